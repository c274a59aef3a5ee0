"""B200-native token-sampling engine for MiniCPM-o 4.5 (sm_100a CUDA kernels behind a C-ABI).

* ``talker_sampler`` -- drop-in for the reference ``engine/talker_sampler.py`` (same names / signatures);
* ``thinker_sampler`` -- the Thinker step: greedy ``argmax`` (the reference's behaviour) and ``sample``;
* ``vocab_shard`` -- vocabulary-sharded sampling across ranks (NCCL all-gather of per-shard candidates).

The directory name is not a Python identifier; ``__graft_entry__.load_package()`` registers it as
``b200_sampler``.
"""

from . import _native, seeds, talker_sampler, thinker_sampler, vocab_shard  # noqa: F401
from .talker_sampler import (  # noqa: F401
    PAD,
    DecodeState,
    RowParams,
    TalkerSampling,
    decode_k,
    draw,
    processed_logits,
    sample,
    step,
    uniform,
)
