"""The bench's workload arithmetic (CPU): the algorithmic bytes behind ``roofline.achieved``, the L2 rule for the
rotating inputs, and the metric text, for the sampling workloads and the two head workloads."""

import bench


def test_bytes_per_row_follow_the_stated_formulas():
    w = bench.WORKLOADS["thinker"]
    assert bench.bytes_per_row(w) == 151_936 * 2 + 4 * 512 + 40
    w = bench.WORKLOADS["talker_head"]  # the head once per step, shared by the batch; the hidden row per row
    assert bench.bytes_per_row(w) * w["rows"] == 6562 * 768 * 2 + w["rows"] * (2 * 768 + 4 * 64 + 40)
    w = bench.WORKLOADS["greedy_head"]
    assert bench.bytes_per_row(w) * w["rows"] == 151_936 * 4096 * 2 + w["rows"] * (2 * 4096 + 8)


def test_rotating_inputs_exceed_the_l2():
    for name, w in bench.WORKLOADS.items():
        if w.get("op") == "lmhead":
            assert w["vocab"] * w["hidden"] * 2 > 2 * bench.L2_BYTES  # one head is already larger
            continue
        if w.get("op") == "head":
            per = w["vocab"] * w["hidden"] * 2
        else:
            per = w["rows"] * w["vocab"] * (2 if w["dtype"] == "bf16" else 4)
        n = bench.rotating_buffers(w)
        assert n * per > bench.L2_BYTES, name  # the timing rule: every sweep is larger than the L2
        assert n * per > 2 * bench.L2_BYTES or n == 8192, name  # twice the L2 unless the buffer count is capped


def test_metric_names_the_fused_head_steps():
    assert "codec head" in bench.metric_of(bench.WORKLOADS["talker_head"])
    assert "LM head" in bench.metric_of(bench.WORKLOADS["greedy_head"])
