"""The DRAM traffic table bench.py reports as roofline.traffic: one entry per batch-1 workload, every kernel of the
chain, and Q8_0 weights (C4) moving about half the bytes of bf16 (C3) in the weight-streaming kernels."""
import json
import os

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
KERNELS = ("qkv_rope", "attention", "oproj", "gate_up", "down", "head")


def test_traffic_table_per_workload():
    t = json.load(open(os.path.join(ROOT, "profiles", "traffic.json")))
    for w in ("c3", "c4"):
        assert set(KERNELS) <= set(t[w]), w
        assert all(t[w][k] > 0 for k in KERNELS)
    for k in ("qkv_rope", "oproj", "gate_up", "down"):  # Q8_0: 34 bytes per 32 weights against 64
        assert 0.45 < t["c4"][k] / t["c3"][k] < 0.6, k
    assert abs(t["c4"]["head"] / t["c3"]["head"] - 1) < 0.01  # the lm_head stays bf16
