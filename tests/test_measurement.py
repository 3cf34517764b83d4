"""The benchmark's workload tables (CPU): the attention configs carry the
shapes and input scales the configs are quoted on, and the algorithmic FLOP
and byte counts that every TFLOP/s and GB/s figure divides by follow the
causal convention (T^2/2 pairs; fwd 2*B*H*T^2*d, bwd 5*B*H*T^2*d; computeD
reads dO and O and writes D)."""
import pytest

from metalllm_b200.inputs import CONFIGS, causal_flops
from metalllm_b200.shards import plan_all


@pytest.mark.parametrize("cfg,shape", [
    ("c1", (16, 256, 6, 64)),
    ("c2", (64, 1024, 12, 64)),
    ("c3", (8, 4096, 16, 128)),
    ("c4", (4, 8192, 32, 64)),
])
def test_config_shapes(cfg, shape):
    c = CONFIGS[cfg]
    assert (c["B"], c["T"], c["H"], c["D"]) == shape
    assert c["qkv_scale"] == (0.5 if cfg == "c3" else 1.0) and c["do_scale"] == 1.0


@pytest.mark.parametrize("cfg,fwd_g,bwd_g,total_g", [
    ("c1", 0.805, 2.013, 2.819),
    ("c2", 103.1, 257.7, 360.8),
    ("c3", 549.8, 1374.4, 1924.1),
    ("c4", 1099.5, 2748.8, 3848.3),
])
def test_causal_flops(cfg, fwd_g, bwd_g, total_g):
    c = CONFIGS[cfg]
    fwd, bwd = causal_flops(c["B"], c["T"], c["H"], c["D"])
    assert bwd == 2.5 * fwd
    assert fwd / 1e9 == pytest.approx(fwd_g, rel=1e-3)
    assert bwd / 1e9 == pytest.approx(bwd_g, rel=1e-3)
    assert (fwd + bwd) / 1e9 == pytest.approx(total_g, rel=1e-3)


@pytest.mark.parametrize("cfg,mb", [("c1", 6.34), ("c2", 202.9), ("c3", 269.5), ("c4", 270.5)])
def test_compute_d_algorithmic_bytes(cfg, mb):
    c = CONFIGS[cfg]
    elems = c["B"] * c["T"] * c["H"] * c["D"]
    rows = c["B"] * c["T"] * c["H"]
    assert (2 * elems * 2 + rows * 2) / 1e6 == pytest.approx(mb, rel=2e-3)


@pytest.mark.parametrize("cfg,world", [("c3", 1), ("c3", 2), ("c3", 4), ("c3", 8), ("c4", 8), ("c2", 2)])
def test_weak_and_strong_shard_counts(cfg, world):
    """Config 3/4's 128 (batch, head) shards split evenly over 1/2/4/8 GPUs."""
    c = CONFIGS[cfg]
    plans = plan_all(c["B"], c["H"], world)
    counts = {p.shards for p in plans}
    assert len(counts) == 1 and counts.pop() * world == c["B"] * c["H"]
