"""bench.py's accounting, on CPU: the algorithmic FLOPs per step of every
workload (selected experts only, visible attention pairs only, fwd+bwd = 3 x
fwd), the skewed-routing bias and the peak table it divides by."""
import json
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))
import bench  # noqa: E402


@pytest.mark.parametrize("name,flops", [("mixtral8x7b_block", 8.08e13), ("dense_block", 5.46e12),
                                        ("small_mixtral_block_f32", 6.27e10)])
def test_block_flops_per_step(name, flops):
    wl = bench.WORKLOADS[name]
    assert bench.flops_per_step(wl["cfg"], wl["batch"], wl["seq"]) == pytest.approx(flops, rel=2e-3)


def test_block_flops_by_hand():
    """One token, window 1: every projection once, one visible pair per head."""
    cfg = dict(dim=8, heads=2, kv_heads=1, head_dim=4, experts=4, top_k=2, intermediate=16,
               sliding_window=1)
    D, H, KV, hd, E, k, I = 8, 2, 1, 4, 4, 2, 16
    fwd = (2 * (D * H * hd + 2 * D * KV * hd + H * hd * D) + 4 * hd * H + 2 * k * 3 * D * I
           + 2 * D * E)
    assert bench.flops_per_step(cfg, 1, 1) == 3 * fwd


def test_mlp_flops():
    assert bench.mlp_flops(bench.WORKLOADS["mlp_f32"]) == 3 * 2 * 64 * (128 * 256 + 256 * 128)


def test_zipf_bias():
    """b_e = 2.0 r_e^-1.2 over a seeded rank permutation: the hottest expert
    gets 2.0 and the biases are the Zipf sequence in some order."""
    b = bench.zipf_bias(8)
    assert float(b.max()) == pytest.approx(2.0)
    expect = sorted(2.0 * r ** -1.2 for r in range(1, 9))
    assert sorted(float(v) for v in b) == pytest.approx(expect, rel=1e-6)
    assert bench.zipf_bias(8).tolist() == b.tolist()  # seeded


def test_measured_peaks_are_read():
    hbm, peak, sustained, src = bench.measured_peaks()
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        assert (hbm, peak, sustained, src) == (d["hbm_gbs"], d["bf16_tflops"],
                                               d["bf16_tflops_sustained"], "measured")
    else:
        assert src == "fallback"
