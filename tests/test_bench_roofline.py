"""bench.py's roofline arithmetic on the CPU: the algorithmic bytes and FLOPs
that every `roofline.achieved` and `binding` figure divides by, checked
against hand-derived per-op figures of the benchmark configurations (decode
bytes, dense FLOPs counting visible (query, key) pairs only) and against the
bytes the dense profiles under profiles/ quote."""
import pytest

import bench


def test_decode_bytes_config1_and_config2():
    # config 1: K+V 8,388,608 + Q 8,192 + O 8,192 + mask 4,096
    assert bench.algo_bytes_per_op(sets=1, kv_len=2048, hq=16, hkv=8) == 8_409_088
    # config 2 headline op: 16 sets x 8192 keys, F16
    assert bench.algo_bytes_per_op() == 537_657_344
    # the same op over a Q8_0 cache (34 B per 32 values)
    assert bench.algo_bytes_per_op(kv_bytes_per_row=128 // 32 * 34) == 285_999_104


@pytest.mark.parametrize("name,gflop", [("prefill1024", 8.60), ("prefill4096", 137.5), ("dit1500", 36.9),
                                        ("dit6000", 589.8), ("cross6000", 45.3)])
def test_dense_flops(name, gflop):
    B, Hq, Hkv, S_q, S_kv, kind, extra = bench.DENSE_WORKLOADS[name][:7]
    flops = 4 * 128 * bench.dense_pairs(S_q, S_kv, kind, extra) * Hq * B
    assert flops / 1e9 == pytest.approx(gflop, rel=2e-3)


@pytest.mark.parametrize("name,mb", [("dit6000", 294.9), ("dit6000_window128", 366.9), ("cross6000", 211.1),
                                     ("prefill4096", 201.3), ("dit6000_gqa8", 245.8), ("dit750", 36.9)])
def test_dense_bytes_match_profiles(name, mb):
    assert bench.dense_bytes(name) / 1e6 == pytest.approx(mb, abs=0.1)


def test_dense_bytes_rule_and_q8():
    # a mask by rule reads no mask tensor
    assert bench.dense_bytes("prefill4096") - bench.dense_bytes("prefill4096", rule=True) == 4096 * 4096 * 2
    # Q8_0 K/V: 136 B per 128-dim row
    B, Hq, Hkv, S, _, _, _ = bench.DENSE_WORKLOADS["prefill512_q8_0"][:7]
    assert bench.dense_bytes("prefill512_q8_0", rule=True) == 2 * B * Hq * S * 128 * 4 + 2 * B * Hkv * S * 136


def test_dense_bound_picks_the_longer_time():
    peak_tf, peak_gbs = 1661.8, 6457.4
    # DiT 6000: 589.8 GFLOP against 294.9 MB -> tensor-bound
    b = bench.dense_bound(589.8e9, 294.9e6, 0.570, peak_tf, peak_gbs)
    assert b["bound"] == "tensor"
    assert b["frac_of_bound"] == pytest.approx(589.8e9 / (peak_tf * 1e12) / 0.570e-3, rel=1e-3)
    # cross 6000x512: 45.3 GFLOP against 211.1 MB -> HBM-bound on the f32 Q/O traffic
    b = bench.dense_bound(45.3e9, 211.1e6, 0.155, peak_tf, peak_gbs)
    assert b["bound"] == "hbm"
    assert b["hbm_frac"] == b["frac_of_bound"]
    assert 0.0 < b["frac_of_bound"] < 1.0
