"""bench.py's reported arithmetic, checked on the CPU.

Beside its measured times the benchmark line carries figures that are pure
functions of the configuration: the algorithmic weight bytes per token, the
full-stream extrapolation, the decode chain floor and the operation count
of the encode FP32 roofline.  These tests pin them to values worked out by
hand from the BASELINE configurations, so that a change to the helpers
cannot silently change what a measured time is divided by.
"""
import pytest

import bench
from detllm_b200 import synth as S

L3 = S.CONFIGS["llama3-8b-q4_k"]


def test_weight_bytes_per_token_of_the_baseline_configs():
    # Q8_0 34/32, Q4_K 144/256, Q6_K 210/256 bytes per weight; every GEMV
    # matrix of one token's forward plus the lm_head (the embedding is one row)
    assert S.weight_bytes_per_token(S.CONFIGS["tinyllama-q8_0"]) == 1_099_071_488
    assert S.weight_bytes_per_token(S.CONFIGS["tinyllama-q4_k_m"]) == 664_178_688
    assert S.weight_bytes_per_token(S.CONFIGS["qwen2.5-0.5b-q8_0"]) == 524_833_792
    assert S.weight_bytes_per_token(L3) == 4_841_250_816


def test_full_stream_estimate_counts_windows_like_the_codec():
    # a 2 MiB segment at n_ctx 8192: the first window codes 8,192 symbols,
    # each later one replays 2,048 and codes 6,144: 1 + 340 windows
    est = bench.full_stream_estimate(2 << 20, 8192, 4.0, 1)
    assert est["windows_per_segment"] == 341
    assert est["est_s"] == pytest.approx(8 * 341 * 4.0)
    assert est["est_tokens_per_s"] == pytest.approx((16 << 20) / (8 * 341 * 4.0))
    # segments are dealt round-robin: ceil(8 / N) per GPU
    assert bench.full_stream_estimate(2 << 20, 8192, 4.0, 8)["est_s"] == pytest.approx(341 * 4.0)
    assert bench.full_stream_estimate(2 << 20, 8192, 4.0, 3)["est_s"] == pytest.approx(3 * 341 * 4.0)
    # a segment that fits one window takes one window
    assert bench.full_stream_estimate(5000, 8192, 1.0, 1)["windows_per_segment"] == 1


def test_decode_chain_floor_of_the_headline_model():
    # 4.3 cycles per dependent add at 1,965 MHz: 4,096 adds = 8.96 us, more
    # than the bytes of q|k|v (2.16 us) or o (1.44 us) at 6,550 GB/s;
    # gate|up (10.09 us) and down (7.35 us) are bound by their bytes
    f = bench.decode_chain_floor(L3, 4.3, 1965.0, 6550.0)
    parts = f["per_layer_launch"]
    assert parts["Q4_K 6144x4096"] == {"us": 8.96, "bound": "chain"}
    assert parts["Q4_K 4096x4096"] == {"us": 8.96, "bound": "chain"}
    assert parts["Q4_K 28672x4096"] == {"us": 10.09, "bound": "hbm"}
    assert parts["Q6_K 4096x14336"] == {"us": 7.35, "bound": "hbm"}
    lm_head_us = 128256 * 4096 * 210 / 256 / 6550e3
    layer_us = 2 * 4096 * 4.3 / 1965.0 + 28672 * 4096 * 144 / 256 / 6550e3 + 4096 * 14336 * 210 / 256 / 6550e3
    assert f["ms_per_token"] == pytest.approx((32 * layer_us + lm_head_us) / 1000.0)
    assert f["ms_per_token"] == pytest.approx(1.1975, abs=1e-4)


def test_encode_roofline_counts_two_ops_per_q4k_weight_and_position():
    # q|k|v (6,144 rows), o (4,096) and gate|up (28,672) at K 4,096, 32 layers
    per_layer = (6144 + 4096 + 28672) * 4096
    assert bench.q4k_weight_positions(L3, 8192) == per_layer * 32 * 8192
    ops = 2.0 * bench.q4k_weight_positions(L3, 8192)
    kprof = {"gemm_qkv": (256, 400.0), "gemm_o": (256, 300.0), "gemm_gate_up": (256, 2300.0),
             "attention": (768, 800.0)}
    r = bench.encode_roofline(kprof, ops, 1965.0, 148)
    assert r["bound"] == "fp32" and r["launches"] == 768 and r["ms"] == pytest.approx(3000.0)
    assert r["peak"] == pytest.approx(148 * 128 * 1965e6 / 1e12)
    assert r["achieved"] == pytest.approx(ops / 3.0 / 1e12)
    assert r["frac"] == pytest.approx(r["achieved"] / r["peak"])
    # no Q4_K launches or no clock sample: no roofline rather than a wrong one
    assert bench.encode_roofline({"attention": (1, 1.0)}, ops, 1965.0, 148) is None
    assert bench.encode_roofline(kprof, ops, None, 148) is None
