"""Host logic of bench.py, on the CPU: the synthetic Q8_0 bytes equal the
oracle's quantizer (Blocks::quantize, src/cpu/gemm.rs:53-76), the
algorithmic bytes of a C1 decode step match the figure the measurement is
quoted against, the clock sampler reads throttle reasons, and the op
sweep's overrides and product-kernel rule parse as documented."""
import argparse

import numpy as np

import bench
from oracle import oracle as O
from tests.synth import presets


def test_q8_0_blocks_equal_the_oracle_quantizer():
    v = np.random.default_rng(5).normal(0, 0.02, (64, 256)).astype(np.float32)
    v[3, :32] = 0.0  # an all-zero block: scale 0, codes 0
    v[7, 5] = 0.5    # a block dominated by one value
    codes, scales = O.q8_0_quantize(v)
    assert np.array_equal(bench.q8_0_blocks(v), O.q8_0_blocks(codes, scales))


def test_c1_algorithmic_bytes():
    cfg = presets.QWEN3_06B
    d, ffn, L = cfg["hidden_size"], cfg["intermediate_size"], cfg["num_hidden_layers"]
    qd, kvd = cfg["num_attention_heads"] * 128, cfg["num_key_value_heads"] * 128
    product_weights = L * ((qd + 2 * kvd) * d + d * qd + 2 * ffn * d + d * ffn)
    assert product_weights == 440_401_920
    table_weights = cfg["vocab_size"] * d
    info = {"hidden_size": d, "num_hidden_layers": L, "head_dim": 128, "num_key_value_heads": 8,
            "qk_norm": True, "product_bytes": product_weights * 34 // 32,
            "output_table_bytes": table_weights * 34 // 32}
    # One step at position 64 with an f16 cache: 633.2 MB of weights and
    # 114,688 B of KV per position read, plus the new row.
    b = bench.algorithmic_bytes(info, 1, [64], 2)
    assert abs(b["weights"] / 1e6 - 633.2) < 0.5
    kv_row = L * 2 * kvd * 2
    assert kv_row == 114_688
    assert b["kv"] == kv_row * 65 + kv_row
    # Streams scale the KV part only.
    b4 = bench.algorithmic_bytes(info, 4, [64], 2)
    assert b4["weights"] == b["weights"] and b4["kv"] == 4 * b["kv"]


def test_clock_summary_reads_reasons():
    c = bench.Clocks(0)
    c.lines = [
        "0, 1965, 1965, 700.1, 0x0, Not Active, Not Active, Not Active, Not Active",
        "0, 1900, 1965, 990.5, 0x4, Not Active, Not Active, Not Active, Active",
        "0, 1950, 1965, 800.0, 0x0, Not Active, Not Active, Not Active, Not Active",
        "garbage line",
    ]
    s = c.summary()
    assert s["sm_mhz"] == 1950 and s["sm_max_mhz"] == 1965 and s["samples"] == 3
    assert s["reasons"] == ["sw_power_cap"]


def test_sweep_overrides_and_kernel_rule():
    none = argparse.Namespace(shapes=None, rows=None)
    assert bench.sweep_shapes(none) == bench.SWEEP_SHAPES
    assert bench.sweep_rows(none) == bench.SWEEP_ROWS
    some = argparse.Namespace(shapes="16384x3072,3072x8192", rows="64,512")
    assert bench.sweep_shapes(some) == [(16384, 3072), (3072, 8192)]
    assert bench.sweep_rows(some) == [64, 512]
    assert bench.dense_kernel(1024, 1) == "k_gemv_slots"
    assert bench.dense_kernel(1024, 4) == "k_gemv_slots"
    assert bench.dense_kernel(1024, 16) == "k_gemm_tc"
    assert bench.dense_kernel(6144, 4) == "k_gemm_tc"
    assert bench.dense_kernel(151936, 1) == "k_gemm_tc"
