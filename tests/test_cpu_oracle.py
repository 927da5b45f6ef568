"""The CPU oracle's operations against independent numpy restatements of
the reference's arithmetic. The oracle is the checker of every GPU parity
test; these tests pin each of its parts to the reference's definitions:
  f32 -> f16            tensors.rs f32_to_f16 (round to nearest, ties even)
  activation quantizer  Quantized::grouped + quantize_scalar,
                        src/cpu/kernels.rs:661-737,760-779
  W8A8 product          Int8 tiles, src/cpu/int8.rs:525-584 (per group
                        acc = fma(f32(dot), ws * xs, acc), groups in order)
  token table product   Q8::matmul, src/cpu/gemm.rs:166-187 (f32 math)
  Cephes exp / SiLU     src/cpu/activation.rs:8-38,54-56
  RmsNorm               src/layers.rs:122-153 (sequential sum)
  Rotary::halves        layers.rs:276-335
  attention             layers.rs:343-504, softmax_rows :571-587
The VNNI tile and the scalar path of the oracle must agree bit for bit, as
the reference's AVX-512 and scalar paths agree (int8.rs:496,567-568)."""
import ctypes

import numpy as np
import pytest

from oracle import oracle

f32 = np.float32


def fma32(a, b, c):
    """fma in float32 via float64: a*b is exact in float64; the sum rounds
    once to float64 and once to float32 (equal to one rounding except in
    rare double-rounding cases, which the callers allow for)."""
    return (np.float64(a) * np.float64(b) + np.float64(c)).astype(np.float32)


def ulps(a, b):
    a = np.asarray(a, np.float32).view(np.int32).astype(np.int64)
    b = np.asarray(b, np.float32).view(np.int32).astype(np.int64)
    a = np.where(a < 0, -(a & 0x7FFFFFFF), a)
    b = np.where(b < 0, -(b & 0x7FFFFFFF), b)
    return np.abs(a - b)


def test_f16_round_trip():
    rng = np.random.default_rng(0)
    vals = np.concatenate([rng.normal(0, 1, 2000), rng.normal(0, 1e-5, 500), rng.normal(0, 3e4, 500),
                           [0.0, -0.0, 65504.0, 65520.0, 1e9, -1e9, 2 ** -24, 2 ** -25, 3 * 2 ** -26, 1.5 * 2 ** -14]])
    vals = vals.astype(np.float32)
    for v in vals:
        with np.errstate(over="ignore"):
            want = np.float16(v)
        h = oracle.f32_to_f16(float(v))
        assert h == int(want.view(np.uint16)), v
        assert oracle.f16_to_f32(h) == np.float32(want)


def quantize_numpy(x, group, half):
    m, k = x.shape
    codes = np.zeros((m, k), np.int8)
    scales = np.zeros((m, k // group), np.float32)
    sums = np.zeros((m, k // group), np.int32)
    for r in range(m):
        for g in range(k // group):
            span = x[r, g * group:(g + 1) * group]
            mx = np.abs(span).max()
            scale = f32(mx / f32(127.0)) if mx > 0 else f32(1.0)
            inv = f32(f32(1.0) / scale)
            c = np.clip(np.rint((span * inv).astype(np.float32)), -127, 127).astype(np.int8)
            codes[r, g * group:(g + 1) * group] = c
            sums[r, g] = int(c.astype(np.int32).sum())
            scales[r, g] = f32(np.float16(scale)) if half else scale
    return codes, scales, sums


@pytest.mark.parametrize("group, half", [(32, True), (128, False), (32, False)])
def test_activation_quantizer(group, half):
    rng = np.random.default_rng(group + half)
    x = rng.normal(0, 1, (5, 512)).astype(np.float32)
    x[1, :group] = 0.0                          # an all-zero group: scale 1
    x[2, 5] = 1e4                               # a dominant value
    x[3, :group] = np.arange(group) - group / 2  # exact halves after scaling
    codes, scales, sums = oracle.quantize(x, group, half)
    c2, s2, u2 = quantize_numpy(x, group, half)
    assert np.array_equal(codes, c2) and np.array_equal(scales, s2) and np.array_equal(sums, u2)


def int_layer_numpy(codes, wscales, wgroup, x, group, half):
    xq, xs, _ = quantize_numpy(x, group, half)
    n, k = codes.shape
    out = np.zeros((x.shape[0], n), np.float32)
    for r in range(x.shape[0]):
        for o in range(n):
            acc = f32(0.0)
            for g in range(k // group):
                dot = int(np.dot(codes[o, g * group:(g + 1) * group].astype(np.int32),
                                 xq[r, g * group:(g + 1) * group].astype(np.int32)))
                ws = wscales[o, (g * group) // wgroup]
                acc = fma32(f32(dot), f32(ws * xs[r, g]), acc)
            out[r, o] = acc
    return out


@pytest.mark.parametrize("group, wgroup, half", [(32, 32, True), (128, 128, False), (128, 1024, False)])
def test_w8a8_product(group, wgroup, half):
    rng = np.random.default_rng(wgroup)
    n, k = 48, 1024
    codes = rng.integers(-127, 128, (n, k)).astype(np.int8)
    wscales = rng.uniform(1e-4, 1e-3, (n, k // wgroup)).astype(np.float32)
    x = rng.normal(0, 1, (3, k)).astype(np.float32)
    layer = oracle.IntLayer(codes, wscales, group, wgroup, half)
    got = layer.forward(x)
    want = int_layer_numpy(codes, wscales, wgroup, x, group, half)
    assert ulps(got, want).max() <= 1
    assert (ulps(got, want) == 0).mean() > 0.99
    oracle.lib().oracle_force_scalar(1)
    try:
        scalar = oracle.IntLayer(codes, wscales, group, wgroup, half).forward(x)
    finally:
        oracle.lib().oracle_force_scalar(0)
    assert np.array_equal(got.view(np.int32), scalar.view(np.int32))


def table_numpy(codes, scales, x):
    """16 lanes (lane l takes k = l mod 16, fma in k order), then the
    _mm512_reduce_add_ps tree: s8[i] = a[i] + a[i+8], s4[i] = s8[i] + s8[i+4],
    (s4[0] + s4[2]) + (s4[1] + s4[3])."""
    n, k = codes.shape
    w = (codes.astype(np.float32) * np.repeat(scales, 32, axis=1)).astype(np.float32)
    out = np.zeros((x.shape[0], n), np.float32)
    for r in range(x.shape[0]):
        for o in range(n):
            lanes = np.zeros(16, np.float32)
            for i in range(0, k, 16):
                lanes = fma32(x[r, i:i + 16], w[o, i:i + 16], lanes)
            s8 = (lanes[:8] + lanes[8:]).astype(np.float32)
            s4 = (s8[:4] + s8[4:]).astype(np.float32)
            out[r, o] = f32(f32(s4[0] + s4[2]) + f32(s4[1] + s4[3]))
    return out


def test_token_table_product():
    rng = np.random.default_rng(5)
    n, k = 40, 256
    codes = rng.integers(-127, 128, (n, k)).astype(np.int8)
    scales = np.float16(rng.uniform(1e-4, 1e-3, (n, k // 32))).astype(np.float32)
    x = rng.normal(0, 1, (2, k)).astype(np.float32)
    got = oracle.Table(codes, scales).forward(x)
    want = table_numpy(codes, scales, x)
    assert ulps(got, want).max() <= 1 and (ulps(got, want) == 0).mean() > 0.99
    oracle.lib().oracle_force_scalar(1)
    try:
        scalar = oracle.Table(codes, scales).forward(x)
    finally:
        oracle.lib().oracle_force_scalar(0)
    assert np.array_equal(got.view(np.int32), scalar.view(np.int32))


def test_exp_and_silu():
    xs = np.concatenate([np.linspace(-87, 88, 20001), np.linspace(-1, 1, 2001)]).astype(np.float32)
    got = np.array([oracle.lib().oracle_exp(float(v)) for v in xs], np.float32)
    want = np.exp(xs.astype(np.float64))
    rel = np.abs(got - want) / want
    assert rel.max() < 3e-7
    assert oracle.lib().oracle_exp(-200.0) == 0.0 or oracle.lib().oracle_exp(-200.0) < 1e-37
    for v in (-30.0, -3.0, -0.5, 0.0, 0.5, 3.0, 30.0):
        e = oracle.lib().oracle_exp(f32(0.0) - f32(v))
        assert oracle.lib().oracle_silu(v) == f32(f32(v) / f32(f32(1.0) + f32(e)))


def test_rmsnorm_sequential_sum():
    rng = np.random.default_rng(9)
    for d in (128, 1024, 3072):
        row = rng.normal(0, 2, d).astype(np.float32)
        w = rng.uniform(0.5, 1.5, d).astype(np.float32)
        got = row.copy()
        oracle.lib().oracle_rmsnorm(got.ctypes.data_as(oracle._f32p), w.ctypes.data_as(oracle._f32p), d, 1e-6)
        s = f32(-0.0)
        for v in row:
            s = f32(s + f32(v * v))
        inv = f32(f32(1.0) / np.sqrt(f32(f32(s / f32(d)) + f32(1e-6))))
        want = (row * (inv * w).astype(np.float32)).astype(np.float32)
        assert np.array_equal(got, want)


def test_rope_halves():
    rng = np.random.default_rng(11)
    rows, heads, hd, first = 5, 3, 128, 37
    x = rng.normal(0, 1, (rows, heads * hd)).astype(np.float32)
    got = x.copy()
    oracle.lib().oracle_rope(got.ctypes.data_as(oracle._f32p), rows, heads * hd, heads, hd, first, 1e6)
    inv = np.power(np.float64(1e6), -np.arange(0, hd, 2) / hd)
    for r in range(rows):
        ang = (first + r) * inv
        for h in range(heads):
            a, b = x[r, h * hd:h * hd + 64].astype(np.float64), x[r, h * hd + 64:(h + 1) * hd].astype(np.float64)
            want = np.concatenate([a * np.cos(ang) - b * np.sin(ang), b * np.cos(ang) + a * np.sin(ang)])
            assert np.abs(got[r, h * hd:(h + 1) * hd] - want).max() < 2e-4


def test_attention_against_float64():
    rng = np.random.default_rng(13)
    tq, tk, heads, kvh, hd = 3, 9, 4, 2, 128
    q = rng.normal(0, 1, (tq, heads * hd)).astype(np.float32)
    k = rng.normal(0, 1, (tk, kvh * hd)).astype(np.float32)
    v = rng.normal(0, 1, (tk, kvh * hd)).astype(np.float32)
    out = np.zeros((tq, heads * hd), np.float32)
    P = oracle._f32p
    oracle.lib().oracle_attention(q.ctypes.data_as(P), heads * hd, k.ctypes.data_as(P), v.ctypes.data_as(P), kvh * hd,
                                  tq, tk, heads, kvh, hd, 1, out.ctypes.data_as(P))
    for i in range(tq):
        for h in range(heads):
            g = h // (heads // kvh)
            s = (k[:, g * hd:(g + 1) * hd].astype(np.float64) @ q[i, h * hd:(h + 1) * hd].astype(np.float64)) / np.sqrt(hd)
            visible = tk - tq + i + 1
            s[visible:] = -np.inf
            p = np.exp(s - s.max())
            p /= p.sum()
            want = p @ v[:, g * hd:(g + 1) * hd].astype(np.float64)
            assert np.abs(out[i, h * hd:(h + 1) * hd] - want).max() < 1e-5
