"""The operator level on the GPU: Dense::forward (src/cpu/gemm.rs:500-542)
of a Q8_0 layer, as the W8A8 product (Int8::from_q8_0, int8.rs:234-289)
and as a token table (Q8::matmul, gemm.rs:166-187), against the CPU
oracle, bit for bit, at the op-sweep shapes including the 151936-row
table shape."""
import numpy as np
import pytest

from oracle import oracle as O
from trit_b200 import Dense

pytestmark = pytest.mark.gpu


def _layer(n, k, seed):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    codes, scales = O.q8_0_quantize(w)
    return codes.reshape(n, k), scales.reshape(n, k // 32)


@pytest.mark.parametrize("n, k", [(1024, 3072), (3072, 1024), (151936, 1024)])
@pytest.mark.parametrize("m", [1, 5, 16, 64])
def test_w8a8_product_matches_oracle(n, k, m):
    codes, scales = _layer(n, k, n + k)
    blocks = O.q8_0_blocks(codes.reshape(-1), scales.reshape(-1))
    x = np.random.default_rng(m).standard_normal((m, k)).astype(np.float32)
    got = Dense.q8_0(blocks, n, k).forward(x)
    ws = scales.view(np.float16).astype(np.float32)  # f16 -> f32 is exact
    want = O.IntLayer(codes, ws, 32, 32, True).forward(x)
    assert np.array_equal(got, want), f"max diff {np.abs(got - want).max()}"


@pytest.mark.parametrize("m", [1, 5, 20])
def test_table_product_matches_oracle(m):
    n, k = 4096, 1024
    codes, scales = _layer(n, k, 77)
    blocks = O.q8_0_blocks(codes.reshape(-1), scales.reshape(-1))
    x = np.random.default_rng(m).standard_normal((m, k)).astype(np.float32)
    got = Dense.q8_0(blocks, n, k, table=True).forward(x)
    ws = scales.view(np.float16).astype(np.float32)
    want = O.Table(codes, ws).forward(x)
    assert np.array_equal(got, want), f"max diff {np.abs(got - want).max()}"
