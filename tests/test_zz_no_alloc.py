"""trit_dense_q8_0_forward_static: the Q8_0 product for callers that cannot
allocate device memory when they run it (inside someone else's graph
capture, on a real-time thread, or with all device memory in their own
pool). Its scratch is a fixed 1 MiB device array in the library, so it must
give what the allocating entry point (trit_dense_forward_device) gives, on
every call, with nothing left over from the call before.

This file is collected last: it must pass alone in a fresh process (the
first call sets up the array's device address) and after every other test.
"""
import ctypes

import numpy as np
import pytest

from oracle import oracle as O
from trit_b200 import Dense, library

pytestmark = pytest.mark.gpu


def _q8_0(n, k, seed):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    codes, scales = O.q8_0_quantize(w)
    return codes.reshape(n, k), scales.reshape(n, k // 32)


def test_static_scratch_equals_allocating_entry_point():
    torch = pytest.importorskip("torch")
    lib = library()
    n, k = 512, 1024
    codes, scales = _q8_0(n, k, 5)
    blocks = O.q8_0_blocks(codes.reshape(-1), scales.reshape(-1))
    dense = Dense.q8_0(blocks, n, k)
    dev = torch.device("cuda", 0)
    codes_d = torch.from_numpy(codes.view(np.int8)).to(dev)
    scales_d = torch.from_numpy(scales.view(np.int16)).to(dev)
    for call, rows in enumerate([16, 5]):  # two calls in a row, the second smaller
        x = np.random.default_rng(100 + call).standard_normal((rows, k)).astype(np.float32)
        x_d = torch.from_numpy(x).to(dev)
        want_d = torch.zeros((rows, n), dtype=torch.float32, device=dev)
        got_d = torch.full((rows, n), float("nan"), dtype=torch.float32, device=dev)
        torch.cuda.synchronize()
        dense.forward_device(x_d.data_ptr(), rows, want_d.data_ptr(), None)
        rc = lib.trit_dense_q8_0_forward_static(codes_d.data_ptr(), scales_d.data_ptr(), n, k, x_d.data_ptr(), rows,
                                                got_d.data_ptr(), None)
        assert rc == 0, lib.trit_last_error().decode()
        torch.cuda.synchronize()
        want, got = want_d.cpu().numpy(), got_d.cpu().numpy()
        # The same kernels on the same inputs: equal bit for bit (the tests'
        # tolerance for products of the same quantized inputs).
        assert np.array_equal(got, want), f"call {call}: max diff {np.abs(got - want).max()}"
        assert np.array_equal(got, dense.forward(x))


def test_static_scratch_rejects_sizes_beyond_its_limit():
    torch = pytest.importorskip("torch")
    lib = library()
    n, k = 32, 8192
    dev = torch.device("cuda", 0)
    codes_d = torch.zeros((n, k), dtype=torch.int8, device=dev)
    scales_d = torch.zeros((n, k // 32), dtype=torch.int16, device=dev)
    rows = 128  # 128 * 8192 * 9 / 8 bytes > 1 MiB
    x_d = torch.zeros((rows, k), dtype=torch.float32, device=dev)
    out_d = torch.zeros((rows, n), dtype=torch.float32, device=dev)
    rc = lib.trit_dense_q8_0_forward_static(codes_d.data_ptr(), scales_d.data_ptr(), n, k, x_d.data_ptr(), rows,
                                            out_d.data_ptr(), None)
    assert rc == -1
    assert "static scratch" in lib.trit_last_error().decode()
