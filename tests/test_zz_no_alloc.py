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
        assert rc == 0, lib.trit_cuda_last_error().decode()
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
    assert "static scratch" in lib.trit_cuda_last_error().decode()


def _device_layer(torch, n, k, seed):
    codes, scales = _q8_0(n, k, seed)
    dense = Dense.q8_0(O.q8_0_blocks(codes.reshape(-1), scales.reshape(-1)), n, k)
    dev = torch.device("cuda", 0)
    return (dense, torch.from_numpy(codes.view(np.int8)).to(dev), torch.from_numpy(scales.view(np.int16)).to(dev))


def test_static_scratch_at_its_size_limit():
    """The largest call the 1 MiB array takes for k = 8192 (113 rows: codes
    plus scales fill 1,041,408 bytes; the GEMV runs it in passes of 8
    frames) equals the allocating entry point; one more row is refused."""
    torch = pytest.importorskip("torch")
    lib = library()
    n, k = 256, 8192
    dense, codes_d, scales_d = _device_layer(torch, n, k, 11)
    dev = torch.device("cuda", 0)
    for call in range(2):
        rows = 113
        x_d = torch.from_numpy(np.random.default_rng(300 + call).standard_normal((rows, k)).astype(np.float32)).to(dev)
        want_d = torch.zeros((rows, n), dtype=torch.float32, device=dev)
        got_d = torch.full((rows, n), float("nan"), dtype=torch.float32, device=dev)
        torch.cuda.synchronize()
        dense.forward_device(x_d.data_ptr(), rows, want_d.data_ptr(), None)
        rc = lib.trit_dense_q8_0_forward_static(codes_d.data_ptr(), scales_d.data_ptr(), n, k, x_d.data_ptr(), rows,
                                                got_d.data_ptr(), None)
        assert rc == 0, lib.trit_cuda_last_error().decode()
        torch.cuda.synchronize()
        assert torch.equal(got_d, want_d), f"call {call}: max diff {(got_d - want_d).abs().max().item()}"
    x_d = torch.zeros((114, k), dtype=torch.float32, device=dev)
    out_d = torch.zeros((114, n), dtype=torch.float32, device=dev)
    assert lib.trit_dense_q8_0_forward_static(codes_d.data_ptr(), scales_d.data_ptr(), n, k, x_d.data_ptr(), 114,
                                              out_d.data_ptr(), None) == -1
    assert "static scratch" in lib.trit_cuda_last_error().decode()


def test_static_entry_recorded_in_a_graph_capture():
    """The case the entry point exists for: after one ordinary call on the
    device (which looks up the array's address and sets every kernel
    attribute), a call with another row count is recorded inside someone
    else's CUDA graph capture and replayed."""
    torch = pytest.importorskip("torch")
    lib = library()
    n, k = 512, 1024
    dense, codes_d, scales_d = _device_layer(torch, n, k, 13)
    dev = torch.device("cuda", 0)
    warm = torch.zeros((2, k), dtype=torch.float32, device=dev)
    warm_out = torch.zeros((2, n), dtype=torch.float32, device=dev)
    assert lib.trit_dense_q8_0_forward_static(codes_d.data_ptr(), scales_d.data_ptr(), n, k, warm.data_ptr(), 2,
                                              warm_out.data_ptr(), None) == 0
    rows = 12
    x_d = torch.empty((rows, k), dtype=torch.float32, device=dev)
    got_d = torch.full((rows, n), float("nan"), dtype=torch.float32, device=dev)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        stream = torch.cuda.current_stream().cuda_stream
        rc = lib.trit_dense_q8_0_forward_static(codes_d.data_ptr(), scales_d.data_ptr(), n, k, x_d.data_ptr(), rows,
                                                got_d.data_ptr(), ctypes.c_void_p(stream))
    assert rc == 0, lib.trit_cuda_last_error().decode()
    for call in range(2):
        x = np.random.default_rng(400 + call).standard_normal((rows, k)).astype(np.float32)
        x_d.copy_(torch.from_numpy(x))
        graph.replay()
        torch.cuda.synchronize()
        assert np.array_equal(got_d.cpu().numpy(), dense.forward(x)), f"replay {call}"
    del graph
