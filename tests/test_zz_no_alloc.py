"""zest_mul_mat_noalloc, the entry point for callers that cannot allocate
device memory on this path (a program whose GPU memory its own allocator
plans and owns, or a latency-sensitive caller that cannot let cudaMalloc /
cudaFree synchronise the device mid-prompt). Its scratch, the bf16 copy of
the activations, lives in a fixed device array inside the library.

Called through the C ABI, twice in a row, and checked against the existing
entry point zest_mul_mat on the same weight copy and inputs. This file sorts
last so that a run stopping at its first failure has run everything else.
"""
import ctypes

import numpy as np
import pytest
import torch

import zest_b200 as Z
from oracle import oracle as O

pytestmark = pytest.mark.gpu

TOL = 1e-3  # the GEMM tests' bar; the two paths run the same kernels, so they agree exactly
MAX_VALUES = 16 * 1024 * 1024


def _noalloc(x, K, w_ptr, N, mode, y, err):
    L = Z.lib()
    return L.zest_mul_mat_noalloc(ctypes.c_void_p(x.data_ptr()), x.shape[0], K, x.stride(0), ctypes.c_void_p(w_ptr),
                                  K, N, mode, ctypes.c_void_p(y.data_ptr()), y.stride(0),
                                  ctypes.c_void_p(err.data_ptr()), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


def test_noalloc_matches_mul_mat_twice():
    torch.cuda.set_device(0)
    npu = Z.Npu(0)
    npu.set_out16(False)
    N, K = 1536, 1024
    raw = O.quantize(O.Q8_0, O.weights_f32(N, K, 3))
    key = Z.Npu.key(raw.ctypes.data, O.Q8_0, K, N)
    npu.add_weight(key, raw.ctypes.data, on_device=False)
    w_ptr, n_pad = npu.weight_bf16(key)
    assert w_ptr and n_pad >= N
    # two calls in a row, the second smaller, so a stale row of the first in
    # the shared scratch would show
    for T, seed in ((2000, 1), (333, 2)):
        x = torch.from_numpy(O.activations(T, K, seed)).cuda()
        want = torch.empty((T, N), dtype=torch.float32, device="cuda")
        torch.cuda.synchronize()
        npu.mul_mat(key, x.data_ptr(), T, want.data_ptr(), on_device=True)
        got = torch.full((T, N), float("nan"), dtype=torch.float32, device="cuda")
        err = torch.zeros(1, dtype=torch.int32, device="cuda")
        rc = _noalloc(x, K, w_ptr, N, Z.MODE_F32, got, err)
        assert rc == 0, Z.lib().zest_last_error().decode()
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        g, w = got.cpu().numpy(), want.cpu().numpy()
        assert O.nmax_err(g, w) <= TOL
        assert np.array_equal(g, w)
    npu.close()


def test_noalloc_rejects_oversized_calls():
    torch.cuda.set_device(0)
    K = 4096
    T = MAX_VALUES // K + 1  # one row over the limit once padded
    x = torch.zeros((1, K), dtype=torch.float32, device="cuda").expand(T, K)
    y = torch.zeros((1, 8), dtype=torch.float32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    L = Z.lib()
    rc = L.zest_mul_mat_noalloc(ctypes.c_void_p(x.data_ptr()), T, K, K, ctypes.c_void_p(x.data_ptr()), K, 8, 0,
                                ctypes.c_void_p(y.data_ptr()), 8, ctypes.c_void_p(err.data_ptr()), None)
    assert rc == -1
    assert "ZEST_NOALLOC_MAX_VALUES" in L.zest_last_error().decode()
