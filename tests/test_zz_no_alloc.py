"""zest_mul_mat_noalloc, the entry point for callers that cannot allocate
device memory on this path (a program whose GPU memory its own allocator
plans and owns, or a latency-sensitive caller that cannot let cudaMalloc /
cudaFree synchronise the device mid-prompt). Its scratch, the bf16 copy of
the activations, lives in a fixed device array inside the library.

Called through the C ABI, twice in a row, and checked against the existing
entry point zest_mul_mat on the same weight copy and inputs, and against the
reference's CPU matmul (xdna_ref_mul_mat, oracle/_ref) on the bfp16-rounded
operands. One shape takes the whole-tile route, one (K = 8192) the stream-K
route, whose partial sums use a second fixed device array. This file sorts
last so that a run stopping at its first failure has run everything else.
"""
import ctypes

import numpy as np
import pytest
import torch

import zest_b200 as Z
from oracle import oracle as O

pytestmark = pytest.mark.gpu

TOL = 1e-3  # the GEMM tests' bar against the reference
MAX_VALUES = 16 * 1024 * 1024


def _noalloc(x, K, w_ptr, N, mode, y, err):
    L = Z.lib()
    return L.zest_mul_mat_noalloc(ctypes.c_void_p(x.data_ptr()), x.shape[0], K, x.stride(0), ctypes.c_void_p(w_ptr),
                                  K, N, mode, ctypes.c_void_p(y.data_ptr()), y.stride(0),
                                  ctypes.c_void_p(err.data_ptr()), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


def _decoded(v: np.ndarray) -> np.ndarray:
    return O.decode_blocks(O.encode_blocks(np.ascontiguousarray(v, np.float32))).reshape(v.shape)


@pytest.mark.parametrize("N,K,calls", [
    (1536, 1024, ((2000, 1), (333, 2))),   # whole tiles; the second call smaller, so a stale row would show
    (2560, 8192, ((2048, 3), (1900, 4))),  # K >= 8192 with a full wave: stream-K; 2048 x 8192 is the limit
])
def test_noalloc_matches_mul_mat_and_reference_twice(N, K, calls):
    torch.cuda.set_device(0)
    npu = Z.Npu(0)
    npu.set_out16(False)
    raw = O.quantize(O.Q8_0, O.weights_f32(N, K, 3))
    key = Z.Npu.key(raw.ctypes.data, O.Q8_0, K, N)
    npu.add_weight(key, raw.ctypes.data, on_device=False)
    w_ptr, n_pad = npu.weight_bf16(key)
    assert w_ptr and n_pad >= N
    wd = _decoded(O.dequant(O.Q8_0, raw, N, K))
    assert Z.plan_gemm(calls[0][0], K, [N])["stream_k"] == (1 if K >= 8192 else 0)
    for T, seed in calls:
        x_host = O.activations(T, K, seed)
        x = torch.from_numpy(x_host).cuda()
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
        # the same kernels on the same operands as zest_mul_mat: identical
        assert np.array_equal(g, w)
        # and the reference's CPU matmul on the bfp16-rounded operands, on the
        # first and last row of every 256-row tile block
        rows = np.unique(np.r_[np.arange(0, T, 256), np.minimum(np.arange(255, T + 255, 256), T - 1)])
        ref = O.ref_mul_mat(O.F32, wd.view(np.uint8), N, K, _decoded(x_host[rows]))
        assert O.nmax_err(g[rows], ref) <= TOL
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
