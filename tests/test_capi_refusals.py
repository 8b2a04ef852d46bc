"""The C ABI's refusals on the host: calls with shapes, strides, modes or
outputs the kernels do not take return -1 with the reason in
zest_last_error(), before any device work, as the reference's service
returns false with its error string. The device pointers here are never
dereferenced on a refused call; so that a refusal that failed to trigger
could never launch a kernel on them, these tests do not run where a GPU is
present (the GPU tests cover the same calls with real buffers)."""
import ctypes

import pytest

import zest_b200 as Z

try:
    import torch
    _gpu = torch.cuda.is_available()
except ImportError:
    _gpu = False

pytestmark = pytest.mark.skipif(_gpu, reason="host-only: fake device pointers")

P = 0x100000   # a 16-byte aligned stand-in for a device pointer (never dereferenced)
ODD = P + 4    # not 16-byte aligned
vp = ctypes.c_void_p


def refused(rc: int, words: str) -> None:
    assert rc == -1
    msg = Z.lib().zest_last_error().decode()
    assert words in msg, msg


def gemm(M=256, N=512, K=128, lda=128, ldb=128, mode=Z.MODE_F32, a=P, b=P, c=P, ldc=512, err=P):
    return Z.lib().zest_gemm(vp(a), lda, vp(b), ldb, M, N, K, mode, vp(c), ldc, vp(err), None)


def test_gemm_refuses_what_the_kernel_cannot_take():
    refused(gemm(K=100, lda=100, ldb=100), "multiples of 8")
    refused(gemm(lda=120), "multiples of 8")
    refused(gemm(a=ODD), "16-byte aligned")
    refused(gemm(b=ODD), "16-byte aligned")
    refused(gemm(err=0), "no device error word")
    refused(gemm(mode=7), "bad output mode")
    refused(gemm(N=520, mode=Z.MODE_SWIGLU), "bad output mode")  # SwiGLU pairs 8 + 8 columns
    refused(gemm(c=0), "no output")
    refused(gemm(ldc=500), "ldc smaller")


def seg(**kw):
    d = dict(b=P, ldb=128, N=512, mode=Z.MODE_BF16, c=P, ldc=512, residual=None, ldr=0, a_next=None, lda_next=0,
             c_multicast=None)
    d.update(kw)
    return Z.GemmSeg(**d)


def segs(*items, M=256, K=128, n=None):
    arr = (Z.GemmSeg * len(items))(*items)
    return Z.lib().zest_gemm_segs(vp(P), K, M, K, len(items) if n is None else n, arr, vp(P), None)


def test_fused_epilogues_refuse_impossible_combinations():
    refused(segs(seg(mode=Z.MODE_SWIGLU, residual=P, ldr=256)), "residual")
    refused(segs(seg(residual=P, ldr=100)), "residual")
    refused(segs(seg(a_next=P, lda_next=256)), "next operand")  # a hand-off needs SwiGLU
    refused(segs(seg(mode=Z.MODE_SWIGLU, a_next=ODD, lda_next=256)), "next operand")
    refused(segs(seg(c_multicast=P)), "multicast")  # with c too
    refused(segs(seg(c=None, c_multicast=P, mode=Z.MODE_SWIGLU)), "multicast")
    refused(segs(seg(), n=0), "1 to 4")
    refused(segs(*[seg()] * 5), "1 to 4")


def test_group_refuses_bad_counts():
    L = Z.lib()
    arr = lambda t, v: (t * len(v))(*v)
    for n in (0, 5):
        k = max(n, 1)
        rc = L.zest_gemm_group(vp(P), 128, 256, 128, n, arr(vp, [P] * k), arr(ctypes.c_int64, [128] * k),
                               arr(ctypes.c_int64, [512] * k), arr(ctypes.c_int, [0] * k), arr(vp, [P] * k),
                               arr(ctypes.c_int64, [512] * k), vp(P), None)
        refused(rc, "1 to 4")


def test_pack_refuses_unaligned_shapes():
    L = Z.lib()
    refused(L.zest_pack_activations(vp(P), 100, 96, 96, 128, None, vp(P), 96, None), "multiple of 64")
    refused(L.zest_pack_activations(vp(P), 100, 128, 128, 100, None, vp(P), 128, None), "multiple of 128")
    refused(L.zest_pack_activations(vp(P), 300, 128, 128, 256, None, vp(P), 128, None), "covering T")
    refused(L.zest_pack_activations(vp(ODD), 100, 128, 128, 128, None, vp(P), 128, None), "16-byte aligned")
    refused(L.zest_pack_activations(vp(P), 100, 128, 128, 128, None, vp(ODD), 128, None), "16-byte aligned")


def test_convert_refuses_bad_rows_types_and_padding():
    L = Z.lib()
    Q8 = Z.TYPE_Q8_0  # type 3 (ggml's Q4_1) has no GPU converter
    refused(L.zest_convert_weight(Q8, vp(P), 100, 90, 20, 128, 512, None, vp(P), None), "rows out of range")
    refused(L.zest_convert_weight(3, vp(P), 100, 0, 100, 128, 512, None, vp(P), None), "unsupported weight type")
    refused(L.zest_convert_weight(Q8, vp(P), 100, 0, 100, 100, 512, None, vp(P), None), "multiple of 64")
    refused(L.zest_convert_weight(Q8, vp(P), 100, 0, 100, 128, 500, None, vp(P), None), "n_pad of 512")
    refused(L.zest_convert_weight(Q8, vp(P), 600, 0, 600, 128, 512, None, vp(P), None), "n_pad too small")
    refused(L.zest_convert_gate_up(Q8, vp(P), vp(P), 300, 0, 300, 128, 300, None, vp(P), None), "multiple of 256")


def test_service_refuses_without_a_service():
    L = Z.lib()
    key = Z.WKey()
    refused(L.zest_mul_mat(None, None, 0, None, 10, None, 1), "no service or key")
    refused(L.zest_mul_mat_group(None, 1, ctypes.byref(key), None, None, 10, None, 1), "not 1 to 4")
    refused(L.zest_take_times(None, None), "no service")
    refused(L.zest_submit_group(None, 0, 1, ctypes.byref(key), None, None, 10, None, 0), "no service")
    refused(L.zest_wait_group(None, 0), "no service")
    refused(L.zest_load_iq3s_grid(None), "no table")


def ptrs(*vals):
    arr = (vp * len(vals))(*vals)
    ptrs._alive.append(arr)
    return ctypes.cast(arr, ctypes.POINTER(vp))


ptrs._alive = []


def test_epilogue_copies_refuse_what_the_epilogue_cannot_store():
    # peer copies (an N-shard's all-gather in f32): a TMA-stored output, 0..7 aligned peers
    refused(segs(seg(c_peers=ptrs(P), n_peers=8)), "0 to 7 peer copies")
    refused(segs(seg(c_peers=None, n_peers=1)), "0 to 7 peer copies")
    refused(segs(seg(c=None, c_multicast=P, c_peers=ptrs(P), n_peers=1)), "peer copies need")
    refused(segs(seg(ldc=513, c_peers=ptrs(P), n_peers=1)), "peer copies need")
    refused(segs(seg(c_peers=ptrs(ODD), n_peers=1)), "16-byte aligned")
    # bf16 copies (the all-gather in bf16): bf16-mode results alone, 1..8 aligned copies
    refused(segs(seg(c=None, c16=ptrs(P), n_c16=1, ldc16=512, mode=Z.MODE_F32)), "bf16 copies take")
    refused(segs(seg(c16=ptrs(P), n_c16=1, ldc16=512)), "bf16 copies take")  # beside an f32 output
    refused(segs(seg(c=None, c16=ptrs(*[P] * 9), n_c16=9, ldc16=512)), "bf16 copies take")
    refused(segs(seg(c=None, c16=ptrs(P), n_c16=1, ldc16=500)), "bf16 copies take")
    refused(segs(seg(c=None, c16=ptrs(ODD), n_c16=1, ldc16=512)), "16-byte aligned")


def test_widen_refuses_unaligned_buffers():
    L = Z.lib()
    refused(L.zest_widen_bf16(vp(ODD), 100, vp(P), None), "16-byte aligned")
    refused(L.zest_widen_bf16(vp(P), 100, vp(ODD), None), "16-byte aligned")
    assert L.zest_widen_bf16(vp(ODD), 0, vp(ODD), None) == 0  # nothing to do
