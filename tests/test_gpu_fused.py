"""The block executor's ops fused into the kernels beside them, through the
C ABI: RMS_NORM + MUL + K2's pack, per-head RMS_NORM + MUL + ROPE, and K3's
epilogues (the residual ADD; SwiGLU writing the next GEMM's packed operand).
Each is held to the bits of the same ops run one after another on the GPU,
and, for the float ops, to the oracle's restatement of the reference's
run_rows within the reference's small-op bar (nrmse 1e-5)."""
import ctypes

import numpy as np
import pytest
import torch

import zest_b200 as Z
from oracle import oracle as O
from gpu_util import dev, host

pytestmark = pytest.mark.gpu
EXACT = 1e-5
_alive = []


def p(t):
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def sp():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def call(name, *args):
    L = Z.lib()
    rc = getattr(L, name)(*args, sp())
    assert rc == 0, L.zest_last_error().decode()


def normal(shape, seed, scale=1.5):
    return (np.random.default_rng(seed).standard_normal(shape) * scale).astype(np.float32)


@pytest.mark.parametrize("with_w", [True, False])
@pytest.mark.parametrize("T,K", [(1000, 2560), (2048, 4096), (37, 512)])
def test_pack_rms_norm_equals_separate_ops(T, K, with_w):
    x = dev(normal((T, K), T + K))
    w = dev(np.random.default_rng(1).uniform(0.5, 1.5, K).astype(np.float32)) if with_w else None
    m_pad = Z.pad_to(T, 128)
    a = torch.full((m_pad, K), 0x5555, dtype=torch.int16, device="cuda")
    y = torch.empty((T, K), device="cuda")
    call("zest_pack_rms_norm", p(x), T, K, K, ctypes.c_float(1e-6), p(w), p(y), K, m_pad, p(a), K)
    # the same ops one after another
    yn = torch.empty((T, K), device="cuda")
    call("zest_rms_norm", p(x), T, K, ctypes.c_float(1e-6), p(yn))
    if with_w:
        call("zest_mul_row", p(yn), p(w), T, K, p(yn))
    _, a_ref = Z.pack_activations(yn, m_pad=m_pad, want_bytes=False)
    torch.cuda.synchronize()
    assert torch.equal(y, yn)
    assert torch.equal(a, a_ref)
    want = O.rms_norm(host(x), K, 1e-6)
    if with_w:
        want = O.mul_row(want, host(w))
    assert O.nrmse(host(y), want) <= EXACT
    # without the f32 output, the same operand
    a2 = torch.empty_like(a)
    call("zest_pack_rms_norm", p(x), T, K, K, ctypes.c_float(1e-6), p(w), None, 0, m_pad, p(a2), K)
    torch.cuda.synchronize()
    assert torch.equal(a2, a)


@pytest.mark.parametrize("mode,n_dims", [(Z.ROPE_NEOX, 128), (Z.ROPE_NORMAL, 128), (Z.ROPE_NEOX, 64)])
def test_norm_rope_equals_separate_ops(mode, n_dims):
    T, H, HD = 300, 8, 128
    x = dev(normal((T, H, HD), 3))
    w = dev(np.random.default_rng(4).uniform(0.5, 1.5, HD).astype(np.float32))
    pos = (5000 + 3 * np.arange(T)).astype(np.int32)
    par = np.array([1000000.0, 1.0, 0.0, 1.0, 32.0, 1.0], np.float32)
    table = torch.empty((T, n_dims), device="cuda")
    posd = dev(pos)
    L = Z.lib()
    assert L.zest_rope_table(p(posd), T, n_dims, 40960, par.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), None,
                             p(table), sp()) == 0
    y = torch.empty((T, H, HD), device="cuda")
    y16 = torch.empty((T, H, HD), dtype=torch.int16, device="cuda")
    call("zest_norm_rope", p(x), T, H, HD, ctypes.c_float(1e-6), p(w), n_dims, mode, p(table), p(y), p(y16))
    # separate ops
    yn = torch.empty((T * H, HD), device="cuda")
    call("zest_rms_norm", p(x), T * H, HD, ctypes.c_float(1e-6), p(yn))
    call("zest_mul_row", p(yn), p(w), T * H, HD, p(yn))
    yr = torch.empty((T, H, HD), device="cuda")
    call("zest_rope", p(yn), T, H, HD, n_dims, mode, p(table), p(yr))
    torch.cuda.synchronize()
    assert O.nrmse(host(y), host(yr)) <= 1e-6  # the per-head sum runs in a warp, not a block
    assert torch.equal(y16, y.to(torch.bfloat16).view(torch.int16))
    want = O.rope(O.mul_row(O.rms_norm(host(x).reshape(T * H, HD), HD, 1e-6), host(w)).reshape(T, H, HD), n_dims,
                  mode, O.rope_table(pos, n_dims, 40960, par))
    assert O.nrmse(host(y), want) <= EXACT


def operands(M, N, K, seed):
    _, ah = Z.pack_activations(dev(O.activations(M, K, seed)))
    _, bh = Z.convert_weight(O.Q8_0, dev(O.quantize(O.Q8_0, O.weights_f32(N, K, seed + 1))), N, K)
    return ah, bh


def segs(*items):
    arr = (Z.GemmSeg * len(items))(*items)
    _alive.append(arr)
    return arr


@pytest.mark.parametrize("M", [900, 100])  # the CTA-pair kernel and the one-CTA kernel
@pytest.mark.parametrize("ldc_pad", [0, 1])  # TMA-stored rows, and direct stores (rows not 16-byte aligned)
def test_gemm_residual_add(M, ldc_pad):
    N, K = 768, 512
    ah, bh = operands(M, N, K, 5)
    ldc = N + ldc_pad
    resid = dev(normal((M, ldc), 6))
    c = torch.empty((M, ldc), device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    s = segs(Z.GemmSeg(bh.data_ptr(), K, N, Z.MODE_BF16, c.data_ptr(), ldc, resid.data_ptr(), ldc, None, 0))
    call("zest_gemm_segs", p(ah), K, M, K, 1, s, p(err))
    plain = host(Z.gemm(ah, bh, M, N, Z.MODE_BF16))
    got = host(c)[:, :N]
    assert np.array_equal(got, host(resid)[:, :N] + plain)  # f32 add of the same operands
    # in place: the residual stream updated where it lies (x += o)
    x = resid.clone()
    s = segs(Z.GemmSeg(bh.data_ptr(), K, N, Z.MODE_BF16, x.data_ptr(), ldc, x.data_ptr(), ldc, None, 0))
    call("zest_gemm_segs", p(ah), K, M, K, 1, s, p(err))
    assert np.array_equal(host(x)[:, :N], got)
    assert int(err.item()) == 0


@pytest.mark.parametrize("with_c", [True, False])
@pytest.mark.parametrize("M", [1000, 128])
def test_gemm_swiglu_writes_next_operand(M, with_c):
    F, K = 600, 512
    gr = O.quantize(O.Q4_K, O.weights_f32(F, K, 7))
    ur = O.quantize(O.Q4_K, O.weights_f32(F, K, 8))
    _, gu = Z.convert_gate_up(O.Q4_K, dev(gr), dev(ur), F, K)
    _, ah = Z.pack_activations(dev(O.activations(M, K, 9)))
    n = gu.shape[0]
    plain = Z.gemm(ah, gu, M, n, Z.MODE_SWIGLU)  # [M][f_pad] f32
    f_pad = n // 2
    _, want = Z.pack_activations(plain.contiguous(), want_bytes=False)
    a_next = torch.full((Z.pad_to(M, 128), f_pad), 0x5555, dtype=torch.int16, device="cuda")
    c = torch.empty((M, f_pad), device="cuda") if with_c else None
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    s = segs(Z.GemmSeg(gu.data_ptr(), K, n, Z.MODE_SWIGLU, c.data_ptr() if with_c else None, f_pad, None, 0,
                       a_next.data_ptr(), f_pad))
    call("zest_gemm_segs", p(ah), K, M, K, 1, s, p(err))
    torch.cuda.synchronize()
    assert torch.equal(a_next[:M], want[:M])
    if with_c:
        assert torch.equal(c, plain)
    assert int(err.item()) == 0


def test_gemm_segs_rejects_bad_epilogues():
    ah, bh = operands(256, 512, 64, 1)
    c = torch.empty((256, 512), device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    L = Z.lib()
    bad = [Z.GemmSeg(bh.data_ptr(), 64, 512, Z.MODE_SWIGLU, c.data_ptr(), 512, c.data_ptr(), 512, None, 0),
           Z.GemmSeg(bh.data_ptr(), 64, 512, Z.MODE_F32, c.data_ptr(), 512, None, 0, c.data_ptr(), 512),
           Z.GemmSeg(bh.data_ptr(), 64, 512, Z.MODE_F32, None, 0, None, 0, None, 0)]
    for sg in bad:
        assert L.zest_gemm_segs(p(ah), 64, 256, 64, 1, segs(sg), p(err), sp()) != 0


def test_gemm_peer_copies_equal_the_output():
    # an N-shard's all-gather from the epilogue: each tile TMA-stored into up
    # to 7 further buffers laid out as c (here buffers of this GPU standing in
    # for the peers' copies), at the slab's column offset in a wider output;
    # every copy holds the output's bits, and columns outside the slab stay
    M, N, K, W, off = 900, 768, 512, 1280, 256  # a 768-column slab at column 256 of a 1280-wide output
    ah, bh = operands(M, N, K, 9)
    outs = [torch.full((M, W), 7.0, device="cuda") for _ in range(8)]
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    peers = (ctypes.c_void_p * 7)(*[o.data_ptr() + 4 * off for o in outs[1:]])
    _alive.append(peers)
    s = segs(Z.GemmSeg(bh.data_ptr(), K, N, Z.MODE_BF16, outs[0].data_ptr() + 4 * off, W, None, 0, None, 0, None, 0,
                       ctypes.cast(peers, ctypes.POINTER(ctypes.c_void_p)), 7))
    call("zest_gemm_segs", p(ah), K, M, K, 1, s, p(err))
    plain = host(Z.gemm(ah, bh, M, N, Z.MODE_BF16))
    for o in outs:
        h = host(o)
        assert np.array_equal(h[:, off:off + N], plain)
        assert (h[:, :off] == 7.0).all() and (h[:, off + N:] == 7.0).all()
    assert int(err.item()) == 0
    # what the epilogue cannot do is refused: peers of a one-CTA launch (M <= 128)
    # or of an output without TMA stores (rows not 16-byte aligned)
    L = Z.lib()
    s = segs(Z.GemmSeg(bh.data_ptr(), K, N, Z.MODE_BF16, outs[0].data_ptr() + 4 * off, W, None, 0, None, 0, None, 0,
                       ctypes.cast(peers, ctypes.POINTER(ctypes.c_void_p)), 7))
    assert L.zest_gemm_segs(p(ah), K, 100, K, 1, s, p(err), sp()) != 0
    assert b"more than 128 rows" in L.zest_last_error()
    s = segs(Z.GemmSeg(bh.data_ptr(), K, N, Z.MODE_BF16, outs[0].data_ptr() + 4 * off + 4, W, None, 0, None, 0, None,
                       0, ctypes.cast(peers, ctypes.POINTER(ctypes.c_void_p)), 7))
    assert L.zest_gemm_segs(p(ah), K, M, K, 1, s, p(err), sp()) != 0
    assert b"peer copies need" in L.zest_last_error()


def test_gemm_bf16_copies_widen_to_the_output():
    # the N-shard's half-bytes all-gather: each tile TMA-stored in bf16 into up
    # to 8 buffers (here this GPU's, standing in for every GPU's whole bf16
    # output) at the slab's column offset; widened back to f32 they hold the
    # bf16-mode output's bits, and the columns outside the slab stay
    M, N, K, W, off = 900, 768, 512, 1280, 256
    ah, bh = operands(M, N, K, 11)
    fill = torch.tensor([7.0], dtype=torch.bfloat16).view(torch.int16).item()
    c16 = [torch.full((M, W), fill, dtype=torch.int16, device="cuda") for _ in range(8)]
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    ptrs = (ctypes.c_void_p * 8)(*[c.data_ptr() + 2 * off for c in c16])
    _alive.append(ptrs)
    cp = ctypes.cast(ptrs, ctypes.POINTER(ctypes.c_void_p))
    s = segs(Z.GemmSeg(bh.data_ptr(), K, N, Z.MODE_BF16, None, 0, None, 0, None, 0, None, 0, None, 0, cp, 8, W))
    call("zest_gemm_segs", p(ah), K, M, K, 1, s, p(err))
    plain = host(Z.gemm(ah, bh, M, N, Z.MODE_BF16))
    for c in c16:
        wide = torch.empty((M, W), device="cuda")
        call("zest_widen_bf16", p(c), M * W, p(wide))
        h = host(wide)
        assert np.array_equal(h[:, off:off + N].view(np.uint32), plain.view(np.uint32))
        assert (h[:, :off] == 7.0).all() and (h[:, off + N:] == 7.0).all()
    assert int(err.item()) == 0
    # a ragged length widens exactly too
    x = torch.randn(1003, device="cuda").to(torch.bfloat16)
    y = torch.empty(1003, device="cuda")
    call("zest_widen_bf16", p(x), 1003, p(y))
    assert torch.equal(y, x.float())
    # bf16 copies of fp32-mode results, or beside an f32 output, are refused
    L = Z.lib()
    for mode, c in ((Z.MODE_F32, None), (Z.MODE_BF16, c16[0].data_ptr())):
        s = segs(Z.GemmSeg(bh.data_ptr(), K, N, mode, c, W, None, 0, None, 0, None, 0, None, 0, cp, 8, W))
        assert L.zest_gemm_segs(p(ah), K, M, K, 1, s, p(err), sp()) != 0
        assert b"bf16 copies take" in L.zest_last_error()
