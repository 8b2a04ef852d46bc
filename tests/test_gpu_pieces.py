"""Claimed pieces end to end through the plugin's graph_compute: the blocks
the reference's block claiming takes (norm -> gate/up -> SwiGLU -> down ->
residual add; norm -> q -> per-head norm -> rope), every op on the GPU, the
SwiGLU fused into one GEMM, checked against the oracle's chain of the same
ops (bf16-rounded matmul outputs, as the reference's default)."""
import os
import sys

import numpy as np
import pytest
import torch

sys.path.insert(0, os.path.join(os.path.dirname(__file__), "ggml_harness"))
from harness import F32, I32, Harness, Q4_K, Q8_0, STATUS_SUCCESS, USAGE_COMPUTE, USAGE_WEIGHTS  # noqa: E402

from oracle import oracle as O  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def h():
    return Harness()


def dec(v: np.ndarray) -> np.ndarray:
    return O.decode_blocks(O.encode_blocks(v)).reshape(v.shape)


def mm_bf16(w_vals: np.ndarray, x: np.ndarray) -> np.ndarray:
    return O.round_bf16(O.mul_mat(dec(w_vals), dec(x)))


class Buffers:
    """Device memory for a piece's tensors, as ggml's allocator would hand out."""

    def __init__(self, h):
        self.h, self.keep = h, []

    def dev(self, a: np.ndarray):
        t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
        self.keep.append(t)
        return t.data_ptr()

    def out(self, *shape, fill=float("nan")):
        t = torch.full(shape, fill, dtype=torch.float32, device="cuda")
        self.keep.append(t)
        return t


@pytest.mark.parametrize("keep", [False, True])
def test_ffn_piece_with_fused_swiglu(h, keep):
    # keep=False: only the block's output is read outside the piece, so the
    # norm rides in the pack, gate/up in one SwiGLU GEMM that hands down its
    # packed result, and the residual ADD in down's epilogue: the
    # intermediates are never written. keep=True: they are graph outputs, so
    # each is computed and written.
    K, F, T = 1024, 2816, 1024
    rng = np.random.default_rng(1)
    x = (rng.standard_normal((T, K)) * 1.5).astype(np.float32)
    wn = rng.uniform(0.5, 1.5, K).astype(np.float32)
    g_raw = O.quantize(Q4_K, O.weights_f32(F, K, 2))
    u_raw = O.quantize(Q4_K, O.weights_f32(F, K, 3))
    d_raw = O.quantize(Q8_0, O.weights_f32(K, F, 4))
    B = Buffers(h)
    W = h.buffer(USAGE_WEIGHTS)
    C = h.buffer(USAGE_COMPUTE)
    xt = h.tensor(F32, [K, T], "x", C, B.dev(x))
    wnt = h.tensor(F32, [K], "blk.0.ffn_norm.weight", W, B.dev(wn))
    n1 = h.rms_norm(xt, 1e-6, name="norm", buffer=C, data=B.out(T, K).data_ptr())
    m = B.out(T, K)
    n2 = h.mul(n1, wnt, name="ffn_inp", buffer=C, data=m.data_ptr())
    gw = h.tensor(Q4_K, [K, F], "blk.0.ffn_gate.weight", W, B.dev(g_raw))
    uw = h.tensor(Q4_K, [K, F], "blk.0.ffn_up.weight", W, B.dev(u_raw))
    dw = h.tensor(Q8_0, [F, K], "blk.0.ffn_down.weight", W, B.dev(d_raw))
    g_out, u_out = B.out(T, F), B.out(T, F)
    g = h.mul_mat(gw, n2, "gate", C, g_out.data_ptr())
    u = h.mul_mat(uw, n2, "up", C, u_out.data_ptr())
    s_out = B.out(T, F)
    s = h.glu(g, u, kind=2, name="swiglu", buffer=C, data=s_out.data_ptr())
    d_out = B.out(T, K)
    dn = h.mul_mat(dw, s, "down", C, d_out.data_ptr())
    y = B.out(T, K)
    out = h.add(dn, xt, name="ffn_out", buffer=C, data=y.data_ptr())
    out.flags = 2  # GGML_TENSOR_FLAG_OUTPUT
    if keep:
        n2.flags = s.flags = dn.flags = 2
    nodes = [n1, n2, g, u, s, dn, out]
    for nd in nodes:  # the scheduler asks about every op: this records who reads what
        h.supports_op(nd)
    assert h.supports_op(s) and h.supports_op(out)
    plan = h.piece_plan(nodes)
    assert (plan["norm"], plan["handoff"], plan["add"]) == ((0, 0, 0) if keep else (1, 1, 1)), plan
    b, _ = h.init_backend()
    torch.cuda.synchronize()
    h.graph_optimize(b, nodes)
    assert h.graph_compute(b, [xt] + nodes) == STATUS_SUCCESS
    torch.cuda.synchronize()
    # the gate and up results were never written: one fused GEMM produced the SwiGLU
    assert torch.isnan(g_out).all() and torch.isnan(u_out).all()
    xm = O.mul_row(O.rms_norm(x, K, 1e-6), wn)
    gv = O.mul_mat(dec(O.dequant(Q4_K, g_raw, F, K)), dec(xm))
    uv = O.mul_mat(dec(O.dequant(Q4_K, u_raw, F, K)), dec(xm))
    sv = O.swiglu_bf16(gv, uv)
    want = O.add(mm_bf16(O.dequant(Q8_0, d_raw, K, F), sv), x)
    assert O.nrmse(y.cpu().numpy(), want) <= 1e-3
    if keep:
        assert O.nrmse(m.cpu().numpy(), xm) <= 1e-5
        assert O.nrmse(s_out.cpu().numpy(), sv) <= 1e-3
        assert O.nrmse(d_out.cpu().numpy(), mm_bf16(O.dequant(Q8_0, d_raw, K, F), sv)) <= 1e-3
    else:
        assert torch.isnan(m).all() and torch.isnan(s_out).all() and torch.isnan(d_out).all()
    h.backend_free(b)


def test_attention_input_piece_with_rope(h):
    K, HD, H, T = 1024, 128, 8, 1024
    rng = np.random.default_rng(5)
    x = (rng.standard_normal((T, K)) * 1.5).astype(np.float32)
    wn = rng.uniform(0.5, 1.5, K).astype(np.float32)
    wqn = rng.uniform(0.5, 1.5, HD).astype(np.float32)
    q_raw = O.quantize(Q4_K, O.weights_f32(H * HD, K, 6))
    pos = (np.arange(T) + 4096).astype(np.int32)
    B = Buffers(h)
    W, C = h.buffer(USAGE_WEIGHTS), h.buffer(USAGE_COMPUTE)
    xt = h.tensor(F32, [K, T], "x", C, B.dev(x))
    n1 = h.rms_norm(xt, name="attn_norm", buffer=C, data=B.out(T, K).data_ptr())
    n2 = h.mul(n1, h.tensor(F32, [K], "blk.0.attn_norm.weight", W, B.dev(wn)), name="attn_inp", buffer=C,
               data=B.out(T, K).data_ptr())
    q_out = B.out(T, H * HD)
    q = h.mul_mat(h.tensor(Q4_K, [K, H * HD], "blk.0.attn_q.weight", W, B.dev(q_raw)), n2, "q", C, q_out.data_ptr())
    q3 = h.tensor(F32, [HD, H, T], "q3", C, q_out.data_ptr(), op="RESHAPE", src=(q,), view_src=q)
    qn = h.rms_norm(q3, name="q_norm", buffer=C, data=B.out(T, H, HD).data_ptr())
    qm = h.mul(qn, h.tensor(F32, [HD], "blk.0.attn_q_norm.weight", W, B.dev(wqn)), name="q_normed", buffer=C,
               data=B.out(T, H, HD).data_ptr())
    post = h.tensor(I32, [T], "pos", h.buffer(USAGE_COMPUTE, host=True), pos.ctypes.data, flags=1)
    r_out = B.out(T, H, HD)
    qr = h.rope(qm, post, HD, 2, freq_base=1000000.0, name="q_rope", buffer=C, data=r_out.data_ptr())
    nodes = [n1, n2, q, q3, qn, qm, qr]
    for nd in nodes:
        h.supports_op(nd)
    plan = h.piece_plan(nodes)
    assert (plan["norm"], plan["rope"]) == (1, 1), plan  # the norms ride in the pack and in the rope kernel
    b, _ = h.init_backend()
    torch.cuda.synchronize()
    assert h.graph_compute(b, nodes) == STATUS_SUCCESS
    torch.cuda.synchronize()
    xm = O.mul_row(O.rms_norm(x, K, 1e-6), wn)
    qv = mm_bf16(O.dequant(Q4_K, q_raw, H * HD, K), xm).reshape(T, H, HD)
    assert O.nrmse(q_out.cpu().numpy().reshape(T, H, HD), qv) <= 1e-3
    qmv = O.mul_row(O.rms_norm(q_out.cpu().numpy().reshape(T * H, HD), HD, 1e-6), wqn).reshape(T, H, HD)
    par = np.array([1000000.0, 1.0, 0.0, 1.0, 32.0, 1.0], np.float32)
    want = O.rope(qmv, HD, 2, O.rope_table(pos, HD, 0, par))
    assert O.nrmse(r_out.cpu().numpy(), want) <= 1e-5
    h.backend_free(b)


@pytest.mark.parametrize("host", [False, True])
def test_qkv_piece_grouped(h, host):
    # q, k and v on one input run as one grouped call at q's turn, with q's
    # per-head norm between them in the node order; inputs and outputs in
    # device memory, or all in host memory (chunked copies)
    K, T = 1024, 1100
    HD, HQ, HK = 128, 8, 2
    rng = np.random.default_rng(9)
    x = (rng.standard_normal((T, K)) * 1.5).astype(np.float32)
    raws = {n: O.quantize(Q4_K, O.weights_f32(rows, K, 10 + i))
            for i, (n, rows) in enumerate([("q", HQ * HD), ("k", HK * HD), ("v", HK * HD)])}
    B = Buffers(h)
    W = h.buffer(USAGE_WEIGHTS)
    C = h.buffer(USAGE_COMPUTE, host=host)
    keep = []

    def buf(*shape, src=None):
        if host:
            a = np.full(shape, np.nan, np.float32) if src is None else np.ascontiguousarray(src)
            keep.append(a)
            return a.ctypes.data, a
        t = B.out(*shape) if src is None else torch.from_numpy(np.ascontiguousarray(src)).cuda()
        keep.append(t)
        return t.data_ptr(), t

    xp, _ = buf(T, K, src=x)
    xt = h.tensor(F32, [K, T], "x", C, xp)
    outs, nodes = {}, []
    wts = {n: h.tensor(Q4_K, [K, r.size // (K // 256 * 144)], f"blk.0.attn_{n}.weight", W, B.dev(r))
           for n, r in raws.items()}
    qp, outs["q"] = buf(T, HQ * HD)
    q = h.mul_mat(wts["q"], xt, "q", C, qp)
    q3 = h.tensor(F32, [HD, HQ, T], "q3", C, qp, op="RESHAPE", src=(q,), view_src=q)
    qnp, qn_out = buf(T, HQ, HD)
    qn = h.rms_norm(q3, name="q_norm", buffer=C, data=qnp)
    kp, outs["k"] = buf(T, HK * HD)
    kk = h.mul_mat(wts["k"], xt, "k", C, kp)
    vp, outs["v"] = buf(T, HK * HD)
    v = h.mul_mat(wts["v"], xt, "v", C, vp)
    nodes = [q, q3, qn, kk, v]
    assert h.piece_groups(nodes) == [3]
    for nd in nodes:
        h.supports_op(nd)
    b, _ = h.init_backend()
    torch.cuda.synchronize()
    assert h.graph_compute(b, nodes) == STATUS_SUCCESS
    torch.cuda.synchronize()
    for n, r in raws.items():
        rows = r.size // (K // 256 * 144)
        got = outs[n] if host else outs[n].cpu().numpy()
        assert O.nrmse(got, mm_bf16(O.dequant(Q4_K, r, rows, K), x)) <= 1e-3, n
    qv = outs["q"] if host else outs["q"].cpu().numpy()
    qnv = qn_out if host else qn_out.cpu().numpy()
    assert O.nrmse(qnv.reshape(T * HQ, HD), O.rms_norm(qv.reshape(T * HQ, HD), HD, 1e-6)) <= 1e-5
    h.backend_free(b)
