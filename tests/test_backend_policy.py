"""The ggml plugin's boundary on the host (no GPU needed): registration,
the device vtable, and the dispatch gate's truth table, mirroring the
reference's tests/test-dispatch-gate.cpp:50-153 (with block claiming off,
as this build claims matmuls only). The plugin is the real
libggml-zest.so, driven through the stand-in ggml-base."""
import ctypes
import os
import subprocess
import sys

import pytest

sys.path.insert(0, os.path.join(os.path.dirname(__file__), "ggml_harness"))
from harness import (DEV_IGPU, F16, F32, FLAG_INPUT, IQ3_S, Harness, Props, Q4_0, Q4_K, Q8_0, Tensor,  # noqa: E402
                     USAGE_COMPUTE, USAGE_WEIGHTS, fn)


@pytest.fixture(scope="module")
def h():
    return Harness()


def mm(h, wtype, k, n, batch, weight_op="NONE"):
    w = h.tensor(wtype, [k, n], name="blk.0.attn_q.weight", buffer=h.buffer(USAGE_WEIGHTS), op=weight_op)
    x = h.tensor(F32, [k, batch], buffer=h.buffer(USAGE_COMPUTE))
    return h.mul_mat(w, x)


def test_abi_sizes():
    assert ctypes.sizeof(Tensor) == 336  # ggml_tensor on LP64
    assert ctypes.sizeof(Props) == 56


def test_registration(h):
    assert h.reg_name() == "XDNA"
    assert h.reg().api_version >= 1
    assert h.plugin.ggml_backend_score() == 1
    assert ctypes.addressof(h.plugin.ggml_backend_init().contents) == ctypes.addressof(h.reg())


def test_device_vtable(h):
    p, d = h.device()
    assert fn(d.iface.get_name, ctypes.c_char_p, ctypes.c_void_p)(p) == b"XDNA0"
    assert fn(d.iface.get_type, ctypes.c_int, ctypes.c_void_p)(p) == DEV_IGPU
    free, total = ctypes.c_size_t(1), ctypes.c_size_t(0)
    fn(d.iface.get_memory, None, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p)(p, ctypes.byref(free),
                                                                                  ctypes.byref(total))
    assert free.value == 0 and total.value > 0, "no free memory: llama.cpp gives it no layers"
    props = Props()
    fn(d.iface.get_props, None, ctypes.c_void_p, ctypes.c_void_p)(p, ctypes.byref(props))
    assert props.name == b"XDNA0" and props.type == DEV_IGPU and not props.caps.async_ and not props.caps.events
    buft = fn(d.iface.get_buffer_type, ctypes.c_void_p, ctypes.c_void_p)(p)
    assert buft == h.fake.fake_cuda_buft(), "its buffer type is the CUDA backend's (no copies between them)"
    sb = fn(d.iface.supports_buft, ctypes.c_bool, ctypes.c_void_p, ctypes.c_void_p)
    assert sb(p, h.fake.fake_cuda_buft()) and sb(p, h.fake.fake_cpu_buft())
    assert not d.iface.offload_op, "no offload_op: that path copies the weights per op"
    assert not d.iface.get_host_buffer_type and not d.iface.event_new


def test_batch_gate(h):
    k = n = 2048
    assert not h.policy(mm(h, Q4_K, k, n, 1)), "batch 1 (reply generation) is not claimed"
    assert not h.policy(mm(h, Q4_K, k, n, 512)), "batch 512 is not claimed"
    assert not h.policy(mm(h, Q4_K, k, n, 1023)), "batch 1023 is not claimed"
    assert h.policy(mm(h, Q4_K, k, n, 1024)), "batch 1024, q4_K 2048x2048 is claimed"
    assert h.policy(mm(h, Q4_0, k, n, 2048)), "batch 2048, q4_0 (dequantised with ggml's to_float) is claimed"
    assert h.policy(mm(h, Q8_0, k, n, 4096))


def test_work_floor(h):
    # 2*1024*64*1024 = 134 MFLOP, under the 256 MFLOP floor
    assert not h.policy(mm(h, Q4_K, 1024, 64, 1024))


def test_weight_must_be_a_plain_leaf(h):
    k, n = 2048, 2048
    cache = h.tensor(F16, [k, 4 * n], buffer=h.buffer(USAGE_COMPUTE))
    view = h.tensor(F16, [k, n], buffer=h.buffer(USAGE_COMPUTE), op="VIEW", view_src=cache)
    x = h.tensor(F32, [k, 1024], buffer=h.buffer(USAGE_COMPUTE))
    assert not h.policy(h.mul_mat(view, x)), "a view (a cache read) is not claimed"
    a = h.tensor(F32, [k, n])
    computed = h.tensor(F32, [k, n], op="ADD", src=(a, a))
    assert not h.policy(h.mul_mat(computed, x)), "a computed left side is not claimed"
    assert not h.policy(computed), "other ops (ADD) are not claimed"


def test_operand_types_and_shapes(h):
    k, n = 2048, 2048
    w = h.tensor(Q4_K, [k, n], buffer=h.buffer(USAGE_WEIGHTS))
    assert not h.policy(h.mul_mat(w, h.tensor(F16, [k, 1024]))), "f16 activations are not claimed"
    assert not h.policy(h.mul_mat(w, h.tensor(F32, [k // 2, 1024]))), "mismatched K is not claimed"
    x3 = h.tensor(F32, [k, 1024, 2])
    assert not h.policy(h.mul_mat(w, x3)), "batched activations are not claimed"
    # K must be a multiple of the bfp16 tile's 64 (the reference's kernel needs K % 64 too)
    w_odd = h.tensor(Q8_0, [65 * 32, 4096], buffer=h.buffer(USAGE_WEIGHTS))
    assert not h.policy(h.mul_mat(w_odd, h.tensor(F32, [65 * 32, 2048])))


def test_mul_mat_id_not_claimed(h):
    experts = h.tensor(Q4_0, [2048, 2048, 8], buffer=h.buffer(USAGE_WEIGHTS))
    rows = h.tensor(F32, [2048, 1, 2048])
    t = h.tensor(F32, [2048, 1, 2048], op="MUL_MAT_ID", src=(experts, rows))
    assert not h.policy(t)
    assert h.policy(mm(h, Q4_0, 2048, 2048, 2048)), "ordinary matmuls are still claimed afterwards"


def test_mixture_of_experts_is_noted(h):
    # src/ggml-zest.cpp:566-655: a MUL_MAT_ID seen while llama.cpp plans the
    # graph makes the first prompt's graph_compute warn that the expert step
    # stays with the GPU backend
    experts = h.tensor(Q4_0, [2048, 2048, 8], buffer=h.buffer(USAGE_WEIGHTS))
    rows = h.tensor(F32, [2048, 1, 2048])
    h.supports_op(h.tensor(F32, [2048, 1, 2048], op="MUL_MAT_ID", src=(experts, rows)))
    notes = h.model_notes()
    assert "mixture-of-experts" in notes and "MUL_MAT_ID" in notes


def test_supports_op_needs_a_usable_gpu(h):
    # supports_op = a usable GPU (start-up self-test) and the policy; without
    # a GPU the plugin still registers but no device is offered and nothing
    # is claimed (tests/test-safe-start.cpp:20-38, its --no-driver case)
    try:
        import torch
        gpu = torch.cuda.is_available()
    except ImportError:
        gpu = False
    t = mm(h, Q4_K, 2048, 2048, 1024)
    assert h.device_count() == (1 if gpu else 0)
    assert h.supports_op(t) == gpu


def test_block_claiming(h):
    # the small ops next to claimed matmuls (test-dispatch-gate.cpp:96-133, the NPU-mode answers)
    k, n = 2048, 2048
    x = h.tensor(F32, [k, 2048], buffer=h.buffer(USAGE_COMPUTE))
    mm1 = h.mul_mat(h.tensor(Q4_0, [k, n], buffer=h.buffer(USAGE_WEIGHTS)), x)
    mm2 = h.mul_mat(h.tensor(Q4_0, [k, n], buffer=h.buffer(USAGE_WEIGHTS)), x)
    assert h.policy(h.add(mm1, mm2)), "an ADD of two claimed matmuls is claimed"
    table = h.tensor(Q4_0, [k, 32000], buffer=h.buffer(USAGE_WEIGHTS))
    emb = h.tensor(F32, [k, 2048], op="GET_ROWS", src=(table, h.tensor(26, [2048])))
    assert not h.policy(h.add(emb, mm1)), "ADD of a matmul and the token embeddings (GET_ROWS) is not claimed"
    assert not h.policy(h.add(mm1, emb)), "... in either order"
    inp = h.tensor(F32, [k, 2048], flags=FLAG_INPUT)
    assert not h.policy(h.add(inp, mm1)), "ADD of a matmul and a graph input is not claimed"
    bias = h.tensor(F32, [n], buffer=h.buffer(USAGE_WEIGHTS))
    assert h.policy(h.add(mm1, bias)), "an ADD of a bias row to a claimed matmul is claimed"
    made = h.scale(h.tensor(F32, [n]), 2.0)
    assert not h.policy(h.add(mm1, made)), "an ADD of a computed row (not a kept leaf) is not claimed"
    assert h.policy(h.scale(mm1, 0.25)), "a SCALE of a claimed matmul is claimed"
    assert h.policy(h.glu(mm1, mm2, kind=1)), "a GeGLU of two claimed matmuls is claimed"
    fused = h.mul_mat(h.tensor(Q4_0, [k, 2 * n], buffer=h.buffer(USAGE_WEIGHTS)), x)
    assert h.policy(h.glu(fused, kind=2)), "a SwiGLU on one matmul holding gate and up is claimed"
    assert not h.policy(h.glu(fused, kind=3)), "an unsupported GLU kind is not claimed"
    normed = h.rms_norm(h.add(mm1, mm2))
    assert h.policy(normed), "an RMS_NORM fed by a claimed ADD is claimed (claims grow out from the matmuls)"
    assert h.policy(h.mul(normed, h.tensor(F32, [k], buffer=h.buffer(USAGE_WEIGHTS))))
    small = h.mul_mat(h.tensor(Q4_0, [k, n], buffer=h.buffer(USAGE_WEIGHTS)), h.tensor(F32, [k, 512]))
    assert not h.policy(h.add(small, small)), "small ops of a short batch are not claimed"


def test_swiglu_fusion_rules(h):
    # find_fusions (src/xdna-exec.cpp:392-431): SiLU(gate) * up as one GEMM only when
    # gate and up share their input and nothing else reads them
    k, f, t = 1024, 2816, 1024

    def ffn(kind=2, split=True, other_input=False, extra_reader=False, gate_output=False):
        x = h.tensor(F32, [k, t], buffer=h.buffer(USAGE_COMPUTE))
        x2 = h.tensor(F32, [k, t], buffer=h.buffer(USAGE_COMPUTE)) if other_input else x
        if split:
            g = h.mul_mat(h.tensor(Q4_K, [k, f], buffer=h.buffer(USAGE_WEIGHTS)), x)
            u = h.mul_mat(h.tensor(Q4_K, [k, f], buffer=h.buffer(USAGE_WEIGHTS)), x2)
            s = h.glu(g, u, kind=kind)
            nodes = [g, u, s]
        else:
            g = h.mul_mat(h.tensor(Q4_K, [k, 2 * f], buffer=h.buffer(USAGE_WEIGHTS)), x)
            s = h.glu(g, kind=kind)
            nodes = [g, s]
        if extra_reader:
            nodes.append(h.scale(g, 2.0))
        if gate_output:
            g.flags = 2
        for nd in nodes:
            h.supports_op(nd)  # records readers, as the scheduler's questions do
        return h.piece_fusions(nodes)

    assert ffn() == 1
    assert ffn(split=False) == 1, "one weight holding gate then up"
    assert ffn(kind=1) == 0, "only SwiGLU runs as the fused epilogue"
    assert ffn(other_input=True) == 0, "gate and up on different inputs"
    assert ffn(extra_reader=True) == 0, "another op in the piece reads the gate"
    assert ffn(gate_output=True) == 0, "the gate is a graph output"


def test_block_ops_env():
    code = ("import sys; sys.path.insert(0, %r); from harness import *; h = Harness(); "
            "x = h.tensor(F32, [2048, 2048]); "
            "mm = h.mul_mat(h.tensor(Q4_K, [2048, 2048], buffer=h.buffer(USAGE_WEIGHTS)), x); "
            "print('ADD', h.policy(h.add(mm, mm)), 'SCALE', h.policy(h.scale(mm, 0.5)))"
            % os.path.join(os.path.dirname(__file__), "ggml_harness"))
    env = dict(os.environ, GGML_XDNA_BLOCK_OPS="ADD")
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env, timeout=120)
    assert "ADD True SCALE False" in out.stdout, out.stdout + out.stderr
    env = dict(os.environ, GGML_XDNA_BLOCK_OPS="SCALE,ADD")
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env, timeout=120)
    assert "ADD True SCALE True" in out.stdout, out.stdout + out.stderr
    env = dict(os.environ, GGML_XDNA_BLOCK_OPS=",")  # given, but naming no op: none taken
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env, timeout=120)
    assert "ADD False SCALE False" in out.stdout, out.stdout + out.stderr
    env = dict(os.environ, GGML_XDNA_BLOCKS="0")
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env, timeout=120)
    assert "ADD False SCALE False" in out.stdout, out.stdout + out.stderr


def test_iq3s_codebook_read_back_through_to_float(h):
    # the plugin builds in no IQ3_S table: it reads ggml's back through the
    # host ggml's to_float (the stand-in's holds the gguf package's codebook)
    got = h.iq3s_codebook()
    assert h.iq3s_grid is not None and got is not None
    assert (got == h.iq3s_grid).all()
    w = h.tensor(IQ3_S, [5120, 17408], buffer=h.buffer(USAGE_WEIGHTS))
    assert h.policy(h.mul_mat(w, h.tensor(F32, [5120, 2048]))), "IQ3_S weights are claimed"


def test_iq3s_not_claimed_without_a_dequantiser():
    # a ggml with no IQ3_S to_float: no codebook, and IQ3_S is not claimed
    code = ("import sys; sys.path.insert(0, %r); "
            "from harness import *; import ctypes; "
            "fake = ctypes.CDLL(str(FAKE), mode=ctypes.RTLD_GLOBAL); "
            "plugin = ctypes.CDLL(str(PLUGIN)); plugin.ggml_zest_iq3s_codebook.argtypes = [ctypes.c_void_p]; "
            "print('CODEBOOK', plugin.ggml_zest_iq3s_codebook(None))"
            % os.path.join(os.path.dirname(__file__), "ggml_harness"))
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=120)
    assert "CODEBOOK 0" in out.stdout, out.stdout + out.stderr


def test_min_batch_env():
    code = ("import sys; sys.path.insert(0, %r); from harness import *; h = Harness(); "
            "w = h.tensor(Q4_K, [2048, 2048], buffer=h.buffer(USAGE_WEIGHTS)); "
            "x = h.tensor(F32, [2048, 512]); print('CLAIMED' if h.policy(h.mul_mat(w, x)) else 'NOT')"
            % os.path.join(os.path.dirname(__file__), "ggml_harness"))
    env = dict(os.environ, GGML_XDNA_MIN_BATCH="512")
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env, timeout=120)
    assert "CLAIMED" in out.stdout, out.stderr
    env = dict(os.environ, GGML_XDNA_MIN_BATCH="")  # empty means unset: the default 1024
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env, timeout=120)
    assert "NOT" in out.stdout, out.stderr


def test_matmul_groups(h):
    # MUL_MATs on one input run as one grouped call at the first one's turn,
    # when no node in between touches a later one's output bytes
    k, t = 1024, 1024
    C, W = h.buffer(USAGE_COMPUTE), h.buffer(USAGE_WEIGHTS)
    base = 0x7f0000000000
    addr = iter(range(base, base + (64 << 30), 1 << 30))  # 1 GiB apart: no overlaps unless asked

    def piece(alias=False, host_out=False, n_extra=0):
        x = h.tensor(F32, [k, t], "x", C, next(addr))
        q = h.mul_mat(h.tensor(Q4_K, [k, 2048], "wq", W, next(addr)), x, "q", C, next(addr))
        qn = h.rms_norm(q, name="q_norm", buffer=C, data=next(addr))
        qs = h.scale(qn, 0.5, name="q_scaled", buffer=C, data=next(addr))
        k_data = qn.data if alias else next(addr)  # the allocator lent q_norm's bytes to k's output
        kk = h.mul_mat(h.tensor(Q4_K, [k, 512], "wk", W, next(addr)), x, "k", h.buffer(USAGE_COMPUTE, host=True)
                       if host_out else C, k_data)
        v = h.mul_mat(h.tensor(Q4_K, [k, 512], "wv", W, next(addr)), x, "v", C, next(addr))
        extra = [h.mul_mat(h.tensor(Q4_K, [k, 256], "we", W, next(addr)), x, "e", C, next(addr))
                 for _ in range(n_extra)]
        other = h.mul_mat(h.tensor(Q4_K, [k, 256], "wo", W, next(addr)), qs, "o", C, next(addr))
        return h.piece_groups([q, qn, qs, kk, v, *extra, other])

    assert piece() == [3], "q, k and v on the same input"
    assert piece(alias=True) == [2], "k's bytes are q_norm's, live between q and k: k runs at its own turn"
    assert piece(host_out=True) == [2], "an output in host memory with the input on the device"
    assert piece(n_extra=2) == [4], "at most 4 to a group"


def test_a_bias_row_is_not_folded_as_a_residual(h):
    # the GEMM epilogue adds a [T][N] residual; a bias row ([N], broadcast
    # over the tokens, Qwen2's q/k/v bias) stays an ADD of its own
    k, n, t = 2048, 2048, 2048
    C, W = h.buffer(USAGE_COMPUTE), h.buffer(USAGE_WEIGHTS)
    base = 0x7f0000000000
    addr = iter(range(base, base + (64 << 30), 1 << 30))

    def T(type_, ne, name, buf=C):
        return h.tensor(type_, ne, name, buf, next(addr))

    def plan(second):
        x = T(F32, [k, t], "x")
        d = h.mul_mat(T(Q4_K, [k, n], "blk.0.attn_q.weight", W), x, "q", C, next(addr))
        out = h.add(d, second, name="q_out", buffer=C, data=next(addr))
        for nd in (d, out):
            h.supports_op(nd)
        return h.piece_plan([d, out])

    assert plan(T(F32, [n], "blk.0.attn_q.bias", W))["add"] == 0
    assert plan(T(F32, [n, t], "resid"))["add"] == 1, "the same piece with a residual folds"


def test_a_sum_half_over_its_residual_is_not_folded(h):
    # the folded epilogue reads each residual element and writes the same one:
    # the sum in place (x += o) folds, a sum placed part-way over the residual
    # does not
    k, n, t = 2048, 2048, 2048
    C, W = h.buffer(USAGE_COMPUTE), h.buffer(USAGE_WEIGHTS)
    base = 0x7b0000000000
    addr = iter(range(base, base + (64 << 30), 1 << 30))

    def plan(out_offset):
        x = h.tensor(F32, [k, t], "x", C, next(addr))
        d = h.mul_mat(h.tensor(Q4_K, [k, n], "blk.0.attn_output.weight", W, next(addr)), x, "o", C, next(addr))
        r_ptr = next(addr)
        r = h.tensor(F32, [n, t], "resid", C, r_ptr)
        out = h.add(d, r, name="o_out", buffer=C, data=r_ptr + out_offset)
        for nd in (d, out):
            h.supports_op(nd)
        return h.piece_plan([d, out])["add"]

    assert plan(0) == 1, "in place"
    assert plan(n * 4 * 16) == 0, "16 rows over"


def test_a_matmul_result_read_elsewhere_is_not_folded_into_its_add(h):
    # the folded epilogue writes only the sum: a second reader of the
    # matmul's own result keeps the ADD separate
    k, n, t = 2048, 2048, 2048
    C, W = h.buffer(USAGE_COMPUTE), h.buffer(USAGE_WEIGHTS)
    base = 0x7c0000000000
    addr = iter(range(base, base + (64 << 30), 1 << 30))

    def T(type_, ne, name, buf=C):
        return h.tensor(type_, ne, name, buf, next(addr))

    x = T(F32, [k, t], "x")
    d = h.mul_mat(T(Q4_K, [k, n], "blk.0.attn_output.weight", W), x, "o", C, next(addr))
    out = h.add(d, T(F32, [n, t], "resid"), name="o_out", buffer=C, data=next(addr))
    other = h.scale(d, 2.0, name="other", buffer=C, data=next(addr))
    for nd in (d, out, other):
        h.supports_op(nd)
    assert h.piece_plan([d, out, other])["add"] == 0


def test_a_swiglu_read_elsewhere_keeps_its_result(h):
    # the hand-off writes down's packed input instead of the f32 SwiGLU
    # result: with another reader of that result there is no hand-off (the
    # gate/up GEMM still applies SwiGLU in its epilogue)
    k, f, t = 2048, 5632, 2048
    C, W = h.buffer(USAGE_COMPUTE), h.buffer(USAGE_WEIGHTS)
    base = 0x7d0000000000
    addr = iter(range(base, base + (64 << 30), 1 << 30))

    def T(type_, ne, name, buf=C):
        return h.tensor(type_, ne, name, buf, next(addr))

    def plan(other_reader):
        x = T(F32, [k, t], "x")
        g = h.mul_mat(T(Q4_K, [k, f], "blk.0.ffn_gate.weight", W), x, "gate", C, next(addr))
        u = h.mul_mat(T(Q4_K, [k, f], "blk.0.ffn_up.weight", W), x, "up", C, next(addr))
        sw = h.glu(g, u, kind=2, name="swiglu", buffer=C, data=next(addr))
        d = h.mul_mat(T(Q4_K, [f, k], "blk.0.ffn_down.weight", W), sw, "down", C, next(addr))
        nodes = [g, u, sw, d]
        if other_reader:
            nodes.append(h.scale(sw, 0.5, name="other", buffer=C, data=next(addr)))
        for nd in nodes:
            h.supports_op(nd)
        return h.piece_plan(nodes)

    p = plan(False)
    assert (p["swiglu"], p["handoff"]) == (1, 1), p
    p = plan(True)
    assert (p["swiglu"], p["handoff"]) == (1, 0), p


def test_piece_plan_folds_the_block_ops(h):
    # what graph_compute folds into its matmul calls: the RMS_NORM (and MUL)
    # before a matmul into the pack, the residual ADD after o/down into the
    # GEMM epilogue, a SwiGLU whose only reader is down into down's packed
    # input, and RMS_NORM -> MUL -> ROPE into one kernel
    k, f, t, hd, heads = 2048, 5632, 2048, 128, 16
    C, W = h.buffer(USAGE_COMPUTE), h.buffer(USAGE_WEIGHTS)
    base = 0x7e0000000000
    addr = iter(range(base, base + (256 << 30), 1 << 30))

    def T(type_, ne, name, buf=C, **kw):
        return h.tensor(type_, ne, name, buf, next(addr), **kw)

    def ffn(extra_norm_reader=False):
        x = T(F32, [k, t], "x")
        nrm = h.rms_norm(x, name="ffn_norm", buffer=C, data=next(addr))
        m = h.mul(nrm, T(F32, [k], "ffn_norm.weight", W), name="ffn_inp", buffer=C, data=next(addr))
        g = h.mul_mat(T(Q4_K, [k, f], "ffn_gate.weight", W), m, "gate", C, next(addr))
        u = h.mul_mat(T(Q4_K, [k, f], "ffn_up.weight", W), m, "up", C, next(addr))
        s = h.glu(g, u, kind=2, name="swiglu", buffer=C, data=next(addr))
        d = h.mul_mat(T(Q4_K, [f, k], "ffn_down.weight", W), s, "down", C, next(addr))
        out = h.add(d, x, name="ffn_out", buffer=C, data=next(addr))
        nodes = [nrm, m, g, u, s, d, out]
        if extra_norm_reader:
            nodes.append(h.scale(nrm, 2.0, name="other", buffer=C, data=next(addr)))
        for nd in nodes:
            h.supports_op(nd)
        return h.piece_plan(nodes)

    p = ffn()
    assert (p["swiglu"], p["norm"], p["add"], p["handoff"]) == (1, 1, 1, 1), p
    assert p["jobs"] == 2  # gate/up and down: two service calls for the whole block
    p = ffn(extra_norm_reader=True)
    assert p["norm"] == 0 and p["swiglu"] == 1, "a norm read by another op is computed on its own"

    x = T(F32, [k, t], "x")
    nrm = h.rms_norm(x, name="attn_norm", buffer=C, data=next(addr))
    m = h.mul(nrm, T(F32, [k], "attn_norm.weight", W), name="attn_inp", buffer=C, data=next(addr))
    q = h.mul_mat(T(Q4_K, [k, heads * hd], "attn_q.weight", W), m, "q", C, next(addr))
    kk = h.mul_mat(T(Q4_K, [k, 4 * hd], "attn_k.weight", W), m, "k", C, next(addr))
    v = h.mul_mat(T(Q4_K, [k, 4 * hd], "attn_v.weight", W), m, "v", C, next(addr))
    q3 = h.tensor(F32, [hd, heads, t], "q3", C, q.data, op="RESHAPE", src=(q,), view_src=q)
    qn = h.rms_norm(q3, name="q_norm", buffer=C, data=next(addr))
    qm = h.mul(qn, T(F32, [hd], "attn_q_norm.weight", W), name="q_normed", buffer=C, data=next(addr))
    pos = h.tensor(26, [t], "pos", h.buffer(USAGE_COMPUTE), next(addr))
    qr = h.rope(qm, pos, hd, 2, name="q_rope", buffer=C, data=next(addr))
    nodes = [nrm, m, q, kk, v, q3, qn, qm, qr]
    for nd in nodes:
        h.supports_op(nd)
    p = h.piece_plan(nodes)
    assert (p["groups"], p["norm"], p["rope"]) == (1, 1, 1), p
    assert p["jobs"] == 1


def test_piece_plan_leaves_unsafe_folds_alone(h):
    # what the plan must NOT fold: a residual ADD that is not the matmul's
    # next node, or whose other operand is a bias row, or is computed after
    # the matmul; a norm feeding a matmul in host memory; a SwiGLU whose
    # result another op reads too
    k, n, t = 2048, 2048, 2048
    C, W, Hm = h.buffer(USAGE_COMPUTE), h.buffer(USAGE_WEIGHTS), h.buffer(USAGE_COMPUTE, host=True)
    base = 0x7d0000000000
    addr = iter(range(base, base + (256 << 30), 1 << 30))

    def T(type_, ne, name, buf=C, **kw):
        return h.tensor(type_, ne, name, buf, next(addr), **kw)

    def plan(nodes):
        for nd in nodes:
            h.supports_op(nd)
        return h.piece_plan(nodes)

    x = T(F32, [k, t], "x")
    r = T(F32, [n, t], "resid")
    mm = h.mul_mat(T(Q4_K, [k, n], "w", W), x, "mm", C, next(addr))
    other = h.scale(x, 2.0, name="between", buffer=C, data=next(addr))
    add = h.add(mm, r, name="out", buffer=C, data=next(addr))
    assert plan([mm, other, add])["add"] == 0, "a node between the matmul and its ADD"
    assert plan([mm, add])["add"] == 1

    mm2 = h.mul_mat(T(Q4_K, [k, n], "w2", W), x, "mm2", C, next(addr))
    bias = h.add(mm2, T(F32, [n], "bias", W), name="biased", buffer=C, data=next(addr))
    assert plan([mm2, bias])["add"] == 0, "a bias row is a small op of its own"

    mm3 = h.mul_mat(T(Q4_K, [k, n], "w3", W), x, "mm3", C, next(addr))
    late = h.scale(T(F32, [n, t], "y"), 1.0, name="late", buffer=C, data=next(addr))
    add3 = h.add(mm3, late, name="out3", buffer=C, data=next(addr))
    assert plan([mm3, late, add3])["add"] == 0, "a residual computed after the matmul"

    xh = T(F32, [k, t], "x_host", Hm)
    nrm = h.rms_norm(xh, name="norm_h", buffer=Hm, data=next(addr))
    mmh = h.mul_mat(T(Q4_K, [k, n], "w4", W), nrm, "mm_h", C, next(addr))
    assert plan([nrm, mmh])["norm"] == 0, "operands in host memory take the staged route"

    f = 5632
    g = h.mul_mat(T(Q4_K, [k, f], "gate", W), x, "g", C, next(addr))
    u = h.mul_mat(T(Q4_K, [k, f], "up", W), x, "u", C, next(addr))
    s = h.glu(g, u, kind=2, name="s", buffer=C, data=next(addr))
    d = h.mul_mat(T(Q4_K, [f, k], "down", W), s, "d", C, next(addr))
    extra = h.scale(s, 0.5, name="s_read_too", buffer=C, data=next(addr))
    p = plan([g, u, s, d, extra])
    assert p["swiglu"] == 1 and p["handoff"] == 0, "the SwiGLU is read by another op: written in f32"


def test_budget_cuts_whole_layers(h):
    # the reference's tests/test-memory-budget.cpp: weight copies fill the
    # budget in the order they are asked for; the first weight that does not
    # fit sends its whole layer back, and every later weight stays on the GPU
    # backend. Each 2048 x 2048 copy takes 2048 * 2048 * (9/8 + 2) bytes = 13.1 MB.
    W = h.buffer(USAGE_WEIGHTS)
    base = 0x7c0000000000
    ws = [h.tensor(Q4_K, [2048, 2048], f"blk.{i // 3}.ffn_{('gate', 'up', 'down')[i % 3]}.weight", W,
                   base + (i << 30)) for i in range(12)]
    # 7 copies fit in 0.1 GB: layer 2 is cut at its second weight, and its first goes back
    assert h.budget_plan(0.1, ws) == [1] * 6 + [0] * 6
    assert h.budget_plan(1.0, ws) == [1] * 12
    assert h.budget_plan(0.0, ws) == [0] * 12
    # a weight without a layer in its name (the output head) is cut alone
    head = h.tensor(Q4_K, [2048, 2048], "output.weight", W, base + (40 << 30))
    assert h.budget_plan(0.03, [ws[0], ws[1], head]) == [1, 1, 0]
