"""The block executor's small ops on the GPU, through the C ABI, against the
oracle's restatement of the reference's run_rows: the 21 cases of the
reference's tests/test-host-ops.cpp:91-153 (D=256, T=8, head dim 64 x 4 heads,
inputs N(0, 1.5), positions 5000 + 300 i, frequency factors U(1, 4)) and a
prompt-sized case. The reference's bar is nrmse <= 1e-5 (3e-3 for the
tanh/quick GELUs against ggml-cpu's 16-bit table); both sides here compute
every activation in float, so all cases are held to 1e-5."""
import ctypes

import numpy as np
import pytest
import torch

import zest_b200 as Z
from oracle import oracle as O

pytestmark = pytest.mark.gpu
EXACT = 1e-5
D, T, HD, H = 256, 8, 64, 4


def rng(seed=42):
    return np.random.default_rng(seed)


def normal(shape, seed):
    return (rng(seed).standard_normal(shape) * 1.5).astype(np.float32)


_alive = []  # device copies must outlive the kernels that read them


def dev(a):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    _alive.append(t)
    return t


def call(name, *args):
    L = Z.lib()
    rc = getattr(L, name)(*args, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, L.zest_last_error().decode()
    torch.cuda.synchronize()
    _alive.clear()


def p(t):
    return ctypes.c_void_p(t.data_ptr())


@pytest.mark.parametrize("rows", [T, 2048])
def test_rms_norm(rows):
    x = normal((rows, D), 1)
    y = torch.empty_like(dev(x))
    call("zest_rms_norm", p(dev(x)), rows, D, ctypes.c_float(1e-6), p(y))
    assert O.nrmse(y.cpu().numpy(), O.rms_norm(x, D, 1e-6)) <= EXACT


def test_rms_norm_per_head():
    # Qwen3's q/k norm: every head's 128 values normalised on their own
    x = normal((T * 32, 128), 2)
    xd = dev(x)
    y = torch.empty_like(xd)
    call("zest_rms_norm", p(xd), T * 32, 128, ctypes.c_float(1e-6), p(y))
    assert O.nrmse(y.cpu().numpy(), O.rms_norm(x, 128, 1e-6)) <= EXACT


def test_mul_by_scale_row():
    x, w = normal((T, D), 3), normal((D,), 4)
    y = torch.empty((T, D), device="cuda")
    call("zest_mul_row", p(dev(x)), p(dev(w)), T, D, p(y))
    assert O.nrmse(y.cpu().numpy(), O.mul_row(x, w)) <= EXACT


@pytest.mark.parametrize("bias", [False, True])
def test_add(bias):
    x = normal((T, D), 5)
    b = normal((D,) if bias else (T, D), 6)
    y = torch.empty((T, D), device="cuda")
    call("zest_add", p(dev(x)), p(dev(b)), int(bias), T, D, p(y))
    assert O.nrmse(y.cpu().numpy(), O.add(x, b)) <= EXACT


def test_scale_and_bias():
    x = normal((T, D), 7)
    y = torch.empty((T, D), device="cuda")
    call("zest_scale", p(dev(x)), T * D, ctypes.c_float(0.37), ctypes.c_float(0.25), p(y))
    assert O.nrmse(y.cpu().numpy(), O.scale(x, 0.37, 0.25)) <= EXACT


GLUS = [("swiglu", 2), ("geglu", 1), ("geglu_erf", 4), ("geglu_quick", 5), ("reglu", 0)]


@pytest.mark.parametrize("name,kind", GLUS)
def test_glu_split(name, kind):
    g, u = normal((T, D), 8), normal((T, D), 9)
    y = torch.empty((T, D), device="cuda")
    call("zest_glu", kind, p(dev(g)), D, p(dev(u)), D, T, D, p(y))
    assert O.nrmse(y.cpu().numpy(), O.glu(kind, g, u)) <= EXACT, name


@pytest.mark.parametrize("name,kind,swapped", [("swiglu", 2, False), ("swiglu", 2, True), ("geglu", 1, False),
                                               ("geglu_erf", 4, False)])
def test_glu_one_tensor(name, kind, swapped):
    x = normal((T, 2 * D), 10)
    xd = dev(x)
    y = torch.empty((T, D), device="cuda")
    base = xd.data_ptr()
    g = ctypes.c_void_p(base + (D * 4 if swapped else 0))
    u = ctypes.c_void_p(base + (0 if swapped else D * 4))
    call("zest_glu", kind, g, 2 * D, u, 2 * D, T, D, p(y))
    assert O.nrmse(y.cpu().numpy(), O.glu(kind, x, swapped=swapped)) <= EXACT, name


ROPES = [  # (n_dims, mode, n_ctx_orig, freq_scale, ext_factor, factors), test-host-ops.cpp:143-149
    (HD, 0, 0, 1.0, 0.0, False), (HD, 2, 0, 1.0, 0.0, False), (HD // 2, 0, 0, 1.0, 0.0, False),
    (HD * 3 // 4, 2, 0, 1.0, 0.0, False), (HD, 2, 4096, 0.25, 1.0, False), (HD, 2, 4096, 1.0, 0.0, True),
    (HD, 0, 4096, 0.25, 1.0, True)]


@pytest.mark.parametrize("n_dims,mode,n_ctx_orig,freq_scale,ext_factor,factors", ROPES)
def test_rope(n_dims, mode, n_ctx_orig, freq_scale, ext_factor, factors):
    x = normal((T, H, HD), 11)
    pos = (5000 + 300 * np.arange(T)).astype(np.int32)
    ff = rng(12).uniform(1.0, 4.0, n_dims // 2).astype(np.float32) if factors else None
    par = np.array([10000.0, freq_scale, ext_factor, 1.0, 32.0, 1.0], np.float32)
    table = torch.empty((T, n_dims), device="cuda")
    ffd = dev(ff) if factors else None
    L = Z.lib()
    rc = L.zest_rope_table(p(dev(pos)), T, n_dims, n_ctx_orig, par.ctypes.data_as(ctypes.POINTER(ctypes.c_float)),
                           p(ffd) if factors else None, p(table), None)
    assert rc == 0, L.zest_last_error().decode()
    y = torch.empty((T, H, HD), device="cuda")
    call("zest_rope", p(dev(x)), T, H, HD, n_dims, mode, p(table), p(y))
    want_t = O.rope_table(pos, n_dims, n_ctx_orig, par, ff)
    assert O.nrmse(table.cpu().numpy(), want_t) <= EXACT
    assert O.nrmse(y.cpu().numpy(), O.rope(x, n_dims, mode, want_t)) <= EXACT


def test_rope_prompt_sized():
    # Qwen3-4B's q: 32 heads x 128, NeoX, a 2048-token chunk
    Tn, Hn, d = 2048, 32, 128
    x = normal((Tn, Hn, d), 13)
    pos = np.arange(Tn, dtype=np.int32) + 4096
    par = np.array([1000000.0, 1.0, 0.0, 1.0, 32.0, 1.0], np.float32)
    table = torch.empty((Tn, d), device="cuda")
    L = Z.lib()
    assert L.zest_rope_table(p(dev(pos)), Tn, d, 0, par.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), None,
                             p(table), None) == 0
    y = torch.empty((Tn, Hn, d), device="cuda")
    call("zest_rope", p(dev(x)), Tn, Hn, d, d, 2, p(table), p(y))
    want = O.rope(x, d, 2, O.rope_table(pos, d, 0, par))
    assert O.nrmse(y.cpu().numpy(), want) <= EXACT
