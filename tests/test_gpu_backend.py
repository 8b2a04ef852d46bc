"""The ggml plugin end to end on the GPU: registration with the start-up
self-test, supports_op, graph_optimize building weight copies at load, and
graph_compute running claimed MUL_MATs in place on device tensors (and on a
host-memory graph input), checked against the oracle; then the failure path
(a failing piece returns GGML_STATUS_FAILED and the backend claims nothing
more), with the failure injected on the host."""
import os
import subprocess
import sys
import textwrap

import numpy as np
import pytest
import torch

sys.path.insert(0, os.path.join(os.path.dirname(__file__), "ggml_harness"))
from harness import F32, Harness, Q4_0, Q4_K, Q8_0, STATUS_FAILED, STATUS_SUCCESS, USAGE_COMPUTE, USAGE_WEIGHTS  # noqa: E402

from oracle import oracle as O  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def h():
    return Harness()


def dequant_q4_0(raw: np.ndarray, n: int, k: int) -> np.ndarray:
    b = raw.reshape(n, k // 32, 18)
    d = b[..., :2].copy().view(np.float16).astype(np.float32)
    q = b[..., 2:]
    lo = (q & 0xF).astype(np.float32) - 8
    hi = (q >> 4).astype(np.float32) - 8
    return (np.concatenate([lo, hi], axis=-1) * d).reshape(n, k).astype(np.float32)


def quant_q4_0(w: np.ndarray) -> np.ndarray:
    n, k = w.shape
    b = w.reshape(n, k // 32, 32)
    amax_i = np.argmax(np.abs(b), axis=-1)
    mx = np.take_along_axis(b, amax_i[..., None], axis=-1)[..., 0]
    d = (mx / -8).astype(np.float16)
    inv = np.where(d != 0, 1.0 / d.astype(np.float32), 0)
    q = np.clip(np.round(b * inv[..., None] + 8), 0, 15).astype(np.uint8)
    out = np.empty((n, k // 32, 18), np.uint8)
    out[..., :2] = d[..., None].view(np.uint8).reshape(n, k // 32, 2)
    out[..., 2:] = q[..., :16] | (q[..., 16:] << 4)
    return out.reshape(-1)


def want(values: np.ndarray, x: np.ndarray) -> np.ndarray:
    n, k = values.shape
    wd = O.decode_blocks(O.encode_blocks(values)).reshape(n, k)
    xd = O.decode_blocks(O.encode_blocks(x)).reshape(x.shape)
    return O.mul_mat(wd, xd)


def test_device_offered(h):
    assert h.device_count() == 1


@pytest.mark.parametrize("qt", [Q4_K, Q8_0, Q4_0])
def test_graph_compute_in_place(h, qt):
    K, N, T = 2560, 1024, 1100
    vals = O.weights_f32(N, K, qt)
    raw = quant_q4_0(vals) if qt == Q4_0 else O.quantize(qt, vals)
    deq = dequant_q4_0(raw, N, K) if qt == Q4_0 else O.dequant(qt, raw, N, K)
    x = O.activations(T, K, 5)
    wd = torch.from_numpy(raw).cuda()
    xd = torch.from_numpy(x).cuda()
    yd = torch.zeros((T, N), dtype=torch.float32, device="cuda")
    w = h.tensor(qt, [K, N], name="blk.0.ffn_down.weight", buffer=h.buffer(USAGE_WEIGHTS), data=wd.data_ptr())
    xt = h.tensor(F32, [K, T], buffer=h.buffer(USAGE_COMPUTE), data=xd.data_ptr())
    node = h.mul_mat(w, xt, buffer=h.buffer(USAGE_COMPUTE), data=yd.data_ptr())
    assert h.supports_op(node)
    b, _ = h.init_backend()
    assert b
    torch.cuda.synchronize()
    h.graph_optimize(b, [node])  # builds the weight copy at load
    assert h.graph_compute(b, [w, xt, node]) == STATUS_SUCCESS
    torch.cuda.synchronize()
    y = yd.cpu().numpy()
    assert np.array_equal(y, O.round_bf16(y)), "GGML_XDNA_OUT16 default: bf16 results"
    assert O.nmax_err(y, want(deq, x)) <= 4e-3
    h.backend_free(b)


def test_host_input(h):
    K, N, T = 2048, 2048, 1024
    raw = O.quantize(Q8_0, O.weights_f32(N, K, 2))
    x = O.activations(T, K, 3)
    wd = torch.from_numpy(raw).cuda()
    yd = torch.zeros((T, N), dtype=torch.float32, device="cuda")
    w = h.tensor(Q8_0, [K, N], buffer=h.buffer(USAGE_WEIGHTS), data=wd.data_ptr())
    xt = h.tensor(F32, [K, T], buffer=h.buffer(USAGE_COMPUTE, host=True), data=x.ctypes.data)
    node = h.mul_mat(w, xt, buffer=h.buffer(USAGE_COMPUTE), data=yd.data_ptr())
    b, _ = h.init_backend()
    torch.cuda.synchronize()
    assert h.graph_compute(b, [node]) == STATUS_SUCCESS
    torch.cuda.synchronize()
    assert O.nmax_err(yd.cpu().numpy(), want(O.dequant(Q8_0, raw, N, K), x)) <= 4e-3
    h.backend_free(b)


def test_failure_is_sticky():
    """A failing matmul (injected on the host, GGML_XDNA_FAIL_AFTER=0) makes
    graph_compute return GGML_STATUS_FAILED and the backend claim nothing
    from then on, so the scheduler hands every later op to the CUDA backend
    (the reference's sticky decline, src/ggml-zest.cpp:120-130,896-899)."""
    here = os.path.dirname(__file__)
    code = textwrap.dedent(f"""
        import sys
        sys.path[:0] = [{os.path.join(here, 'ggml_harness')!r}, {os.path.dirname(here)!r}]
        import numpy as np, torch
        from harness import *
        from oracle import oracle as O
        h = Harness()
        K, N, T = 2048, 2048, 1024
        raw = O.quantize(Q8_0, O.weights_f32(N, K, 2))
        wd = torch.from_numpy(raw).cuda(); xd = torch.randn(T, K, device="cuda")
        yd = torch.zeros((T, N), device="cuda")
        w = h.tensor(Q8_0, [K, N], buffer=h.buffer(USAGE_WEIGHTS), data=wd.data_ptr())
        xt = h.tensor(F32, [K, T], buffer=h.buffer(USAGE_COMPUTE), data=xd.data_ptr())
        node = h.mul_mat(w, xt, buffer=h.buffer(USAGE_COMPUTE), data=yd.data_ptr())
        b, _ = h.init_backend(); torch.cuda.synchronize()
        print("before", h.supports_op(node))
        print("status", h.graph_compute(b, [node]))
        print("after", h.supports_op(node))
    """)
    env = dict(os.environ, GGML_XDNA_FAIL_AFTER="0")
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    assert "before True" in r.stdout
    assert f"status {STATUS_FAILED}" in r.stdout
    assert "after False" in r.stdout, "after a failure the backend claims nothing"
    assert "claiming nothing from now on" in r.stderr


def test_no_device_when_the_gpu_cannot_run():
    """tests/test-safe-start.cpp:20-38: when the device cannot run the path,
    the plugin still registers but offers no device, so it claims nothing.
    The reference simulates it with a kernel path that names nothing; here
    the CUDA device index names no device, which fails the same start-up
    check a missing GPU or a non-B200 one does."""
    here = os.path.dirname(__file__)
    code = textwrap.dedent(f"""
        import sys
        sys.path[:0] = [{os.path.join(here, 'ggml_harness')!r}, {os.path.dirname(here)!r}]
        from harness import *
        h = Harness()
        print("reg", h.reg_name())
        print("devices", h.device_count())
        x = h.tensor(F32, [2048, 2048], buffer=h.buffer(USAGE_COMPUTE))
        w = h.tensor(Q4_K, [2048, 2048], buffer=h.buffer(USAGE_WEIGHTS))
        print("policy", h.policy(h.mul_mat(w, x)))
    """)
    env = dict(os.environ, GGML_ZEST_CUDA_DEVICE="64")
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    assert "reg XDNA" in r.stdout, "the plugin loads"
    assert "devices 0" in r.stdout, "no device offered"
    assert "policy True" in r.stdout, "the host-side policy alone would take the matmul"
    assert "not offering" in r.stderr and "no such CUDA device" in r.stderr
