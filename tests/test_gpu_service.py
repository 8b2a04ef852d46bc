"""The matmul service zest_npu (xdna_npu's counterpart) through the C ABI:
self-test, weight cache, y = x * W^T on host and device buffers, output
modes, and the failure paths the reference tests with its injection
variables (GGML_XDNA_FAIL_AFTER / GGML_XDNA_NAN_AFTER), on the host side."""
import os
import subprocess
import sys
import textwrap

import numpy as np
import pytest
import torch

import zest_b200 as Z
from oracle import oracle as O
from gpu_util import bf16_to_f32, dev, host, same_up_to_sum_order

pytestmark = pytest.mark.gpu
ROOT = Z.PKG_DIR.parent


def test_usable():
    ok, why = Z.usable(0)
    assert ok, why


@pytest.mark.parametrize("qt", [O.Q8_0, O.Q4_K, O.Q6_K, O.IQ3_S])
def test_mul_mat_host_buffers(qt):
    Z.load_iq3s_grid()
    npu = Z.Npu(0)
    npu.set_out16(False)
    N, K, T = 1024, 512, 300
    raw = O.quantize(qt, O.weights_f32(N, K, qt))
    x = O.activations(T, K, 1)
    key = Z.Npu.key(raw.ctypes.data, qt, K, N)
    npu.add_weight(key, raw.ctypes.data, on_device=False)
    assert npu.has_weight(key) and npu.out_width(key) == N
    y = np.empty((T, N), np.float32)
    npu.mul_mat(key, x.ctypes.data, T, y.ctypes.data, on_device=False)
    a_dec = O.decode_blocks(O.encode_blocks(x)).reshape(T, K)
    w_dec = O.decode_blocks(O.encode_blocks(O.dequant(qt, raw, N, K))).reshape(N, K)
    assert O.nmax_err(y, O.mul_mat(w_dec, a_dec)) <= 1e-3
    t = npu.take_times()
    assert t.calls == 1 and t.gemm_ms > 0
    npu.close()


def test_mul_mat_out16_and_device_buffers():
    npu = Z.Npu(0)  # GGML_XDNA_OUT16 unset: bf16 output, as the reference's default
    N, K, T = 512, 256, 1024
    raw = O.quantize(O.Q8_0, O.weights_f32(N, K, 4))
    key = Z.Npu.key(raw.ctypes.data, O.Q8_0, K, N)
    npu.add_weight(key, raw.ctypes.data, on_device=False)
    xd = dev(O.activations(T, K, 2))
    yd = torch.empty((T, N), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    npu.mul_mat(key, xd.data_ptr(), T, yd.data_ptr(), on_device=True)
    y = host(yd)
    assert np.array_equal(y, O.round_bf16(y))  # every value a bf16
    a_dec = O.decode_blocks(O.encode_blocks(host(xd))).reshape(T, K)
    w_dec = O.decode_blocks(O.encode_blocks(O.dequant(O.Q8_0, raw, N, K))).reshape(N, K)
    assert O.nmax_err(y, O.mul_mat(w_dec, a_dec)) <= 4e-3  # bf16 output rounding (2^-9) included
    npu.close()


def test_fused_gate_up():
    npu = Z.Npu(0)
    F, K, T = 1000, 512, 200
    g = O.quantize(O.Q4_K, O.weights_f32(F, K, 1))
    u = O.quantize(O.Q4_K, O.weights_f32(F, K, 2))
    key = Z.Npu.key(g.ctypes.data, O.Q4_K, K, F)
    npu.add_fused(key, g.ctypes.data, u.ctypes.data, on_device=False)
    assert npu.out_width(key, fused=True) == F
    x = O.activations(T, K, 3)
    y = np.empty((T, F), np.float32)
    npu.mul_mat(key, x.ctypes.data, T, y.ctypes.data, on_device=False, fused=True)
    a_dec = O.decode_blocks(O.encode_blocks(x)).reshape(T, K)
    gd = O.decode_blocks(O.encode_blocks(O.dequant(O.Q4_K, g, F, K))).reshape(F, K)
    ud = O.decode_blocks(O.encode_blocks(O.dequant(O.Q4_K, u, F, K))).reshape(F, K)
    want = O.swiglu_bf16(O.mul_mat(gd, a_dec), O.mul_mat(ud, a_dec))
    assert O.nmax_err(y, want) <= 4e-3
    npu.close()


def _child(env_extra: dict, body: str) -> subprocess.CompletedProcess:
    env = dict(os.environ, **env_extra)
    code = textwrap.dedent(f"""
        import sys
        sys.path[:0] = [{str(ROOT)!r}, {str(ROOT / 'ggml-xdna_b200')!r}]
        import numpy as np, zest_b200 as Z
        from oracle import oracle as O
        npu = Z.Npu(0)
        N, K, T = 512, 256, 128
        raw = O.quantize(O.Q8_0, O.weights_f32(N, K, 1))
        key = Z.Npu.key(raw.ctypes.data, O.Q8_0, K, N)
        npu.add_weight(key, raw.ctypes.data, on_device=False)
        x = O.activations(T, K, 2)
        y = np.empty((T, N), np.float32)
    """) + textwrap.dedent(body)
    return subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env, timeout=300)


def test_injected_failure():
    r = _child({"GGML_XDNA_FAIL_AFTER": "1"}, """
        npu.mul_mat(key, x.ctypes.data, T, y.ctypes.data, on_device=False)
        try:
            npu.mul_mat(key, x.ctypes.data, T, y.ctypes.data, on_device=False)
        except Z.ZestError as e:
            print("FAILED:", e)
    """)
    assert r.returncode == 0, r.stderr
    assert "FAILED:" in r.stdout and "GGML_XDNA_FAIL_AFTER" in r.stdout


def test_injected_nan_is_caught():
    r = _child({"GGML_XDNA_NAN_AFTER": "0"}, """
        try:
            npu.mul_mat(key, x.ctypes.data, T, y.ctypes.data, on_device=False)
        except Z.ZestError as e:
            print("FAILED:", e)
    """)
    assert r.returncode == 0, r.stderr
    assert "NaN or infinity" in r.stdout


@pytest.mark.parametrize("on_device", [False, True])
def test_mul_mat_group_equals_separate_calls(on_device):
    # q, k, v and a fused gate/up sharing one input: one pack, one launch,
    # the results of a call per weight (up to the sum order)
    npu = Z.Npu(0)
    npu.set_out16(False)
    K, T = 512, 700
    raws = [O.quantize(O.Q4_K, O.weights_f32(N, K, 50 + i)) for i, N in enumerate((1024, 256, 256))]
    keys = [Z.Npu.key(r.ctypes.data, O.Q4_K, K, N) for r, N in zip(raws, (1024, 256, 256))]
    for k, r in zip(keys, raws):
        npu.add_weight(k, r.ctypes.data, on_device=False)
    F = 600
    g = O.quantize(O.Q6_K, O.weights_f32(F, K, 60))
    u = O.quantize(O.Q6_K, O.weights_f32(F, K, 61))
    gkey = Z.Npu.key(g.ctypes.data, O.Q6_K, K, F)
    npu.add_fused(gkey, g.ctypes.data, u.ctypes.data, on_device=False)
    keys.append(gkey)
    fused = [False, False, False, True]
    widths = [1024, 256, 256, F]
    x = O.activations(T, K, 62)
    if on_device:
        xd = dev(x)
        ys = [torch.empty((T, w), dtype=torch.float32, device="cuda") for w in widths]
        solo = [torch.empty((T, w), dtype=torch.float32, device="cuda") for w in widths]
        torch.cuda.synchronize()
        npu.mul_mat_group(keys, xd.data_ptr(), T, [y.data_ptr() for y in ys], True, fused)
        for k, f, y in zip(keys, fused, solo):
            npu.mul_mat(k, xd.data_ptr(), T, y.data_ptr(), True, fused=f)
        got, want = [host(y) for y in ys], [host(y) for y in solo]
    else:
        got = [np.empty((T, w), np.float32) for w in widths]
        want = [np.empty((T, w), np.float32) for w in widths]
        npu.mul_mat_group(keys, x.ctypes.data, T, [y.ctypes.data for y in got], False, fused)
        for k, f, y in zip(keys, fused, want):
            npu.mul_mat(k, x.ctypes.data, T, y.ctypes.data, False, fused=f)
    for a, b in zip(got, want):
        assert same_up_to_sum_order(a, b, rounded=False)
    t = npu.take_times()
    assert t.calls == 8
    npu.close()


def test_mul_mat_group_rejects_mixed_k():
    npu = Z.Npu(0)
    r1 = O.quantize(O.Q8_0, O.weights_f32(512, 256, 1))
    r2 = O.quantize(O.Q8_0, O.weights_f32(512, 512, 2))
    k1, k2 = Z.Npu.key(r1.ctypes.data, O.Q8_0, 256, 512), Z.Npu.key(r2.ctypes.data, O.Q8_0, 512, 512)
    npu.add_weight(k1, r1.ctypes.data, on_device=False)
    npu.add_weight(k2, r2.ctypes.data, on_device=False)
    x = O.activations(128, 256, 3)
    y1, y2 = np.empty((128, 512), np.float32), np.empty((128, 512), np.float32)
    with pytest.raises(Z.ZestError, match="differ in K"):
        npu.mul_mat_group([k1, k2], x.ctypes.data, 128, [y1.ctypes.data, y2.ctypes.data], False)
    npu.close()


def test_host_buffer_chunks_equal_one_pass():
    # host buffers cut into 256-row chunks (the last one ragged) overlap their
    # copies with the kernels; the results are those of one device-buffer pass
    # (up to the sum order: the chunks' launches split their tiles differently)
    code = textwrap.dedent(f"""
        import sys
        sys.path[:0] = [{str(ROOT)!r}, {str(ROOT / 'ggml-xdna_b200')!r}, {str(ROOT / 'tests')!r}]
        import numpy as np, torch, zest_b200 as Z
        from oracle import oracle as O
        from gpu_util import same_up_to_sum_order
        npu = Z.Npu(0)
        npu.set_out16(False)
        K, T = 512, 1000
        raws = [O.quantize(O.Q8_0, O.weights_f32(N, K, 70 + N)) for N in (768, 512)]
        keys = [Z.Npu.key(r.ctypes.data, O.Q8_0, K, N) for r, N in zip(raws, (768, 512))]
        for k, r in zip(keys, raws):
            npu.add_weight(k, r.ctypes.data, on_device=False)
        x = O.activations(T, K, 71)
        ys = [torch.empty((T, N), dtype=torch.float32).pin_memory() for N in (768, 512)]
        npu.mul_mat_group(keys, torch.from_numpy(x).pin_memory().data_ptr(), T, [y.data_ptr() for y in ys], False)
        xd = torch.from_numpy(x).cuda()
        yd = [torch.empty((T, N), dtype=torch.float32, device="cuda") for N in (768, 512)]
        torch.cuda.synchronize()
        npu.mul_mat_group(keys, xd.data_ptr(), T, [y.data_ptr() for y in yd], True)
        ok = all(same_up_to_sum_order(a.numpy(), b.cpu().numpy(), False) for a, b in zip(ys, yd))
        ph = np.empty((T, 768), np.float32)  # pageable host memory takes the same path
        npu.mul_mat(keys[0], x.ctypes.data, T, ph.ctypes.data, False)
        ok = ok and same_up_to_sum_order(ph, ys[0].numpy(), False)
        print("CHUNKS", "OK" if ok else "DIFFER")
    """)
    env = dict(os.environ, GGML_ZEST_CHUNK_ROWS="256")
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env, timeout=300)
    assert "CHUNKS OK" in r.stdout, r.stdout + r.stderr


_WIRE_CHILD = """
import sys
sys.path[:0] = [{root!r}, {pkg!r}, {tests!r}]
import numpy as np, torch, zest_b200 as Z
from oracle import oracle as O
npu = Z.Npu(0)  # GGML_XDNA_OUT16 unset: bf16-rounded results
K, T, F = 512, 1000, 300
raws = [O.quantize(O.Q8_0, O.weights_f32(N, K, 80 + N)) for N in (768, 512)]
keys = [Z.Npu.key(r.ctypes.data, O.Q8_0, K, N) for r, N in zip(raws, (768, 512))]
for k, r in zip(keys, raws):
    npu.add_weight(k, r.ctypes.data, on_device=False)
g, u = (O.quantize(O.Q8_0, O.weights_f32(F, K, s)) for s in (90, 91))
gkey = Z.Npu.key(g.ctypes.data, O.Q8_0, K, F)
npu.add_fused(gkey, g.ctypes.data, u.ctypes.data, on_device=False)
x = O.activations(T, K, 92)
xp = torch.from_numpy(x).pin_memory()
ys = [torch.empty((T, N), dtype=torch.float32).pin_memory() for N in (768, 512)]
npu.mul_mat_group(keys, xp.data_ptr(), T, [y.data_ptr() for y in ys], False)
sw = np.empty((T, F), np.float32)  # pageable host memory, SwiGLU results
npu.mul_mat(gkey, x.ctypes.data, T, sw.ctypes.data, False, fused=True)
np.savez({out!r}, y0=ys[0].numpy(), y1=ys[1].numpy(), sw=sw)
"""


def test_host_results_cross_pcie_as_bf16_exactly(tmp_path):
    # host-buffer calls send bf16-rounded results (the default output mode,
    # SwiGLU) to the host as bf16 and widen them there: the same f32 bits as
    # sending the f32 values (GGML_ZEST_WIRE16=0), chunk by chunk
    root = Z.PKG_DIR.parent
    got = {}
    for wire in ("1", "0"):
        out = tmp_path / f"wire{wire}.npz"
        code = _WIRE_CHILD.format(root=str(root), pkg=str(Z.PKG_DIR), tests=str(root / "tests"), out=str(out))
        env = dict(os.environ, GGML_ZEST_CHUNK_ROWS="256", GGML_ZEST_WIRE16=wire)
        r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env, timeout=300)
        assert r.returncode == 0, r.stdout + r.stderr
        got[wire] = np.load(out)
    for k in ("y0", "y1", "sw"):
        a, b = got["1"][k], got["0"][k]
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), k
        assert np.array_equal(a, O.round_bf16(a)), k


def test_async_weight_copies_equal_synchronous_ones():
    # with zest_set_load_async, copies from device-resident raw bytes are
    # built on the service's load stream and the add returns at once; the
    # first matmul waits for them on the GPU (the reference builds its copies
    # on a background thread, src/ggml-zest.cpp:261-330)
    N, K, T = 2048, 2560, 512
    raws = [O.quantize(O.Q4_K, O.weights_f32(N, K, 100 + i)) for i in range(4)]
    devs = [torch.from_numpy(r).cuda() for r in raws]
    keys = [Z.Npu.key(d.data_ptr(), O.Q4_K, K, N) for d in devs]
    x = dev(O.activations(T, K, 7))
    torch.cuda.synchronize()
    outs = {}
    for mode in ("async", "sync"):
        npu = Z.Npu(0)
        npu.set_out16(False)
        npu.set_load_async(mode == "async")
        for k, d in zip(keys, devs):
            npu.add_weight(k, d.data_ptr(), on_device=True)
        ys = [torch.empty((T, N), dtype=torch.float32, device="cuda") for _ in keys]
        for k, y in zip(keys, ys):
            npu.mul_mat(k, x.data_ptr(), T, y.data_ptr(), on_device=True)
        w_ptr, n_pad = npu.weight_bf16(keys[-1])  # waits for the copy on the host
        assert w_ptr and n_pad == N
        npu.wait_weights()
        outs[mode] = [host(y) for y in ys]
        npu.close()
    for a, b in zip(outs["async"], outs["sync"]):
        assert np.array_equal(a, b)


def test_submitted_groups_equal_synchronous_calls():
    # group calls in flight in every slot at once (their copies in and out
    # overlapping on PCIe), then each slot reused after its wait: the same
    # results, bit for bit, as the same calls made one at a time
    npu = Z.Npu(0)  # bf16-rounded results: they cross PCIe as bf16
    K, T, F = 512, 2600, 300  # 512-row chunks, the last one ragged
    Ns = (768, 256, 512)
    raws = [O.quantize(O.Q8_0, O.weights_f32(N, K, 100 + N)) for N in Ns]
    keys = [Z.Npu.key(r.ctypes.data, O.Q8_0, K, N) for r, N in zip(raws, Ns)]
    for k, r in zip(keys, raws):
        npu.add_weight(k, r.ctypes.data, on_device=False)
    g, u = (O.quantize(O.Q4_K, O.weights_f32(F, K, s)) for s in (110, 111))
    gkey = Z.Npu.key(g.ctypes.data, O.Q4_K, K, F)
    npu.add_fused(gkey, g.ctypes.data, u.ctypes.data, on_device=False)
    # (keys, fused, widths, input seed, pinned): five groups on four slots
    groups = [([keys[0], keys[1]], [False, False], [768, 256], 120, True),
              ([gkey], [True], [F], 121, True),
              ([keys[2]], [False], [512], 122, False),
              ([keys[0], gkey, keys[2]], [False, True, False], [768, F, 512], 123, True),
              ([keys[1]], [False], [256], 124, True)]

    def buffers(pinned, seed, widths):
        x = torch.from_numpy(O.activations(T, K, seed))
        ys = [torch.full((T, w), float("nan"), dtype=torch.float32) for w in widths]
        if pinned:
            x, ys = x.pin_memory(), [y.pin_memory() for y in ys]
        return x, ys

    want = []
    for ks, fu, widths, seed, pinned in groups:
        x, ys = buffers(pinned, seed, widths)
        npu.mul_mat_group(ks, x.data_ptr(), T, [y.data_ptr() for y in ys], False, fu)
        want.append([y.numpy().copy() for y in ys])
    bufs = [buffers(p, s, w) for _, _, w, s, p in groups]
    for rnd in range(2):  # twice: every slot takes a second call after its wait
        for y in (y for _, ys in bufs for y in ys):
            y.fill_(float("nan"))
        slot_of = {}
        for i, (ks, fu, _, _, _) in enumerate(groups):
            slot = i % Z.SLOTS
            if any(s == slot for s in slot_of.values()):
                j = next(j for j, s in slot_of.items() if s == slot)
                npu.wait_group(slot)
                del slot_of[j]
            x, ys = bufs[i]
            npu.submit_group(slot, ks, x.data_ptr(), T, [y.data_ptr() for y in ys], False, fu)
            slot_of[i] = slot
        for i, slot in slot_of.items():
            npu.wait_group(slot)
        for i in range(len(groups)):
            for got, exp in zip(bufs[i][1], want[i]):
                assert np.array_equal(got.numpy().view(np.uint32), exp.view(np.uint32)), (rnd, i)
    x, ys = bufs[0]
    with pytest.raises(Z.ZestError, match="nothing submitted"):
        npu.wait_group(0)
    npu.submit_group(0, groups[0][0], x.data_ptr(), T, [y.data_ptr() for y in ys], False, groups[0][1])
    with pytest.raises(Z.ZestError, match="not finished"):
        npu.submit_group(0, groups[0][0], x.data_ptr(), T, [y.data_ptr() for y in ys], False, groups[0][1])
    npu.wait_group(0)
    with pytest.raises(Z.ZestError, match="no such slot"):
        npu.wait_group(Z.SLOTS)
    npu.close()
