"""K3, the tensor-core GEMM, through the C ABI.

Parity bar (the north star's): max|C_gpu - C_ref| / max|C_ref| <= 1e-3, where
C_ref is the reference's CPU matmul (xdna-ref) on the bfp16-decoded operands.
The products are exact in bf16 x bf16 -> fp32, so only the summation order
differs; the measured error is ~1e-6. Integer operands must match exactly.
"""
import numpy as np
import pytest
import torch

import zest_b200 as Z
from oracle import oracle as O
from gpu_util import bf16_to_f32, dev, host, same_up_to_sum_order

pytestmark = pytest.mark.gpu

TOL = 1e-3


def operands(M, N, K, qt=O.Q8_0, seed=0, outliers=False):
    raw = O.quantize(qt, O.weights_f32(N, K, seed + 1))
    x = O.activations(M, K, seed + 2, outliers=outliers)
    _, bh = Z.convert_weight(qt, dev(raw), N, K)
    _, ah = Z.pack_activations(dev(x))
    a_dec = bf16_to_f32(host(ah)[:M].view(np.uint16))
    b_dec = bf16_to_f32(host(bh)[:N].view(np.uint16))
    return ah, bh, a_dec, b_dec, raw, x


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 512, 128), (1000, 1000, 320), (96, 4096, 2560),
                                   (513, 777, 1024)])
def test_gemm_f32_vs_oracle(M, N, K):
    ah, bh, a_dec, b_dec, _, _ = operands(M, N, K, seed=M + N)
    c = host(Z.gemm(ah, bh, M, N))
    want = O.mul_mat(b_dec, a_dec)
    assert O.nmax_err(c, want) <= TOL


@pytest.mark.parametrize("bn", ["256", "192", "160", "128"])
@pytest.mark.parametrize("mode", [Z.MODE_F32, Z.MODE_BF16])
def test_gemm_pair_tile_widths(bn, mode, monkeypatch):
    # every N tile of the CTA-pair kernel, on a ragged shape (M, N not tile multiples)
    monkeypatch.setenv("ZEST_GEMM_BN", bn)
    M, N, K = 777, 1000, 576
    ah, bh, a_dec, b_dec, _, _ = operands(M, N, K, seed=int(bn))
    c = host(Z.gemm(ah, bh, M, N, mode))
    want = O.mul_mat(b_dec, a_dec)
    if mode == Z.MODE_BF16:
        assert np.array_equal(c, O.round_bf16(c))
        assert O.nmax_err(c, want) <= 4e-3
    else:
        assert O.nmax_err(c, want) <= TOL


def test_gemm_pair_and_single_agree(monkeypatch):
    # the CTA-pair kernel and the one-CTA kernel accumulate in the same k order
    M, N, K = 640, 768, 1024
    ah, bh, _, _, _, _ = operands(M, N, K, seed=4)
    monkeypatch.setenv("ZEST_GEMM_PAIR", "0")
    c1 = host(Z.gemm(ah, bh, M, N))
    monkeypatch.setenv("ZEST_GEMM_PAIR", "1")
    c2 = host(Z.gemm(ah, bh, M, N))
    assert O.nmax_err(c2, c1) <= 1e-6


def test_gemm_exact_integers():
    a, w = O.selftest_operands(512, 128, 512)
    ah = dev(O.decode_blocks(O.encode_blocks(a.astype(np.float32))).reshape(512, 128))
    _, ah = Z.pack_activations(ah)
    _, bh = Z.convert_weight(O.F32, dev(w.astype(np.float32).view(np.uint8)), 512, 128)
    c = host(Z.gemm(ah, bh, 512, 512))
    want = a.astype(np.int64) @ w.astype(np.int64).T
    assert np.array_equal(c, want.astype(np.float32))


def test_gemm_matches_reference_golden():
    g = np.load(Z.PKG_DIR.parent / "tests" / "golden" / "mul_mat_q8_0.npz")
    N, K, M = int(g["N"]), int(g["K"]), int(g["M"])
    _, bh = Z.convert_weight(O.Q8_0, dev(g["raw"]), N, K)
    _, ah = Z.pack_activations(dev(g["x"]))
    c = host(Z.gemm(ah, bh, M, N))
    assert O.nmax_err(c, g["y_decoded"]) <= TOL
    # against the reference on the unrounded operands: the bfp16 rounding's own error
    assert O.nmax_err(c, g["y"]) < 5e-2


def test_gemm_config1_rows():
    # config 1: 1024 x 2560 activations, Q8_0 9728 x 2560 weight; 64 rows checked in full
    M, N, K = 1024, 9728, 2560
    ah, bh, a_dec, b_dec, _, _ = operands(M, N, K, seed=1)
    c = host(Z.gemm(ah, bh, M, N))
    rows = np.r_[0:32, 992:1024]
    assert O.nmax_err(c[rows], O.mul_mat(b_dec, a_dec[rows])) <= TOL


def test_gemm_bf16_mode_is_rounded_f32():
    M, N, K = 384, 768, 512
    ah, bh, _, _, _, _ = operands(M, N, K, seed=3)
    c0 = host(Z.gemm(ah, bh, M, N, Z.MODE_F32))
    c1 = host(Z.gemm(ah, bh, M, N, Z.MODE_BF16))
    assert np.array_equal(c1, O.round_bf16(c0))


def test_gemm_swiglu_mode():
    M, F, K = 256, 300, 512
    gr = O.quantize(O.Q4_K, O.weights_f32(F, K, 1))
    ur = O.quantize(O.Q4_K, O.weights_f32(F, K, 2))
    _, bh = Z.convert_gate_up(O.Q4_K, dev(gr), dev(ur), F, K)
    _, ah = Z.pack_activations(dev(O.activations(M, K, 3)))
    n = bh.shape[0]  # 2 * f_pad
    acc = host(Z.gemm(ah, bh, M, n, Z.MODE_F32))
    got = host(Z.gemm(ah, bh, M, n, Z.MODE_SWIGLU))
    idx = np.arange(F)
    at = (idx // 8) * 16 + idx % 8
    want = O.swiglu_bf16(acc[:, at], acc[:, at + 8])
    assert got.shape == (M, n // 2)
    g = got[:, :F]
    # one bf16 ulp at most (SiLU's exp differs in its last fp32 bits)
    ulp = np.abs(g.view(np.int32).astype(np.int64) - want.view(np.int32).astype(np.int64)) >> 16
    assert ulp.max() <= 1
    assert not got[:, F:].any()


def test_gemm_flags_non_finite():
    M, N, K = 128, 512, 64
    w = O.weights_f32(N, K, 1)
    w[7, 3] = np.inf
    _, bh = Z.convert_weight(O.F32, dev(w.view(np.uint8)), N, K)
    _, ah = Z.pack_activations(dev(O.activations(M, K, 2)))
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    Z.gemm(ah, bh, M, N, err=err)
    assert int(err.item()) & Z.ERR_NOT_FINITE


def test_gemm_full_size_vs_torch_fp32():
    # config 2's largest projection shape at M=8192 against cuBLAS fp32 on the same decoded operands
    torch.backends.cuda.matmul.allow_tf32 = False
    M, N, K = 8192, 9728, 2560
    g = torch.Generator("cuda").manual_seed(5)
    x = torch.randn(M, K, device="cuda", generator=g)
    w = torch.randn(N, K, device="cuda", generator=g) * 0.02
    _, ah = Z.pack_activations(x)
    _, bh = Z.convert_weight(O.F32, w.contiguous().view(torch.uint8), N, K)
    c = Z.gemm(ah, bh, M, N)
    a32 = (ah.to(torch.int32) << 16).view(torch.float32)
    b32 = (bh[:N].to(torch.int32) << 16).view(torch.float32)
    ref = a32 @ b32.T
    err = ((c - ref).abs().max() / ref.abs().max()).item()
    assert err <= TOL, err


@pytest.mark.parametrize("pair", ["1", "0"])
@pytest.mark.parametrize("bn", ["256", "128"])
def test_gemm_group_equals_separate_launches(pair, bn, monkeypatch):
    # q/k/v-like segments of ragged widths plus a SwiGLU gate/up segment sharing A:
    # one grouped launch gives what a launch per weight gives (up to the sum order)
    monkeypatch.setenv("ZEST_GEMM_PAIR", pair)
    monkeypatch.setenv("ZEST_GEMM_BN", bn)
    M, K = 900, 640
    _, ah = Z.pack_activations(dev(O.activations(M, K, 7)))
    Ns, modes, bs = [1000, 300, 512], [Z.MODE_F32, Z.MODE_BF16, Z.MODE_F32], []
    for i, N in enumerate(Ns):
        _, bh = Z.convert_weight(O.Q8_0, dev(O.quantize(O.Q8_0, O.weights_f32(N, K, 20 + i))), N, K)
        bs.append(bh)
    F = 200
    gr = O.quantize(O.Q8_0, O.weights_f32(F, K, 30))
    ur = O.quantize(O.Q8_0, O.weights_f32(F, K, 31))
    _, gu = Z.convert_gate_up(O.Q8_0, dev(gr), dev(ur), F, K)
    bs.append(gu)
    Ns.append(gu.shape[0])
    modes.append(Z.MODE_SWIGLU)
    outs = Z.gemm_group(ah, bs, M, Ns, modes)
    for b, N, m, o in zip(bs, Ns, modes, outs):
        assert same_up_to_sum_order(host(o), host(Z.gemm(ah, b, M, N, m)), rounded=m != Z.MODE_F32)


def test_gemm_group_vs_oracle():
    M, K = 1300, 512
    x = O.activations(M, K, 9)
    _, ah = Z.pack_activations(dev(x))
    a_dec = bf16_to_f32(host(ah)[:M].view(np.uint16))
    Ns, bs, decs = [768, 256], [], []
    for i, N in enumerate(Ns):
        _, bh = Z.convert_weight(O.Q6_K, dev(O.quantize(O.Q6_K, O.weights_f32(N, K, 40 + i))), N, K)
        bs.append(bh)
        decs.append(bf16_to_f32(host(bh)[:N].view(np.uint16)))
    outs = Z.gemm_group(ah, bs, M, Ns, [Z.MODE_F32, Z.MODE_F32])
    for o, d in zip(outs, decs):
        assert O.nmax_err(host(o), O.mul_mat(d, a_dec)) <= TOL


def test_gemm_group_rejects_bad_groups():
    _, ah = Z.pack_activations(dev(O.activations(256, 64, 1)))
    _, bh = Z.convert_weight(O.F32, dev(O.weights_f32(512, 64, 2).view(np.uint8)), 512, 64)
    with pytest.raises(Z.ZestError, match="1 to 4"):
        Z.gemm_group(ah, [bh] * 5, 256, [512] * 5, [Z.MODE_F32] * 5)
    with pytest.raises(Z.ZestError, match="mode"):
        Z.gemm_group(ah, [bh, bh], 256, [512, 500], [Z.MODE_F32, Z.MODE_SWIGLU])


_SK_CHILD = """
import sys
sys.path[:0] = [{root!r}, {pkg!r}, {tests!r}]
import numpy as np, torch, zest_b200 as Z
from oracle import oracle as O
from gpu_util import dev, host, bf16_to_f32, same_up_to_sum_order
ok = True
for M, N, K, mode in [(2048, 2560, 4096, 0), (512, 2560, 4096, 0), (1024, 9728, 2560, 1), (2048, 2560, 9728, 1)]:
    _, bh = Z.convert_weight(O.Q8_0, dev(O.quantize(O.Q8_0, O.weights_f32(N, K, M + 1))), N, K)
    x = O.activations(M, K, M + 2)
    _, ah = Z.pack_activations(dev(x))
    c_sk = host(Z.gemm(ah, bh, M, N, mode))
    import os
    os.environ["ZEST_GEMM_PAIR"] = "0"
    c_whole = host(Z.gemm(ah, bh, M, N, mode))
    del os.environ["ZEST_GEMM_PAIR"]
    ok &= same_up_to_sum_order(c_sk, c_whole, rounded=mode != 0)
    rows = np.r_[0:16, M - 16:M]
    a_dec = bf16_to_f32(host(ah)[:M].view(np.uint16))[rows]
    b_dec = bf16_to_f32(host(bh)[:N].view(np.uint16))
    ok &= O.nmax_err(c_sk[rows], O.mul_mat(b_dec, a_dec)) <= (4e-3 if mode else 1e-3)
# the tile that collects other pairs' partial sums applies SwiGLU to the completed sum
M, F, K = 2048, 2560, 4096
gr = O.quantize(O.Q8_0, O.weights_f32(F, K, 11))
ur = O.quantize(O.Q8_0, O.weights_f32(F, K, 12))
_, gu = Z.convert_gate_up(O.Q8_0, dev(gr), dev(ur), F, K)
_, ah = Z.pack_activations(dev(O.activations(M, K, 13)))
n = gu.shape[0]
acc = host(Z.gemm(ah, gu, M, n, 0))
got = host(Z.gemm(ah, gu, M, n, 2))
idx = np.arange(F)
at = (idx // 8) * 16 + idx % 8
ok &= same_up_to_sum_order(got[:, :F], O.swiglu_bf16(acc[:, at], acc[:, at + 8]), rounded=True)
# the residual ADD on completed sums: the same split as the plain launch, so
# the sum order matches and the result is the plain one plus the residual
import ctypes
M, N, K = 2048, 2560, 4096
_, bh = Z.convert_weight(O.Q8_0, dev(O.quantize(O.Q8_0, O.weights_f32(N, K, 14))), N, K)
_, ah = Z.pack_activations(dev(O.activations(M, K, 15)))
resid = torch.randn((M, N), device="cuda", generator=torch.Generator("cuda").manual_seed(16))
c = torch.empty((M, N), device="cuda")
err = torch.zeros(1, dtype=torch.int32, device="cuda")
seg = (Z.GemmSeg * 1)(Z.GemmSeg(bh.data_ptr(), K, N, Z.MODE_BF16, c.data_ptr(), N, resid.data_ptr(), N, None, 0))
L = Z.lib()
rc = L.zest_gemm_segs(ctypes.c_void_p(ah.data_ptr()), K, M, K, 1, seg, ctypes.c_void_p(err.data_ptr()),
                      ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
assert rc == 0, L.zest_last_error().decode()
plain = host(Z.gemm(ah, bh, M, N, Z.MODE_BF16))
ok &= bool(np.array_equal(host(c), host(resid) + plain)) and int(err.item()) == 0
print("STREAMK", "OK" if ok else "DIFFER")
"""


def test_stream_k_matches_whole_tiles():
    # with ZEST_GEMM_SK=1, launches whose last wave would leave pairs idle
    # split it in k across all pairs (tiles of 80, 20, 152 and 80 on 74 pairs,
    # SwiGLU on the completed sums); the one-CTA kernel runs every tile whole
    import os
    import subprocess
    import sys
    root = Z.PKG_DIR.parent
    code = _SK_CHILD.format(root=str(root), pkg=str(Z.PKG_DIR), tests=str(root / "tests"))
    env = dict(os.environ, ZEST_GEMM_SK="1")
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env, timeout=600)
    assert "STREAMK OK" in r.stdout, r.stdout + r.stderr


def test_stream_k_order_survives_a_capture():
    # Stream-K launches share one workspace per device. A live launch on
    # stream A (held back behind a GPU sleep), then one captured into a CUDA
    # graph on stream B, then a live one on stream C: C must still wait for
    # A, whatever the capture did in between.
    import time
    M, N, K = 2048, 2560, 9728
    assert Z.plan_gemm(M, K, [N])["stream_k"] == 1
    _, bh = Z.convert_weight(O.Q8_0, dev(O.quantize(O.Q8_0, O.weights_f32(N, K, 61))), N, K)
    _, ah = Z.pack_activations(dev(O.activations(M, K, 62)))
    torch.cuda.synchronize()
    outs = [torch.zeros((M, N), dtype=torch.float32, device="cuda") for _ in range(3)]
    errs = [torch.zeros(1, dtype=torch.int32, device="cuda") for _ in range(3)]
    sa, sb, sc = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream()
    with torch.cuda.stream(sa):
        torch.cuda._sleep(1_000_000_000)  # about half a second or more
        Z.gemm(ah, bh, M, N, out=outs[0], err=errs[0])
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(sb):  # capture_begin, unlike torch.cuda.graph, does not synchronize first
        g.capture_begin(capture_error_mode="relaxed")
        Z.gemm(ah, bh, M, N, out=outs[1], err=errs[1])
        g.capture_end()
    with torch.cuda.stream(sc):
        Z.gemm(ah, bh, M, N, out=outs[2], err=errs[2])
        done_c = torch.cuda.Event()
        done_c.record(sc)
    time.sleep(0.1)
    waited = not done_c.query()
    torch.cuda.synchronize()
    g.replay()
    torch.cuda.synchronize()
    assert waited, "the launch on C ran while the one on A was still held back"
    assert all(int(e.item()) == 0 for e in errs)
    want = host(outs[0])
    assert np.array_equal(host(outs[2]), want)
    assert same_up_to_sum_order(host(outs[1]), want, rounded=False)
