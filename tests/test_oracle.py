"""The oracle pinned before it is trusted (CPU only).

1. against the golden fixtures, which hold the reference's own outputs
   (tests/golden/make_golden.py) and gguf-py's dequantised values;
2. against the reference build (oracle/_ref), where it exists, on fresh
   inputs and every shape and tiling of tests/test-bfp16-pack.cpp:101,134-135;
3. the reference's own test binary, tests/test-bfp16-pack.cpp, built from its
   sources, must print ALL PASS.
"""
import subprocess
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O

GOLD = Path(__file__).resolve().parent / "golden"


def load(name):
    return np.load(GOLD / name)


def test_codec_matches_golden():
    g = load("codec.npz")
    assert np.array_equal(O.encode_blocks(g["x"]), g["bytes"])


def test_decode_every_exponent_byte():
    # tests/test-bfp16-pack.cpp:180-191: every exponent byte, mantissas -128..127
    blocks = []
    want = []
    for e in range(256):
        for base in range(-128, 128, 8):
            blocks.append([e] + [(base + i) & 0xFF for i in range(8)])
            want.extend(np.ldexp(np.arange(base, base + 8, dtype=np.float64), e - 133))
    got = O.decode_blocks(np.array(blocks, dtype=np.uint8))
    assert np.array_equal(got, np.array(want, dtype=np.float32))


def test_saturation_kat():
    # tests/test-bfp16-pack.cpp:168-175
    blk = np.array([127.75, 1.0, -3.5, 0.0, 64.0, -127.5, 0.25, 100.5], np.float32) / 64
    enc = O.encode_blocks(blk)
    assert enc[0] == 127 and np.int8(enc[1]) == 127 and np.int8(enc[6]) == -128 and np.int8(enc[8]) == 100


def test_zero_block():
    z = np.array([0.0, -0.0, 0.0, 0.0, -0.0, 0.0, 0.0, 0.0], np.float32)
    assert not O.encode_blocks(z).any()


def test_pack_a_matches_golden():
    g = load("pack_a_256x128.npz")
    assert np.array_equal(O.pack_a(g["x"]), g["bytes"])


def test_pack_b_matches_golden():
    g = load("pack_b_512x128.npz")
    assert np.array_equal(O.pack_b(g["w"]), g["bytes"])


def test_gate_up_matches_golden():
    g = load("gate_up_256x64.npz")
    assert np.array_equal(O.pack_b(O.interleave_gate_up(g["gate"], g["up"])), g["bytes"])


@pytest.mark.parametrize("name,qt", [("q8_0", O.Q8_0), ("q4_k", O.Q4_K), ("q6_k", O.Q6_K), ("iq3_s", O.IQ3_S)])
def test_dequant_matches_gguf_golden(name, qt):
    g = load(f"dequant_{name}.npz")
    got = O.dequant(qt, g["raw"], 16, 512)
    assert np.array_equal(got.view(np.uint32), g["values"].view(np.uint32))


def test_mul_mat_matches_reference_golden():
    g = load("mul_mat_q8_0.npz")
    N, K, M = int(g["N"]), int(g["K"]), int(g["M"])
    W = O.dequant(O.Q8_0, g["raw"], N, K)
    assert O.nmax_err(O.mul_mat(W, g["x"]), g["y"]) < 1e-6
    Xd = O.decode_blocks(O.encode_blocks(g["x"])).reshape(M, K)
    Wd = O.decode_blocks(O.encode_blocks(W)).reshape(N, K)
    assert O.nmax_err(O.mul_mat(Wd, Xd), g["y_decoded"]) < 1e-6


def test_unpack_inverts_pack():
    x = O.make_data(256 * 192, 9).reshape(256, 192)
    b = O.pack_a(x)
    want = O.decode_blocks(O.encode_blocks(x)).reshape(256, 192)
    assert np.array_equal(O.unpack_a(b, 256, 192), want)
    w = O.make_data(512 * 64, 10).reshape(512, 64)
    assert np.array_equal(O.unpack_b(O.pack_b(w), 512, 64), O.decode_blocks(O.encode_blocks(w)).reshape(512, 64))


def test_quantisers_round_trip():
    for qt, tol in ((O.Q8_0, 0.01), (O.Q4_K, 0.1), (O.Q6_K, 0.03), (O.IQ3_S, 0.3)):
        w = O.weights_f32(8, 512, 3)
        d = O.dequant(qt, O.quantize(qt, w), 8, 512)
        assert np.abs(d - w).max() / np.abs(w).max() < tol, qt


def test_bf16_rounding():
    x = np.array([1.0, 1.00390625, 1.005859375, -2.5e-3, 3e38], np.float32)
    r = O.round_bf16(x)
    assert r[0] == 1.0 and r[1] == 1.0 and r[2] == np.float32(1.0078125)
    assert np.array_equal(r.view(np.uint32) & 0xFFFF, np.zeros(5, np.uint32))


needs_ref = pytest.mark.skipif(not O.has_ref(), reason="oracle/_ref not built here (needs the reference sources)")


@needs_ref
def test_codec_matches_reference_build():
    x = O.make_data(8 * 20000, 77)
    assert np.array_equal(O.encode_blocks(x), O.ref_encode_blocks(x))


@needs_ref
@pytest.mark.parametrize("M,K,m,k", [(512, 256, 128, 64), (256, 384, 64, 128), (1024, 6144, 128, 64)])
def test_pack_a_matches_reference_build(M, K, m, k):
    x = O.make_data(M * K, 1 + M + K).reshape(M, K)
    assert np.array_equal(O.pack_a(x, O.tiling(m, k)), O.ref_pack_a(x, m, k))


@needs_ref
@pytest.mark.parametrize("N,K,n,k,cols", [(1024, 256, 64, 64, 8), (4096, 2048, 64, 64, 8), (2048, 6144, 64, 128, 8),
                                          (512, 128, 32, 64, 4)])
def test_pack_b_matches_reference_build(N, K, n, k, cols):
    w = O.make_data(N * K, 7 + N + K).reshape(N, K)
    assert np.array_equal(O.pack_b(w, O.tiling(128, k, n, cols)), O.ref_pack_b(w, n, k, cols))


@needs_ref
@pytest.mark.parametrize("qt", [O.Q8_0, O.Q4_K, O.Q6_K, O.IQ3_S])
def test_mul_mat_matches_reference_build(qt):
    N, K, M = 256, 512, 32
    raw = O.quantize(qt, O.weights_f32(N, K, qt))
    X = O.activations(M, K, 5)
    want = O.ref_mul_mat(qt, raw, N, K, X, n_threads=4)
    assert O.nmax_err(O.mul_mat(O.dequant(qt, raw, N, K), X), want) < 1e-6


@pytest.mark.skipif(not O.REF_TEST.exists(), reason="the reference's test binary is not built here")
def test_reference_pack_test_passes():
    out = subprocess.run([str(O.REF_TEST)], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0 and "ALL PASS" in out.stdout, out.stdout[-2000:]


def test_selftest_operands():
    a, w = O.selftest_operands()
    assert a.min() >= -2 and a.max() <= 2 and w.min() >= -3 and w.max() <= 3
    assert a.shape == (512, 128) and w.shape == (512, 128)


def _host_ops():
    import json
    import sys
    sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
    import host_ops as HO
    g = np.load(Path(__file__).resolve().parent / "golden" / "host_ops.npz")
    cases = json.loads(str(g["cases"]))
    for i, (name, spec) in enumerate(cases):
        inp = {k.split("/", 1)[1]: g[k] for k in g.files if k.startswith(f"{i}/") and not k.endswith("/y")}
        yield HO, i, name, spec, inp, g[f"{i}/y"]


def test_small_ops_match_the_reference_executor_fixtures():
    # the oracle's restatement of run_rows (and its rope table) against the
    # outputs of the reference's own executor (tests/golden/host_ops.npz), the
    # 21 cases of tests/test-host-ops.cpp plus the two fused forms, at the
    # reference's own bar (nrmse <= 1e-5)
    n = 0
    for HO, i, name, spec, inp, want in _host_ops():
        got = HO.run(i, spec, HO.oracle_ops(O), inp)
        assert O.nrmse(got, want) <= 1e-5, name
        n += 1
    assert n == 23


@pytest.mark.skipif(not O.has_ref(), reason="oracle/_ref not built (needs the reference sources)")
def test_reference_executor_reproduces_its_fixtures():
    # the reference build here gives the committed fixtures back
    for HO, i, name, spec, inp, want in _host_ops():
        got = HO.run(i, spec, HO.reference_ops(O), inp)
        assert O.nrmse(got, want) <= 1e-6, name
