"""ctypes wrappers over the CPU oracle: TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
legs may import this module, as the checker. The product (libzest_b200.so,
libggml-zest.so) never calls it.

Two libraries:
  oracle/libzest_oracle.so    the plain-C restatement (zest_oracle.c)
  oracle/_ref/libzest_ref.so  the reference's own bfp16_pack.cpp and
                              xdna-ref.cpp, compiled from its sources
                              (oracle/Makefile); present wherever it was built
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "libzest_oracle.so"
REF_SO = HERE / "_ref" / "libzest_ref.so"
REF_TEST = HERE / "_ref" / "test-bfp16-pack"

F32, F16, Q8_0, Q4_K, Q6_K, IQ3_S = 0, 1, 8, 12, 14, 21
QUANT = {F32: (1, 4), F16: (1, 2), Q8_0: (32, 34), Q4_K: (256, 144), Q6_K: (256, 210), IQ3_S: (256, 110)}

_i64, _vp, _int = ctypes.c_int64, ctypes.c_void_p, ctypes.c_int


class Tiling(ctypes.Structure):
    _fields_ = [("m", _int), ("k", _int), ("n", _int), ("cols", _int)]


DEFAULT_TILING = (128, 64, 64, 8)  # bfp16_tiling (src/npu/bfp16_pack.h:37-41)

_orc = None
_ref = None


def _p(a: np.ndarray):
    return a.ctypes.data_as(_vp)


def orc() -> ctypes.CDLL:
    global _orc
    if _orc is None:
        if not ORACLE_SO.exists():
            raise RuntimeError(f"{ORACLE_SO} missing: make -C oracle")
        L = ctypes.CDLL(str(ORACLE_SO))
        L.zo_a_offset.restype = ctypes.c_size_t
        L.zo_a_offset.argtypes = [_i64, _i64, _i64, ctypes.POINTER(Tiling)]
        L.zo_b_offset.restype = ctypes.c_size_t
        L.zo_b_offset.argtypes = [_i64, _i64, _i64, _i64, ctypes.POINTER(Tiling)]
        for n in ("zo_pack_a", "zo_pack_b", "zo_unpack_a", "zo_unpack_b"):
            getattr(L, n).argtypes = [_vp, _i64, _i64, ctypes.POINTER(Tiling), _vp]
        L.zo_encode_blocks.argtypes = [_vp, _i64, _vp]
        L.zo_decode_blocks.argtypes = [_vp, _i64, _vp]
        L.zo_interleave_gate_up.argtypes = [_vp, _vp, _i64, _i64, _vp]
        L.zo_set_iq3s_grid.argtypes = [_vp]
        L.zo_dequant.argtypes = [_int, _vp, _i64, _i64, _vp]
        L.zo_quantize.argtypes = [_int, _vp, _i64, _i64, _vp]
        L.zo_mul_mat.argtypes = [_vp, _i64, _vp, _i64, _i64, _vp, _int]
        L.zo_mul_mat_f64.argtypes = [_vp, _i64, _vp, _i64, _i64, _vp, _int]
        L.zo_round_bf16.restype = ctypes.c_float
        L.zo_round_bf16.argtypes = [ctypes.c_float]
        L.zo_swiglu_bf16.restype = ctypes.c_float
        L.zo_swiglu_bf16.argtypes = [ctypes.c_float, ctypes.c_float]
        L.zo_selftest_operands.argtypes = [_i64, _i64, _i64, _vp, _vp]
        L.zo_row_bytes.restype = _i64
        L.zo_row_bytes.argtypes = [_int, _i64]
        try:  # the codebook goes in before any other thread can see the library
            g = np.ascontiguousarray(iq3s_grid(), dtype=np.uint32)
            L.zo_set_iq3s_grid(_p(g))
        except ImportError:
            pass
        _orc = L
    return _orc


def has_ref() -> bool:
    return REF_SO.exists()


def ref() -> ctypes.CDLL:
    global _ref
    if _ref is None:
        if not REF_SO.exists():
            raise RuntimeError(f"{REF_SO} missing: make -C oracle ref (needs the reference sources)")
        orc()  # the reference build's to_float needs the codebook too
        L = ctypes.CDLL(str(REF_SO))
        L.zr_encode_block.argtypes = [_vp, _vp]
        L.zr_decode_block.argtypes = [_vp, _vp]
        L.zr_pack_a.argtypes = [_vp, _i64, _i64, _int, _int, _vp, _int]
        L.zr_pack_b.argtypes = [_vp, _i64, _i64, _int, _int, _int, _vp, _int]
        L.zr_unpack_a.argtypes = [_vp, _i64, _i64, _int, _int, _vp]
        L.zr_unpack_b.argtypes = [_vp, _i64, _i64, _int, _int, _int, _vp]
        L.zr_interleave_gate_up.argtypes = [_vp, _vp, _i64, _i64, _vp]
        L.zr_mul_mat.argtypes = [_int, _vp, _i64, _i64, _vp, _i64, _vp, _int]
        _f = ctypes.c_float
        L.zr_rms_norm.argtypes = [_vp, _i64, _i64, _f, _vp, _int]
        L.zr_mul_row.argtypes = [_vp, _vp, _i64, _i64, _vp, _int]
        L.zr_add.argtypes = [_vp, _vp, _int, _i64, _i64, _vp, _int]
        L.zr_scale.argtypes = [_vp, _i64, _i64, _f, _f, _vp, _int]
        L.zr_glu.argtypes = [_int, _int, _vp, _vp, _i64, _i64, _vp, _int]
        L.zr_rope.argtypes = [_vp, _i64, _i64, _i64, _vp, _int, _int, _int, _vp, _vp, _vp, _int]
        L.zr_norm_mul.argtypes = [_vp, _i64, _i64, _f, _vp, _vp, _int]
        L.zr_norm_mul_rope.argtypes = [_vp, _i64, _i64, _i64, _f, _vp, _vp, _int, _int, _int, _vp, _vp, _vp, _int]
        for n in ("zr_rms_norm", "zr_mul_row", "zr_add", "zr_scale", "zr_glu", "zr_rope", "zr_norm_mul",
                  "zr_norm_mul_rope"):
            getattr(L, n).restype = _int
        # the reference build links its own copy of the oracle's dequantisers
        L.zo_set_iq3s_grid.argtypes = [_vp]
        try:
            g = np.ascontiguousarray(iq3s_grid())
            L.zo_set_iq3s_grid(_p(g))
        except ImportError:
            pass
        _ref = L
    return _ref


def iq3s_grid() -> np.ndarray:
    """ggml's IQ3_S codebook from the installed gguf package (uint32 x 512)."""
    from gguf.quants import IQ3_S as _IQ3S
    _IQ3S.init_grid()
    g = np.asarray(_IQ3S.grid, dtype=np.float32).reshape(512, 4).astype(np.uint32)
    return (g[:, 0] | (g[:, 1] << 8) | (g[:, 2] << 16) | (g[:, 3] << 24)).astype(np.uint32)


def set_iq3s_grid(g: np.ndarray) -> None:
    g = np.ascontiguousarray(g, dtype=np.uint32)
    orc().zo_set_iq3s_grid(_p(g))


def tiling(m=128, k=64, n=64, cols=8) -> Tiling:
    return Tiling(m, k, n, cols)


# --- codec and layouts ---------------------------------------------------------

def encode_blocks(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    out = np.empty(x.size // 8 * 9, dtype=np.uint8)
    orc().zo_encode_blocks(_p(x), x.size // 8, _p(out))
    return out


def decode_blocks(b: np.ndarray) -> np.ndarray:
    b = np.ascontiguousarray(b, dtype=np.uint8).reshape(-1)
    out = np.empty(b.size // 9 * 8, dtype=np.float32)
    orc().zo_decode_blocks(_p(b), b.size // 9, _p(out))
    return out


def pack_a(x: np.ndarray, t: Tiling | None = None) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    M, K = x.shape
    out = np.zeros(M * K // 8 * 9, dtype=np.uint8)
    orc().zo_pack_a(_p(x), M, K, ctypes.byref(t or tiling()), _p(out))
    return out


def pack_b(w: np.ndarray, t: Tiling | None = None) -> np.ndarray:
    w = np.ascontiguousarray(w, dtype=np.float32)
    N, K = w.shape
    out = np.zeros(N * K // 8 * 9, dtype=np.uint8)
    orc().zo_pack_b(_p(w), N, K, ctypes.byref(t or tiling()), _p(out))
    return out


def unpack_a(b: np.ndarray, M: int, K: int, t: Tiling | None = None) -> np.ndarray:
    out = np.empty((M, K), dtype=np.float32)
    orc().zo_unpack_a(_p(np.ascontiguousarray(b)), M, K, ctypes.byref(t or tiling()), _p(out))
    return out


def unpack_b(b: np.ndarray, N: int, K: int, t: Tiling | None = None) -> np.ndarray:
    out = np.empty((N, K), dtype=np.float32)
    orc().zo_unpack_b(_p(np.ascontiguousarray(b)), N, K, ctypes.byref(t or tiling()), _p(out))
    return out


def interleave_gate_up(g: np.ndarray, u: np.ndarray) -> np.ndarray:
    g = np.ascontiguousarray(g, dtype=np.float32)
    u = np.ascontiguousarray(u, dtype=np.float32)
    F, K = g.shape
    out = np.empty((2 * F, K), dtype=np.float32)
    orc().zo_interleave_gate_up(_p(g), _p(u), F, K, _p(out))
    return out


# --- GGUF ----------------------------------------------------------------------

def row_bytes(qtype: int, k: int) -> int:
    qk, bb = QUANT[qtype]
    return k // qk * bb


def quantize(qtype: int, x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, k = x.shape
    out = np.zeros(rows * row_bytes(qtype, k), dtype=np.uint8)
    if orc().zo_quantize(qtype, _p(x), rows, k, _p(out)):
        raise ValueError(f"cannot quantise type {qtype} with k={k}")
    return out


def dequant(qtype: int, raw: np.ndarray, rows: int, k: int) -> np.ndarray:
    out = np.empty((rows, k), dtype=np.float32)
    if orc().zo_dequant(qtype, _p(np.ascontiguousarray(raw, dtype=np.uint8)), rows, k, _p(out)):
        raise ValueError(f"cannot dequantise type {qtype} with k={k}")
    return out


# --- matmul ----------------------------------------------------------------------

def mul_mat(W: np.ndarray, X: np.ndarray, n_threads: int = 8) -> np.ndarray:
    """Y[M][N] = X[M][K] * W[N][K]^T, float accumulation in k order (xdna-ref)."""
    W = np.ascontiguousarray(W, dtype=np.float32)
    X = np.ascontiguousarray(X, dtype=np.float32)
    N, K = W.shape
    M = X.shape[0]
    Y = np.empty((M, N), dtype=np.float32)
    orc().zo_mul_mat(_p(W), N, _p(X), M, K, _p(Y), n_threads)
    return Y


def mul_mat_f64(W: np.ndarray, X: np.ndarray, n_threads: int = 8) -> np.ndarray:
    W = np.ascontiguousarray(W, dtype=np.float32)
    X = np.ascontiguousarray(X, dtype=np.float32)
    N, K = W.shape
    M = X.shape[0]
    Y = np.empty((M, N), dtype=np.float64)
    orc().zo_mul_mat_f64(_p(W), N, _p(X), M, K, _p(Y), n_threads)
    return Y


def round_bf16(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = np.where(nan, (u | 0x00400000).astype(np.uint32), r)
    return r.view(np.float32)


def swiglu_bf16(g: np.ndarray, u: np.ndarray) -> np.ndarray:
    g64 = g.astype(np.float64)
    return round_bf16((g64 / (1.0 + np.exp(-g64)) * u.astype(np.float64)).astype(np.float32))


def selftest_operands(M=512, K=128, N=512):
    a = np.empty(M * K, dtype=np.int8)
    w = np.empty(N * K, dtype=np.int8)
    orc().zo_selftest_operands(M, K, N, _p(a), _p(w))
    return a.reshape(M, K), w.reshape(N, K)


# --- the reference build ------------------------------------------------------------

def ref_pack_a(x: np.ndarray, m=128, k=64, n_threads=8) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    M, K = x.shape
    out = np.zeros(M * K // 8 * 9, dtype=np.uint8)
    ref().zr_pack_a(_p(x), M, K, m, k, _p(out), n_threads)
    return out


def ref_pack_b(w: np.ndarray, n=64, k=64, cols=8, n_threads=8) -> np.ndarray:
    w = np.ascontiguousarray(w, dtype=np.float32)
    N, K = w.shape
    out = np.zeros(N * K // 8 * 9, dtype=np.uint8)
    ref().zr_pack_b(_p(w), N, K, n, k, cols, _p(out), n_threads)
    return out


def ref_encode_blocks(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, 8)
    out = np.empty((x.shape[0], 9), dtype=np.uint8)
    L = ref()
    for i in range(x.shape[0]):
        L.zr_encode_block(_p(x[i]), _p(out[i]))
    return out.reshape(-1)


def ref_mul_mat(qtype: int, raw_w: np.ndarray, N: int, K: int, X: np.ndarray, n_threads: int = 8) -> np.ndarray:
    """xdna_ref_mul_mat on a raw GGUF weight [N rows of K] and f32 X [M][K]."""
    X = np.ascontiguousarray(X, dtype=np.float32)
    M = X.shape[0]
    Y = np.empty((M, N), dtype=np.float32)
    ref().zr_mul_mat(qtype, _p(np.ascontiguousarray(raw_w)), N, K, _p(X), M, _p(Y), n_threads)
    return Y


# --- the reference's block executor (src/xdna-exec.cpp, xdna_exec_piece with no
# NPU: its host path, so run_rows and the rope table are the reference's own) -------

def _ref_ok(rc: int, what: str) -> None:
    if rc:
        raise RuntimeError(f"the reference's executor failed the {what} piece")


def ref_rms_norm(x: np.ndarray, d: int, eps: float, n_threads: int = 4) -> np.ndarray:
    x = _f32(x)
    y = np.empty_like(x)
    _ref_ok(ref().zr_rms_norm(_p(x), x.size // d, d, eps, _p(y), n_threads), "RMS_NORM")
    return y


def ref_mul_row(x: np.ndarray, w: np.ndarray, n_threads: int = 4) -> np.ndarray:
    x, w = _f32(x), _f32(w)
    y = np.empty_like(x)
    _ref_ok(ref().zr_mul_row(_p(x), _p(w), x.size // w.size, w.size, _p(y), n_threads), "MUL")
    return y


def ref_add(x: np.ndarray, b: np.ndarray, n_threads: int = 4) -> np.ndarray:
    x, b = _f32(x), _f32(b)
    y = np.empty_like(x)
    bias = int(b.size != x.size)
    d = b.size if bias else x.shape[-1]
    _ref_ok(ref().zr_add(_p(x), _p(b), bias, x.size // d, d, _p(y), n_threads), "ADD")
    return y


def ref_scale(x: np.ndarray, s: float, bias: float, n_threads: int = 4) -> np.ndarray:
    x = _f32(x)
    y = np.empty_like(x)
    _ref_ok(ref().zr_scale(_p(x), x.shape[0], x.size // x.shape[0], s, bias, _p(y), n_threads), "SCALE")
    return y


def ref_glu(kind: int, g: np.ndarray, u: np.ndarray | None = None, swapped: bool = False,
            n_threads: int = 4) -> np.ndarray:
    g = _f32(g)
    rows = g.shape[0]
    f = g.shape[1] if u is not None else g.shape[1] // 2
    y = np.empty((rows, f), np.float32)
    up = _p(_f32(u)) if u is not None else None
    _ref_ok(ref().zr_glu(kind, int(swapped), _p(g), up, rows, f, _p(y), n_threads), "GLU")
    return y


def ref_rope(x: np.ndarray, pos: np.ndarray, n_dims: int, mode: int, n_ctx_orig: int, par,
             ff: np.ndarray | None = None, n_threads: int = 4) -> np.ndarray:
    """x [T][heads][d]; par: freq_base, freq_scale, ext_factor, attn_factor, beta_fast, beta_slow."""
    x = _f32(x)
    T, H, d = x.shape
    pos = np.ascontiguousarray(pos, dtype=np.int32)
    par = _f32(par)
    y = np.empty_like(x)
    ffp = _p(_f32(ff)) if ff is not None else None
    _ref_ok(ref().zr_rope(_p(x), T, H, d, _p(pos), n_dims, mode, n_ctx_orig, _p(par), ffp, _p(y), n_threads),
            "ROPE")
    return y


def ref_norm_mul(x: np.ndarray, eps: float, w: np.ndarray, n_threads: int = 4) -> np.ndarray:
    x, w = _f32(x), _f32(w)
    y = np.empty_like(x)
    _ref_ok(ref().zr_norm_mul(_p(x), x.size // w.size, w.size, eps, _p(w), _p(y), n_threads), "RMS_NORM + MUL")
    return y


def ref_norm_mul_rope(x: np.ndarray, eps: float, w: np.ndarray, pos: np.ndarray, n_dims: int, mode: int,
                      n_ctx_orig: int, par, ff: np.ndarray | None = None, n_threads: int = 4) -> np.ndarray:
    x, w = _f32(x), _f32(w)
    T, H, d = x.shape
    pos = np.ascontiguousarray(pos, dtype=np.int32)
    par = _f32(par)
    y = np.empty_like(x)
    ffp = _p(_f32(ff)) if ff is not None else None
    _ref_ok(ref().zr_norm_mul_rope(_p(x), T, H, d, eps, _p(w), _p(pos), n_dims, mode, n_ctx_orig, _p(par), ffp,
                                   _p(y), n_threads), "RMS_NORM + MUL + ROPE")
    return y


# --- seeded synthetic inputs (the shapes and distributions of the configs) ---------

def make_data(n: int, seed: int) -> np.ndarray:
    """Values spanning many exponents per block, with zeros, ties and maxima
    that round up to +128 (the kinds of tests/test-bfp16-pack.cpp:77-91,
    drawn from numpy's generator rather than std::mt19937)."""
    rng = np.random.default_rng(seed)
    kind = rng.integers(0, 10, n)
    ex = rng.integers(-24, 13, n).astype(np.int32)
    x = np.ldexp(rng.standard_normal(n).astype(np.float32), ex).astype(np.float32)
    x = np.where(kind == 0, np.float32(0), x)
    x = np.where(kind == 1, np.ldexp(np.float32(127.75), ex).astype(np.float32), x)
    tie = (0.5 + rng.integers(0, 64, n)).astype(np.float32)
    x = np.where(kind == 2, np.ldexp(tie, ex).astype(np.float32), x)
    return x.astype(np.float32)


def activations(M: int, K: int, seed: int, outliers: bool = False) -> np.ndarray:
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((M, K), dtype=np.float32)
    if outliers:  # 1% of entries x50 (a Bernoulli mask from its own seed)
        mask = np.random.default_rng(seed + 7919).random((M, K)) < 0.01
        x = np.where(mask, x * np.float32(50), x).astype(np.float32)
    return x


def weights_f32(N: int, K: int, seed: int, std: float = 0.02) -> np.ndarray:
    return (np.random.default_rng(seed).standard_normal((N, K), dtype=np.float32) * np.float32(std)).astype(np.float32)


def nmax_err(got: np.ndarray, want: np.ndarray) -> float:
    """max |got - want| / max |want|: the parity metric of the GEMM."""
    w = np.asarray(want, dtype=np.float64)
    return float(np.max(np.abs(np.asarray(got, dtype=np.float64) - w)) / max(np.max(np.abs(w)), 1e-30))


# --- the block executor's small ops (src/xdna-exec.cpp:253-346) ---------------------

def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def rms_norm(x: np.ndarray, d: int, eps: float) -> np.ndarray:
    x = _f32(x)
    y = np.empty_like(x)
    orc().zo_rms_norm(_p(x), _i64(x.size // d), _i64(d), ctypes.c_float(eps), _p(y))
    return y


def mul_row(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    x, w = _f32(x), _f32(w)
    y = np.empty_like(x)
    orc().zo_mul_row(_p(x), _p(w), _i64(x.size // w.size), _i64(w.size), _p(y))
    return y


def add(x: np.ndarray, b: np.ndarray) -> np.ndarray:
    x, b = _f32(x), _f32(b)
    y = np.empty_like(x)
    d = b.size if b.size != x.size else x.shape[-1]
    orc().zo_add(_p(x), _p(b), ctypes.c_int(int(b.size != x.size)), _i64(x.size // d), _i64(d), _p(y))
    return y


def scale(x: np.ndarray, s: float, bias: float) -> np.ndarray:
    x = _f32(x)
    y = np.empty_like(x)
    orc().zo_scale(_p(x), _i64(x.size), ctypes.c_float(s), ctypes.c_float(bias), _p(y))
    return y


def glu(kind: int, g: np.ndarray, u: np.ndarray | None = None, swapped: bool = False) -> np.ndarray:
    """split: g, u [rows][f]; one tensor: g [rows][2f] holding gate then up (or up then gate when swapped)."""
    g = _f32(g)
    if u is not None:
        u = _f32(u)
        rows, f = g.shape
        gp, up, gs, us = g, u, f, f
        y = np.empty((rows, f), np.float32)
        orc().zo_glu(ctypes.c_int(kind), _p(gp), _i64(gs), _p(up), _i64(us), _i64(rows), _i64(f), _p(y))
        return y
    rows, f2 = g.shape
    f = f2 // 2
    y = np.empty((rows, f), np.float32)
    gate = g[:, f:] if swapped else g[:, :f]
    upv = g[:, :f] if swapped else g[:, f:]
    base = g.ctypes.data
    gp = ctypes.c_void_p(base + (f * 4 if swapped else 0))
    upp = ctypes.c_void_p(base + (0 if swapped else f * 4))
    orc().zo_glu(ctypes.c_int(kind), gp, _i64(f2), upp, _i64(f2), _i64(rows), _i64(f), _p(y))
    del gate, upv
    return y


def rope_table(pos: np.ndarray, n_dims: int, n_ctx_orig: int, par, ff: np.ndarray | None = None) -> np.ndarray:
    pos = np.ascontiguousarray(pos, dtype=np.int32)
    par = _f32(par)
    t = np.empty((pos.size, n_dims), np.float32)
    ffp = _p(_f32(ff)) if ff is not None else None
    orc().zo_rope_table(_p(pos), _i64(pos.size), ctypes.c_int(n_dims), ctypes.c_int(n_ctx_orig), _p(par), ffp, _p(t))
    return t


def rope(x: np.ndarray, n_dims: int, mode: int, table: np.ndarray) -> np.ndarray:
    """x [T][heads][d]"""
    x = _f32(x)
    T, H, d = x.shape
    y = np.empty_like(x)
    orc().zo_rope(_p(x), _i64(T), _i64(H), _i64(d), ctypes.c_int(n_dims), ctypes.c_int(mode), _p(_f32(table)), _p(y))
    return y


def nrmse(got: np.ndarray, want: np.ndarray) -> float:
    g = np.asarray(got, np.float64)
    w = np.asarray(want, np.float64)
    return float(np.sqrt(np.sum((g - w) ** 2) / max(np.sum(w ** 2), 1e-300)))
