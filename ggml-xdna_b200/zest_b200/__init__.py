"""ctypes binding of libzest_b200.so (include/zest_b200.h) for tests and bench.

Torch is used only for device memory and streams: every call passes plain
device pointers and the current CUDA stream through the C ABI. There is no
CPU fallback: if the library or a GPU is missing, the calls raise.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

import numpy as np

PKG_DIR = Path(__file__).resolve().parent.parent
LIB_PATH = PKG_DIR / "libzest_b200.so"
BACKEND_PATH = PKG_DIR / "libggml-zest.so"

TYPE_F32, TYPE_F16, TYPE_Q8_0, TYPE_Q4_K, TYPE_Q6_K, TYPE_IQ3_S = 0, 1, 8, 12, 14, 21
MODE_F32, MODE_BF16, MODE_SWIGLU = 0, 1, 2
ERR_NOT_FINITE, ERR_TIMEOUT = 1, 2
GLU_REGLU, GLU_GEGLU, GLU_SWIGLU, GLU_GEGLU_ERF, GLU_GEGLU_QUICK = 0, 1, 2, 4, 5
ROPE_NORMAL, ROPE_NEOX = 0, 2
BLOCK_BYTES = 9
SLOTS = 4  # ZEST_SLOTS: group calls in flight at once (zest_submit_group)
# (values per quant block, bytes per quant block)
QUANT = {TYPE_F32: (1, 4), TYPE_F16: (1, 2), TYPE_Q8_0: (32, 34), TYPE_Q4_K: (256, 144),
         TYPE_Q6_K: (256, 210), TYPE_IQ3_S: (256, 110)}

_i64, _vp, _int, _u32p = ctypes.c_int64, ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(ctypes.c_uint32)
_vpp, _i64p, _intp = ctypes.POINTER(_vp), ctypes.POINTER(_i64), ctypes.POINTER(_int)


class ZestError(RuntimeError):
    pass


class WKey(ctypes.Structure):
    """zest_wkey: a weight's identity (xdna_npu::wkey, src/xdna-npu.h:46-52)."""
    _fields_ = [("buffer", _vp), ("data", _vp), ("type", _int), ("K", _i64), ("N", _i64)]


class GemmSeg(ctypes.Structure):
    """zest_gemm_seg: one weight of zest_gemm_segs with its fused epilogue."""
    _fields_ = [("b", _vp), ("ldb", _i64), ("N", _i64), ("mode", _int), ("c", _vp), ("ldc", _i64),
                ("residual", _vp), ("ldr", _i64), ("a_next", _vp), ("lda_next", _i64), ("c_multicast", _vp),
                ("multicast_store", _int), ("c_peers", _vpp), ("n_peers", _int),
                ("c16", _vpp), ("n_c16", _int), ("ldc16", _i64)]


class GemmPlan(ctypes.Structure):
    """zest_gemm_plan: how K3 runs a launch."""
    _fields_ = [("pair_kernel", _int), ("tile_n", _int), ("tiles_m", _int), ("tiles_n", _int), ("k_blocks", _int),
                ("tiles", _i64), ("ctas", _int), ("raster", _int), ("stream_k", _int), ("whole_tiles", _int),
                ("split_tiles", _int), ("run_k_blocks", _i64)]


class MmOut(ctypes.Structure):
    """zest_mm_out: where one weight's result of zest_mul_mat_group_ex goes."""
    _fields_ = [("y", _vp), ("residual", _vp), ("a_next", _vp)]


class Times(ctypes.Structure):
    _fields_ = [("encode_ms", ctypes.c_double), ("gemm_ms", ctypes.c_double), ("copy_ms", ctypes.c_double),
                ("pack_ms", ctypes.c_double), ("calls", _int)]


_lib = None


def lib() -> ctypes.CDLL:
    """The loaded library; raises if it was never built."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise ZestError(f"{LIB_PATH} is missing: run __graft_entry__.build() (make -C ggml-xdna_b200)")
    L = ctypes.CDLL(str(LIB_PATH))
    sig = {
        "zest_version": (_int, []),
        "zest_last_error": (ctypes.c_char_p, []),
        "zest_load_iq3s_grid": (_int, [_u32p]),
        "zest_pack_activations": (_int, [_vp, _i64, _i64, _i64, _i64, _vp, _vp, _i64, _vp]),
        "zest_convert_weight": (_int, [_int, _vp, _i64, _i64, _i64, _i64, _i64, _vp, _vp, _vp]),
        "zest_convert_gate_up": (_int, [_int, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _vp, _vp, _vp]),
        "zest_gemm": (_int, [_vp, _i64, _vp, _i64, _i64, _i64, _i64, _int, _vp, _i64, _vp, _vp]),
        "zest_gemm_group": (_int, [_vp, _i64, _i64, _i64, _int, _vpp, _i64p, _i64p, _intp, _vpp, _i64p, _vp, _vp]),
        "zest_gemm_segs": (_int, [_vp, _i64, _i64, _i64, _int, ctypes.POINTER(GemmSeg), _vp, _vp]),
        "zest_plan_gemm": (_int, [_i64, _i64, _int, _i64p, _int, ctypes.POINTER(GemmPlan)]),
        "zest_pack_rms_norm": (_int, [_vp, _i64, _i64, _i64, ctypes.c_float, _vp, _vp, _i64, _i64, _vp, _i64, _vp]),
        "zest_norm_rope": (_int, [_vp, _i64, _i64, _i64, ctypes.c_float, _vp, _int, _int, _vp, _vp, _vp, _vp]),
        "zest_mul_mat_noalloc": (_int, [_vp, _i64, _i64, _i64, _vp, _i64, _i64, _int, _vp, _i64, _vp, _vp]),
        "zest_rms_norm": (_int, [_vp, _i64, _i64, ctypes.c_float, _vp, _vp]),
        "zest_mul_row": (_int, [_vp, _vp, _i64, _i64, _vp, _vp]),
        "zest_add": (_int, [_vp, _vp, _int, _i64, _i64, _vp, _vp]),
        "zest_scale": (_int, [_vp, _i64, ctypes.c_float, ctypes.c_float, _vp, _vp]),
        "zest_glu": (_int, [_int, _vp, _i64, _vp, _i64, _i64, _i64, _vp, _vp]),
        "zest_rope_table": (_int, [_vp, _i64, _int, _int, ctypes.POINTER(ctypes.c_float), _vp, _vp, _vp]),
        "zest_rope": (_int, [_vp, _i64, _i64, _i64, _int, _int, _vp, _vp, _vp]),
        "zest_usable": (_int, [_int, ctypes.c_char_p, ctypes.c_size_t]),
        "zest_open": (_vp, [_int]),
        "zest_close": (None, [_vp]),
        "zest_set_out16": (None, [_vp, _int]),
        "zest_has_weight": (_int, [_vp, ctypes.POINTER(WKey)]),
        "zest_add_weight": (_int, [_vp, ctypes.POINTER(WKey), _vp, _int]),
        "zest_add_fused": (_int, [_vp, ctypes.POINTER(WKey), _vp, _vp, _int]),
        "zest_add_weight_values": (_int, [_vp, ctypes.POINTER(WKey), _vp, _int]),
        "zest_out_width": (_i64, [_vp, ctypes.POINTER(WKey), _int]),
        "zest_weight_bfp16": (_vp, [_vp, ctypes.POINTER(WKey), _int]),
        "zest_weight_bf16": (_vp, [_vp, ctypes.POINTER(WKey), _int, ctypes.POINTER(_i64)]),
        "zest_set_load_async": (None, [_vp, _int]),
        "zest_wait_weights": (_int, [_vp]),
        "zest_mul_mat": (_int, [_vp, ctypes.POINTER(WKey), _int, _vp, _i64, _vp, _int]),
        "zest_mul_mat_group": (_int, [_vp, _int, ctypes.POINTER(WKey), _intp, _vp, _i64, _vpp, _int]),
        "zest_widen_bf16": (_int, [_vp, _i64, _vp, _vp]),
        "zest_submit_group": (_int, [_vp, _int, _int, ctypes.POINTER(WKey), _intp, _vp, _i64, _vpp, _int]),
        "zest_wait_group": (_int, [_vp, _int]),
        "zest_mul_mat_group_ex": (_int, [_vp, _int, ctypes.POINTER(WKey), _intp, _vp, ctypes.c_float, _vp, _vp, _vp,
                                         _i64, ctypes.POINTER(MmOut)]),
        "zest_stream": (_vp, [_vp]),
        "zest_take_times": (_int, [_vp, ctypes.POINTER(Times)]),
    }
    for name, (res, args) in sig.items():
        f = getattr(L, name)
        f.restype, f.argtypes = res, args
    _lib = L
    return L


def exported_symbols() -> list[str]:
    return [n for n in ("zest_version", "zest_last_error", "zest_load_iq3s_grid", "zest_pack_activations",
                        "zest_convert_weight", "zest_convert_gate_up", "zest_gemm", "zest_gemm_group",
                        "zest_gemm_segs", "zest_plan_gemm", "zest_mul_mat_noalloc",
                        "zest_rms_norm", "zest_mul_row", "zest_add", "zest_scale", "zest_glu", "zest_rope_table",
                        "zest_rope", "zest_pack_rms_norm", "zest_norm_rope", "zest_widen_bf16",
                        "zest_usable", "zest_open",
                        "zest_close", "zest_set_out16", "zest_has_weight", "zest_add_weight", "zest_add_fused",
                        "zest_add_weight_values",
                        "zest_out_width", "zest_weight_bfp16", "zest_weight_bf16", "zest_set_load_async",
                        "zest_wait_weights", "zest_mul_mat",
                        "zest_mul_mat_group", "zest_submit_group", "zest_wait_group", "zest_mul_mat_group_ex",
                        "zest_stream", "zest_take_times")]


def _check(rc: int, what: str) -> None:
    if rc != 0:
        raise ZestError(f"{what}: {lib().zest_last_error().decode()}")


def iq3s_grid() -> np.ndarray:
    """ggml's IQ3_S codebook (512 x 4 magnitudes) packed as uint32, read
    from the installed gguf package at run time."""
    from gguf.quants import IQ3_S
    IQ3_S.init_grid()
    g = np.asarray(IQ3_S.grid, dtype=np.float32).reshape(512, 4).astype(np.uint32)
    return (g[:, 0] | (g[:, 1] << 8) | (g[:, 2] << 16) | (g[:, 3] << 24)).astype(np.uint32)


def load_iq3s_grid() -> None:
    g = np.ascontiguousarray(iq3s_grid())
    _check(lib().zest_load_iq3s_grid(g.ctypes.data_as(_u32p)), "zest_load_iq3s_grid")


def row_bytes(qtype: int, k: int) -> int:
    qk, bb = QUANT[qtype]
    return k // qk * bb


def pad_to(x: int, m: int) -> int:
    return (x + m - 1) // m * m


# --- stream-level kernels on torch tensors -----------------------------------

def _stream():
    import torch
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _ptr(t):
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def pack_activations(x, m_pad: int | None = None, want_bytes: bool = True, want_bf16: bool = True):
    """K2: f32 [T][K] cuda tensor -> (bfp16 bytes uint8 [m_pad*K/8*9], bf16 int16 [m_pad][K])."""
    import torch
    T, K = x.shape
    m_pad = m_pad or pad_to(max(T, 1), 128)
    ab = torch.empty(m_pad * K // 8 * 9, dtype=torch.uint8, device=x.device) if want_bytes else None
    ah = torch.empty((m_pad, K), dtype=torch.int16, device=x.device) if want_bf16 else None
    _check(lib().zest_pack_activations(_ptr(x), T, K, x.stride(0), m_pad, _ptr(ab), _ptr(ah), K, _stream()),
           "zest_pack_activations")
    return ab, ah


def convert_weight(qtype: int, raw, N: int, K: int, row0: int = 0, n_rows: int | None = None,
                   n_pad: int | None = None, want_bytes: bool = True, want_bf16: bool = True):
    """K1: raw GGUF rows (uint8 cuda tensor of N rows) -> (bfp16 B operand, bf16 [n_pad][K])."""
    import torch
    n_rows = N - row0 if n_rows is None else n_rows
    n_pad = n_pad or pad_to(max(n_rows, 1), 512)
    bb = torch.empty(n_pad * K // 8 * 9, dtype=torch.uint8, device=raw.device) if want_bytes else None
    bh = torch.empty((n_pad, K), dtype=torch.int16, device=raw.device) if want_bf16 else None
    _check(lib().zest_convert_weight(qtype, _ptr(raw), N, row0, n_rows, K, n_pad, _ptr(bb), _ptr(bh), _stream()),
           "zest_convert_weight")
    return bb, bh


def convert_gate_up(qtype: int, gate, up, F: int, K: int, row0: int = 0, n_rows: int | None = None,
                    f_pad: int | None = None, want_bytes: bool = True, want_bf16: bool = True):
    import torch
    n_rows = F - row0 if n_rows is None else n_rows
    f_pad = f_pad or pad_to(max(n_rows, 1), 256)
    bb = torch.empty(2 * f_pad * K // 8 * 9, dtype=torch.uint8, device=gate.device) if want_bytes else None
    bh = torch.empty((2 * f_pad, K), dtype=torch.int16, device=gate.device) if want_bf16 else None
    _check(lib().zest_convert_gate_up(qtype, _ptr(gate), _ptr(up), F, row0, n_rows, K, f_pad, _ptr(bb), _ptr(bh),
                                      _stream()), "zest_convert_gate_up")
    return bb, bh


def gemm(a_bf16, b_bf16, M: int, N: int, mode: int = MODE_F32, out=None, err=None):
    """K3: out[M][N or N/2] f32 = A * B^T; err: int32 cuda word (cleared by the caller)."""
    import torch
    K = a_bf16.shape[1]
    n_out = N // 2 if mode == MODE_SWIGLU else N
    if out is None:
        out = torch.empty((M, n_out), dtype=torch.float32, device=a_bf16.device)
    own_err = err is None
    if own_err:
        err = torch.zeros(1, dtype=torch.int32, device=a_bf16.device)
    _check(lib().zest_gemm(_ptr(a_bf16), a_bf16.stride(0), _ptr(b_bf16), b_bf16.stride(0), M, N, K, mode, _ptr(out),
                           out.stride(0), _ptr(err), _stream()), "zest_gemm")
    if own_err:
        e = int(err.item())
        if e:
            raise ZestError(f"zest_gemm raised device error bits {e:#x}")
    return out


def gemm_group(a_bf16, bs, M: int, Ns, modes, outs=None, err=None):
    """K3 over up to 4 weights sharing A in one launch: outs[i] = A * bs[i]^T."""
    import torch
    n = len(bs)
    K = a_bf16.shape[1]
    if outs is None:
        outs = [torch.empty((M, N // 2 if m == MODE_SWIGLU else N), dtype=torch.float32, device=a_bf16.device)
                for N, m in zip(Ns, modes)]
    own_err = err is None
    if own_err:
        err = torch.zeros(1, dtype=torch.int32, device=a_bf16.device)
    arr = lambda t, vals: (t * n)(*vals)
    _check(lib().zest_gemm_group(_ptr(a_bf16), a_bf16.stride(0), M, K, n, arr(_vp, [b.data_ptr() for b in bs]),
                                 arr(_i64, [b.stride(0) for b in bs]), arr(_i64, Ns), arr(_int, modes),
                                 arr(_vp, [o.data_ptr() for o in outs]), arr(_i64, [o.stride(0) for o in outs]),
                                 _ptr(err), _stream()), "zest_gemm_group")
    if own_err:
        e = int(err.item())
        if e:
            raise ZestError(f"zest_gemm_group raised device error bits {e:#x}")
    return outs


def plan_gemm(M: int, K: int, Ns, sms: int = 0) -> dict:
    """How K3 would run A [M][K] against weights of Ns rows (no GPU needed)."""
    n = len(Ns)
    out = GemmPlan()
    _check(lib().zest_plan_gemm(M, K, n, (_i64 * n)(*Ns), sms, ctypes.byref(out)), "zest_plan_gemm")
    return {name: getattr(out, name) for name, _ in GemmPlan._fields_}


# --- the matmul service -------------------------------------------------------

class Npu:
    """zest_npu: per-GPU weight cache + y = x * W^T (xdna_npu, src/xdna-npu.h:40-136)."""

    def __init__(self, device: int = 0):
        self.h = lib().zest_open(device)
        if not self.h:
            raise ZestError(f"zest_open: {lib().zest_last_error().decode()}")

    def close(self):
        if self.h:
            lib().zest_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_out16(self, on: bool):
        lib().zest_set_out16(self.h, int(on))

    def set_load_async(self, on: bool):
        lib().zest_set_load_async(self.h, int(on))

    def wait_weights(self):
        _check(lib().zest_wait_weights(self.h), "zest_wait_weights")

    @staticmethod
    def key(data_addr: int, qtype: int, K: int, N: int, buffer: int = 0) -> WKey:
        return WKey(buffer, data_addr, qtype, K, N)

    def add_weight(self, key: WKey, raw_ptr: int, on_device: bool):
        _check(lib().zest_add_weight(self.h, ctypes.byref(key), ctypes.c_void_p(raw_ptr), int(on_device)),
               "zest_add_weight")

    def add_fused(self, key: WKey, gate_ptr: int, up_ptr: int, on_device: bool):
        _check(lib().zest_add_fused(self.h, ctypes.byref(key), ctypes.c_void_p(gate_ptr), ctypes.c_void_p(up_ptr),
                                    int(on_device)), "zest_add_fused")

    def has_weight(self, key: WKey) -> bool:
        return bool(lib().zest_has_weight(self.h, ctypes.byref(key)))

    def out_width(self, key: WKey, fused: bool = False) -> int:
        return int(lib().zest_out_width(self.h, ctypes.byref(key), int(fused)))

    def weight_bf16(self, key: WKey, fused: bool = False):
        n_pad = _i64(0)
        p = lib().zest_weight_bf16(self.h, ctypes.byref(key), int(fused), ctypes.byref(n_pad))
        return p, n_pad.value

    def mul_mat(self, key: WKey, x_ptr: int, T: int, y_ptr: int, on_device: bool, fused: bool = False):
        _check(lib().zest_mul_mat(self.h, ctypes.byref(key), int(fused), ctypes.c_void_p(x_ptr), T,
                                  ctypes.c_void_p(y_ptr), int(on_device)), "zest_mul_mat")

    def mul_mat_group(self, keys, x_ptr: int, T: int, y_ptrs, on_device: bool, fused=None):
        """One activation pack and one GEMM launch for weights sharing x."""
        n = len(keys)
        fused = fused or [False] * n
        _check(lib().zest_mul_mat_group(self.h, n, (WKey * n)(*keys), (_int * n)(*[int(f) for f in fused]),
                                        ctypes.c_void_p(x_ptr), T, (_vp * n)(*y_ptrs), int(on_device)),
               "zest_mul_mat_group")

    def submit_group(self, slot: int, keys, x_ptr: int, T: int, y_ptrs, on_device: bool, fused=None):
        """zest_mul_mat_group queued in `slot` (0 .. SLOTS-1); finish it with wait_group(slot).
        The arrays behind x_ptr and y_ptrs must outlive the wait."""
        n = len(keys)
        fused = fused or [False] * n
        _check(lib().zest_submit_group(self.h, slot, n, (WKey * n)(*keys), (_int * n)(*[int(f) for f in fused]),
                                       ctypes.c_void_p(x_ptr), T, (_vp * n)(*y_ptrs), int(on_device)),
               "zest_submit_group")

    def wait_group(self, slot: int):
        _check(lib().zest_wait_group(self.h, slot), "zest_wait_group")

    def mul_mat_group_ex(self, keys, outs, T: int, x_ptr: int = 0, a_ptr: int = 0, norm_eps: float = -1.0,
                         norm_w_ptr: int = 0, x_normed_ptr: int = 0, fused=None):
        """Device buffers; outs: [(y, residual, a_next)] pointers (0 for none)."""
        n = len(keys)
        fused = fused or [False] * n
        _check(lib().zest_mul_mat_group_ex(self.h, n, (WKey * n)(*keys), (_int * n)(*[int(f) for f in fused]),
                                           ctypes.c_void_p(x_ptr), ctypes.c_float(norm_eps),
                                           ctypes.c_void_p(norm_w_ptr), ctypes.c_void_p(x_normed_ptr),
                                           ctypes.c_void_p(a_ptr), T, (MmOut * n)(*[MmOut(*o) for o in outs])),
               "zest_mul_mat_group_ex")

    def stream(self) -> int:
        return int(lib().zest_stream(self.h) or 0)

    def take_times(self) -> Times:
        t = Times()
        _check(lib().zest_take_times(self.h, ctypes.byref(t)), "zest_take_times")
        return t


def usable(device: int = 0) -> tuple[bool, str]:
    buf = ctypes.create_string_buffer(512)
    rc = lib().zest_usable(device, buf, len(buf))
    return rc == 0, buf.value.decode()


def env_threads() -> int:
    return os.cpu_count() or 1
