"""Drives libggml-zest.so through its ggml vtables, with the stand-in
ggml-base (libfake_ggml.so) underneath. TEST INFRASTRUCTURE ONLY.

The ctypes structures mirror ggml_abi.h: ggml_tensor, the reg / device /
backend interfaces in the slot order of the reference's initialisers.
"""
from __future__ import annotations

import ctypes
import struct
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
FAKE = HERE / "libfake_ggml.so"
PLUGIN = ROOT / "ggml-xdna_b200" / "libggml-zest.so"

_vp, _i64, _int = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int

F32, F16, Q4_0, Q8_0, Q4_K, Q6_K, IQ3_S, I32 = 0, 1, 2, 8, 12, 14, 21, 26
USAGE_ANY, USAGE_WEIGHTS, USAGE_COMPUTE = 0, 1, 2
FLAG_INPUT, FLAG_OUTPUT = 1, 2
DEV_CPU, DEV_GPU, DEV_IGPU, DEV_ACCEL = 0, 1, 2, 3
STATUS_FAILED, STATUS_SUCCESS = -1, 0
BLCK = {F32: (1, 4), F16: (1, 2), Q4_0: (32, 18), Q8_0: (32, 34), Q4_K: (256, 144), Q6_K: (256, 210),
        IQ3_S: (256, 110), I32: (1, 4)}


class Tensor(ctypes.Structure):
    _fields_ = [("type", _int), ("buffer", _vp), ("ne", _i64 * 4), ("nb", ctypes.c_size_t * 4), ("op", _int),
                ("op_params", ctypes.c_int32 * 16), ("flags", ctypes.c_int32), ("src", _vp * 10), ("view_src", _vp),
                ("view_offs", ctypes.c_size_t), ("data", _vp), ("name", ctypes.c_char * 64), ("extra", _vp),
                ("padding", ctypes.c_char * 8)]


class RegI(ctypes.Structure):
    _fields_ = [("get_name", _vp), ("get_device_count", _vp), ("get_device", _vp), ("get_proc_address", _vp)]


class Reg(ctypes.Structure):
    _fields_ = [("api_version", _int), ("iface", RegI), ("context", _vp)]


class DeviceI(ctypes.Structure):
    _fields_ = [(n, _vp) for n in ("get_name", "get_description", "get_memory", "get_type", "get_props",
                                   "init_backend", "get_buffer_type", "get_host_buffer_type", "buffer_from_host_ptr",
                                   "supports_op", "supports_buft", "offload_op", "event_new", "event_free",
                                   "event_synchronize")]


class Device(ctypes.Structure):
    _fields_ = [("iface", DeviceI), ("reg", _vp), ("context", _vp)]


class BackendI(ctypes.Structure):
    _fields_ = [(n, _vp) for n in ("get_name", "free", "set_tensor_async", "get_tensor_async", "set_tensor_2d_async",
                                   "get_tensor_2d_async", "cpy_tensor_async", "synchronize", "graph_plan_create",
                                   "graph_plan_free", "graph_plan_update", "graph_plan_compute", "graph_compute",
                                   "event_record", "event_wait", "graph_optimize")]


class Backend(ctypes.Structure):
    _fields_ = [("guid", _vp), ("iface", BackendI), ("device", _vp), ("context", _vp)]


class Caps(ctypes.Structure):
    _fields_ = [(n, ctypes.c_bool) for n in ("async_", "host_buffer", "buffer_from_host_ptr", "events",
                                             "mmap_support")]


class Props(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("description", ctypes.c_char_p), ("memory_free", ctypes.c_size_t),
                ("memory_total", ctypes.c_size_t), ("type", _int), ("device_id", ctypes.c_char_p), ("caps", Caps)]


_KEEP: list = []


def fn(ptr, restype, *argtypes):
    return ctypes.CFUNCTYPE(restype, *argtypes)(ptr)


class Harness:
    """The fake ggml-base and the plugin, loaded into this process."""

    def __init__(self):
        self.fake = ctypes.CDLL(str(FAKE), mode=ctypes.RTLD_GLOBAL)
        self.fake.fake_buffer_new.restype = _vp
        self.fake.fake_buffer_new.argtypes = [_int, _int]
        self.fake.fake_graph_new.restype = _vp
        self.fake.fake_graph_new.argtypes = [_int, _vp]
        self.fake.fake_cuda_buft.restype = _vp
        self.fake.fake_cpu_buft.restype = _vp
        self.fake.fake_op_id.argtypes = [ctypes.c_char_p]
        # ggml's IQ3_S dequantiser needs its codebook, here the installed
        # gguf package's (the plugin reads it back through to_float)
        self.fake.fake_ggml_set_iq3s_grid.argtypes = [_vp]
        try:
            import numpy as np
            from gguf.quants import IQ3_S as _IQ3S
            _IQ3S.init_grid()
            g = np.asarray(_IQ3S.grid, dtype=np.float32).reshape(512, 4).astype(np.uint32)
            self.iq3s_grid = np.ascontiguousarray(g[:, 0] | (g[:, 1] << 8) | (g[:, 2] << 16) | (g[:, 3] << 24),
                                                  dtype=np.uint32)
            self.fake.fake_ggml_set_iq3s_grid(self.iq3s_grid.ctypes.data)
        except ImportError:
            self.iq3s_grid = None
        self.plugin = ctypes.CDLL(str(PLUGIN))
        self.plugin.ggml_backend_xdna_reg.restype = ctypes.POINTER(Reg)
        self.plugin.ggml_backend_init.restype = ctypes.POINTER(Reg)
        self.plugin.ggml_backend_score.restype = _int
        self.plugin.ggml_zest_policy_supports.argtypes = [ctypes.POINTER(Tensor)]
        self.plugin.ggml_zest_piece_fusions.argtypes = [_vp]
        self.plugin.ggml_zest_piece_plan.argtypes = [_vp, ctypes.POINTER(ctypes.c_int)]
        self.plugin.ggml_zest_budget_plan.argtypes = [ctypes.c_double, _vp, ctypes.c_int, ctypes.POINTER(ctypes.c_int)]
        self.plugin.ggml_zest_piece_groups.argtypes = [_vp, ctypes.POINTER(ctypes.c_int), ctypes.c_int]
        self.plugin.ggml_zest_model_notes.argtypes = [ctypes.c_char_p, ctypes.c_int]
        self.plugin.ggml_zest_iq3s_codebook.argtypes = [_vp]
        # ctypes objects the C side points at, kept for the whole process: the
        # plugin remembers who read each tensor by address (as the reference
        # does), and a freed tensor's address reused by a later test's tensor
        # would carry stale readers into it
        self.keep = _KEEP

    def piece_fusions(self, nodes: list[Tensor]) -> int:
        arr = (ctypes.POINTER(Tensor) * len(nodes))(*[ctypes.pointer(n) for n in nodes])
        self.keep.append(arr)
        return self.plugin.ggml_zest_piece_fusions(self.fake.fake_graph_new(len(nodes), ctypes.cast(arr, _vp)))

    def piece_plan(self, nodes: list[Tensor]) -> dict:
        """graph_compute's plan for a piece: its service calls and what it folds in."""
        arr = (ctypes.POINTER(Tensor) * len(nodes))(*[ctypes.pointer(n) for n in nodes])
        self.keep.append(arr)
        c = (ctypes.c_int * 6)()
        jobs = self.plugin.ggml_zest_piece_plan(self.fake.fake_graph_new(len(nodes), ctypes.cast(arr, _vp)), c)
        return dict(jobs=jobs, swiglu=c[0], groups=c[1], norm=c[2], add=c[3], handoff=c[4], rope=c[5])

    def budget_plan(self, limit_gb: float, weights: list[Tensor]) -> list[int]:
        """The weight-copy budget's answers for these weights, asked in order."""
        arr = (ctypes.POINTER(Tensor) * len(weights))(*[ctypes.pointer(w) for w in weights])
        self.keep.append(arr)
        taken = (ctypes.c_int * len(weights))()
        self.plugin.ggml_zest_budget_plan(limit_gb, ctypes.cast(arr, _vp), len(weights), taken)
        return list(taken)

    def piece_groups(self, nodes: list[Tensor]) -> list[int]:
        arr = (ctypes.POINTER(Tensor) * len(nodes))(*[ctypes.pointer(n) for n in nodes])
        self.keep.append(arr)
        sizes = (ctypes.c_int * 16)()
        n = self.plugin.ggml_zest_piece_groups(self.fake.fake_graph_new(len(nodes), ctypes.cast(arr, _vp)), sizes, 16)
        return list(sizes[:n])

    def graph(self, nodes: list[Tensor]):
        arr = (ctypes.POINTER(Tensor) * len(nodes))(*[ctypes.pointer(n) for n in nodes])
        self.keep.append(arr)
        return self.fake.fake_graph_new(len(nodes), ctypes.cast(arr, _vp))

    def iq3s_codebook(self):
        """The IQ3_S codebook the plugin read back through ggml's to_float
        (uint32 x 512), or None when it has none."""
        import numpy as np
        out = np.zeros(512, dtype=np.uint32)
        return out if self.plugin.ggml_zest_iq3s_codebook(out.ctypes.data) else None

    def model_notes(self) -> str:
        """What graph_compute would say about the model as the first prompt runs."""
        buf = ctypes.create_string_buffer(2048)
        self.plugin.ggml_zest_model_notes(buf, len(buf))
        return buf.value.decode()

    # --- registry / device / backend ------------------------------------------
    def reg(self):
        return self.plugin.ggml_backend_xdna_reg().contents

    def reg_name(self) -> str:
        r = self.plugin.ggml_backend_xdna_reg()
        return fn(r.contents.iface.get_name, ctypes.c_char_p, _vp)(ctypes.cast(r, _vp)).decode()

    def device_count(self) -> int:
        r = self.plugin.ggml_backend_xdna_reg()
        return fn(r.contents.iface.get_device_count, ctypes.c_size_t, _vp)(ctypes.cast(r, _vp))

    def device(self):
        r = self.plugin.ggml_backend_xdna_reg()
        p = fn(r.contents.iface.get_device, _vp, _vp, ctypes.c_size_t)(ctypes.cast(r, _vp), 0)
        return p, ctypes.cast(p, ctypes.POINTER(Device)).contents

    def dev_call(self, name, restype, *args, argtypes=()):
        p, d = self.device()
        return fn(getattr(d.iface, name), restype, _vp, *argtypes)(p, *args)

    def supports_op(self, t: Tensor) -> bool:
        return bool(self.dev_call("supports_op", ctypes.c_bool, ctypes.byref(t), argtypes=(ctypes.POINTER(Tensor),)))

    def policy(self, t: Tensor) -> bool:
        return bool(self.plugin.ggml_zest_policy_supports(ctypes.byref(t)))

    def init_backend(self):
        p = self.dev_call("init_backend", _vp, None, argtypes=(ctypes.c_char_p,))
        return p, (ctypes.cast(p, ctypes.POINTER(Backend)).contents if p else None)

    def graph_compute(self, backend_ptr, nodes: list[Tensor]) -> int:
        arr = (ctypes.POINTER(Tensor) * len(nodes))(*[ctypes.pointer(n) for n in nodes])
        self.keep.append(arr)
        g = self.fake.fake_graph_new(len(nodes), ctypes.cast(arr, _vp))
        b = ctypes.cast(backend_ptr, ctypes.POINTER(Backend)).contents
        return fn(b.iface.graph_compute, _int, _vp, _vp)(backend_ptr, g)

    def graph_optimize(self, backend_ptr, nodes: list[Tensor]) -> None:
        arr = (ctypes.POINTER(Tensor) * len(nodes))(*[ctypes.pointer(n) for n in nodes])
        self.keep.append(arr)
        g = self.fake.fake_graph_new(len(nodes), ctypes.cast(arr, _vp))
        b = ctypes.cast(backend_ptr, ctypes.POINTER(Backend)).contents
        fn(b.iface.graph_optimize, None, _vp, _vp, _vp)(backend_ptr, g, None)

    def backend_free(self, backend_ptr) -> None:
        b = ctypes.cast(backend_ptr, ctypes.POINTER(Backend)).contents
        fn(b.iface.free, None, _vp)(backend_ptr)

    # --- tensors ---------------------------------------------------------------
    def buffer(self, usage=USAGE_COMPUTE, host=False):
        return self.fake.fake_buffer_new(usage, int(host))

    def op(self, name: str) -> int:
        return self.fake.fake_op_id(name.encode())

    def tensor(self, type_: int, ne, name="t", buffer=None, data=None, op="NONE", src=(), view_src=None,
               flags=0, params=None) -> Tensor:
        """params: op_params as a list of ints and floats (floats stored as their bits)."""
        t = Tensor()
        for i, v in enumerate(params or []):
            if isinstance(v, float):
                t.op_params[i] = struct.unpack("<i", struct.pack("<f", v))[0]
            elif v is not None:
                t.op_params[i] = int(v)
        t.type = type_
        t.buffer = buffer
        ne = list(ne) + [1] * (4 - len(ne))
        blck, size = BLCK[type_]
        t.ne[:] = ne
        t.nb[0] = size
        t.nb[1] = size * (ne[0] // blck)
        t.nb[2] = t.nb[1] * ne[1]
        t.nb[3] = t.nb[2] * ne[2]
        t.op = self.op(op)
        for i, s in enumerate(src):
            t.src[i] = ctypes.cast(ctypes.pointer(s), _vp)
        if view_src is not None:
            t.view_src = ctypes.cast(ctypes.pointer(view_src), _vp)
        t.data = data
        t.name = name.encode()[:63]
        t.flags = flags
        self.keep.append(t)
        return t

    def mul_mat(self, w: Tensor, x: Tensor, name="mm", buffer=None, data=None) -> Tensor:
        # ggml_mul_mat: dst ne = [w.ne1, x.ne1, x.ne2, x.ne3], f32
        return self.tensor(F32, [w.ne[1], x.ne[1], x.ne[2], x.ne[3]], name=name, buffer=buffer, data=data,
                           op="MUL_MAT", src=(w, x))

    # the small ops, shaped as ggml builds them
    def like(self, a: Tensor, op: str, src, name="op", params=None, buffer=None, data=None, ne=None) -> Tensor:
        return self.tensor(F32, list(ne or a.ne), name=name, buffer=buffer, data=data, op=op, src=src,
                           params=params)

    def rms_norm(self, a, eps=1e-6, **kw):
        return self.like(a, "RMS_NORM", (a,), params=[eps], **kw)

    def mul(self, a, w, **kw):
        return self.like(a, "MUL", (a, w), **kw)

    def add(self, a, b, **kw):
        return self.like(a, "ADD", (a, b), **kw)

    def scale(self, a, s, bias=0.0, **kw):
        return self.like(a, "SCALE", (a,), params=[float(s), float(bias)], **kw)

    def glu(self, a, b=None, kind=2, swapped=0, **kw):
        ne = list(a.ne) if b is not None else [a.ne[0] // 2, a.ne[1], a.ne[2], a.ne[3]]
        return self.like(a, "GLU", (a, b) if b is not None else (a,), params=[kind, swapped], ne=ne, **kw)

    def rope(self, a, pos, n_dims, mode, n_ctx_orig=0, freq_base=10000.0, freq_scale=1.0, ext_factor=0.0,
             attn_factor=1.0, beta_fast=32.0, beta_slow=1.0, ff=None, **kw):
        params = [0, n_dims, mode, 0, n_ctx_orig, float(freq_base), float(freq_scale), float(ext_factor),
                  float(attn_factor), float(beta_fast), float(beta_slow)]
        return self.like(a, "ROPE", (a, pos, ff) if ff is not None else (a, pos), params=params, **kw)
