"""The block executor's small-op cases, shared by the fixture script
(make_golden.py, which runs them through the reference's own executor) and
the tests that hold the oracle and the GPU kernels to those fixtures.

The 21 cases are the reference's tests/test-host-ops.cpp:91-153: rows of
D=256 for 8 tokens, rope over 4 heads of 64, inputs N(0, 1.5), positions
5000 + 300 i, frequency factors U(1, 4) (numpy's seeded generator here, not
std::mt19937). Two more are the fused forms this build runs: RMS_NORM + MUL
(the attention and FFN norms, Qwen3-4B's hidden 2560) and per-head RMS_NORM +
MUL + ROPE (Qwen3's q, 32 heads of 128, NeoX, base 1e6).
"""
from __future__ import annotations

import numpy as np

D, T, HD, H = 256, 8, 64, 4

# (name, spec); glu kinds in ggml's order: REGLU 0, GEGLU 1, SWIGLU 2, GEGLU_ERF 4, GEGLU_QUICK 5
CASES = [
    ("rms_norm", dict(kind="rms_norm", eps=1e-6)),
    ("mul by a scale row", dict(kind="mul_row")),
    ("add", dict(kind="add", bias=False)),
    ("add a bias row", dict(kind="add", bias=True)),
    ("scale and bias", dict(kind="scale", s=0.37, b=0.25)),
    ("swiglu, split", dict(kind="glu", glu=2, split=True, swapped=False)),
    ("geglu, split", dict(kind="glu", glu=1, split=True, swapped=False)),
    ("geglu_erf, split", dict(kind="glu", glu=4, split=True, swapped=False)),
    ("geglu_quick, split", dict(kind="glu", glu=5, split=True, swapped=False)),
    ("reglu, split", dict(kind="glu", glu=0, split=True, swapped=False)),
    ("swiglu, one tensor", dict(kind="glu", glu=2, split=False, swapped=False)),
    ("swiglu, one tensor, swapped", dict(kind="glu", glu=2, split=False, swapped=True)),
    ("geglu, one tensor", dict(kind="glu", glu=1, split=False, swapped=False)),
    ("geglu_erf, one tensor", dict(kind="glu", glu=4, split=False, swapped=False)),
    ("rope, normal", dict(kind="rope", n_dims=HD, mode=0, n_ctx_orig=0, freq_scale=1.0, ext=0.0, factors=False)),
    ("rope, neox", dict(kind="rope", n_dims=HD, mode=2, n_ctx_orig=0, freq_scale=1.0, ext=0.0, factors=False)),
    ("rope, normal, half the head", dict(kind="rope", n_dims=HD // 2, mode=0, n_ctx_orig=0, freq_scale=1.0, ext=0.0,
                                         factors=False)),
    ("rope, neox, three quarters", dict(kind="rope", n_dims=HD * 3 // 4, mode=2, n_ctx_orig=0, freq_scale=1.0,
                                        ext=0.0, factors=False)),
    ("rope, neox, yarn", dict(kind="rope", n_dims=HD, mode=2, n_ctx_orig=4096, freq_scale=0.25, ext=1.0,
                              factors=False)),
    ("rope, neox, frequency factors", dict(kind="rope", n_dims=HD, mode=2, n_ctx_orig=4096, freq_scale=1.0, ext=0.0,
                                           factors=True)),
    ("rope, normal, yarn and factors", dict(kind="rope", n_dims=HD, mode=0, n_ctx_orig=4096, freq_scale=0.25,
                                            ext=1.0, factors=True)),
    ("rms_norm + mul, qwen3 hidden", dict(kind="norm_mul", eps=1e-6, rows=16, d=2560)),
    ("rms_norm + mul + rope, qwen3 q heads", dict(kind="norm_mul_rope", eps=1e-6, tokens=8, heads=32, hd=128,
                                                  mode=2, base=1e6)),
]


def normal(shape, seed: int) -> np.ndarray:
    return (np.random.default_rng(seed).standard_normal(shape) * 1.5).astype(np.float32)


def rope_par(spec: dict, base: float = 10000.0) -> np.ndarray:
    """freq_base, freq_scale, ext_factor, attn_factor, beta_fast, beta_slow (test-host-ops.cpp:84-85)."""
    return np.array([base, spec.get("freq_scale", 1.0), spec.get("ext", 0.0), 1.0, 32.0, 1.0], np.float32)


def inputs(i: int, spec: dict) -> dict:
    """Case i's inputs, seeded by its index."""
    s = 1000 * (i + 1)
    k = spec["kind"]
    if k == "rms_norm" or k == "scale":
        return {"x": normal((T, D), s)}
    if k == "mul_row":
        return {"x": normal((T, D), s), "w": normal((D,), s + 1)}
    if k == "add":
        return {"x": normal((T, D), s), "b": normal((D,) if spec["bias"] else (T, D), s + 1)}
    if k == "glu":
        if spec["split"]:
            return {"g": normal((T, D), s), "u": normal((T, D), s + 1)}
        return {"g": normal((T, 2 * D), s)}
    if k == "rope":
        d = {"x": normal((T, H, HD), s), "pos": (5000 + 300 * np.arange(T)).astype(np.int32)}
        if spec["factors"]:
            d["ff"] = np.random.default_rng(s + 2).uniform(1.0, 4.0, spec["n_dims"] // 2).astype(np.float32)
        return d
    if k == "norm_mul":
        return {"x": normal((spec["rows"], spec["d"]), s), "w": normal((spec["d"],), s + 1)}
    if k == "norm_mul_rope":
        Tn, Hn, d = spec["tokens"], spec["heads"], spec["hd"]
        return {"x": normal((Tn, Hn, d), s), "w": normal((d,), s + 1),
                "pos": (4096 + np.arange(Tn)).astype(np.int32)}
    raise ValueError(k)


def run(i: int, spec: dict, ops, inp: dict | None = None) -> np.ndarray:
    """Case i through a set of op functions with the oracle's signatures
    (the reference's executor: oracle.ref_*; the restatement: oracle.*)."""
    inp = inp or inputs(i, spec)
    k = spec["kind"]
    if k == "rms_norm":
        return ops["rms_norm"](inp["x"], D, spec["eps"])
    if k == "mul_row":
        return ops["mul_row"](inp["x"], inp["w"])
    if k == "add":
        return ops["add"](inp["x"], inp["b"])
    if k == "scale":
        return ops["scale"](inp["x"], spec["s"], spec["b"])
    if k == "glu":
        if spec["split"]:
            return ops["glu"](spec["glu"], inp["g"], inp["u"])
        return ops["glu"](spec["glu"], inp["g"], None, spec["swapped"])
    if k == "rope":
        return ops["rope"](inp["x"], inp["pos"], spec["n_dims"], spec["mode"], spec["n_ctx_orig"], rope_par(spec),
                           inp.get("ff"))
    if k == "norm_mul":
        return ops["norm_mul"](inp["x"], spec["eps"], inp["w"])
    if k == "norm_mul_rope":
        par = rope_par({}, spec["base"])
        return ops["norm_mul_rope"](inp["x"], spec["eps"], inp["w"], inp["pos"], spec["hd"], spec["mode"], 0, par)
    raise ValueError(k)


def reference_ops(O) -> dict:
    return {"rms_norm": O.ref_rms_norm, "mul_row": O.ref_mul_row, "add": O.ref_add, "scale": O.ref_scale,
            "glu": lambda kind, g, u=None, swapped=False: O.ref_glu(kind, g, u, swapped),
            "rope": O.ref_rope, "norm_mul": O.ref_norm_mul, "norm_mul_rope": O.ref_norm_mul_rope}


def oracle_ops(O) -> dict:
    """The oracle's restatement composed into the same cases."""
    def rope(x, pos, n_dims, mode, n_ctx_orig, par, ff=None):
        return O.rope(x, n_dims, mode, O.rope_table(pos, n_dims, n_ctx_orig, par, ff))

    def norm_mul(x, eps, w):
        return O.mul_row(O.rms_norm(x, w.size, eps), w)

    def norm_mul_rope(x, eps, w, pos, n_dims, mode, n_ctx_orig, par, ff=None):
        y = O.mul_row(O.rms_norm(x, w.size, eps), w).reshape(x.shape)
        return rope(y, pos, n_dims, mode, n_ctx_orig, par, ff)

    return {"rms_norm": O.rms_norm, "mul_row": O.mul_row, "add": O.add, "scale": O.scale,
            "glu": lambda kind, g, u=None, swapped=False: O.glu(kind, g, u, swapped),
            "rope": rope, "norm_mul": norm_mul, "norm_mul_rope": norm_mul_rope}
