"""Writes the golden fixtures under tests/golden/ from the REFERENCE's own code.

Run in a container that has the reference sources, after `make -C oracle ref`:

    python tests/golden/make_golden.py

    python tests/golden/make_golden.py host_ops    # only the small-op fixture

Every output byte / value here comes from oracle/_ref/libzest_ref.so, i.e.
the reference's src/npu/bfp16_pack.cpp, src/xdna-ref.cpp and
src/xdna-exec.cpp compiled unmodified, except the dequantised weights, which
come from gguf-py's numpy dequantisers (the independent cross-check of the
restated ggml to_float).
Inputs are seeded (numpy PCG64) and stored alongside, so the fixtures stand
on their own where neither the reference nor gguf is present.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle import oracle as O  # noqa: E402

OUT = Path(__file__).resolve().parent


def host_ops() -> None:
    """5. the block executor's small ops (run_rows, src/xdna-exec.cpp:253-346,
    and its rope table, :199-239), run by the reference's own executor with
    no NPU: the cases of tests/golden/host_ops.py, inputs stored beside."""
    import json

    sys.path.insert(0, str(OUT))
    import host_ops as HO

    arrays = {"cases": np.array(json.dumps(HO.CASES))}
    ops = HO.reference_ops(O)
    for i, (name, spec) in enumerate(HO.CASES):
        inp = HO.inputs(i, spec)
        for k, v in inp.items():
            arrays[f"{i}/{k}"] = v
        arrays[f"{i}/y"] = HO.run(i, spec, ops, inp)
    np.savez_compressed(OUT / "host_ops.npz", **arrays)


def main() -> None:
    import gguf
    from gguf import GGMLQuantizationType as GT

    if not O.has_ref():
        raise SystemExit("oracle/_ref/libzest_ref.so is missing: make -C oracle ref")
    if sys.argv[1:] == ["host_ops"]:
        host_ops()
        print("wrote host_ops.npz")
        return

    # 1. the codec: adversarial blocks and special values (bfp16_pack.cpp:85-144)
    x = O.make_data(8 * 4096, 20261201)
    specials = np.array([np.inf, 1, 2, 3, 4, 5, 6, 7,
                         -np.inf, 1e30, 0, 0, 0, 0, 0, 0,
                         np.nan, 1, 1, 1, 1, 1, 1, 1,
                         1e-45, 2e-45, -3e-40, 0, 0, 0, 0, 0,
                         -0.0, 0.0, -0.0, 0, 0, 0, 0, 0,
                         3e38, -3e38, 1, 2, 3, 4, 5, 6,
                         127.75 / 64, 1.0 / 64, -3.5 / 64, 0, 1, -127.5 / 64, 0.25 / 64, 100.5 / 64], np.float32)
    specials[-4] = 0.0
    specials[-8:] = np.array([127.75, 1.0, -3.5, 0.0, 64.0, -127.5, 0.25, 100.5], np.float32) / 64
    xs = np.concatenate([x, specials]).astype(np.float32)
    np.savez_compressed(OUT / "codec.npz", x=xs, bytes=O.ref_encode_blocks(xs))

    # 2. operand layouts at the reference's default tiling (m=128, k=64, n=64, 8 columns)
    xa = O.make_data(256 * 128, 1 + 256 + 128).reshape(256, 128)
    np.savez_compressed(OUT / "pack_a_256x128.npz", x=xa, bytes=O.ref_pack_a(xa))
    wb = O.make_data(512 * 128, 7 + 512 + 128).reshape(512, 128)
    np.savez_compressed(OUT / "pack_b_512x128.npz", w=wb, bytes=O.ref_pack_b(wb))
    # a fused gate/up weight (bfp16_interleave_gate_up), F=256 -> 512 rows
    g = O.make_data(256 * 64, 31).reshape(256, 64)
    u = O.make_data(256 * 64, 32).reshape(256, 64)
    inter = np.empty((512, 64), np.float32)
    O.ref().zr_interleave_gate_up(O._p(g), O._p(u), 256, 64, O._p(inter))
    np.savez_compressed(OUT / "gate_up_256x64.npz", gate=g, up=u, bytes=O.ref_pack_b(inter))

    # 3. dequantisers: gguf-py's numpy output on our synthetic encodings
    for name, qt, gt in (("q8_0", O.Q8_0, GT.Q8_0), ("q4_k", O.Q4_K, GT.Q4_K), ("q6_k", O.Q6_K, GT.Q6_K),
                         ("iq3_s", O.IQ3_S, GT.IQ3_S)):
        w = O.weights_f32(16, 512, 100 + qt)
        raw = O.quantize(qt, w)
        deq = gguf.quants.dequantize(raw.reshape(16, -1), gt).astype(np.float32)
        np.savez_compressed(OUT / f"dequant_{name}.npz", raw=raw, values=deq)

    # 4. the reference's CPU matmul (xdna_ref_mul_mat) on a Q8_0 weight,
    #    config 1's distributions at a small size
    N, K, M = 512, 256, 64
    w = O.weights_f32(N, K, 41)
    raw = O.quantize(O.Q8_0, w)
    X = O.activations(M, K, 42)
    Y = O.ref_mul_mat(O.Q8_0, raw, N, K, X, n_threads=4)
    # the same on the bfp16-decoded operands: the GEMM parity target
    Xd = O.decode_blocks(O.ref_encode_blocks(X)).reshape(M, K)
    Wd = O.decode_blocks(O.ref_encode_blocks(O.dequant(O.Q8_0, raw, N, K))).reshape(N, K)
    Yd = O.ref_mul_mat(O.F32, Wd, N, K, Xd, n_threads=4)
    np.savez_compressed(OUT / "mul_mat_q8_0.npz", raw=raw, x=X, y=Y, y_decoded=Yd, N=N, K=K, M=M)
    host_ops()
    print("wrote", sorted(p.name for p in OUT.glob("*.npz")))


if __name__ == "__main__":
    main()
