"""K1 -> K2 -> K3 at the configs' own shapes and weight types, against the
reference's CPU matmul.

Each case runs the GPU path from the raw GGUF bytes (K1 weight conversion,
K2 activation pack, K3 grouped launches as bench.py makes them) and checks
it against xdna_ref_mul_mat, the reference's src/xdna-ref.cpp compiled
unmodified into oracle/_ref, run on the same operands rounded to bfp16 by
the oracle (dequant, bfp16 encode, decode): the north star's bar,
max|C_gpu - C_ref| / max|C_ref| <= 1e-3, on fp32 outputs.

The CPU side checks the first and the last row of every 256-row block (the
pair kernel's tile height) and a few rows between, in every output column,
so every tile of every launch, the stream-K-split ones included, is checked
in part. The launch plans are asserted to take the routes the configs take
(stream-K on the long-K down projections).

Configs: C2 the Qwen3-4B layer, Q4_K, M=8192; C4 the
27B-class layer's IQ3_S gate (through the ggml plugin, as llama.cpp would
run it) and down (K=17408) at M=2048 and 8192; C5 the LFM-style Q8_0 FFN at
M=16384 with 1% of the activations x50.
"""
import os
import sys

import numpy as np
import pytest
import torch

import zest_b200 as Z
from oracle import oracle as O
from gpu_util import dev

pytestmark = pytest.mark.gpu

TOL = 1e-3
THREADS = os.cpu_count() or 8


def sample_rows(M: int, seed: int) -> np.ndarray:
    """First and last row of every 256-row block, plus 16 rows drawn at random."""
    edges = [r for b in range(0, M, 256) for r in (b, min(M, b + 256) - 1)]
    extra = np.random.default_rng(seed).integers(0, M, 16)
    return np.unique(np.r_[edges, extra]).astype(np.int64)


def decoded(values: np.ndarray) -> np.ndarray:
    """The values as the bfp16 operand holds them (oracle encode + decode)."""
    return O.decode_blocks(O.encode_blocks(np.ascontiguousarray(values, np.float32))).reshape(values.shape)


def random_iq3s(N: int, K: int, seed: int) -> np.ndarray:
    """Valid IQ3_S rows: every byte of qs, qh, signs and scales random (so all
    512 codebook entries and every sign and scale occur), d a small positive
    fp16. Parity is on the dequantised values both sides share, so any
    valid encoding serves."""
    rng = np.random.default_rng(seed)
    nb = N * K // 256
    blk = rng.integers(0, 256, size=(nb, 110), dtype=np.uint8)
    d = rng.uniform(2e-4, 8e-4, nb).astype(np.float16)
    blk[:, :2] = d.view(np.uint8).reshape(nb, 2)
    return blk.reshape(-1)


def quantized(qt: int, N: int, K: int, seed: int) -> np.ndarray:
    if qt == O.IQ3_S:
        return random_iq3s(N, K, seed)
    from concurrent.futures import ThreadPoolExecutor
    w = O.weights_f32(N, K, seed)
    step = max(1, N // THREADS)
    with ThreadPoolExecutor(THREADS) as ex:
        parts = list(ex.map(lambda r: O.quantize(qt, w[r:r + step]), range(0, N, step)))
    return np.concatenate(parts)


def ref_rows(qt: int, raw: np.ndarray, N: int, K: int, x_rows: np.ndarray) -> np.ndarray:
    """xdna_ref_mul_mat (oracle/_ref) on the bfp16-rounded operands."""
    wd = decoded(O.dequant(qt, raw, N, K))
    return O.ref_mul_mat(O.F32, wd.view(np.uint8), N, K, decoded(x_rows), n_threads=THREADS)


def run_groups(qt: int, M: int, groups, seed: int, outliers: bool = False):
    """groups: [(K, [(name, N), ...])], one pack and one grouped launch each,
    fp32 outputs. Returns {name: (rows checked, GPU rows, reference rows)}."""
    if qt == O.IQ3_S:
        Z.load_iq3s_grid()
    rows = sample_rows(M, seed)
    got = {}
    for gi, (K, members) in enumerate(groups):
        x = O.activations(M, K, seed + 17 * gi, outliers=outliers)
        _, ah = Z.pack_activations(dev(x))
        raws, bhs = [], []
        for name, N in members:
            raw = quantized(qt, N, K, seed + 1000 * gi + N)
            _, bh = Z.convert_weight(qt, dev(raw), N, K, want_bytes=False)
            raws.append(raw)
            bhs.append(bh)
        Ns = [N for _, N in members]
        outs = Z.gemm_group(ah, bhs, M, Ns, [Z.MODE_F32] * len(members))
        idx = torch.from_numpy(rows).cuda()
        for (name, N), raw, o in zip(members, raws, outs):
            g = o.index_select(0, idx).cpu().numpy()
            got[name] = (rows, g, ref_rows(qt, raw, N, K, x[rows]))
        del ah, bhs, outs
        torch.cuda.empty_cache()
    return got


def check(got: dict):
    worst = {name: O.nmax_err(g, w) for name, (_, g, w) in got.items()}
    for name, e in worst.items():
        assert e <= TOL, f"{name}: {e:.3g} > {TOL}"
    return worst


def test_c2_qwen3_4b_layer_q4k_m8192():
    M = 8192
    groups = [(2560, [("q", 4096), ("k", 1024), ("v", 1024)]), (4096, [("o", 2560)]),
              (2560, [("gate", 9728), ("up", 9728)]), (9728, [("down", 2560)])]
    assert Z.plan_gemm(M, 9728, [2560])["stream_k"] == 1, "C2 down runs stream-K"
    check(run_groups(O.Q4_K, M, groups, seed=21))


@pytest.mark.parametrize("M", [2048, 8192])
def test_c4_down_iq3s_k17408_stream_k(M):
    p = Z.plan_gemm(M, 17408, [5120])
    assert p["stream_k"] == 1 and p["split_tiles"] > 0, "C4 down runs stream-K"
    check(run_groups(O.IQ3_S, M, [(17408, [("down", 5120)])], seed=40 + M))


def test_c4_qkv_iq3s_m2048():
    check(run_groups(O.IQ3_S, 2048, [(5120, [("q", 6144), ("k", 1024), ("v", 1024)])], seed=43))


def test_c5_lfm_q8_0_m16384_outliers():
    M = 16384
    groups = [(2048, [("gate", 10752), ("up", 10752)]), (10752, [("down", 2048)])]
    check(run_groups(O.Q8_0, M, groups, seed=50, outliers=True))


def test_c4_iq3s_gate_through_the_plugin(monkeypatch):
    """An IQ3_S weight through the ggml plugin, as llama.cpp runs C4: the
    plugin reads ggml's IQ3_S codebook back through to_float, converts the
    raw GGUF rows on the GPU and runs the matmul in place. fp32 outputs
    (GGML_XDNA_OUT16=0) against xdna_ref at 1e-3; with the default bf16
    rounding, every value within one bf16 step of the rounded reference."""
    sys.path.insert(0, os.path.join(os.path.dirname(__file__), "ggml_harness"))
    from harness import F32, IQ3_S, STATUS_SUCCESS, USAGE_COMPUTE, USAGE_WEIGHTS, Harness

    h = Harness()
    assert h.iq3s_codebook() is not None
    K, N, T = 5120, 17408, 2048
    raw = random_iq3s(N, K, 44)
    x = O.activations(T, K, 45)
    rows = sample_rows(T, 46)
    want = ref_rows(O.IQ3_S, raw, N, K, x[rows])
    wd = torch.from_numpy(raw).cuda()
    xd = torch.from_numpy(x).cuda()
    for out16 in ("0", "1"):
        monkeypatch.setenv("GGML_XDNA_OUT16", out16)
        yd = torch.zeros((T, N), dtype=torch.float32, device="cuda")
        w = h.tensor(IQ3_S, [K, N], name="blk.0.ffn_gate.weight", buffer=h.buffer(USAGE_WEIGHTS),
                     data=wd.data_ptr())
        xt = h.tensor(F32, [K, T], buffer=h.buffer(USAGE_COMPUTE), data=xd.data_ptr())
        node = h.mul_mat(w, xt, buffer=h.buffer(USAGE_COMPUTE), data=yd.data_ptr())
        assert h.supports_op(node), "IQ3_S is claimed"
        b, _ = h.init_backend()
        assert b
        torch.cuda.synchronize()
        assert h.graph_compute(b, [w, xt, node]) == STATUS_SUCCESS
        torch.cuda.synchronize()
        got = yd.index_select(0, torch.from_numpy(rows).cuda()).cpu().numpy()
        h.backend_free(b)
        if out16 == "0":
            assert O.nmax_err(got, want) <= TOL
        else:
            assert np.array_equal(got, O.round_bf16(got))
            r = O.round_bf16(want).astype(np.float64)
            assert np.all(np.abs(got - r) <= np.abs(r) * 2.0 ** -7 + 1e-30)
