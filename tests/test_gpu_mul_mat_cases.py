"""The reference's tests/test-mul-mat.cpp:140-157 restated: its twelve weight
types and shapes (K x N x batch), weights and activations drawn N(0, 1),
each product held against the fp64 truth built from the dequantised weight
bytes and the raw f32 activations (test-mul-mat.cpp:100-125), by the same
two measures (nrmse and cosine, test-mul-mat.cpp:42-57).

The reference passes a case when the NPU's nrmse is within twice the CPU
backend's plus 1e-6 and the cosine is above 0.9999
(test-mul-mat.cpp:200-204). ggml-cpu is not in this image; its error comes
from quantising the activations to the weight type's vec_dot_type before
the dot product (ggml's published CPU matmul: q8_0 blocks of 32 for Q4_0 and
Q8_0, q8_K blocks of 256 for the K-quants, f16 for f16 weights, f32 for f32
weights), so the CPU leg here restates that quantisation and takes the exact
product of what it keeps.

Every case runs through the plugin's graph_compute in a child process with
the batch and work gates lowered (GGML_XDNA_MIN_BATCH=1,
GGML_XDNA_MIN_MFLOP=0) and the weights in a weight buffer, so that all
twelve reach the GPU; the reference runs the seven "weights=false" cases on
its CPU path instead, and the last test checks that the plugin leaves them
alone the same way at its default gates. f32 and f16 weights cannot meet a
bar relative to an f32 or f16 CPU product on a bfp16 path (the reference
keeps them off the NPU for that reason); they are held to the bfp16 level,
nrmse <= 1e-2 with the same cosine bound."""
import json
import os
import subprocess
import sys
import textwrap

import numpy as np
import pytest

HERE = os.path.dirname(__file__)
sys.path.insert(0, os.path.join(HERE, "ggml_harness"))
from harness import F16, F32, Q4_0, Q4_K, Q6_K, Q8_0  # noqa: E402

pytestmark = pytest.mark.gpu

# (name, type, K, N, batch, weights) as test-mul-mat.cpp:140-157 lists them
CASES = [
    ("f32 256x128 x 64", F32, 256, 128, 64, False),
    ("f16 256x128 x 64", F16, 256, 128, 64, False),
    ("q8_0 512x256 x 64", Q8_0, 512, 256, 64, False),
    ("q4_0 512x256 x 64", Q4_0, 512, 256, 64, False),
    ("q4_K 512x256 x 64", Q4_K, 512, 256, 64, False),
    ("q4_K 2048x512 x 512", Q4_K, 2048, 512, 512, False),
    ("q6_K 512x256 x 64", Q6_K, 512, 256, 64, False),
    ("q4_0 2048x1024 x 512 w", Q4_0, 2048, 1024, 512, True),
    ("q4_K 2048x1024 x 600 w", Q4_K, 2048, 1024, 600, True),
    ("q4_0 1536x896 x 512 w", Q4_0, 1536, 896, 512, True),
    ("q8_0 1536x256 x 512 w", Q8_0, 1536, 256, 512, True),
    ("q4_K 1536x8960 x 520 w", Q4_K, 1536, 8960, 520, True),
]

CHILD = textwrap.dedent("""
    import json, sys
    sys.path[:0] = [{harness!r}, {tests!r}, {root!r}]
    import numpy as np, torch
    from harness import *
    from oracle import oracle as O
    from test_gpu_backend import dequant_q4_0, quant_q4_0

    def compare(got, truth):
        se = float(np.sum((got - truth) ** 2)); ss = float(np.sum(truth ** 2))
        cos = float(np.sum(got * truth) / max(np.sqrt(np.sum(got ** 2) * ss), 1e-300))
        return float(np.sqrt(se / max(ss, 1e-300))), cos

    def q8_blocks(x, blk, scale16):
        # ggml-cpu's activation quantisation for a dot product: blocks of blk
        # values on one scale amax/127, values rounded to it; q8_0 keeps the
        # scale as f16, q8_K as f32.
        b = x.reshape(-1, blk).astype(np.float32)
        d = np.abs(b).max(axis=1, keepdims=True) / np.float32(127)
        if scale16:
            d = d.astype(np.float16).astype(np.float32)
        inv = np.where(d > 0, 1 / np.where(d > 0, d, 1), 0).astype(np.float32)
        q = np.clip(np.rint(b * inv), -128, 127)
        return (q * d).reshape(x.shape)

    def cpu_leg(qt, x, deq):
        if qt == F32:
            return (x @ deq.T).astype(np.float64)
        if qt == F16:
            xa = x.astype(np.float16).astype(np.float64)
        elif qt in (Q4_0, Q8_0):
            xa = q8_blocks(x, 32, True).astype(np.float64)
        else:
            xa = q8_blocks(x, 256, False).astype(np.float64)
        return xa @ deq.astype(np.float64).T

    def weights_of(qt, vals):
        n, k = vals.shape
        if qt == F32:
            return vals.view(np.uint8).reshape(-1), vals
        if qt == F16:
            h16 = vals.astype(np.float16)
            return h16.view(np.uint8).reshape(-1), h16.astype(np.float32)
        if qt == Q4_0:
            raw = quant_q4_0(vals)
            return raw, dequant_q4_0(raw, n, k)
        raw = O.quantize(qt, vals)
        return raw, O.dequant(qt, raw, n, k)

    h = Harness()
    out = {{}}
    rng = np.random.default_rng(1234)
    for name, qt, K, N, M in {cases!r}:
        vals = rng.standard_normal((N, K)).astype(np.float32)
        x = rng.standard_normal((M, K)).astype(np.float32)
        raw, deq = weights_of(qt, vals)
        truth = x.astype(np.float64) @ deq.astype(np.float64).T
        wd = torch.from_numpy(np.ascontiguousarray(raw)).cuda()
        xd = torch.from_numpy(x).cuda()
        yd = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
        w = h.tensor(qt, [K, N], name="blk.0.ffn_up.weight", buffer=h.buffer(USAGE_WEIGHTS), data=wd.data_ptr())
        xt = h.tensor(F32, [K, M], buffer=h.buffer(USAGE_COMPUTE), data=xd.data_ptr())
        node = h.mul_mat(w, xt, buffer=h.buffer(USAGE_COMPUTE), data=yd.data_ptr())
        claimed = h.supports_op(node)
        b, _ = h.init_backend()
        torch.cuda.synchronize()
        st = h.graph_compute(b, [node])
        torch.cuda.synchronize()
        got = yd.cpu().numpy().astype(np.float64)
        h.backend_free(b)
        ex = compare(got, truth)
        ec = compare(cpu_leg(qt, x, deq), truth)
        out[name] = dict(claimed=claimed, status=st, ex=ex, ec=ec)
        print(f"{{name:24s}} gpu nrmse {{ex[0]:.2e}} cos {{ex[1]:.6f}}   cpu nrmse {{ec[0]:.2e}} cos {{ec[1]:.6f}}",
              file=sys.stderr)
    print(json.dumps(out))
""")


@pytest.fixture(scope="module")
def results():
    code = CHILD.format(harness=os.path.join(HERE, "ggml_harness"), tests=HERE, root=os.path.dirname(HERE),
                        cases=[c[:5] for c in CASES])
    env = dict(os.environ, GGML_XDNA_MIN_BATCH="1", GGML_XDNA_MIN_MFLOP="0")
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    print(r.stderr[-3000:])
    return json.loads(r.stdout.strip().splitlines()[-1])


@pytest.mark.parametrize("name,qt", [(c[0], c[1]) for c in CASES], ids=[c[0] for c in CASES])
def test_mul_mat_case_against_fp64_truth(results, name, qt):
    r = results[name]
    assert r["claimed"], "with the gates lowered every case is the plugin's"
    assert r["status"] == 0
    ex_nrmse, ex_cos = r["ex"]
    ec_nrmse, _ = r["ec"]
    bar = 1e-2 if qt in (F32, F16) else ec_nrmse * 2.0 + 1e-6
    assert ex_nrmse <= bar and ex_cos > 0.9999, (ex_nrmse, ex_cos, ec_nrmse)


def test_unweighted_cases_stay_off_at_default_gates():
    """test-mul-mat.cpp:143-149: the cases whose weights are not in a weight
    buffer, and whose batch is below the prompt gate, are not the backend's;
    the weight-buffer cases at batch 512-600 are below the default prompt
    gate (1024 rows) too and also stay with the host at default settings."""
    import torch
    from harness import F32 as _F32, Harness, USAGE_COMPUTE, USAGE_WEIGHTS
    h = Harness()
    for name, qt, K, N, M, weights in CASES:
        wd = torch.zeros(1, device="cuda")
        xt = h.tensor(_F32, [K, M], buffer=h.buffer(USAGE_COMPUTE), data=wd.data_ptr())
        w = h.tensor(qt, [K, N], buffer=h.buffer(USAGE_WEIGHTS if weights else USAGE_COMPUTE), data=wd.data_ptr())
        node = h.mul_mat(w, xt, buffer=h.buffer(USAGE_COMPUTE), data=wd.data_ptr())
        assert not h.supports_op(node), name
