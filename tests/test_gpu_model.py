"""The whole-model prefill driver behind bench.py's qwen3-4b-model workload,
on a two-layer model of the same structure: the chunks run through the C ABI
(every claimed op on our kernels) against the same chunks run as torch ops
on the same bf16 weight copies (the path an unclaimed chunk takes). The
claimed path rounds activations to bfp16 (8 significant bits per value, a
shared exponent per 8) where torch rounds them to bf16, so the two agree to
about 1e-2, not bit for bit; a wiring mistake (a rope pairing, the gate/up
interleave, a stride) shows up as an O(1) difference."""
import numpy as np
import pytest
import torch

import bench
from oracle import oracle as O

pytestmark = pytest.mark.gpu

TINY = dict(bench.MODEL, layers=2, hidden=1024, heads=8, kv_heads=2, head_dim=128, ffn=2048, vocab=2000,
            prompt=2048 + 1024 + 40, chunk=1024)


def test_prefill_claimed_matches_torch_chunks():
    m = bench.Prefill(TINY, seed=1, threads=8)
    assert [t for _, t in m.chunks] == [1024, 1024, 1024, 40]
    ids = torch.randint(0, TINY["vocab"], (TINY["prompt"],), generator=torch.Generator().manual_seed(3),
                        dtype=torch.int64).pin_memory()
    m.fused = False  # every claimed op its own kernel
    m.run(ids)
    torch.cuda.synchronize()
    unfused = m.logits.clone().numpy()
    m.fused = True  # the norms in the packs, q/k norm with rope, ADDs and SwiGLU's operand in the epilogues
    m.run(ids)
    torch.cuda.synchronize()
    got = m.logits.clone().numpy()
    # the per-head norm sums in a warp rather than a block: last-bit
    # differences, which a bf16 rounding downstream can widen to 2^-8
    assert O.nrmse(got, unfused) <= 1e-2
    kc_claimed = m.kc[:, :3072].float().cpu().numpy()
    m.capture()  # the claimed chunks replayed from CUDA graphs: the same launches, the same bits
    m.run(ids, graphs=True)
    torch.cuda.synchronize()
    assert np.array_equal(m.logits.clone().numpy(), got)
    m.run(ids, claim=False)
    torch.cuda.synchronize()
    want = m.logits.clone().numpy()
    assert np.isfinite(got).all() and int(m.err.item()) == 0
    assert O.nrmse(got, want) <= 3e-2
    # the keys each path cached for the claimed chunks (post norm and rope)
    assert O.nrmse(kc_claimed, m.kc[:, :3072].float().cpu().numpy()) <= 3e-2
