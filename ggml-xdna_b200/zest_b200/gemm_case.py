"""K3 launches of the benchmark configs' shapes, for profiling and tuning.

    python -m zest_b200.gemm_case C1                 # six launches (for an ncu capture of the 6th)
    python -m zest_b200.gemm_case --plan             # the launch plans, on the host (no GPU)

Operands are bf16 on the device (A ~ N(0, 0.25), B ~ N(0, 0.0004), seeded); the
output is f32 holding bf16-rounded values, as the plugin's default.
"""
from __future__ import annotations

import argparse
import json

# (M, the N of each weight sharing A, K): one grouped launch of each config's layer
SHAPES = {
    "C1": (1024, [9728], 2560),
    "C3 qkv": (2048, [4096, 1024, 1024], 2560), "C3 o": (2048, [2560], 4096),
    "C3 gate+up": (2048, [9728, 9728], 2560), "C3 down": (2048, [2560], 9728),
    "C2 qkv": (8192, [4096, 1024, 1024], 2560), "C2 o": (8192, [2560], 4096),
    "C2 gate+up": (8192, [9728, 9728], 2560), "C2 down": (8192, [2560], 9728),
    "C5 m1024 gu": (1024, [10752, 10752], 2048), "C5 m1024 down": (1024, [2048], 10752),
    "C5 m2048 gu": (2048, [10752, 10752], 2048), "C5 m2048 down": (2048, [2048], 10752),
    "C4 m2048 qkv": (2048, [6144, 1024, 1024], 5120), "C4 m2048 gu": (2048, [17408, 17408], 5120),
    "C4 m2048 down": (2048, [5120], 17408),
    # not a config's launch: one k-block, so the epilogue is nearly all of the
    # launch (8192 x 8192 f32 out), for profiling the epilogue alone
    "K64 probe": (8192, [8192], 64),
}


def operands(M: int, Ns: list[int], K: int, seed: int = 0):
    import torch
    g = torch.Generator("cuda").manual_seed(seed)
    a = (torch.randn((M + 127) // 128 * 128, K, device="cuda", generator=g) * 0.5).to(torch.bfloat16)
    bs = [(torch.randn(N, K, device="cuda", generator=g) * 0.02).to(torch.bfloat16) for N in Ns]
    outs = [torch.empty(M, N, device="cuda") for N in Ns]
    return a.view(torch.int16), [b.view(torch.int16) for b in bs], outs


def run(name: str, launches: int = 6) -> None:
    import torch
    from . import MODE_BF16, gemm_group
    M, Ns, K = SHAPES[name]
    a, bs, outs = operands(M, Ns, K)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    for _ in range(launches):
        gemm_group(a, bs, M, Ns, [MODE_BF16] * len(Ns), outs, err=err)
    torch.cuda.synchronize()
    if int(err.item()):
        raise RuntimeError(f"{name}: device error bits {int(err.item()):#x}")


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("shapes", nargs="*", help=f"shape names (default: all): {', '.join(SHAPES)}")
    ap.add_argument("--plan", action="store_true", help="print each shape's launch plan (no GPU needed)")
    ap.add_argument("--sms", type=int, default=148, help="--plan: the SMs to plan for")
    ap.add_argument("--launches", type=int, default=6)
    args = ap.parse_args(argv)
    names = args.shapes or list(SHAPES)
    for s in names:
        if s not in SHAPES:
            ap.error(f"unknown shape {s!r}")
    if args.plan:
        from . import plan_gemm
        for s in names:
            M, Ns, K = SHAPES[s]
            print(json.dumps({"shape": s, **plan_gemm(M, K, Ns, args.sms)}))
        return
    for s in names:
        run(s, args.launches)
    print("ok")


if __name__ == "__main__":
    main()
