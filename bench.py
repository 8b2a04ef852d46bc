#!/usr/bin/env python
"""Benchmark of the prefill MUL_MAT path (BASELINE.json's metric).

    python bench.py [--gpus N --steps K --warmup W] [--impl ours|reference] [--workload NAME]

One step = one prefill chunk through every projection of a layer: the
activation pack (K2) of each distinct input, then each projection's GEMM
(K3), weights converted once beforehand (K1), as the reference converts them
at load. Inputs are seeded synthetic tensors with the configs' shapes and
distributions (no model files exist here). Multi-GPU: one process per GPU,
each converting and multiplying its N-slab of every weight, then an NCCL
all-gather of the output slabs.

--impl reference times the reference's own CPU path (xdna_ref_mul_mat,
oracle/_ref, compiled from the reference sources) on the host cores.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path[:0] = [str(ROOT), str(ROOT / "ggml-xdna_b200")]

METRIC = "prefill MUL_MAT TFLOP/s and tokens/s at 8K prompt; % of bf16 tensor-core peak"
Q8_0, Q4_K, Q6_K, IQ3_S = 8, 12, 14, 21
QNAME = {Q8_0: "Q8_0", Q4_K: "Q4_K", Q6_K: "Q6_K", IQ3_S: "IQ3_S"}

# (name, N, K, input) per projection; projections sharing an input share one pack
WORKLOADS = {
    "qwen3-4b-layer": dict(config="BASELINE configs[1]: Qwen3-4B-shaped layer, 7 projections", M=8192, qtype=Q4_K,
                           profiled="down",
                           proj=[("q", 4096, 2560, "attn"), ("k", 1024, 2560, "attn"), ("v", 1024, 2560, "attn"),
                                 ("o", 2560, 4096, "o"), ("gate", 9728, 2560, "ffn"), ("up", 9728, 2560, "ffn"),
                                 ("down", 2560, 9728, "down")]),
    "single-q8_0": dict(config="BASELINE configs[0]: one MUL_MAT, Q8_0", M=1024, qtype=Q8_0,
                        proj=[("w", 9728, 2560, "x")]),
    "27b-layer-m8192": dict(config="BASELINE configs[3]: 27B-class layer, IQ3_S, M=8192", M=8192, qtype=IQ3_S,
                            proj=[("q", 6144, 5120, "attn"), ("k", 1024, 5120, "attn"), ("v", 1024, 5120, "attn"),
                                  ("gate", 17408, 5120, "ffn"), ("up", 17408, 5120, "ffn"),
                                  ("down", 5120, 17408, "down")]),
    "27b-layer-m2048": dict(config="BASELINE configs[3]: 27B-class layer, IQ3_S, M=2048", M=2048, qtype=IQ3_S,
                            proj=[("q", 6144, 5120, "attn"), ("k", 1024, 5120, "attn"), ("v", 1024, 5120, "attn"),
                                  ("gate", 17408, 5120, "ffn"), ("up", 17408, 5120, "ffn"),
                                  ("down", 5120, 17408, "down")]),
}
for _m in (1024, 2048, 4096, 8192, 16384):
    WORKLOADS[f"lfm-m{_m}"] = dict(config=f"BASELINE configs[4]: LFM-style Q8_0 FFN, M={_m}, 1% x50 outliers", M=_m,
                                   qtype=Q8_0, outliers=True,
                                   proj=[("gate", 10752, 2048, "ffn"), ("up", 10752, 2048, "ffn"),
                                         ("down", 2048, 10752, "down")])

DEFAULT = "qwen3-4b-layer"


def flops(w: dict) -> float:
    return float(sum(2.0 * w["M"] * n * k for _, n, k, _ in w["proj"]))


def launch_groups(w: dict) -> list:
    """[(input, [(name, N, K), ...])]: the projections sharing an input, in
    order; each group is one pack and one grouped K3 launch."""
    g = {}
    for name, N, K, kind in w["proj"]:
        g.setdefault(kind, []).append((name, N, K))
    return list(g.items())


def seed_of(name: str, salt: int = 0) -> int:
    return (sum((i + 1) * ord(c) for i, c in enumerate(name)) * 7919 + salt) % (2 ** 31)


def quantize_threaded(qtype: int, w: np.ndarray, threads: int) -> np.ndarray:
    from oracle import oracle as O
    O.orc()  # load the library (and the IQ3_S codebook) before the worker threads use it
    rows = w.shape[0]
    chunks = [(i, min(rows, i + max(1, rows // threads))) for i in range(0, rows, max(1, rows // threads))]
    with ThreadPoolExecutor(threads) as ex:
        parts = list(ex.map(lambda c: O.quantize(qtype, w[c[0]:c[1]]), chunks))
    return np.concatenate(parts)


def weight_raw(qtype: int, name: str, N: int, K: int, threads: int) -> np.ndarray:
    """A projection's GGUF bytes: N(0, 0.02) floats quantised (seeded)."""
    from oracle import oracle as O
    return quantize_threaded(qtype, O.weights_f32(N, K, seed_of(name, 1)), threads)


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------

class ClockSampler:
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu, self.proc, self.lines = gpu, None, []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 7:
                continue
            try:
                sm.append(float(f[0]))
                mx = float(f[1])
            except ValueError:
                continue
            for n, v in zip(names, f[3:7]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"tflops_burst": d.get("bf16_tflops"), "tflops_sustained": d.get("bf16_tflops_sustained"),
                "hbm_gbs": d.get("hbm_gbs"), "source": "measured"}
    return {"tflops_burst": 1590.0, "tflops_sustained": 1400.0, "hbm_gbs": 6650.0, "source": "fallback"}


def profiled_traffic(kernel: str, workload: str):
    """DRAM bytes per launch of `kernel` from the committed ncu summary for this
    workload (profiles/<kernel>_<workload>.md, line 'traffic_bytes_per_launch: X'),
    or None when no capture exists."""
    p = ROOT / "profiles" / f"{kernel}_{workload}.md"
    if not p.exists():
        return None
    for ln in p.read_text().splitlines():
        if ln.startswith("traffic_bytes_per_launch:"):
            try:
                return float(ln.split(":", 1)[1].strip())
            except ValueError:
                return None
    return None


# ---------------------------------------------------------------------------
# the reference's CPU path
# ---------------------------------------------------------------------------

def cpu_reference_run(w: dict, rows: int, threads: int, raws: dict) -> tuple[float, float]:
    """xdna_ref_mul_mat (oracle/_ref) over `rows` tokens of every projection,
    all host threads. Returns (flops, seconds)."""
    from oracle import oracle as O
    kinds = {}
    fl, t = 0.0, 0.0
    for name, N, K, kind in w["proj"]:
        if kind not in kinds:
            kinds[kind] = O.activations(rows, K, seed_of(kind, 2), outliers=w.get("outliers", False))
        x = kinds[kind]
        t0 = time.perf_counter()
        if O.has_ref():
            O.ref_mul_mat(w["qtype"], raws[name], N, K, x, n_threads=threads)
        else:
            O.mul_mat(O.dequant(w["qtype"], raws[name], N, K), x, n_threads=threads)
        t += time.perf_counter() - t0
        fl += 2.0 * rows * N * K
    return fl, t


def cpu_baseline(w: dict, raws: dict, budget_s: float = 12.0) -> dict:
    from oracle import oracle as O
    threads = os.cpu_count() or 1
    fl, t = cpu_reference_run(w, 16, threads, raws)  # calibration
    rows = int(max(16, min(w["M"], 16 * budget_s / max(t, 1e-3))))
    fl, t = cpu_reference_run(w, rows, threads, raws)
    return {"value": fl / t / 1e12, "unit": "TFLOP/s", "cores": threads,
            "kind": "reference" if O.has_ref() else "port",
            "sample": f"{rows} of {w['M']} token rows through every projection ({fl / 1e9:.1f} GFLOP, {t:.1f} s)",
            "tokens_per_s": rows / t}


def run_reference(args, w: dict) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return  # the CPU path runs once, on rank 0
    from oracle import oracle as O
    threads = os.cpu_count() or 1
    raws = {name: weight_raw(w["qtype"], name, N, K, threads) for name, N, K, _ in w["proj"]}
    # rows per step: a bounded sample sized so all steps take about a minute
    _, t16 = cpu_reference_run(w, 16, threads, raws)
    rows = int(max(8, min(128, 16 * 60.0 / (args.steps + args.warmup) / max(t16, 1e-3))))
    for _ in range(args.warmup):
        cpu_reference_run(w, rows, threads, raws)
    fl, t = 0.0, 0.0
    for _ in range(args.steps):
        f, s = cpu_reference_run(w, rows, threads, raws)
        fl += f
        t += s
    value = fl / t / 1e12
    kind = "reference" if O.has_ref() else "port"
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": t / args.steps * 1e3, "higher_is_better": True,
        "scaling": "none", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": args.workload, "desc": w["config"], "M": w["M"], "weights": QNAME[w["qtype"]],
                   "sample_rows_per_step": rows},
        "tokens_per_s": rows * args.steps / t,
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": kind,
                         "sample": f"{rows} of {w['M']} token rows through every projection per step"},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


# ---------------------------------------------------------------------------
# ours
# ---------------------------------------------------------------------------

def run_ours(args, w: dict) -> None:
    import torch
    import torch.distributed as dist

    import zest_b200 as Z

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    threads = max(1, (os.cpu_count() or 1) // max(1, world))
    if w["qtype"] == IQ3_S:
        Z.load_iq3s_grid()
    M, qt = w["M"], w["qtype"]

    # tokens: every rank its own prompt chunk through whole weights (no
    # collective); nshard: every rank an N-slab of each weight, outputs
    # all-gathered into ggml's row-major [M][N]
    from zest_b200.shard import gather_slabs, shard_rows, slab_width
    nshard = world > 1 and args.mode != "tokens"
    gather = nshard and args.mode == "nshard"

    # --- load: every projection's (slab of) weight converted once (K1) ---------
    raws, bh, slabs = {}, {}, {}
    for name, N, K, _ in w["proj"]:
        raws[name] = weight_raw(qt, name, N, K, threads)
        row0, n = shard_rows(N, world, rank) if nshard else (0, N)
        slabs[name] = (row0, n)
        raw_dev = torch.from_numpy(raws[name]).cuda()
        _, bh[name] = Z.convert_weight(qt, raw_dev, N, K, row0=row0, n_rows=n, want_bytes=False)
        del raw_dev
    torch.cuda.synchronize()

    # --- inputs and outputs ------------------------------------------------
    kinds = {}
    for name, N, K, kind in w["proj"]:
        kinds.setdefault(kind, K)
    x, ah = {}, {}
    gen = torch.Generator("cuda").manual_seed(1234 + (0 if nshard else rank))  # tokens: each rank its own chunk
    for kind, K in kinds.items():
        x[kind] = torch.randn(M, K, device="cuda", generator=gen)
        if w.get("outliers"):
            mask = torch.rand(M, K, device="cuda", generator=gen) < 0.01
            x[kind] = torch.where(mask, x[kind] * 50, x[kind])
        ah[kind] = torch.empty((Z.pad_to(M, 128), K), dtype=torch.int16, device="cuda")
    width = {name: (slab_width(N, world) if nshard else N) for name, N, *_ in w["proj"]}
    out = {name: torch.zeros((M, max(1, width[name])), dtype=torch.float32, device="cuda") for name, *_ in w["proj"]}
    full = {}
    if gather:
        for name, N, K, _ in w["proj"]:
            full[name] = torch.empty((M, N), dtype=torch.float32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream()
    L = Z.lib()
    sp = ctypes.c_void_p(stream.cuda_stream)

    # one K3 launch per input: the projections that share it (q, k, v; gate, up)
    # are the segments of one grouped launch
    groups = launch_groups(w)
    gargs = []
    for kind, members in groups:
        n = len(members)
        gargs.append((kind, (ctypes.c_void_p * n)(*[bh[name].data_ptr() for name, _, _ in members]),
                      (ctypes.c_int64 * n)(*[K for _, _, K in members]),
                      (ctypes.c_int64 * n)(*[slabs[name][1] for name, _, _ in members]),
                      (ctypes.c_int * n)(*[Z.MODE_BF16] * n),
                      (ctypes.c_void_p * n)(*[out[name].data_ptr() for name, _, _ in members]),
                      (ctypes.c_int64 * n)(*[out[name].shape[1] for name, _, _ in members]), members))

    def step(events=None):
        for kind, K in kinds.items():
            rc = L.zest_pack_activations(ctypes.c_void_p(x[kind].data_ptr()), M, K, K, ah[kind].shape[0], None,
                                         ctypes.c_void_p(ah[kind].data_ptr()), K, sp)
            if rc:
                raise Z.ZestError(L.zest_last_error().decode())
        for i, (kind, bp, ldb, ns, modes, cp, ldc, members) in enumerate(gargs):
            K = kinds[kind]
            if events is not None:
                events[i][0].record(stream)
            rc = L.zest_gemm_group(ctypes.c_void_p(ah[kind].data_ptr()), K, M, K, len(members), bp, ldb, ns, modes,
                                   cp, ldc, ctypes.c_void_p(err.data_ptr()), sp)
            if events is not None:
                events[i][1].record(stream)
            if rc:
                raise Z.ZestError(L.zest_last_error().decode())
            if gather:
                for name, N, _ in members:
                    gather_slabs(out[name], full[name], world, N)

    # --- warm-up, then K timed steps ---------------------------------------
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if int(err.item()):
        raise Z.ZestError(f"device error bits {int(err.item()):#x} during warm-up")
    ev = [[[torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)] for _ in groups]
          for _ in range(args.steps)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        t0.record(stream)
        for s in range(args.steps):
            step(ev[s])
        t1.record(stream)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = t0.elapsed_time(t1) / args.steps
    gemm_ms = [sum(ev[s][i][0].elapsed_time(ev[s][i][1]) for s in range(args.steps)) / args.steps
               for i in range(len(groups))]
    if int(err.item()):
        raise Z.ZestError(f"device error bits {int(err.item()):#x} in the timed region")
    t = torch.tensor([ms], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())

    total_flops = flops(w) * (1 if nshard else world)  # the whole job: all ranks' tokens
    local_gemm_flops = sum(2.0 * M * slabs[name][1] * K for name, N, K, _ in w["proj"])
    peaks = measured_peaks()
    gemm_total_ms = sum(gemm_ms)
    # the roofline's launch: the group holding the profiled projection (the
    # one the committed ncu capture profiles), else the one with the most work
    gflops = [sum(2.0 * M * slabs[name][1] * K for name, _, K in members) for _, members in groups]
    names = [[name for name, _, _ in members] for _, members in groups]
    top = next((i for i, ns in enumerate(names) if w.get("profiled") in ns), None)
    if top is None:
        top = max(range(len(groups)), key=lambda i: gflops[i])
    top_flops = gflops[top]
    top_desc = " + ".join(f"{name} {M}x{slabs[name][1]}x{K}" for name, _, K in groups[top][1])
    achieved = top_flops / (gemm_ms[top] * 1e-3) / 1e12
    traffic = profiled_traffic("k3_gemm", args.workload) if world == 1 else None

    # --- end to end through the C ABI, host buffers: each rank its own chunk ----
    e2e = None
    if not nshard:
        if world > 1:
            dist.barrier()
        e2e = e2e_run(args, w, raws, Z, torch)
        if world > 1:
            t = torch.tensor([e2e["ms_per_step"]], dtype=torch.float64, device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e2e["ms_per_step"] = float(t.item())
            e2e["value"] = world * flops(w) / (e2e["ms_per_step"] * 1e-3) / 1e12
            e2e["tokens_per_s"] = world * M / (e2e["ms_per_step"] * 1e-3)
            e2e["h2d_bytes_per_step"] *= world
            e2e["d2h_bytes_per_step"] *= world

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline(w, raws)

    if rank == 0:
        value = total_flops / (ms_max * 1e-3) / 1e12
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max, "higher_is_better": True,
            "scaling": ("strong" if nshard else "weak") if world > 1 else "none", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic",
            "config": {"workload": args.workload, "desc": w["config"], "M": M, "weights": QNAME[qt],
                       "projections": {name: [N, K] for name, N, K, _ in w["proj"]},
                       "parallelism": (f"n-shard{world}" + ("+allgather" if gather else "")) if nshard else
                                      f"tokens{world} (each GPU its own {M}-token chunk, no collective)",
                       "global_tokens_per_step": M * (1 if nshard else world),
                       "output": "f32 holding bf16-rounded values (reference default GGML_XDNA_OUT16=1)",
                       "l2": "no flush: each step reads %.0f MB of inputs and weights (> 126 MB L2)" %
                             (sum(M * K * 4 for K in kinds.values()) / 1e6 +
                              sum(slabs[n][1] * K * 2 for n, N, K, _ in w["proj"]) / 1e6)},
            "tokens_per_s": M * (1 if nshard else world) / (ms_max * 1e-3),
            "pct_of_bf16_peak": 100.0 * value / (world * peaks["tflops_sustained"]),
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peaks["tflops_sustained"],
                         "unit": "TFLOP/s", "frac": achieved / peaks["tflops_sustained"],
                         "traffic": traffic, "kernel": "k3 gemm_bf16_tc_kernel",
                         "launch": f"{top_desc}: {top_flops / 1e9:.1f} GFLOP, {gemm_ms[top] * 1e3:.1f} us avg",
                         "peak_kind": f"bf16 sustained ({peaks['source']})", "peak_burst": peaks["tflops_burst"],
                         "all_gemms": {"ms_per_step": gemm_total_ms,
                                       "tflops": local_gemm_flops / (gemm_total_ms * 1e-3) / 1e12,
                                       "per_launch_us": {"+".join(ns): round(t * 1e3, 1)
                                                         for ns, t in zip(names, gemm_ms)}}},
            "gpu_launches": args.steps * (len(kinds) + len(groups)),
            "clocks": clocks.summary(),
        }
        if e2e:
            line["e2e"] = e2e
        if cpu:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def e2e_run(args, w: dict, raws: dict, Z, torch) -> dict:
    """The same step through the C ABI's matmul service, host (pinned) inputs
    and outputs, host<->device copies inside the timed region."""
    M = w["M"]
    npu = Z.Npu(torch.cuda.current_device())
    keys = {}
    for name, N, K, _ in w["proj"]:
        keys[name] = Z.Npu.key(raws[name].ctypes.data, w["qtype"], K, N)
        npu.add_weight(keys[name], raws[name].ctypes.data, on_device=False)
    xs = {}
    for name, N, K, kind in w["proj"]:
        if kind not in xs:
            xs[kind] = torch.randn(M, K, generator=torch.Generator().manual_seed(seed_of(kind))).pin_memory()
    ys = {name: torch.empty((M, N), dtype=torch.float32).pin_memory() for name, N, *_ in w["proj"]}
    st = torch.cuda.ExternalStream(npu.stream())

    groups = launch_groups(w)

    def step():
        for kind, members in groups:
            npu.mul_mat_group([keys[name] for name, _, _ in members], xs[kind].data_ptr(), M,
                              [ys[name].data_ptr() for name, _, _ in members], on_device=False)

    for _ in range(max(1, min(args.warmup, 2))):
        step()
    steps = max(1, min(args.steps, 5))
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    a.record(st)
    for _ in range(steps):
        step()
    b.record(st)
    b.synchronize()
    ms = a.elapsed_time(b) / steps
    h2d = sum(M * members[0][2] * 4 for _, members in groups)
    d2h = sum(sum(M * N * 4 for _, N, _ in members) + 4 for _, members in groups)
    npu.close()
    return {"value": flops(w) / (ms * 1e-3) / 1e12, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "ms_per_step": ms, "tokens_per_s": M / (ms * 1e-3), "steps": steps,
            "api": "zest_mul_mat_group (include/zest_b200.h), host buffers, one call per shared input"}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default=DEFAULT)
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--mode", choices=["tokens", "nshard", "nshard-nogather"], default="tokens",
                    help="N>1: each GPU its own token chunk (default, no collective), or N-slabs of every weight "
                         "with (nshard) or without the NCCL all-gather of the output slabs")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)  # at least 3 untimed warm-up steps
    w = WORKLOADS[args.workload]
    if args.impl == "reference":
        run_reference(args, w)
    else:
        run_ours(args, w)


if __name__ == "__main__":
    main()
