#!/usr/bin/env python
"""Benchmark of the prefill MUL_MAT path (BASELINE.json's metric).

    python bench.py [--gpus N --steps K --warmup W] [--impl ours|reference] [--workload NAME]

One step = one prefill chunk through every projection of a layer: the
activation pack (K2) of each distinct input, then one grouped GEMM launch
(K3) per input (q+k+v, o, gate+up, down), weights converted once beforehand
(K1), as the reference converts them at load. Inputs are seeded synthetic
tensors with the configs' shapes and distributions (no model files exist
here). --workload picks BASELINE's configs: qwen3-4b-layer (the default,
configs[1]), single-q8_0, qwen3-4b-model (configs[2], a whole
36-layer prefill in tok/s), 27b-layer-m8192/m2048 and
lfm-m1024..16384.

Multi-GPU (one process per GPU under torchrun, NCCL): --mode tokens (the
default) gives every rank its own prompt chunk, no collective; nshard /
nshard-nogather split every weight's rows with / without the all-gather of
the output slabs; tp runs the layer as one tensor-parallel block (o/down
K-sharded, one all-reduce of their partials, by NCCL or by the GEMM itself
through NVLink multicast).

--impl reference times the reference's own CPU path (xdna_ref_mul_mat,
oracle/_ref, compiled from the reference sources) on the host cores.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import math
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

WORKLOADS["qwen3-4b-model"] = dict(config="BASELINE configs[2]: 36-layer Qwen3-4B-shaped Q4_K_M-style prefill, "
                                          "8,296-token prompt in chunks of 2048", M=2048, qtype=Q4_K, model=True,
                                   proj=WORKLOADS["qwen3-4b-layer"]["proj"])

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
    """SM clocks and clock-event reasons read (never set) every 10 ms through
    NVML while the timed region runs; nvidia-smi -lms 50 where NVML is
    missing. The first sample is in before __enter__ returns."""
    REASONS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40}
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu, self.proc, self.lines = gpu, None, []
        self.samples, self.max_mhz, self.stop, self.thread = [], None, threading.Event(), None

    def _nvml(self) -> bool:
        try:
            import pynvml
            import torch
            pynvml.nvmlInit()
            pr = torch.cuda.get_device_properties(self.gpu)
            try:
                bus = f"{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
                h = pynvml.nvmlDeviceGetHandleByPciBusId(bus.encode())
            except Exception:
                h = pynvml.nvmlDeviceGetHandleByIndex(self.gpu)
            reasons = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                pynvml.nvmlDeviceGetCurrentClocksThrottleReasons
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))

            def loop():
                while not self.stop.is_set():
                    self.samples.append((float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)),
                                         int(reasons(h))))
                    self.stop.wait(0.01)

            self.thread = threading.Thread(target=loop, daemon=True)
            self.thread.start()
            t = time.time()
            while not self.samples and self.thread.is_alive() and time.time() - t < 5:
                time.sleep(0.001)
            return bool(self.samples)
        except Exception:
            return False

    def __enter__(self):
        if self._nvml():
            return self
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
            t = time.time()
            while not self.lines and self.proc.poll() is None and time.time() - t < 10:
                time.sleep(0.005)
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        self.stop.set()
        if self.thread:
            self.thread.join(timeout=1)
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], self.max_mhz, set()
        for mhz, bits in self.samples:
            sm.append(mhz)
            reasons.update(n for n, b in self.REASONS.items() if bits & b)
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
                "samples": len(sm), "source": "nvml" if self.samples else "nvidia-smi"}


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"tflops_burst": d.get("bf16_tflops"), "tflops_sustained": d.get("bf16_tflops_sustained"),
                "hbm_gbs": d.get("hbm_gbs"), "source": "measured"}
    return {"tflops_burst": 1590.0, "tflops_sustained": 1400.0, "hbm_gbs": 6650.0, "source": "fallback"}


def choose_peak(peaks: dict, timed_s: float, clocks: dict) -> tuple[float, str]:
    """The bf16 roofline denominator for a timed region. MEASURED_PEAKS.json
    holds cuBLAS's bf16 GEMM timed alone at full clock (burst) and back to
    back for seconds under the 1 kW cap (sustained). A region of under two
    seconds, or one whose sampled SM clock stayed near its maximum, runs as
    the burst did; only a region of seconds whose median clock sat well
    below the maximum is held to the sustained figure."""
    sm, mx = clocks.get("sm_mhz"), clocks.get("sm_max_mhz")
    capped = sm is not None and mx and sm < 0.9 * mx
    if timed_s >= 2.0 and capped:
        return peaks["tflops_sustained"], (f"bf16 sustained ({peaks['source']}): {timed_s:.1f} s timed at a median "
                                           f"{sm:.0f} of {mx:.0f} MHz")
    return peaks["tflops_burst"], (f"bf16 burst ({peaks['source']}): {timed_s * 1e3:.0f} ms timed at a median "
                                   f"{sm} of {mx} MHz")


def profiled_traffic(workload: str, launch: str):
    """DRAM bytes (read + write) per launch of `launch` from the committed ncu
    summary of this workload's K3 launches (profiles/k3_gemm_<workload>.md,
    a line 'traffic_bytes_per_launch[<launch>]: X'), or None."""
    p = ROOT / "profiles" / f"k3_gemm_{workload}.md"
    if not p.exists():
        return None
    key = f"traffic_bytes_per_launch[{launch}]:"
    for ln in p.read_text().splitlines():
        if ln.startswith(key):
            try:
                return float(ln[len(key):].strip())
            except ValueError:
                return None
    return None


# ---------------------------------------------------------------------------
# the reference's CPU path
# ---------------------------------------------------------------------------

def ref_activations(w: dict) -> dict:
    """Every input of the layer, all M token rows (seeded), for the CPU path."""
    from oracle import oracle as O
    xs = {}
    for _, _, K, kind in w["proj"]:
        if kind not in xs:
            xs[kind] = O.activations(w["M"], K, seed_of(kind, 2), outliers=w.get("outliers", False))
    return xs


def cpu_reference_sample(w: dict, raws: dict, xs: dict, frac: float, threads: int) -> tuple[float, float, int]:
    """xdna_ref_mul_mat (oracle/_ref; the oracle's port where it is not built)
    over ALL M token rows and the first max(threads, frac * N) weight rows of
    every projection. The reference splits its threads over weight rows and
    streams every token row past each one, so a slice of weight rows costs
    per flop what the whole weight does. Returns (flops, seconds, rows)."""
    from oracle import oracle as O
    M, qt = w["M"], w["qtype"]
    fl, t, rows = 0.0, 0.0, 0
    for name, N, K, kind in w["proj"]:
        n = min(N, max(threads, int(round(N * frac))))
        raw = raws[name][:n * O.row_bytes(qt, K)]
        t0 = time.perf_counter()
        if O.has_ref():
            O.ref_mul_mat(qt, raw, n, K, xs[kind], n_threads=threads)
        else:
            O.mul_mat(O.dequant(qt, raw, n, K), xs[kind], n_threads=threads)
        t += time.perf_counter() - t0
        fl += 2.0 * M * n * K
        rows += n
    return fl, t, rows


def cpu_sample_frac(w: dict, raws: dict, xs: dict, threads: int, seconds: float) -> float:
    """The weight-row fraction whose sample takes about `seconds` (calibrated
    on a sample of `threads` rows per projection)."""
    fl, t, _ = cpu_reference_sample(w, raws, xs, 0.0, threads)
    return min(1.0, seconds * fl / max(t, 1e-6) / flops(w))


def cpu_baseline(w: dict, raws: dict, budget_s: float = 12.0) -> dict:
    from oracle import oracle as O
    threads = os.cpu_count() or 1
    xs = ref_activations(w)
    frac = cpu_sample_frac(w, raws, xs, threads, budget_s)
    fl, t, rows = cpu_reference_sample(w, raws, xs, frac, threads)
    total_rows = sum(N for _, N, _, _ in w["proj"])
    return {"value": fl / t / 1e12, "unit": "TFLOP/s", "cores": threads,
            "kind": "reference" if O.has_ref() else "port",
            "sample": f"all {w['M']} token rows x {rows} of the {total_rows} weight rows (every projection's first "
                      f"{100 * rows / total_rows:.0f} %): {fl / 1e9:.1f} GFLOP in {t:.1f} s",
            "tokens_per_s": w["M"] * fl / flops(w) / t}


def run_reference(args, w: dict) -> None:
    """The reference's CPU path on the host cores, on our arm's config: each
    step all M token rows through a slice of every projection's weight rows,
    the slice sized so the whole run takes about a minute (ZEST_REF_SECONDS)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return  # the CPU path runs once, on rank 0
    from oracle import oracle as O
    threads = os.cpu_count() or 1
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    raws = {name: weight_raw(w["qtype"], name, N, K, threads) for name, N, K, _ in w["proj"]}
    xs = ref_activations(w)
    budget = float(os.environ.get("ZEST_REF_SECONDS") or 60.0)  # the whole run's CPU time, about
    frac = cpu_sample_frac(w, raws, xs, threads, budget / (args.steps + args.warmup))
    for _ in range(args.warmup):
        cpu_reference_sample(w, raws, xs, frac, threads)
    fl, t, rows = 0.0, 0.0, 0
    for _ in range(args.steps):
        f, s_, rows = cpu_reference_sample(w, raws, xs, frac, threads)
        fl += f
        t += s_
    value = fl / t / 1e12
    kind = "reference" if O.has_ref() else "port"
    total_rows = sum(N for _, N, _, _ in w["proj"])
    sample = (f"each step all {w['M']} token rows x {rows} of the {total_rows} weight rows (every projection's "
              f"first {100 * rows / total_rows:.1f} %), {fl / args.steps / 1e9:.1f} GFLOP")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": t / args.steps * 1e3, "higher_is_better": True,
        "scaling": layer_scaling(world, args.mode), "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": layer_config(w, args.workload, world, args.mode),
        "tokens_per_s": w["M"] * fl / flops(w) / t,
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": kind, "sample": sample},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


# ---------------------------------------------------------------------------
# ours
# ---------------------------------------------------------------------------

def layer_mode(world: int, mode) -> str:
    """--mode, defaulted: one GPU runs the whole layer; N > 1 the north
    star's partition, N-slabs of every weight with the output all-gather."""
    return mode or ("tokens" if world == 1 else "nshard")


def layer_scaling(world: int, mode) -> str:
    if world == 1:
        return "none"
    return "weak" if layer_mode(world, mode) == "tokens" else "strong"


def layer_config(w: dict, workload: str, world: int, mode) -> dict:
    """The run's config, the same in both arms."""
    from zest_b200.shard import slab_width
    mode = layer_mode(world, mode)
    nshard = world > 1 and mode != "tokens"
    M = w["M"]
    kinds = {}
    for _, _, K, kind in w["proj"]:
        kinds.setdefault(kind, K)
    if not nshard:
        par = "1 GPU" if world == 1 else f"tokens{world} (each GPU its own {M}-token chunk, no collective)"
    elif mode == "nshard":
        par = (f"n-shard{world}: every GPU a slab of each weight's rows (whole 128-row granules), the output "
               "slabs all-gathered into ggml's row-major f32 [M][N] on every GPU: by the GEMM epilogue through "
               "an NVLink multicast address as the tiles finish, or over NCCL (bf16 on the wire) where a GPU "
               "has no multicast (the line's 'gather' says which)")
    else:
        par = f"n-shard{world}, no gather: every GPU a slab of each weight's rows, the output slabs left in place"
    wbytes = sum((slab_width(N, world) if nshard else N) * K * 2 for _, N, K, _ in w["proj"])
    return {"workload": workload, "desc": w["config"], "M": M, "weights": QNAME[w["qtype"]],
            "projections": {name: [N, K] for name, N, K, _ in w["proj"]},
            "parallelism": par, "global_tokens_per_step": M * (1 if nshard else world),
            "output": "f32 holding bf16-rounded values (reference default GGML_XDNA_OUT16=1)",
            "l2": "no flush: each step reads %.0f MB of inputs and weights (> 126 MB L2)" %
                  ((sum(M * K * 4 for K in kinds.values()) + wbytes) / 1e6)}


class LayerStep:
    """One layer's MUL_MATs on this rank as the bench runs them: per distinct
    input one K2 pack, then one grouped K3 launch per input (q+k+v, o,
    gate+up, down), weights converted beforehand (K1) as the reference
    converts them at load. nshard: this rank's N-slab of every weight; with
    gather, every rank gets the whole [M][N] output of every weight: by
    default each launch's epilogue stores its slab's tiles through an NVLink
    multicast address into every rank's copy (multimem.st; the NVSwitch does
    the all-gather as the tiles finish, and a one-float all-reduce ends the
    step as the group's fence), else (gather_how "nccl", or no multicast on
    some rank) the slabs are all-gathered over NCCL, bf16 on the wire, on a
    side stream while the next launch runs."""

    def __init__(self, w: dict, raws: dict, world: int, rank: int, nshard: bool, gather: bool, Z, torch,
                 gather_how: str = "peer16"):
        from zest_b200.shard import any_rank, shard_rows, slab_width
        self.w, self.world, self.nshard, self.gather, self.Z, self.torch = w, world, nshard, gather, Z, torch
        M, qt = w["M"], w["qtype"]
        self.bh, self.slabs = {}, {}
        for name, N, K, _ in w["proj"]:
            row0, n = shard_rows(N, world, rank) if nshard else (0, N)
            self.slabs[name] = (row0, n)
            raw_dev = torch.from_numpy(raws[name]).cuda()
            _, self.bh[name] = Z.convert_weight(qt, raw_dev, N, K, row0=row0, n_rows=n, want_bytes=False)
            del raw_dev
        torch.cuda.synchronize()
        self.kinds = {}
        for name, N, K, kind in w["proj"]:
            self.kinds.setdefault(kind, K)
        self.x, self.ah = {}, {}
        gen = torch.Generator("cuda").manual_seed(1234 + (0 if nshard else rank))  # tokens: each rank its own chunk
        for kind, K in self.kinds.items():
            self.x[kind] = torch.randn(M, K, device="cuda", generator=gen)
            if w.get("outliers"):
                mask = torch.rand(M, K, device="cuda", generator=gen) < 0.01
                self.x[kind] = torch.where(mask, self.x[kind] * 50, self.x[kind])
            self.ah[kind] = torch.empty((Z.pad_to(M, 128), K), dtype=torch.int16, device="cuda")
        width = {name: (slab_width(N, world) if nshard else N) for name, N, *_ in w["proj"]}
        self.out = {name: torch.zeros((M, max(1, width[name])), dtype=torch.float32, device="cuda")
                    for name, *_ in w["proj"]}
        self.full = {name: torch.empty((M, N), dtype=torch.float32, device="cuda")
                     for name, N, _, _ in w["proj"]} if gather else {}
        # the whole outputs in symmetric memory: bound to an NVLink multicast
        # object (multicast), or reached through every peer's pointer (peer)
        self.mc, self.mc_why, self.how = {}, None, gather_how if gather else "none"
        if gather and gather_how in ("multicast", "peer", "peer16"):
            import torch.distributed as dist
            try:
                import torch.distributed._symmetric_memory as symm_mem
                for name, N, _, _ in w["proj"]:
                    t = symm_mem.empty((M, N), dtype=torch.bfloat16 if gather_how == "peer16" else torch.float32,
                                       device="cuda")
                    hdl = symm_mem.rendezvous(t, dist.group.WORLD)
                    if gather_how == "multicast" and not hdl.multicast_ptr:
                        raise RuntimeError("no multicast support")
                    self.mc[name] = (t, hdl, int(hdl.multicast_ptr or 0), [int(p) for p in hdl.buffer_ptrs])
            except Exception as e:  # every rank falls back to NCCL below
                self.mc, self.mc_why = {}, f"{type(e).__name__}: {e}"
            if any_rank(not self.mc):
                self.mc_why = self.mc_why or "symmetric memory unavailable on another rank"
                self.mc = {}
                self.how = "nccl"
            self.tick = torch.zeros(1, device="cuda")
        self.err = torch.zeros(1, dtype=torch.int32, device="cuda")
        self.stream = torch.cuda.current_stream()
        self.comm = torch.cuda.Stream() if gather else None
        self.sp = ctypes.c_void_p(self.stream.cuda_stream)
        self.groups = launch_groups(w)
        self.gargs = []
        for kind, members in self.groups:
            n = len(members)
            self.gargs.append((kind, (ctypes.c_void_p * n)(*[self.bh[nm].data_ptr() for nm, _, _ in members]),
                               (ctypes.c_int64 * n)(*[K for _, _, K in members]),
                               (ctypes.c_int64 * n)(*[self.slabs[nm][1] for nm, _, _ in members]),
                               (ctypes.c_int * n)(*[Z.MODE_BF16] * n),
                               (ctypes.c_void_p * n)(*[self.out[nm].data_ptr() for nm, _, _ in members]),
                               (ctypes.c_int64 * n)(*[self.out[nm].shape[1] for nm, _, _ in members]), members))
        self.launches = len(self.kinds) + len(self.groups)
        # multicast gather: each group's segments write their slab into every rank's whole output
        self.msegs, self.peer_arrays = [], []
        if self.mc:
            for kind, members in self.groups:
                segs = []
                for nm, _, K in members:
                    t, _, mcp, ptrs = self.mc[nm]
                    N, off = t.shape[1], 4 * self.slabs[nm][0]
                    if self.how == "peer16":
                        c16 = (ctypes.c_void_p * world)(*[ptrs[j] + off // 2 for j in range(world)])
                        self.peer_arrays.append(c16)
                        segs.append(Z.GemmSeg(self.bh[nm].data_ptr(), K, self.slabs[nm][1], Z.MODE_BF16, None, 0,
                                              None, 0, None, 0, None, 0, None, 0,
                                              ctypes.cast(c16, ctypes.POINTER(ctypes.c_void_p)), world, N))
                    elif self.how == "multicast":
                        segs.append(Z.GemmSeg(self.bh[nm].data_ptr(), K, self.slabs[nm][1], Z.MODE_BF16, None, N,
                                              None, 0, None, 0, mcp + off, 1))
                    else:
                        peers = (ctypes.c_void_p * (world - 1))(*[ptrs[j] + off for j in range(world) if j != rank])
                        self.peer_arrays.append(peers)
                        segs.append(Z.GemmSeg(self.bh[nm].data_ptr(), K, self.slabs[nm][1], Z.MODE_BF16,
                                              t.data_ptr() + off, N, None, 0, None, 0, None, 0,
                                              ctypes.cast(peers, ctypes.POINTER(ctypes.c_void_p)), world - 1))
                self.msegs.append((Z.GemmSeg * len(segs))(*segs))

    def gather_desc(self) -> str:
        if not self.gather:
            return "none"
        if self.mc and self.how == "peer16":
            return ("TMA stores of each launch's tiles in bf16 into every rank's whole bf16 output (peer pointers "
                    "over NVLink), widened to f32 on every rank after each launch's fence")
        if self.mc and self.how == "multicast":
            return "multimem.st of each launch's tiles into every rank's whole output (NVLink multicast)"
        if self.mc:
            return "TMA stores of each launch's tiles into every rank's whole output (peer pointers over NVLink)"
        return "NCCL all-gather of the slabs, bf16 on the wire" + (f" (multicast: {self.mc_why})" if self.mc_why else "")

    def check_gather(self) -> float:
        """The outputs gathered by the GEMM epilogue (multicast, peer or bf16
        peer stores) against the NCCL all-gather of the same slabs computed
        into local buffers: the largest difference over this rank's outputs
        (0 when they agree bit for bit). Collective."""
        import torch.distributed as dist
        from zest_b200.shard import gather_slabs
        torch, Z, L = self.torch, self.Z, self.Z.lib()
        self.step()
        dist.all_reduce(self.tick)
        torch.cuda.synchronize()
        M = self.w["M"]
        worst = 0.0
        for i, (kind, bp, ldb, ns, modes, cp, ldc, members) in enumerate(self.gargs):
            K = self.kinds[kind]
            rc = L.zest_gemm_group(ctypes.c_void_p(self.ah[kind].data_ptr()), K, M, K, len(members), bp, ldb, ns,
                                   modes, cp, ldc, ctypes.c_void_p(self.err.data_ptr()), self.sp)
            if rc:
                raise Z.ZestError(L.zest_last_error().decode())
            for name, N, _ in members:
                ref = torch.empty((M, N), dtype=torch.float32, device="cuda")
                gather_slabs(self.out[name], ref, self.world, N)
                got = self.full[name] if self.how == "peer16" else self.mc[name][0]
                worst = max(worst, float((ref - got).abs().max().item()))
        return worst

    def step(self, events=None):
        from zest_b200.shard import gather_slabs
        torch, Z, L = self.torch, self.Z, self.Z.lib()
        M = self.w["M"]
        for kind, K in self.kinds.items():
            rc = L.zest_pack_activations(ctypes.c_void_p(self.x[kind].data_ptr()), M, K, K, self.ah[kind].shape[0],
                                         None, ctypes.c_void_p(self.ah[kind].data_ptr()), K, self.sp)
            if rc:
                raise Z.ZestError(L.zest_last_error().decode())
        for i, (kind, bp, ldb, ns, modes, cp, ldc, members) in enumerate(self.gargs):
            K = self.kinds[kind]
            if events is not None:
                events[i][0].record(self.stream)
            if self.mc:
                rc = L.zest_gemm_segs(ctypes.c_void_p(self.ah[kind].data_ptr()), K, M, K, len(members), self.msegs[i],
                                      ctypes.c_void_p(self.err.data_ptr()), self.sp)
            else:
                rc = L.zest_gemm_group(ctypes.c_void_p(self.ah[kind].data_ptr()), K, M, K, len(members), bp, ldb,
                                       ns, modes, cp, ldc, ctypes.c_void_p(self.err.data_ptr()), self.sp)
            if events is not None:
                events[i][1].record(self.stream)
            if rc:
                raise Z.ZestError(L.zest_last_error().decode())
            if self.how == "peer16":
                # every rank's tiles of this launch are in every bf16 copy once
                # the fence completes; the widening overlaps the next launch
                import torch.distributed as dist
                self.comm.wait_stream(self.stream)
                with torch.cuda.stream(self.comm):
                    dist.all_reduce(self.tick)
                    cs = ctypes.c_void_p(self.comm.cuda_stream)
                    for name, N, _ in members:
                        if L.zest_widen_bf16(ctypes.c_void_p(self.mc[name][0].data_ptr()), M * N,
                                             ctypes.c_void_p(self.full[name].data_ptr()), cs):
                            raise Z.ZestError(L.zest_last_error().decode())
            elif self.gather and not self.mc:
                # the gather of this launch's slabs overlaps the next launch
                self.comm.wait_stream(self.stream)
                with torch.cuda.stream(self.comm):
                    for name, N, _ in members:
                        gather_slabs(self.out[name], self.full[name], self.world, N, wire=torch.bfloat16)
        if self.how == "peer16":
            import torch.distributed as dist
            self.stream.wait_stream(self.comm)
            dist.all_reduce(self.tick)  # every rank has widened its copies before the next step writes them
        elif self.mc:
            import torch.distributed as dist
            dist.all_reduce(self.tick)  # every rank's tiles are in every copy before the step ends
        elif self.gather:
            self.stream.wait_stream(self.comm)

    def timed(self, steps: int, warmup: int, local: int, clocked: bool = True):
        """(ms per step on this rank, per-launch ms, clock summary)."""
        import torch.distributed as dist
        from zest_b200.shard import any_rank
        torch, Z = self.torch, self.Z
        for _ in range(warmup):
            self.step()
        torch.cuda.synchronize()
        if any_rank(int(self.err.item()) != 0):  # every rank stops together
            raise Z.ZestError(f"device error bits {int(self.err.item()):#x} during warm-up (this rank)")
        mk = lambda: [torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)]
        ev = [[mk() for _ in self.groups] for _ in range(steps)]
        t0, t1 = mk()
        if self.world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        with ClockSampler(local) as clocks:
            t0.record(self.stream)
            for s_ in range(steps):
                self.step(ev[s_])
            t1.record(self.stream)
            torch.cuda.synchronize()
        if self.world > 1:
            dist.barrier()
        if any_rank(int(self.err.item()) != 0):
            raise Z.ZestError(f"device error bits {int(self.err.item()):#x} in the timed region (this rank)")
        ms = t0.elapsed_time(t1) / steps
        gemm_ms = [sum(ev[s_][i][0].elapsed_time(ev[s_][i][1]) for s_ in range(steps)) / steps
                   for i in range(len(self.groups))]
        return ms, gemm_ms, clocks.summary()


def max_over_ranks(v: float, world: int, torch) -> float:
    if world == 1:
        return v
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


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
    mode = layer_mode(world, args.mode)
    nshard = world > 1 and mode != "tokens"
    gather = nshard and mode == "nshard"
    raws = {name: weight_raw(qt, name, N, K, threads) for name, N, K, _ in w["proj"]}

    layer = LayerStep(w, raws, world, rank, nshard, gather, Z, torch, args.gather)
    ms, gemm_ms, clocks = layer.timed(args.steps, args.warmup, local)
    ms_max = max_over_ranks(ms, world, torch)
    groups, slabs = layer.groups, layer.slabs
    launches = layer.launches
    gather_desc = layer.gather_desc()
    if layer.mc:
        from zest_b200.shard import any_rank
        worst = layer.check_gather()
        if any_rank(not worst == 0.0):
            raise Z.ZestError(f"the epilogue's gather differs from NCCL's by {worst} (this rank)")
    del layer
    torch.cuda.empty_cache()

    # N > 1 with the N-shard: the token split's figure beside it (every rank
    # its own chunk through whole weights, no collective)
    tokens_leg = None
    if nshard:
        tl = LayerStep(w, raws, world, rank, False, False, Z, torch)
        t_ms, _, _ = tl.timed(args.steps, args.warmup, local)
        del tl
        torch.cuda.empty_cache()
        t_max = max_over_ranks(t_ms, world, torch)
        tokens_leg = {"value": world * flops(w) / (t_max * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": t_max,
                      "parallelism": f"tokens{world}: each GPU its own {M}-token chunk through whole weights, "
                                     "no collective (weak scaling)"}

    total_flops = flops(w) * (1 if nshard else world)  # the whole job: all ranks' tokens
    local_gemm_flops = sum(2.0 * M * slabs[name][1] * K for name, N, K, _ in w["proj"])
    peaks = measured_peaks()
    peak, peak_kind = choose_peak(peaks, ms * args.steps * 1e-3, clocks)
    gemm_total_ms = sum(gemm_ms)
    # the roofline's launch: the one with the most work (gate+up at C2)
    gflops = [sum(2.0 * M * slabs[name][1] * K for name, _, K in members) for _, members in groups]
    names = ["+".join(name for name, _, _ in members) for _, members in groups]
    top = max(range(len(groups)), key=lambda i: gflops[i])
    top_desc = " + ".join(f"{name} {M}x{slabs[name][1]}x{K}" for name, _, K in groups[top][1])
    achieved = gflops[top] / (gemm_ms[top] * 1e-3) / 1e12
    traffic = profiled_traffic(args.workload, names[top]) if world == 1 else None
    algo_bytes = sum(2.0 * M * K + 2.0 * slabs[name][1] * K + 4.0 * M * slabs[name][1]
                     for name, _, K in groups[top][1])
    algo_bytes -= 2.0 * M * groups[top][1][0][2] * (len(groups[top][1]) - 1)  # one A per launch

    # --- end to end through the C ABI, host buffers: each rank its own chunk ----
    if world > 1:
        dist.barrier()
    e2e = e2e_run(args, w, raws, Z, torch)
    if world > 1:
        e2e["ms_per_step"] = max_over_ranks(e2e["ms_per_step"], world, torch)
        e2e["value"] = world * flops(w) / (e2e["ms_per_step"] * 1e-3) / 1e12
        e2e["tokens_per_s"] = world * M / (e2e["ms_per_step"] * 1e-3)
        e2e["h2d_bytes_per_step"] *= world
        e2e["d2h_bytes_per_step"] *= world
        e2e["api"] += f"; each of the {world} GPUs its own {M}-token chunk"

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline(w, raws)

    if rank == 0:
        value = total_flops / (ms_max * 1e-3) / 1e12
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max, "higher_is_better": True,
            "scaling": layer_scaling(world, args.mode), "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic",
            "config": layer_config(w, args.workload, world, args.mode),
            "tokens_per_s": M * (1 if nshard else world) / (ms_max * 1e-3),
            "pct_of_bf16_peak": 100.0 * value / (world * peak),
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak, "traffic": traffic,
                         "traffic_vs_algorithmic": traffic / algo_bytes if traffic else None,
                         "algorithmic_bytes": algo_bytes,
                         "kernel": "k3 gemm_bf16_tc_pair_kernel<256> (whole tiles; the stream-K instance where "
                                   "zest_plan_gemm says so)",
                         "launch": f"{top_desc}: {gflops[top] / 1e9:.1f} GFLOP, {gemm_ms[top] * 1e3:.1f} us avg",
                         "peak_kind": peak_kind, "peak_burst": peaks["tflops_burst"],
                         "peak_sustained": peaks["tflops_sustained"],
                         "per_launch": {n: {"us": round(t * 1e3, 1), "tflops": round(f / (t * 1e-3) / 1e12, 1),
                                            "frac": round(f / (t * 1e-3) / 1e12 / peak, 3)}
                                        for n, t, f in zip(names, gemm_ms, gflops)},
                         "all_gemms": {"ms_per_step": gemm_total_ms,
                                       "tflops": local_gemm_flops / (gemm_total_ms * 1e-3) / 1e12,
                                       "frac": local_gemm_flops / (gemm_total_ms * 1e-3) / 1e12 / peak}},
            "gpu_launches": args.steps * launches,
            "clocks": clocks,
        }
        if nshard:
            line["gather"] = gather_desc
        if tokens_leg:
            line["tokens_mode"] = tokens_leg
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
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1 and "GGML_ZEST_HOST_THREADS" not in os.environ:
        # the ranks share the host's cores: each service's widening pool takes its share
        os.environ["GGML_ZEST_HOST_THREADS"] = str(max(1, (os.cpu_count() or 1) // world))
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
        # every group of the step in flight at once, one slot each (the
        # reference's streams, xdna_exec_piece): one group's copy in overlaps
        # another's copy out and the host's widening of a third's results
        slots = []
        for i, (kind, members) in enumerate(groups):
            if len(slots) == Z.SLOTS:
                npu.wait_group(slots.pop(0))
            slot = i % Z.SLOTS
            npu.submit_group(slot, [keys[name] for name, _, _ in members], xs[kind].data_ptr(), M,
                             [ys[name].data_ptr() for name, _, _ in members], on_device=False)
            slots.append(slot)
        for slot in slots:
            npu.wait_group(slot)

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
    # results that hold bf16 values (GGML_XDNA_OUT16=1, the default) cross
    # PCIe as bf16 and are widened to f32 on host threads inside the call
    # (GGML_ZEST_WIRE16=0 sends the f32)
    out_bytes = 2 if os.environ.get("GGML_ZEST_WIRE16", "1") != "0" and \
        os.environ.get("GGML_XDNA_OUT16", "1") != "0" else 4
    d2h = sum(sum(M * N * out_bytes for _, N, _ in members) + 4 for _, members in groups)
    npu.close()
    return {"value": flops(w) / (ms * 1e-3) / 1e12, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "ms_per_step": ms, "tokens_per_s": M / (ms * 1e-3), "steps": steps,
            "api": "zest_submit_group / zest_wait_group (include/zest_b200.h), host buffers, one group call per "
                   "shared input, all of a step's groups in flight at once; f32 in, f32 out (bf16-rounded results "
                   "cross PCIe as bf16 and are widened on the host)"}


# ---------------------------------------------------------------------------
# C3: a whole Qwen3-4B-shaped prefill
# ---------------------------------------------------------------------------

MODEL = dict(layers=36, hidden=2560, heads=32, kv_heads=8, head_dim=128, ffn=9728, vocab=151936, prompt=8296,
             chunk=2048, min_batch=1024, eps=1e-6, rope_base=1e6, n_ctx_orig=40960, published_tok_s=380.4)


def q4_k_m_six(i: int, n: int) -> bool:
    """Layers whose attn_v and ffn_down take Q6_K in this Q4_K_M-style mix:
    the first and last eighth of the layers and every third one between."""
    return i < n // 8 or i >= n - n // 8 or (i - n // 8) % 3 == 2


class Prefill:
    """A Qwen3-shaped model's prompt prefill in chunks. The chunks the gate
    claims (>= min_batch tokens) run every claimed op through the C ABI:
    RMS_NORM and its MUL, the q/k/v group, the per-head q/k norms, ROPE
    (NeoX), o, the residual ADDs, the fused gate/up SwiGLU and down.
    Attention, the embedding lookup, the LM head (last token) and chunks
    below the floor run as torch ops, as the sibling backend would."""

    def __init__(self, c: dict, seed: int = 0, threads: int = 1):
        import torch

        import zest_b200 as Z
        self.c, self.Z, self.torch = c, Z, torch
        self.L = Z.lib()
        nL, H, hq, hk, hd, F = c["layers"], c["hidden"], c["heads"], c["kv_heads"], c["head_dim"], c["ffn"]
        self.dims = (nL, H, hq, hk, hd, F)
        self.shapes = {"q": (hq * hd, H), "k": (hk * hd, H), "v": (hk * hd, H), "o": (H, hq * hd), "gate": (F, H),
                       "up": (F, H), "down": (H, F)}
        # seeded raw bytes: one Q4_K set, and a Q6_K set for v and down;
        # every layer converted (K1) into its own device copy
        raw4 = {n: torch.from_numpy(weight_raw(Q4_K, n, N, K, threads)).cuda() for n, (N, K) in self.shapes.items()}
        raw6 = {n: torch.from_numpy(weight_raw(Q6_K, n + "6", *self.shapes[n], threads)).cuda()
                for n in ("v", "down")}
        g = torch.Generator("cuda").manual_seed(4242 + seed)
        self.layers = []
        torch.cuda.synchronize()
        t = time.perf_counter()
        for i in range(nL):
            six = q4_k_m_six(i, nL)
            d = {}
            for n in ("q", "k", "v", "o", "down"):
                qt, raw = (Q6_K, raw6[n]) if six and n in raw6 else (Q4_K, raw4[n])
                _, d[n] = Z.convert_weight(qt, raw, *self.shapes[n], want_bytes=False)
            _, d["gate_up"] = Z.convert_gate_up(Q4_K, raw4["gate"], raw4["up"], F, H, want_bytes=False)
            for n, dim in (("attn_norm", H), ("ffn_norm", H), ("q_norm", hd), ("k_norm", hd)):
                d[n] = torch.rand(dim, device="cuda", generator=g) + 0.5
            self.layers.append(d)
        torch.cuda.synchronize()
        self.load_s = time.perf_counter() - t
        self.emb = (torch.randn(c["vocab"], H, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
        self.lm_head = (torch.randn(c["vocab"], H, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
        self.out_norm = torch.rand(H, device="cuda", generator=g) + 0.5
        # per-chunk buffers, the cache, the rope table
        P, CH = c["prompt"], c["chunk"]
        self.chunks = [(p0, min(CH, P - p0)) for p0 in range(0, P, CH)]
        Tm = max(t for _, t in self.chunks)
        mp = Z.pad_to(Tm, 128)
        f32 = lambda *s: torch.empty(*s, dtype=torch.float32, device="cuda")
        self.x, self.xm = f32(Tm, H), f32(Tm, H)
        self.q, self.k, self.v = f32(Tm, hq * hd), f32(Tm, hk * hd), f32(Tm, hk * hd)
        self.qn, self.kn, self.qr, self.kr = f32(Tm, hq * hd), f32(Tm, hk * hd), f32(Tm, hq * hd), f32(Tm, hk * hd)
        self.att, self.o_out, self.s, self.d_out = f32(Tm, hq * hd), f32(Tm, H), f32(Tm, F), f32(Tm, H)
        self.q16 = torch.empty((Tm, hq * hd), dtype=torch.bfloat16, device="cuda")
        self.fused = True
        self.a_h = {K: torch.empty((mp, K), dtype=torch.int16, device="cuda") for K in (H, hq * hd, F)}
        self.page = 64
        Pp = Z.pad_to(P, self.page)  # the cache in 64-token pages for the paged attention kernel
        self.kc = torch.zeros((nL, Pp, hk, hd), dtype=torch.bfloat16, device="cuda")
        self.vc = torch.zeros((nL, Pp, hk, hd), dtype=torch.bfloat16, device="cuda")
        self.att16 = torch.empty((Tm, hq, hd), dtype=torch.bfloat16, device="cuda")
        self.attn_impl = self._pick_attention()
        self.table = f32(Tm, hd)
        self.pos = torch.arange(P, dtype=torch.int32, device="cuda")
        self.par = (ctypes.c_float * 6)(c["rope_base"], 1.0, 0.0, 1.0, 32.0, 1.0)
        self.err = torch.zeros(1, dtype=torch.int32, device="cuda")
        self.ids = torch.empty(P, dtype=torch.int64, device="cuda")
        self.logits = torch.empty(c["vocab"], dtype=torch.float32).pin_memory()
        self.gi = None

    # --- the C ABI calls ------------------------------------------------------
    def _ok(self, rc):
        if rc:
            raise self.Z.ZestError(self.L.zest_last_error().decode())

    @staticmethod
    def _p(t):
        return ctypes.c_void_p(t.data_ptr())

    def _sp(self):
        return ctypes.c_void_p(self.torch.cuda.current_stream().cuda_stream)

    def _gemm(self, K, T, bs, ns, modes, outs, ev):
        n, p = len(bs), self._p
        if ev is not None:
            ev[0].record()
        self._ok(self.L.zest_gemm_group(p(self.a_h[K]), K, T, K, n, (ctypes.c_void_p * n)(*[p(b) for b in bs]),
                                        (ctypes.c_int64 * n)(*[K] * n), (ctypes.c_int64 * n)(*ns),
                                        (ctypes.c_int * n)(*modes), (ctypes.c_void_p * n)(*[p(o) for o in outs]),
                                        (ctypes.c_int64 * n)(*[o.shape[1] for o in outs]), p(self.err), self._sp()))
        if ev is not None:
            ev[1].record()

    def _pack(self, src, T, K):
        self._ok(self.L.zest_pack_activations(self._p(src), T, K, K, self.Z.pad_to(T, 128), None,
                                              self._p(self.a_h[K]), K, self._sp()))

    def _norm(self, src, rows, d, wt, dst):
        self._ok(self.L.zest_rms_norm(self._p(src), rows, d, ctypes.c_float(self.c["eps"]), self._p(dst),
                                      self._sp()))
        self._ok(self.L.zest_mul_row(self._p(dst), self._p(wt), rows, d, self._p(dst), self._sp()))

    def _pick_attention(self) -> str:
        """Attention outside the path: flashinfer's trtllm-gen paged context
        kernel for chunks that attend over earlier ones (2-3x torch SDPA
        there on B200), torch SDPA for a chunk on its own. Checked once
        against SDPA; SDPA everywhere if the library is missing or differs."""
        torch = self.torch
        try:
            from flashinfer.prefill import trtllm_batch_context_with_kv_cache
            nL, H, hq, hk, hd, F = self.dims
            Pp = self.kc.shape[1]
            self._trt = trtllm_batch_context_with_kv_cache
            self._ws = torch.zeros(128 << 20, dtype=torch.uint8, device="cuda")
            self._blocks = torch.arange(Pp // self.page, dtype=torch.int32, device="cuda")[None]
            self._meta = {}
            for p0, T in self.chunks:
                S = p0 + T
                self._meta[p0] = (torch.tensor([S], dtype=torch.int32, device="cuda"),
                                  torch.tensor([0, T], dtype=torch.int32, device="cuda"),
                                  torch.tensor([0, S], dtype=torch.int32, device="cuda"))
            # check on the second chunk's shape with random keys
            p0, T = self.chunks[1] if len(self.chunks) > 1 else self.chunks[0]
            g = torch.Generator("cuda").manual_seed(7)
            self.kc[0, :p0 + T] = torch.randn(p0 + T, hk, hd, device="cuda", generator=g).to(torch.bfloat16)
            self.vc[0, :p0 + T] = torch.randn(p0 + T, hk, hd, device="cuda", generator=g).to(torch.bfloat16)
            q = torch.randn(T, hq, hd, device="cuda", generator=g).to(torch.bfloat16)
            got = self._attend_paged(0, p0, T, q).float()
            want = self._attend(q, self.kc[0, :p0 + T], self.vc[0, :p0 + T]).float()
            torch.cuda.synchronize()
            if ((got - want).abs().max() / want.abs().max()).item() > 2e-2:
                return "torch SDPA (trtllm-gen disagreed)"
            return "flashinfer trtllm-gen paged context attention; torch SDPA for the first chunk"
        except Exception as e:  # the library is optional: SDPA is the stock path
            self._trt = None
            return f"torch SDPA ({type(e).__name__} from flashinfer)"

    def _attend_paged(self, li, p0, T, q):
        """A chunk's queries q [T, hq, hd] over layer li's cache up to the chunk's end."""
        nL, H, hq, hk, hd, F = self.dims
        Pp, ps = self.kc.shape[1], self.page
        seq, cq, ckv = self._meta[p0]
        out = self.att16[:T]
        self._trt(q, (self.kc[li].view(Pp // ps, ps, hk, hd), self.vc[li].view(Pp // ps, ps, hk, hd)), self._ws,
                  self._blocks, seq, T, p0 + T, 1.0 / math.sqrt(hd), 1.0, 1, cq, ckv, out=out, kv_layout="NHD",
                  causal=True)
        return out

    def _attention(self, li, p0, T, q):
        """Layer li's attention for a chunk (queries q [T, hq, hd] bf16)."""
        if self._trt is not None and p0 > 0:
            return self._attend_paged(li, p0, T, q)
        return self._attend(q, self.kc[li, :p0 + T], self.vc[li, :p0 + T])

    def _attend(self, q, k, v):
        """Causal attention of a chunk's queries over the cache up to the
        chunk's end (row i sees every position up to its own): torch SDPA
        with a lower-right causal bias and grouped kv heads."""
        import torch.nn.functional as Fnn
        from torch.nn.attention.bias import causal_lower_right
        T, S = q.shape[0], k.shape[0]
        qh, kh, vh = (t.transpose(0, 1).unsqueeze(0) for t in (q, k, v))
        return Fnn.scaled_dot_product_attention(qh, kh, vh, attn_mask=causal_lower_right(T, S),
                                                enable_gqa=True)[0].transpose(0, 1)

    def capture(self):
        """One CUDA graph per claimed chunk (each chunk attends over its own
        number of cached keys), replayed by run(graphs=True): a chunk's
        36 x 20 launches then cost the host nothing."""
        torch = self.torch
        claimed = [(ci, p0, T) for ci, (p0, T) in enumerate(self.chunks) if T >= self.c["min_batch"]]
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _, p0, T in claimed:
                self.claimed_chunk(p0, T)
        torch.cuda.current_stream().wait_stream(side)
        self.graphs = {}
        for ci, p0, T in claimed:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self.claimed_chunk(p0, T)
            self.graphs[ci] = g
        # the unclaimed tail and the LM head as one more graph (torch ops only)
        self.tail_graph = None
        p0, T = self.chunks[-1]
        if T < self.c["min_batch"]:
            self.head_out = torch.empty(self.c["vocab"], dtype=torch.float32, device="cuda")
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                self._tail_and_head(p0, T)
            torch.cuda.current_stream().wait_stream(side)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self._tail_and_head(p0, T)
            self.tail_graph = g
        torch.cuda.synchronize()

    def _tail_and_head(self, p0, T):
        torch = self.torch
        last = self.unclaimed_chunk(p0, T)[-1:]
        h = last * torch.rsqrt(last.pow(2).mean(-1, keepdim=True) + self.c["eps"]) * self.out_norm
        self.head_out.copy_((h.to(torch.bfloat16) @ self.lm_head.T).float()[0])

    def _segs(self, K, T, items, ev):
        """One zest_gemm_segs launch: items = [(weight, N, mode, c, residual, a_next)]."""
        Z, p = self.Z, self._p
        n = len(items)
        arr = (Z.GemmSeg * n)(*[Z.GemmSeg(b.data_ptr(), K, N, mode, c.data_ptr() if c is not None else None,
                                          c.shape[1] if c is not None else 0,
                                          r.data_ptr() if r is not None else None, r.shape[1] if r is not None else 0,
                                          a.data_ptr() if a is not None else None, a.shape[1] if a is not None else 0)
                                for b, N, mode, c, r, a in items])
        if ev is not None:
            ev[0].record()
        self._ok(self.L.zest_gemm_segs(p(self.a_h[K]), K, T, K, n, arr, p(self.err), self._sp()))
        if ev is not None:
            ev[1].record()

    def claimed_chunk(self, p0, T, evs=None, att_ev=None):
        """Every op of a claimed chunk through the C ABI (attention aside);
        the chunk's hidden state ends in self.x[:T]. With self.fused the
        block executor's ops ride in the kernels beside them (the norm in
        the pack, q/k norm with rope, the residual ADDs in the GEMM epilogue,
        SwiGLU writing the down projection's operand): 8 launches of ours a
        layer instead of 20."""
        if self.fused:
            return self._claimed_chunk_fused(p0, T, evs, att_ev)
        torch, Z, L, p, sp = self.torch, self.Z, self.L, self._p, self._sp()
        nL, H, hq, hk, hd, F = self.dims
        B = Z.MODE_BF16
        x, xm, q, k, v = self.x, self.xm, self.q, self.k, self.v
        x[:T] = self.emb[self.ids[p0:p0 + T]].float()
        self._ok(L.zest_rope_table(p(self.pos[p0:]), T, hd, self.c["n_ctx_orig"], self.par, None, p(self.table), sp))
        for li, d in enumerate(self.layers):
            ev = evs[li] if evs is not None else [None] * 4
            self._norm(x, T, H, d["attn_norm"], xm)
            self._pack(xm, T, H)
            self._gemm(H, T, [d["q"], d["k"], d["v"]], [hq * hd, hk * hd, hk * hd], [B, B, B], [q, k, v], ev[0])
            self._norm(q, T * hq, hd, d["q_norm"], self.qn)
            self._norm(k, T * hk, hd, d["k_norm"], self.kn)
            self._ok(L.zest_rope(p(self.qn), T, hq, hd, hd, Z.ROPE_NEOX, p(self.table), p(self.qr), sp))
            self._ok(L.zest_rope(p(self.kn), T, hk, hd, hd, Z.ROPE_NEOX, p(self.table), p(self.kr), sp))
            self.kc[li, p0:p0 + T] = self.kr[:T].view(T, hk, hd)
            self.vc[li, p0:p0 + T] = v[:T].view(T, hk, hd)
            if att_ev is not None:
                att_ev[li][0].record()
            self.att[:T] = self._attend(self.qr[:T].view(T, hq, hd).to(torch.bfloat16), self.kc[li, :p0 + T],
                                        self.vc[li, :p0 + T]).reshape(T, hq * hd)
            if att_ev is not None:
                att_ev[li][1].record()
            self._pack(self.att, T, hq * hd)
            self._gemm(hq * hd, T, [d["o"]], [H], [B], [self.o_out], ev[1])
            self._ok(L.zest_add(p(x), p(self.o_out), 0, T, H, p(x), sp))
            self._norm(x, T, H, d["ffn_norm"], xm)
            self._pack(xm, T, H)
            self._gemm(H, T, [d["gate_up"]], [d["gate_up"].shape[0]], [Z.MODE_SWIGLU], [self.s], ev[2])
            self._pack(self.s, T, F)
            self._gemm(F, T, [d["down"]], [H], [B], [self.d_out], ev[3])
            self._ok(L.zest_add(p(x), p(self.d_out), 0, T, H, p(x), sp))
        return x[:T]

    LAUNCHES_PER_LAYER = 20  # our kernels per layer of a claimed chunk, unfused
    LAUNCHES_PER_LAYER_FUSED = 8

    def _claimed_chunk_fused(self, p0, T, evs, att_ev):
        torch, Z, L, p, sp = self.torch, self.Z, self.L, self._p, self._sp()
        nL, H, hq, hk, hd, F = self.dims
        B, eps, mp = Z.MODE_BF16, ctypes.c_float(self.c["eps"]), Z.pad_to(T, 128)
        x = self.x
        x[:T] = self.emb[self.ids[p0:p0 + T]].float()
        self._ok(L.zest_rope_table(p(self.pos[p0:]), T, hd, self.c["n_ctx_orig"], self.par, None, p(self.table), sp))
        for li, d in enumerate(self.layers):
            ev = evs[li] if evs is not None else [None] * 4
            self._ok(L.zest_pack_rms_norm(p(x), T, H, H, eps, p(d["attn_norm"]), None, 0, mp, p(self.a_h[H]), H, sp))
            self._segs(H, T, [(d["q"], hq * hd, B, self.q, None, None), (d["k"], hk * hd, B, self.k, None, None),
                              (d["v"], hk * hd, B, self.v, None, None)], ev[0])
            kc = self.kc[li, p0:p0 + T]
            self._ok(L.zest_norm_rope(p(self.q), T, hq, hd, eps, p(d["q_norm"]), hd, Z.ROPE_NEOX, p(self.table),
                                      None, p(self.q16), sp))
            self._ok(L.zest_norm_rope(p(self.k), T, hk, hd, eps, p(d["k_norm"]), hd, Z.ROPE_NEOX, p(self.table),
                                      None, p(kc), sp))
            self.vc[li, p0:p0 + T] = self.v[:T].view(T, hk, hd)
            if att_ev is not None:
                att_ev[li][0].record()
            self.att[:T] = self._attention(li, p0, T, self.q16[:T].view(T, hq, hd)).reshape(T, hq * hd)
            if att_ev is not None:
                att_ev[li][1].record()
            self._pack(self.att, T, hq * hd)
            self._segs(hq * hd, T, [(d["o"], H, B, x, x, None)], ev[1])
            self._ok(L.zest_pack_rms_norm(p(x), T, H, H, eps, p(d["ffn_norm"]), None, 0, mp, p(self.a_h[H]), H, sp))
            self._segs(H, T, [(d["gate_up"], d["gate_up"].shape[0], Z.MODE_SWIGLU, None, None, self.a_h[F])], ev[2])
            self._segs(F, T, [(d["down"], H, B, x, x, None)], ev[3])
        return x[:T]

    def unclaimed_chunk(self, p0, T):
        """A chunk below the gate's batch floor, as the sibling backend runs
        it: torch ops on the same bf16 weight copies."""
        torch = self.torch
        nL, H, hq, hk, hd, F = self.dims
        bf, eps = torch.bfloat16, self.c["eps"]
        rms = lambda t, wt: t * torch.rsqrt(t.pow(2).mean(-1, keepdim=True) + eps) * wt
        mm = lambda a, wt, n: (a.to(bf) @ wt.view(bf)[:n].T).float()
        inv = self.c["rope_base"] ** (-torch.arange(0, hd, 2, device="cuda", dtype=torch.float32) / hd)
        ang = self.pos[p0:p0 + T].float()[:, None] * inv[None]
        cos, sin = ang.cos()[:, None], ang.sin()[:, None]

        def rope(t):  # NeoX: the two halves of each head rotate together
            a, b = t[..., :hd // 2], t[..., hd // 2:]
            return torch.cat([a * cos - b * sin, a * sin + b * cos], -1)

        if self.gi is None:
            idx = torch.arange(F, device="cuda")
            self.gi = (idx // 8) * 16 + idx % 8  # gate columns of the interleaved copy; up = +8
        xt = self.emb[self.ids[p0:p0 + T]].float()
        for li, d in enumerate(self.layers):
            h = rms(xt, d["attn_norm"])
            qq = rope(rms(mm(h, d["q"], hq * hd).view(T, hq, hd), d["q_norm"]))
            kk = rope(rms(mm(h, d["k"], hk * hd).view(T, hk, hd), d["k_norm"]))
            self.kc[li, p0:p0 + T] = kk
            self.vc[li, p0:p0 + T] = mm(h, d["v"], hk * hd).view(T, hk, hd)
            a = self._attend(qq.to(bf), self.kc[li, :p0 + T], self.vc[li, :p0 + T]).reshape(T, hq * hd)
            xt = xt + mm(a, d["o"], H)
            gu = mm(rms(xt, d["ffn_norm"]), d["gate_up"], d["gate_up"].shape[0])
            xt = xt + mm(torch.nn.functional.silu(gu[:, self.gi]) * gu[:, self.gi + 8], d["down"], H)
        return xt

    def run(self, ids_host, evs=None, claim=True, graphs=False, att_evs=None, tail_ev=None):
        """One prefill: token ids (pinned host) in, last-token logits (pinned
        host) out. claim=False runs every chunk as an unclaimed one;
        graphs=True replays the captured claimed chunks (and the tail)."""
        torch = self.torch
        self.ids.copy_(ids_host, non_blocking=True)
        last = None
        if graphs and claim and self.tail_graph is not None:
            for ci in range(len(self.chunks) - 1):
                self.graphs[ci].replay()
            self.tail_graph.replay()
            self.logits.copy_(self.head_out, non_blocking=True)
            return self.logits
        for ci, (p0, T) in enumerate(self.chunks):
            if claim and T >= self.c["min_batch"]:
                if graphs:
                    self.graphs[ci].replay()
                    last = self.x[T - 1:T]
                else:
                    last = self.claimed_chunk(p0, T, evs[ci] if evs is not None else None,
                                              att_evs[ci] if att_evs is not None else None)[-1:]
            else:
                if tail_ev is not None:
                    tail_ev[0].record()
                last = self.unclaimed_chunk(p0, T)[-1:]
        h = last * torch.rsqrt(last.pow(2).mean(-1, keepdim=True) + self.c["eps"]) * self.out_norm
        self.logits.copy_((h.to(torch.bfloat16) @ self.lm_head.T).float()[0], non_blocking=True)
        if tail_ev is not None:
            tail_ev[1].record()
        return self.logits


def run_model(args, w: dict) -> None:
    """C3: prefill of an 8,296-token prompt through 36 Qwen3-4B-shaped layers
    in chunks of 2048 (Prefill); N>1: every GPU its own prompt."""
    import torch

    import zest_b200 as Z
    from zest_b200.shard import any_rank

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    c = MODEL
    threads = max(1, (os.cpu_count() or 1) // max(1, world))
    m = Prefill(c, seed=0, threads=threads)
    nL, H, hq, hk, hd, F = m.dims
    P, CH = c["prompt"], c["chunk"]
    ids_host = torch.randint(0, c["vocab"], (P,), generator=torch.Generator().manual_seed(1000 + rank),
                             dtype=torch.int64).pin_memory()
    steps = min(args.steps, 20)
    for _ in range(args.warmup):
        m.run(ids_host)
    torch.cuda.synchronize()
    if any_rank(int(m.err.item()) != 0):  # every rank stops together
        raise Z.ZestError(f"device error bits {int(m.err.item()):#x} during warm-up (this rank)")
    if not torch.isfinite(m.logits).all():
        raise Z.ZestError("non-finite logits")
    # eager prefills with events around every MUL_MAT launch and attention:
    # the per-launch figures and the breakdown (graphs cannot carry them)
    mk = lambda: [torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)]
    n_prof = 2
    evs = [[[[mk() for _ in range(4)] for _ in range(nL)] for _ in m.chunks] for _ in range(n_prof)]
    aevs = [[[mk() for _ in range(nL)] for _ in m.chunks] for _ in range(n_prof)]
    tevs = [mk() for _ in range(n_prof)]
    e0, e1 = mk()
    torch.cuda.synchronize()
    e0.record()
    for si in range(n_prof):
        m.run(ids_host, evs[si], att_evs=aevs[si], tail_ev=tevs[si])
    e1.record()
    torch.cuda.synchronize()
    eager_ms = e0.elapsed_time(e1) / n_prof
    # the timed prefills: claimed chunks replayed from CUDA graphs
    m.capture()
    for _ in range(2):
        m.run(ids_host, graphs=True)
    t0, t1 = mk()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        t0.record()
        for si in range(steps):
            m.run(ids_host, graphs=True)
        t1.record()
        torch.cuda.synchronize()
    if any_rank(int(m.err.item()) != 0):
        raise Z.ZestError(f"device error bits {int(m.err.item()):#x} in the timed region (this rank)")
    ms = t0.elapsed_time(t1) / steps
    t = torch.tensor([ms], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    # per claimed chunk: its MUL_MATs' time (four launches per layer)
    names = ["q+k+v", "o", "gate+up", "down"]
    claimed = [ci for ci, (_, T) in enumerate(m.chunks) if T >= c["min_batch"]]
    per_chunk, per_launch, att_ms = [], {n: 0.0 for n in names}, 0.0
    for ci in claimed:
        tot = 0.0
        for li in range(nL):
            for j in range(4):
                e = sum(evs[si][ci][li][j][0].elapsed_time(evs[si][ci][li][j][1]) for si in range(n_prof)) / n_prof
                tot += e
                per_launch[names[j]] += e / (nL * len(claimed))
            att_ms += sum(aevs[si][ci][li][0].elapsed_time(aevs[si][ci][li][1]) for si in range(n_prof)) / n_prof
        per_chunk.append(tot)
    tail_ms = sum(a.elapsed_time(b) for a, b in tevs) / n_prof if m.chunks[-1][1] < c["min_batch"] else 0.0
    per_token_fl = 2.0 * nL * sum(N * K for N, K in m.shapes.values())
    claimed_fl = per_token_fl * sum(m.chunks[ci][1] for ci in claimed)
    mm_ms = sum(per_chunk)
    down_fl = 2.0 * CH * H * F
    achieved = down_fl / (per_launch["down"] * 1e-3) / 1e12
    peaks = measured_peaks()
    clk = clocks.summary()
    peak, peak_kind = choose_peak(peaks, ms * steps * 1e-3, clk)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        lw = WORKLOADS["qwen3-4b-layer"]
        cb = cpu_baseline(lw, {n: weight_raw(Q4_K, n, N, K, threads) for n, N, K, _ in lw["proj"]})
        cpu = {"value": cb["tokens_per_s"] / nL, "unit": "tok/s", "cores": cb["cores"], "kind": cb["kind"],
               "sample": cb["sample"] + "; the 36 layers' MUL_MATs only (attention and the other ops not counted), "
                                        "so an upper bound for the CPU path"}
    if rank == 0:
        value = world * P / (ms_max * 1e-3)
        n_six = sum(q4_k_m_six(i, nL) for i in range(nL))
        line = {
            "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": steps,
            "warmup": args.warmup, "ms_per_step": ms_max, "higher_is_better": True,
            "scaling": "weak" if world > 1 else "none", "vs_baseline": value / c["published_tok_s"],
            "dtype": "bf16", "data": "synthetic",
            "config": {"workload": args.workload, "desc": w["config"], "layers": nL, "prompt_tokens": P,
                       "chunks": [T for _, T in m.chunks],
                       "weights": f"Q4_K; Q6_K for attn_v and ffn_down on {n_six} of {nL} layers (first and last "
                                  "eighth, every third between). One seeded set of raw bytes per type, converted "
                                  "into every layer's own device copy",
                       "attention": m.attn_impl + " (outside the path)",
                       "graphs": "each claimed chunk, and the tail with the LM head, replayed from CUDA graphs",
                       "fused": "norm in the pack, q/k norm with rope, residual ADDs and SwiGLU's packed output in "
                                "the GEMM epilogues" if m.fused else "every op its own kernel",
                       "unclaimed": f"the {m.chunks[-1][1]}-token tail (< {c['min_batch']} tokens) in torch ops",
                       "parallelism": f"tokens{world} (each GPU its own prompt, no collective)" if world > 1
                       else "1 GPU",
                       "l2": "no flush: a chunk streams 7.3 GB of weight copies (> 126 MB L2)"},
            "vs_baseline_of": f"{c['published_tok_s']} tok/s: the reference's NPU + iGPU prefill of an 8,296-token "
                              "prompt on Qwen3-4B Q4_K_M",
            "tokens_per_s": value,
            "mul_mat": {"ms_per_prefill": mm_ms, "tflops": claimed_fl / (mm_ms * 1e-3) / 1e12,
                        "ms_per_claimed_chunk": [round(x, 3) for x in per_chunk],
                        "share_of_prefill": mm_ms / ms_max,
                        "per_launch_us": {n: round(v * 1e3, 1) for n, v in per_launch.items()}},
            "breakdown_ms": {"prefill_graphs": ms_max, "prefill_eager": eager_ms, "mul_mat": mm_ms,
                             "attention_claimed_chunks": att_ms, "tail_and_head_eager": tail_ms,
                             "rest": eager_ms - mm_ms - att_ms - tail_ms,
                             "note": "eager prefills with events around each launch; the rest is the small ops, "
                                     "packs, cache writes, the unclaimed tail, the LM head and the host gaps"},
            "load": {"weight_conversion_s": m.load_s, "layers": nL},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak,
                         "unit": "TFLOP/s", "frac": achieved / peak, "traffic": None,
                         "kernel": "k3 gemm_bf16_tc_pair_kernel",
                         "launch": f"down {CH}x{H}x{F}: {down_fl / 1e9:.1f} GFLOP, "
                                   f"{per_launch['down'] * 1e3:.1f} us avg over layers and chunks",
                         "peak_kind": peak_kind},
            "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": P * 8 * world,
                    "d2h_bytes_per_step": c["vocab"] * 4 * world,
                    "api": "token ids in, last-token logits out; claimed ops through include/zest_b200.h"},
            "gpu_launches": steps * len(claimed) * (1 + nL * (Prefill.LAUNCHES_PER_LAYER_FUSED if m.fused
                                                              else Prefill.LAUNCHES_PER_LAYER)),
            "steps_note": f"{steps} timed prefills of {P} tokens (--steps capped at 20 for this workload)",
            "clocks": clk,
        }
        if cpu:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


# ---------------------------------------------------------------------------
# tensor-parallel layer (--mode tp)
# ---------------------------------------------------------------------------

TP_KSHARDED = ("o", "down")  # inputs the block leaves split by columns: attention heads, the SwiGLU


def run_tp(args, w: dict) -> None:
    """The layer's MUL_MATs as one tensor-parallel block on N GPUs: q/k/v and
    gate/up N-sharded (each rank its slab of output columns, left where they
    are, as a head-parallel attention and the FFN's SwiGLU consume them);
    o and down K-sharded (each rank multiplies its column slab of their input
    by the same slab of the weight), and their partial products summed by
    one NCCL all-reduce per row chunk, issued as each chunk's GEMMs finish so
    it overlaps the next chunk's. Strong scaling: the job is one layer of M
    tokens however many GPUs share it."""
    import torch
    import torch.distributed as dist

    import zest_b200 as Z
    from zest_b200.shard import all_reduce_rows, any_rank, shard_cols, shard_rows

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    from datetime import timedelta
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    threads = max(1, (os.cpu_count() or 1) // max(1, world))
    if w["qtype"] == IQ3_S:
        Z.load_iq3s_grid()
    M, qt = w["M"], w["qtype"]
    kinds = {}
    for name, N, K, kind in w["proj"]:
        kinds.setdefault(kind, K)
    ksh = {kind for kind in kinds if kind in TP_KSHARDED}

    # weights: N-sharded projections convert their row slab; K-sharded ones
    # convert whole and multiply the column slab of the bf16 copy in place
    bh, n_of, kcols = {}, {}, {}
    for name, N, K, kind in w["proj"]:
        raw = torch.from_numpy(weight_raw(qt, name, N, K, threads)).cuda()
        if kind in ksh:
            _, bh[name] = Z.convert_weight(qt, raw, N, K, want_bytes=False)
            n_of[name] = N
            kcols[kind] = shard_cols(K, world, rank)
        else:
            row0, n = shard_rows(N, world, rank)
            _, bh[name] = Z.convert_weight(qt, raw, N, K, row0=row0, n_rows=n, want_bytes=False)
            n_of[name] = n
        del raw
    for kind in kinds:
        kcols.setdefault(kind, (0, kinds[kind]))
    torch.cuda.synchronize()

    gen = torch.Generator("cuda").manual_seed(1234)  # the same layer input on every rank
    x, ah = {}, {}
    mp = Z.pad_to(M, 128)
    for kind, K in kinds.items():
        x[kind] = torch.randn(M, K, device="cuda", generator=gen)
        ah[kind] = torch.empty((mp, kcols[kind][1]), dtype=torch.int16, device="cuda")
    out = {name: torch.zeros((M, max(1, n_of[name])), dtype=torch.float32, device="cuda")
           for name, N, K, kind in w["proj"]}
    # the K-sharded partials summed by the GEMM itself: its epilogue adds them
    # into a symmetric buffer bound to an NVLink multicast object (every rank
    # a copy), the NVSwitch doing the reduction, when the box supports it
    mc = {}
    reduce_how = "NCCL all-reduce"
    if world > 1 and args.tp_reduce == "multicast":
        try:
            import torch.distributed._symmetric_memory as symm_mem
            for name, N, K, kind in w["proj"]:
                if kind in ksh:
                    t = symm_mem.empty((M, N), dtype=torch.float32, device="cuda")
                    hdl = symm_mem.rendezvous(t, dist.group.WORLD)
                    if not hdl.multicast_ptr:
                        raise RuntimeError("no multicast support")
                    out[name] = t
                    mc[name] = (hdl, int(hdl.multicast_ptr))
            reduce_how = "multimem.red into an NVLink multicast buffer from the GEMM epilogue"
        except Exception as e:  # fall back to NCCL
            mc = {}
            reduce_how = f"NCCL all-reduce (multicast unavailable: {type(e).__name__}: {e})"
        # the ranks take the same collective steps: if any rank has no
        # multicast buffers, every rank sums through NCCL
        if any_rank(not mc):
            if mc:
                reduce_how = "NCCL all-reduce (multicast unavailable on another rank)"
            mc = {}
            for name, N, K, kind in w["proj"]:
                if kind in ksh:
                    out[name] = torch.zeros((M, max(1, n_of[name])), dtype=torch.float32, device="cuda")
    tick = torch.zeros(1, dtype=torch.float32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream()
    L = Z.lib()
    sp = ctypes.c_void_p(stream.cuda_stream)
    groups = launch_groups(w)
    CH = Z.pad_to(max(128, M // (1 if mc else args.tp_chunks)), 128)
    chunks = [(r0, min(CH, M - r0)) for r0 in range(0, M, CH)]

    def ok(rc):
        if rc:
            raise Z.ZestError(L.zest_last_error().decode())

    def step(events=None):
        works = []
        if mc:
            # zero this rank's copies, and no rank adds before every rank has
            # (a one-float all-reduce as the group's stream-ordered fence)
            for name in mc:
                out[name].zero_()
            dist.all_reduce(tick)
        for ci, (r0, m) in enumerate(chunks):
            for kind, K in kinds.items():
                k0, k = kcols[kind]
                ok(L.zest_pack_activations(ctypes.c_void_p(x[kind][r0:].data_ptr() + 4 * k0), m, k, K,
                                           Z.pad_to(m, 128), None, ctypes.c_void_p(ah[kind][r0:].data_ptr()), k,
                                           sp))
            for gi, (kind, members) in enumerate(groups):
                k0, k = kcols[kind]
                n = len(members)
                partial = kind in ksh
                if events is not None:
                    events[gi][ci][0].record(stream)
                if partial and mc:
                    segs = (Z.GemmSeg * n)(*[Z.GemmSeg(bh[nm].data_ptr() + 2 * k0, K, n_of[nm], Z.MODE_F32, None,
                                                       out[nm].shape[1], None, 0, None, 0,
                                                       mc[nm][1] + 4 * r0 * out[nm].shape[1])
                                             for nm, _, _ in members])
                    ok(L.zest_gemm_segs(ctypes.c_void_p(ah[kind][r0:].data_ptr()), k, m, k, n, segs,
                                        ctypes.c_void_p(err.data_ptr()), sp))
                else:
                    ok(L.zest_gemm_group(
                        ctypes.c_void_p(ah[kind][r0:].data_ptr()), k, m, k, n,
                        (ctypes.c_void_p * n)(*[bh[nm].data_ptr() + 2 * k0 for nm, _, _ in members]),
                        (ctypes.c_int64 * n)(*[K for _, _, K in members]),
                        (ctypes.c_int64 * n)(*[n_of[nm] for nm, _, _ in members]),
                        (ctypes.c_int * n)(*[Z.MODE_F32 if partial else Z.MODE_BF16] * n),
                        (ctypes.c_void_p * n)(*[out[nm][r0:].data_ptr() for nm, _, _ in members]),
                        (ctypes.c_int64 * n)(*[out[nm].shape[1] for nm, _, _ in members]),
                        ctypes.c_void_p(err.data_ptr()), sp))
                if events is not None:
                    events[gi][ci][1].record(stream)
                if partial and world > 1 and not mc:
                    for nm, _, _ in members:
                        works.append(all_reduce_rows(out[nm], r0, m))
        for wk in works:
            wk.wait()  # the stream waits for the reductions, not the host
        if mc:
            dist.all_reduce(tick)  # every rank's reductions are in before anyone reads the sums

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if any_rank(int(err.item()) != 0):  # every rank stops together
        raise Z.ZestError(f"device error bits {int(err.item()):#x} during warm-up (this rank)")
    check = None
    if mc:
        # the multicast sums against the same partials summed by NCCL
        worst = 0.0
        for kind in ksh:
            k0, k = kcols[kind]
            for nm, N, K in dict(groups)[kind]:
                part = torch.empty((M, n_of[nm]), dtype=torch.float32, device="cuda")
                ok(L.zest_gemm(ctypes.c_void_p(ah[kind].data_ptr()), k, ctypes.c_void_p(bh[nm].data_ptr() + 2 * k0),
                               K, M, n_of[nm], k, Z.MODE_F32, ctypes.c_void_p(part.data_ptr()), n_of[nm],
                               ctypes.c_void_p(err.data_ptr()), sp))
                dist.all_reduce(part)
                worst = max(worst, ((out[nm] - part).abs().max() / part.abs().max()).item())
        check = {"max_rel_diff_vs_nccl": worst}
        if any_rank(not worst <= 1e-5):
            raise Z.ZestError(f"multicast sums differ from NCCL's by {worst} (this rank)")
    mk = lambda: [torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)]
    ev = [[[mk() for _ in chunks] for _ in groups] for _ in range(args.steps)]
    t0, t1 = mk()
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
    if any_rank(int(err.item()) != 0):
        raise Z.ZestError(f"device error bits {int(err.item()):#x} in the timed region (this rank)")
    ms = t0.elapsed_time(t1) / args.steps
    t = torch.tensor([ms], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    gemm_ms = [sum(ev[s][gi][ci][0].elapsed_time(ev[s][gi][ci][1]) for s in range(args.steps)
                   for ci in range(len(chunks))) / args.steps for gi in range(len(groups))]
    peaks = measured_peaks()
    clk = clocks.summary()
    peak, peak_kind = choose_peak(peaks, ms * args.steps * 1e-3, clk)
    if rank == 0:
        value = flops(w) / (ms_max * 1e-3) / 1e12
        names = ["+".join(nm for nm, _, _ in members) for _, members in groups]
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max, "higher_is_better": True,
            "scaling": "strong" if world > 1 else "none", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic",
            "config": {"workload": args.workload, "desc": w["config"], "M": M, "weights": QNAME[qt],
                       "parallelism": f"tp{world}: q/k/v and gate/up N-sharded, o/down K-sharded, their partials "
                                      f"summed by {reduce_how}" + (f", per {CH}-row chunk" if len(chunks) > 1 else ""),
                       "outputs": "N-sharded projections: bf16-rounded slabs left on their rank; K-sharded: the "
                                  "f32 sums of the partials on every rank",
                       "global_tokens_per_step": M},
            "tokens_per_s": M / (ms_max * 1e-3),
            "pct_of_bf16_peak": 100.0 * value / (world * peak), "peak_kind": peak_kind,
            "per_rank_gemm_us": {nm: round(v * 1e3, 1) for nm, v in zip(names, gemm_ms)},
            "reduce_check": check,
            "gpu_launches": args.steps * len(chunks) * (len(kinds) + len(groups)),
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        # every rank is done with the multicast buffers before any releases them
        torch.cuda.synchronize()
        dist.barrier()
        mc.clear()
        out.clear()
        torch.cuda.synchronize()
        dist.barrier()
        dist.destroy_process_group()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default=DEFAULT)
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--mode", choices=["tokens", "nshard", "nshard-nogather", "tp"], default=None,
                    help="N>1: N-slabs of every weight with (nshard, the default) or without the NCCL all-gather "
                         "of the output slabs, each GPU its own token chunk (tokens, no collective), or the layer "
                         "as one tensor-parallel block (tp: o/down K-sharded, one all-reduce per row chunk)")
    ap.add_argument("--gather", choices=["peer16", "peer", "multicast", "nccl"], default="peer16",
                    help="nshard: the output all-gather from the GEMM epilogue, by TMA stores into every GPU's "
                         "copy in bf16 then widened (peer16, the default) or in f32 (peer), or by multimem.st "
                         "through NVLink multicast, or by NCCL (also where a rank has no symmetric memory)")
    ap.add_argument("--tp-chunks", type=int, default=1, help="tp with NCCL: row chunks whose all-reduce overlaps the next")
    ap.add_argument("--tp-reduce", choices=["multicast", "nccl"], default="nccl",
                    help="tp: K-sharded partials summed by NCCL, or in the GEMM epilogue through NVLink multicast "
                         "(multimem.red; exact, faster at 2 GPUs, slower at 8)")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)  # at least 3 untimed warm-up steps
    w = WORKLOADS[args.workload]
    if args.impl == "reference":
        run_reference(args, w)
    elif w.get("model"):
        run_model(args, w)
    elif args.mode == "tp":
        run_tp(args, w)
    else:
        run_ours(args, w)


if __name__ == "__main__":
    main()
