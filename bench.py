"""MaxSim scoring benchmark on B200 (one process per GPU; torchrun for N > 1).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c2] [--extra c1,c3,c4,c5]
                    [--impl ours|reference]

Headline workload ("c2"): batched shared-docs scoring,
Q [100, 32, 128] fp16 against D [100000, 300, 128] fp16 (7.68 GB), docs
sharded across ranks (strong scaling: the 100000 docs are split N ways) and
the per-rank score blocks combined with one NCCL all-gather. Inputs are
synthetic: N(0, 1) entries, every token row L2-normalised, seeded per rank.
At N = 1 the other BASELINE configurations (c1, c3, c4, c5) are measured in
the same run and reported under "configs" of the same JSON line.

A step = one pass of the hot path over the whole batch: the fused sm_100a
MaxSim kernel on every rank, then the all-gather. Inputs (7.68 GB) exceed the
126 MB L2, so no flush is needed between steps (configs whose documents are
smaller than 4x L2 rotate over enough copies of them that no step finds its
batch in L2). `value` is query-doc scores (or docs) per second of the
whole job, device-timed with CUDA events, max over ranks. `e2e` repeats the
step through the public API from pinned host buffers: host->device copy of Q
and the rank's document shard, the kernel, the all-gather, and the
device->host copy of the scores, all inside the timed region.

After each timed region a seeded sample of documents of the timed output is
checked against the CPU oracle (`parity`), and the reference's own Triton
kernels (installed unmodified under baseline/_ref) are timed on the same
inputs (`reference_gpu`).

`--impl reference` times the reference's own CPU path instead (its torch
maxsim_naive from baseline/_ref on every host thread; the numpy restatement
in oracle/ when the reference is not installed), on a bounded sample of the
same workload per step; rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "docs scored/sec per B200 and 8-GPU box; % of HBM or tensor-core roofline"
L2_BYTES = 126 * 1024 * 1024

# name: (description, Nq, Lq, B, Ld, d, kind)
CONFIGS = {
    "c1": ("textual single-query MaxSim Q[32,128] x D[1000,300,128] fp16", 1, 32, 1000, 300, 128, "single"),
    "c2": ("batched shared-docs MaxSim Q[100,32,128] x D[100000,300,128] fp16, doc-sharded",
           100, 32, 100000, 300, 128, "batched"),
    "c3": ("visual late-interaction Q[16,1024,128] x D[4000,1024,128] fp16", 16, 1024, 4000, 1024, 128,
           "batched"),
    "c4": ("INT8 fused-dequant MaxSim Q[32,128] x u8 D[200000,300,128] + scale/min", 1, 32, 200000, 300,
           128, "int8"),
    "c4fp8": ("FP8 e4m3 documents (per-token fp32 scale) MaxSim Q[32,128] x e4m3 D[200000,300,128]", 1, 32,
              200000, 300, 128, "fp8"),
    "c5": ("varlen train fwd+bwd Q[64,64,256] x D[4096,1024,256], lengths U[32,1024]", 64, 64, 4096, 1024,
           256, "train"),
}


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        j = json.loads(p.read_text())
        return {"hbm_gbs": j["hbm_gbs"], "tflops": j["bf16_tflops"],
                "tflops_sustained": j.get("bf16_tflops_sustained"), "source": "measured"}
    return {"hbm_gbs": 6650.0, "tflops": 1590.0, "tflops_sustained": 1400.0, "source": "fallback"}


def load_traffic(cfg: str):
    p = ROOT / "profiles" / "traffic.json"
    if p.exists():
        return json.loads(p.read_text()).get(cfg)
    return None


# ---------------------------------------------------------------------------
# distributed plumbing
# ---------------------------------------------------------------------------

def dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}: launch N>1 with torchrun")
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return rank, world, torch.device("cuda", torch.cuda.current_device())


def physical_gpu_index(local: int) -> int:
    """nvidia-smi index of CUDA device `local` (honours CUDA_VISIBLE_DEVICES)."""
    vis = os.environ.get("CUDA_VISIBLE_DEVICES", "").strip()
    if vis:
        parts = [p.strip() for p in vis.split(",") if p.strip()]
        if local < len(parts) and parts[local].isdigit():
            return int(parts[local])
    return local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x: float, world: int, device) -> float:
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------------------
# clocks sampler (nvidia-smi during the timed region)
# ---------------------------------------------------------------------------

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        loaded = [s for s in sm if smax and s > 0.5 * smax] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
# synthetic inputs
# ---------------------------------------------------------------------------

def synth(shape, seed: int, device, chunk_rows: int = 4096) -> torch.Tensor:
    """N(0, 1) entries, last-axis rows L2-normalised, fp16, built in chunks."""
    g = torch.Generator(device=device).manual_seed(seed)
    out = torch.empty(shape, dtype=torch.float16, device=device)
    flat = out.view(-1, shape[-1])
    rows = flat.shape[0]
    step = max(1, chunk_rows * 300)
    for r0 in range(0, rows, step):
        n = min(step, rows - r0)
        x = torch.randn(n, shape[-1], generator=g, device=device, dtype=torch.float32)
        flat[r0:r0 + n] = F.normalize(x, dim=-1).half()
    return out


def shard(B: int, rank: int, world: int):
    lo = B * rank // world
    hi = B * (rank + 1) // world
    return lo, hi


# ---------------------------------------------------------------------------
# our implementation
# ---------------------------------------------------------------------------

class Workload:
    """Inputs of one configuration on this rank (documents of its shard)."""

    def __init__(self, args, cfg, rank, world, dev):
        import flash_maxsim_b200 as fm
        desc, Nq, Lq, B, Ld, d, kind = CONFIGS[cfg]
        if args.docs:
            # smaller document count, for ncu captures (same per-doc shapes)
            B = args.docs
            desc += f" [B overridden to {B}]"
        for name in ("nq", "lq", "ld", "dim"):
            v = getattr(args, "shape_" + name)
            if v:
                Nq, Lq, Ld, d = [v if n == name else o for n, o in zip(("nq", "lq", "ld", "dim"), (Nq, Lq, Ld, d))]
                desc += f" [{name} overridden to {v}]"
        self.cfg, self.desc, self.kind = cfg, desc, kind
        self.Nq, self.Lq, self.B, self.Ld, self.d = Nq, Lq, B, Ld, d
        lo, hi = shard(B, rank, world)
        self.lo, self.Bl = lo, hi - lo
        self.Q = synth((Nq, Lq, d) if kind not in ("single", "int8", "fp8") else (Lq, d), 1, dev)
        D = synth((self.Bl, Ld, d), 1000 + rank, dev)
        self.lengths = None
        if kind == "train":
            gl = torch.Generator(device=dev).manual_seed(77 + rank)
            self.lengths = torch.randint(32, Ld + 1, (self.Bl,), generator=gl, device=dev, dtype=torch.int32)
        self.Du8 = self.sc = self.mn = None
        if kind == "int8":
            self.Du8, self.sc, self.mn = fm.quantize_int8(D)
            del D
            D = None
            torch.cuda.empty_cache()
        if kind == "fp8":
            self.Du8, self.sc = fm.quantize_fp8(D)
            self.mn = torch.empty(0, device=dev)
            del D
            D = None
            torch.cuda.empty_cache()
        self.D = D
        self.grad = None
        if kind == "train":
            self.grad = torch.randn(Nq, self.Bl, device=dev, generator=torch.Generator(device=dev).manual_seed(5))
        if kind == "int8":
            self.in_bytes = self.Du8.numel() + self.sc.numel() * 2 + self.mn.numel() * 2
        elif kind == "fp8":
            self.in_bytes = self.Du8.numel() + self.sc.numel() * 4
        else:
            self.in_bytes = D.numel() * 2
        # inputs smaller than 4x L2: rotate over enough copies of the documents
        # that every step reads its batch from HBM (no step finds it in L2)
        self.n_copies = 1
        if self.in_bytes < 4 * L2_BYTES:
            self.n_copies = -(-4 * L2_BYTES // self.in_bytes)
        self.D_copies = [D] + [D.clone() for _ in range(self.n_copies - 1)] if D is not None else [None]
        self.U_copies = ([(self.Du8, self.sc, self.mn)] +
                         [(self.Du8.clone(), self.sc.clone(), self.mn.clone()) for _ in range(self.n_copies - 1)]
                         if self.Du8 is not None else [None])

    def call(self, i):
        """One public-API scoring call on document copy i."""
        import flash_maxsim_b200 as fm
        if self.kind == "single":
            return fm.flash_maxsim(self.Q, self.D_copies[i])
        if self.kind == "batched":
            return fm.flash_maxsim_batched(self.Q, self.D_copies[i])
        u, s_, m_ = self.U_copies[i]
        if self.kind == "fp8":
            return fm.flash_maxsim_fp8(self.Q, u, s_)
        return fm.flash_maxsim_int8(self.Q, u, s_, m_)

    def units(self):
        return (self.Nq * self.B) if self.kind in ("batched", "train") else self.B

    def unit_name(self):
        return "query-doc scores/s" if self.kind in ("batched", "train") else "docs/s"


def parity(w: Workload, out, dev) -> dict:
    """Check a seeded sample of documents of the timed launch's output (copy 0
    for rotated inputs) against the CPU oracle, after the timed region."""
    from oracle import sampled_check as SC
    import flash_maxsim_b200 as fm
    npy = lambda t: t.detach().cpu().numpy()  # noqa: E731
    t0 = time.perf_counter()
    if w.kind in ("single", "batched"):
        n = 24 if w.Lq * w.Ld > 100000 else 256
        idx = SC.sample_docs(w.Bl, n, seed=11)
        it = torch.from_numpy(idx).to(dev)
        Q3 = w.Q if w.Q.dim() == 3 else w.Q.unsqueeze(0)
        got = out if out.dim() == 2 else out.unsqueeze(0)
        res = SC.check_scores(npy(Q3), npy(w.D_copies[0][it]), npy(got[:, it]))
    elif w.kind == "int8":
        idx = SC.sample_docs(w.Bl, 256, seed=11)
        it = torch.from_numpy(idx).to(dev)
        res = SC.check_int8(npy(w.Q), npy(w.Du8[it]), npy(w.sc[it]), npy(w.mn[it]), npy(out[it]))
    elif w.kind == "fp8":
        idx = SC.sample_docs(w.Bl, 256, seed=11)
        it = torch.from_numpy(idx).to(dev)
        res = SC.check_fp8(npy(w.Q), npy(w.Du8[it].view(torch.float8_e4m3fn).float()), npy(w.sc[it]), npy(out[it]))
    else:
        from flash_maxsim_b200 import api
        Qg = w.Q.detach().clone().requires_grad_(True)
        Dg = w.D.detach().clone().requires_grad_(True)
        s = fm.flash_maxsim_train(Qg, Dg, w.lengths)
        s.backward(w.grad)
        _, am = api._fwd(w.Q, w.D, w.lengths, w.Nq, w.Bl, w.Lq, w.Ld, True, True)
        am = am.view(w.Nq, w.Bl, w.Lq)
        idx = SC.sample_docs(w.Bl, 16, seed=11)
        it = torch.from_numpy(idx).to(dev)
        rows = [(0, 0), (w.Nq // 2, w.Lq - 1), (w.Nq - 1, w.Lq // 3)]
        Dsel = []
        ar = torch.arange(w.Bl, device=dev)
        for n, q in rows:
            a = am[n, :, q].long()
            sel = w.D[ar, a.clamp(min=0)].float()
            Dsel.append(npy(torch.where((a >= 0)[:, None], sel, torch.zeros_like(sel))))
        sd = s.detach()
        g_eff = torch.where(torch.isfinite(sd), w.grad, torch.zeros_like(w.grad))
        res = SC.check_train(npy(w.Q), npy(w.D[it]), npy(w.lengths[it]), npy(w.grad[:, it]), npy(sd[:, it]),
                             npy(am[:, it]), npy(Dg.grad[it].float()), rows,
                             np.stack([npy(Qg.grad[n, q].float()) for n, q in rows]), (npy(g_eff), Dsel))
        res = {k: v for k, v in res.items() if k != "parts"} | {
            "parts": {k: v["ok"] for k, v in res["parts"].items()}}
    res["docs_sampled"] = int(len(idx))
    res["seconds"] = round(time.perf_counter() - t0, 1)
    res["oracle"] = "oracle/maxsim_oracle.py (numpy restatement of maxsim_naive, pinned to reference golden vectors)"
    return res


def run_config(args, cfg, rank, world, dev, headline: bool) -> dict:
    import flash_maxsim_b200 as fm
    from flash_maxsim_b200 import sharded

    peaks = load_peaks()
    torch.manual_seed(0)
    w = Workload(args, cfg, rank, world, dev)
    kind, Nq, Lq, B, Ld, d, Bl = w.kind, w.Nq, w.Lq, w.B, w.Ld, w.d, w.Bl
    stream = torch.cuda.current_stream(dev)

    # Scoring calls are captured once per document copy in a CUDA graph and
    # replayed, so short launches are not limited by Python dispatch; the
    # training step (autograd) is launched eagerly.
    graphs, graph_out = [], []
    if kind != "train" and not args.no_graph:
        side = torch.cuda.Stream(dev)
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            for i in range(w.n_copies):
                w.call(i)
        stream.wait_stream(side)
        torch.cuda.synchronize(dev)
        for i in range(w.n_copies):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                graph_out.append(w.call(i))
            graphs.append(g)
        torch.cuda.synchronize(dev)
    only_kernel = world == 1 and kind != "train"
    ev_pool = [torch.cuda.Event(enable_timing=True) for _ in range(2 * (args.steps + args.warmup))]
    step_idx = [0]

    def kernel_step():
        """The hot path once; returns (result, kernel start/end events)."""
        k = step_idx[0]
        step_idx[0] += 1
        i = k % w.n_copies
        e0, e1 = ev_pool[(2 * k) % len(ev_pool)], ev_pool[(2 * k + 1) % len(ev_pool)]
        if only_kernel:
            # the step is this one launch: the timed region's own events time it
            e0 = e1 = None
        if e0 is not None:
            e0.record(stream)
        if graphs:
            graphs[i].replay()
            out = graph_out[i]
        elif kind != "train":
            out = w.call(i)
        else:
            Qg = w.Q.detach().requires_grad_(True)
            Dg = w.D.detach().requires_grad_(True)
            s = fm.flash_maxsim_train(Qg, Dg, w.lengths)
            s.backward(w.grad)
            out = s.detach()
        if e1 is not None:
            e1.record(stream)
        return out, (e0, e1)

    def step():
        out, ev = kernel_step()
        if world > 1:
            out = sharded.all_gather_scores(out if out.dim() == 2 else out.unsqueeze(0), B)
        return out, ev

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    fm.check_status(dev)

    sampler = ClockSampler(physical_gpu_index(dev.index))
    sampler.start()
    barrier(world)
    torch.cuda.synchronize(dev)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    evs = []
    t0.record(stream)
    for _ in range(args.steps):
        _, ev = step()
        evs.append(ev)
    t1.record(stream)
    torch.cuda.synchronize(dev)
    barrier(world)
    clocks = sampler.stop()
    fm.check_status(dev)
    total_ms = max_over_ranks(t0.elapsed_time(t1), world, dev)
    if only_kernel:
        kern_avg_ms = total_ms / args.steps
    else:
        kern_ms = [a.elapsed_time(b) for a, b in evs]
        kern_avg_ms = max_over_ranks(sum(kern_ms) / len(kern_ms), world, dev)

    value = w.units() / (total_ms / 1e3 / args.steps)

    # roofline of the dominant kernel (per rank, per launch)
    flops = 2.0 * Nq * Lq * Ld * d * Bl
    if kind == "train":
        flops = 2.0 * Nq * Lq * float(w.lengths.sum().item()) * d
    if kind in ("single", "int8", "fp8"):
        alg_bytes = w.in_bytes + w.Q.numel() * 2 + Bl * 4
        achieved = alg_bytes / (kern_avg_ms / 1e3) / 1e9
        roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": round(achieved / peaks["hbm_gbs"], 4), "peak_source": peaks["source"],
                "algorithmic_bytes_per_launch": alg_bytes}
    else:
        achieved = flops / (kern_avg_ms / 1e3) / 1e12
        roof = {"bound": "tensor", "achieved": round(achieved, 1), "peak": peaks["tflops"],
                "unit": "TFLOP/s", "frac": round(achieved / peaks["tflops"], 4),
                "peak_source": peaks["source"] + " (burst bf16 cuBLAS; fp16 dense taken equal)",
                "algorithmic_flops_per_launch": flops,
                # the same against cuBLAS held for seconds under the 1 kW power cap
                "frac_of_sustained_peak": (round(achieved / peaks["tflops_sustained"], 4)
                                           if peaks.get("tflops_sustained") else None),
                "hbm_achieved_GBs": round(w.in_bytes / (kern_avg_ms / 1e3) / 1e9, 1)}
        if kind == "train":
            roof["note"] = ("step = forward with argmax + backward (dQ, dD); flops of the forward on "
                            "valid tokens over the whole step's time")
    tr = load_traffic(cfg)
    roof["traffic"] = tr.get("bytes_per_launch") if tr else None
    if tr:
        roof["traffic_source"] = tr.get("source")
    roof["kernel_ms"] = round(kern_avg_ms, 4)

    out_for_check = graph_out[0] if graphs else None
    if out_for_check is None and kind != "train":
        out_for_check = w.call(0)
    par = None
    if rank == 0 and not args.no_parity:
        par = parity(w, out_for_check, dev)

    # the same scoring with the per-query top-10 kept by the kernel (reranking)
    topk = None
    if kind in ("single", "batched") and world == 1 and not args.no_topk:
        topk = time_topk(args, w, dev, 10, out_for_check)

    # end to end through the public API from pinned host memory
    e2e = None if args.no_e2e else run_e2e(args, w, fm, sharded, world, dev)

    ref_gpu = None
    if rank == 0 and world == 1 and not args.no_ref_gpu:
        ref_gpu = reference_gpu(args, w, dev)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline(cfg, args.cpu_seconds if headline else min(args.cpu_seconds, 4.0))

    res = {
        "value": round(value, 1), "unit": w.unit_name(), "ms_per_step": round(total_ms / args.steps, 4),
        "config": {"workload": w.desc, "config": cfg, "Nq": Nq, "Lq": Lq, "B": B, "Ld": Ld, "d": d,
                   "docs_per_rank": Bl,
                   "parallelism": f"doc-shard x{world} + NCCL all-gather" if world > 1 else "single GPU",
                   "launch": "CUDA graph replay of the public API call" if graphs else "eager public API call",
                   "l2": "inputs larger than L2" if w.n_copies == 1 else
                   f"documents rotated over {w.n_copies} copies ({w.n_copies * w.in_bytes / 1e6:.0f} MB > 4x L2) "
                   "between steps"},
        "roofline": roof, "kernel_ms": round(kern_avg_ms, 4), "clocks": clocks, "parity": par,
        "e2e": e2e, "cpu_baseline": cpu, "reference_gpu": ref_gpu, "topk": topk,
        # this library's kernels per step: one scoring launch, or for training
        # the forward, dQ (+ its range reduction when the documents are split)
        # and dD
        "gpu_launches": args.steps * ((3 + (1 if fm._lib.lib.fm_maxsim_bwd_workspace_size(Nq, Bl, Lq, Ld, d) > 0 else 0))
                                      if kind == "train" else 1),
    }
    del w, graphs, graph_out, out_for_check
    torch.cuda.synchronize(dev)
    torch.cuda.empty_cache()
    return res


def time_topk(args, w: Workload, dev, k: int, full_out):
    """flash_maxsim(_batched)_topk on the same documents: device time per
    call (graph replay, documents rotated like the main step) and whether
    its ids are exactly the stable top-k of the full scores."""
    import flash_maxsim_b200 as fm

    def call(i):
        if w.kind == "single":
            return fm.flash_maxsim_topk(w.Q, w.D_copies[i], k)
        return fm.flash_maxsim_batched_topk(w.Q, w.D_copies[i], k)

    stream = torch.cuda.current_stream(dev)
    side = torch.cuda.Stream(dev)
    side.wait_stream(stream)
    with torch.cuda.stream(side):
        for i in range(w.n_copies):
            call(i)
    stream.wait_stream(side)
    torch.cuda.synchronize(dev)
    graphs, outs = [], []
    for i in range(w.n_copies):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            outs.append(call(i))
        graphs.append(g)
    for j in range(args.warmup):
        graphs[j % w.n_copies].replay()
    torch.cuda.synchronize(dev)
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for j in range(args.steps):
        graphs[j % w.n_copies].replay()
    b.record(stream)
    torch.cuda.synchronize(dev)
    fm.check_status(dev)
    ms = a.elapsed_time(b) / args.steps
    v, i = outs[0]
    full = full_out if full_out.dim() == 2 else full_out.unsqueeze(0)
    v2 = v if v.dim() == 2 else v.unsqueeze(0)
    i2 = i if i.dim() == 2 else i.unsqueeze(0)
    # stable order: score descending, then id ascending
    o1 = torch.argsort(full, dim=1, descending=True, stable=True)[:, :k]
    exact = bool(torch.equal(o1, i2) and torch.equal(torch.gather(full, 1, o1), v2))
    return {"k": k, "value": round(w.units() / (ms / 1e3), 1), "unit": w.unit_name(), "ms_per_step": round(ms, 4),
            "ids_equal_stable_topk_of_full_scores": exact,
            "launches_per_step": 2}


def run_e2e(args, w: Workload, fm, sharded, world, dev):
    """Same step through the public API, inputs from pinned host buffers."""
    kind = w.kind
    steps = max(2, min(args.steps, args.e2e_steps))
    hQ = w.Q.cpu().pin_memory()
    if kind == "int8":
        hD = [w.Du8.cpu().pin_memory(), w.sc.cpu().pin_memory(), w.mn.cpu().pin_memory()]
        dD = [torch.empty_like(w.Du8), torch.empty_like(w.sc), torch.empty_like(w.mn)]
    elif kind == "fp8":
        hD = [w.Du8.cpu().pin_memory(), w.sc.cpu().pin_memory()]
        dD = [torch.empty_like(w.Du8), torch.empty_like(w.sc)]
    else:
        hD = [w.D.cpu().pin_memory()]
        dD = [] if kind == "batched" else [torch.empty_like(w.D)]
    hL = w.lengths.cpu().pin_memory() if w.lengths is not None else None
    h2d = hQ.numel() * hQ.element_size() + sum(t.numel() * t.element_size() for t in hD)
    if hL is not None:
        h2d += hL.numel() * 4
    out_host = None
    d2h = 0

    def one():
        nonlocal out_host, d2h
        if kind == "batched":
            # the public host-corpus entry point: the documents cross PCIe in
            # pieces on a copy stream while the pieces already copied are scored
            out = fm.flash_maxsim_batched_from_host(hQ, hD[0], hL, device=dev)
        else:
            out = step_from_device_copies()
        if world > 1:
            out = sharded.all_gather_scores(out if out.dim() == 2 else out.unsqueeze(0), w.B)
        if out_host is None:
            out_host = torch.empty(out.shape, dtype=out.dtype, pin_memory=True)
            d2h = out.numel() * out.element_size()
        out_host.copy_(out, non_blocking=True)

    def step_from_device_copies():
        q = hQ.to(dev, non_blocking=True)
        for h, dd in zip(hD, dD):
            dd.copy_(h, non_blocking=True)
        ln = hL.to(dev, non_blocking=True) if hL is not None else None
        if kind == "single":
            out = fm.flash_maxsim(q, dD[0])
        elif kind == "int8":
            out = fm.flash_maxsim_int8(q, dD[0], dD[1], dD[2])
        elif kind == "fp8":
            out = fm.flash_maxsim_fp8(q, dD[0], dD[1])
        else:
            qg = q.requires_grad_(True)
            dg = dD[0].requires_grad_(True)
            s = fm.flash_maxsim_train(qg, dg, ln)
            s.backward(w.grad)
            out = s.detach()
            dD[0] = dg.detach()
        return out

    one()
    torch.cuda.synchronize(dev)
    barrier(world)
    stream = torch.cuda.current_stream(dev)
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(steps):
        one()
    b.record(stream)
    torch.cuda.synchronize(dev)
    ms = max_over_ranks(a.elapsed_time(b), world, dev) / steps
    return {"value": round(w.units() / (ms / 1e3), 1), "unit": w.unit_name(),
            "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h), "steps": steps,
            "ms_per_step": round(ms, 3)}


# ---------------------------------------------------------------------------
# the reference implementation (installed unmodified under baseline/_ref)
# ---------------------------------------------------------------------------

def reference_module():
    """The reference package from baseline/_ref, or None when it is absent or
    does not import."""
    p = ROOT / "baseline" / "_ref"
    if not (p / "flash_maxsim").exists():
        return None
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))
    try:
        import flash_maxsim
        return flash_maxsim
    except Exception:  # noqa: BLE001 (any import failure means "not available")
        return None


def reference_gpu(args, w: Workload, dev):
    """The reference's own Triton kernels on this GPU, same inputs, for
    comparison (median of a few launches after its autotuning)."""
    ref = reference_module()
    if ref is None:
        return {"unavailable": "reference package not installed under baseline/_ref"}
    if w.kind == "fp8":
        return {"unavailable": "the reference has no FP8 document format (its quantised path is INT8)"}
    if w.kind == "train":
        return {"unavailable": "the reference's training path takes one query and no doc_lengths "
                               "(flash_maxsim/flash_maxsim.py:253-291)"}
    # The reference kernels index documents with 32-bit offsets
    # (doc * stride, flash_maxsim/flash_maxsim.py:118-121,
    # flash_maxsim_quant.py:80-83): past 2**31 elements they address memory
    # outside the tensor (an illegal-address fault on this GPU at 100000
    # documents of 300 x 128). They only ever run on the largest leading
    # slice of documents whose offsets fit, and the throughput is per document.
    per_doc = w.Ld * w.d
    nb = min(w.Bl, (2 ** 31 - 1) // per_doc - 1)
    if nb < 1:
        return {"unavailable": "one document exceeds the reference kernels' 32-bit offsets"}
    try:
        D = w.D_copies[0][:nb] if w.D_copies[0] is not None else None
        if w.kind == "single":
            fn = lambda: ref.flash_maxsim(w.Q, D)  # noqa: E731
        elif w.kind == "batched":
            fn = lambda: ref.flash_maxsim_batched(w.Q, D)  # noqa: E731
        else:
            fn = lambda: ref.flash_maxsim_int8(w.Q, w.Du8[:nb], w.sc[:nb], w.mn[:nb])  # noqa: E731
        fn()
        fn()  # autotuning happens on the first calls
        torch.cuda.synchronize(dev)
        times = []
        for _ in range(3):
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record()
            out = fn()
            b.record()
            torch.cuda.synchronize(dev)
            times.append(a.elapsed_time(b))
        ms = statistics.median(times)
        ours = graph_out_first(w)
        same = None
        if ours is not None:
            ours = ours[..., :nb]
            o = out if out.dim() == ours.dim() else out.view_as(ours)
            same = float((o.float() - ours.float()).abs().max().item())
        units = w.units() * nb / w.Bl
        res = {"value": round(units / (ms / 1e3), 1), "unit": w.unit_name(), "ms_per_step": round(ms, 4),
               "impl": "reference Triton kernels (baseline/_ref, unmodified)", "docs": nb,
               "max_abs_diff_vs_ours": same}
        if nb < w.Bl:
            res["note"] = (f"first {nb} of {w.Bl} documents: the reference's 32-bit document offsets "
                           "overflow beyond them")
        return res
    except Exception as e:  # noqa: BLE001
        return {"unavailable": f"{type(e).__name__}: {str(e).splitlines()[0][:200]}"}


def graph_out_first(w: Workload):
    try:
        with torch.no_grad():
            return w.call(0)
    except Exception:  # noqa: BLE001
        return None


# ---------------------------------------------------------------------------
# CPU baseline (the reference's own CPU path, maxsim_naive, on the host cores)
# ---------------------------------------------------------------------------

def _cpu_sample_docs(kind, Lq, Ld, d) -> int:
    # a sample whose one pass is well under a second on a many-core host
    work = Lq * Ld * d
    return max(8, min(256, int(2.5e9 // work)))


def cpu_baseline(cfg: str, seconds: float):
    """The reference's maxsim_naive (torch, fp32, baseline/_ref) on a bounded
    sample of the workload with every host thread, or, if the reference does
    not import, the numpy restatement in oracle/; returns units per second.
    Training samples run the forward and the autograd backward."""
    from oracle import maxsim_oracle as O
    desc, Nq, Lq, B, Ld, d, kind = CONFIGS[cfg]
    n_docs = _cpu_sample_docs(kind, Lq, Ld, d)
    nq = 1 if kind in ("single", "int8", "fp8") else min(Nq, 4)
    Q, D = O.seeded_inputs(123, (nq, Lq, d), (n_docs, Ld, d))
    lens = None
    if kind == "train":
        lens = np.random.default_rng(5).integers(32, Ld + 1, n_docs).astype(np.int32)
    if kind == "int8":
        u8, s, m = O.quantize_int8(D)
        D = O.dequantize_int8(u8, s, m)
    if kind == "fp8":
        D = O.dequantize_fp8(*O.quantize_fp8(D))
    threads = os.cpu_count() or 1
    ref = reference_module()
    old_threads = torch.get_num_threads()
    if ref is not None:
        torch.set_num_threads(threads)
        Qt = torch.from_numpy(np.asarray(Q, dtype=np.float32))
        Dt = torch.from_numpy(np.asarray(D, dtype=np.float32))
        Lt = torch.from_numpy(lens) if lens is not None else None
        g = torch.randn(n_docs, generator=torch.Generator().manual_seed(1))

        def one_pass():
            for n in range(nq):
                if kind == "train":
                    q = Qt[n].clone().requires_grad_(True)
                    dd = Dt.clone().requires_grad_(True)
                    s = ref.maxsim_naive(q, dd, Lt)
                    (s * g).sum().backward()
                else:
                    ref.maxsim_naive(Qt[n], Dt)
        what = ("the reference's maxsim_naive (torch fp32 einsum, baseline/_ref)"
                + (" forward + autograd backward" if kind == "train" else ""))
        used = torch.get_num_threads()
        kind_s = "reference"
    else:
        from threadpoolctl import threadpool_limits

        def one_pass():
            with threadpool_limits(limits=threads):
                for n in range(nq):
                    O.maxsim(Q[n], D, lens)
        what = "numpy fp32 restatement of maxsim_naive (oracle/maxsim_oracle.py; reference not installed)"
        used = threads
        kind_s = "port"
    try:
        t0 = time.perf_counter()
        done = 0
        while True:
            one_pass()
            done += 1
            el = time.perf_counter() - t0
            if el >= seconds:
                break
    finally:
        torch.set_num_threads(old_threads)
    units = done * n_docs * (nq if kind in ("batched", "train") else 1)
    unit_name = "query-doc scores/s" if kind in ("batched", "train") else "docs/s"
    return {"value": round(units / el, 1), "unit": unit_name, "cores": int(used), "kind": kind_s,
            "torch_threads": int(used) if ref is not None else None, "os_cpu_count": os.cpu_count(),
            "sample": f"{nq} queries x {n_docs} docs of the {cfg} shapes, repeated for {el:.1f} s ({what})"}


def run_reference(args, cfg):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    desc, Nq, Lq, B, Ld, d, kind = CONFIGS[cfg]
    per_step = max(0.2, min(args.cpu_seconds, 120.0 / max(1, args.steps + args.warmup)))
    for _ in range(args.warmup):
        cpu_baseline(cfg, per_step / 2)
    vals = [cpu_baseline(cfg, per_step) for _ in range(args.steps)]
    v = statistics.median(x["value"] for x in vals)
    base = vals[0]
    line = {
        "metric": METRIC, "impl": "reference", "value": v, "unit": base["unit"], "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic N(0,1), rows L2-normalised, seeded",
        "ms_per_step": round(per_step * 1e3, 1),
        "config": {"workload": desc, "config": cfg, "Nq": Nq, "Lq": Lq, "B": B, "Ld": Ld, "d": d},
        "cpu_baseline": {k: base[k] for k in ("unit", "cores", "kind", "sample", "torch_threads", "os_cpu_count")}
        | {"value": v},
        "e2e": {"value": v, "unit": base["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_ours(args):
    rank, world, dev = dist_setup(args.gpus)
    head = run_config(args, args.config, rank, world, dev, headline=True)
    extras = {}
    if world == 1 and args.extra:
        for c in [c.strip() for c in args.extra.split(",") if c.strip()]:
            if c != args.config:
                extras[c] = run_config(args, c, rank, world, dev, headline=False)
    if rank == 0:
        line = {
            "metric": METRIC, "value": head["value"], "unit": head["unit"], "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": head["ms_per_step"],
            "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f16 (fp32 accumulate)",
            "data": "synthetic N(0,1), rows L2-normalised, seeded",
            "config": head["config"], "roofline": head["roofline"], "cpu_baseline": head["cpu_baseline"],
            "e2e": head["e2e"], "gpu_launches": head["gpu_launches"], "clocks": head["clocks"],
            "parity": head["parity"], "reference_gpu": head["reference_gpu"], "topk": head["topk"],
        }
        if extras:
            line["configs"] = extras
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", default="c2", choices=sorted(CONFIGS), help="headline configuration")
    ap.add_argument("--extra", default="c1,c3,c4,c4fp8,c5",
                    help="further configurations measured in the same run at N=1 (empty: none)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-parity", action="store_true")
    ap.add_argument("--no-topk", action="store_true", help="skip timing the top-k variant")
    ap.add_argument("--no-ref-gpu", action="store_true", help="skip timing the reference's Triton kernels")
    ap.add_argument("--no-graph", action="store_true", help="launch every step eagerly (no CUDA graph)")
    for name in ("nq", "lq", "ld", "dim"):
        ap.add_argument(f"--shape-{name}", type=int, default=0, help="override a shape (tuning)")
    ap.add_argument("--docs", type=int, default=0, help="override B (profiling captures)")
    args = ap.parse_args()
    if args.warmup < 3:
        print("warning: fewer than 3 warm-up steps", file=sys.stderr)
    if args.impl == "reference":
        run_reference(args, args.config)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
