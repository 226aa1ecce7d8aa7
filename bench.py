"""Throughput of the fused exact KV patch on the Llama-3-8B-shaped workload.

One step = one pass of the exact/zeroth-order patch route over a full cache: pack the
rank-16 k/v LoRA factors of 32 layers, then patch 64 sequences x 4096 tokens x 32 layers
(8,388,608 token-layers) from fp8-e4m3 stored activations (per-token scale, RMSNorm
folded in) into bf16 paged K/V (block 16, permuted block table), RoPE on K.

    python bench.py [--gpus N --steps K --warmup W]          # this implementation
    python bench.py --impl reference ...                       # CPU reference arm
    python bench.py --workload smollm2-exact ...               # exact route, SmolLM2-135M shape
    python bench.py --workload rl-dense ...                    # dense-dW (RL step) route
    python bench.py --workload multi-lora-kivi ...             # int4 KIVI subspace route

The rl-dense workload is one GPU's share of the Llama-3-70B-shaped RL step (10 of 80
layers, d=8192, 8 KV heads x 128, 16 seqs x 8192 tokens, bf16 X, full-rank dW_K / dW_V at
||dW||/||W|| = 1e-3): one tensor-core GEMM launch of 44 TFLOP per step with RoPE and the
paged read-add-write fused; its roofline is the measured sustained bf16 GEMM rate.

Under torchrun (N>1) every rank patches its own request shard of the same size (weak
scaling; no data-path collective).  Rank 0 prints one JSON line.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "patched token·layers/s (Llama-8B shape, rank-16 k/v LoRA)"
UNIT = "token·layers/s"
BYTES_PER_UNIT = 4096 + 4 + 4 + 4096 + 4096  # X fp8 + scale + sum of squares + K read/write + V read/write
WORKLOAD = ("Llama-3-8B-shaped exact patch: 32 layers, d=4096, 8 KV heads x 128, 64 seqs x 4096 tokens, "
            "rank-16 k/v LoRA (rel. norm 1e-2), fp8-e4m3 stored X + per-token scale, RMSNorm folded, "
            "RoPE (theta 5e5), bf16 paged KV block 16")


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="llama8b-exact",
                    choices=["llama8b-exact", "smollm2-exact", "rl-dense", "multi-lora-kivi", "analytic"])
    ap.add_argument("--adapters", type=int, default=8)
    ap.add_argument("--layers", type=int, default=None)
    ap.add_argument("--seqs", type=int, default=None)
    ap.add_argument("--seq-len", type=int, default=None)
    ap.add_argument("--e2e-seqs", type=int, default=4)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    return ap.parse_args()


class Geo:
    """The exact-route workload being measured (rebound by --workload)."""
    d_model, n_kv, hd, rank, bs, eps, rope_theta = 4096, 8, 128, 16, 16, 1e-5, 500000.0
    layers, seqs, seq_len = 32, 64, 4096
    x_torch, x_kind = torch.float8_e4m3fn, "e4m3"


class SmolGeo(Geo):
    """SmolLM2-135M shape: 30 layers, d=576, 3 KV heads x 64, rank-8 k/v LoRA, fp16 stored X."""
    d_model, n_kv, hd, rank, bs, eps, rope_theta = 576, 3, 64, 8, 16, 1e-5, 10000.0
    layers, seqs, seq_len = 30, 32, 2048
    x_torch, x_kind = torch.float16, "f16"


SMOL_METRIC = "patched token·layers/s (SmolLM2-135M shape, rank-8 k/v LoRA)"
SMOL_BYTES_PER_UNIT = 1152 + 4 + 4 + 768 + 768  # X f16 + row scale + sum of squares + K read/write + V read/write
SMOL_WORKLOAD = ("SmolLM2-135M-shaped exact patch: 30 layers, d=576, 3 KV heads x 64, 32 seqs x 2048 tokens, "
                 "rank-8 k/v LoRA (rel. norm 1e-2), f16 stored X + power-of-two row scale, RMSNorm folded, "
                 "RoPE (theta 1e4), bf16 paged KV block 16")


class DenseGeo:
    """One GPU's share (10 of 80 layers) of the Llama-3-70B-shaped RL step."""
    layers, seqs, seq_len, d_model, n_kv, hd, bs, rope_theta = 10, 16, 8192, 8192, 8, 128, 16, 500000.0


# ---------------------------------------------------------------------------
# workload
# ---------------------------------------------------------------------------
def make_factors(n_layers, device, gen):
    G = Geo
    d, d_kv, r = G.d_model, G.n_kv * G.hd, G.rank
    w_norm = 0.02 * math.sqrt(d_kv * d)  # ||W_k|| of an N(0, 0.02^2) projection
    out = {}
    for name in ("k", "v"):
        A = torch.randn(n_layers, r, d, generator=gen, device=device) / math.sqrt(d)
        B = torch.randn(n_layers, d_kv, r, generator=gen, device=device)
        # scale so ||s B A||_F / ||W||_F = 1e-2 per layer (use the mean over layers)
        ba = torch.stack([(B[l] @ A[l]).norm() for l in range(n_layers)]).mean().item()
        out[name] = (A, B, 1e-2 * w_norm / ba)
    norm_w = 1.0 + 0.05 * torch.randn(n_layers, d, generator=gen, device=device)
    return out, norm_w


def make_workload(n_layers, n_seqs, seq_len, device, seed):
    import deltakv_b200 as dkv
    from deltakv_b200 import ops

    G = Geo
    gen = torch.Generator(device=device).manual_seed(seed)
    rows = n_seqs * seq_len
    x = torch.empty(n_layers, rows, G.d_model, dtype=G.x_torch, device=device)
    xs = torch.empty(n_layers, rows, dtype=torch.float32, device=device)
    xq = torch.empty(n_layers, rows, dtype=torch.float32, device=device)  # per-row sum of squared codes
    for l in range(n_layers):
        # residual-stream-like rows: N(0,1) with a per-token magnitude spread
        h = torch.randn(rows, G.d_model, generator=gen, device=device)
        h *= (0.5 + torch.rand(rows, 1, generator=gen, device=device))
        q, s, ssq = dkv.quantize_rows(h, G.x_torch, with_sumsq=True)
        x[l].copy_(q)
        xs[l].copy_(s)
        xq[l].copy_(ssq)
        del h, q, s, ssq
    blocks_per_seq = (seq_len + G.bs - 1) // G.bs
    nb = n_seqs * blocks_per_seq
    perm = torch.randperm(nb, generator=torch.Generator().manual_seed(seed + 2)).to(torch.int32)
    tables = perm.view(n_seqs, blocks_per_seq).to(device)
    caches = []  # vLLM flash-attention layout per layer: [2, num_blocks, block, n_kv, head_dim]
    for _ in range(n_layers):
        c = torch.empty(2, nb, G.bs, G.n_kv, G.hd, dtype=torch.bfloat16, device=device)
        c.normal_(generator=gen)
        caches.append(c)
    facs, norm_w = make_factors(n_layers, device, gen)
    cu = torch.arange(0, n_seqs + 1, dtype=torch.int32, device=device) * seq_len
    seqs = ops.SeqBatchTensors(cu_seqlens=cu, block_tables=tables, max_seq_len=seq_len)
    rope = dkv.RotaryEmbedding(G.hd, max_seq=seq_len, base=G.rope_theta)
    return dict(x=x, xs=xs, xq=xq, caches=caches, facs=facs, norm_w=norm_w, seqs=seqs, rope=rope, tables=tables)


# ---------------------------------------------------------------------------
# clocks during the timed region (NVML, polled in a thread)
# ---------------------------------------------------------------------------
class ClockSampler:
    REASONS = {
        "gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4, "hw_slowdown": 0x8,
        "sync_boost": 0x10, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
        "hw_power_brake_slowdown": 0x80, "display_clock_setting": 0x100,
    }

    def __init__(self, device_index: int):
        self.samples, self.reasons = [], 0
        self.stop_evt = threading.Event()
        self.ok = False
        try:
            import pynvml

            pynvml.nvmlInit()
            vis = os.environ.get("CUDA_VISIBLE_DEVICES")
            phys = int(vis.split(",")[device_index]) if vis else device_index
            self.h = pynvml.nvmlDeviceGetHandleByIndex(phys)
            self.nv = pynvml
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            self.max_mhz = None

    def _run(self):
        while not self.stop_evt.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                fn = getattr(self.nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                    getattr(self.nv, "nvmlDeviceGetCurrentClocksThrottleReasons")
                self.reasons |= fn(self.h)
            except Exception:
                pass
            time.sleep(0.01)

    def __enter__(self):
        if self.ok:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        if self.ok:
            self.stop_evt.set()
            self.t.join()

    def summary(self):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unavailable"]}
        names = [n for n, b in self.REASONS.items() if self.reasons & b and n != "gpu_idle"]
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz, "reasons": names,
                "samples": len(self.samples)}


# ---------------------------------------------------------------------------
# CPU oracle port (cpu_baseline and the reference arm)
# ---------------------------------------------------------------------------
def cpu_pool_threads() -> int:
    """Host threads for the CPU arm: every core, capped so each worker's ~0.5 GB of
    fp32 temporaries (one 4096-token sequence of one layer) fits in free memory."""
    try:
        cores = len(os.sched_getaffinity(0))
    except AttributeError:
        cores = os.cpu_count() or 1
    try:
        import psutil

        cap = int(psutil.virtual_memory().available * 0.6 // (512 << 20))
        return max(1, min(cores, cap))
    except Exception:
        return cores


class CpuSample:
    """A bounded sample of the workload on the host: P distinct (layer, sequence) inputs,
    one private paged K/V per worker thread (a single sequence's blocks)."""

    def __init__(self, n_inputs: int, seq_len: int, seed: int = 5):
        from oracle import exact as OX

        G = Geo
        g = torch.Generator().manual_seed(seed)
        self.seq_len = seq_len
        self.inputs = []
        facs, norm_w = make_factors(n_inputs, "cpu", g)
        for i in range(n_inputs):
            h = torch.randn(seq_len, G.d_model, generator=g) * (0.5 + torch.rand(seq_len, 1, generator=g))
            amax = h.abs().amax(-1).clamp_min(1e-12)
            s = (amax / 448.0).float()
            if G.x_kind == "e4m3":
                xb = (h / s[:, None]).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
            else:
                xb = (h / s[:, None]).to(torch.float16).numpy()
            fk = (facs["k"][0][i].numpy(), facs["k"][1][i].numpy(), facs["k"][2])
            fv = (facs["v"][0][i].numpy(), facs["v"][1][i].numpy(), facs["v"][2])
            self.inputs.append((xb, s.numpy(), norm_w[i].numpy(), fk, fv))
        self.rope = OX.rope_tables(G.hd, seq_len, G.rope_theta)
        nblk = (seq_len + G.bs - 1) // G.bs
        self.table = list(np.random.default_rng(seed).permutation(nblk))
        self.nblk = nblk

    def new_pages(self):
        G = Geo
        rng = np.random.default_rng(0)
        shape = (self.nblk, G.bs, G.n_kv, G.hd)
        return (rng.integers(0x3C00, 0x3F80, size=shape, dtype=np.uint16),
                rng.integers(0x3C00, 0x3F80, size=shape, dtype=np.uint16))

    def patch_one(self, i: int, kp, vp) -> int:
        """The reference's exact branch on one (layer, sequence): dequant -> RMSNorm ->
        exact_kv_patch -> materialize -> scatter_into_paged (K and V).  Returns units."""
        from oracle import exact as OX

        G = Geo
        xb, s, w, fk, fv = self.inputs[i % len(self.inputs)]
        x = OX.dequant_x(xb, G.x_kind, s)
        x = OX.rmsnorm(x, w, G.eps)
        dk, dv = OX.exact_kv_delta(x, fk, fv, G.n_kv, G.hd, self.rope)
        OX.scatter_into_paged(dk, kp, self.table, G.bs, kind="bf16")
        OX.scatter_into_paged(dv, vp, self.table, G.bs, kind="bf16")
        return self.seq_len

    def run(self, threads: int, seconds: float | None = None, pairs: int | None = None):
        """Process pairs on `threads` workers for `seconds` (or `pairs` pairs); returns
        (units, elapsed_s)."""
        from concurrent.futures import ThreadPoolExecutor

        from threadpoolctl import threadpool_limits

        pages = [self.new_pages() for _ in range(threads)]
        counter = [0]
        lock = threading.Lock()
        deadline = None if seconds is None else time.perf_counter() + seconds

        def worker(wi):
            done = 0
            while True:
                with lock:
                    if pairs is not None and counter[0] >= pairs:
                        return done
                    if deadline is not None and time.perf_counter() >= deadline:
                        return done
                    k = counter[0]
                    counter[0] += 1
                done += self.patch_one(k, *pages[wi])

        with threadpool_limits(1):
            t0 = time.perf_counter()
            with ThreadPoolExecutor(threads) as ex:
                units = sum(ex.map(worker, range(threads)))
            el = time.perf_counter() - t0
        return units, el


def cpu_baseline(seconds: float, seq_len: int) -> dict:
    threads = cpu_pool_threads()
    sample = CpuSample(n_inputs=4, seq_len=seq_len)
    sample.run(threads, pairs=threads)  # warm-up: every thread once
    units, el = sample.run(threads, seconds=seconds)
    return {"value": units / el, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{units // seq_len} (layer, sequence) pairs of {seq_len} tokens in {el:.1f} s "
                      f"(oracle numpy port of the reference's exact branch, {threads} threads)"}


# ---------------------------------------------------------------------------
# arms
# ---------------------------------------------------------------------------
def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def run_reference(args):
    world, rank, _ = dist_setup(args)
    if rank != 0:
        return 0
    threads = cpu_pool_threads()
    sample = CpuSample(n_inputs=4, seq_len=args.seq_len)
    for _ in range(args.warmup):
        sample.run(threads, pairs=threads)
    units_tot, el_tot = 0, 0.0
    for _ in range(args.steps):
        u, el = sample.run(threads, pairs=threads)
        units_tot += u
        el_tot += el
    value = units_tot / el_tot
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * el_tot / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "step": f"{threads} (layer, sequence) pairs of {args.seq_len} tokens "
                   "(bounded sample of the workload)"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"{threads} (layer, sequence) pairs per step, oracle numpy port of the "
                                   "reference's exact branch (dequant, RMSNorm, exact_kv_patch, materialize, "
                                   "scatter_into_paged)"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_ours(args):
    import deltakv_b200 as dkv

    world, rank, local = dist_setup(args)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=dev)
    G = Geo
    wl = make_workload(args.layers, args.seqs, args.seq_len, dev, seed=1000 + rank)
    facs = wl["facs"]
    patcher = dkv.ExactPatcher(G.d_model, G.n_kv, G.hd, rank_k=G.rank, rank_v=G.rank,
                               x_dtype=G.x_torch, rope=wl["rope"], norm_eps=G.eps)
    packed = torch.empty(args.layers, patcher.packed_bytes, dtype=torch.uint8, device=dev)
    kpages = [c[0] for c in wl["caches"]]
    vpages = [c[1] for c in wl["caches"]]
    units = args.layers * args.seqs * args.seq_len
    stream = torch.cuda.current_stream()

    def step(ev=None):
        patcher.pack(facs["k"][0], facs["k"][1], facs["v"][0], facs["v"][1], facs["k"][2], facs["v"][2],
                     norm_weight=wl["norm_w"], out=packed)
        if ev is not None:
            ev[0].record(stream)
        patcher.apply(wl["x"], packed, kpages, vpages, wl["seqs"], x_scale=wl["xs"], apply_norm=True,
                      x_sumsq=wl["xq"])
        if ev is not None:
            ev[1].record(stream)

    # correctness guard before timing: device status clean after one step
    step()
    torch.cuda.synchronize()
    from deltakv_b200 import ops

    ops.status_word(dev).raise_if_set("bench warm-up")
    for _ in range(max(0, args.warmup - 1)):
        step()
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        t_start.record(stream)
        for i in range(args.steps):
            step(kev[i])
        t_end.record(stream)
        torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    ms = t_start.elapsed_time(t_end)
    kern_ms = [a.elapsed_time(b) for a, b in kev]
    if world > 1:
        t = torch.tensor([ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    ops.status_word(dev).raise_if_set("bench timed region")
    ms_step = ms / args.steps
    value = units * world / (ms_step / 1e3)
    kmean = sum(kern_ms) / len(kern_ms)
    achieved = units * BYTES_PER_UNIT / (kmean / 1e3) / 1e9
    peaks = {}
    try:
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except Exception:
        pass
    peak = peaks.get("hbm_gbs")
    peak_kind = "of measured (MEASURED_PEAKS.json hbm_gbs, burst copy)" if peak else "of fallback (6650 GB/s)"
    peak = peak or 6650.0
    traffic = None  # DRAM bytes per launch from the committed ncu summary (full workload)
    tfile = ROOT / "profiles" / "exact_patch_kernel.md"
    if tfile.exists() and args.layers == 32 and args.seqs == 64 and args.seq_len == 4096:
        for line in tfile.read_text().splitlines():
            if line.startswith("traffic_bytes_per_launch_full_workload:"):
                traffic = int(line.split(":", 1)[1])

    layer_errors = measure_layer_errors(args, wl["seqs"], kpages, vpages, step, dev, world)
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(args, patcher, dev, world)
    del wl, kpages, vpages
    torch.cuda.empty_cache()
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline(args.cpu_seconds, args.seq_len)
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16 tensor-core products, fp32 accumulate (e4m3 X, bf16 pages)",
            "data": "synthetic",
            "config": {"workload": WORKLOAD, "layers": args.layers, "seqs_per_gpu": args.seqs,
                       "seq_len": args.seq_len, "units_per_step_per_gpu": units,
                       "parallelism": f"request shards x{world} (weak)",
                       "l2": f"inputs {units * BYTES_PER_UNIT / 1e9:.1f} GB per GPU >> 126 MB L2, no flush needed",
                       "launches_per_step": 2},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic, "peak_source": peak_kind,
                         "kernel": "patch_kernel", "kernel_ms": kmean,
                         "algorithmic_bytes_per_unit": BYTES_PER_UNIT},
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": 2 * args.steps,
            "clocks": clk.summary(),
            "layer_errors": layer_errors,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()
    return 0


def measure_layer_errors(args, seqs, kpages, vpages, step, dev, world):
    """After the timed region: per-layer measured error (compose.py:147-163 formula) of one
    more patch step on sequence 0 — the stale pages against the patched ones, i.e. the error a
    cache would carry without the patch — then the NCCL all-gather of those scalars over the
    ranks (the path's only collective)."""
    from deltakv_b200 import metrics, ops

    n = args.seq_len
    one = ops.SeqBatchTensors(cu_seqlens=seqs.cu_seqlens[:2].clone(), block_tables=seqs.block_tables[:1].contiguous(),
                              max_seq_len=n)
    L_ = len(kpages)
    nkv, hd = kpages[0].shape[2], kpages[0].shape[3]
    stale_k = torch.empty(L_, n, nkv, hd, dtype=kpages[0].dtype, device=dev)
    stale_v = torch.empty_like(stale_k)
    for l in range(L_):
        ops.gather_paged(kpages[l], one, stale_k[l])
        ops.gather_paged(vpages[l], one, stale_v[l])
    step()
    local = metrics.measured_error_paged(kpages, vpages, stale_k, stale_v, one, check=True)
    t0 = time.perf_counter()
    gathered = metrics.gather_layer_errors(local)
    torch.cuda.synchronize()
    gather_ms = 1e3 * (time.perf_counter() - t0)
    g = gathered.cpu()
    return {"what": "per-layer relative KV change of one patch step on sequence 0 (stale vs patched)",
            "max": float(g.max()), "mean": float(g.mean()), "ranks": world, "layers_per_rank": L_,
            "collective": "all_gather_into_tensor (nccl)" if world > 1 else "none (single rank)",
            "gather_wall_ms": gather_ms}


def run_e2e(args, patcher, dev, world):
    """Same metric through the public API with host buffers: every step copies the step's
    stored activations, scales, factors, block tables and the touched pages host->device,
    patches, and copies the pages back."""
    import deltakv_b200 as dkv
    from deltakv_b200 import ops

    G = Geo
    n_seqs = args.e2e_seqs
    cpu = make_workload(args.layers, n_seqs, args.seq_len, dev, seed=77)
    host = {
        "x": cpu["x"].view(torch.uint8).cpu().pin_memory(),
        "xs": cpu["xs"].cpu().pin_memory(),
        "xq": cpu["xq"].cpu().pin_memory(),
        "caches": torch.stack(cpu["caches"]).cpu().pin_memory(),
        "tables": cpu["tables"].cpu().pin_memory(),
        "a_k": cpu["facs"]["k"][0].cpu().pin_memory(), "b_k": cpu["facs"]["k"][1].cpu().pin_memory(),
        "a_v": cpu["facs"]["v"][0].cpu().pin_memory(), "b_v": cpu["facs"]["v"][1].cpu().pin_memory(),
        "norm_w": cpu["norm_w"].cpu().pin_memory(),
    }
    sk, sv = cpu["facs"]["k"][2], cpu["facs"]["v"][2]
    del cpu
    torch.cuda.empty_cache()
    d = {k: torch.empty_like(v, device=dev) for k, v in host.items()}
    packed = torch.empty(args.layers, patcher.packed_bytes, dtype=torch.uint8, device=dev)
    cu = torch.arange(0, n_seqs + 1, dtype=torch.int32, device=dev) * args.seq_len
    stream = torch.cuda.current_stream()
    h2d = sum(v.numel() * v.element_size() for v in host.values())
    d2h = host["caches"].numel() * host["caches"].element_size()

    # Layer-pipelined: host->device copies of layer l+1 (one copy engine), the patch of layer l
    # (compute stream) and the device->host copy of layer l-1 (the other copy engine) overlap.
    h2d_s, d2h_s = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    seqs = ops.SeqBatchTensors(cu_seqlens=cu, block_tables=d["tables"], max_seq_len=args.seq_len)
    small = ("tables", "a_k", "b_k", "a_v", "b_v", "norm_w")
    n_layers = args.layers

    def step():
        start = torch.cuda.Event()
        start.record(stream)
        h2d_s.wait_event(start)  # the previous step's copies back have finished
        with torch.cuda.stream(h2d_s):
            for k in small:
                d[k].copy_(host[k], non_blocking=True)
            ev_small = torch.cuda.Event()
            ev_small.record(h2d_s)
            ev_in = []
            for l in range(n_layers):
                d["x"][l].copy_(host["x"][l], non_blocking=True)
                d["xs"][l].copy_(host["xs"][l], non_blocking=True)
                d["xq"][l].copy_(host["xq"][l], non_blocking=True)
                d["caches"][l].copy_(host["caches"][l], non_blocking=True)
                e = torch.cuda.Event()
                e.record(h2d_s)
                ev_in.append(e)
        stream.wait_event(ev_small)
        patcher.pack(d["a_k"], d["b_k"], d["a_v"], d["b_v"], sk, sv, norm_weight=d["norm_w"], out=packed)
        xv = d["x"].view(G.x_torch)
        for l in range(n_layers):
            stream.wait_event(ev_in[l])
            patcher.apply(xv[l:l + 1], packed[l:l + 1], [d["caches"][l][0]], [d["caches"][l][1]], seqs,
                          x_scale=d["xs"][l:l + 1], apply_norm=True, x_sumsq=d["xq"][l:l + 1])
            e = torch.cuda.Event()
            e.record(stream)
            d2h_s.wait_event(e)
            with torch.cuda.stream(d2h_s):
                host["caches"][l].copy_(d["caches"][l], non_blocking=True)
        done = torch.cuda.Event()
        done.record(d2h_s)
        stream.wait_event(done)

    for _ in range(2):
        step()
    torch.cuda.synchronize()
    n = 3
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        torch.distributed.barrier()
    a.record(stream)
    for _ in range(n):
        step()
    b.record(stream)
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / n
    if world > 1:
        t = torch.tensor([ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    units = args.layers * n_seqs * args.seq_len * world
    del d, host
    torch.cuda.empty_cache()
    return {"value": units / (ms / 1e3), "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "ms_per_step": ms, "sample": f"{n_seqs} seqs x {args.layers} layers per GPU, pinned host buffers, "
                                        "host->device / patch / device->host pipelined by layer"}


# ---------------------------------------------------------------------------
# rl-dense workload: full-rank dW on k_proj / v_proj (tensor-core GEMM route)
# ---------------------------------------------------------------------------
DENSE_METRIC = "patched token·layers/s (Llama-70B shape, dense dW RL step)"
DENSE_WORKLOAD = ("Llama-3-70B-shaped RL-step dense delta, one GPU's share: 10 of 80 layers, d=8192, 8 KV heads "
                  "x 128, 16 seqs x 8192 tokens, bf16 stored X (post-norm), full-rank dW_K/dW_V Gaussian with "
                  "||dW||/||W|| = 1e-3, RoPE (theta 5e5) on K, bf16 paged KV block 16, permuted block table")


def dense_flops_per_unit() -> float:
    G = DenseGeo
    return 2.0 * G.d_model * 2 * G.n_kv * G.hd


def make_dense_workload(n_layers, n_seqs, seq_len, device, seed):
    import deltakv_b200 as dkv
    from deltakv_b200 import ops

    G = DenseGeo
    gen = torch.Generator(device=device).manual_seed(seed)
    rows = n_seqs * seq_len
    d_kv = G.n_kv * G.hd
    x = torch.empty(n_layers, rows, G.d_model, dtype=torch.bfloat16, device=device)
    for l in range(n_layers):
        x[l].normal_(generator=gen)
    sigma = 1e-3 * 0.02  # ||dW|| / ||W|| = 1e-3 for W ~ N(0, 0.02^2)
    dw_k = (torch.randn(n_layers, d_kv, G.d_model, generator=gen, device=device) * sigma).to(torch.bfloat16)
    dw_v = (torch.randn(n_layers, d_kv, G.d_model, generator=gen, device=device) * sigma).to(torch.bfloat16)
    blocks_per_seq = (seq_len + G.bs - 1) // G.bs
    nb = n_seqs * blocks_per_seq
    perm = torch.randperm(nb, generator=torch.Generator().manual_seed(seed + 2)).to(torch.int32)
    tables = perm.view(n_seqs, blocks_per_seq).to(device)
    caches = []
    for _ in range(n_layers):
        c = torch.empty(2, nb, G.bs, G.n_kv, G.hd, dtype=torch.bfloat16, device=device)
        c.normal_(generator=gen)
        caches.append(c)
    cu = torch.arange(0, n_seqs + 1, dtype=torch.int32, device=device) * seq_len
    seqs = ops.SeqBatchTensors(cu_seqlens=cu, block_tables=tables, max_seq_len=seq_len)
    rope = dkv.RotaryEmbedding(G.hd, max_seq=seq_len, base=G.rope_theta)
    return dict(x=x, dw_k=dw_k, dw_v=dw_v, caches=caches, seqs=seqs, rope=rope, tables=tables)


class DenseCpuSample:
    """Bounded host sample of the dense route: (layer, 256-token chunk) items through the
    oracle port of the reference's exact route with A = dW, B = I (one chunk per worker)."""

    CHUNK = 256

    def __init__(self, seed: int = 5):
        from oracle import dense as OD
        from oracle import exact as OX

        G = DenseGeo
        g = torch.Generator().manual_seed(seed)
        d_kv = G.n_kv * G.hd
        self.x = (torch.randn(self.CHUNK, G.d_model, generator=g)).to(torch.bfloat16).float().numpy()
        sig = 1e-3 * 0.02
        self.fk, self.fv = OD.dense_factors((torch.randn(d_kv, G.d_model, generator=g) * sig).numpy(),
                                            (torch.randn(d_kv, G.d_model, generator=g) * sig).numpy())
        self.rope = OX.rope_tables(G.hd, self.CHUNK, G.rope_theta)
        self.nblk = self.CHUNK // G.bs
        self.table = list(np.random.default_rng(seed).permutation(self.nblk))

    def new_pages(self):
        G = DenseGeo
        rng = np.random.default_rng(0)
        shape = (self.nblk, G.bs, G.n_kv, G.hd)
        return (rng.integers(0x3C00, 0x3F80, size=shape, dtype=np.uint16),
                rng.integers(0x3C00, 0x3F80, size=shape, dtype=np.uint16))

    def patch_one(self, kp, vp) -> int:
        from oracle import exact as OX

        G = DenseGeo
        dk, dv = OX.exact_kv_delta(self.x, self.fk, self.fv, G.n_kv, G.hd, self.rope)
        OX.scatter_into_paged(dk, kp, self.table, G.bs, kind="bf16")
        OX.scatter_into_paged(dv, vp, self.table, G.bs, kind="bf16")
        return self.CHUNK

    def run(self, threads: int, seconds: float | None = None, items: int | None = None):
        from concurrent.futures import ThreadPoolExecutor

        from threadpoolctl import threadpool_limits

        pages = [self.new_pages() for _ in range(threads)]
        counter = [0]
        lock = threading.Lock()
        deadline = None if seconds is None else time.perf_counter() + seconds

        def worker(wi):
            done = 0
            while True:
                with lock:
                    if items is not None and counter[0] >= items:
                        return done
                    if deadline is not None and time.perf_counter() >= deadline:
                        return done
                    counter[0] += 1
                done += self.patch_one(*pages[wi])

        with threadpool_limits(1):
            t0 = time.perf_counter()
            with ThreadPoolExecutor(threads) as ex:
                units = sum(ex.map(worker, range(threads)))
            el = time.perf_counter() - t0
        return units, el


def dense_cpu_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def run_dense_reference(args):
    world, rank, _ = dist_setup(args)
    if rank != 0:
        return 0
    threads = dense_cpu_threads()
    sample = DenseCpuSample()
    for _ in range(args.warmup):
        sample.run(threads, items=threads)
    units_tot, el_tot = 0, 0.0
    for _ in range(args.steps):
        u, el = sample.run(threads, items=threads)
        units_tot += u
        el_tot += el
    value = units_tot / el_tot
    line = {
        "impl": "reference", "metric": DENSE_METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * el_tot / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": DENSE_WORKLOAD, "step": f"{threads} (layer, {DenseCpuSample.CHUNK}-token chunk) "
                   "items (bounded sample of the workload)"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"{threads} items per step, oracle numpy port of the reference's exact route "
                                   "with A=dW, B=I (x @ dW^T, RoPE, scatter_into_paged)"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_dense_ours(args):
    import deltakv_b200 as dkv
    from deltakv_b200 import ops

    world, rank, local = dist_setup(args)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    G = DenseGeo
    wl = make_dense_workload(args.layers, args.seqs, args.seq_len, dev, seed=2000 + rank)
    patcher = dkv.DensePatcher(G.d_model, G.n_kv, G.hd, rope=wl["rope"])
    packed = torch.empty(args.layers, 2 * G.n_kv * G.hd, G.d_model, dtype=torch.bfloat16, device=dev)
    kpages = [c[0] for c in wl["caches"]]
    vpages = [c[1] for c in wl["caches"]]
    units = args.layers * args.seqs * args.seq_len
    stream = torch.cuda.current_stream()

    def step(ev=None):
        patcher.pack(wl["dw_k"], wl["dw_v"], out=packed)
        if ev is not None:
            ev[0].record(stream)
        patcher.apply(wl["x"], packed, kpages, vpages, wl["seqs"])
        if ev is not None:
            ev[1].record(stream)

    step()
    torch.cuda.synchronize()
    ops.status_word(dev).raise_if_set("bench warm-up")
    for _ in range(max(0, args.warmup - 1)):
        step()
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        t_start.record(stream)
        for i in range(args.steps):
            step(kev[i])
        t_end.record(stream)
        torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    ms = t_start.elapsed_time(t_end)
    kern_ms = [a.elapsed_time(b) for a, b in kev]
    if world > 1:
        t = torch.tensor([ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    ops.status_word(dev).raise_if_set("bench timed region")
    ms_step = ms / args.steps
    value = units * world / (ms_step / 1e3)
    kmean = sum(kern_ms) / len(kern_ms)
    achieved = units * dense_flops_per_unit() / (kmean / 1e3) / 1e12
    peaks = {}
    try:
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except Exception:
        pass
    peak = peaks.get("bf16_tflops_sustained")
    peak_kind = ("of measured (MEASURED_PEAKS.json bf16_tflops_sustained: a seconds-long step)" if peak
                 else "of fallback (1400 TFLOP/s sustained)")
    peak = peak or 1400.0
    traffic = None
    tfile = ROOT / "profiles" / "dense_patch_kernel.md"
    if tfile.exists() and args.layers == G.layers and args.seqs == G.seqs and args.seq_len == G.seq_len:
        for line in tfile.read_text().splitlines():
            if line.startswith("traffic_bytes_per_launch_full_workload:"):
                traffic = int(line.split(":", 1)[1])
    e2e = None
    if not args.no_e2e:
        e2e = run_dense_e2e(args, patcher, dev, world)
    del wl, kpages, vpages
    torch.cuda.empty_cache()
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        threads = dense_cpu_threads()
        sample = DenseCpuSample()
        sample.run(threads, items=threads)
        u, el = sample.run(threads, seconds=args.cpu_seconds)
        cpu = {"value": u / el, "unit": UNIT, "cores": threads, "kind": "port",
               "sample": f"{u // DenseCpuSample.CHUNK} (layer, {DenseCpuSample.CHUNK}-token chunk) items in "
                         f"{el:.1f} s (oracle numpy port of the reference's exact route with A=dW, B=I, "
                         f"{threads} threads)"}
    if rank == 0:
        line = {
            "metric": DENSE_METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16 tensor-core products, fp32 accumulate (bf16 X and pages)",
            "data": "synthetic",
            "config": {"workload": DENSE_WORKLOAD, "layers": args.layers, "seqs_per_gpu": args.seqs,
                       "seq_len": args.seq_len, "units_per_step_per_gpu": units,
                       "parallelism": f"layer shards x{world} (weak)",
                       "l2": f"X {units * G.d_model * 2 / 1e9:.1f} GB per GPU >> 126 MB L2, no flush needed",
                       "launches_per_step": 2},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak, "traffic": traffic, "peak_source": peak_kind,
                         "kernel": "dense_patch_kernel", "kernel_ms": kmean,
                         "algorithmic_flops_per_unit": dense_flops_per_unit()},
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": 2 * args.steps,
            "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()
    return 0


def run_dense_e2e(args, patcher, dev, world):
    """Same metric through DensePatcher with pinned host buffers: X, dW, tables and pages
    copied in, pages copied back, every step (1 layer x 2 sequences per GPU)."""
    from deltakv_b200 import ops

    n_layers, n_seqs = 1, 2
    cpu = make_dense_workload(n_layers, n_seqs, args.seq_len, dev, seed=78)
    host = {k: cpu[k].cpu().pin_memory() for k in ("x", "dw_k", "dw_v", "tables")}
    host["caches"] = torch.stack(cpu["caches"]).cpu().pin_memory()
    del cpu
    torch.cuda.empty_cache()
    d = {k: torch.empty_like(v, device=dev) for k, v in host.items()}
    G = DenseGeo
    packed = torch.empty(n_layers, 2 * G.n_kv * G.hd, G.d_model, dtype=torch.bfloat16, device=dev)
    cu = torch.arange(0, n_seqs + 1, dtype=torch.int32, device=dev) * args.seq_len
    stream = torch.cuda.current_stream()
    h2d = sum(v.numel() * v.element_size() for v in host.values())
    d2h = host["caches"].numel() * host["caches"].element_size()

    def step():
        for k, v in host.items():
            d[k].copy_(v, non_blocking=True)
        patcher.pack(d["dw_k"], d["dw_v"], out=packed)
        seqs = ops.SeqBatchTensors(cu_seqlens=cu, block_tables=d["tables"], max_seq_len=args.seq_len)
        patcher.apply(d["x"], packed, [c[0] for c in d["caches"]], [c[1] for c in d["caches"]], seqs)
        host["caches"].copy_(d["caches"], non_blocking=True)

    for _ in range(2):
        step()
    torch.cuda.synchronize()
    n = 3
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        torch.distributed.barrier()
    a.record(stream)
    for _ in range(n):
        step()
    b.record(stream)
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / n
    if world > 1:
        t = torch.tensor([ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    units = n_layers * n_seqs * args.seq_len * world
    del d, host
    torch.cuda.empty_cache()
    return {"value": units / (ms / 1e3), "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "ms_per_step": ms, "sample": f"{n_seqs} seqs x {n_layers} layer per GPU, pinned host buffers"}



# ---------------------------------------------------------------------------
# multi-lora-kivi workload: int4 KIVI shared prefix corrected per adapter view
# ---------------------------------------------------------------------------
KIVI_METRIC = "patched token·layers/s (Llama-8B shape, int4 KIVI prefix, subspace route per adapter view)"
KIVI_WORKLOAD = ("Multi-LoRA shared prefix on the Llama-3-8B shape: 32 layers, 8 KV heads x 128, one 32768-token "
                 "prefix stored KIVI int4 (K per-channel, V per-token, group 32, fp16 scale/zero); adapter views "
                 "with k/v ranks {8,8,16,16,32,32,64,64}; per view and layer: K basis = top-r right singular "
                 "subspace of the probe residual, V basis = the adapter's LoRA B; probes 10 %; dequant -> subspace "
                 "correction -> requant into the view's own int4 cache")
KIVI_BYTES_PER_UNIT = 1024 + 256 + 4096 + 1024 + 256  # base int4 K+V, scale/zero, fresh bf16 K+V, out int4, scale/zero
KIVI_RANKS = (8, 8, 16, 16, 32, 32, 64, 64)


class KiviGeo:
    layers, seq_len, n_kv, hd, probe_ratio = 32, 32768, 8, 128, 0.10


def make_kivi_workload(args, device, rank_ids):
    """Base int4 prefix (shared), and per adapter view: fresh bf16 K/V per layer, V basis,
    probes.  fresh = dequant(base) + rank-r structure + 10 % drift on the non-probes."""
    from deltakv_b200 import kivi as K

    G = KiviGeo
    n, d = args.seq_len, G.n_kv * G.hd
    gen = torch.Generator(device=device).manual_seed(4000)
    base = []
    for _ in range(args.layers):
        kv = []
        for mode in ("k", "v"):
            x = torch.randn(n, d, generator=gen, device=device)
            kv.append(K.quantize(x, mode))
            del x
        base.append(kv)
    n_p = int(round(G.probe_ratio * n))
    adapters = []
    for a in rank_ids:
        r = KIVI_RANKS[a % len(KIVI_RANKS)]
        g = torch.Generator(device=device).manual_seed(5000 + a)
        probes = torch.unique(torch.cat([torch.zeros(1, dtype=torch.long, device=device),
                                         torch.randperm(n, generator=g, device=device)[: n_p - 1]]))
        layers = []
        for l in range(args.layers):
            views = []
            for m, mode in enumerate(("k", "v")):
                B = torch.randn(d, r, generator=g, device=device) / math.sqrt(d)
                codes = torch.randn(n, r, generator=g, device=device) * 0.5
                fresh = K.dequantize(base[l][m])
                fresh += codes @ B.T
                drift = 0.1 * fresh.std() * torch.randn(n, d, generator=g, device=device)
                drift[probes] = 0
                fresh += drift
                views.append({"fresh": fresh.to(torch.bfloat16), "basis": B if mode == "v" else None,
                              "out": K.KiviTensor.empty(n, d, mode, device)})
                del codes, drift, fresh
            layers.append(views)
        adapters.append({"rank": r, "probes": probes, "layers": layers})
    return base, adapters


def kivi_problems(base, adapter, k_bases=None):
    from deltakv_b200 import kivi as K

    probs = []
    for l, views in enumerate(adapter["layers"]):
        for m in range(2):
            v = views[m]
            basis = v["basis"] if m == 1 else (None if k_bases is None else k_bases[l])
            probs.append(K.SubspaceProblem(base=base[l][m], fresh=v["fresh"], probe_index=adapter["probes"],
                                           basis=basis, rank=adapter["rank"], out=v["out"]))
    return probs


def kivi_e2e(args, base, adapter, dev, world, stream, n_layers: int = 4) -> dict:
    """The same metric through the public call from pinned host buffers, on a bounded sample:
    one adapter view's first ``n_layers`` layers — its fresh bf16 K / V copied in, corrected by
    ``subspace_correct_views``, the corrected int4 K / V (codes, scales, zeros) copied out; the
    shared base cache stays resident."""
    from deltakv_b200 import kivi as K

    nl = min(n_layers, args.layers)
    views = [adapter["layers"][l][m] for l in range(nl) for m in range(2)]
    fresh_host = [v["fresh"].cpu().pin_memory() for v in views]
    outs = [v["out"] for v in views]
    out_host = [[t.cpu().pin_memory() for t in (o.codes, o.scale, o.zero)] for o in outs]
    h2d = sum(t.numel() * t.element_size() for t in fresh_host)
    d2h = sum(t.numel() * t.element_size() for ts in out_host for t in ts)

    def step():
        probs = []
        for i, (v, fh) in enumerate(zip(views, fresh_host)):
            l, m = divmod(i, 2)
            probs.append(K.SubspaceProblem(base=base[l][m], fresh=fh.to(dev, non_blocking=True),
                                           probe_index=adapter["probes"], basis=v["basis"] if m == 1 else None,
                                           rank=adapter["rank"], out=v["out"]))
        K.subspace_correct_views([probs], check=False)
        for o, hs in zip(outs, out_host):
            for hst, t in zip(hs, (o.codes, o.scale, o.zero)):
                hst.copy_(t, non_blocking=True)

    step()  # untimed: the pinned buffers' first transfers
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n = 3
    a.record(stream)
    for _ in range(n):
        step()
    b.record(stream)
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / n
    if world > 1:
        t = torch.tensor([ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    units = nl * args.seq_len * world
    return {"value": units / (ms / 1e3), "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "ms_per_step": ms, "sample": f"1 adapter view (rank {adapter['rank']}) x {nl} layers x "
                                        f"{args.seq_len} tokens per GPU, pinned host buffers"}


def run_kivi_ours(args):
    from deltakv_b200 import kivi as K
    from deltakv_b200 import ops

    world, rank, local = dist_setup(args)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    # weak scaling: every rank maintains its own `--adapters` views (distinct adapters, the same
    # rank mix {8, 8, 16, 16, 32, 32, 64, 64} on each GPU, so the ranks stay balanced)
    per_rank = max(1, args.adapters)
    ids = [rank * per_rank + i for i in range(per_rank)]
    base, adapters = make_kivi_workload(args, dev, ids)
    units = args.layers * args.seq_len * per_rank
    stream = torch.cuda.current_stream()

    problems = [kivi_problems(base, ad) for ad in adapters]

    def step():
        # all views; view v + 1's K bases overlap view v's route (side stream)
        K.subspace_correct_views(problems, check=False)

    step()
    torch.cuda.synchronize()
    ops.status_word(dev).raise_if_set("bench warm-up")
    for _ in range(max(0, args.warmup - 1)):
        step()
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        t_start.record(stream)
        for i in range(args.steps):
            step()
        t_end.record(stream)
        torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    # the two halves alone (after the timed region, same work, one stream): K bases, route
    split = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    n_split = 2
    basis_ms = route_ms = 0.0
    for it in range(n_split + 1):  # the first pass warms the main stream's allocator pool
        split[0].record(stream)
        kbs = [K.k_bases(pb) for pb in problems]
        split[1].record(stream)
        for pb, kb in zip(problems, kbs):
            K.subspace_correct(pb, check=False, bases=kb)
        split[2].record(stream)
        torch.cuda.synchronize()
        if it:
            basis_ms += split[0].elapsed_time(split[1]) / n_split
            route_ms += split[1].elapsed_time(split[2]) / n_split
    ms = t_start.elapsed_time(t_end)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    ops.status_word(dev).raise_if_set("bench timed region")
    ms_step = ms / args.steps
    value = units * world / (ms_step / 1e3)
    achieved = units * KIVI_BYTES_PER_UNIT / (route_ms / 1e3) / 1e9
    peaks = {}
    try:
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except Exception:
        pass
    peak = peaks.get("hbm_gbs") or 6650.0
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = kivi_cpu_sample(args.cpu_seconds)
    e2e = None
    if not args.no_e2e:
        e2e = kivi_e2e(args, base, adapters[0], dev, world, stream)
    if rank == 0:
        line = {
            "metric": KIVI_METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int4 KIVI cache, bf16 tensor-core products, fp32 accumulate",
            "data": "synthetic",
            "config": {"workload": KIVI_WORKLOAD, "layers": args.layers, "prefix_tokens": args.seq_len,
                       "adapter_views_per_gpu": per_rank, "ranks": [a["rank"] for a in adapters],
                       "units_per_step_per_gpu": units, "parallelism": f"adapter shards x{world}",
                       "l2": f"{units * KIVI_BYTES_PER_UNIT / 1e9:.1f} GB per step per GPU >> 126 MB L2",
                       "k_basis_ms_per_step": basis_ms, "subspace_route_ms_per_step": route_ms},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "traffic": None, "peak_source": "of measured (MEASURED_PEAKS.json hbm_gbs, burst copy)",
                         "kernel": "int4 subspace route (flags, pack, pass1 x2, psum, solve, fitb, pass2 x2) per view",
                         "kernel_ms": route_ms, "algorithmic_bytes_per_unit": KIVI_BYTES_PER_UNIT},
            "cpu_baseline": cpu,
            "e2e": e2e,
            # per view: flags, pack, pass1 K/V, psum, solve, fitb, pass2 K/V (9) + the K bases'
            # batched probe residual and Jacobi eigensolver (2); library calls not counted
            "gpu_launches": args.steps * len(adapters) * 11,
            "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()
    return 0


def kivi_cpu_sample(seconds: float, n: int = 4096) -> dict:
    """Oracle port of the route (dequant, subspace_correct, requant) on (layer, view) items of
    `n` tokens, one item per worker thread."""
    from concurrent.futures import ThreadPoolExecutor

    from threadpoolctl import threadpool_limits

    from oracle import kivi as OK
    from oracle import subspace as OS

    G = KiviGeo
    d = G.n_kv * G.hd
    rng = np.random.default_rng(7)
    base = OK.quantize(rng.standard_normal((n, d), dtype=np.float32), "v")
    B = (rng.standard_normal((d, 16), dtype=np.float32) / np.sqrt(d)).astype(np.float32)
    fresh = (OK.dequantize(*base, "v") + (rng.standard_normal((n, 16), dtype=np.float32) * 0.5) @ B.T).astype(np.float32)
    probes = np.unique(np.concatenate([[0], rng.permutation(n)[: int(0.1 * n)]]))
    threads = dense_cpu_threads()

    def item():
        reused = OK.dequantize(*base, "v")
        corr, _, _ = OS.subspace_correct(reused.reshape(n, G.n_kv, G.hd), fresh.reshape(n, G.n_kv, G.hd), probes,
                                         basis=B, rank=16)
        OK.quantize(corr.reshape(n, d), "v")
        return n

    deadline = time.perf_counter() + seconds
    lock = threading.Lock()
    done = [0]

    def worker(_):
        u = 0
        while time.perf_counter() < deadline:
            u += item()
        with lock:
            done[0] += u
        return u

    with threadpool_limits(1):
        t0 = time.perf_counter()
        with ThreadPoolExecutor(threads) as ex:
            list(ex.map(worker, range(threads)))
        el = time.perf_counter() - t0
    return {"value": done[0] / el, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{done[0] // n} (layer, view) items of {n} tokens, rank 16, V grouping, in {el:.1f} s "
                      f"(oracle numpy port: dequant, subspace_correct, requant; {threads} threads)"}


def run_kivi_reference(args):
    world, rank, _ = dist_setup(args)
    if rank != 0:
        return 0
    res = [kivi_cpu_sample(max(2.0, args.cpu_seconds / max(1, args.steps))) for _ in range(args.steps)]
    value = sum(r["value"] for r in res) / len(res)
    line = {
        "impl": "reference", "metric": KIVI_METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": None, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": KIVI_WORKLOAD, "step": res[0]["sample"]},
        "cpu_baseline": {**res[0], "value": value},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# analytic route (Route A): first-order propagation through the stack
# ---------------------------------------------------------------------------
ANALYTIC_METRIC = "patched token·layers/s (analytic route, SmolLM2-135M shape)"
FP32_FMA_NOMINAL_TFLOPS = 148 * 128 * 2 * 1.965e9 / 1e12  # SMs x FP32 lanes x 2 x max SM clock


class AnalyticGeo:
    layers, d_model, n_heads, n_kv, hd, d_ff, rank = 30, 576, 9, 3, 64, 1536, 8
    seqs, seq_len, eps, rope_theta, propagator_rank, hidden_stride = 4, 2048, 1e-5, 10000.0, 64, 4


ANALYTIC_WORKLOAD = ("SmolLM2-135M-shaped analytic route (engine loop of the reference): 30 layers, d=576, 9 query / 3 "
                     "KV heads x 64, SwiGLU 1536, fp32 weights N(0, 0.02), rank-8 LoRA on q/k/v/o of every layer, "
                     "stored hidden states N(0,1) (layer input and post-attention), 2048 tokens per sequence, "
                     "propagator rank 64, hidden stride 4")


def make_analytic_workload(args, device, seed):
    import types as _t

    from deltakv_b200.rope import RotaryEmbedding
    from deltakv_b200.types import LayerDelta, LowRankFactors

    G = AnalyticGeo
    g = torch.Generator(device=device).manual_seed(seed)
    rnd = lambda *shape, s=0.02: torch.randn(*shape, generator=g, device=device) * s
    dq, dkv = G.n_heads * G.hd, G.n_kv * G.hd
    blocks, layers = [], {}
    for l in range(args.layers):
        mod = lambda w: _t.SimpleNamespace(weight=w)
        b = _t.SimpleNamespace(
            attn_norm=mod(1 + rnd(G.d_model, s=0.1)), mlp_norm=mod(1 + rnd(G.d_model, s=0.1)),
            q_proj=mod(rnd(dq, G.d_model)), k_proj=mod(rnd(dkv, G.d_model)), v_proj=mod(rnd(dkv, G.d_model)),
            o_proj=mod(rnd(G.d_model, dq)), gate_proj=mod(rnd(G.d_ff, G.d_model)), up_proj=mod(rnd(G.d_ff, G.d_model)),
            down_proj=mod(rnd(G.d_model, G.d_ff)))
        blocks.append(b)
        proj = {}
        for name, (fin, fout) in (("q_proj", (G.d_model, dq)), ("k_proj", (G.d_model, dkv)),
                                  ("v_proj", (G.d_model, dkv)), ("o_proj", (dq, G.d_model))):
            proj[name] = LowRankFactors(A=rnd(G.rank, fin, s=fin ** -0.5), B=rnd(fout, G.rank, s=1.0), scale=0.01)
        layers[l] = LayerDelta(layer_idx=l, projections=proj)
    cfg = _t.SimpleNamespace(n_heads=G.n_heads, n_kv_heads=G.n_kv, head_dim=G.hd, d_model=G.d_model, rms_eps=G.eps)
    model = _t.SimpleNamespace(cfg=cfg, blocks=blocks, rope=RotaryEmbedding(G.hd, max_seq=args.seq_len, base=G.rope_theta))
    conf = _t.SimpleNamespace(hidden_stride=G.hidden_stride, propagator_rank=G.propagator_rank)
    hidden = []
    for _ in range(args.seqs):
        h = torch.randn(args.layers, args.seq_len, G.d_model, generator=g, device=device)
        hm = torch.randn(args.layers, args.seq_len, G.d_model, generator=g, device=device)
        hidden.append((h, hm))
    return model, _t.SimpleNamespace(layers=layers), conf, hidden


def _snapshot(h, hm):
    import types as _t

    return _t.SimpleNamespace(layer_in=lambda l: h[l], layer_mid=lambda l: hm[l], seq_len=int(h.shape[1]))


def analytic_cpu_sample(seconds: float, n: int = 2048, layers: int = 1) -> dict:
    """The oracle port (numpy fp64) of the engine's analytic loop on ``layers`` layers of one
    ``n``-token sequence of the same shape, repeated for about ``seconds``."""
    from oracle import analytic as OA

    G = AnalyticGeo
    rng = np.random.default_rng(0)
    rnd = lambda *shape, s=0.02: rng.standard_normal(shape) * s
    dq, dkv = G.n_heads * G.hd, G.n_kv * G.hd
    W, Ls = [], {}
    for l in range(layers):
        W.append({"q": rnd(dq, G.d_model), "k": rnd(dkv, G.d_model), "v": rnd(dkv, G.d_model), "o": rnd(G.d_model, dq),
                  "gate": rnd(G.d_ff, G.d_model), "up": rnd(G.d_ff, G.d_model), "down": rnd(G.d_model, G.d_ff),
                  "attn_norm": 1 + rnd(G.d_model, s=0.1), "mlp_norm": 1 + rnd(G.d_model, s=0.1)})
        Ls[l] = {p: (rnd(G.rank, fin, s=fin ** -0.5), rnd(fout, G.rank, s=1.0), 0.01)
                 for p, (fin, fout) in (("q", (G.d_model, dq)), ("k", (G.d_model, dkv)), ("v", (G.d_model, dkv)),
                                        ("o", (dq, G.d_model)))}
    cfg = dict(n_heads=G.n_heads, n_kv=G.n_kv, hd=G.hd, d_model=G.d_model, eps=G.eps, rope_base=G.rope_theta,
               hidden_stride=G.hidden_stride, propagator_rank=G.propagator_rank)
    h, hm = rng.standard_normal((layers, n, G.d_model)), rng.standard_normal((layers, n, G.d_model))
    t0, done = time.perf_counter(), 0
    while True:
        OA.analytic_patches(h, hm, W, Ls, cfg)
        done += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    return {"value": done * layers * n / el, "unit": UNIT, "cores": cpu_pool_threads(), "kind": "port",
            "sample": f"{done} x ({layers} layer x {n} tokens) of the engine's analytic loop in {el:.1f} s "
                      "(oracle numpy fp64 port, attention materialised; BLAS threads for the matrix products)"}


def run_analytic_ours(args):
    from deltakv_b200 import analytic as AN
    from deltakv_b200 import ops

    world, rank, local = dist_setup(args)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    G = AnalyticGeo
    model, delta, conf, hidden = make_analytic_workload(args, dev, 7000 + rank)
    units = args.layers * args.seq_len * args.seqs
    stream = torch.cuda.current_stream()

    def step():
        for h, hm in hidden:
            AN.analytic_patches(_snapshot(h, hm), delta, model, conf)

    for _ in range(max(1, args.warmup)):
        step()
    torch.cuda.synchronize()
    ops.status_word(dev).raise_if_set("bench warm-up")
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    from deltakv_b200 import subspace as SUB

    trunc0 = SUB.gram_launches
    with ClockSampler(local) as clk:
        t_start.record(stream)
        for _ in range(args.steps):
            step()
        t_end.record(stream)
        torch.cuda.synchronize()
    trunc_launches = SUB.gram_launches - trunc0
    if world > 1:
        torch.distributed.barrier()
    ms = t_start.elapsed_time(t_end)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    ms_step = ms / args.steps
    # the attention core alone on one layer's tensors (same shapes as inside the loop)
    n = args.seq_len
    gq = torch.Generator(device=dev).manual_seed(1)
    mk = lambda hh: torch.randn(n, hh, G.hd, generator=gq, device=dev)
    qs = [mk(G.n_heads), mk(G.n_heads), mk(G.n_kv), mk(G.n_kv), mk(G.n_kv), mk(G.n_kv)]
    AN.attention_core(*qs, want_ctx=True)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 10
    e0.record(stream)
    for _ in range(reps):
        AN.attention_core(*qs, want_ctx=True)
    e1.record(stream)
    torch.cuda.synchronize()
    core_ms = e0.elapsed_time(e1) / reps
    core_flops = 2 * 6 * G.hd * (n * (n + 1) / 2) * G.n_heads  # S, dS (2), O, OS, OD MACs per causal pair
    achieved = core_flops / (core_ms / 1e3) / 1e12
    peaks = {}
    try:
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except Exception:
        pass
    bf16_peak = peaks.get("bf16_tflops") or 1590.0
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = analytic_cpu_sample(args.cpu_seconds)
    e2e = None
    if not args.no_e2e:
        # through the public API from pinned host buffers: hidden states in, the K / V patches out
        h_host = [(h.cpu().pin_memory(), hm.cpu().pin_memory()) for h, hm in hidden]
        out_bytes = 2 * args.layers * n * G.n_kv * G.hd * 4
        outs = [torch.empty(2, args.layers, n, G.n_kv, G.hd).pin_memory() for _ in hidden]

        def e2e_step():
            for (hh, hmh), o in zip(h_host, outs):
                h_d, hm_d = hh.to(dev, non_blocking=True), hmh.to(dev, non_blocking=True)
                pt = AN.analytic_patches(_snapshot(h_d, hm_d), delta, model, conf)
                o[0].copy_(torch.stack([pt[l].k_dense for l in range(args.layers)]), non_blocking=True)
                o[1].copy_(torch.stack([pt[l].v_dense for l in range(args.layers)]), non_blocking=True)

        e2e_step()  # untimed: the pinned buffers' first transfers
        torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier()
        e2 = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        e2[0].record(stream)
        e2e_step()
        e2[1].record(stream)
        torch.cuda.synchronize()
        e2e_ms = e2[0].elapsed_time(e2[1])
        if world > 1:
            t = torch.tensor([e2e_ms], device=dev)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            e2e_ms = float(t.item())
        e2e = {"value": units * world / (e2e_ms / 1e3), "unit": UNIT,
               "h2d_bytes_per_step": sum(a.numel() * 4 + b.numel() * 4 for a, b in h_host),
               "d2h_bytes_per_step": out_bytes * len(hidden), "ms_per_step": e2e_ms}
    if rank == 0:
        line = {
            "metric": ANALYTIC_METRIC, "value": units * world / (ms_step / 1e3), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": ANALYTIC_WORKLOAD, "layers": args.layers, "seqs_per_gpu": args.seqs,
                       "seq_len": n, "parallelism": f"request shards x{world}",
                       "l2": "per sequence 283 MB of stored hidden states >> 126 MB L2"},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": bf16_peak, "unit": "TFLOP/s",
                         "frac": achieved / bf16_peak, "traffic": None,
                         "peak_source": "of measured (MEASURED_PEAKS.json bf16_tflops, burst)",
                         "kernel": "attention core (dkv_attn_first_order, mma.sync bf16 three-term split), one layer",
                         "kernel_ms": core_ms, "algorithmic_flops_per_launch": core_flops,
                         # the split issues 3 bf16 products per fp32-level product; S / dS are formed by
                         # both column-half warps of a row group
                         "issued_mma_flops_per_launch": core_flops * (3 * 3 * 2 + 3 * 3) / 6,
                         "fp32_fma_equivalent": {"peak": FP32_FMA_NOMINAL_TFLOPS,
                                                 "frac": achieved / FP32_FMA_NOMINAL_TFLOPS,
                                                 "peak_source": "of nominal (148 SMs x 128 lanes x 2 x 1965 MHz)"}},
            "cpu_baseline": cpu, "e2e": e2e,
            # per layer and sequence: rmsnorm x2, rope x4, attention core, swiglu; plus the rank
            # truncations' subspace-iteration and Jacobi kernels, as counted
            "gpu_launches": args.steps * args.seqs * args.layers * 8 + trunc_launches,
            "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()
    return 0


def run_analytic_reference(args):
    world, rank, _ = dist_setup(args)
    if rank != 0:
        return 0
    res = [analytic_cpu_sample(max(2.0, args.cpu_seconds / max(1, args.steps))) for _ in range(args.steps)]
    value = sum(r["value"] for r in res) / len(res)
    line = {
        "impl": "reference", "metric": ANALYTIC_METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": None, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
        "config": {"workload": ANALYTIC_WORKLOAD, "step": res[0]["sample"]},
        "cpu_baseline": {**res[0], "value": value},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def main():
    args = parse()
    if args.workload == "analytic":
        for k, v in (("layers", AnalyticGeo.layers), ("seqs", AnalyticGeo.seqs), ("seq_len", AnalyticGeo.seq_len)):
            if getattr(args, k) is None:
                setattr(args, k, v)
        return run_analytic_reference(args) if args.impl == "reference" else run_analytic_ours(args)
    if args.workload == "multi-lora-kivi":
        for k, v in (("layers", KiviGeo.layers), ("seqs", 1), ("seq_len", KiviGeo.seq_len)):
            if getattr(args, k) is None:
                setattr(args, k, v)
        return run_kivi_reference(args) if args.impl == "reference" else run_kivi_ours(args)
    if args.workload == "smollm2-exact":
        global Geo, METRIC, WORKLOAD, BYTES_PER_UNIT
        Geo, METRIC, WORKLOAD, BYTES_PER_UNIT = SmolGeo, SMOL_METRIC, SMOL_WORKLOAD, SMOL_BYTES_PER_UNIT
    dense = args.workload == "rl-dense"
    for k, v in (("layers", DenseGeo.layers if dense else Geo.layers), ("seqs", DenseGeo.seqs if dense else Geo.seqs),
                 ("seq_len", DenseGeo.seq_len if dense else Geo.seq_len)):
        if getattr(args, k) is None:
            setattr(args, k, v)
    if dense:
        return run_dense_reference(args) if args.impl == "reference" else run_dense_ours(args)
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
