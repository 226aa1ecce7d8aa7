"""Throughput of ΔKV's cache-maintenance hot path on B200, one JSON line.

Default run (the headline): the exact/zeroth-order patch route on the Llama-3-8B-shaped cache
— 32 layers, d=4096, 8 KV heads x 128, 64 sequences x 4096 tokens, rank-16 k/v LoRA, fp8-e4m3
stored activations (per-token scale, per-row sums of squared codes stored beside them),
RMSNorm folded in, RoPE on K, bf16 paged K/V (block 16, permuted block table).  One step =
pack the factors of the layers this GPU holds, then one fused launch over its (layer,
sequence) tiles.  The same line carries a ``workloads`` object with the other measured
configurations, each with its own value, roofline, CPU baseline, end-to-end figure, parity
spot check and clocks:

* ``smollm2-exact``   exact route, SmolLM2-135M shape (30 layers, d=576, 3 KV heads x 64,
                      32 x 2048 tokens, rank-8 k/v LoRA, f16 stored activations);
* ``multi-lora-kivi`` subspace route on a KIVI int4 shared prefix (Llama-3-8B shape,
                      32768 tokens, 8 adapter views of ranks {8,8,16,16,32,32,64,64});
* ``rl-dense``        dense-dW route of an RL step (Llama-3-70B shape: 80 layers, d=8192,
                      16 x 8192 tokens, full-rank dW_K / dW_V), a tcgen05 GEMM;
* ``analytic``        the analytic route's engine loop (SmolLM2-135M shape, 30 layers, 4 x 2048
                      tokens, rank-8 q/k/v/o LoRA, propagator rank 64).

    python bench.py [--gpus N --steps K --warmup W]      # this implementation
    python bench.py --impl reference ...                   # the CPU reference arm
    python bench.py --workload NAME ...                    # one workload alone (also: analytic)

Under torchrun (N > 1) the fixed workload is split across the ranks without any data-path
collective (strong scaling): layers round-robin (layer l on rank l mod N) for the exact and
dense routes, adapter views for the int4 route (the shared base cache broadcast once over
NCCL before timing).  The per-layer error scalars are all-gathered after the timed region.
Rank 0 prints the line; ``value`` = all units of the step / the slowest rank's time.
"""

from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics
import sys
import threading
import time
import traceback
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

UNIT = "token·layers/s"


def parse(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="llama8b-exact",
                    choices=["llama8b-exact", "smollm2-exact", "rl-dense", "multi-lora-kivi", "dense-subspace",
                             "analytic"])
    ap.add_argument("--shard", default="layer", choices=["layer", "request"],
                    help="N>1 split of the exact / dense routes: layers of one fixed cache (strong "
                         "scaling) or a request shard of the same size per rank (weak scaling)")
    ap.add_argument("--adapters", type=int, default=8)
    ap.add_argument("--layers", type=int, default=None)
    ap.add_argument("--seqs", type=int, default=None)
    ap.add_argument("--seq-len", type=int, default=None)
    ap.add_argument("--e2e-seqs", type=int, default=4)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--sub-cpu-seconds", type=float, default=6.0)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-workloads", action="store_true", help="headline only (no workloads object)")
    return ap.parse_args(argv)


# ---------------------------------------------------------------------------
# ranks, timing, clocks, peaks
# ---------------------------------------------------------------------------
class Dist:
    """One process per GPU; NCCL process group when WORLD_SIZE > 1."""

    def __init__(self):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.dev = None

    def init(self):
        torch.cuda.set_device(self.local)
        self.dev = torch.device("cuda", self.local)
        if self.world > 1:
            torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=self.dev)
        return self

    def barrier(self):
        if self.world > 1:
            torch.distributed.barrier()

    def reduce(self, x: float, op) -> float:
        if self.world == 1:
            return float(x)
        t = torch.tensor([float(x)], device=self.dev, dtype=torch.float64)
        torch.distributed.all_reduce(t, op=op)
        return float(t.item())

    def max(self, x: float) -> float:
        return self.reduce(x, torch.distributed.ReduceOp.MAX if self.world > 1 else None)

    def min(self, x: float) -> float:
        return self.reduce(x, torch.distributed.ReduceOp.MIN if self.world > 1 else None)

    def finish(self):
        if self.world > 1:
            torch.distributed.destroy_process_group()


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


def timed(dist: Dist, step, steps: int, kernel_events: bool = True):
    """Exactly ``steps`` steps between a barrier + synchronize on each side; returns
    (max-over-ranks ms of the whole region, this rank's per-step kernel ms, clocks)."""
    stream = torch.cuda.current_stream()
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(dist.local) as clk:
        t0.record(stream)
        for i in range(steps):
            step(kev[i] if kernel_events else None)
        t1.record(stream)
        torch.cuda.synchronize()
    dist.barrier()
    ms = dist.max(t0.elapsed_time(t1))
    kern = [a.elapsed_time(b) for a, b in kev] if kernel_events else []
    return ms, kern, clk.summary()


def peaks() -> dict:
    try:
        return json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except Exception:
        return {}


def hbm_peak():
    p = peaks().get("hbm_gbs")
    if p:
        return p, "of measured (MEASURED_PEAKS.json hbm_gbs, burst copy)"
    return 6650.0, "of fallback (6650 GB/s)"


def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except Exception:
        pass
    return "unknown"


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_pool_threads() -> int:
    """Host threads for the CPU arm: every core, capped so each worker's ~0.5 GB of fp32
    temporaries (one 4096-token sequence of one layer) fits in free memory."""
    cores = host_threads()
    try:
        import psutil

        cap = int(psutil.virtual_memory().available * 0.6 // (512 << 20))
        return max(1, min(cores, cap))
    except Exception:
        return cores


class torch_threads:
    """torch's intra-op thread count set to `n` inside the block, restored after"""

    def __init__(self, n: int):
        self.n = n

    def __enter__(self):
        self.old = torch.get_num_threads()
        torch.set_num_threads(self.n)

    def __exit__(self, *exc):
        torch.set_num_threads(self.old)


def _pool_run(item, threads: int, seconds: float | None = None, count: int | None = None):
    """`item()` (returns units) on `threads` workers, one intra-op thread each, for `seconds` or
    `count` items; returns (units, elapsed_s)"""
    from concurrent.futures import ThreadPoolExecutor

    lock = threading.Lock()
    started = [0]
    deadline = None if seconds is None else time.perf_counter() + seconds

    def worker(_):
        u = 0
        while True:
            with lock:
                if count is not None and started[0] >= count:
                    return u
                if deadline is not None and time.perf_counter() >= deadline:
                    return u
                started[0] += 1
            u += item()

    with torch_threads(1):
        t0 = time.perf_counter()
        with ThreadPoolExecutor(threads) as ex:
            units = sum(ex.map(worker, range(threads)))
        return units, time.perf_counter() - t0


def _serial_run(item, threads: int, seconds: float | None = None, count: int | None = None):
    """`item()` one after another with `threads` intra-op threads inside each operation"""
    with torch_threads(threads):
        t0 = time.perf_counter()
        units = k = 0
        while (count is None or k < count) and (seconds is None or time.perf_counter() - t0 < seconds):
            units += item()
            k += 1
        return units, time.perf_counter() - t0


HOST_MODES = {"pool": (_pool_run, "one item per thread"),
              "serial": (_serial_run, "items in turn, every thread inside each operation")}


def host_rate(item, threads: int, seconds: float):
    """Runs `item` for `seconds` the faster of the two ways to spread it over the cores (each
    warmed up and timed on `threads` items first); returns (units, elapsed_s, mode text)."""
    rate = {}
    for mode, (run, _) in HOST_MODES.items():
        run(item, threads, count=threads)
        u, el = run(item, threads, count=threads)
        rate[mode] = u / el
    mode = max(rate, key=rate.get)
    run, text = HOST_MODES[mode]
    u, el = run(item, threads, seconds=seconds)
    return u, el, text


def my_layers(n_layers: int, dist: Dist, shard: str) -> list[int]:
    """Layer l on rank l mod N (layer sharding); every layer on every rank otherwise."""
    if dist.world == 1 or shard != "layer":
        return list(range(n_layers))
    return [l for l in range(n_layers) if l % dist.world == dist.rank]


def rel_l2(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.double(), b.double()
    return float((a - b).norm() / (b.norm() + 1e-30))


# ---------------------------------------------------------------------------
# exact route (Llama-3-8B and SmolLM2-135M shapes)
# ---------------------------------------------------------------------------
class Llama8B:
    name = "llama8b-exact"
    metric = "patched token·layers/s (Llama-8B shape, rank-16 k/v LoRA)"
    d_model, n_kv, hd, rank, bs, eps, rope_theta = 4096, 8, 128, 16, 16, 1e-5, 500000.0
    layers, seqs, seq_len = 32, 64, 4096
    x_torch, x_kind = torch.float8_e4m3fn, "e4m3"
    bytes_per_unit = 4096 + 4 + 4 + 4096 + 4096  # X fp8 + scale + sum of squares + K read/write + V read/write
    workload = ("Llama-3-8B-shaped exact patch: 32 layers, d=4096, 8 KV heads x 128, 64 seqs x 4096 tokens, "
                "rank-16 k/v LoRA (rel. norm 1e-2), fp8-e4m3 stored X + per-token scale + per-row sum of squared "
                "codes (formed when the activations are stored), RMSNorm folded, RoPE (theta 5e5), bf16 paged KV "
                "block 16, permuted block table")
    profile = "exact_patch_kernel.md"
    dtype = "f16 tensor-core products, fp32 accumulate (e4m3 X, bf16 pages)"


class Smol135M(Llama8B):
    name = "smollm2-exact"
    metric = "patched token·layers/s (SmolLM2-135M shape, rank-8 k/v LoRA)"
    d_model, n_kv, hd, rank, bs, eps, rope_theta = 576, 3, 64, 8, 16, 1e-5, 10000.0
    layers, seqs, seq_len = 30, 32, 2048
    x_torch, x_kind = torch.float16, "f16"
    bytes_per_unit = 1152 + 4 + 4 + 768 + 768  # X f16 + row scale + sum of squares + K read/write + V read/write
    workload = ("SmolLM2-135M-shaped exact patch: 30 layers, d=576, 3 KV heads x 64, 32 seqs x 2048 tokens, "
                "rank-8 k/v LoRA (rel. norm 1e-2), f16 stored X + power-of-two row scale + per-row sum of squared "
                "codes, RMSNorm folded, RoPE (theta 1e4), bf16 paged KV block 16, permuted block table")
    profile = "smollm2_exact_patch.md"
    dtype = "f16 tensor-core products, fp32 accumulate (f16 X, bf16 pages)"


def lora_scale(G) -> float:
    """LoRA scale with E||s B A||_F = 1e-2 ||W||_F for W ~ N(0, 0.02^2), A ~ N(0, 1/d), B ~ N(0, 1)
    (E||B A||_F^2 = d_kv * r): the same for every layer, whatever the split across ranks."""
    d_kv = G.n_kv * G.hd
    return 1e-2 * 0.02 * math.sqrt(d_kv * G.d_model) / math.sqrt(d_kv * G.rank)


def make_exact_workload(G, layers, n_seqs, seq_len, device, seed):
    """Synthetic inputs of the given layers; each layer's data comes from its own seed, so a
    layer holds the same values whichever rank it lands on."""
    import deltakv_b200 as dkv
    from deltakv_b200 import ops

    rows = n_seqs * seq_len
    nl = len(layers)
    d_kv = G.n_kv * G.hd
    x = None
    xs = torch.empty(nl, rows, dtype=torch.float32, device=device)
    xq = torch.empty(nl, rows, dtype=torch.float32, device=device)  # per-row sum of squared codes
    blocks_per_seq = (seq_len + G.bs - 1) // G.bs
    nb = n_seqs * blocks_per_seq
    caches = []
    a_k = torch.empty(nl, G.rank, G.d_model, device=device)
    b_k = torch.empty(nl, d_kv, G.rank, device=device)
    a_v = torch.empty_like(a_k)
    b_v = torch.empty_like(b_k)
    norm_w = torch.empty(nl, G.d_model, device=device)
    for i, l in enumerate(layers):
        gen = torch.Generator(device=device).manual_seed(seed + 7919 * l)
        # residual-stream-like rows: N(0,1) with a per-token magnitude spread
        h = torch.randn(rows, G.d_model, generator=gen, device=device)
        h *= (0.5 + torch.rand(rows, 1, generator=gen, device=device))
        q, s, ssq = dkv.quantize_rows(h, G.x_torch, with_sumsq=True)
        if x is None:
            x = torch.empty(nl, rows, q.shape[-1], dtype=q.dtype, device=device)
        x[i].copy_(q)
        xs[i].copy_(s)
        xq[i].copy_(ssq)
        del h, q, s, ssq
        c = torch.empty(2, nb, G.bs, G.n_kv, G.hd, dtype=torch.bfloat16, device=device)
        c.normal_(generator=gen)
        caches.append(c)
        a_k[i] = torch.randn(G.rank, G.d_model, generator=gen, device=device) / math.sqrt(G.d_model)
        b_k[i] = torch.randn(d_kv, G.rank, generator=gen, device=device)
        a_v[i] = torch.randn(G.rank, G.d_model, generator=gen, device=device) / math.sqrt(G.d_model)
        b_v[i] = torch.randn(d_kv, G.rank, generator=gen, device=device)
        norm_w[i] = 1.0 + 0.05 * torch.randn(G.d_model, generator=gen, device=device)
    perm = torch.randperm(nb, generator=torch.Generator().manual_seed(seed + 2)).to(torch.int32)
    tables = perm.view(n_seqs, blocks_per_seq).to(device)
    s = lora_scale(G)
    cu = torch.arange(0, n_seqs + 1, dtype=torch.int32, device=device) * seq_len
    seqs = ops.SeqBatchTensors(cu_seqlens=cu, block_tables=tables, max_seq_len=seq_len)
    rope = dkv.RotaryEmbedding(G.hd, max_seq=seq_len, base=G.rope_theta)
    return dict(x=x, xs=xs, xq=xq, caches=caches, a_k=a_k, b_k=b_k, a_v=a_v, b_v=b_v, s=s, norm_w=norm_w,
                seqs=seqs, rope=rope, tables=tables)


def exact_reference_delta(G, wl, i, r0, r1, rope_tabs):
    """Plain PyTorch fp32 restatement of the reference's exact branch for rows [r0, r1) of
    held layer i: dequantise, RMSNorm (x * rsqrt(mean(x^2) + eps) * w, src/deltakv/model.py:
    48-56), codes = s x A^T and delta = codes B^T (deltas/factors.py:61-67), RoPE on K with the
    rotate-half pairing at positions 0.. (rope.py:9-25).  Returns (dK, dV) [n, n_kv, hd] fp32."""
    n = r1 - r0
    x = wl["x"][i, r0:r1, :G.d_model].float() * wl["xs"][i, r0:r1, None]
    x = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + G.eps) * wl["norm_w"][i]
    s = wl["s"]
    dk = ((s * (x @ wl["a_k"][i].T)) @ wl["b_k"][i].T).view(n, G.n_kv, G.hd)
    dv = ((s * (x @ wl["a_v"][i].T)) @ wl["b_v"][i].T).view(n, G.n_kv, G.hd)
    cos, sin = rope_tabs
    c, sn = cos[:n, None, :], sin[:n, None, :]
    h = G.hd // 2
    k1, k2 = dk[..., :h], dk[..., h:]
    dk = torch.cat([k1 * c - k2 * sn, k2 * c + k1 * sn], dim=-1)
    return dk, dv


class CpuSample:
    """A bounded sample of the exact workload on the host: P distinct (layer, sequence)
    inputs, one private paged K/V per worker (a single sequence's blocks).  The work is the
    reference's exact branch in its own torch CPU operations (`oracle.exact_torch`)."""

    def __init__(self, G, n_inputs: int, seq_len: int, seed: int = 5):
        from oracle import exact as OX
        from oracle import exact_torch as OT

        self.G = G
        g = torch.Generator().manual_seed(seed)
        self.seq_len = seq_len
        self.inputs = []
        d_kv = G.n_kv * G.hd
        s = lora_scale(G)
        for _ in range(n_inputs):
            h = torch.randn(seq_len, G.d_model, generator=g) * (0.5 + torch.rand(seq_len, 1, generator=g))
            amax = h.abs().amax(-1).clamp_min(1e-12)
            sc = (amax / 448.0).float()
            if G.x_kind == "e4m3":
                xb = (h / sc[:, None]).to(torch.float8_e4m3fn).view(torch.uint8)
            else:
                xb = (h / sc[:, None]).to(torch.float16)
            fk = (torch.randn(G.rank, G.d_model, generator=g) / math.sqrt(G.d_model),
                  torch.randn(d_kv, G.rank, generator=g), s)
            fv = (torch.randn(G.rank, G.d_model, generator=g) / math.sqrt(G.d_model),
                  torch.randn(d_kv, G.rank, generator=g), s)
            w = 1.0 + 0.05 * torch.randn(G.d_model, generator=g)
            self.inputs.append((xb, sc, w, fk, fv))
        cos_h, sin_h = OX.rope_tables(G.hd, seq_len, G.rope_theta)
        self.rope = OT.rope_full(torch.from_numpy(cos_h), torch.from_numpy(sin_h), seq_len)
        nblk = (seq_len + G.bs - 1) // G.bs
        self.table = torch.from_numpy(np.random.default_rng(seed).permutation(nblk))
        self.nblk = nblk

    def new_pages(self):
        G = self.G
        g = torch.Generator().manual_seed(0)
        shape = (self.nblk, G.bs, G.n_kv, G.hd)
        return ((1.0 + torch.rand(shape, generator=g)).to(torch.bfloat16),
                (1.0 + torch.rand(shape, generator=g)).to(torch.bfloat16))

    def patch_one(self, i: int, kp, vp) -> int:
        """The reference's exact branch on one (layer, sequence): dequant -> RMSNorm ->
        exact_kv_patch -> materialize -> scatter_into_paged (K and V).  Returns units."""
        from oracle import exact_torch as OT

        G = self.G
        xb, s, w, fk, fv = self.inputs[i % len(self.inputs)]
        with torch.no_grad():
            x = OT.dequant_x(xb, G.x_kind, s)
            x = OT.rmsnorm(x, w, G.eps)
            dk, dv = OT.exact_kv_delta(x, fk, fv, G.n_kv, G.hd, self.rope)
            OT.scatter_into_paged(dk, kp, self.table, G.bs)
            OT.scatter_into_paged(dv, vp, self.table, G.bs)
        return self.seq_len

    def dequant_share(self, threads: int, reps: int = 2) -> float:
        """Fraction of one pair's time (all `threads` inside each operation) spent in the
        fp8/f16 dequantisation (which has no counterpart in the reference, whose activations
        are fp32)."""
        from oracle import exact_torch as OT

        kp, vp = self.new_pages()
        xb, s, *_ = self.inputs[0]
        with torch_threads(threads):
            OT.dequant_x(xb, self.G.x_kind, s)
            t0 = time.perf_counter()
            for _ in range(reps):
                OT.dequant_x(xb, self.G.x_kind, s)
            t_deq = time.perf_counter() - t0
            t0 = time.perf_counter()
            for _ in range(reps):
                self.patch_one(0, kp, vp)
            return t_deq / (time.perf_counter() - t0)

    def run(self, threads: int, seconds: float | None = None, pairs: int | None = None,
            mode: str = "pool"):
        """Process pairs for `seconds` (or `pairs` pairs); returns (units, elapsed_s).
        mode "pool": one pair per worker on `threads` workers, one intra-op thread each;
        "serial": pairs one after another, `threads` intra-op threads inside each operation."""
        from concurrent.futures import ThreadPoolExecutor

        deadline = None if seconds is None else time.perf_counter() + seconds
        if mode == "serial":
            kp, vp = self.new_pages()
            units, k = 0, 0
            with torch_threads(threads):
                t0 = time.perf_counter()
                while (pairs is None or k < pairs) and (deadline is None or time.perf_counter() < deadline):
                    units += self.patch_one(k, kp, vp)
                    k += 1
                return units, time.perf_counter() - t0
        pages = [self.new_pages() for _ in range(threads)]
        counter = [0]
        lock = threading.Lock()

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

        with torch_threads(1):
            t0 = time.perf_counter()
            with ThreadPoolExecutor(threads) as ex:
                units = sum(ex.map(worker, range(threads)))
            el = time.perf_counter() - t0
        return units, el

    def best_mode(self, threads: int) -> str:
        """The faster of the two ways to spread the sample over the cores (each warmed up and
        timed on `threads` pairs)."""
        rate = {}
        for mode in ("pool", "serial"):
            self.run(threads, pairs=threads, mode=mode)
            u, el = self.run(threads, pairs=threads, mode=mode)
            rate[mode] = u / el
        return max(rate, key=rate.get)


MODE_TEXT = {"pool": "one pair per thread", "serial": "pairs in turn, every thread inside each operation"}


def exact_cpu_baseline(G, seconds: float, seq_len: int) -> dict:
    threads = cpu_pool_threads()
    sample = CpuSample(G, n_inputs=4, seq_len=seq_len)
    share = sample.dequant_share(threads)
    mode = sample.best_mode(threads)
    units, el = sample.run(threads, seconds=seconds, mode=mode)
    return {"value": units / el, "unit": UNIT, "cores": threads, "cpu_model": cpu_model(), "kind": "port",
            "sample": f"{units // seq_len} (layer, sequence) pairs of {seq_len} tokens in {el:.1f} s (the "
                      f"reference's exact branch in its own torch CPU operations: dequant, RMSNorm, exact_kv_patch, "
                      f"materialize, scatter_into_paged; {threads} threads, {MODE_TEXT[mode]})",
            "dequant_share": share,
            "dequant_note": "fraction of a pair's time in the stored-activation dequantisation, timed on its own "
                            "(the reference keeps fp32 activations and has no such step)",
            "sumsq_note": "the CPU port forms RMSNorm's sum of squares from X; the GPU arm reads the per-row sums "
                          "stored with X"}


def run_exact(args, dist: Dist, G) -> dict:
    import deltakv_b200 as dkv
    from deltakv_b200 import metrics, ops

    dev = dist.dev
    L_total, n_seqs, n = args.layers, args.seqs, args.seq_len
    layers = my_layers(L_total, dist, args.shard)
    weak = args.shard != "layer" and dist.world > 1
    seed = 1000 + (dist.rank * 100003 if weak else 0)
    wl = make_exact_workload(G, layers, n_seqs, n, dev, seed)
    patcher = dkv.ExactPatcher(G.d_model, G.n_kv, G.hd, rank_k=G.rank, rank_v=G.rank, x_dtype=G.x_torch,
                               rope=wl["rope"], norm_eps=G.eps)
    packed = torch.empty(len(layers), patcher.packed_bytes, dtype=torch.uint8, device=dev)
    kpages = [c[0] for c in wl["caches"]]
    vpages = [c[1] for c in wl["caches"]]
    units_rank = len(layers) * n_seqs * n
    units_step = (L_total * n_seqs * n) if not weak else units_rank * dist.world
    stream = torch.cuda.current_stream()

    def pack():
        patcher.pack(wl["a_k"], wl["b_k"], wl["a_v"], wl["b_v"], wl["s"], wl["s"], norm_weight=wl["norm_w"],
                     out=packed)

    def apply():
        patcher.apply(wl["x"], packed, kpages, vpages, wl["seqs"], x_scale=wl["xs"], apply_norm=True,
                      x_sumsq=wl["xq"])

    pack()
    apply()
    torch.cuda.synchronize()
    ops.status_word(dev).raise_if_set("bench warm-up")
    # the step's two launches as CUDA graphs, replayed: the host's argument marshalling (tens to
    # a hundred microseconds of Python per call, a tenth of a SmolLM2-sized launch) stays off
    # the device timeline, as in a serving loop; the end-to-end figure below calls the Python
    # API every step
    graphs = [torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()]
    cap = torch.cuda.Stream(device=dev)
    cap.wait_stream(stream)
    for g, fn in zip(graphs, (pack, apply)):
        with torch.cuda.graph(g, stream=cap):
            fn()
    stream.wait_stream(cap)

    def step(ev=None):
        graphs[0].replay()
        if ev is not None:
            ev[0].record(stream)
        graphs[1].replay()
        if ev is not None:
            ev[1].record(stream)

    for _ in range(max(0, args.warmup - 1)):
        step()
    ms, kern, clocks = timed(dist, step, args.steps)
    ops.status_word(dev).raise_if_set("bench timed region")
    ms_step = ms / args.steps
    kmean = sum(kern) / len(kern)
    kmax = dist.max(kmean)
    achieved = units_rank * G.bytes_per_unit / (kmean / 1e3) / 1e9
    peak, peak_kind = hbm_peak()
    frac_min = dist.min(achieved / peak)
    traffic = traffic_from_profile(G.profile, units_rank)

    # --- after the timed region: one more step with sequence 0 of every held layer gathered
    # before and after it -> the parity spot check and the per-layer measured errors
    one = ops.SeqBatchTensors(cu_seqlens=wl["seqs"].cu_seqlens[:2].clone(),
                              block_tables=wl["seqs"].block_tables[:1].contiguous(), max_seq_len=n)
    nl = len(layers)
    stale_k = torch.empty(nl, n, G.n_kv, G.hd, dtype=torch.bfloat16, device=dev)
    stale_v = torch.empty_like(stale_k)
    for i in range(nl):
        ops.gather_paged(kpages[i], one, stale_k[i])
        ops.gather_paged(vpages[i], one, stale_v[i])
    step()
    local_err = metrics.measured_error_paged(kpages, vpages, stale_k, stale_v, one, check=True)
    t0 = time.perf_counter()
    if weak:  # every rank holds the same layer indices of its own cache
        full_err = metrics.gather_layer_errors(local_err).reshape(-1)
    else:
        full_err = metrics.gather_sharded_layer_errors(local_err, layers, L_total)
    torch.cuda.synchronize()
    gather_ms = 1e3 * (time.perf_counter() - t0)
    fe = full_err.cpu()
    layer_errors = {"what": "per-layer relative KV change of one patch step on sequence 0 (stale vs patched), "
                            "compose.py:147-163's formula summed from the pages",
                    "layers": int(fe.numel()), "max": float(fe.max()), "mean": float(fe.mean()),
                    "ranks": dist.world, "layers_per_rank": nl,
                    "collective": ("all_gather_into_tensor (nccl) of [layers] vectors over disjoint layer sets"
                                   if dist.world > 1 else "none (single rank)"),
                    "gather_wall_ms": gather_ms}
    parity = exact_parity(G, wl, patcher, packed, kpages, vpages, stale_k, stale_v, layers, n, dev)
    e2e = None
    if not args.no_e2e:
        e2e = run_exact_e2e(args, G, patcher, dist, layers, weak)
    del wl, kpages, vpages, stale_k, stale_v
    torch.cuda.empty_cache()
    cpu = None
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu:
        cpu = exact_cpu_baseline(G, args.cpu_seconds if G is Llama8B else args.sub_cpu_seconds, n)
    return {
        "metric": G.metric, "value": units_step / (ms_step / 1e3), "unit": UNIT, "n_gpus": dist.world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "weak" if weak else "strong", "vs_baseline": None, "dtype": G.dtype, "data": "synthetic",
        "config": {"workload": G.workload, "layers": L_total, "seqs": n_seqs, "seq_len": n,
                   "units_per_step": units_step, "layers_per_rank": nl,
                   "parallelism": (f"request shards x{dist.world} (weak)" if weak else
                                   f"layer shards x{dist.world}: layer l on rank l mod {dist.world} (strong)"),
                   "l2": f"inputs {units_rank * G.bytes_per_unit / 1e9:.1f} GB per GPU >> 126 MB L2, no flush needed",
                   "launches_per_step": 2,
                   "e2e_sample": None if e2e is None else e2e["sample"]},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": traffic, "peak_source": peak_kind, "kernel": "exact::patch_kernel_tc",
                     "kernel_ms": kmean, "kernel_ms_max_over_ranks": kmax, "frac_min_over_ranks": frac_min,
                     "algorithmic_bytes_per_unit": G.bytes_per_unit, "units_per_launch": units_rank},
        "parity": parity,
        "cpu_baseline": cpu,
        "e2e": e2e,
        "gpu_launches": 2 * args.steps,
        "clocks": clocks,
        "layer_errors": layer_errors,
    }


def traffic_from_profile(name, units_rank):
    """DRAM bytes per launch from the committed ncu summary, scaled to this launch's units
    (the summary states bytes per token-layer measured on a capture whose writes exceed L2)."""
    if not name:
        return None
    f = ROOT / "profiles" / name
    if not f.exists():
        return None
    for line in f.read_text().splitlines():
        if line.startswith("dram_bytes_per_unit:"):
            try:
                return int(float(line.split(":", 1)[1]) * units_rank)
            except ValueError:
                return None
    return None


def exact_parity(G, wl, patcher, packed, kpages, vpages, stale_k, stale_v, layers, n, dev):
    """Spot check of the timed workload: held layer 0, sequence 0, after the step above.
    (1) the bf16 pages against round_bf16(stale + delta_ref); (2) the delta alone, written by
    the same kernel into zeroed fp32 pages, against delta_ref (a plain PyTorch fp32
    restatement of the reference's exact branch)."""
    from deltakv_b200 import ops
    from deltakv_b200.rope import half_tables

    i = 0
    tabs = half_tables(wl["rope"], dev)
    one = ops.SeqBatchTensors(cu_seqlens=wl["seqs"].cu_seqlens[:2].clone(),
                              block_tables=wl["seqs"].block_tables[:1].contiguous(), max_seq_len=n)
    dk, dv = exact_reference_delta(G, wl, i, 0, n, tabs)
    got_k = torch.empty(n, G.n_kv, G.hd, dtype=torch.bfloat16, device=dev)
    got_v = torch.empty_like(got_k)
    ops.gather_paged(kpages[i], one, got_k)
    ops.gather_paged(vpages[i], one, got_v)
    out = {}
    eq, err = [], []
    for got, stale, d in ((got_k, stale_k[i], dk), (got_v, stale_v[i], dv)):
        want = (stale.float() + d).to(torch.bfloat16)
        err.append(rel_l2(got.float(), want.float()))
        eq.append(float((got.view(torch.int16) == want.view(torch.int16)).float().mean()))
    out["pages_rel_l2"] = max(err)
    out["pages_bit_equal"] = min(eq)
    # (2) delta alone into fp32 pages
    nblk = (n + G.bs - 1) // G.bs
    kp32 = torch.zeros(nblk, G.bs, G.n_kv, G.hd, device=dev)
    vp32 = torch.zeros_like(kp32)
    tab = ops.SeqBatchTensors(cu_seqlens=wl["seqs"].cu_seqlens[:2].clone(),
                              block_tables=torch.arange(nblk, dtype=torch.int32, device=dev)[None].contiguous(),
                              max_seq_len=n)
    patcher.apply(wl["x"][i:i + 1], packed[i:i + 1], [kp32], [vp32], tab, x_scale=wl["xs"][i:i + 1],
                  apply_norm=True, x_sumsq=wl["xq"][i:i + 1], check=True)
    dk_got = kp32.view(-1, G.n_kv, G.hd)[:n]
    dv_got = vp32.view(-1, G.n_kv, G.hd)[:n]
    out["delta_rel_l2"] = max(rel_l2(dk_got, dk), rel_l2(dv_got, dv))
    out["tolerance"] = 1e-3
    out["pass"] = bool(out["pages_rel_l2"] <= 1e-3 and out["delta_rel_l2"] <= 1e-3)
    out["sample"] = f"layer {layers[i]}, sequence 0 ({n} tokens), K and V"
    out["reference"] = "plain PyTorch fp32 restatement of RMSNorm -> exact_kv_patch -> materialize (+ scatter)"
    return out


def run_exact_e2e(args, G, patcher, dist: Dist, layers, weak):
    """Same metric through the public API with host buffers: every step copies the step's
    stored activations, scales, sums of squares, factors, block tables and the touched pages
    host->device, patches, and copies the pages back (pipelined by layer)."""
    from deltakv_b200 import ops

    dev = dist.dev
    n_seqs = args.e2e_seqs
    cpu = make_exact_workload(G, layers, n_seqs, args.seq_len, dev, seed=77)
    host = {
        "x": cpu["x"].view(torch.uint8).cpu().pin_memory(),
        "xs": cpu["xs"].cpu().pin_memory(),
        "xq": cpu["xq"].cpu().pin_memory(),
        "caches": torch.stack(cpu["caches"]).cpu().pin_memory(),
        "tables": cpu["tables"].cpu().pin_memory(),
        "a_k": cpu["a_k"].cpu().pin_memory(), "b_k": cpu["b_k"].cpu().pin_memory(),
        "a_v": cpu["a_v"].cpu().pin_memory(), "b_v": cpu["b_v"].cpu().pin_memory(),
        "norm_w": cpu["norm_w"].cpu().pin_memory(),
    }
    s = cpu["s"]
    del cpu
    torch.cuda.empty_cache()
    d = {k: torch.empty_like(v, device=dev) for k, v in host.items()}
    nl = len(layers)
    packed = torch.empty(nl, patcher.packed_bytes, dtype=torch.uint8, device=dev)
    cu = torch.arange(0, n_seqs + 1, dtype=torch.int32, device=dev) * args.seq_len
    stream = torch.cuda.current_stream()
    h2d = sum(v.numel() * v.element_size() for v in host.values())
    d2h = host["caches"].numel() * host["caches"].element_size()
    h2d_s, d2h_s = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    seqs = ops.SeqBatchTensors(cu_seqlens=cu, block_tables=d["tables"], max_seq_len=args.seq_len)
    small = ("tables", "a_k", "b_k", "a_v", "b_v", "norm_w")

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
            for l in range(nl):
                for k in ("x", "xs", "xq", "caches"):
                    d[k][l].copy_(host[k][l], non_blocking=True)
                e = torch.cuda.Event()
                e.record(h2d_s)
                ev_in.append(e)
        stream.wait_event(ev_small)
        patcher.pack(d["a_k"], d["b_k"], d["a_v"], d["b_v"], s, s, norm_weight=d["norm_w"], out=packed)
        xv = d["x"].view(G.x_torch)
        for l in range(nl):
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
    reps = 3
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    dist.barrier()
    a.record(stream)
    for _ in range(reps):
        step()
    b.record(stream)
    torch.cuda.synchronize()
    ms = dist.max(a.elapsed_time(b) / reps)
    # layer shards (or one GPU): all layers of the sample across the ranks; request shards: every rank's
    units = (nl * dist.world if weak else args.layers) * n_seqs * args.seq_len
    del d, host
    torch.cuda.empty_cache()
    return {"value": units / (ms / 1e3), "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "ms_per_step": ms,
            "sample": f"{n_seqs} seqs x {nl} layers per GPU ({n_seqs} of {args.seqs} sequences), pinned host "
                      "buffers, host->device / patch / device->host pipelined by layer"}


def run_exact_reference(args, G) -> dict:
    threads = cpu_pool_threads()
    sample = CpuSample(G, n_inputs=4, seq_len=args.seq_len)
    mode = sample.best_mode(threads)
    for _ in range(args.warmup):
        sample.run(threads, pairs=threads, mode=mode)
    units_tot, el_tot = 0, 0.0
    for _ in range(args.steps):
        u, el = sample.run(threads, pairs=threads, mode=mode)
        units_tot += u
        el_tot += el
    value = units_tot / el_tot
    return {
        "impl": "reference", "metric": G.metric, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * el_tot / args.steps,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": G.workload, "step": f"{threads} (layer, sequence) pairs of {args.seq_len} tokens "
                   "(bounded sample of the workload)"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "cpu_model": cpu_model(), "kind": "port",
                         "sample": f"{threads} (layer, sequence) pairs per step, the reference's exact branch in "
                                   "its own torch CPU operations (dequant, RMSNorm, exact_kv_patch, materialize, "
                                   f"scatter_into_paged), {MODE_TEXT[mode]}"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


# ---------------------------------------------------------------------------
# rl-dense workload: full-rank dW on k_proj / v_proj (tensor-core GEMM route)
# ---------------------------------------------------------------------------
class Dense70B:
    name = "rl-dense"
    metric = "patched token·layers/s (Llama-70B shape, dense dW RL step)"
    layers, seqs, seq_len, d_model, n_kv, hd, bs, rope_theta = 80, 16, 8192, 8192, 8, 128, 16, 500000.0
    x_buffers = 10  # distinct stored-X buffers; layer l reads buffer l mod 10
    layers_per_launch = 10
    workload = ("Llama-3-70B-shaped RL-step dense delta: 80 layers, d=8192, 8 KV heads x 128, 16 seqs x 8192 "
                "tokens, bf16 stored X (post-norm), full-rank dW_K/dW_V Gaussian with ||dW||/||W|| = 1e-3, RoPE "
                "(theta 5e5) on K, bf16 paged KV block 16, permuted block table")


def dense_flops_per_unit() -> float:
    G = Dense70B
    return 2.0 * G.d_model * 2 * G.n_kv * G.hd


def make_dense_workload(layers, n_seqs, seq_len, device, seed, x_buffers: int | None = None):
    """Pages and dW of the given layers (per-layer seeds) and the stored X.  The 80 layers'
    X would take 172 GB; ``x_buffers`` distinct [tokens, d] buffers stand in for it and
    layer l reads buffer l mod x_buffers (2.1 GB each, far beyond L2, so every layer's
    launch still streams its X from HBM)."""
    import deltakv_b200 as dkv
    from deltakv_b200 import ops

    G = Dense70B
    rows = n_seqs * seq_len
    d_kv = G.n_kv * G.hd
    nxb = x_buffers or len(layers)
    x = torch.empty(nxb, rows, G.d_model, dtype=torch.bfloat16, device=device)
    for j in range(nxb):
        x[j].normal_(generator=torch.Generator(device=device).manual_seed(seed + 31 * j))
    sigma = 1e-3 * 0.02  # ||dW|| / ||W|| = 1e-3 for W ~ N(0, 0.02^2)
    nl = len(layers)
    dw_k = torch.empty(nl, d_kv, G.d_model, dtype=torch.bfloat16, device=device)
    dw_v = torch.empty_like(dw_k)
    blocks_per_seq = (seq_len + G.bs - 1) // G.bs
    nb = n_seqs * blocks_per_seq
    caches = []
    for i, l in enumerate(layers):
        gen = torch.Generator(device=device).manual_seed(seed + 7919 * (l + 1))
        dw_k[i] = (torch.randn(d_kv, G.d_model, generator=gen, device=device) * sigma).to(torch.bfloat16)
        dw_v[i] = (torch.randn(d_kv, G.d_model, generator=gen, device=device) * sigma).to(torch.bfloat16)
        c = torch.empty(2, nb, G.bs, G.n_kv, G.hd, dtype=torch.bfloat16, device=device)
        c.normal_(generator=gen)
        caches.append(c)
    perm = torch.randperm(nb, generator=torch.Generator().manual_seed(seed + 2)).to(torch.int32)
    tables = perm.view(n_seqs, blocks_per_seq).to(device)
    cu = torch.arange(0, n_seqs + 1, dtype=torch.int32, device=device) * seq_len
    seqs = ops.SeqBatchTensors(cu_seqlens=cu, block_tables=tables, max_seq_len=seq_len)
    rope = dkv.RotaryEmbedding(G.hd, max_seq=seq_len, base=G.rope_theta)
    return dict(x=x, dw_k=dw_k, dw_v=dw_v, caches=caches, seqs=seqs, rope=rope, tables=tables)


class DenseCpuSample:
    """Bounded host sample of the dense route: (layer, 256-token chunk) items through the
    reference's exact route with A = dW, B = I in its torch CPU operations (`oracle.exact_torch`)."""

    CHUNK = 256

    def __init__(self, seed: int = 5):
        from oracle import exact as OX
        from oracle import exact_torch as OT

        G = Dense70B
        g = torch.Generator().manual_seed(seed)
        d_kv = G.n_kv * G.hd
        self.x = torch.randn(self.CHUNK, G.d_model, generator=g).to(torch.bfloat16).float()
        sig = 1e-3 * 0.02
        eye = torch.eye(d_kv)
        self.fk = (torch.randn(d_kv, G.d_model, generator=g) * sig, eye, 1.0)
        self.fv = (torch.randn(d_kv, G.d_model, generator=g) * sig, eye, 1.0)
        cos_h, sin_h = OX.rope_tables(G.hd, self.CHUNK, G.rope_theta)
        self.rope = OT.rope_full(torch.from_numpy(cos_h), torch.from_numpy(sin_h), self.CHUNK)
        self.nblk = self.CHUNK // G.bs
        self.table = torch.from_numpy(np.random.default_rng(seed).permutation(self.nblk))
        self.pages = threading.local()

    def item(self) -> int:
        from oracle import exact_torch as OT

        G = Dense70B
        pg = getattr(self.pages, "kv", None)
        if pg is None:  # one private paged K / V per worker thread
            shape = (self.nblk, G.bs, G.n_kv, G.hd)
            pg = self.pages.kv = ((1.0 + torch.rand(shape)).to(torch.bfloat16),
                                  (1.0 + torch.rand(shape)).to(torch.bfloat16))
        with torch.no_grad():
            dk, dv = OT.exact_kv_delta(self.x, self.fk, self.fv, G.n_kv, G.hd, self.rope)
            OT.scatter_into_paged(dk, pg[0], self.table, G.bs)
            OT.scatter_into_paged(dv, pg[1], self.table, G.bs)
        return self.CHUNK

    def measure(self, threads: int, seconds: float) -> dict:
        u, el, how = host_rate(self.item, threads, seconds)
        return {"value": u / el, "unit": UNIT, "cores": threads, "cpu_model": cpu_model(), "kind": "port",
                "sample": f"{u // self.CHUNK} (layer, {self.CHUNK}-token chunk) items in {el:.1f} s (the "
                          f"reference's exact route with A=dW, B=I in its torch CPU operations: x @ dW^T, RoPE, "
                          f"scatter_into_paged; {threads} threads, {how})"}


def run_dense_reference(args) -> dict:
    threads = host_threads()
    sample = DenseCpuSample()
    res = [sample.measure(threads, max(2.0, args.cpu_seconds / max(1, args.steps))) for _ in range(args.steps)]
    value = sum(r["value"] for r in res) / len(res)
    return {
        "impl": "reference", "metric": Dense70B.metric, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": None,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": Dense70B.workload, "step": res[0]["sample"]},
        "cpu_baseline": {**res[0], "value": value},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def run_dense(args, dist: Dist) -> dict:
    import deltakv_b200 as dkv
    from deltakv_b200 import ops
    from deltakv_b200.rope import half_tables

    G = Dense70B
    dev = dist.dev
    weak = args.shard != "layer" and dist.world > 1
    layers = my_layers(args.layers, dist, args.shard)
    nl = len(layers)
    per = min(G.layers_per_launch, nl)
    nxb = min(G.x_buffers, per)
    wl = make_dense_workload(layers, args.seqs, args.seq_len, dev,
                             seed=2000 + (dist.rank * 100003 if weak else 0), x_buffers=nxb)
    patcher = dkv.DensePatcher(G.d_model, G.n_kv, G.hd, rope=wl["rope"])
    packed = torch.empty(nl, 2 * G.n_kv * G.hd, G.d_model, dtype=torch.bfloat16, device=dev)
    kpages = [c[0] for c in wl["caches"]]
    vpages = [c[1] for c in wl["caches"]]
    units_rank = nl * args.seqs * args.seq_len
    units_step = units_rank * dist.world if weak else args.layers * args.seqs * args.seq_len
    stream = torch.cuda.current_stream()
    groups = [list(range(j, min(j + per, nl))) for j in range(0, nl, per)]

    def step(ev=None):
        patcher.pack(wl["dw_k"], wl["dw_v"], out=packed)
        if ev is not None:
            ev[0].record(stream)
        for grp in groups:  # each launch: `per` layers, layer g reads X buffer g mod nxb
            patcher.apply(wl["x"][:len(grp)], packed[grp[0]:grp[-1] + 1], kpages[grp[0]:grp[-1] + 1],
                          vpages[grp[0]:grp[-1] + 1], wl["seqs"])
        if ev is not None:
            ev[1].record(stream)

    step()
    torch.cuda.synchronize()
    ops.status_word(dev).raise_if_set("bench warm-up")
    for _ in range(max(0, args.warmup - 1)):
        step()
    ms, kern, clocks = timed(dist, step, args.steps)
    ops.status_word(dev).raise_if_set("bench timed region")
    ms_step = ms / args.steps
    kmean = sum(kern) / len(kern)
    achieved = units_rank * dense_flops_per_unit() / (kmean / 1e3) / 1e12
    pk = peaks()
    burst = pk.get("bf16_tflops") or 1590.0
    sustained = pk.get("bf16_tflops_sustained") or 1400.0
    src = "of measured (MEASURED_PEAKS.json bf16_tflops, burst)" if pk.get("bf16_tflops") else "of fallback (1590)"
    parity = dense_parity(G, wl, patcher, packed, kpages, vpages, layers, args.seq_len, dev)
    e2e = None
    if not args.no_e2e:
        e2e = run_dense_e2e(args, patcher, dist, weak)
    del wl, kpages, vpages
    torch.cuda.empty_cache()
    cpu = None
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu:
        cpu = DenseCpuSample().measure(host_threads(), args.sub_cpu_seconds)
    return {
        "metric": G.metric, "value": units_step / (ms_step / 1e3), "unit": UNIT, "n_gpus": dist.world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "weak" if weak else "strong", "vs_baseline": None,
        "dtype": "bf16 tensor-core products, fp32 accumulate (bf16 X and pages)", "data": "synthetic",
        "config": {"workload": G.workload, "layers": args.layers, "seqs": args.seqs, "seq_len": args.seq_len,
                   "units_per_step": units_step, "layers_per_rank": nl,
                   "parallelism": (f"request shards x{dist.world} (weak)" if weak else
                                   f"layer shards x{dist.world}: layer l on rank l mod {dist.world} (strong)"),
                   "stored_x": f"{nxb} distinct X buffers on this GPU, held layer i reads buffer i mod {nxb} "
                               "(the 80 layers' X would not fit: 172 GB)",
                   "l2": f"X {args.seqs * args.seq_len * G.d_model * 2 / 1e9:.1f} GB per buffer >> 126 MB L2",
                   "launches_per_step": 1 + len(groups),
                   "e2e_sample": None if e2e is None else e2e["sample"]},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": burst, "unit": "TFLOP/s",
                     "frac": achieved / burst, "peak_source": src,
                     "frac_of_sustained": achieved / sustained,
                     "sustained_peak": sustained, "traffic": traffic_from_profile("dense_patch_kernel.md", units_rank),
                     "kernel": "dense_patch_kernel", "kernel_ms": kmean,
                     "algorithmic_flops_per_unit": dense_flops_per_unit(), "units_per_step_this_gpu": units_rank},
        "parity": parity,
        "cpu_baseline": cpu,
        "e2e": e2e,
        "gpu_launches": (1 + len(groups)) * args.steps,
        "clocks": clocks,
    }


def dense_parity(G, wl, patcher, packed, kpages, vpages, layers, n, dev):
    """Spot check: held layer 0, sequence 0 — the delta written by the same kernel in store
    mode into f16 pages against a plain PyTorch fp32 x @ dW^T (+ RoPE on K)."""
    from deltakv_b200 import ops
    from deltakv_b200.rope import half_tables

    i = 0
    x = wl["x"][0, :n].float()
    d_kv = G.n_kv * G.hd
    dk = (x @ wl["dw_k"][i].float().T).view(n, G.n_kv, G.hd)
    dv = (x @ wl["dw_v"][i].float().T).view(n, G.n_kv, G.hd)
    cos, sin = half_tables(wl["rope"], dev)
    h = G.hd // 2
    c, sn = cos[:n, None, :], sin[:n, None, :]
    dk = torch.cat([dk[..., :h] * c - dk[..., h:] * sn, dk[..., h:] * c + dk[..., :h] * sn], dim=-1)
    nblk = (n + G.bs - 1) // G.bs
    kp = torch.zeros(nblk, G.bs, G.n_kv, G.hd, dtype=torch.float16, device=dev)
    vp = torch.zeros_like(kp)
    tab = ops.SeqBatchTensors(cu_seqlens=wl["seqs"].cu_seqlens[:2].clone(),
                              block_tables=torch.arange(nblk, dtype=torch.int32, device=dev)[None].contiguous(),
                              max_seq_len=n)
    patcher.apply(wl["x"][0:1], packed[i:i + 1], [kp], [vp], tab, accumulate=False, check=True)
    err = max(rel_l2(kp.view(-1, G.n_kv, G.hd)[:n].float(), dk), rel_l2(vp.view(-1, G.n_kv, G.hd)[:n].float(), dv))
    return {"delta_rel_l2": err, "tolerance": 1e-3, "pass": bool(err <= 1e-3),
            "sample": f"layer {layers[i]}, sequence 0 ({n} tokens), K and V, store mode into f16 pages",
            "reference": "plain PyTorch fp32 x @ dW^T with rotate-half RoPE on K"}


def run_dense_e2e(args, patcher, dist: Dist, weak):
    """Same metric through DensePatcher with pinned host buffers: X, dW, tables and pages
    copied in, pages copied back, every step (1 layer x 2 sequences per GPU)."""
    from deltakv_b200 import ops

    dev = dist.dev
    n_layers, n_seqs = 1, 2
    cpu = make_dense_workload([0], n_seqs, args.seq_len, dev, seed=78)
    host = {k: cpu[k].cpu().pin_memory() for k in ("x", "dw_k", "dw_v", "tables")}
    host["caches"] = torch.stack(cpu["caches"]).cpu().pin_memory()
    del cpu
    torch.cuda.empty_cache()
    d = {k: torch.empty_like(v, device=dev) for k, v in host.items()}
    G = Dense70B
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
    reps = 3
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    dist.barrier()
    a.record(stream)
    for _ in range(reps):
        step()
    b.record(stream)
    torch.cuda.synchronize()
    ms = dist.max(a.elapsed_time(b) / reps)
    units = n_layers * n_seqs * args.seq_len * dist.world
    del d, host
    torch.cuda.empty_cache()
    return {"value": units / (ms / 1e3), "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "ms_per_step": ms, "sample": f"{n_seqs} seqs x {n_layers} layer per GPU, pinned host buffers"}


# ---------------------------------------------------------------------------
# multi-lora-kivi workload: int4 KIVI shared prefix corrected per adapter view
# ---------------------------------------------------------------------------
KIVI_METRIC = "patched token·layers/s (Llama-8B shape, int4 KIVI prefix, subspace route per adapter view)"
KIVI_WORKLOAD = ("Multi-LoRA shared prefix on the Llama-3-8B shape: 32 layers, 8 KV heads x 128, one 32768-token "
                 "prefix stored KIVI int4 (K per-channel, V per-token, group 32, fp16 scale/zero); 8 adapter views "
                 "with k/v ranks {8,8,16,16,32,32,64,64}; per view and layer: K basis = top-r right singular "
                 "subspace of the probe residual, V basis = the adapter's LoRA B; probes 10 %; dequant -> subspace "
                 "correction -> requant into the view's own int4 cache")
KIVI_BYTES_PER_UNIT = 1024 + 256 + 4096 + 1024 + 256  # base int4 K+V, scale/zero, fresh bf16 K+V, out int4, scale/zero
KIVI_RANKS = (8, 8, 16, 16, 32, 32, 64, 64)


class KiviGeo:
    layers, seq_len, n_kv, hd, probe_ratio = 32, 32768, 8, 128, 0.10


def kivi_owner(n_views: int, world: int) -> dict[int, int]:
    """Adapter views dealt to ranks in a snake order of their rank (8, 8, 16, 16, ...), so each
    GPU gets a similar mix of cheap and costly views."""
    order = sorted(range(n_views), key=lambda v: (KIVI_RANKS[v % len(KIVI_RANKS)], v))
    owner = {}
    for i, v in enumerate(order):
        cyc, pos = divmod(i, world)
        owner[v] = pos if cyc % 2 == 0 else world - 1 - pos
    return owner


def make_kivi_base(args, dist: Dist):
    """The shared int4 prefix: made on rank 0 and broadcast once over NCCL to the others."""
    from deltakv_b200 import kivi as K

    G = KiviGeo
    dev = dist.dev
    n, d = args.seq_len, G.n_kv * G.hd
    base = []
    if dist.rank == 0:
        gen = torch.Generator(device=dev).manual_seed(4000)
        for _ in range(args.layers):
            kv = []
            for mode in ("k", "v"):
                x = torch.randn(n, d, generator=gen, device=dev)
                kv.append(K.quantize(x, mode))
                del x
            base.append(kv)
    else:
        base = [[K.KiviTensor.empty(n, d, mode, dev) for mode in ("k", "v")] for _ in range(args.layers)]
    if dist.world > 1:
        for kv in base:
            for t in kv:
                for part in (t.codes, t.scale, t.zero):
                    torch.distributed.broadcast(part, src=0)
        torch.cuda.synchronize()
    return base


def make_kivi_views(args, base, dev, view_ids):
    """Per adapter view: fresh bf16 K/V per layer, V basis, probes.  fresh = dequant(base) +
    rank-r structure + 10 % drift on the non-probes."""
    from deltakv_b200 import kivi as K

    G = KiviGeo
    n, d = args.seq_len, G.n_kv * G.hd
    n_p = int(round(G.probe_ratio * n))
    adapters = []
    for a in view_ids:
        r = KIVI_RANKS[a % len(KIVI_RANKS)]
        g = torch.Generator(device=dev).manual_seed(5000 + a)
        probes = torch.unique(torch.cat([torch.zeros(1, dtype=torch.long, device=dev),
                                         torch.randperm(n, generator=g, device=dev)[: n_p - 1]]))
        layers = []
        for l in range(args.layers):
            views = []
            for m, mode in enumerate(("k", "v")):
                B = torch.randn(d, r, generator=g, device=dev) / math.sqrt(d)
                codes = torch.randn(n, r, generator=g, device=dev) * 0.5
                fresh = K.dequantize(base[l][m])
                fresh += codes @ B.T
                drift = 0.1 * fresh.std() * torch.randn(n, d, generator=g, device=dev)
                drift[probes] = 0
                fresh += drift
                views.append({"fresh": fresh.to(torch.bfloat16), "basis": B if mode == "v" else None,
                              "out": K.KiviTensor.empty(n, d, mode, dev)})
                del codes, drift, fresh
            layers.append(views)
        adapters.append({"id": a, "rank": r, "probes": probes, "layers": layers})
    return adapters


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


def kivi_parity(base, adapter) -> dict:
    """One problem of the timed work (the view's layer 0, V) corrected alone into a fresh int4
    cache and checked against a plain PyTorch fp32 restatement of the composition the oracle
    pins: KIVI dequantise -> subspace_correct (src/deltakv/patches/subspace.py:45-106) ->
    KIVI quantise (scale = fp16((max - min) / 15), zero = fp16(min), q = rint((x - zero) /
    scale) clamped to [0, 15]).  Codes agree except next to rounding ties."""
    from deltakv_b200 import kivi as K

    view, b = adapter["layers"][0][1], base[0][1]
    n, d = b.n_tokens, b.d
    out = K.KiviTensor.empty(n, d, "v", b.codes.device)
    pb = K.SubspaceProblem(base=b, fresh=view["fresh"], probe_index=adapter["probes"], basis=view["basis"],
                           rank=adapter["rank"], out=out)
    K.subspace_correct([pb], check=True)

    def unpack(c):
        c = c.to(torch.int32)
        return torch.stack([c & 15, c >> 4], dim=-1).flatten(1).float()

    g = 32
    reused = (unpack(b.codes).view(n, d // g, g) * b.scale.float()[..., None] + b.zero.float()[..., None]).view(n, d)
    fresh = view["fresh"].float().view(n, d)
    idx = torch.unique(adapter["probes"].long())
    B = view["basis"].float()
    R = fresh - reused
    G = (B.double().T @ B.double() + 1e-6 * torch.eye(B.shape[1], device=B.device, dtype=torch.float64))
    codes = torch.linalg.solve(G, (R @ B).double().T).T.float()
    fitted = codes @ B.T
    mu = (R[idx] - fitted[idx]).mean(0)
    dist_ = R.norm(dim=-1)
    w = (dist_ / dist_.mean().clamp_min(1e-8)).clamp(max=1.0)
    corr = reused + fitted + w[:, None] * mu[None]
    corr[idx] = fresh[idx]
    grp = corr.view(n, d // g, g)
    lo, hi = grp.min(-1).values, grp.max(-1).values
    s16 = ((hi - lo).clamp_min(1e-8) / 15).half()
    z16 = lo.half()
    q = torch.where(s16.float()[..., None] > 0, torch.round((grp - z16.float()[..., None]) / s16.float()[..., None]),
                    torch.zeros_like(grp)).clamp(0, 15).view(n, d)
    got = unpack(out.codes)
    codes_eq = float((got == q).float().mean())
    sz_eq = float(((out.scale == s16) & (out.zero == z16)).float().mean())
    return {"codes_equal": codes_eq, "scale_zero_equal": sz_eq, "pass": codes_eq >= 0.999,
            "tolerance": "codes equal on >= 99.9 % (the rest at rounding ties)",
            "sample": f"view {adapter['id']} (rank {adapter['rank']}), layer 0, V ({n} tokens)",
            "reference": "plain PyTorch fp32 restatement of dequantise -> subspace_correct -> quantise"}


def kivi_e2e(args, base, adapter, dist: Dist, stream, n_layers: int = 4) -> dict:
    """The same metric through the public call from pinned host buffers, on a bounded sample:
    one adapter view's first ``n_layers`` layers — its fresh bf16 K / V copied in, corrected by
    ``subspace_correct_views``, the corrected int4 K / V (codes, scales, zeros) copied out; the
    shared base cache stays resident."""
    from deltakv_b200 import kivi as K

    dev = dist.dev
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
    dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 3
    a.record(stream)
    for _ in range(reps):
        step()
    b.record(stream)
    torch.cuda.synchronize()
    ms = dist.max(a.elapsed_time(b) / reps)
    units = nl * args.seq_len * dist.world
    return {"value": units / (ms / 1e3), "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "ms_per_step": ms, "sample": f"1 adapter view (rank {adapter['rank']}) x {nl} layers x "
                                        f"{args.seq_len} tokens per GPU, pinned host buffers"}


def run_kivi(args, dist: Dist) -> dict:
    from deltakv_b200 import kivi as K
    from deltakv_b200 import ops

    dev = dist.dev
    n_views = max(1, args.adapters)
    owner = kivi_owner(n_views, dist.world)
    mine = [v for v in range(n_views) if owner[v] == dist.rank]
    base = make_kivi_base(args, dist)
    adapters = make_kivi_views(args, base, dev, mine)
    units_rank = args.layers * args.seq_len * len(mine)
    units_step = args.layers * args.seq_len * n_views
    stream = torch.cuda.current_stream()
    problems = [kivi_problems(base, ad) for ad in adapters]

    def step(ev=None):
        # all held views; view v + 1's K bases overlap view v's route (side stream)
        if problems:
            K.subspace_correct_views(problems, check=False)

    step()
    torch.cuda.synchronize()
    ops.status_word(dev).raise_if_set("bench warm-up")
    for _ in range(max(0, args.warmup - 1)):
        step()
    ms, _, clocks = timed(dist, step, args.steps, kernel_events=False)
    # the two halves alone (after the timed region, same work, one stream): K bases, route
    split = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    per_view = [torch.cuda.Event(enable_timing=True) for _ in range(len(problems) + 1)]
    n_split = 2
    basis_ms = route_ms = host_ms = 0.0
    view_ms = [0.0] * len(problems)
    for it in range(n_split + 1):  # the first pass warms the main stream's allocator pool
        split[0].record(stream)
        kbs = [K.k_bases(pb) for pb in problems]
        split[1].record(stream)
        per_view[0].record(stream)
        h0 = time.perf_counter()
        for j, (pb, kb) in enumerate(zip(problems, kbs)):
            K.subspace_correct(pb, check=False, bases=kb)
            per_view[j + 1].record(stream)
        h1 = time.perf_counter()
        split[2].record(stream)
        torch.cuda.synchronize()
        if it:
            host_ms += (h1 - h0) * 1e3 / n_split
            basis_ms += split[0].elapsed_time(split[1]) / n_split
            route_ms += split[1].elapsed_time(split[2]) / n_split
            for j in range(len(problems)):
                view_ms[j] += per_view[j].elapsed_time(per_view[j + 1]) / n_split
    ops.status_word(dev).raise_if_set("bench timed region")
    ms_step = ms / args.steps
    achieved = units_rank * KIVI_BYTES_PER_UNIT / (route_ms / 1e3) / 1e9 if route_ms > 0 else 0.0
    peak, peak_kind = hbm_peak()
    cpu = None
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu:
        cpu = kivi_cpu_sample(args.sub_cpu_seconds)
    parity = kivi_parity(base, adapters[0]) if adapters else None
    e2e = None
    if not args.no_e2e and adapters:
        e2e = kivi_e2e(args, base, adapters[0], dist, stream)
    del problems, adapters, base
    torch.cuda.empty_cache()
    return {
        "metric": KIVI_METRIC, "value": units_step / (ms_step / 1e3), "unit": UNIT, "n_gpus": dist.world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "int4 KIVI cache, bf16 tensor-core products, fp32 accumulate",
        "data": "synthetic",
        "config": {"workload": KIVI_WORKLOAD, "layers": args.layers, "prefix_tokens": args.seq_len,
                   "adapter_views": n_views, "views_this_gpu": mine,
                   "ranks_this_gpu": [KIVI_RANKS[v % len(KIVI_RANKS)] for v in mine],
                   "units_per_step": units_step,
                   "parallelism": f"adapter shards x{dist.world} (base int4 cache broadcast once over NCCL)",
                   "l2": f"{units_rank * KIVI_BYTES_PER_UNIT / 1e9:.1f} GB per step per GPU >> 126 MB L2",
                   "k_basis_ms_per_step": basis_ms, "subspace_route_ms_per_step": route_ms,
                   "route_ms_per_view": [round(x, 3) for x in view_ms],
                   "route_host_enqueue_ms_per_step": host_ms,
                   "e2e_sample": None if e2e is None else e2e["sample"]},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": None, "peak_source": peak_kind,
                     "kernel": "int4 subspace route (flags, pack, pass1 x2, psum, solve, fitb, pass2 x2) per view",
                     "kernel_ms": route_ms, "algorithmic_bytes_per_unit": KIVI_BYTES_PER_UNIT},
        "parity": parity,
        "cpu_baseline": cpu,
        "e2e": e2e,
        # per view: flags, pack, pass1 K/V, psum, solve, fitb, pass2 K/V (9) + the K bases'
        # batched probe residual and Jacobi eigensolver (2); library calls not counted
        "gpu_launches": args.steps * len(mine) * 11,
        "clocks": clocks,
    }


def kivi_cpu_sample(seconds: float, n: int = 4096) -> dict:
    """The route on the host (dequantise, subspace_correct, requantise; K and V of one (layer,
    view) of `n` tokens per item) in the reference's torch CPU operations (`oracle.subspace_torch`)."""
    from oracle import subspace_torch as OST

    G = KiviGeo
    d = G.n_kv * G.hd
    g = torch.Generator().manual_seed(7)
    B = torch.randn(d, 16, generator=g) / math.sqrt(d)
    probes = torch.unique(torch.cat([torch.zeros(1, dtype=torch.int64), torch.randperm(n, generator=g)[: n // 10]]))
    problems = []
    for mode in ("k", "v"):
        base = OST.quantize(torch.randn(n, d, generator=g), mode)
        fresh = OST.dequantize(*base, mode) + (torch.randn(n, 16, generator=g) * 0.5) @ B.T
        problems.append((mode, base, fresh))
    threads = host_threads()

    def item():
        with torch.no_grad():
            for mode, base, fresh in problems:
                corr, _, _ = OST.subspace_correct(OST.dequantize(*base, mode), fresh, probes, B)
                OST.quantize(corr, mode)
        return n

    units, el, how = host_rate(item, threads, seconds)
    return {"value": units / el, "unit": UNIT, "cores": threads, "cpu_model": cpu_model(), "kind": "port",
            "sample": f"{units // n} (layer, view) items of {n} tokens (K and V), rank 16, in {el:.1f} s (the "
                      f"route in the reference's torch CPU operations: dequant, subspace_correct, requant; "
                      f"{threads} threads, {how})"}


def run_kivi_reference(args) -> dict:
    res = [kivi_cpu_sample(max(2.0, args.cpu_seconds / max(1, args.steps))) for _ in range(args.steps)]
    value = sum(r["value"] for r in res) / len(res)
    return {
        "impl": "reference", "metric": KIVI_METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": None, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": KIVI_WORKLOAD, "step": res[0]["sample"]},
        "cpu_baseline": {**res[0], "value": value},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


# ---------------------------------------------------------------------------
# subspace route on a dense bf16 cache: the probe path's per-layer K / V correction
# ---------------------------------------------------------------------------
DSUB_METRIC = "patched token·layers/s (subspace route on a bf16 KV cache, Llama-8B shape)"


class DsubGeo:
    layers, seq_len, n_kv, hd, rank, probe_ratio = 32, 32768, 8, 128, 16, 0.10


# K and V per token·layer: read reused + fresh, write corrected, bf16, d = n_kv * hd
DSUB_BYTES_PER_UNIT = 2 * 3 * DsubGeo.n_kv * DsubGeo.hd * 2
DSUB_WORKLOAD = ("Subspace route (subspace_correct) on a dense bf16 KV cache, Llama-3-8B shape: 32 layers x (K, V), "
                 "8 KV heads x 128, one 32768-token sequence, rank-16 bases (V: the adapter's LoRA B; K: a given "
                 "top-16 basis), 10 % probes; each rank's layers in one dkv_subspace_correct_batched call per step")


def make_dsub_problems(args, dist: Dist, layer_ids) -> list[dict]:
    """Per layer a K and a V problem from the layer's own seed: reused ~ N(0, 1) bf16, fresh =
    reused + codes B^T (B orthonormal, rank 16) + 1 % noise, bf16; one shared probe set."""
    G = DsubGeo
    d, n, dev = G.n_kv * G.hd, args.seq_len, dist.dev
    pg = torch.Generator(device=dev).manual_seed(4999)
    probes = torch.randperm(n, generator=pg, device=dev)[: int(G.probe_ratio * n)].sort().values
    probs = []
    for l in layer_ids:
        gen = torch.Generator(device=dev).manual_seed(5000 + 7919 * l)
        for _ in range(2):
            reused = torch.randn(n, G.n_kv, G.hd, generator=gen, device=dev).to(torch.bfloat16)
            B = torch.linalg.qr(torch.randn(d, G.rank, generator=gen, device=dev))[0].contiguous()
            codes = torch.randn(n, G.rank, generator=gen, device=dev) * 0.3
            noise = 0.01 * torch.randn(n, d, generator=gen, device=dev)
            fresh = (reused.float().view(n, d) + codes @ B.T + noise).view(n, G.n_kv, G.hd).to(torch.bfloat16)
            del codes, noise
            probs.append(dict(reused=reused, fresh=fresh, probe_index=probes, basis=B, rank=G.rank))
    return probs


def dsub_parity(probs) -> dict:
    """One problem of the timed batch (layer 0's V) recomputed by a plain PyTorch fp32
    restatement of subspace_correct (src/deltakv/patches/subspace.py:45-106) and compared."""
    import deltakv_b200 as dkv

    p = probs[1]
    got = dkv.subspace_correct_batched([p])[0][0].float()
    rf, ff = p["reused"].float().flatten(1), p["fresh"].float().flatten(1)
    idx, B = p["probe_index"], p["basis"]
    R = ff - rf
    codes = torch.linalg.solve(B.T @ B + 1e-6 * torch.eye(B.shape[1], device=B.device), (R @ B).T).T
    fitted = codes @ B.T
    mu = (R[idx] - fitted[idx]).mean(0)
    dist_ = R.norm(dim=-1)
    w = (dist_ / dist_.mean().clamp_min(1e-8)).clamp(max=1.0)
    ref = rf + fitted + w[:, None] * mu[None]
    ref[idx] = ff[idx]
    ref = ref.to(torch.bfloat16).float()
    err = float((got.flatten(1) - ref).norm() / ref.norm())
    return {"corrected_rel_l2": err, "tolerance": 2e-3, "pass": err < 2e-3,
            "sample": "layer 0, V (32768 tokens)", "reference": "plain PyTorch fp32 restatement of subspace_correct"}


def dsub_cpu_sample(seconds: float, n: int = 4096) -> dict:
    """subspace_correct on the host (K and V of one layer of `n` tokens per item) in the
    reference's torch CPU operations (`oracle.subspace_torch`)."""
    from oracle import subspace_torch as OST

    G = DsubGeo
    d = G.n_kv * G.hd
    g = torch.Generator().manual_seed(11)
    probes = torch.sort(torch.randperm(n, generator=g)[: int(G.probe_ratio * n)]).values
    problems = []
    for _ in range(2):
        reused = torch.randn(n, d, generator=g)
        B = torch.linalg.qr(torch.randn(d, G.rank, generator=g))[0]
        problems.append((reused, reused + (torch.randn(n, G.rank, generator=g) * 0.3) @ B.T, B))
    threads = host_threads()

    def item():
        with torch.no_grad():
            for reused, fresh, B in problems:
                OST.subspace_correct(reused, fresh, probes, B)
        return n

    units, el, how = host_rate(item, threads, seconds)
    return {"value": units / el, "unit": UNIT, "cores": threads, "cpu_model": cpu_model(), "kind": "port",
            "sample": f"{units // n} layers of {n} tokens (K and V), rank 16, in {el:.1f} s (subspace_correct in "
                      f"the reference's torch CPU operations; {threads} threads, {how})"}


def dsub_e2e(args, probs, dist: Dist, stream, n_layers: int = 4) -> dict:
    """The same metric through the public call from pinned host buffers on a bounded sample:
    the first `n_layers` layers' reused and fresh K / V copied in, corrected, copied out."""
    import deltakv_b200 as dkv

    sample = probs[: 2 * min(n_layers, len(probs) // 2)]
    host = [(p["reused"].cpu().pin_memory(), p["fresh"].cpu().pin_memory()) for p in sample]
    outs = [torch.empty(p["reused"].shape, dtype=p["reused"].dtype).pin_memory() for p in sample]
    h2d = sum(a.numel() * a.element_size() + b.numel() * b.element_size() for a, b in host)
    d2h = sum(o.numel() * o.element_size() for o in outs)

    def step():
        dev_probs = [dict(p, reused=r.to(dist.dev, non_blocking=True), fresh=f.to(dist.dev, non_blocking=True))
                     for p, (r, f) in zip(sample, host)]
        res = dkv.subspace_correct_batched(dev_probs)
        for o, (corr, _, _) in zip(outs, res):
            o.copy_(corr, non_blocking=True)

    step()
    torch.cuda.synchronize()
    dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 3
    a.record(stream)
    for _ in range(reps):
        step()
    b.record(stream)
    torch.cuda.synchronize()
    ms = dist.max(a.elapsed_time(b) / reps)
    units = len(sample) // 2 * args.seq_len * dist.world
    return {"value": units / (ms / 1e3), "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "ms_per_step": ms, "sample": f"{len(sample) // 2} layers x {args.seq_len} tokens per GPU (K and V), "
                                        "pinned host buffers"}


def run_dsub(args, dist: Dist) -> dict:
    import deltakv_b200 as dkv

    mine = [l for l in range(args.layers) if l % dist.world == dist.rank]
    probs = make_dsub_problems(args, dist, mine)
    units_step = args.layers * args.seq_len
    stream = torch.cuda.current_stream()

    def step(ev=None):
        dkv.subspace_correct_batched(probs)

    step()
    torch.cuda.synchronize()
    for _ in range(max(0, args.warmup - 1)):
        step()
    ms, _, clocks = timed(dist, step, args.steps, kernel_events=False)
    ms_step = ms / args.steps
    units_rank = len(mine) * args.seq_len
    achieved = units_rank * DSUB_BYTES_PER_UNIT / (ms_step / 1e3) / 1e9
    peak, peak_kind = hbm_peak()
    parity = dsub_parity(probs) if dist.rank == 0 else None
    cpu = None
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu:
        cpu = dsub_cpu_sample(args.sub_cpu_seconds)
    e2e = None if args.no_e2e else dsub_e2e(args, probs, dist, stream)
    del probs
    torch.cuda.empty_cache()
    return {
        "metric": DSUB_METRIC, "value": units_step / (ms_step / 1e3), "unit": UNIT, "n_gpus": dist.world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16 cache, split-bf16 tensor-core products, fp32",
        "data": "synthetic",
        "config": {"workload": DSUB_WORKLOAD, "layers": args.layers, "seq_len": args.seq_len,
                   "layers_this_gpu": len(mine), "units_per_step": units_step,
                   "parallelism": f"layer shards x{dist.world}: layer l on rank l mod {dist.world} (strong)",
                   "l2": f"{units_rank * DSUB_BYTES_PER_UNIT / 1e9:.1f} GB per step per GPU >> 126 MB L2",
                   "e2e_sample": None if e2e is None else e2e["sample"]},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": None, "peak_source": peak_kind,
                     "kernel": "subspace route, dense form (flags, pack, pass1, psum, solve, fitb, dpass2, dprobe) "
                               "over this rank's layers, host wrapper included",
                     "algorithmic_bytes_per_unit": DSUB_BYTES_PER_UNIT},
        "parity": parity,
        "cpu_baseline": cpu,
        "e2e": e2e,
        "gpu_launches": args.steps * 8,
        "clocks": clocks,
    }


def run_dsub_reference(args) -> dict:
    res = [dsub_cpu_sample(max(2.0, args.cpu_seconds / max(1, args.steps))) for _ in range(args.steps)]
    value = sum(r["value"] for r in res) / len(res)
    return {
        "impl": "reference", "metric": DSUB_METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": None, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": DSUB_WORKLOAD, "step": res[0]["sample"]},
        "cpu_baseline": {**res[0], "value": value},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


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
    """The engine's analytic loop on ``layers`` layers of one ``n``-token sequence of the same
    shape, in the reference's fp32 torch CPU operations (`oracle.analytic_torch`), repeated for
    about ``seconds``."""
    from oracle import analytic_torch as OAT

    G = AnalyticGeo
    g = torch.Generator().manual_seed(0)
    rnd = lambda *shape, s=0.02: torch.randn(*shape, generator=g) * s  # noqa: E731
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
    h, hm = torch.randn(layers, n, G.d_model, generator=g), torch.randn(layers, n, G.d_model, generator=g)

    def item():
        with torch.no_grad():
            OAT.analytic_patches(h, hm, W, Ls, cfg)
        return layers * n

    # each item holds ~1 GB of [heads, n, n] fp32 matrices
    threads = host_threads()
    try:
        import psutil

        threads = max(1, min(threads, int(psutil.virtual_memory().available * 0.5 // (1 << 30))))
    except Exception:
        pass
    units, el, how = host_rate(item, threads, seconds)
    return {"value": units / el, "unit": UNIT, "cores": threads, "cpu_model": cpu_model(), "kind": "port",
            "sample": f"{units // (layers * n)} x ({layers} layer x {n} tokens) of the engine's analytic loop in "
                      f"{el:.1f} s (the reference's fp32 torch CPU operations, attention materialised; {threads} "
                      f"threads, {how})"}


def run_analytic(args, dist: Dist) -> dict:
    from deltakv_b200 import analytic as AN
    from deltakv_b200 import ops
    from deltakv_b200 import subspace as SUB

    G = AnalyticGeo
    dev = dist.dev
    model, delta, conf, hidden = make_analytic_workload(args, dev, 7000 + dist.rank)
    units = args.layers * args.seq_len * args.seqs
    stream = torch.cuda.current_stream()

    def step(ev=None):
        for h, hm in hidden:
            AN.analytic_patches(_snapshot(h, hm), delta, model, conf)

    for _ in range(max(1, args.warmup)):
        step()
    torch.cuda.synchronize()
    ops.status_word(dev).raise_if_set("bench warm-up")
    trunc0 = SUB.gram_launches
    ms, _, clocks = timed(dist, step, args.steps, kernel_events=False)
    trunc_launches = SUB.gram_launches - trunc0
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
    bf16_peak = peaks().get("bf16_tflops") or 1590.0
    cpu = None
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu:
        cpu = analytic_cpu_sample(args.sub_cpu_seconds)
    e2e = None
    if not args.no_e2e:
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
        dist.barrier()
        e2 = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        e2[0].record(stream)
        e2e_step()
        e2[1].record(stream)
        torch.cuda.synchronize()
        e2e_ms = dist.max(e2[0].elapsed_time(e2[1]))
        e2e = {"value": units * dist.world / (e2e_ms / 1e3), "unit": UNIT,
               "h2d_bytes_per_step": sum(a.numel() * 4 + b.numel() * 4 for a, b in h_host),
               "d2h_bytes_per_step": out_bytes * len(hidden), "ms_per_step": e2e_ms}
    return {
        "metric": ANALYTIC_METRIC, "value": units * dist.world / (ms_step / 1e3), "unit": UNIT, "n_gpus": dist.world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": ANALYTIC_WORKLOAD, "layers": args.layers, "seqs_per_gpu": args.seqs,
                   "seq_len": n, "parallelism": f"request shards x{dist.world}",
                   "l2": "per sequence 283 MB of stored hidden states >> 126 MB L2"},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": bf16_peak, "unit": "TFLOP/s",
                     "frac": achieved / bf16_peak, "traffic": None,
                     "peak_source": "of measured (MEASURED_PEAKS.json bf16_tflops, burst)",
                     "kernel": "attention core (dkv_attn_first_order, mma.sync bf16 three-term split), one layer",
                     "kernel_ms": core_ms, "algorithmic_flops_per_launch": core_flops,
                     "issued_mma_flops_per_launch": core_flops * (3 * 3 * 2 + 3 * 3) / 6,
                     "fp32_fma_equivalent": {"peak": FP32_FMA_NOMINAL_TFLOPS,
                                             "frac": achieved / FP32_FMA_NOMINAL_TFLOPS,
                                             "peak_source": "of nominal (148 SMs x 128 lanes x 2 x 1965 MHz)"}},
        "cpu_baseline": cpu, "e2e": e2e,
        "gpu_launches": args.steps * args.seqs * args.layers * 8 + trunc_launches,
        "clocks": clocks,
    }


def run_analytic_reference(args) -> dict:
    res = [analytic_cpu_sample(max(2.0, args.cpu_seconds / max(1, args.steps))) for _ in range(args.steps)]
    value = sum(r["value"] for r in res) / len(res)
    return {
        "impl": "reference", "metric": ANALYTIC_METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": None, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": ANALYTIC_WORKLOAD, "step": res[0]["sample"]},
        "cpu_baseline": {**res[0], "value": value},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


# ---------------------------------------------------------------------------
# driver
# ---------------------------------------------------------------------------
DEFAULTS = {
    "llama8b-exact": (Llama8B.layers, Llama8B.seqs, Llama8B.seq_len),
    "smollm2-exact": (Smol135M.layers, Smol135M.seqs, Smol135M.seq_len),
    "rl-dense": (Dense70B.layers, Dense70B.seqs, Dense70B.seq_len),
    "multi-lora-kivi": (KiviGeo.layers, 1, KiviGeo.seq_len),
    "dense-subspace": (DsubGeo.layers, 1, DsubGeo.seq_len),
    "analytic": (AnalyticGeo.layers, AnalyticGeo.seqs, AnalyticGeo.seq_len),
}


def with_defaults(args, workload):
    import copy

    a = copy.copy(args)
    a.workload = workload
    L_, S, N = DEFAULTS[workload]
    a.layers = args.layers if args.layers is not None else L_
    a.seqs = args.seqs if args.seqs is not None else S
    a.seq_len = args.seq_len if args.seq_len is not None else N
    return a


def run_one(args, dist: Dist) -> dict:
    w = args.workload
    if w == "llama8b-exact":
        return run_exact(args, dist, Llama8B)
    if w == "smollm2-exact":
        return run_exact(args, dist, Smol135M)
    if w == "rl-dense":
        return run_dense(args, dist)
    if w == "multi-lora-kivi":
        return run_kivi(args, dist)
    if w == "dense-subspace":
        return run_dsub(args, dist)
    return run_analytic(args, dist)


def run_reference(args) -> dict:
    w = args.workload
    if w == "llama8b-exact":
        return run_exact_reference(args, Llama8B)
    if w == "smollm2-exact":
        return run_exact_reference(args, Smol135M)
    if w == "rl-dense":
        return run_dense_reference(args)
    if w == "multi-lora-kivi":
        return run_kivi_reference(args)
    if w == "dense-subspace":
        return run_dsub_reference(args)
    return run_analytic_reference(args)


SUB_WORKLOADS = ("smollm2-exact", "multi-lora-kivi", "rl-dense", "dense-subspace", "analytic")


def main(argv=None):
    args = parse(argv)
    if args.impl == "reference":
        # the CPU reference arm: rank 0 alone times the host path; other ranks exit at once
        if int(os.environ.get("RANK", "0")) != 0:
            return 0
        print(json.dumps(run_reference(with_defaults(args, args.workload))), flush=True)
        return 0
    dist = Dist().init()
    line = run_one(with_defaults(args, args.workload), dist)
    if args.workload == "llama8b-exact" and not args.no_workloads:
        # the other configurations, one after another on the same GPUs (each frees its memory)
        sub_args = argparse.Namespace(**{**vars(args), "layers": None, "seqs": None, "seq_len": None})
        workloads = {}
        for w in SUB_WORKLOADS:
            try:
                workloads[w] = run_one(with_defaults(sub_args, w), dist)
            except Exception as e:  # recorded, not hidden: the line says which workload failed and why
                workloads[w] = {"error": f"{type(e).__name__}: {e}", "trace": traceback.format_exc()[-2000:]}
                try:
                    torch.cuda.synchronize()
                except Exception:
                    pass
            try:
                torch.cuda.empty_cache()
            except Exception:
                pass
        line["workloads"] = workloads
    if dist.rank == 0:
        print(json.dumps(line), flush=True)
    dist.finish()
    return 0


if __name__ == "__main__":
    sys.exit(main())
