"""Test infrastructure: times the reference's own CPU exact branch beside the oracle's ports.

The CPU baseline the benchmark reports is a port (the reference is Python and is not installed
where the benchmark runs): `oracle.exact_torch`, the reference's steps in torch CPU operations.
This script checks, on the machine that has the reference's sources, that this port is not a
slower stand-in for the reference: it runs the reference, the numpy parity oracle and the torch
port on the same Llama-3-8B-shaped (layer, sequence) pairs with the same cores and prints one
JSON line.

Per pair (4096 tokens, d_model 4096, 8 KV heads x 128, rank-16 LoRA on k_proj / v_proj, RoPE
theta 5e5, bf16 pages of block 16 through a permuted block table):

* reference: ``RMSNorm`` (src/deltakv/model.py:48-56, the engine's ``rmsnorm_tensors``,
  model.py:310-314) -> ``exact_kv_patch`` (src/deltakv/patches/exact.py:14-63) ->
  ``LowRankKVPatch.materialize`` (src/deltakv/patches/tensors.py:105-123) ->
  ``scatter_into_paged`` for K and V (src/deltakv/paged.py:8-43), on fp32 activations as the
  reference keeps them;
* numpy port: ``oracle.exact`` (the parity oracle) rmsnorm -> exact_kv_delta -> scatter_into_paged
  on the same fp32 activations (no fp8 dequantisation, so every arm does the same work);
* torch port: ``oracle.exact_torch``, the form the benchmark's CPU baseline times, on the same
  fp32 activations.

Every arm is timed two ways — one pair per worker thread with one BLAS / intra-op thread each,
and pairs one after another with every core inside each operation — and the faster of the two
is each arm's figure.

Usage: python oracle/time_reference_exact.py --reference-src <reference checkout>/src [--pairs N]
"""
from __future__ import annotations

import argparse
import json
import math
import os
import sys
import threading
import time
from concurrent.futures import ThreadPoolExecutor

import numpy as np

D_MODEL, N_KV, HD, RANK, THETA, BS, SEQ, EPS = 4096, 8, 128, 16, 500000.0, 16, 4096, 1e-5


def make_inputs(n_inputs: int, seed: int = 0):
    rng = np.random.default_rng(seed)
    s = 1.0 / RANK
    out = []
    for _ in range(n_inputs):
        x = (rng.standard_normal((SEQ, D_MODEL)) * (0.5 + rng.random((SEQ, 1)))).astype(np.float32)
        w = (1.0 + 0.05 * rng.standard_normal(D_MODEL)).astype(np.float32)
        fk = ((rng.standard_normal((RANK, D_MODEL)) / math.sqrt(D_MODEL)).astype(np.float32),
              rng.standard_normal((N_KV * HD, RANK)).astype(np.float32), s)
        fv = ((rng.standard_normal((RANK, D_MODEL)) / math.sqrt(D_MODEL)).astype(np.float32),
              rng.standard_normal((N_KV * HD, RANK)).astype(np.float32), s)
        out.append((x, w, fk, fv))
    nblk = (SEQ + BS - 1) // BS
    table = [int(b) for b in rng.permutation(nblk)]
    return out, table, nblk


class ReferenceArm:
    def __init__(self, src: str, inputs, table, nblk):
        sys.path.insert(0, src)
        import torch

        from deltakv.deltas.descriptor import LayerDelta
        from deltakv.deltas.factors import LowRankFactors
        from deltakv.model import RMSNorm
        from deltakv.paged import scatter_into_paged
        from deltakv.patches.exact import exact_kv_patch
        from deltakv.rope import RotaryEmbedding

        self.torch = torch
        self.exact_kv_patch, self.scatter = exact_kv_patch, scatter_into_paged
        self.rope = RotaryEmbedding(HD, max_seq=SEQ, base=THETA)
        self.items = []
        for x, w, fk, fv in inputs:
            norm = RMSNorm(D_MODEL, EPS)
            with torch.no_grad():
                norm.weight.copy_(torch.from_numpy(w))
            layer = LayerDelta(0, {
                "k_proj": LowRankFactors(A=torch.from_numpy(fk[0]), B=torch.from_numpy(fk[1]), scale=fk[2]),
                "v_proj": LowRankFactors(A=torch.from_numpy(fv[0]), B=torch.from_numpy(fv[1]), scale=fv[2]),
            })
            self.items.append((torch.from_numpy(x), norm, layer))
        self.table, self.nblk = table, nblk

    def new_pages(self):
        t = self.torch
        g = t.Generator().manual_seed(0)
        return (t.randn(self.nblk, BS, N_KV, HD, generator=g).to(t.bfloat16),
                t.randn(self.nblk, BS, N_KV, HD, generator=g).to(t.bfloat16))

    def patch_one(self, i: int, pages) -> int:
        x, norm, layer = self.items[i % len(self.items)]
        with self.torch.no_grad():
            xn = norm(x)
            patch = self.exact_kv_patch(xn, layer, n_kv_heads=N_KV, head_dim=HD, rope=self.rope)
            dk, dv = patch.materialize(N_KV, HD)
            self.scatter(dk.to(pages[0].dtype), pages[0], self.table, BS)
            self.scatter(dv.to(pages[1].dtype), pages[1], self.table, BS)
        return SEQ

    def threads_ctx(self, n: int):
        arm = self

        class _Ctx:
            def __enter__(self):
                self.old = arm.torch.get_num_threads()
                arm.torch.set_num_threads(n)

            def __exit__(self, *a):
                arm.torch.set_num_threads(self.old)

        return _Ctx()


class PortArm:
    def __init__(self, inputs, table, nblk):
        from oracle import exact as OX

        self.OX = OX
        self.items = inputs
        self.tabs = OX.rope_tables(HD, SEQ, THETA)
        self.table, self.nblk = table, nblk

    def new_pages(self):
        rng = np.random.default_rng(0)
        shape = (self.nblk, BS, N_KV, HD)
        return (rng.integers(0x3C00, 0x3F80, size=shape, dtype=np.uint16),
                rng.integers(0x3C00, 0x3F80, size=shape, dtype=np.uint16))

    def patch_one(self, i: int, pages) -> int:
        OX = self.OX
        x, w, fk, fv = self.items[i % len(self.items)]
        xn = OX.rmsnorm(x, w, EPS)
        dk, dv = OX.exact_kv_delta(xn, fk, fv, N_KV, HD, self.tabs)
        OX.scatter_into_paged(dk, pages[0], self.table, BS, kind="bf16")
        OX.scatter_into_paged(dv, pages[1], self.table, BS, kind="bf16")
        return SEQ

    def threads_ctx(self, n: int):
        from threadpoolctl import threadpool_limits

        return threadpool_limits(n)


class TorchPortArm:
    """`oracle.exact_torch`, the form the benchmark's CPU baseline times"""

    def __init__(self, inputs, table, nblk):
        import torch

        from oracle import exact as OX
        from oracle import exact_torch as OT

        self.torch, self.OT = torch, OT
        self.items = [(torch.from_numpy(x), torch.from_numpy(w),
                       (torch.from_numpy(fk[0]), torch.from_numpy(fk[1]), fk[2]),
                       (torch.from_numpy(fv[0]), torch.from_numpy(fv[1]), fv[2])) for x, w, fk, fv in inputs]
        cos_h, sin_h = OX.rope_tables(HD, SEQ, THETA)
        self.rope = OT.rope_full(torch.from_numpy(cos_h), torch.from_numpy(sin_h), SEQ)
        self.table, self.nblk = torch.tensor(table), nblk

    new_pages = ReferenceArm.new_pages
    threads_ctx = ReferenceArm.threads_ctx

    def patch_one(self, i: int, pages) -> int:
        OT = self.OT
        x, w, fk, fv = self.items[i % len(self.items)]
        with self.torch.no_grad():
            xn = OT.rmsnorm(x, w, EPS)
            dk, dv = OT.exact_kv_delta(xn, fk, fv, N_KV, HD, self.rope)
            OT.scatter_into_paged(dk, pages[0], self.table, BS)
            OT.scatter_into_paged(dv, pages[1], self.table, BS)
        return SEQ


def time_pool(arm, threads: int, pairs: int) -> float:
    """pairs on `threads` workers, one intra-op thread each; token·layers per second"""
    pages = [arm.new_pages() for _ in range(threads)]
    counter = [0]
    lock = threading.Lock()

    def worker(wi):
        done = 0
        while True:
            with lock:
                if counter[0] >= pairs:
                    return done
                k = counter[0]
                counter[0] += 1
            done += arm.patch_one(k, pages[wi])

    with arm.threads_ctx(1):
        with ThreadPoolExecutor(threads) as ex:  # warm-up: every worker once
            counter[0] = pairs - threads
            list(ex.map(worker, range(threads)))
        counter[0] = 0
        t0 = time.perf_counter()
        with ThreadPoolExecutor(threads) as ex:
            units = sum(ex.map(worker, range(threads)))
        return units / (time.perf_counter() - t0)


def time_serial(arm, threads: int, pairs: int) -> float:
    """pairs one after another, every core inside each operation"""
    pages = arm.new_pages()
    with arm.threads_ctx(threads):
        arm.patch_one(0, pages)
        t0 = time.perf_counter()
        units = sum(arm.patch_one(k, pages) for k in range(pairs))
        return units / (time.perf_counter() - t0)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-src", required=True, help="the reference checkout's src directory")
    ap.add_argument("--pairs", type=int, default=0, help="pairs per timing (default 2 x cores)")
    ap.add_argument("--threads", type=int, default=len(os.sched_getaffinity(0)))
    a = ap.parse_args()
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    pairs = a.pairs or 2 * a.threads
    inputs, table, nblk = make_inputs(4)
    ref = ReferenceArm(a.reference_src, inputs, table, nblk)
    port = PortArm(inputs, table, nblk)
    tport = TorchPortArm(inputs, table, nblk)
    out = {"workload": f"exact patch, {SEQ} tokens x d_model {D_MODEL}, {N_KV}x{HD} KV heads, rank {RANK}, "
                       f"fp32 X, bf16 pages (block {BS})", "unit": "token·layers/s", "cores": a.threads,
           "pairs": pairs}
    for name, arm in (("reference", ref), ("numpy_port", port), ("torch_port", tport)):
        out[name] = {"pool": time_pool(arm, a.threads, pairs), "serial": time_serial(arm, a.threads, pairs)}
        out[name]["best"] = max(out[name]["pool"], out[name]["serial"])
    for name in ("numpy_port", "torch_port"):
        out[f"{name}_over_reference"] = out[name]["best"] / out["reference"]["best"]
    print(json.dumps(out))


if __name__ == "__main__":
    main()
