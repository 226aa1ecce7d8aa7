"""Probe scoring/selection, the residual gate, apply_probe_to_cache and the no-clone replay on
the GPU against the reference's golden outputs (tests/golden/probe.npz, replay.npz).

Tolerances: scores 1e-5 relative (fp32); probe indices, gate set and extra tokens exact;
corrected KV within 1e-4 absolute of the reference (fp32 subspace kernels on O(1) values);
replayed KV within rel-L2 1e-3 of the reference for an fp32 cache (the codes of a codes@basis
patch pass through the fused kernel's f16 activation format) and 4e-3 for a bf16 cache (one
bf16 rounding of the base and of each stage's sum).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from deltakv_b200 import probe as P
from deltakv_b200.exact import replay
from deltakv_b200.types import KVCache, LayerDelta, LowRankFactors, LowRankKVPatch
from tests.conftest import golden

pytestmark = pytest.mark.gpu


class _Delta:
    def __init__(self, layers):
        self.layers = layers
        self.first_modified_layer = min(layers)


def _setup(cuda):
    g = golden("probe")
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    fk = LowRankFactors(A=t(g["a_k"]), B=t(g["b_k"]), scale=float(g["s_k"]), name="k_proj")
    fv = LowRankFactors(A=t(g["a_v"]), B=t(g["b_v"]), scale=float(g["s_v"]), name="v_proj")
    layers = {l: LayerDelta(l, {"k_proj": fk, "v_proj": fv}) for l in range(2)}
    return g, t, layers


def test_weight_axis_scores_and_select_probes(cuda):
    g, t, layers = _setup(cuda)
    sc = P.weight_axis_scores(t(g["x_norm"]), _Delta(layers), 0)
    assert np.allclose(sc.cpu().numpy(), g["scores"], rtol=1e-5, atol=1e-6)
    pr = P.select_probes(t(g["scores"]), 0.15, 4, 0.5)
    assert np.array_equal(pr.cpu().numpy(), g["probes"])


def test_residual_gate_and_apply_probe_to_cache(cuda):
    g, t, layers = _setup(cuda)
    probes = t(g["probes"])
    gate = P.residual_gate(t(g["base_k"][0]), t(g["out_k"][0]), t(g["fresh_k"][0]), probes, 0.15, 0.40)
    assert np.array_equal(np.sort(gate.cpu().numpy()), np.sort(g["gate"]))
    kv = KVCache(k=t(g["base_k"]), v=t(g["base_v"]))
    fresh = {l: (t(g["fresh_k"][l]), t(g["fresh_v"][l])) for l in range(2)}
    out, patches, extra = P.apply_probe_to_cache(kv, fresh, probes, 0.15, 0.40, layer_deltas=layers,
                                                 subspace_rank=4, probe_layers={0})
    torch.cuda.synchronize()
    assert np.array_equal(extra.cpu().numpy(), g["extra"])
    assert np.abs(out.k.cpu().numpy() - g["out_k"]).max() < 1e-4
    assert np.abs(out.v.cpu().numpy() - g["out_v"]).max() < 1e-4
    assert np.array_equal(patches[0].k_dense.cpu().numpy(), g["patch_k0"])  # the reference's ordering
    assert torch.equal(kv.k, t(g["base_k"]))  # input untouched


class _Applied:
    def __init__(self, layer_patches, target):
        self.layer_patches = layer_patches
        self.target = target


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("inplace", [False, True])
def test_replay_without_clones(cuda, dtype, inplace):
    r = golden("replay")
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    chain = []
    for si in range(2):
        stage = {}
        for l in range(3):
            f = lambda nm: t(r[f"s{si}_l{l}_{nm}"]) if f"s{si}_l{l}_{nm}" in r else None
            if f"s{si}_l{l}_k_codes" in r or f"s{si}_l{l}_k_dense" in r:
                stage[l] = LowRankKVPatch(l, f("k_codes"), f("k_basis"), f("v_codes"), f("v_basis"),
                                          k_dense=f("k_dense"), v_dense=f("v_dense"))
        chain.append(_Applied(stage, f"v{si + 1}"))
    base = KVCache(k=t(r["base_k"]).to(dtype), v=t(r["base_v"]).to(dtype), version="base")
    base_copy = base.k.clone()
    out = replay(base, chain, inplace=inplace)
    torch.cuda.synchronize()
    tol = 1e-3 if dtype == torch.float32 else 4e-3
    for got, ref in ((out.k, r["out_k"]), (out.v, r["out_v"])):
        a = got.float().cpu().numpy()
        assert np.linalg.norm(a - ref) / np.linalg.norm(ref) < tol
    assert out.version == "v2"
    assert (out is base) == inplace
    if not inplace:
        assert torch.equal(base.k, base_copy)
