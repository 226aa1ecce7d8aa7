"""The reference engine's routes end to end through this build's operators, on the GPU.

``tests/golden/engine.npz`` records a run of the reference's own ``DeltaKVEngine`` (CPU toy:
4 layers, d=64, GQA 4/2, 64 tokens, rank-4 q/k/v LoRA at scale 0.01): ``prefill``,
``commit_delta``, ``evaluate_against_fresh`` for route exact, hybrid and subspace, with the
arguments and results of every hot-path call its ``_patch`` made (src/deltakv/engine.py:
263-359) and the connector's ``patch_paged`` (connectors/vllm.py:70-81).  The reference
cannot be imported where these tests run, so each test drives the same calls, in the
engine's order, through the drop-ins that :func:`deltakv_b200.install` binds into the
engine module — ``zeroth_order_patches`` -> ``apply_layer_patches`` for the exact branch;
then ``weight_axis_scores`` -> ``select_probes`` -> ``apply_probe_to_cache`` for the probe
branch, with the engine's own fresh probe K/V and plan — and the subspace route through the
mapping itself (``routes.wrap_materialize`` around a stand-in ``materialize`` whose probe
branch calls the engine module's rebound ``apply_probe_to_cache``).

Tolerances: zeroth-order KV within rel-L2 1e-5 of the reference's (fp32); probe scores 1e-5;
probe indices and gate sets exact; corrected KV within 1e-4 absolute (fp32 subspace kernels
on O(1) values, as in tests/test_gpu_probe.py); next-token KL within 1e-4 nats of the
reference's report; connector pages bit-identical.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import deltakv_b200 as dkv
from deltakv_b200 import routes
from oracle.model import logits_from_kv, next_token_kl, weights_from_golden
from tests.conftest import golden
from tests.helpers import bf16_from_bits, bits_from_bf16, rel_l2

pytestmark = pytest.mark.gpu


class _Delta:
    def __init__(self, layers):
        self.layers = layers
        self.first_modified_layer = min(layers)


def _setup(cuda):
    g = golden("engine")
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    L_ = int(g["n_layers"])
    layers = {}
    for l in range(L_):
        proj = {f"{p}_proj": dkv.LowRankFactors(A=t(g[f"a_{p}"][l]), B=t(g[f"b_{p}"][l]), scale=float(g[f"s_{p}"][l]),
                                               name=f"{p}_proj") for p in ("k", "v", "q")}
        layers[l] = dkv.LayerDelta(l, proj)
    rope = (torch.from_numpy(g["rope_cos"]), torch.from_numpy(g["rope_sin"]))
    return g, t, _Delta(layers), rope


def _kl(g, k, v):
    w = weights_from_golden(g)
    kw = dict(n_layers=int(g["n_layers"]), n_heads=int(g["n_heads"]), n_kv=int(g["n_kv_heads"]),
              hd=int(g["head_dim"]), eps=float(g["eps"]), rope=(g["rope_cos"], g["rope_sin"]))
    fresh = logits_from_kv(w, g["tokens"], g["fresh_k"], g["fresh_v"], **kw)
    return next_token_kl(fresh, logits_from_kv(w, g["tokens"], k, v, **kw))


def _zeroth(g, t, delta, rope, route):
    n_kv, hd = int(g["n_kv_heads"]), int(g["head_dim"])
    xn = {l: t(g[f"{route}_xn"][l]) for l in range(g[f"{route}_xn"].shape[0])}
    patches = dkv.zeroth_order_patches(xn, delta, n_kv_heads=n_kv, head_dim=hd, rope=rope)
    base = dkv.KVCache(t(g[f"{route}_base_k"]), t(g[f"{route}_base_v"]))
    return dkv.apply_layer_patches(base, patches)


def test_engine_exact_route(cuda):
    g, t, delta, rope = _setup(cuda)
    kv = _zeroth(g, t, delta, rope, "exact")
    k, v = kv.k.cpu().numpy(), kv.v.cpu().numpy()
    assert rel_l2(k, g["exact_k"]) < 1e-5 and rel_l2(v, g["exact_v"]) < 1e-5
    assert abs(_kl(g, k, v) - float(g["exact_kl"])) < 1e-4
    # the report's max relative L2 against the fresh prefill, through the compare_kv drop-in
    rep = dkv.compare_kv(kv, dkv.KVCache(t(g["fresh_k"]), t(g["fresh_v"])))
    assert abs(rep.max_relative_l2 - float(g["exact_max_rel_l2"])) < 1e-5


def _probe_branch(g, t, delta, rope, route, apply_probe):
    kv = _zeroth(g, t, delta, rope, route)
    assert rel_l2(kv.k.cpu().numpy(), g[f"{route}_kv_in_k"]) < 1e-5
    assert rel_l2(kv.v.cpu().numpy(), g[f"{route}_kv_in_v"]) < 1e-5
    scores = dkv.weight_axis_scores(t(g[f"{route}_score_x"]), delta, int(g[f"{route}_score_layer"]))
    assert np.allclose(scores.cpu().numpy(), g[f"{route}_scores"], rtol=1e-5, atol=1e-6)
    probes = dkv.select_probes(scores, float(g[f"{route}_ratio"]), int(g[f"{route}_min_tokens"]),
                               float(g[f"{route}_max_ratio"]))
    assert np.array_equal(probes.cpu().numpy(), g[f"{route}_probes"])
    fresh = {int(l): (t(g[f"{route}_fresh_k"][i]), t(g[f"{route}_fresh_v"][i]))
             for i, l in enumerate(g[f"{route}_fresh_layers"])}
    dec = lambda a: None if (a.size == 1 and a[0] == -1) else {int(x) for x in a}
    out, _, extra = apply_probe(kv, fresh, probes, float(g[f"{route}_thr"]), float(g[f"{route}_maxr"]),
                                layer_deltas=delta.layers, subspace_rank=int(g[f"{route}_subspace_rank"]),
                                probe_layers=dec(g[f"{route}_probe_layers"]),
                                skip_layers=dec(g[f"{route}_skip_layers"]))
    torch.cuda.synchronize()
    assert np.array_equal(extra.cpu().numpy(), g[f"{route}_extra"])
    k, v = out.k.cpu().numpy(), out.v.cpu().numpy()
    assert np.abs(k - g[f"{route}_kv_out_k"]).max() < 1e-4 and np.abs(v - g[f"{route}_kv_out_v"]).max() < 1e-4
    assert np.abs(k - g[f"{route}_k"]).max() < 1e-4 and np.abs(v - g[f"{route}_v"]).max() < 1e-4
    assert abs(_kl(g, k, v) - float(g[f"{route}_kl"])) < 1e-4
    return out


def test_engine_hybrid_route(cuda):
    g, t, delta, rope = _setup(cuda)
    assert str(g["hybrid_decision_route"]) == "hybrid"
    _probe_branch(g, t, delta, rope, "hybrid", dkv.apply_probe_to_cache)


def test_engine_subspace_route_through_the_mapping(cuda):
    """``materialize(route="subspace")`` -> the probe route with the gate off: the recorded
    reference run passed probe_layers=set(); here the stand-in probe branch passes None (as
    the engine's probe route does) and the mapping must turn it into set()."""
    g, t, delta, rope = _setup(cuda)
    assert g["subspace_probe_layers"].size == 0 and str(g["subspace_decision_route"]) == "probe"
    seen = {}

    class _Result:
        def __init__(self, kv):
            self.kv = kv
            self.decision = type("D", (), {"reason": "", "extra": {}})()

    def materialize(self, token_ids, route=None):
        assert route == "probe"

        def engine_call(kv, fresh, probes, thr, maxr, *, layer_deltas, subspace_rank, probe_layers, skip_layers):
            seen["skip_layers"] = skip_layers
            # the engine's probe route passes no gate plan (engine.py:315-317)
            return routes.engine_apply_probe_to_cache(kv, fresh, probes, thr, maxr, layer_deltas=layer_deltas,
                                                      subspace_rank=subspace_rank, probe_layers=None,
                                                      skip_layers=skip_layers)

        return _Result(_probe_branch(g, t, delta, rope, "subspace", engine_call))

    res = routes.wrap_materialize(materialize)(None, g["tokens"], route="subspace")
    assert res.decision.extra["route_requested"] == "subspace"
    assert seen["skip_layers"] is None


def test_connector_patch_paged(cuda):
    """DeltaKVConnector.patch_paged: every layer's K and V scattered (additively, kv_dim 0)
    into vLLM's per-layer paged buffers through the block table."""
    g, t, *_ = _setup(cuda)
    table, bs = [int(b) for b in g["conn_table"]], int(g["conn_bs"])
    for l in range(int(g["n_layers"])):
        kc, vc = bf16_from_bits(g["conn_k_in"][l], cuda), bf16_from_bits(g["conn_v_in"][l], cuda)
        dkv.scatter_into_paged(t(g["exact_k"][l]), kc, table, bs, kv_dim=0)
        dkv.scatter_into_paged(t(g["exact_v"][l]), vc, table, bs, kv_dim=0)
        assert np.array_equal(bits_from_bf16(kc), g["conn_k_out"][l])
        assert np.array_equal(bits_from_bf16(vc), g["conn_v_out"][l])
