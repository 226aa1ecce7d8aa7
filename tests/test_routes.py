"""The engine's ``route="subspace"`` mapping, on a stand-in engine module (host logic, no GPU).

The stand-in mimics the two things :func:`deltakv_b200.install` relies on in
src/deltakv/engine.py: ``DeltaKVEngine.materialize(token_ids, route=None)``, which
``evaluate_against_fresh`` calls, and its probe branch calling the module-level name
``apply_probe_to_cache(kv, fresh, probes, thr, max_ratio, *, layer_deltas, subspace_rank,
probe_layers, skip_layers)`` (engine.py:329-339).  The recorder replaces the corrector so
no kernel runs.
"""

from __future__ import annotations

import sys
import types
from dataclasses import dataclass, field

import pytest

import deltakv_b200 as dkv
from deltakv_b200 import routes


@dataclass
class _Decision:
    route: str
    reason: str = ""
    extra: dict = field(default_factory=dict)


@dataclass
class _Result:
    kv: object
    decision: _Decision


def _fake_engine_module():
    mod = types.ModuleType("deltakv.engine")

    def apply_probe_to_cache(kv, fresh, probes, thr, max_ratio, *, layer_deltas=None, subspace_rank=8,
                             probe_layers=None, skip_layers=None):
        raise AssertionError("install() must rebind the engine's apply_probe_to_cache")

    class DeltaKVEngine:
        def materialize(self, token_ids, route=None):
            if route not in (None, "exact", "zeroth", "analytic", "probe", "hybrid", "recompute"):
                route = None  # the reference drops strings that are not a PatchRoute
            if route in ("probe", "hybrid"):
                # the probe branch: gate on every layer for "probe", the planner's set for "hybrid"
                plan = None if route == "probe" else {1, 3}
                mod.apply_probe_to_cache("kv", {0: None}, "probes", 0.15, 0.4, layer_deltas=None, subspace_rank=4,
                                         probe_layers=plan, skip_layers=None)
            return _Result(kv="kv", decision=_Decision(route=route or "lattice-default"))

        def evaluate_against_fresh(self, token_ids, route=None):
            return self.materialize(token_ids, route=route)

    mod.apply_probe_to_cache = apply_probe_to_cache
    mod.DeltaKVEngine = DeltaKVEngine
    return mod


@pytest.fixture
def fake_engine(monkeypatch):
    mod = _fake_engine_module()
    monkeypatch.setitem(sys.modules, "deltakv.engine", mod)
    calls = []

    def recorder(kv, fresh, probes, *args, probe_layers=None, **kwargs):
        calls.append(probe_layers)
        return kv, {}, None

    monkeypatch.setattr(routes, "_apply_probe", recorder)
    return mod, calls


def test_install_maps_subspace_to_probe_with_the_gate_off(fake_engine):
    mod, calls = fake_engine
    done = dkv.install({"deltakv.engine": {"apply_probe_to_cache": routes.engine_apply_probe_to_cache}})
    assert "deltakv.engine.apply_probe_to_cache" in done
    assert "deltakv.engine.DeltaKVEngine.materialize" in done
    eng = mod.DeltaKVEngine()
    res = eng.evaluate_against_fresh([1, 2, 3], route="subspace")
    assert res.decision.route == "probe"
    assert res.decision.extra["route_requested"] == "subspace"
    assert "gate off" in res.decision.reason
    assert calls == [set()]  # pure subspace_correct on every layer, no residual gate


def test_other_routes_pass_through_unchanged(fake_engine):
    mod, calls = fake_engine
    dkv.install({"deltakv.engine": {"apply_probe_to_cache": routes.engine_apply_probe_to_cache}})
    eng = mod.DeltaKVEngine()
    assert eng.materialize([1], route="probe").decision.route == "probe"
    assert eng.materialize([1], route="hybrid").decision.route == "hybrid"
    assert eng.materialize([1], route="exact").decision.route == "exact"
    assert eng.materialize([1], route="bogus").decision.route == "lattice-default"
    assert calls == [None, {1, 3}]  # the gate state of the probe and hybrid routes is untouched
    # a second install does not wrap twice
    before = mod.DeltaKVEngine.materialize
    dkv.install({"deltakv.engine": {}})
    assert mod.DeltaKVEngine.materialize is before


def test_gate_flag_does_not_leak_after_an_error(fake_engine):
    mod, calls = fake_engine

    def failing(self, token_ids, route=None):
        raise RuntimeError("engine failure")

    mod.DeltaKVEngine.materialize = failing
    dkv.install({"deltakv.engine": {"apply_probe_to_cache": routes.engine_apply_probe_to_cache}})
    with pytest.raises(RuntimeError):
        mod.DeltaKVEngine().materialize([1], route="subspace")
    routes.engine_apply_probe_to_cache("kv", {}, "p", probe_layers={2})
    assert calls == [{2}]
