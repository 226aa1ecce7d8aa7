"""The engine's ``route="subspace"``, which the reference accepts but does not have.

``DeltaKVEngine.materialize`` turns its ``route`` string into a ``PatchRoute``
(src/deltakv/engine.py:112-116) and silently keeps the lattice's own choice when the string
is not one of the enum's values (src/deltakv/types.py:28-36 has exact, zeroth, analytic,
probe, hybrid, recompute).  ``"subspace"`` — pure ``subspace_correct`` on every layer, with
no CacheBlend residual gate — is therefore mapped onto the probe route with the gate off:
the engine's probe branch (engine.py:290-359) calls
``apply_probe_to_cache(..., probe_layers=set())``, i.e. every layer is corrected by the
rank-r subspace shift plus the orthogonal residual mu and no token is recomputed.

:func:`wrap_materialize` wraps the engine's ``materialize`` (``evaluate_against_fresh`` and
``maintain_all`` call it) so that ``route="subspace"`` runs the probe route inside a context
in which :func:`engine_apply_probe_to_cache` — the name the engine module is rebound to —
passes ``probe_layers=set()``.  Every other route string goes through unchanged.  The
decision of a subspace call records the request (``decision.extra["route_requested"]``,
``decision.reason``); its ``route`` stays ``PatchRoute.PROBE``, the enum having no member
for it.
"""

from __future__ import annotations

import contextvars
import functools

from deltakv_b200.probe import apply_probe_to_cache

SUBSPACE_ROUTE = "subspace"
_gate_off = contextvars.ContextVar("deltakv_b200_subspace_route", default=False)
_apply_probe = apply_probe_to_cache


def engine_apply_probe_to_cache(kv, fresh_layers, probe_index, *args, probe_layers=None, **kwargs):
    """``apply_probe_to_cache`` as the engine module sees it: within a ``route="subspace"``
    call the residual gate is off on every layer (``probe_layers = set()``)."""
    if _gate_off.get():
        probe_layers = set()
    return _apply_probe(kv, fresh_layers, probe_index, *args, probe_layers=probe_layers, **kwargs)


def wrap_materialize(materialize):
    """``DeltaKVEngine.materialize`` with the ``"subspace"`` route mapped (idempotent)."""
    if getattr(materialize, "_dkv_subspace_route", False):
        return materialize

    @functools.wraps(materialize)
    def wrapped(self, token_ids, route=None):
        if route != SUBSPACE_ROUTE:
            return materialize(self, token_ids, route=route)
        token = _gate_off.set(True)
        try:
            result = materialize(self, token_ids, route="probe")
        finally:
            _gate_off.reset(token)
        decision = getattr(result, "decision", None)
        if decision is not None:
            extra = getattr(decision, "extra", None)
            if isinstance(extra, dict):
                extra["route_requested"] = SUBSPACE_ROUTE
            if hasattr(decision, "reason"):
                note = "subspace route: probe route with the residual gate off"
                decision.reason = f"{decision.reason}; {note}" if decision.reason else note
        return result

    wrapped._dkv_subspace_route = True
    return wrapped
