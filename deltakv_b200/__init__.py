"""deltakv_b200 — ΔKV's cache-maintenance hot path as hand-written sm_100a kernels.

Operators keep the reference's names and signatures (adityaraj-09/DeltaKV), so a ΔKV
deployment swaps them in (see :func:`install`):

* ``scatter_into_paged`` / ``gather_from_paged``   (deltakv.paged)
* ``exact_kv_patch`` / ``zeroth_order_patches``    (deltakv.patches.exact)
* ``apply_layer_patches`` / ``measured_error``     (deltakv.patches.compose)
* ``compare_kv``                                   (deltakv.metrics)
* ``rmsnorm_first_order`` / ``attention_first_order`` / ``mlp_first_order`` /
  ``rank_truncate`` / ``softmax_jacobian_product`` (deltakv.patches.analytic) and the engine's
  analytic loop (``analytic.analytic_patches``)
* ``subspace_correct`` / ``svd_basis``             (deltakv.patches.subspace)
* ``apply_probe_to_cache`` / ``select_probes`` / ``weight_axis_scores`` / ``residual_gate``
  (deltakv.patches.probe), ``lora_activation_scores`` (deltakv.patches.exact)

plus the fused batched forms the engine and connector use: :class:`ExactPatcher` (LoRA
deltas) and :class:`DensePatcher` (full-rank dW of an RL step, a tensor-core GEMM).
All computation runs in ``libdkv_b200.so``; a missing library raises (no CPU path).
"""

from __future__ import annotations

from deltakv_b200 import analytic, kivi, routes
from deltakv_b200._lib import DkvError
from deltakv_b200.dense import DensePatcher
from deltakv_b200.exact import (
    ExactPatcher,
    apply_layer_patches,
    apply_layer_patches_,
    replay,
    exact_kv_patch,
    materialize_codes,
    zeroth_order_patches,
)
from deltakv_b200.metrics import compare_kv, measured_error
from deltakv_b200.ops import SeqBatchTensors, quantize_rows
from deltakv_b200.probe import (
    apply_probe_to_cache,
    lora_activation_scores,
    residual_gate,
    select_probes,
    weight_axis_scores,
)
from deltakv_b200.paged import gather_from_paged, scatter_into_paged, scatter_into_paged_batched
from deltakv_b200.rope import RotaryEmbedding
from deltakv_b200.subspace import subspace_correct, subspace_correct_batched, svd_basis
from deltakv_b200.types import KVCache, LayerDelta, LowRankFactors, LowRankKVPatch

__version__ = "0.1.0"

__all__ = [
    "DensePatcher",
    "DkvError",
    "ExactPatcher",
    "KVCache",
    "LayerDelta",
    "LowRankFactors",
    "LowRankKVPatch",
    "RotaryEmbedding",
    "SeqBatchTensors",
    "analytic",
    "apply_layer_patches",
    "apply_layer_patches_",
    "apply_probe_to_cache",
    "compare_kv",
    "exact_kv_patch",
    "gather_from_paged",
    "install",
    "kivi",
    "lora_activation_scores",
    "materialize_codes",
    "measured_error",
    "quantize_rows",
    "replay",
    "residual_gate",
    "routes",
    "scatter_into_paged",
    "scatter_into_paged_batched",
    "select_probes",
    "subspace_correct",
    "subspace_correct_batched",
    "svd_basis",
    "weight_axis_scores",
    "zeroth_order_patches",
]

# reference module -> {attribute: replacement}
_INSTALL_MAP = {
    "deltakv.paged": {"scatter_into_paged": scatter_into_paged, "gather_from_paged": gather_from_paged},
    "deltakv.patches.exact": {"exact_kv_patch": exact_kv_patch, "zeroth_order_patches": zeroth_order_patches,
                              "lora_activation_scores": lora_activation_scores},
    "deltakv.patches.compose": {"apply_layer_patches": apply_layer_patches, "measured_error": measured_error},
    "deltakv.metrics": {"compare_kv": compare_kv},
    "deltakv.patches.analytic": {"rmsnorm_first_order": analytic.rmsnorm_first_order,
                                 "attention_first_order": analytic.attention_first_order,
                                 "mlp_first_order": analytic.mlp_first_order,
                                 "rank_truncate": analytic.rank_truncate,
                                 "softmax_jacobian_product": analytic.softmax_jacobian_product},
    # modules that imported the names with `from ... import`
    "deltakv.engine": {"zeroth_order_patches": zeroth_order_patches, "exact_kv_patch": exact_kv_patch,
                       "apply_layer_patches": apply_layer_patches,
                       "apply_probe_to_cache": routes.engine_apply_probe_to_cache,
                       "select_probes": select_probes, "weight_axis_scores": weight_axis_scores,
                       "compare_kv": compare_kv, "measured_error": measured_error,
                       "rmsnorm_first_order": analytic.rmsnorm_first_order,
                       "attention_first_order": analytic.attention_first_order,
                       "mlp_first_order": analytic.mlp_first_order, "rank_truncate": analytic.rank_truncate},
    "deltakv.connectors.vllm": {"scatter_into_paged": scatter_into_paged},
    "deltakv.patches.subspace": {"subspace_correct": subspace_correct, "svd_basis": svd_basis},
    "deltakv.patches.probe": {"subspace_correct": subspace_correct, "apply_probe_to_cache": apply_probe_to_cache,
                              "select_probes": select_probes, "weight_axis_scores": weight_axis_scores,
                              "residual_gate": residual_gate, "lora_activation_scores": lora_activation_scores},
    "deltakv.patches": {"exact_kv_patch": exact_kv_patch, "zeroth_order_patches": zeroth_order_patches,
                        "apply_layer_patches": apply_layer_patches, "subspace_correct": subspace_correct},
}


def install(modules: dict | None = None) -> list[str]:
    """Point an imported ``deltakv`` package at these kernels.

    Rebinds the operator names in the reference's modules (and in the modules that
    imported them by name), so ``DeltaKVEngine`` and ``DeltaKVConnector`` run the B200
    path unchanged, and gives ``DeltaKVEngine.materialize`` (hence ``evaluate_against_fresh``
    and ``maintain_all``) the ``route="subspace"`` the reference accepts but drops: the probe
    route with the residual gate off on every layer (:mod:`deltakv_b200.routes`).  Returns
    the ``module.attribute`` names that were replaced.
    """
    import importlib
    import sys

    done = []
    for mod_name, attrs in (modules or _INSTALL_MAP).items():
        mod = sys.modules.get(mod_name)
        if mod is None:
            try:
                mod = importlib.import_module(mod_name)
            except ImportError:
                continue
        for attr, fn in attrs.items():
            if hasattr(mod, attr):
                setattr(mod, attr, fn)
                done.append(f"{mod_name}.{attr}")
        engine_cls = getattr(mod, "DeltaKVEngine", None) if mod_name == "deltakv.engine" else None
        if engine_cls is not None and hasattr(engine_cls, "materialize"):
            engine_cls.materialize = routes.wrap_materialize(engine_cls.materialize)
            done.append(f"{mod_name}.DeltaKVEngine.materialize")
    return done
