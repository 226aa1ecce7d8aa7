"""ctypes binding of ``libdkv_b200.so`` (the C ABI declared in ``include/dkv_b200.h``).

The library is built in-tree by :mod:`deltakv_b200.build`.  Loading never falls back to
another implementation: a missing or stale library raises immediately.
"""

from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libdkv_b200.so"

# status codes (dkv_b200.h)
DKV_OK = 0
ABI_VERSION = 2  # the struct layouts below (dkv_abi_version() of the library must match)
DKV_ERR_INVALID_ARGUMENT = -1
DKV_ERR_BLOCK_TABLE_SHORT = -2
DKV_ERR_LAYOUT = -3
DKV_ERR_UNSUPPORTED = -4
DKV_ERR_ALIGNMENT = -5
DKV_ERR_ROPE_RANGE = -6
DKV_ERR_BASIS_DIM = -7
DKV_ERR_CUDA = -8
DKV_ERR_TIMEOUT = -9
DKV_ERR_PAGE_RANGE = -10
DKV_ERR_WORKSPACE = -11

# element types
DKV_F32, DKV_F16, DKV_BF16, DKV_E4M3, DKV_I32, DKV_U8 = 0, 1, 2, 3, 4, 5
DKV_MAX_LAYERS = 128

EXPORTED = (
    "dkv_status_string",
    "dkv_abi_version",
    "dkv_last_cuda_error",
    "dkv_scatter_paged",
    "dkv_gather_paged",
    "dkv_paged_error_sums",
    "dkv_paged_compare_sums",
    "dkv_quantize_rows",
    "dkv_quantize_rows_sumsq",
    "dkv_exact_packed_bytes",
    "dkv_pack_exact_factors",
    "dkv_exact_patch_paged",
    "dkv_pack_dense_delta",
    "dkv_dense_patch_paged",
    "dkv_row_inv_rms",
    "dkv_kivi_quantize",
    "dkv_kivi_dequantize",
    "dkv_kivi_patch",
    "dkv_kivi_probe_residual",
    "dkv_kivi_probe_residual_batched",
    "dkv_kivi_subspace_workspace_bytes",
    "dkv_kivi_subspace_correct",
    "dkv_lora_scores",
    "dkv_row_diff_norms",
    "dkv_sym_eig_batched",
    "dkv_gram_subspace_iterate",
    "dkv_split_gemm_batched",
    "dkv_attn_first_order",
    "dkv_rmsnorm_first_order",
    "dkv_swiglu_first_order",
    "dkv_rope_rows",
    "dkv_subspace_workspace_bytes",
    "dkv_subspace_correct",
    "dkv_subspace_correct_noalloc",
    "dkv_subspace_correct_batched_workspace_bytes",
    "dkv_subspace_correct_batched",
    "dkv_subspace_probe_residual",
)


class PagedCache(C.Structure):
    _fields_ = [
        ("base", C.c_void_p),
        ("dtype", C.c_int32),
        ("block_size", C.c_int32),
        ("n_heads", C.c_int32),
        ("head_dim", C.c_int32),
        ("num_blocks", C.c_int64),
        ("stride_block", C.c_int64),
        ("stride_slot", C.c_int64),
        ("stride_head", C.c_int64),
    ]


class SeqBatch(C.Structure):
    _fields_ = [
        ("cu_seqlens", C.c_void_p),
        ("block_tables", C.c_void_p),
        ("table_lens", C.c_void_p),
        ("positions", C.c_void_p),
        ("table_stride", C.c_int64),
        ("n_seqs", C.c_int32),
        ("max_seq_len", C.c_int32),
    ]


class LoraFactors(C.Structure):
    _fields_ = [
        ("a_k", C.c_void_p),
        ("b_k", C.c_void_p),
        ("a_v", C.c_void_p),
        ("b_v", C.c_void_p),
        ("dtype", C.c_int32),
        ("rank_k", C.c_int32),
        ("rank_v", C.c_int32),
        ("n_layers", C.c_int32),
        ("scale_k", C.c_float),
        ("scale_v", C.c_float),
        ("a_k_layer_stride", C.c_int64),
        ("b_k_layer_stride", C.c_int64),
        ("a_v_layer_stride", C.c_int64),
        ("b_v_layer_stride", C.c_int64),
        ("norm_weight", C.c_void_p),
        ("norm_dtype", C.c_int32),
        ("norm_layer_stride", C.c_int64),
    ]


class ExactGeometry(C.Structure):
    _fields_ = [
        ("d_model", C.c_int32),
        ("n_kv_heads", C.c_int32),
        ("head_dim", C.c_int32),
        ("x_dtype", C.c_int32),
        ("rank_k", C.c_int32),
        ("rank_v", C.c_int32),
    ]


class ExactPatchArgs(C.Structure):
    _fields_ = [
        ("geom", ExactGeometry),
        ("x", C.c_void_p),
        ("x_layer_stride", C.c_int64),
        ("x_row_stride", C.c_int64),
        ("x_rows", C.c_int64),
        ("x_scale", C.c_void_p),
        ("x_scale_layer_stride", C.c_int64),
        ("apply_norm", C.c_int32),
        ("norm_eps", C.c_float),
        ("packed", C.c_void_p),
        ("packed_layer_stride", C.c_int64),
        ("rope_cos", C.c_void_p),
        ("rope_sin", C.c_void_p),
        ("rope_max_pos", C.c_int32),
        ("n_layers", C.c_int32),
        ("seqs", SeqBatch),
        ("k_pages", C.POINTER(PagedCache)),
        ("v_pages", C.POINTER(PagedCache)),
        ("accumulate", C.c_int32),
        ("status", C.c_void_p),
        ("x_sumsq", C.c_void_p),
        ("x_sumsq_layer_stride", C.c_int64),
    ]


DKV_KIVI_PER_CHANNEL, DKV_KIVI_PER_TOKEN = 0, 1


class KiviCache(C.Structure):
    _fields_ = [
        ("codes", C.c_void_p),
        ("scale", C.c_void_p),
        ("zero", C.c_void_p),
        ("code_row_stride", C.c_int64),
        ("sz_row_stride", C.c_int64),
        ("n_tokens", C.c_int64),
        ("d", C.c_int64),
        ("mode", C.c_int32),
    ]


class KiviProbeJob(C.Structure):
    _fields_ = [
        ("base", KiviCache),
        ("fresh", C.c_void_p),
        ("fresh_row_stride", C.c_int64),
        ("rows", C.c_void_p),
    ]


class KiviSubspaceProblem(C.Structure):
    _fields_ = [
        ("base", KiviCache),
        ("out", KiviCache),
        ("fresh", C.c_void_p),
        ("fresh_dtype", C.c_int32),
        ("fresh_row_stride", C.c_int64),
        ("probe_index", C.c_void_p),
        ("n_probes", C.c_int64),
        ("basis", C.c_void_p),
        ("rank", C.c_int32),
        ("subspace_out", C.c_void_p),
        ("orth_mu_out", C.c_void_p),
    ]


class DenseGeometry(C.Structure):
    _fields_ = [("d_model", C.c_int32), ("n_kv_heads", C.c_int32), ("head_dim", C.c_int32)]


class DenseDelta(C.Structure):
    _fields_ = [
        ("dw_k", C.c_void_p),
        ("dw_v", C.c_void_p),
        ("dtype", C.c_int32),
        ("n_layers", C.c_int32),
        ("dw_k_layer_stride", C.c_int64),
        ("dw_v_layer_stride", C.c_int64),
        ("norm_weight", C.c_void_p),
        ("norm_dtype", C.c_int32),
        ("norm_layer_stride", C.c_int64),
        ("scale_k", C.c_float),
        ("scale_v", C.c_float),
    ]


class DensePatchArgs(C.Structure):
    _fields_ = [
        ("geom", DenseGeometry),
        ("x", C.c_void_p),
        ("x_layer_stride", C.c_int64),
        ("x_row_stride", C.c_int64),
        ("x_rows", C.c_int64),
        ("x_scale", C.c_void_p),
        ("x_scale_layer_stride", C.c_int64),
        ("packed", C.c_void_p),
        ("packed_layer_stride", C.c_int64),
        ("rope_cos", C.c_void_p),
        ("rope_sin", C.c_void_p),
        ("rope_max_pos", C.c_int32),
        ("n_layers", C.c_int32),
        ("do_k", C.c_int32),
        ("do_v", C.c_int32),
        ("seqs", SeqBatch),
        ("k_pages", C.POINTER(PagedCache)),
        ("v_pages", C.POINTER(PagedCache)),
        ("accumulate", C.c_int32),
        ("status", C.c_void_p),
    ]


class SubspaceArgs(C.Structure):
    _fields_ = [
        ("reused", C.c_void_p),
        ("fresh", C.c_void_p),
        ("kv_dtype", C.c_int32),
        ("n_tokens", C.c_int64),
        ("d", C.c_int64),
        ("reused_row_stride", C.c_int64),
        ("fresh_row_stride", C.c_int64),
        ("probe_index", C.c_void_p),
        ("n_probes", C.c_int64),
        ("basis", C.c_void_p),
        ("rank", C.c_int32),
        ("token_weights", C.c_void_p),
        ("corrected", C.c_void_p),
        ("out_dtype", C.c_int32),
        ("out_row_stride", C.c_int64),
        ("subspace_out", C.c_void_p),
        ("orth_mu_out", C.c_void_p),
        ("workspace", C.c_void_p),
        ("workspace_bytes", C.c_int64),
    ]


_lib: C.CDLL | None = None


def _declare(lib: C.CDLL) -> None:
    P, I32, I64 = C.c_void_p, C.c_int32, C.c_int64
    lib.dkv_status_string.restype = C.c_char_p
    lib.dkv_status_string.argtypes = [C.c_int]
    lib.dkv_abi_version.restype = C.c_int
    lib.dkv_abi_version.argtypes = []
    lib.dkv_last_cuda_error.restype = C.c_char_p
    lib.dkv_last_cuda_error.argtypes = []
    lib.dkv_scatter_paged.restype = C.c_int
    lib.dkv_scatter_paged.argtypes = [P, I32, I64, I64, C.POINTER(PagedCache), C.POINTER(SeqBatch), P, P]
    lib.dkv_gather_paged.restype = C.c_int
    lib.dkv_gather_paged.argtypes = [C.POINTER(PagedCache), C.POINTER(SeqBatch), P, I32, I64, I64, P, P]
    lib.dkv_paged_error_sums.restype = C.c_int
    lib.dkv_paged_error_sums.argtypes = [C.POINTER(PagedCache), I32, P, I32, I64, I64, I64, C.POINTER(SeqBatch),
                                         P, P, P]
    lib.dkv_paged_compare_sums.restype = C.c_int
    lib.dkv_paged_compare_sums.argtypes = [C.POINTER(PagedCache), I32, P, I32, I64, I64, I64, C.POINTER(SeqBatch),
                                           P, P, P]
    lib.dkv_quantize_rows.restype = C.c_int
    lib.dkv_quantize_rows.argtypes = [P, I32, I64, I64, I64, P, I32, I64, I64, P, P]
    lib.dkv_quantize_rows_sumsq.restype = C.c_int
    lib.dkv_quantize_rows_sumsq.argtypes = [P, I32, I64, I64, I64, P, I32, I64, I64, P, P, P]
    lib.dkv_exact_packed_bytes.restype = C.c_int
    lib.dkv_exact_packed_bytes.argtypes = [C.POINTER(ExactGeometry), C.POINTER(C.c_int64)]
    lib.dkv_pack_exact_factors.restype = C.c_int
    lib.dkv_pack_exact_factors.argtypes = [C.POINTER(ExactGeometry), C.POINTER(LoraFactors), P, I64, P]
    lib.dkv_exact_patch_paged.restype = C.c_int
    lib.dkv_exact_patch_paged.argtypes = [C.POINTER(ExactPatchArgs), P]
    lib.dkv_pack_dense_delta.restype = C.c_int
    lib.dkv_pack_dense_delta.argtypes = [C.POINTER(DenseGeometry), C.POINTER(DenseDelta), P, I64, P]
    lib.dkv_dense_patch_paged.restype = C.c_int
    lib.dkv_dense_patch_paged.argtypes = [C.POINTER(DensePatchArgs), P]
    lib.dkv_row_inv_rms.restype = C.c_int
    lib.dkv_row_inv_rms.argtypes = [P, I32, I64, I64, I64, C.c_float, P, P]
    lib.dkv_kivi_quantize.restype = C.c_int
    lib.dkv_kivi_quantize.argtypes = [P, I32, I64, C.POINTER(KiviCache), P]
    lib.dkv_kivi_dequantize.restype = C.c_int
    lib.dkv_kivi_dequantize.argtypes = [C.POINTER(KiviCache), P, I32, I64, P]
    lib.dkv_kivi_patch.restype = C.c_int
    lib.dkv_kivi_patch.argtypes = [C.POINTER(KiviCache), P, I32, I64, C.POINTER(KiviCache), P]
    lib.dkv_kivi_probe_residual.restype = C.c_int
    lib.dkv_kivi_probe_residual.argtypes = [C.POINTER(KiviCache), P, I32, I64, P, I64, P, I64, P, P]
    lib.dkv_kivi_probe_residual_batched.restype = C.c_int
    lib.dkv_kivi_probe_residual_batched.argtypes = [C.POINTER(KiviProbeJob), I32, I32, I64, P, I64, I64, P, P]
    lib.dkv_kivi_subspace_workspace_bytes.restype = C.c_int
    lib.dkv_kivi_subspace_workspace_bytes.argtypes = [C.POINTER(KiviSubspaceProblem), I32, C.POINTER(C.c_int64)]
    lib.dkv_kivi_subspace_correct.restype = C.c_int
    lib.dkv_kivi_subspace_correct.argtypes = [C.POINTER(KiviSubspaceProblem), I32, P, I64, P, P]
    lib.dkv_lora_scores.restype = C.c_int
    lib.dkv_lora_scores.argtypes = [P, I32, I64, I64, I64, P, I32, C.c_float, P, I32, P]
    lib.dkv_row_diff_norms.restype = C.c_int
    lib.dkv_row_diff_norms.argtypes = [P, P, I32, I64, I64, I64, I64, P, I64, P, P, P]
    lib.dkv_sym_eig_batched.restype = C.c_int
    lib.dkv_sym_eig_batched.argtypes = [P, I64, I32, I64, I32, P, P, P, P]
    lib.dkv_gram_subspace_iterate.restype = C.c_int
    lib.dkv_gram_subspace_iterate.argtypes = [P, I32, P, I32, I32, P, P, P, P, P]
    lib.dkv_split_gemm_batched.restype = C.c_int
    lib.dkv_split_gemm_batched.argtypes = [P, I64, I64, I32, P, I64, I64, P, I64, I64, I64, I32, I32, I32, P]
    lib.dkv_attn_first_order.restype = C.c_int
    lib.dkv_attn_first_order.argtypes = [P, P, I64, P, P, P, P, I64, I32, I32, I32, I32, I32, C.c_float, P, P, I64,
                                         P]
    lib.dkv_rmsnorm_first_order.restype = C.c_int
    lib.dkv_rmsnorm_first_order.argtypes = [P, P, P, C.c_float, I64, I32, I64, I64, P, P, I64, I64, P]
    lib.dkv_swiglu_first_order.restype = C.c_int
    lib.dkv_swiglu_first_order.argtypes = [P, P, P, P, I64, P, P, P]
    lib.dkv_rope_rows.restype = C.c_int
    lib.dkv_rope_rows.argtypes = [P, I64, I32, I32, I64, P, P, I64, P]
    lib.dkv_subspace_workspace_bytes.restype = C.c_int
    lib.dkv_subspace_workspace_bytes.argtypes = [I64, I64, I32, C.POINTER(C.c_int64)]
    lib.dkv_subspace_correct.restype = C.c_int
    lib.dkv_subspace_correct.argtypes = [C.POINTER(SubspaceArgs), P]
    lib.dkv_subspace_correct_noalloc.restype = C.c_int
    lib.dkv_subspace_correct_noalloc.argtypes = [C.POINTER(SubspaceArgs), P]
    lib.dkv_subspace_correct_batched_workspace_bytes.restype = C.c_int
    lib.dkv_subspace_correct_batched_workspace_bytes.argtypes = [C.POINTER(SubspaceArgs), I32, C.POINTER(C.c_int64)]
    lib.dkv_subspace_correct_batched.restype = C.c_int
    lib.dkv_subspace_correct_batched.argtypes = [C.POINTER(SubspaceArgs), I32, P, I64, P]
    lib.dkv_subspace_probe_residual.restype = C.c_int
    lib.dkv_subspace_probe_residual.argtypes = [P, P, I32, I64, I64, I64, I64, P, I64, P, P]


def lib() -> C.CDLL:
    """The loaded library; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(
                f"{LIB_PATH.name} is not built; run `python -m deltakv_b200.build` "
                "(the CUDA path has no fallback)"
            )
        handle = C.CDLL(str(LIB_PATH))
        _declare(handle)
        if handle.dkv_abi_version() != ABI_VERSION:
            raise ImportError(f"{LIB_PATH.name} ABI version mismatch; rebuild the library")
        _lib = handle
    return _lib


class DkvError(RuntimeError):
    def __init__(self, status: int, where: str = ""):
        self.status = status
        msg = lib().dkv_status_string(status).decode()
        if status == DKV_ERR_CUDA:
            msg += f" [{lib().dkv_last_cuda_error().decode()}]"
        super().__init__(f"{where}: {msg} (status {status})" if where else msg)


def check(status: int, where: str = "") -> None:
    if status != DKV_OK:
        raise DkvError(status, where)
