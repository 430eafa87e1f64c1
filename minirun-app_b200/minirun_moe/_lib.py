"""ctypes binding of libminirun_moe.so (include/minirun_moe.h).

This module is the reference-side binding a host would add: every struct and
function below mirrors the C header one to one. Loading fails loudly when the
library has not been built — there is no CPU fallback anywhere in the package.
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
# MINIRUN_MOE_LIB selects another build of the same library (e.g. one built
# with different compile flags); the default is the in-tree build.
LIB_PATH = os.environ.get("MINIRUN_MOE_LIB") or os.path.join(_HERE, "_lib", "libminirun_moe.so")

MR_OK = 0
MR_ERR_INVALID_ARGUMENT = 1
MR_ERR_UNSUPPORTED = 2
MR_ERR_CUDA = 3
MR_ERR_OUT_OF_MEMORY = 4
MR_ERR_DEVICE = 5
MR_ERR_TIMEOUT = 6
MR_ERR_BUDGET = 7
MR_ERR_NCCL = 8
MR_ERR_STATE = 9
MR_ERR_IO = 10
MR_ERR_INTEGRITY = 11
MR_DEVERR_BAD_TOKEN_ID = 0x10

MR_DTYPE_BF16, MR_DTYPE_F16, MR_DTYPE_F32, MR_DTYPE_E8M0 = 0, 1, 2, 3
MR_SCORING_SIGMOID, MR_SCORING_SOFTMAX, MR_SCORING_SQRT_SOFTPLUS = 0, 1, 2
MR_RENORM_NONE, MR_RENORM_PLAIN, MR_RENORM_EPS = 0, 1, 2
MR_WEIGHT_BEFORE_DOWN, MR_WEIGHT_AFTER_DOWN = 0, 1
MR_DEVERR_BAD_EXPERT_ID, MR_DEVERR_NONFINITE_SCORE, MR_DEVERR_RENORM_ZERO = 1, 2, 4

vp = C.c_void_p


class mr_affine_desc(C.Structure):
    _fields_ = [("packed", vp), ("scales", vp), ("biases", vp), ("experts", C.c_int32),
                ("out_features", C.c_int64), ("in_features", C.c_int64),
                ("group_size", C.c_int32), ("bits", C.c_int32), ("scale_dtype", C.c_int)]


class mr_mxfp4_desc(C.Structure):
    _fields_ = [("packed", vp), ("scales", vp), ("experts", C.c_int32),
                ("out_features", C.c_int64), ("in_features", C.c_int64)]


class mr_router_config(C.Structure):
    _fields_ = [("experts", C.c_int32), ("top_k", C.c_int32), ("scoring", C.c_int),
                ("renorm", C.c_int), ("renorm_eps", C.c_float), ("routed_scale", C.c_float),
                ("correction_bias", vp)]


class mr_k3_projection(C.Structure):
    _fields_ = [("kind", C.c_int32), ("dense", vp), ("dense_dtype", C.c_int),
                ("out_features", C.c_int64), ("in_features", C.c_int64), ("mx", mr_mxfp4_desc)]


class mr_k3_moe(C.Structure):
    _fields_ = [("router", mr_router_config), ("gate_weight", vp), ("gate_dtype", C.c_int),
                ("routed_down", mr_k3_projection), ("routed_up", mr_k3_projection),
                ("routed_norm", vp), ("norm_dtype", C.c_int), ("rms_eps", C.c_float),
                ("w1", mr_mxfp4_desc), ("w3", mr_mxfp4_desc), ("w2", mr_mxfp4_desc),
                ("shared_gate", mr_k3_projection), ("shared_up", mr_k3_projection),
                ("shared_down", mr_k3_projection), ("hidden", C.c_int64), ("latent", C.c_int64),
                ("inter", C.c_int64), ("shared_inter", C.c_int64), ("situ_beta", C.c_float),
                ("situ_linear_beta", C.c_float)]


MR_K3_PROJ_DENSE, MR_K3_PROJ_MXFP4 = 0, 1


class mr_expert_ptrs(C.Structure):
    _fields_ = [("packed", vp * 3), ("scales", vp * 3), ("biases", vp * 3)]


class mr_moe_layer(C.Structure):
    _fields_ = [("hidden", C.c_int64), ("inter", C.c_int64), ("shared_inter", C.c_int64),
                ("router", mr_router_config), ("router_w", vp),
                ("gate", mr_affine_desc), ("up", mr_affine_desc), ("down", mr_affine_desc),
                ("expert_table", vp),
                ("shared_gate", mr_affine_desc), ("shared_up", mr_affine_desc),
                ("shared_down", mr_affine_desc),
                ("swiglu_limit", C.c_float), ("weight_placement", C.c_int)]


class mr_expert_host(C.Structure):
    _fields_ = [("packed", vp * 3), ("scales", vp * 3), ("biases", vp * 3),
                ("packed_bytes", C.c_size_t * 3), ("scale_bytes", C.c_size_t * 3)]


class mr_tile_layout(C.Structure):
    _fields_ = [("rows", C.c_int32), ("cols", C.c_int32), ("group_size", C.c_int32),
                ("bits", C.c_int32), ("quant_mode", C.c_int32), ("scale_dtype", C.c_int32),
                ("scale_block_rows", C.c_int32), ("version", C.c_int32),
                ("content_kind", C.c_int32), ("feature_flags", C.c_uint32),
                ("tile_count", C.c_int64), ("seed", C.c_uint64),
                ("packed_bytes", C.c_int64), ("scale_bytes", C.c_int64),
                ("bias_bytes", C.c_int64), ("scale_offset", C.c_int64),
                ("bias_offset", C.c_int64), ("tile_stride", C.c_int64),
                ("first_tile_offset", C.c_int64), ("total_bytes", C.c_int64),
                ("packed_region_bytes", C.c_int64), ("scale_region_bytes", C.c_int64)]


class mr_cache_stats(C.Structure):
    _fields_ = [("slots", C.c_int64), ("resident", C.c_int64), ("hits", C.c_int64),
                ("misses", C.c_int64), ("evictions", C.c_int64), ("bytes_copied", C.c_int64),
                ("prefetched", C.c_int64)]


# name -> (restype, argtypes); the complete exported surface of the header
SIGNATURES = {
    "mr_abi_version": (C.c_int, []),
    "mr_status_string": (C.c_char_p, [C.c_int]),
    "mr_ctx_create": (C.c_int, [C.c_int, C.POINTER(vp)]),
    "mr_ctx_destroy": (C.c_int, [vp]),
    "mr_last_error": (C.c_char_p, [vp]),
    "mr_ctx_check": (C.c_int, [vp, vp, C.POINTER(C.c_uint32)]),
    "mr_ctx_reserve": (C.c_int, [vp, C.c_int64, C.c_int32, C.c_int32, C.c_int64, C.c_int64]),
    "mr_ctx_set_kernel_path": (C.c_int, [vp, C.c_int]),
    "mr_affine_validate": (C.c_int, [C.POINTER(mr_affine_desc), C.c_char_p, C.c_size_t]),
    "mr_affine_mm": (C.c_int, [vp, vp, C.c_int64, C.POINTER(mr_affine_desc), vp, vp]),
    "mr_affine_gather_mm": (C.c_int, [vp, vp, C.c_int64, vp, C.c_int32,
                                      C.POINTER(mr_affine_desc), vp, vp]),
    "mr_affine_dequantize": (C.c_int, [vp, C.POINTER(mr_affine_desc), vp, vp]),
    "mr_affine_gather_mm_noalloc": (C.c_int, [vp, C.c_int64, vp, C.c_int32,
                                              C.POINTER(mr_affine_desc), vp, vp, C.c_char_p,
                                              C.c_size_t]),
    "mr_ep_set_fused": (C.c_int, [vp, C.c_int]),
    "mr_ep_set_mode": (C.c_int, [vp, C.c_int]),
    "mr_ep_set_placement": (C.c_int, [vp, C.c_int]),
    "mr_ep_set_capacity": (C.c_int, [vp, C.c_int64]),
    "mr_ep_init": (C.c_int, [vp, vp, C.c_int, C.c_int, C.POINTER(vp)]),
    "mr_test_expire_ep_wait": (C.c_int, [vp, C.c_int64, C.c_int64, C.c_uint32, vp, vp]),
    "mr_mxfp4_validate": (C.c_int, [C.POINTER(mr_mxfp4_desc), C.c_char_p, C.c_size_t]),
    "mr_mxfp4_mm": (C.c_int, [vp, vp, C.c_int64, C.POINTER(mr_mxfp4_desc), vp, vp]),
    "mr_mxfp4_gather_mm": (C.c_int, [vp, vp, C.c_int64, vp, C.c_int32,
                                     C.POINTER(mr_mxfp4_desc), vp, vp]),
    "mr_mxfp4_dequantize": (C.c_int, [vp, C.POINTER(mr_mxfp4_desc), vp, vp]),
    "mr_mxfp4_mm_f32": (C.c_int, [vp, vp, C.c_int64, C.POINTER(mr_mxfp4_desc), vp, vp]),
    "mr_mxfp4_gather_mm_f32": (C.c_int, [vp, vp, C.c_int64, vp, C.c_int32,
                                         C.POINTER(mr_mxfp4_desc), vp, vp]),
    "mr_dense_mm_f32": (C.c_int, [vp, vp, C.c_int64, vp, C.c_int, C.c_int64, C.c_int64, vp, vp]),
    "mr_k3_situ": (C.c_int, [vp, vp, C.c_int64, C.c_int64, C.c_float, C.c_float, vp, vp]),
    "mr_k3_moe_validate": (C.c_int, [C.POINTER(mr_k3_moe), C.c_char_p, C.c_size_t]),
    "mr_k3_moe_forward": (C.c_int, [vp, C.POINTER(mr_k3_moe), vp, C.c_int64, vp, vp, vp, vp]),
    "mr_router_config_validate": (C.c_int, [C.POINTER(mr_router_config), C.c_char_p,
                                            C.c_size_t]),
    "mr_router_select": (C.c_int, [vp, vp, C.c_int64, C.c_int64, vp,
                                   C.POINTER(mr_router_config), vp, vp, vp, vp, vp]),
    "mr_router_select_logits": (C.c_int, [vp, vp, C.c_int64, C.POINTER(mr_router_config),
                                          vp, vp, vp, vp]),
    "mr_moe_layer_validate": (C.c_int, [C.POINTER(mr_moe_layer), C.c_char_p, C.c_size_t]),
    "mr_moe_layer_forward": (C.c_int, [vp, C.POINTER(mr_moe_layer), vp, C.c_int64, vp, vp, vp,
                                       vp, vp]),
    "mr_moe_layer_forward_host": (C.c_int, [vp, C.POINTER(mr_moe_layer), vp, C.c_int64, vp, vp,
                                            vp]),
    "mr_ep_unique_id": (C.c_int, [vp]),
    "mr_ep_create": (C.c_int, [vp, vp, C.c_int, C.c_int, C.POINTER(vp)]),
    "mr_ep_destroy": (C.c_int, [vp]),
    "mr_moe_layer_forward_ep": (C.c_int, [vp, vp, C.POINTER(mr_moe_layer), vp, C.c_int64, vp, vp,
                                          vp]),
    "mr_cache_create": (C.c_int, [vp, C.c_size_t, C.c_size_t, C.POINTER(vp)]),
    "mr_cache_destroy": (C.c_int, [vp]),
    "mr_cache_register": (C.c_int, [vp, C.c_int32, C.c_int32, C.POINTER(mr_expert_host)]),
    "mr_cache_get_stats": (C.c_int, [vp, C.POINTER(mr_cache_stats)]),
    "mr_cache_set_policy": (C.c_int, [vp, C.c_int, vp, vp, C.c_int64]),
    "mr_cache_prefetch": (C.c_int, [vp, C.c_int32, vp, C.c_int64, vp]),
    "mr_cache_register_tiles": (C.c_int, [vp, C.c_int32, C.c_int32, vp * 3, C.c_int64 * 3]),
    "mr_tiles_open": (C.c_int, [C.c_char_p, C.c_int, C.POINTER(vp), C.c_char_p, C.c_size_t]),
    "mr_tiles_close": (C.c_int, [vp]),
    "mr_tiles_get_layout": (C.c_int, [vp, C.POINTER(mr_tile_layout)]),
    "mr_tiles_read": (C.c_int, [vp, C.c_int64, vp, C.c_size_t, C.c_char_p, C.c_size_t]),
    "mr_tiles_layout_for": (C.c_int, [C.POINTER(mr_tile_layout), C.c_int64, C.c_int,
                                      C.c_char_p, C.c_size_t]),
    "mr_tiles_encode_header": (C.c_int, [C.POINTER(mr_tile_layout), vp, vp, C.c_char_p,
                                         C.c_size_t]),
    "mr_sha256": (C.c_int, [vp, C.c_size_t, vp]),
    "mr_token_map_validate": (C.c_int, [vp, C.c_int64, C.c_int32, C.c_int32, C.c_char_p,
                                        C.c_size_t]),
    "mr_router_select_hashed": (C.c_int, [vp, vp, C.c_int64, C.c_int64, vp,
                                          C.POINTER(mr_router_config), vp, vp, C.c_int64, vp,
                                          vp, vp, vp]),
    "mr_moe_layer_forward_hashed": (C.c_int, [vp, C.POINTER(mr_moe_layer), vp, vp, C.c_int64,
                                              vp, C.c_int64, vp, vp, vp, vp]),
    "mr_moe_layer_forward_cached": (C.c_int, [vp, vp, C.c_int32, C.POINTER(mr_moe_layer), vp,
                                              C.c_int64, vp, vp, vp]),
    "mr_ctx_profile": (C.c_int, [vp, C.c_int]),
    "mr_ctx_profile_read": (C.c_int, [vp, C.POINTER(C.c_double), C.POINTER(C.c_int64), C.c_int]),
    "mr_synth_label": (C.c_uint64, [C.c_uint32] * 4),
    "mr_synth_derive": (C.c_uint64, [C.c_uint64, C.c_uint64]),
    "mr_synth_words": (C.c_int, [vp, C.c_uint64, C.c_int64, vp, vp]),
    "mr_synth_normal_bf16": (C.c_int, [vp, C.c_uint64, C.c_int64, C.c_double, C.c_int, vp, vp]),
    "mr_synth_affine_biases": (C.c_int, [vp, vp, C.c_int64, C.c_int32, vp, vp]),
}

_lib = None


class LibraryMissing(RuntimeError):
    pass


def load():
    """Load the built library (raises LibraryMissing if it was not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise LibraryMissing(
                f"{LIB_PATH} is missing: build it with `make -C minirun-app_b200/csrc` "
                "(or __graft_entry__.build()); there is no CPU fallback")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib
