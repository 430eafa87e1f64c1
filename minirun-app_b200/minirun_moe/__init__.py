"""minirun_moe — B200 (sm_100a) MoE-expert hot path of Minirun, over a C ABI.

The package is the host-side mirror of the reference's MLXBridge affine op
API and its MoE block (nanguoyu/minirun-app); all arithmetic runs in
libminirun_moe.so (``minirun-app_b200/csrc``), which must be built — there is
no CPU fallback.
"""
from ._lib import LIB_PATH, LibraryMissing, load as load_library
from .bridge import (AffineBridgeError, AffineWeights, Context, MoeError, Selection,
                     affine_dequantize, affine_gather_mm, affine_mm, validate_desc)
from .cache import CachedLayer, ExpertCache
from .ep import ExpertGroup, MoELayerShard
from .moe import (MoELayer, ResidentExpertBackend, RouterConfig, TokenExpertMap, router_select,
                  router_select_hashed, router_select_logits)
from .checkpoint import Checkpoint, SafetensorsError, SafetensorsFile, write_safetensors
from .mxfp4 import (MXFP4BridgeError, MXFP4Weights, mxfp4_dequantize, mxfp4_gather_mm,
                    mxfp4_gather_mm_f32, mxfp4_mm, mxfp4_mm_f32, mxfp4_validate)
from .k3 import K3MoE, K3Projection, dense_mm_f32, situ
from .tiles import (ExpertContainers, TileContainer, TileContainerError, write_container,
                    write_expert_containers)

__all__ = [
    "LIB_PATH", "LibraryMissing", "load_library", "AffineBridgeError", "AffineWeights",
    "Context", "MoeError", "Selection", "affine_dequantize", "affine_gather_mm", "affine_mm",
    "validate_desc", "MoELayer", "ResidentExpertBackend", "RouterConfig", "router_select",
    "router_select_logits", "ExpertGroup", "MoELayerShard", "CachedLayer", "ExpertCache",
    "ExpertContainers", "TileContainer", "TileContainerError", "write_container",
    "write_expert_containers", "Checkpoint", "SafetensorsError", "SafetensorsFile",
    "write_safetensors", "TokenExpertMap", "router_select_hashed", "MXFP4BridgeError",
    "MXFP4Weights", "mxfp4_dequantize", "mxfp4_gather_mm", "mxfp4_mm", "mxfp4_validate",
    "mxfp4_gather_mm_f32", "mxfp4_mm_f32", "K3MoE", "K3Projection", "dense_mm_f32", "situ",
]
