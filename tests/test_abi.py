"""The C ABI and the host-side logic, without a GPU.

* libminirun_moe.so loads and exports every function include/minirun_moe.h
  declares (no compute call is made here);
* the host-only validators (mr_affine_validate, mr_router_config_validate,
  mr_moe_layer_validate) refuse what the reference refuses
  (AffineWeights.swift:84-157, DeepSeekV4Routing.swift:133-146,
  DeepSeekV4HashFFN.swift:132-151) and accept the BASELINE configs;
* the Python AffineWeights mirror raises the reference's AffineBridgeError
  messages.
"""
import ctypes as C
import os
import re

import pytest
import torch

import minirun_moe as M
from minirun_moe import _lib as L

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "minirun_moe.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(mr_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    lib = L.load()
    names = declared_functions()
    assert len(names) >= 20
    for n in names:
        assert hasattr(lib, n), n
    assert set(names) == set(L.SIGNATURES), set(names) ^ set(L.SIGNATURES)


def test_abi_version_and_status_strings():
    lib = L.load()
    assert lib.mr_abi_version() == 1
    assert lib.mr_status_string(L.MR_ERR_BUDGET) == b"budget refused"
    assert lib.mr_status_string(99) == b"unknown status"


def test_struct_layout_matches_c_compiler(tmp_path):
    """ctypes mirrors of the header structs agree with gcc on size and offsets."""
    import subprocess
    prog = tmp_path / "layout.c"
    checks = [("mr_affine_desc", ["packed", "experts", "out_features", "bits", "scale_dtype"]),
              ("mr_router_config", ["top_k", "renorm_eps", "correction_bias"]),
              ("mr_expert_ptrs", ["scales", "biases"]),
              ("mr_moe_layer", ["router", "router_w", "gate", "expert_table", "shared_down",
                                "swiglu_limit", "weight_placement"]),
              ("mr_expert_host", ["scales", "biases", "packed_bytes", "scale_bytes"]),
              ("mr_cache_stats", ["resident", "hits", "evictions", "bytes_copied"]),
              ("mr_tile_layout", ["bits", "feature_flags", "tile_count", "seed", "packed_bytes",
                                  "bias_offset", "total_bytes", "scale_region_bytes"]),
              ("mr_mxfp4_desc", ["packed", "scales", "experts", "out_features", "in_features"]),
              ("mr_k3_projection", ["kind", "dense", "dense_dtype", "in_features", "mx"]),
              ("mr_k3_moe", ["router", "gate_weight", "routed_down", "routed_norm", "rms_eps",
                             "w1", "w2", "shared_down", "shared_inter", "situ_linear_beta"])]
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "minirun_moe.h"',
             "int main(void) {"]
    for s, fields in checks:
        lines.append(f'printf("{s} %zu\\n", sizeof({s}));')
        for f in fields:
            lines.append(f'printf("{s}.{f} %zu\\n", offsetof({s}, {f}));')
    lines.append("return 0; }")
    prog.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), str(prog), "-o", str(exe)],
                   check=True)
    got = dict(line.split() for line in subprocess.check_output([str(exe)]).decode().split("\n")
               if line)
    for s, fields in checks:
        cls = getattr(L, s)
        assert int(got[s]) == C.sizeof(cls), s
        for f in fields:
            assert int(got[f"{s}.{f}"]) == getattr(cls, f).offset, f"{s}.{f}"


def _desc(**kw):
    d = dict(packed=16, scales=32, biases=48, experts=4, out_features=64, in_features=128,
             group_size=64, bits=4, scale_dtype=L.MR_DTYPE_BF16)
    d.update(kw)
    return L.mr_affine_desc(**d)


@pytest.mark.parametrize("kw,status,needle", [
    ({}, L.MR_OK, ""),
    ({"bits": 3}, L.MR_ERR_INVALID_ARGUMENT, "must divide 32"),
    ({"group_size": 0}, L.MR_ERR_INVALID_ARGUMENT, "group size must be positive"),
    ({"in_features": 96}, L.MR_ERR_INVALID_ARGUMENT, "not a multiple of the group size"),
    ({"scale_dtype": 7}, L.MR_ERR_INVALID_ARGUMENT, "floating-point type"),
    ({"packed": 0}, L.MR_ERR_INVALID_ARGUMENT, "non-NULL"),
    ({"bits": 16}, L.MR_ERR_UNSUPPORTED, "not built here"),
    ({"group_size": 32}, L.MR_ERR_UNSUPPORTED, "not built here"),
])
def test_affine_validate(kw, status, needle):
    buf = C.create_string_buffer(256)
    d = _desc(**kw)
    assert L.load().mr_affine_validate(C.byref(d), buf, 256) == status
    assert needle in buf.value.decode()


@pytest.mark.parametrize("cfg,status", [
    (M.RouterConfig(256, 8, routed_scale=2.5), L.MR_OK),
    (M.RouterConfig.deepseek_v4(256, 6, scale=1.5), L.MR_OK),
    (M.RouterConfig.qwen(128, 8), L.MR_OK),
    (M.RouterConfig(8, 8), L.MR_ERR_INVALID_ARGUMENT),
    (M.RouterConfig(8, 0), L.MR_ERR_INVALID_ARGUMENT),
    (M.RouterConfig(8, 2, routed_scale=0.0), L.MR_ERR_INVALID_ARGUMENT),
    (M.RouterConfig(2048, 8), L.MR_ERR_UNSUPPORTED),
])
def test_router_config_validate(cfg, status):
    assert cfg.validate()[0] == status


def _cpu_affine(E, out, inn, bits=4, dtype=torch.bfloat16):
    lead = [E] if E else []
    return M.AffineWeights(torch.zeros(lead + [out, inn * bits // 32], dtype=torch.int32),
                           torch.zeros(lead + [out, inn // 64], dtype=dtype),
                           torch.zeros(lead + [out, inn // 64], dtype=dtype), 64, bits)


def _layer_struct(E=16, k=2, H=1024, I=512, S=512, bits=4, shared_bits=None, swiglu=0.0):
    c = L.mr_moe_layer()
    c.hidden, c.inter, c.shared_inter = H, I, S
    c.router = M.RouterConfig(E, k).c()
    c.router_w = 4096
    c.gate = _cpu_affine(E, I, H, bits).desc()
    c.up = _cpu_affine(E, I, H, bits).desc()
    c.down = _cpu_affine(E, H, I, bits).desc()
    if S:
        sb = shared_bits or bits
        c.shared_gate = _cpu_affine(None, S, H, sb).desc()
        c.shared_up = _cpu_affine(None, S, H, sb).desc()
        c.shared_down = _cpu_affine(None, H, S, sb).desc()
    c.swiglu_limit = swiglu
    return c


@pytest.mark.parametrize("kw,status,needle", [
    ({}, L.MR_OK, ""),
    ({"S": 0}, L.MR_OK, ""),
    ({"E": 16, "k": 16}, L.MR_ERR_INVALID_ARGUMENT, "expertsPerToken"),
    ({"swiglu": -1.0}, L.MR_ERR_INVALID_ARGUMENT, "SwiGLU limit"),
    ({"shared_bits": 8}, L.MR_ERR_UNSUPPORTED, "shared expert must share bits"),
])
def test_layer_validate(kw, status, needle):
    c = _layer_struct(**kw)
    buf = C.create_string_buffer(256)
    assert L.load().mr_moe_layer_validate(C.byref(c), buf, 256) == status
    assert needle in buf.value.decode()


def test_layer_validate_catches_wrong_stack_shape():
    c = _layer_struct()
    c.down = _cpu_affine(16, 512, 1024).desc()  # transposed down projection
    buf = C.create_string_buffer(256)
    assert L.load().mr_moe_layer_validate(C.byref(c), buf, 256) == L.MR_ERR_INVALID_ARGUMENT
    assert "down stack must be [16, 1024, 512]" in buf.value.decode()


@pytest.mark.parametrize("make,needle", [
    (lambda: M.AffineWeights(torch.zeros(4, 16), torch.zeros(4, 2, dtype=torch.bfloat16),
                             torch.zeros(4, 2, dtype=torch.bfloat16), 64, 4), ".uint32"),
    (lambda: M.AffineWeights(torch.zeros(4, 16, dtype=torch.int32), torch.zeros(4, 2),
                             torch.zeros(4, 2, dtype=torch.bfloat16), 64, 4), "MLX emits both"),
    (lambda: M.AffineWeights(torch.zeros(4, 16, dtype=torch.int32),
                             torch.zeros(4, 3, dtype=torch.bfloat16),
                             torch.zeros(4, 3, dtype=torch.bfloat16), 64, 4),
     "need 2 scales per row, got 3"),
    (lambda: M.AffineWeights(torch.zeros(2, 4, 16, dtype=torch.int32),
                             torch.zeros(3, 4, 2, dtype=torch.bfloat16),
                             torch.zeros(3, 4, 2, dtype=torch.bfloat16), 64, 4),
     "expert count differs"),
    (lambda: M.AffineWeights(torch.zeros(4, 16, dtype=torch.int32),
                             torch.zeros(4, 2, dtype=torch.bfloat16),
                             torch.zeros(4, 2, dtype=torch.bfloat16), 64, 5), "must divide 32"),
])
def test_affine_weights_errors_mirror_reference(make, needle):
    with pytest.raises(M.AffineBridgeError, match=re.escape(needle)):
        make()


def test_expert_stack_and_expert_keep_or_drop_axis():
    w = _cpu_affine(4, 64, 128)
    assert w.expert_stack(2).experts == 1
    assert w.expert(2).experts is None
    with pytest.raises(M.AffineBridgeError, match="requested from a stack of 4"):
        w.expert(4)
    with pytest.raises(M.AffineBridgeError, match="stack of none"):
        w.expert(0).expert(0)


def test_gather_refuses_single_matrix_and_bad_rank():
    w = _cpu_affine(None, 64, 128)
    with pytest.raises(M.AffineBridgeError, match="needs a stacked AffineWeights"):
        M.affine_gather_mm(torch.zeros(2, 128, dtype=torch.bfloat16), w,
                           torch.zeros(2, 1, dtype=torch.int32))
    ws = _cpu_affine(4, 64, 128)
    with pytest.raises(M.AffineBridgeError, match="inserts the broadcast axes"):
        M.affine_gather_mm(torch.zeros(2, 1, 128, dtype=torch.bfloat16), ws,
                           torch.zeros(2, 1, dtype=torch.int32))
