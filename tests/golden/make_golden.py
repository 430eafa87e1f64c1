"""Regenerates the committed golden fixtures of tests/golden/ from the C oracle.

    python tests/golden/make_golden.py

Fixtures (all small):
  kat.json        SplitMix64 known answers and the MLX affine packing known
                  answer (hand-computed, independent of the oracle).
  config0_T4.npz  BASELINE config 0 (H 1024, 16+1 experts, top-2, I 512,
                  4-bit g64, T=4), seeded: x, router logits, ids, weights,
                  margins, layer output (bf16 bits and fp32).
  gather_b{2,4,8}.npz  affineGatherMM on a 4-expert [48, 128] stack with
                  repeated and unsorted ids, seeded.
The oracle restates MLX's affine gather_qmm semantics (mlx-swift 0.31.4 is not
available here), so these pin the oracle against itself across revisions and
pin the CUDA path against the oracle; they are not MLX outputs.
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import oracle as O  # noqa: E402


def kat() -> dict:
    return {
        # SplitMix64, seed 0: the published first outputs of the algorithm
        "splitmix64_seed0": ["0xe220a8397b1dcdaf", "0x6e789e6aa1b965f4", "0x06c45d188009454f"],
        # MLX affine 4-bit: word 0x76543210 holds codes 0..7, element j at bits 4j
        "pack4_word": "0x76543210",
        "pack4_codes": list(range(8)),
        # 2-bit: codes 0,1,2,3 repeated -> 0xE4E4E4E4; 8-bit: 1,2,3,4 -> 0x04030201
        "pack2_word": "0xe4e4e4e4",
        "pack2_codes": [0, 1, 2, 3] * 4,
        "pack8_word": "0x04030201",
        "pack8_codes": [1, 2, 3, 4],
    }


def gather_case(bits: int, seed: int = 0x6A7E0000):
    E, out, inn, T, k = 4, 48, 128, 5, 3
    parts = [O.gen_affine(seed + bits, 0, e, 0, out, inn, bits, 64) for e in range(E)]
    w = O._stack(parts)
    x = O.gen_normal_bf16(O.sm_derive(seed, 99), T * inn, 1.0).reshape(T, inn)
    ids = np.array([[3, 0, 3], [1, 1, 2], [3, 2, 0], [2, 3, 1], [0, 0, 0]], np.int32)
    y, yf = O.affine_gather_mm(x, w, ids)
    return dict(packed=w.packed, scales=w.scales, biases=w.biases, x=x, ids=ids, out=y,
                out_f32=yf, bits=np.int32(bits))


def main() -> None:
    with open(os.path.join(HERE, "kat.json"), "w") as f:
        json.dump(kat(), f, indent=1)
    cfg = O.CONFIGS[0]
    L = O.gen_layer(cfg)
    x = O.gen_x(cfg, 4)
    logits = O.router_logits(x, L.router_w)
    out, f, ids, w, m = O.moe_layer_forward(L, x)
    np.savez_compressed(os.path.join(HERE, "config0_T4.npz"), x=x, logits=logits, ids=ids,
                        weights=w, margins=m, out=out, out_f32=f)
    for b in (2, 4, 8):
        np.savez_compressed(os.path.join(HERE, f"gather_b{b}.npz"), **gather_case(b))
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
