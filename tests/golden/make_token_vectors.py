"""Writes tests/golden/token_vectors.json: known answers for the token input side.

1. Literal vectors of the reference's own unit tests for the patch projection and
   the position assembly (crates/da-engine/src/patch_embed.rs:281-350,
   crates/da-engine/src/pos_embed.rs:358-443), each with its source lines.
2. An independent pin of the bicubic position interpolation: PyTorch's
   F.interpolate(mode="bicubic", align_corners=False, scale_factor=((gh+0.1)/M,
   (gw+0.1)/M)) in float64 (the upstream DINOv2 formulation the reference's
   interpolate_pos_embed restates, pos_embed.rs:122-172) on a small seeded grid.
   Inputs are regenerated from the recorded seed with numpy PCG64.

Run: python tests/golden/make_token_vectors.py   (CPU only; writes next to this file)
"""
from __future__ import annotations

import json
import os

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
BICUBIC_SEED, BICUBIC_GRID, BICUBIC_EMBED = 7, 5, 3
BICUBIC_SIZES = [(3, 2), (5, 5), (7, 4), (1, 1)]


def bicubic_inputs():
    rng = np.random.default_rng(BICUBIC_SEED)
    return rng.standard_normal((BICUBIC_GRID * BICUBIC_GRID + 1, BICUBIC_EMBED)).astype(np.float32)


def main():
    pe = bicubic_inputs()
    m, e = BICUBIC_GRID, BICUBIC_EMBED
    grid = torch.from_numpy(pe[1:].astype(np.float64)).reshape(1, m, m, e).permute(0, 3, 1, 2)
    bicubic = []
    for gh, gw in BICUBIC_SIZES:
        t = torch.nn.functional.interpolate(grid, scale_factor=((gh + 0.1) / m, (gw + 0.1) / m), mode="bicubic",
                                            align_corners=False)
        bicubic.append({"gh": gh, "gw": gw, "table": t.permute(0, 2, 3, 1).reshape(-1, e).tolist()})
    vectors = {
        "bias_broadcast": {"patch": 2, "embed": 3, "h": 4, "w": 4, "image_value": 1.0, "bias": [1.0, 2.0, 3.0],
                           "gh": 2, "gw": 2, "source": "crates/da-engine/src/patch_embed.rs:281-301"},
        "row_major_order": {"patch": 2, "embed": 1, "h": 4, "w": 4, "tokens": [10.0, 18.0, 42.0, 50.0],
                            "source": "crates/da-engine/src/patch_embed.rs:304-340"},
        "misaligned": {"patch": 2, "h": 3, "w": 4, "message": "must be a multiple of patch_size",
                       "source": "crates/da-engine/src/patch_embed.rs:343-350"},
        "infer_grid": {"cases": [[20, 2, 3], [257 * 384, 384, 16]], "rejected": [38, 2],
                       "message": "not a perfect square", "source": "crates/da-engine/src/pos_embed.rs:358-370"},
        "cls_row": {"grid": 3, "embed": 2, "cls": [100.0, -100.0], "tokens_cls": [100.0, -100.0],
                    "native_cls": [0.0, -0.0], "source": "crates/da-engine/src/pos_embed.rs:407-443"},
        "bicubic": {"seed": BICUBIC_SEED, "grid": m, "embed": e, "offset": 0.1, "cases": bicubic,
                    "source": "torch.nn.functional.interpolate bicubic, float64"},
    }
    with open(os.path.join(HERE, "token_vectors.json"), "w") as f:
        json.dump(vectors, f, indent=1)
    print("wrote token_vectors.json")


if __name__ == "__main__":
    main()
