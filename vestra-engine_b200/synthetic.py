"""Seeded synthetic inputs of the benchmark shapes (no dataset or checkpoint exists here).

Hidden states ~ N(0,1) F32, QKV/proj weights ~ N(0, 0.02), QK-norm gamma 1 / beta 0,
biases 0 unless asked, ls1 absent unless asked; camera slots ~ N(0,1).  Weights use
the reference's [in, out] orientation (engine.rs:110-126).  Generator: numpy PCG64,
one independent stream per (seed, purpose) so that inputs and weights do not
depend on the order they are drawn in.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass(frozen=True)
class Workload:
    name: str
    embed: int
    heads: int
    views: int
    gh: int
    gw: int
    n_special: int
    global_: bool

    @property
    def tokens_per_view(self) -> int:
        return self.n_special + self.gh * self.gw

    @property
    def rows(self) -> int:
        return self.views * self.tokens_per_view

    @property
    def seg_len(self) -> int:
        return self.rows if self.global_ else self.tokens_per_view

    def attention_flops(self) -> float:
        """4 * N^2 * d * heads summed over the attention segments (the metric's FLOP count)."""
        segs = self.rows // self.seg_len
        return 4.0 * segs * self.seg_len ** 2 * 64 * self.heads


# Benchmark configs (504x336 -> 36x24 patches; 1008x672 -> 72x48), n_special = 2.
CONFIGS = {
    "cfg1_single_view": Workload("cfg1_single_view", 768, 12, 1, 36, 24, 2, False),
    "cfg2_s2_global": Workload("cfg2_s2_global", 768, 12, 2, 36, 24, 2, True),
    "cfg3_s12_global": Workload("cfg3_s12_global", 768, 12, 12, 36, 24, 2, True),
    "cfg4_s12_local": Workload("cfg4_s12_local", 768, 12, 12, 36, 24, 2, False),
    "cfg5_large_s32_global": Workload("cfg5_large_s32_global", 1024, 16, 32, 72, 48, 2, True),
}


def rng(seed: int, purpose: int) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64([seed, purpose]))


def hidden_states(rows: int, embed: int, seed: int = 0) -> np.ndarray:
    return rng(seed, 1).standard_normal((rows, embed), dtype=np.float32)


def layer_weights(embed: int, seed: int = 0, layer: int = 0, qknorm: bool = True, ls1: bool = False,
                  bias: bool = False, norm1: bool = False, perturb_norm: bool = False, mlp: bool = False,
                  ls2: bool = False, mlp_ratio: int = 4) -> dict:
    """One block's weights, [in, out] orientation: attention (always), LN1 (norm1),
    and the MLP sub-block (mlp: norm2, fc1 [E, ratio*E], fc2 [ratio*E, E], ls2)."""
    r = rng(seed, 1000 + layer)
    p = {
        "qkv_w": (0.02 * r.standard_normal((embed, 3 * embed))).astype(np.float32),
        "qkv_b": ((0.02 * r.standard_normal(3 * embed)) if bias else np.zeros(3 * embed)).astype(np.float32),
        "proj_w": (0.02 * r.standard_normal((embed, embed))).astype(np.float32),
        "proj_b": ((0.02 * r.standard_normal(embed)) if bias else np.zeros(embed)).astype(np.float32),
    }
    if qknorm:
        if perturb_norm:
            p["q_g"] = (1.0 + 0.1 * r.standard_normal(64)).astype(np.float32)
            p["q_b"] = (0.1 * r.standard_normal(64)).astype(np.float32)
            p["k_g"] = (1.0 + 0.1 * r.standard_normal(64)).astype(np.float32)
            p["k_b"] = (0.1 * r.standard_normal(64)).astype(np.float32)
        else:
            p["q_g"] = np.ones(64, np.float32)
            p["q_b"] = np.zeros(64, np.float32)
            p["k_g"] = np.ones(64, np.float32)
            p["k_b"] = np.zeros(64, np.float32)
    if ls1:
        p["ls1"] = (0.1 + 0.05 * r.standard_normal(embed)).astype(np.float32)
    if norm1:
        p["norm1_w"] = (1.0 + 0.1 * r.standard_normal(embed)).astype(np.float32)
        p["norm1_b"] = (0.1 * r.standard_normal(embed)).astype(np.float32)
    if mlp:
        m = rng(seed, 2000 + layer)
        hidden = mlp_ratio * embed
        p["norm2_w"] = (1.0 + 0.1 * m.standard_normal(embed)).astype(np.float32)
        p["norm2_b"] = (0.1 * m.standard_normal(embed)).astype(np.float32)
        p["fc1_w"] = (0.02 * m.standard_normal((embed, hidden))).astype(np.float32)
        p["fc1_b"] = (0.02 * m.standard_normal(hidden)).astype(np.float32)
        p["fc2_w"] = (0.02 * m.standard_normal((hidden, embed))).astype(np.float32)
        p["fc2_b"] = (0.02 * m.standard_normal(embed)).astype(np.float32)
        if ls2:
            p["ls2"] = (0.1 + 0.05 * m.standard_normal(embed)).astype(np.float32)
    return p


def camera_tokens(embed: int, seed: int = 0) -> np.ndarray:
    return rng(seed, 7).standard_normal(2 * embed, dtype=np.float32)


def images(views: int, height: int, width: int, seed: int = 0) -> np.ndarray:
    """Normalised NCHW images [views, 3, H, W] (preprocessed pixels are roughly N(0, 1))."""
    return rng(seed, 8).standard_normal((views, 3, height, width), dtype=np.float32)


def patch_embed_weights(embed: int, patch: int = 14, grid: int = 37, num_register: int = 0,
                        seed: int = 0) -> dict:
    """Patch filter [E, 3, p, p] (OIHW), bias [E], CLS [E], learned positions
    [grid*grid + 1, E] and register tokens [num_register, E] (DA3: patch 14, 37x37)."""
    r = rng(seed, 9)
    p = {
        "weight": (0.02 * r.standard_normal((embed, 3, patch, patch))).astype(np.float32),
        "bias": (0.02 * r.standard_normal(embed)).astype(np.float32),
        "cls": (0.02 * r.standard_normal(embed)).astype(np.float32),
        "pos_embed": (0.02 * r.standard_normal((grid * grid + 1, embed))).astype(np.float32),
        "registers": None,
    }
    if num_register:
        p["registers"] = (0.02 * r.standard_normal((num_register, embed))).astype(np.float32)
    return p
