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


# --------------------------------------------------------------------------- GGUF files
def quantize_q8_0(x: np.ndarray) -> bytes:
    """F32 values (a multiple of 32) -> Q8_0 blocks: scale d = max|x| / 127 stored as
    an IEEE half, quants round(x / d) (half away from zero) as int8 (ggml's block_q8_0)."""
    x = np.asarray(x, np.float32).reshape(-1, 32)
    d = np.abs(x).max(axis=1) / np.float32(127.0)
    inv = np.divide(1.0, d, out=np.zeros_like(d), where=d > 0)
    v = x * inv[:, None]
    q = np.clip(np.trunc(v + np.copysign(0.5, v)), -127, 127).astype(np.int8)
    out = np.empty((x.shape[0], 34), np.uint8)
    out[:, :2] = d.astype("<f2").view(np.uint8).reshape(-1, 2)
    out[:, 2:] = q.view(np.uint8)
    return out.tobytes()


class GgufWriter:
    """GGUF container bytes (the layout the reference's test builders write,
    e2e_native.rs:144-260): header, metadata, tensor infos, padding to the
    alignment, then each tensor's bytes at an aligned offset."""

    GGML = {"f32": 0, "f16": 1, "q8_0": 8}

    def __init__(self, version: int = 3, alignment: int | None = None):
        self.version = version
        self.alignment = alignment or 32
        self.kv = bytearray()
        self.n_kv = 0
        self.info = bytearray()
        self.n_tensors = 0
        self.data = bytearray()
        if alignment is not None:
            self.kv_u32("general.alignment", alignment)

    @staticmethod
    def _s(buf: bytearray, s) -> None:
        b = s.encode() if isinstance(s, str) else bytes(s)
        buf += np.uint64(len(b)).tobytes() + b

    def kv_raw(self, key, vtype: int, payload: bytes) -> None:
        self._s(self.kv, key)
        self.kv += np.uint32(vtype).tobytes() + payload
        self.n_kv += 1

    def kv_u8(self, k, v): self.kv_raw(k, 0, np.uint8(v).tobytes())
    def kv_i8(self, k, v): self.kv_raw(k, 1, np.int8(v).tobytes())
    def kv_u16(self, k, v): self.kv_raw(k, 2, np.uint16(v).tobytes())
    def kv_i16(self, k, v): self.kv_raw(k, 3, np.int16(v).tobytes())
    def kv_u32(self, k, v): self.kv_raw(k, 4, np.uint32(v).tobytes())
    def kv_i32(self, k, v): self.kv_raw(k, 5, np.int32(v).tobytes())
    def kv_f32(self, k, v): self.kv_raw(k, 6, np.float32(v).tobytes())
    def kv_bool(self, k, v): self.kv_raw(k, 7, np.uint8(1 if v else 0).tobytes())
    def kv_u64(self, k, v): self.kv_raw(k, 10, np.uint64(v).tobytes())
    def kv_i64(self, k, v): self.kv_raw(k, 11, np.int64(v).tobytes())
    def kv_f64(self, k, v): self.kv_raw(k, 12, np.float64(v).tobytes())

    def kv_str(self, k, v):
        b = bytearray()
        self._s(b, v)
        self.kv_raw(k, 8, bytes(b))

    def kv_arr(self, k, elem: int, values) -> None:
        """Array of element type `elem` (GGUF value type codes)."""
        b = bytearray(np.uint32(elem).tobytes() + np.uint64(len(values)).tobytes())
        fmt = {0: "<u1", 1: "<i1", 2: "<u2", 3: "<i2", 4: "<u4", 5: "<i4", 6: "<f4", 7: "<u1", 10: "<u8",
               11: "<i8", 12: "<f8"}
        if elem == 8:
            for s in values:
                self._s(b, s)
        else:
            b += np.asarray(values, fmt[elem]).tobytes()
        self.kv_raw(k, 9, bytes(b))

    def tensor(self, name, values, dtype: str = "f32", shape=None) -> None:
        """values (any shape) stored with `shape` (outer -> inner; default values.shape)."""
        a = np.asarray(values, np.float32)
        shape = list(a.shape if shape is None else shape)
        assert int(np.prod(shape, dtype=np.int64)) == a.size
        raw = {"f32": lambda: a.astype("<f4").tobytes(), "f16": lambda: a.astype("<f2").tobytes(),
               "q8_0": lambda: quantize_q8_0(a)}[dtype]()
        self.tensor_raw(name, raw, self.GGML[dtype], shape)

    def tensor_raw(self, name, raw: bytes, ggml_type: int, shape) -> None:
        pad = (self.alignment - len(self.data) % self.alignment) % self.alignment
        self.data += bytes(pad)
        self._s(self.info, name)
        self.info += np.uint32(len(shape)).tobytes()
        for d in reversed(shape):  # innermost first
            self.info += np.uint64(d).tobytes()
        self.info += np.uint32(ggml_type).tobytes() + np.uint64(len(self.data)).tobytes()
        self.data += raw
        self.n_tensors += 1

    def to_bytes(self) -> bytes:
        head = bytearray(b"GGUF" + np.uint32(self.version).tobytes() + np.uint64(self.n_tensors).tobytes() +
                         np.uint64(self.n_kv).tobytes())
        head += self.kv + self.info
        head += bytes((self.alignment - len(head) % self.alignment) % self.alignment)
        return bytes(head + self.data)


def model_metadata(w: GgufWriter, embed: int, depth: int, heads: int, mlp_hidden: int, num_register: int = 0,
                   patch: int = 14, rope_start: int = 4, qknorm_start: int = 4, alt_start: int = 4) -> None:
    """The depthanything3.* keys ModelConfig::from_gguf reads (config.rs:17-71)."""
    p = "depthanything3."
    w.kv_str(p + "arch", "depthanything3")
    w.kv_u32(p + "patch_size", patch)
    w.kv_u32(p + "image_size", 518)
    w.kv_u32(p + "vit.embed_dim", embed)
    w.kv_u32(p + "vit.depth", depth)
    w.kv_u32(p + "vit.num_heads", heads)
    w.kv_u32(p + "vit.head_dim", embed // heads)
    w.kv_u32(p + "vit.mlp_hidden", mlp_hidden)
    w.kv_u32(p + "vit.num_register_tokens", num_register)
    w.kv_i32(p + "vit.rope_start", rope_start)
    w.kv_i32(p + "vit.qknorm_start", qknorm_start)
    w.kv_f32(p + "vit.rope_freq", 100.0)
    w.kv_f32(p + "vit.ln_eps", 1e-6)
    w.kv_arr(p + "vit.out_layers", 5, [max(0, depth * (i + 1) // 4 - 1) for i in range(4)])
    w.kv_str(p + "vit.ffn_type", "mlp")
    w.kv_i32(p + "vit.alt_start", alt_start)
    w.kv_u32(p + "head.features", 128)
    w.kv_arr(p + "img.mean", 6, [0.485, 0.456, 0.406])
    w.kv_arr(p + "img.std", 6, [0.229, 0.224, 0.225])
    w.kv_str(p + "img.resize_mode", "bicubic")
    w.kv_u32(p + "cam.dim_in", 2 * embed)


def gguf_model(embed: int = 768, depth: int = 12, heads: int = 12, mlp_ratio: int = 4, num_register: int = 0,
               patch: int = 14, grid: int = 37, dtype: str = "q8_0", layout: str = "rank2", seed: int = 0,
               layers=None, patch_embed: bool = True, version: int = 3, alignment: int | None = None) -> bytes:
    """A DA3-style model file from the synthetic weights above: metadata, every
    block's norm1/attn_qkv/attn_q,knorm/attn_proj/ls1/norm2/mlp_fc1/mlp_fc2/ls2, the
    patch embedding, positions, CLS/register tokens and vit.norm.  Linear weights
    use `dtype`; vectors stay F32.  layout "rank2" stores linear weights as GGUF
    [out, in] (what converters write); "flat" stores the [in, out] values as one
    dimension (what the reference's e2e_native.rs builder writes)."""
    w = GgufWriter(version=version, alignment=alignment)
    hidden = mlp_ratio * embed
    model_metadata(w, embed, depth, heads, hidden, num_register, patch)

    def linear(name, m):  # m: [in, out]
        if layout == "rank2":
            w.tensor(name, np.ascontiguousarray(m.T), dtype)
        else:
            w.tensor(name, m.reshape(-1), dtype)

    if patch_embed:
        pe = patch_embed_weights(embed, patch, grid, num_register, seed)
        w.tensor("vit.patch_embed.weight", pe["weight"], dtype if dtype != "q8_0" or (3 * patch * patch * embed) % 32 == 0 else "f32")
        w.tensor("vit.patch_embed.bias", pe["bias"])
        w.tensor("vit.cls_token", pe["cls"], shape=[1, 1, embed])
        w.tensor("vit.pos_embed", pe["pos_embed"], shape=[1, grid * grid + 1, embed])
        if num_register:
            w.tensor("vit.register_tokens", pe["registers"], shape=[1, num_register, embed])
    r = rng(seed, 11)
    w.tensor("vit.norm.weight", (1.0 + 0.1 * r.standard_normal(embed)).astype(np.float32))
    w.tensor("vit.norm.bias", (0.1 * r.standard_normal(embed)).astype(np.float32))
    for i in (range(depth) if layers is None else layers):
        p = layer_weights(embed, seed=seed, layer=i, qknorm=True, ls1=True, bias=True, norm1=True,
                          perturb_norm=True, mlp=True, ls2=True, mlp_ratio=mlp_ratio)
        b = f"vit.blk.{i}."
        w.tensor(b + "norm1.weight", p["norm1_w"])
        w.tensor(b + "norm1.bias", p["norm1_b"])
        linear(b + "attn_qkv.weight", p["qkv_w"])
        w.tensor(b + "attn_qkv.bias", p["qkv_b"])
        w.tensor(b + "attn_qnorm.weight", p["q_g"])
        w.tensor(b + "attn_qnorm.bias", p["q_b"])
        w.tensor(b + "attn_knorm.weight", p["k_g"])
        w.tensor(b + "attn_knorm.bias", p["k_b"])
        linear(b + "attn_proj.weight", p["proj_w"])
        w.tensor(b + "attn_proj.bias", p["proj_b"])
        w.tensor(b + "ls1", p["ls1"])
        w.tensor(b + "norm2.weight", p["norm2_w"])
        w.tensor(b + "norm2.bias", p["norm2_b"])
        linear(b + "mlp_fc1.weight", p["fc1_w"])
        w.tensor(b + "mlp_fc1.bias", p["fc1_b"])
        linear(b + "mlp_fc2.weight", p["fc2_w"])
        w.tensor(b + "mlp_fc2.bias", p["fc2_b"])
        w.tensor(b + "ls2", p["ls2"])
    return w.to_bytes()
