"""Writes tests/golden/gguf_vectors.json: known answers for the GGUF model-file reader.

Every case rebuilds, byte for byte, a file or byte sequence that one of the
reference's own tests constructs, with the answer that test asserts (paths inside
the vestra-engine project):

  q8_0_block      crates/da-gguf/tests/q8_0_roundtrip.rs:5-27  (d = 0.5, qs = -16..15)
  bool_array_skip crates/da-gguf/src/reader.rs:387-479  (bool array skipped, sentinel u32)
  u16_array_skip  crates/da-gguf/src/reader.rs:481-540  (u16 array skipped, sentinel i32 -42)
  misaligned_q8_0 crates/da-gguf/src/reader.rs:543-620  (33-element Q8_0 tensor rejected)
  config_full     crates/da-engine/src/config.rs:362-415 full_valid_entries +
                  from_gguf_parses_all_fields (defaults alt_start -1, cat_token, head_pos_embed)
  config_alt4     config.rs alt_start_explicit_value_round_trips
  config_cat_off  config.rs cat_token_explicit_false_round_trips
  e2e_tiny        crates/da-engine/tests/e2e_native.rs:301-350 (the synthetic model's
                  metadata and a few of its rank-1 F32 tensors)

The two kv sequences of reader.rs's unit tests are wrapped in a version-2 header
with zero tensors so that a whole-file reader can take them.  The bytes are built
here with struct.pack, independently of the writer in synthetic.py, so these
fixtures pin both the oracle and that writer.

Run: python tests/golden/make_gguf_vectors.py   (CPU only; writes next to this file)
"""
from __future__ import annotations

import json
import os
import struct

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def s(x: str) -> bytes:
    b = x.encode()
    return struct.pack("<Q", len(b)) + b


def kv(key: str, vtype: int, payload: bytes) -> bytes:
    return s(key) + struct.pack("<I", vtype) + payload


def header(version: int, n_tensors: int, n_kv: int) -> bytes:
    return b"GGUF" + struct.pack("<IQQ", version, n_tensors, n_kv)


def pad32(b: bytes) -> bytes:
    return b + bytes((32 - len(b) % 32) % 32)


def q8_0_block():
    d = np.float16(0.5).tobytes()
    qs = bytes((i - 16) & 0xFF for i in range(32))
    block = d + qs
    return {"source": "crates/da-gguf/tests/q8_0_roundtrip.rs:5-27", "block_hex": block.hex(),
            "expect_f32": [0.5 * (i - 16) for i in range(32)]}


def bool_array_skip():
    body = kv("unmodeled_bool_array", 9, struct.pack("<IQ", 7, 3) + bytes([1, 0, 1]))
    body += kv("sentinel", 4, struct.pack("<I", 0x12345678))
    return {"source": "crates/da-gguf/src/reader.rs:387-479", "kv_hex": body.hex(),
            "file_hex": pad32(header(2, 0, 2) + body).hex(),
            "expect_kv": [["sentinel", "u32", 0x12345678]]}


def u16_array_skip():
    body = kv("unmodeled_u16_array", 9, struct.pack("<IQ", 2, 5) +
              struct.pack("<5H", 0x1111, 0x2222, 0x3333, 0x4444, 0x5555))
    body += kv("sentinel_i", 5, struct.pack("<i", -42))
    return {"source": "crates/da-gguf/src/reader.rs:481-540", "kv_hex": body.hex(),
            "file_hex": pad32(header(2, 0, 2) + body).hex(),
            "expect_kv": [["sentinel_i", "i32", -42]]}


def misaligned_q8_0():
    b = header(2, 1, 0) + s("misaligned") + struct.pack("<I", 1) + struct.pack("<Q", 33)
    b += struct.pack("<I", 8) + struct.pack("<Q", 0)
    b = pad32(b) + bytes(68)
    return {"source": "crates/da-gguf/src/reader.rs:543-620", "file_hex": b.hex(), "tensor": "misaligned",
            "expect_error": "malformed", "expect_message_contains": "not a multiple of block size"}


FULL = [
    ("str", "depthanything3.arch", "depthanything3"),
    ("u32", "depthanything3.patch_size", 14),
    ("u32", "depthanything3.image_size", 518),
    ("u32", "depthanything3.vit.embed_dim", 384),
    ("u32", "depthanything3.vit.depth", 12),
    ("u32", "depthanything3.vit.num_heads", 6),
    ("u32", "depthanything3.vit.head_dim", 64),
    ("u32", "depthanything3.vit.mlp_hidden", 1536),
    ("u32", "depthanything3.vit.num_register_tokens", 4),
    ("i32", "depthanything3.vit.rope_start", 0),
    ("i32", "depthanything3.vit.qknorm_start", 0),
    ("f32", "depthanything3.vit.rope_freq", 100.0),
    ("f32", "depthanything3.vit.ln_eps", 1e-6),
    ("arr_i32", "depthanything3.vit.out_layers", [2, 5, 8, 11]),
    ("u32", "depthanything3.head.features", 256),
    ("f32", "depthanything3.head.max_depth", 20.0),
    ("arr_f32", "depthanything3.img.mean", [0.485, 0.456, 0.406]),
    ("arr_f32", "depthanything3.img.std", [0.229, 0.224, 0.225]),
    ("str", "depthanything3.img.resize_mode", "bicubic"),
    ("u32", "depthanything3.cam.dim_in", 8),
]


def encode(kind, key, v) -> bytes:
    if kind == "str":
        return kv(key, 8, s(v))
    if kind == "u32":
        return kv(key, 4, struct.pack("<I", v))
    if kind == "i32":
        return kv(key, 5, struct.pack("<i", v))
    if kind == "f32":
        return kv(key, 6, struct.pack("<f", v))
    if kind == "bool":
        return kv(key, 7, bytes([1 if v else 0]))
    if kind == "arr_f32":
        return kv(key, 9, struct.pack("<IQ", 6, len(v)) + struct.pack(f"<{len(v)}f", *v))
    if kind == "arr_i32":
        return kv(key, 9, struct.pack("<IQ", 5, len(v)) + struct.pack(f"<{len(v)}i", *v))
    raise ValueError(kind)


def config_file(entries) -> bytes:
    body = b"".join(encode(*e) for e in entries)
    return pad32(header(2, 0, len(entries)) + body)


def f32(x):
    return float(np.float32(x))


FULL_EXPECT = {
    "arch": "depthanything3", "patch_size": 14, "image_size": 518, "embed_dim": 384, "depth": 12,
    "num_heads": 6, "head_dim": 64, "mlp_hidden": 1536, "num_register": 4, "rope_start": 0, "qknorm_start": 0,
    "rope_freq": 100.0, "ln_eps": f32(1e-6), "out_layers": [2, 5, 8, 11], "ffn_type": "mlp", "alt_start": -1,
    "cat_token": True, "head_features": 256, "head_max_depth": 20.0, "head_pos_embed": True,
    "img_mean": [f32(0.485), f32(0.456), f32(0.406)], "img_std": [f32(0.229), f32(0.224), f32(0.225)],
    "img_resize_mode": "bicubic", "cam_dim_in": 8,
}


def configs():
    out = {}
    out["config_full"] = {"source": "crates/da-engine/src/config.rs:362-415", "file_hex": config_file(FULL).hex(),
                          "expect": FULL_EXPECT}
    alt = FULL + [("i32", "depthanything3.vit.alt_start", 4)]
    out["config_alt4"] = {"source": "crates/da-engine/src/config.rs (alt_start_explicit_value_round_trips)",
                          "file_hex": config_file(alt).hex(), "expect": dict(FULL_EXPECT, alt_start=4)}
    cat = FULL + [("bool", "depthanything3.vit.cat_token", False)]
    out["config_cat_off"] = {"source": "crates/da-engine/src/config.rs (cat_token_explicit_false_round_trips)",
                             "file_hex": config_file(cat).hex(), "expect": dict(FULL_EXPECT, cat_token=False)}
    no_arch = [e for e in FULL if e[1] != "depthanything3.arch"]
    out["config_no_arch"] = {"source": "crates/da-engine/src/config.rs:219-223 (UnsupportedModel)",
                             "file_hex": config_file(no_arch).hex(), "expect_error": "unsupported",
                             "expect_message": "unsupported model architecture: expected 'depthanything3', found None"}
    no_heads = [e for e in FULL if e[1] != "depthanything3.vit.num_heads"]
    out["config_missing_heads"] = {"source": "crates/da-engine/src/config.rs:187-189 (MissingKey)",
                                   "file_hex": config_file(no_heads).hex(), "expect_error": "missing",
                                   "expect_message": "missing required gguf metadata key: depthanything3.vit.num_heads"}
    return out


def e2e_tiny():
    """The synthetic model's metadata (e2e_native.rs:316-341) and its first tensors
    (:343-350), with seeded values in place of its Xorshift32 stream."""
    meta = [
        ("str", "depthanything3.arch", "depthanything3"),
        ("u32", "depthanything3.patch_size", 2),
        ("u32", "depthanything3.image_size", 4),
        ("u32", "depthanything3.vit.embed_dim", 4),
        ("u32", "depthanything3.vit.depth", 4),
        ("u32", "depthanything3.vit.num_heads", 2),
        ("u32", "depthanything3.vit.head_dim", 2),
        ("u32", "depthanything3.vit.mlp_hidden", 8),
        ("u32", "depthanything3.vit.num_register_tokens", 0),
        ("i32", "depthanything3.vit.rope_start", -1),
        ("i32", "depthanything3.vit.qknorm_start", -1),
        ("f32", "depthanything3.vit.rope_freq", 100.0),
        ("f32", "depthanything3.vit.ln_eps", 1e-6),
        ("arr_i32", "depthanything3.vit.out_layers", [0, 1, 2, 3]),
        ("str", "depthanything3.vit.ffn_type", "mlp"),
        ("i32", "depthanything3.vit.alt_start", -1),
        ("u32", "depthanything3.head.features", 8),
        ("f32", "depthanything3.head.max_depth", 20.0),
        ("arr_f32", "depthanything3.img.mean", [0.0, 0.0, 0.0]),
        ("arr_f32", "depthanything3.img.std", [1.0, 1.0, 1.0]),
        ("str", "depthanything3.img.resize_mode", "bilinear"),
        ("u32", "depthanything3.cam.dim_in", 8),
    ]
    rng = np.random.default_rng(5)
    tensors = [("vit.patch_embed.weight", rng.standard_normal(4 * 3 * 2 * 2).astype(np.float32)),
               ("vit.patch_embed.bias", rng.standard_normal(4).astype(np.float32)),
               ("vit.pos_embed", rng.standard_normal(5 * 4).astype(np.float32)),
               ("vit.cls_token", rng.standard_normal(4).astype(np.float32))]
    info, data = b"", b""
    for name, v in tensors:  # rank 1, F32, offsets = running data length (e2e_native.rs:223-234)
        info += s(name) + struct.pack("<IQIQ", 1, v.size, 0, len(data))
        data += v.astype("<f4").tobytes()
    body = b"".join(encode(*e) for e in meta)
    b = pad32(header(3, len(tensors), len(meta)) + body + info) + data
    expect = {"arch": "depthanything3", "patch_size": 2, "image_size": 4, "embed_dim": 4, "depth": 4,
              "num_heads": 2, "head_dim": 2, "mlp_hidden": 8, "num_register": 0, "rope_start": -1,
              "qknorm_start": -1, "rope_freq": 100.0, "ln_eps": f32(1e-6), "out_layers": [0, 1, 2, 3],
              "ffn_type": "mlp", "alt_start": -1, "cat_token": True, "head_features": 8, "head_max_depth": 20.0,
              "head_pos_embed": True, "img_mean": [0.0, 0.0, 0.0], "img_std": [1.0, 1.0, 1.0],
              "img_resize_mode": "bilinear", "cam_dim_in": 8}
    return {"source": "crates/da-engine/tests/e2e_native.rs:301-350", "file_hex": b.hex(), "expect": expect,
            "tensors": {name: {"shape": [int(v.size)], "f32": [float(x) for x in v]} for name, v in tensors}}


def main():
    vec = {"q8_0_block": q8_0_block(), "bool_array_skip": bool_array_skip(), "u16_array_skip": u16_array_skip(),
           "misaligned_q8_0": misaligned_q8_0(), "e2e_tiny": e2e_tiny()}
    vec.update(configs())
    with open(os.path.join(HERE, "gguf_vectors.json"), "w") as f:
        json.dump(vec, f, indent=1)
        f.write("\n")


if __name__ == "__main__":
    main()
