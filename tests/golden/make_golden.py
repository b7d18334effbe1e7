"""Generates the committed golden fixtures under tests/golden/.

1. attention_block_small.npz — outputs of an independent float64 restatement (torch
   ops: F.layer_norm, matmul, softmax) of the reference attention sub-block
   (crates/da-engine/src/vit_block.rs:772-992) and of Op::Attention
   (crates/da-graph/src/cpu_backend.rs:198-298) on small seeded cases.  Inputs are
   NOT stored: they are regenerated from the recorded seeds with numpy PCG64
   (vestra-engine_b200/synthetic.py), which is deterministic across platforms.
2. reference_vectors.json — the known-answer vectors of the reference's own unit
   tests for this path (literal values from the cited test functions).

Run: python tests/golden/make_golden.py   (CPU only; writes next to this file)
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "vestra-engine_b200"))
import synthetic as syn  # noqa: E402

torch.set_default_dtype(torch.float64)


def rope_f64(x, pos_yx, base=100.0):
    """x [heads, n, d]; the first d/2 channels rotate with y, the rest with x.
    Per half of width h: angles pos * base^(-(0,2,..,h-2)/h) concatenated twice and
    rotate-half (x1, x2) -> (-x2, x1)."""
    d = x.shape[-1]
    half = d // 2
    inv = 1.0 / (base ** (torch.arange(0, half, 2, dtype=torch.float64) / half))
    out = []
    for axis in range(2):
        seg = x[..., axis * half:(axis + 1) * half]
        ang = pos_yx[:, axis:axis + 1].to(torch.float64) * inv[None, :]
        ang = torch.cat([ang, ang], dim=-1)
        x1, x2 = seg[..., : half // 2], seg[..., half // 2:]
        rot = torch.cat([-x2, x1], dim=-1)
        out.append(seg * torch.cos(ang) + rot * torch.sin(ang))
    return torch.cat(out, dim=-1)


def attention_f64(q, k, v, seg_len):
    heads, n, d = q.shape
    out = torch.empty_like(q)
    for s0 in range(0, n, seg_len):
        sl = slice(s0, s0 + seg_len)
        w = torch.softmax(q[:, sl] @ k[:, sl].transpose(1, 2) / d ** 0.5, dim=-1)
        out[:, sl] = w @ v[:, sl]
    return out


def block_f64(x, p, heads, pos, seg_len, use_qknorm, eps=1e-5):
    x = torch.from_numpy(x).double()
    e = x.shape[1]
    d = e // heads
    qkv = x @ torch.from_numpy(p["qkv_w"]).double() + torch.from_numpy(p["qkv_b"]).double()
    q, k, v = (qkv[:, i * e:(i + 1) * e].reshape(-1, heads, d).transpose(0, 1) for i in range(3))
    if use_qknorm:
        q = torch.nn.functional.layer_norm(q, (d,), torch.from_numpy(p["q_g"]).double(),
                                           torch.from_numpy(p["q_b"]).double(), eps)
        k = torch.nn.functional.layer_norm(k, (d,), torch.from_numpy(p["k_g"]).double(),
                                           torch.from_numpy(p["k_b"]).double(), eps)
    if pos is not None:
        pt = torch.from_numpy(pos).round().long()
        q, k = rope_f64(q, pt), rope_f64(k, pt)
    o = attention_f64(q, k, v, seg_len).transpose(0, 1).reshape(-1, e)
    y = o @ torch.from_numpy(p["proj_w"]).double() + torch.from_numpy(p["proj_b"]).double()
    if "ls1" in p:
        y = y * torch.from_numpy(p["ls1"]).double()
    return y.numpy()


def positions(rows, views, n_special, gh, gw, glob):
    per = n_special + gh * gw
    p = np.zeros((views, per, 2), np.float32)
    if glob:
        p[:, n_special:] = 1
    else:
        i = np.arange(gh * gw)
        p[:, n_special:, 0] = i // gw + 1
        p[:, n_special:, 1] = i % gw + 1
    return p.reshape(rows, 2)


# (name, embed, views, gh, gw, n_special, global, use_qknorm, use_rope, ls1, seed)
BLOCK_CASES = [
    ("local_s1", 128, 1, 3, 4, 2, False, True, True, False, 11),
    ("local_s3", 128, 3, 2, 3, 1, False, True, True, True, 12),
    ("global_s2", 128, 2, 3, 4, 2, True, True, True, True, 13),
    ("global_s3_plain", 128, 3, 2, 2, 1, True, False, False, False, 14),
]
# (name, heads, n, d, qknorm, rope, seed)
OP_CASES = [
    ("op_plain_d4", 2, 3, 4, False, False, 21),
    ("op_norm_rope_d4", 2, 5, 4, True, True, 22),
    ("op_norm_rope_d64", 3, 37, 64, True, True, 23),
]


def op_inputs(heads, n, d, seed):
    r = syn.rng(seed, 5)
    q, k, v = (r.standard_normal((heads, n, d)).astype(np.float32) for _ in range(3))
    g = (1 + 0.1 * r.standard_normal(d)).astype(np.float32)
    b = (0.1 * r.standard_normal(d)).astype(np.float32)
    pos = np.stack([r.integers(0, 9, n), r.integers(0, 9, n)], 1).astype(np.float32)
    return q, k, v, g, b, pos


def main():
    out = {}
    for name, e, views, gh, gw, ns, glob, qk, rp, ls1, seed in BLOCK_CASES:
        rows = views * (ns + gh * gw)
        x = syn.hidden_states(rows, e, seed=seed)
        p = syn.layer_weights(e, seed=seed, layer=0, qknorm=qk, ls1=ls1, bias=True, perturb_norm=True)
        pos = positions(rows, views, ns, gh, gw, glob) if rp else None
        seg = rows if glob else rows // views
        out[name] = block_f64(x, p, e // 64, pos, seg, qk).astype(np.float32)
    for name, heads, n, d, qk, rp, seed in OP_CASES:
        q, k, v, g, b, pos = op_inputs(heads, n, d, seed)
        qt, kt, vt = (torch.from_numpy(a).double() for a in (q, k, v))
        if qk:
            qt = torch.nn.functional.layer_norm(qt, (d,), torch.from_numpy(g).double(), torch.from_numpy(b).double(), 1e-5)
            kt = torch.nn.functional.layer_norm(kt, (d,), torch.from_numpy(g[::-1].copy()).double(),
                                                torch.from_numpy(b[::-1].copy()).double(), 1e-5)
        if rp:
            pt = torch.from_numpy(pos).long()
            qt, kt = rope_f64(qt, pt), rope_f64(kt, pt)
        out[name] = attention_f64(qt, kt, vt, n).numpy().astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "attention_block_small.npz"), **out)

    vectors = {
        "qk_norm_eps": {"value": 1e-5, "source": "crates/da-engine/src/backbone.rs:1340-1342"},
        "saddle": {"cls": [[1.0, 0.0, 0.0, 0.0], [0.7, 0.6, 0.1, 0.0], [0.0, 1.0, 0.0, 0.0], [-1.0, 0.0, 0.0, 0.0]],
                   "reference": 0, "source": "crates/da-engine/src/backbone.rs:1446-1455"},
        "reference_first_order": [{"views": 5, "reference": 3, "order": [3, 0, 1, 2, 4]},
                                  {"views": 3, "reference": 0, "order": [0, 1, 2]}],
        "reference_first_order_source": "crates/da-engine/src/backbone.rs:1457-1460",
        "restore": {"ordered": ["reference", "first", "second", "third"], "reference": 3,
                    "restored": ["first", "second", "third", "reference"],
                    "source": "crates/da-engine/src/engine.rs:743-749"},
        "plain_attention_tolerance": {"value": 1e-6,
                                      "source": "crates/da-graph/tests/attention_and_layerscale_op.rs:39-74"},
        "eps_discriminator": {"correct_max_diff": 1e-6, "wrong_min_diff": 1e-8, "base": 100.0, "spread": 1e-3,
                              "source": "crates/da-graph/tests/attention_and_layerscale_op.rs:92-196"},
        "rope_changes_output": {"min_diff": 1e-4, "pos_yx": [0.0, 0.0, 1.0, 2.0], "freq": 100.0,
                                "source": "crates/da-graph/tests/attention_and_layerscale_op.rs:203-260"},
    }
    with open(os.path.join(HERE, "reference_vectors.json"), "w") as f:
        json.dump(vectors, f, indent=1)
    print("wrote", sorted(out))


if __name__ == "__main__":
    main()
