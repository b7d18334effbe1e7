"""CPU checks of the token input side's oracle (oracle/tokens.py) against the
reference's own unit-test vectors and an independent bicubic restatement."""
import json
import os

import numpy as np
import pytest

import tokens as tk

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "token_vectors.json")


@pytest.fixture(scope="module")
def vec():
    with open(GOLDEN) as f:
        return json.load(f)


def test_zero_filter_gives_bias_on_every_patch(vec):
    # patch_embed.rs:281-301
    v = vec["bias_broadcast"]
    p, e = v["patch"], v["embed"]
    img = np.full((3, v["h"], v["w"]), v["image_value"], np.float32)
    gh, gw, t = tk.patch_embed(img, np.zeros((e, 3, p, p), np.float32), np.array(v["bias"], np.float32), p)
    assert (gh, gw) == (v["gh"], v["gw"])
    assert t.shape == (gh * gw, e)
    for row in t:
        assert row.tolist() == v["bias"]


def test_patch_order_is_row_major_over_the_grid(vec):
    # patch_embed.rs:304-340: channel-0 taps = 1, pixel value = row-major index
    v = vec["row_major_order"]
    p, h, w = v["patch"], v["h"], v["w"]
    img = np.zeros((3, h, w), np.float32)
    img[0] = np.arange(h * w, dtype=np.float32).reshape(h, w)
    wt = np.zeros((1, 3, p, p), np.float32)
    wt[0, 0] = 1.0
    _, _, t = tk.patch_embed(img, wt, np.zeros(1, np.float32), p)
    assert t.ravel().tolist() == v["tokens"]


def test_misaligned_image_is_rejected(vec):
    # patch_embed.rs:343-350
    v = vec["misaligned"]
    with pytest.raises(ValueError, match=v["message"]):
        tk.patch_embed(np.zeros((3, v["h"], v["w"]), np.float32), np.zeros((1, 3, 2, 2), np.float32),
                       np.zeros(1, np.float32), v["patch"])


def test_infer_grid(vec):
    # pos_embed.rs:358-370
    v = vec["infer_grid"]
    for length, embed, m in v["cases"]:
        assert tk.infer_grid(length, embed) == m
    with pytest.raises(ValueError, match=v["message"]):
        tk.infer_grid(*v["rejected"])


def _grid3(embed=2):
    # pos_embed.rs:346-356: row r of the 3x3 table is [r, -r]
    pos = np.zeros((10, embed), np.float32)
    pos[:, 0] = np.arange(10, dtype=np.float32)
    pos[:, 1] = -np.arange(10, dtype=np.float32)  # -0.0 in row 0, as in the reference
    return pos


def test_cls_rows(vec):
    # pos_embed.rs:407-443
    v = vec["cls_row"]
    pos = _grid3(v["embed"])
    table = tk.interpolate_pos_embed(pos, v["grid"], v["embed"], 3, 3)
    assert table[0].tolist() == v["native_cls"]
    assert np.signbit(table[0, 1])
    _, _, tok = tk.prepare_tokens(np.zeros((3, 4, 4), np.float32), np.zeros((2, 3, 2, 2), np.float32),
                                  np.zeros(2, np.float32), np.array(v["cls"], np.float32), pos, 2)
    assert tok.shape == (5, 2)
    assert tok[0].tolist() == v["tokens_cls"]


def test_interpolation_matches_torch_bicubic(vec):
    v = vec["bicubic"]
    rng = np.random.default_rng(v["seed"])
    pe = rng.standard_normal((v["grid"] * v["grid"] + 1, v["embed"])).astype(np.float32)
    for case in v["cases"]:
        ours = tk.interpolate_pos_embed(pe, v["grid"], v["embed"], case["gh"], case["gw"], np.float32(v["offset"]))
        ref = np.array(case["table"], np.float64)
        assert ours.shape == (1 + case["gh"] * case["gw"], v["embed"])
        assert np.array_equal(ours[0], pe[0])
        # F32 positions and taps against float64: a few ulp of the table's scale
        assert np.abs(ours[1:] - ref).max() < 2e-5, case


def test_patch_projection_matches_direct_convolution():
    rng = np.random.default_rng(3)
    p, e, h, w = 3, 5, 6, 9
    img = rng.standard_normal((3, h, w)).astype(np.float32)
    wt = rng.standard_normal((e, 3, p, p)).astype(np.float32)
    b = rng.standard_normal(e).astype(np.float32)
    gh, gw, t = tk.patch_embed(img, wt, b, p)
    ref = np.zeros((gh * gw, e))
    for py in range(gh):
        for px in range(gw):
            win = img[:, py * p:(py + 1) * p, px * p:(px + 1) * p].astype(np.float64)
            for o in range(e):
                ref[py * gw + px, o] = (win * wt[o]).sum() + b[o]
    assert np.abs(t - ref).max() < 1e-5


def test_registers_follow_cls_without_positions():
    # pos_embed.rs:277-299: [CLS, registers, patches]; registers get no position
    e = 4
    patches = np.ones((6, e), np.float32)
    pos = np.arange(7 * e, dtype=np.float32).reshape(7, e)
    regs = np.full((2, e), 5.0, np.float32)
    out = tk.assemble_tokens(patches, 2, 3, np.zeros(e, np.float32), pos, regs)
    assert out.shape == (9, e)
    assert np.array_equal(out[0], pos[0])
    assert np.array_equal(out[1:3], regs)
    assert np.array_equal(out[3:], 1.0 + pos[1:])
