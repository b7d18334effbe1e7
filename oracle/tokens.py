"""NumPy restatement of the reference's token input side: the conv patch
projection and the CLS / register / learned-position assembly.

TEST INFRASTRUCTURE ONLY: imported by tests/ and bench.py's CPU leg as the
checker.  The product path (vestra-engine_b200/) never imports this module.

Each function names the reference code it restates (paths inside the
vestra-engine project).  The conv itself is `vestra_kernels::conv::conv2d` from the
vestra-kernels crate (git rev 783bd66c, not vendored in the reference tree); what
its call site fixes (kernel = stride = patch, no padding, OIHW filter, NCHW image,
output [embed][gh*gw] transposed to token-major) is restated here as one matrix
product accumulated in float64.  The position interpolation is restated in F32
with the reference's operation order, so a device table computed with separately
rounded F32 operations in the same order is bit-identical to it.
"""
from __future__ import annotations

import numpy as np

CHANNELS = 3
DEFAULT_INTERP_OFFSET = np.float32(0.1)  # pos_embed.rs:41-55


def patch_embed(img_nchw, weight, bias, patch):
    """patch_embed.rs:53-133.  img [3, H, W] (batch 1), weight [E, 3, p, p] (OIHW),
    bias [E] -> (gh, gw, tokens [gh*gw, E]), tokens row-major over the patch grid."""
    img = np.asarray(img_nchw, np.float32)
    if img.ndim != 3 or img.shape[0] != CHANNELS:
        raise ValueError("img_nchw must be [3, h, w]")
    _, h, w = img.shape
    if h % patch:
        raise ValueError(f"h ({h}) must be a multiple of patch_size ({patch})")
    if w % patch:
        raise ValueError(f"w ({w}) must be a multiple of patch_size ({patch})")
    weight = np.asarray(weight, np.float32)
    embed = weight.shape[0]
    if weight.size != embed * CHANNELS * patch * patch:
        raise ValueError("patch filter shape mismatch: expected embed_dim*3*patch*patch")
    gh, gw = h // patch, w // patch
    # rows[p] = the patch's pixels in (c, ky, kx) order, the OIHW filter's flattening
    rows = img.reshape(CHANNELS, gh, patch, gw, patch).transpose(1, 3, 0, 2, 4).reshape(gh * gw, -1)
    out = rows.astype(np.float64) @ weight.reshape(embed, -1).astype(np.float64).T
    out += np.asarray(bias, np.float64)[None, :]
    return gh, gw, out.astype(np.float32)


def cubic(x):
    """Keys' cubic convolution kernel, a = -0.75 (pos_embed.rs:73-83), F32."""
    a = np.float32(-0.75)
    x = np.float32(abs(np.float32(x)))
    if x < 1:
        return ((a + np.float32(2)) * x - (a + np.float32(3))) * x * x + np.float32(1)
    if x < 2:
        return (((x - np.float32(5)) * x + np.float32(8)) * x - np.float32(4)) * a
    return np.float32(0)


def infer_grid(length, embed):
    """pos_embed.rs:89-106: side M of the square grid in a [(M*M + 1), E] table."""
    if length % embed:
        raise ValueError("pos_embed length not a multiple of embed_dim")
    rows = length // embed
    if rows < 1:
        raise ValueError("pos_embed must have at least the CLS row")
    patch_rows = rows - 1
    m = int(round(patch_rows ** 0.5))
    if m * m != patch_rows:
        raise ValueError(f"pos_embed patch-row count {patch_rows} is not a perfect square")
    return m


def interpolate_pos_embed(pos_embed, grid, embed, gh, gw, interp_offset=DEFAULT_INTERP_OFFSET):
    """pos_embed.rs:122-172: bicubic resampling of the learned grid to (gh, gw) with
    half-pixel centres and clamp-to-edge taps; CLS row copied.  Every operation in
    F32, in the reference's order.  Returns [(1 + gh*gw), E]."""
    src = np.asarray(pos_embed, np.float32).reshape(grid * grid + 1, embed)
    out = np.zeros((1 + gh * gw, embed), np.float32)
    out[0] = src[0]
    m = np.float32(grid)
    off = np.float32(interp_offset)
    sx = (np.float32(gw) + off) / m
    sy = (np.float32(gh) + off) / m
    for oy in range(gh):
        iy = (np.float32(oy) + np.float32(0.5)) / sy - np.float32(0.5)
        y0 = int(np.floor(iy))
        fy = iy - np.float32(y0)
        for ox in range(gw):
            ix = (np.float32(ox) + np.float32(0.5)) / sx - np.float32(0.5)
            x0 = int(np.floor(ix))
            fx = ix - np.float32(x0)
            acc = np.zeros(embed, np.float32)
            for dy in range(-1, 3):
                wy = cubic(fy - np.float32(dy))
                yy = min(max(y0 + dy, 0), grid - 1)
                for dx in range(-1, 3):
                    wx = cubic(fx - np.float32(dx))
                    xx = min(max(x0 + dx, 0), grid - 1)
                    acc = acc + (wy * wx) * src[1 + yy * grid + xx]
            out[1 + oy * gw + ox] = acc
    return out


def assemble_tokens(patch_tokens, gh, gw, cls_token, pos_table, register_tokens=None):
    """assemble_tokens_from_patch_tokens (pos_embed.rs:254-300): [CLS, registers,
    patches]; positions added to the CLS row and the patch rows only."""
    patch_tokens = np.asarray(patch_tokens, np.float32)
    embed = patch_tokens.shape[1]
    regs = np.zeros((0, embed), np.float32) if register_tokens is None else \
        np.asarray(register_tokens, np.float32).reshape(-1, embed)
    out = np.concatenate([np.asarray(cls_token, np.float32).reshape(1, embed), regs, patch_tokens], 0)
    pos = np.asarray(pos_table, np.float32)
    out[0] = out[0] + pos[0]
    out[1 + regs.shape[0]:] = out[1 + regs.shape[0]:] + pos[1:]
    return out


def prepare_tokens(img_nchw, weight, bias, cls_token, pos_embed, patch, register_tokens=None,
                   interp_offset=DEFAULT_INTERP_OFFSET, pos_table=None):
    """prepare_tokens (pos_embed.rs:236-252) for one image: returns (gh, gw, tokens)."""
    gh, gw, patch_tokens = patch_embed(img_nchw, weight, bias, patch)
    embed = patch_tokens.shape[1]
    if pos_table is None:
        pe = np.asarray(pos_embed, np.float32)
        grid = infer_grid(pe.size, embed)
        pos_table = interpolate_pos_embed(pe, grid, embed, gh, gw, interp_offset)
    return gh, gw, assemble_tokens(patch_tokens, gh, gw, cls_token, pos_table, register_tokens)
