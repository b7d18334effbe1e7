"""GPU parity of the token input side (va_prepare_tokens_*, va_pos_embed_device)
against the NumPy restatement in oracle/tokens.py: patch_embed (patch_embed.rs:53-133),
interpolate_pos_embed (pos_embed.rs:122-172) and the token assembly
(pos_embed.rs:236-300), for DA3-BASE widths (E = 768, patch 14, 37 x 37 positions).

The position table is built with separately rounded F32 operations in the
reference's order, so it is compared bit for bit; the special rows are exact F32
adds and copies, also bit for bit; the patch rows go through the bf16 tcgen05
projection and are held to the path's parity gates (max-abs <= 2e-2, cosine >=
0.9999).
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")]

import synthetic as syn  # noqa: E402
import tokens as tk  # noqa: E402
import vestra_attn as va  # noqa: E402

E, PATCH, GRID = 768, 14, 37


def _close(got, ref, what):
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    err = float(np.abs(got - ref).max())
    cos = float(got.ravel() @ ref.ravel() / (np.linalg.norm(got) * np.linalg.norm(ref)))
    assert err <= 2e-2 and cos >= 0.9999, f"{what}: max-abs {err:.3e} cos {cos:.7f}"


def _ctx(num_register, max_rows=12 * 866):
    return va.Context(va.default_config(max_rows=max_rows, num_register=num_register), 0)


def _load(c, w):
    c.load_patch_embed(w["weight"], w["bias"], w["cls"], w["pos_embed"], w["registers"], PATCH)


def _oracle_tokens(img, w, pos_table):
    out = []
    for v in range(img.shape[0]):
        _, _, t = tk.prepare_tokens(img[v], w["weight"], w["bias"], w["cls"], w["pos_embed"], PATCH,
                                    w["registers"], pos_table=pos_table)
        out.append(t)
    return np.stack(out)


@pytest.mark.parametrize("gh,gw", [(36, 24), (3, 2), (37, 37), (72, 48)])
def test_position_table_is_bit_identical(gh, gw):
    w = syn.patch_embed_weights(E, PATCH, GRID, 0, seed=1)
    c = _ctx(0, max_rows=16 * 1024)
    try:
        _load(c, w)
        out = torch.empty(1 + gh * gw, E, device="cuda")
        c.pos_embed_device(gh, gw, out)
        again = torch.empty_like(out)
        c.pos_embed_device(gh, gw, again)  # cached table
        torch.cuda.synchronize()
        c.check_device()
        ref = tk.interpolate_pos_embed(w["pos_embed"], GRID, E, gh, gw)
        got = out.cpu().numpy()
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), \
            f"{gh}x{gw}: {np.count_nonzero(got != ref)} differing values, max {np.abs(got - ref).max():.3e}"
        assert torch.equal(out, again)
    finally:
        c.close()


@pytest.mark.parametrize("views,h,w,nreg", [(2, 504, 336, 0), (3, 504, 336, 1), (5, 42, 28, 1), (1, 14, 14, 0)])
def test_prepare_tokens_device_matches_oracle(views, h, w, nreg):
    wts = syn.patch_embed_weights(E, PATCH, GRID, nreg, seed=2)
    img = syn.images(views, h, w, seed=3)
    gh, gw = h // PATCH, w // PATCH
    n = 1 + nreg + gh * gw
    c = _ctx(nreg)
    try:
        _load(c, wts)
        out = torch.full((views * n, E), float("nan"), device="cuda")
        c.prepare_tokens_device(torch.from_numpy(img).cuda(), views, h, w, out)
        torch.cuda.synchronize()
        c.check_device()
        got = out.cpu().numpy().reshape(views, n, E)
        ref = _oracle_tokens(img, wts, tk.interpolate_pos_embed(wts["pos_embed"], GRID, E, gh, gw))
        assert np.isfinite(got).all(), "rows left unwritten"
        special = 1 + nreg
        assert np.array_equal(got[:, :special], ref[:, :special]), "CLS / register rows"
        _close(got[:, special:], ref[:, special:], f"patch rows {views}x{h}x{w}")
    finally:
        c.close()


def test_host_path_equals_device_path_and_takes_a_position_table():
    views, h, w, nreg = 2, 504, 336, 1
    wts = syn.patch_embed_weights(E, PATCH, GRID, nreg, seed=4)
    img = syn.images(views, h, w, seed=5)
    gh, gw = h // PATCH, w // PATCH
    n = 1 + nreg + gh * gw
    c = _ctx(nreg)
    try:
        _load(c, wts)
        dev = torch.empty(views * n, E, device="cuda")
        c.prepare_tokens_device(torch.from_numpy(img).cuda(), views, h, w, dev)
        torch.cuda.synchronize()
        host = c.prepare_tokens_host(img, h, w)
        assert np.array_equal(host.reshape(-1, E), dev.cpu().numpy())
        # The reference's run() takes the position table from its PosEmbedCache; the
        # oracle's table is bit-identical to the device's, so the result is too.
        table = tk.interpolate_pos_embed(wts["pos_embed"], GRID, E, gh, gw)
        given = c.prepare_tokens_host(img, h, w, position=table)
        assert np.array_equal(given, host)
        # A different table changes exactly the CLS and patch rows.
        shifted = c.prepare_tokens_host(img, h, w, position=table + 1.0)
        assert np.array_equal(shifted[:, 1:1 + nreg], host[:, 1:1 + nreg])
        assert np.abs(shifted[:, 0] - host[:, 0] - 1.0).max() < 1e-5
        assert np.abs(shifted[:, 1 + nreg:] - host[:, 1 + nreg:] - 1.0).max() < 1e-5
    finally:
        c.close()


def test_executor_mirror_runs_one_image():
    cfg = va.ModelConfig(num_register=0)
    wts = syn.patch_embed_weights(E, PATCH, GRID, 0, seed=6)
    weights = {va.PATCH_EMBED_WEIGHT: wts["weight"], va.PATCH_EMBED_BIAS: wts["bias"],
               va.CLS_TOKEN_WEIGHT: wts["cls"], va.POS_EMBED_WEIGHT: wts["pos_embed"]}
    ex = va.CudaPatchEmbedExecutor(cfg, weights, 0, max_rows=2048)
    try:
        img = syn.images(1, 252, 182, seed=7)[0]
        gh, gw, t = ex.run(img, 252, 182)
        assert (gh, gw) == (18, 13) and t.shape == (1 + 18 * 13, E)
        _, _, ref = tk.prepare_tokens(img, wts["weight"], wts["bias"], wts["cls"], wts["pos_embed"], PATCH)
        _close(t, ref, "executor run")
    finally:
        ex.ctx.close()


def test_bad_shapes_are_rejected():
    wts = syn.patch_embed_weights(E, PATCH, GRID, 0, seed=8)
    c = _ctx(0, max_rows=1024)
    try:
        with pytest.raises(va.VestraError, match="perfect square"):
            c.load_patch_embed(wts["weight"], wts["bias"], wts["cls"], wts["pos_embed"][:-1], None, PATCH)
        with pytest.raises(va.VestraError, match="num_register"):
            c.load_patch_embed(wts["weight"], wts["bias"], wts["cls"], wts["pos_embed"],
                               np.zeros((1, E), np.float32), PATCH)
        with pytest.raises(va.VestraError, match="not loaded"):
            c.pos_embed_device(2, 2, torch.empty(5, E, device="cuda"))
        _load(c, wts)
        out = torch.empty(64, E, device="cuda")
        with pytest.raises(va.VestraError, match="multiples of patch_size"):
            c.prepare_tokens_device(torch.zeros(3, 30, 28, device="cuda"), 1, 30, 28, out)
        with pytest.raises(va.VestraError, match="max_rows"):
            c.prepare_tokens_device(torch.zeros(2, 3, 504, 336, device="cuda"), 2, 504, 336, out)
    finally:
        c.close()


def test_tokens_feed_a_global_block(oracle_mod):
    """prepare_tokens -> one global block on the device, against the oracle chain."""
    views, h, w, nreg = 2, 126, 84, 1
    gh, gw = h // PATCH, w // PATCH
    n = 1 + nreg + gh * gw
    wts = syn.patch_embed_weights(E, PATCH, GRID, nreg, seed=9)
    img = syn.images(views, h, w, seed=10)
    layer = 5
    p = syn.layer_weights(E, seed=11, layer=layer, bias=True, norm1=True, perturb_norm=True, ls1=True,
                          mlp=True, ls2=True)
    c = _ctx(nreg, max_rows=views * n)
    try:
        _load(c, wts)
        c.load_layer(layer, p)
        c.load_mlp(layer, p)
        t = torch.empty(views * n, E, device="cuda")
        c.prepare_tokens_device(torch.from_numpy(img).cuda(), views, h, w, t)
        c.block_device(layer, t, gh, gw, views, True)
        torch.cuda.synchronize()
        c.check_device()
        x = _oracle_tokens(img, wts, tk.interpolate_pos_embed(wts["pos_embed"], GRID, E, gh, gw)).reshape(-1, E)
        pos = va.positions_yx(views * n, views, 1 + nreg, gh, gw, True)
        ref = oracle_mod.block(x, p, E // 64, pos_yx=pos, seg_len=0)
        _close(t.cpu().numpy(), ref, "tokens -> global block")
    finally:
        c.close()
