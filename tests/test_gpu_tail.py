"""GPU parity of the device-resident transformer tail (whole ViT block) against the
CPU F32 restatement: x += attention(LN1 x) (*ls1); x += fc2(GELU_erf(fc1(LN2 x)))
(*ls2) (vit_block.rs:1019-1139, device form run_tail_device :489-583).

Gates as for the attention branch: max-abs <= 2e-2 and cosine >= 0.9999 on the
block output; the host entry (TransformerTailExecutor::run_tail) must equal the
device entry bit for bit.  Every call goes through the C ABI.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")]

import synthetic as syn  # noqa: E402
import vestra_attn as va  # noqa: E402

MAX_ABS, MIN_COS = 2e-2, 0.9999


def _close(got, ref, what):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    assert np.isfinite(got).all(), what
    err = float(np.abs(got - ref).max())
    cos = float((got.ravel() @ ref.ravel()) / (np.linalg.norm(got) * np.linalg.norm(ref)))
    assert err <= MAX_ABS and cos >= MIN_COS, f"{what}: max-abs {err:.3e} cos {cos:.7f}"


@pytest.fixture(scope="module")
def ctx():
    c = va.Context(va.default_config(max_rows=12 * 866, num_register=1, depth=12), 0)
    yield c
    c.close()


def _weights(ctx, layer, seed, ls):
    p = syn.layer_weights(768, seed=seed, layer=layer, bias=True, norm1=True, perturb_norm=True,
                          ls1=ls, mlp=True, ls2=ls)
    ctx.load_layer(layer, p)
    ctx.load_mlp(layer, p)
    return p


def _oracle_block(oracle_mod, ctx, x, p, wl, layer, rows=None):
    use_qk, use_rope = ctx.layer_flags(layer)
    pos = va.positions_yx(wl.rows, wl.views, wl.n_special, wl.gh, wl.gw, wl.global_) if use_rope else None
    ln1 = oracle_mod.layernorm(x, p["norm1_w"], p["norm1_b"], 1e-6)
    attn = oracle_mod.attention_block(ln1, p, wl.heads, pos_yx=pos, seg_len=wl.seg_len, use_qknorm=use_qk,
                                      q_rows=rows)
    x1 = (x if rows is None else x[rows]) + attn
    return oracle_mod.mlp_block(x1, p, 1e-6)


@pytest.mark.parametrize("name,ls", [("cfg1_single_view", False), ("cfg2_s2_global", True)])
def test_block_device_matches_oracle(ctx, oracle_mod, name, ls):
    wl = syn.CONFIGS[name]
    layer = 5
    p = _weights(ctx, layer, seed=21, ls=ls)
    x = syn.hidden_states(wl.rows, 768, seed=21)
    t = torch.from_numpy(x.copy()).cuda()
    ctx.block_device(layer, t, wl.gh, wl.gw, wl.views, wl.global_)
    torch.cuda.synchronize()
    ctx.check_device()
    _close(t.cpu().numpy(), _oracle_block(oracle_mod, ctx, x, p, wl, layer), name)


def test_block_s12_global_row_subset(ctx, oracle_mod):
    wl = syn.CONFIGS["cfg3_s12_global"]
    layer = 7
    p = _weights(ctx, layer, seed=22, ls=True)
    x = syn.hidden_states(wl.rows, 768, seed=22)
    t = torch.from_numpy(x.copy()).cuda()
    ctx.block_device(layer, t, wl.gh, wl.gw, wl.views, True)
    torch.cuda.synchronize()
    rows = np.sort(np.random.default_rng(22).choice(wl.rows, 96, replace=False)).astype(np.int64)
    _close(t.cpu().numpy()[rows], _oracle_block(oracle_mod, ctx, x, p, wl, layer, rows), "S=12 block")


def test_run_tail_host_equals_device_and_executor(ctx):
    wl = syn.CONFIGS["cfg2_s2_global"]
    layer = 6
    p = _weights(ctx, layer, seed=23, ls=True)
    x = syn.hidden_states(wl.rows, 768, seed=23)
    host = ctx.run_tail(layer, x, wl.gh, wl.gw, wl.views, True)
    t = torch.from_numpy(x.copy()).cuda()
    ctx.block_device(layer, t, wl.gh, wl.gw, wl.views, True)
    torch.cuda.synchronize()
    assert np.array_equal(host, t.cpu().numpy())
    # The executor mirror built from the reference's weight names gives the same.
    names = {"norm1_w": "norm1.weight", "norm1_b": "norm1.bias", "qkv_w": "attn_qkv.weight",
             "qkv_b": "attn_qkv.bias", "q_g": "attn_qnorm.weight", "q_b": "attn_qnorm.bias",
             "k_g": "attn_knorm.weight", "k_b": "attn_knorm.bias", "proj_w": "attn_proj.weight",
             "proj_b": "attn_proj.bias", "ls1": "ls1", "norm2_w": "norm2.weight", "norm2_b": "norm2.bias",
             "fc1_w": "mlp_fc1.weight", "fc1_b": "mlp_fc1.bias", "fc2_w": "mlp_fc2.weight",
             "fc2_b": "mlp_fc2.bias", "ls2": "ls2"}
    weights = {va.wname(layer, v): p[k] for k, v in names.items()}
    cfg = va.ModelConfig(num_register=1, depth=12)
    ex = va.CudaTransformerTailExecutor(cfg, weights, device=0, max_rows=wl.rows)
    got = ex.run_tail(layer, x, None, wl.rows, wl.gh, wl.gw, True, wl.views)
    assert np.array_equal(got, host)
    ex.ctx.close()


def test_tail_needs_mlp_weights(ctx):
    c = va.Context(va.default_config(max_rows=866, num_register=1), 0)
    try:
        c.load_layer(4, syn.layer_weights(768, seed=1, layer=4, norm1=True))
        t = torch.zeros(866, 768, device="cuda")
        with pytest.raises(va.VestraError):
            c.block_device(4, t, 36, 24, 1, False)
    finally:
        c.close()
