"""The attention kernel's fixed exponent offset.  QK-normalised layers whose norm
weights bound |q.k| * scale * log2(e) by 64 run the softmax with exponents relative
to 0 instead of the running row max; the result must match the row-max form to
bf16 rounding and pass the oracle gates, layers whose bound is larger must keep the
row-max form (bit-identical with the offset switched off), and the raw entry point
accepts the offset only with bf16 V.  Every call goes through the C ABI."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")]

import synthetic as syn  # noqa: E402
import vestra_attn as va  # noqa: E402

MAX_ABS, MIN_COS = 2e-2, 0.9999


def _run(monkeypatch, fixed, wl, p, x):
    monkeypatch.setenv("VA_SOFTMAX_FIXED_OFFSET", "1" if fixed else "0")
    ctx = va.Context(va.default_config(max_rows=wl.rows, num_register=wl.n_special - 1), 0)
    try:
        ctx.load_layer(5, p)
        y = ctx.attention_host(5, x, wl.gh, wl.gw, wl.views, wl.global_)
        ctx.check_device()
        return y
    finally:
        ctx.close()


def _cmp(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.abs(a - b).max()), float((a.ravel() @ b.ravel()) / (np.linalg.norm(a) * np.linalg.norm(b)))


@pytest.mark.parametrize("name", ["cfg2_s2_global", "cfg3_s12_global"])
def test_fixed_offset_matches_row_max_and_oracle(monkeypatch, oracle_mod, name):
    wl = syn.CONFIGS[name]
    p = syn.layer_weights(wl.embed, seed=6, layer=5, perturb_norm=True, ls1=True, bias=True)
    x = syn.hidden_states(wl.rows, wl.embed, seed=6)
    fixed = _run(monkeypatch, True, wl, p, x)
    rowmax = _run(monkeypatch, False, wl, p, x)
    err, cos = _cmp(fixed, rowmax)
    assert err <= 4e-3 and cos >= 0.99999, f"fixed vs row max: max-abs {err:.3e} cos {cos:.8f}"
    assert fixed.tobytes() != rowmax.tobytes()  # the two forms really ran
    rows = np.sort(np.random.default_rng(2).choice(wl.rows, 512, replace=False))
    pos = va.positions_yx(wl.rows, wl.views, wl.n_special, wl.gh, wl.gw, wl.global_)
    ref = oracle_mod.attention_block(x, p, wl.heads, pos_yx=pos, seg_len=0, q_rows=rows)
    err, cos = _cmp(fixed[rows], ref)
    assert err <= MAX_ABS and cos >= MIN_COS, f"fixed vs oracle: max-abs {err:.3e} cos {cos:.7f}"


def test_large_norm_weights_keep_the_row_max(monkeypatch):
    wl = syn.CONFIGS["cfg2_s2_global"]
    p = syn.layer_weights(wl.embed, seed=7, layer=5, perturb_norm=True)
    p["q_g"] = (10.0 * p["q_g"]).astype(np.float32)  # bound ~ 1e3 > 64: row max required
    x = syn.hidden_states(wl.rows, wl.embed, seed=7)
    a = _run(monkeypatch, True, wl, p, x)
    b = _run(monkeypatch, False, wl, p, x)
    assert np.isfinite(a).all() and a.tobytes() == b.tobytes()


def test_raw_entry_fixed_offset(monkeypatch):
    ctx = va.Context(va.default_config(max_rows=2048), 0)
    try:
        g = torch.Generator(device="cuda").manual_seed(3)

        def rows(n):
            x = torch.randn(n, 12, 64, device="cuda", generator=g)
            return torch.nn.functional.layer_norm(x, (64,)).view(n, 768).to(torch.bfloat16)

        q, k = rows(1000), rows(1800)
        v = torch.randn(1800, 768, device="cuda", generator=g).to(torch.bfloat16)
        o1 = torch.empty(1000, 768, device="cuda", dtype=torch.bfloat16)
        o2 = torch.empty_like(o1)
        ctx.flash_bf16(q, k, v, 12, o1, variant=256 + 24)
        ctx.flash_bf16(q, k, v, 12, o2, variant=24)
        torch.cuda.synchronize()
        ctx.check_device()
        err, cos = _cmp(o1.float().cpu().numpy(), o2.float().cpu().numpy())
        assert err <= 1e-2 and cos >= 0.99999
        with pytest.raises(va.VestraError):
            ctx.flash_bf16(q, k, v.to(torch.float16), 12, o1, variant=256 + 24)
    finally:
        ctx.close()
