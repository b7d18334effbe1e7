"""The CPU F32 restatement (oracle/) pinned against the reference's own known-answer
tests and against an independent float64 restatement (tests/golden/).  CPU only."""
import json
import os

import numpy as np
import pytest

import synthetic as syn

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = os.path.join(HERE, "golden")


@pytest.fixture(scope="module")
def vectors():
    with open(os.path.join(GOLD, "reference_vectors.json")) as f:
        return json.load(f)


@pytest.fixture(scope="module")
def golden():
    return np.load(os.path.join(GOLD, "attention_block_small.npz"))


def _rng(seed):
    return np.random.default_rng(seed)


def _positions(oracle_mod, rows, views, ns, gh, gw, glob):
    return oracle_mod.positions(rows, views, ns, gh, gw, glob)


# --------------------------------------------------------------- golden fixtures
def test_block_cases_match_float64_restatement(oracle_mod, golden):
    import make_golden as mg  # tests/golden/make_golden.py
    for name, e, views, gh, gw, ns, glob, qk, rp, ls1, seed in mg.BLOCK_CASES:
        rows = views * (ns + gh * gw)
        x = syn.hidden_states(rows, e, seed=seed)
        p = syn.layer_weights(e, seed=seed, layer=0, qknorm=qk, ls1=ls1, bias=True, perturb_norm=True)
        pos = _positions(oracle_mod, rows, views, ns, gh, gw, glob) if rp else None
        seg = 0 if glob else rows // views
        got = oracle_mod.attention_block(x, p, e // 64, pos_yx=pos, seg_len=seg, use_qknorm=qk)
        np.testing.assert_allclose(got, golden[name], atol=2e-5, rtol=1e-4, err_msg=name)


def test_op_cases_match_float64_restatement(oracle_mod, golden):
    import make_golden as mg
    for name, heads, n, d, qk, rp, seed in mg.OP_CASES:
        q, k, v, g, b, pos = mg.op_inputs(heads, n, d, seed)
        got = oracle_mod.op_attention(q, k, v, qnorm=(g, b) if qk else None,
                                      knorm=(g[::-1].copy(), b[::-1].copy()) if qk else None,
                                      rope=(pos, 100.0) if rp else None)
        np.testing.assert_allclose(got, golden[name], atol=2e-5, rtol=1e-4, err_msg=name)


@pytest.fixture(autouse=True, scope="module")
def _golden_path():
    import sys
    if GOLD not in sys.path:
        sys.path.insert(0, GOLD)


# --------------------------------------------------------------- reference relation tests
def _xorshift(seed, n):
    """The reference tests' Xorshift32 mapped to [-1, 1] (attention_and_layerscale_op.rs:291-303)."""
    out = np.empty(n, np.float32)
    x = seed
    for i in range(n):
        x ^= (x << 13) & 0xFFFFFFFF
        x ^= x >> 17
        x ^= (x << 5) & 0xFFFFFFFF
        out[i] = np.float32(x) / np.float32(4294967295.0) * 2 - 1
    return out, x


def test_plain_op_attention_equals_naive(oracle_mod, vectors):
    # attention_and_layerscale_op.rs:39-74 (heads 2, n 3, head_dim 4)
    vals, _ = _xorshift(0xA5A51234, 3 * 24)
    q, k, v = (vals[i * 24:(i + 1) * 24].reshape(2, 3, 4) for i in range(3))
    got = oracle_mod.op_attention(q, k, v)
    ref = oracle_mod.attention_naive_f64(q, k, v)
    assert np.abs(got - ref).max() < vectors["plain_attention_tolerance"]["value"]


def test_qk_norm_uses_1e5_not_1e6(oracle_mod, vectors):
    # attention_and_layerscale_op.rs:92-196: near-constant rows separate the epsilons.
    heads, n, d = 2, 2, 4
    vals, state = _xorshift(0xC0DEF00D, 2 * heads * n * d)
    q = np.empty((heads * n, d), np.float32)
    k = np.empty((heads * n, d), np.float32)
    it = iter(vals)
    for row in range(heads * n):
        base = 100.0 + row
        for c in range(d):
            q[row, c] = base + next(it) * 1e-3
            k[row, c] = base - next(it) * 1e-3
    v, _ = _xorshift(state, heads * n * d)
    q, k, v = q.reshape(heads, n, d), k.reshape(heads, n, d), v.reshape(heads, n, d)
    g, b = np.ones(d, np.float32), np.zeros(d, np.float32)
    got = oracle_mod.op_attention(q, k, v, qnorm=(g, b), knorm=(g, b), qk_norm_eps=1e-5)

    def manual(eps):
        qn = oracle_mod.layernorm(q.reshape(-1, d), g, b, eps).reshape(q.shape)
        kn = oracle_mod.layernorm(k.reshape(-1, d), g, b, eps).reshape(k.shape)
        return oracle_mod.attention_naive_f64(qn, kn, v)

    ev = vectors["eps_discriminator"]
    assert np.abs(got - manual(1e-5)).max() < ev["correct_max_diff"]
    assert np.abs(got - manual(1e-6)).max() > ev["wrong_min_diff"]


def test_rope_changes_output(oracle_mod, vectors):
    # attention_and_layerscale_op.rs:203-260 (heads 1, n 2, head_dim 4)
    vals, _ = _xorshift(0x12345678, 3 * 8)
    q, k, v = (vals[i * 8:(i + 1) * 8].reshape(1, 2, 4) for i in range(3))
    rv = vectors["rope_changes_output"]
    pos = np.array(rv["pos_yx"], np.float32).reshape(2, 2)
    a = oracle_mod.op_attention(q, k, v)
    b = oracle_mod.op_attention(q, k, v, rope=(pos, rv["freq"]))
    assert np.abs(a - b).max() > rv["min_diff"]


def test_qk_norm_eps_constant(vectors):
    assert vectors["qk_norm_eps"]["value"] == 1e-5


# --------------------------------------------------------------- restatement properties
def test_positions_follow_vit_block_rule(oracle_mod):
    # vit_block.rs:841-881: specials (0,0); local patch p at (p/gw+1, p%gw+1); global (1,1).
    loc = oracle_mod.positions(2 * 8, 2, 2, 2, 3, False)
    np.testing.assert_array_equal(loc[:2], 0)
    np.testing.assert_array_equal(loc[2:8], [[1, 1], [1, 2], [1, 3], [2, 1], [2, 2], [2, 3]])
    np.testing.assert_array_equal(loc[8:10], 0)
    glo = oracle_mod.positions(2 * 8, 2, 2, 2, 3, True)
    np.testing.assert_array_equal(glo[[0, 1, 8, 9]], 0)
    np.testing.assert_array_equal(glo[2:8], 1)


def test_core_matches_naive_f64(oracle_mod):
    rng = _rng(0)
    for heads, n, d, seg in [(3, 133, 64, 0), (2, 99, 64, 33), (2, 9, 4, 0), (1, 40, 8, 8)]:
        q, k, v = (rng.standard_normal((heads, n, d)).astype(np.float32) for _ in range(3))
        got = oracle_mod.attention_core(q, k, v, seg_len=seg)
        ref = oracle_mod.attention_naive_f64(q, k, v, seg_len=seg)
        assert np.abs(got - ref).max() < 5e-6


def test_rope_identity_at_zero_and_norm_preserving(oracle_mod):
    rng = _rng(1)
    x = rng.standard_normal((2, 5, 64)).astype(np.float32)
    z = oracle_mod.rope2d(x, np.zeros((5, 2), np.float32))
    np.testing.assert_array_equal(z, x)
    pos = rng.integers(0, 40, (5, 2)).astype(np.float32)
    for pairing in (0, 1):
        y = oracle_mod.rope2d(x, pos, pairing=pairing)
        np.testing.assert_allclose(np.linalg.norm(y, axis=-1), np.linalg.norm(x, axis=-1), rtol=1e-5)


def test_nodiff_rope_only_affects_special_patch_pairs(oracle_mod):
    # Global blocks rotate every patch by the same angle: patch-patch scores keep
    # their values, scores against the unrotated special tokens change.
    rng = _rng(2)
    q = rng.standard_normal((1, 6, 64)).astype(np.float32)
    k = rng.standard_normal((1, 6, 64)).astype(np.float32)
    pos = oracle_mod.positions(6, 1, 2, 2, 2, True)
    qr, kr = oracle_mod.rope2d(q, pos), oracle_mod.rope2d(k, pos)
    s0 = q[0] @ k[0].T
    s1 = qr[0] @ kr[0].T
    np.testing.assert_allclose(s1[2:, 2:], s0[2:, 2:], rtol=1e-4, atol=1e-4)
    np.testing.assert_allclose(s1[:2, :2], s0[:2, :2], rtol=1e-6, atol=1e-6)
    assert np.abs(s1[:2, 2:] - s0[:2, 2:]).max() > 1e-3


def test_row_subset_equals_full(oracle_mod):
    wl = syn.Workload("t", 128, 2, 3, 2, 3, 2, True)
    x = syn.hidden_states(wl.rows, 128, seed=3)
    p = syn.layer_weights(128, seed=3, ls1=True, bias=True)
    pos = oracle_mod.positions(wl.rows, wl.views, 2, 2, 3, True)
    full = oracle_mod.attention_block(x, p, 2, pos_yx=pos, seg_len=0)
    rows = np.array([0, 5, 7, 23], np.int64)
    sub = oracle_mod.attention_block(x, p, 2, pos_yx=pos, seg_len=0, q_rows=rows)
    np.testing.assert_allclose(sub, full[rows], rtol=1e-5, atol=1e-6)


def test_global_couples_views_local_does_not(oracle_mod):
    # backbone.rs:1422-1443 at the attention-branch level.
    wl = syn.Workload("t", 128, 2, 2, 2, 2, 1, False)
    n = wl.tokens_per_view
    x = syn.hidden_states(wl.rows, 128, seed=4)
    y = x.copy()
    y[n:] = 2.0 - y[n:]
    p = syn.layer_weights(128, seed=4)
    for glob in (True, False):
        pos = oracle_mod.positions(wl.rows, 2, 1, 2, 2, glob)
        seg = 0 if glob else n
        a = oracle_mod.attention_block(x, p, 2, pos_yx=pos, seg_len=seg)[:n]
        b = oracle_mod.attention_block(y, p, 2, pos_yx=pos, seg_len=seg)[:n]
        assert (not np.array_equal(a, b)) == glob


def test_layerscale_presence_changes_output(oracle_mod):
    # vit_block.rs:1369-1401 at the attention-branch level.
    x = syn.hidden_states(10, 128, seed=5)
    p = syn.layer_weights(128, seed=5, ls1=True)
    a = oracle_mod.attention_block(x, p, 2)
    q = dict(p)
    del q["ls1"]
    b = oracle_mod.attention_block(x, q, 2)
    assert not np.array_equal(a, b)
    np.testing.assert_allclose(a, b * p["ls1"], rtol=1e-5, atol=1e-7)


def test_qknorm_gating_changes_output(oracle_mod):
    # vit_block.rs:1404-1453: blocks below qknorm_start skip QK-norm even with the tensors present.
    x = syn.hidden_states(10, 128, seed=6)
    p = syn.layer_weights(128, seed=6, perturb_norm=True)
    a = oracle_mod.attention_block(x, p, 2, use_qknorm=True)
    b = oracle_mod.attention_block(x, p, 2, use_qknorm=False)
    assert not np.array_equal(a, b)


def test_mlp_block_matches_float64_restatement(oracle_mod):
    # vit_block.rs:1092-1129: x + (GELU_erf(LN2(x) fc1 + b1) fc2 + b2) * ls2, restated
    # independently in float64 torch (exact erf GELU).
    torch = pytest.importorskip("torch")
    x = syn.hidden_states(40, 256, seed=11)
    for with_ls2 in (False, True):
        p = syn.layer_weights(256, seed=11, layer=3, mlp=True, ls2=with_ls2)
        got = oracle_mod.mlp_block(x, p, ln_eps=1e-6)
        t = lambda a: torch.from_numpy(np.asarray(a, np.float64))  # noqa: E731
        xt = t(x)
        ln = torch.nn.functional.layer_norm(xt, (256,), t(p["norm2_w"]), t(p["norm2_b"]), eps=1e-6)
        h = torch.nn.functional.gelu(ln @ t(p["fc1_w"]) + t(p["fc1_b"]), approximate="none")
        m = h @ t(p["fc2_w"]) + t(p["fc2_b"])
        if with_ls2:
            m = m * t(p["ls2"])
        ref = (xt + m).numpy()
        assert np.abs(got - ref).max() <= 2e-5, (with_ls2, np.abs(got - ref).max())


def test_mlp_ls2_presence_changes_output(oracle_mod):
    # LayerScale presence gating holds for ls2 as for ls1 (vit_block.rs:1369-1401).
    x = syn.hidden_states(16, 256, seed=12)
    p = syn.layer_weights(256, seed=12, layer=2, mlp=True, ls2=True)
    q = {k: v for k, v in p.items() if k != "ls2"}
    assert np.abs(oracle_mod.mlp_block(x, p) - oracle_mod.mlp_block(x, q)).max() > 1e-3
