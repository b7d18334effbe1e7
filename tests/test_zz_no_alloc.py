"""va_op_attention_noalloc: Op::Attention for callers that cannot allocate device memory.

Such callers (a process whose allocator owns the whole GPU, or a block loop that
must not stall on, or fail in, cudaMalloc) get the same result as the context-based
entry point, computed with the library's fixed scratch array instead of any
allocation.  Each case is checked against that entry point and against the CPU
restatement (oracle/) directly.  This file is collected last so a failure here
leaves every other test already run; it needs nothing from them and also passes
alone in a fresh process.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")]

import vestra_attn as va  # noqa: E402

MAX_ABS = 2e-2   # the tolerance of the other GPU parity tests
MIN_COS = 0.9999


def _case(heads, n, seed, pos_max=40):
    rng = np.random.default_rng(seed)
    q, k, v = (rng.standard_normal((heads, n, 64)).astype(np.float32) for _ in range(3))
    g = (1 + 0.1 * rng.standard_normal(64)).astype(np.float32)
    b = (0.1 * rng.standard_normal(64)).astype(np.float32)
    pos = np.stack([rng.integers(0, pos_max, n), rng.integers(0, pos_max, n)], 1).astype(np.float32)
    return q, k, v, g, b, pos


def _close(a, r, what):
    a, r = np.asarray(a, np.float64), np.asarray(r, np.float64)
    assert np.isfinite(a).all(), what
    err = np.abs(a - r).max()
    cos = (a.ravel() @ r.ravel()) / (np.linalg.norm(a) * np.linalg.norm(r))
    assert err <= MAX_ABS and cos >= MIN_COS, (what, err, cos)


def _run(oracle_mod, heads, n, seed, norm=True, rope=True, pairing=0, pos_max=40):
    q, k, v, g, b, pos = _case(heads, n, seed, pos_max)
    ctx = va.Context(va.default_config(max_rows=1024, rope_pairing=pairing), 0)
    try:
        tq, tk, tv = (torch.from_numpy(x).cuda() for x in (q, k, v))
        tg, tb = torch.from_numpy(g).cuda(), torch.from_numpy(b).cuda()
        kg, kb = torch.flip(tg, [0]).contiguous(), torch.flip(tb, [0]).contiguous()
        qn, kn = ((tg, tb), (kg, kb)) if norm else (None, None)
        ref = torch.empty_like(tq)
        ctx.op_attention(tq, tk, tv, ref, qnorm=qn, knorm=kn, rope=(pos, 100.0) if rope else None)
        torch.cuda.synchronize()
        ctx.check_device()
    finally:
        ctx.close()
    got = torch.full_like(tq, float("nan"))
    rc = va.op_attention_noalloc(tq, tk, tv, got, qnorm=qn, knorm=kn,
                                 pos_yx_dev=torch.from_numpy(pos).cuda() if rope else None, freq=100.0,
                                 rope_pairing=pairing)
    assert rc == va.VA_OK
    what = f"h{heads} n{n} norm={norm} rope={rope} pairing={pairing} pos<{pos_max}"
    _close(got.cpu().numpy(), ref.cpu().numpy(), what + " vs context entry point")
    oref = oracle_mod.op_attention(q, k, v, qnorm=(g, b) if norm else None,
                                   knorm=(g[::-1].copy(), b[::-1].copy()) if norm else None,
                                   rope=(pos, 100.0) if rope else None, pairing=pairing)
    _close(got.cpu().numpy(), oref, what + " vs oracle")


def test_noalloc_matches_context_entry_point_on_two_calls_in_a_row(oracle_mod):
    # Two different shapes back to back: the second call runs on scratch the first
    # one left behind.
    _run(oracle_mod, 12, 866, 1)
    _run(oracle_mod, 3, 197, 2)


@pytest.mark.parametrize("norm,rope,pairing,pos_max", [(True, True, 1, 40), (False, False, 0, 40),
                                                       (False, True, 0, 40), (True, True, 0, 3000)])
def test_noalloc_norm_rope_variants(oracle_mod, norm, rope, pairing, pos_max):
    # Interleaved pairing, neither norm nor RoPE, RoPE alone, and positions in the
    # thousands (the angles are formed in double on the device).
    _run(oracle_mod, 4, 300, 7, norm=norm, rope=rope, pairing=pairing, pos_max=pos_max)


def test_noalloc_rejects_requests_beyond_its_scratch():
    heads, n = 16, va.NOALLOC_MAX_ELEMS // (16 * 64) + 1
    t = torch.empty(1, device="cuda")
    assert va.load_library().va_op_attention_noalloc(
        t.data_ptr(), t.data_ptr(), t.data_ptr(), heads, n, 64, None, None, None, None, 1e-5,
        None, 100.0, 0, t.data_ptr(), None) == va.VA_ERR_CAPACITY


def test_noalloc_rejects_positions_out_of_range():
    q = torch.randn(2, 50, 64, device="cuda")
    out = torch.empty_like(q)
    pos = torch.zeros(50, 2, device="cuda")
    pos[17, 1] = 70000.0  # above the 16-bit range of the context entry points
    assert va.op_attention_noalloc(q, q, q, out, pos_yx_dev=pos) == va.VA_ERR_INVALID
    pos[17, 1] = -0.6  # rounds to -1
    assert va.op_attention_noalloc(q, q, q, out, pos_yx_dev=pos) == va.VA_ERR_INVALID
    pos[17, 1] = 0.5   # rounds half away from zero to 1: valid
    assert va.op_attention_noalloc(q, q, q, out, pos_yx_dev=pos) == va.VA_OK
