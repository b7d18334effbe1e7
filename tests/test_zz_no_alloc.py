"""va_op_attention_noalloc: Op::Attention for callers that cannot allocate device memory.

Such callers (a process whose allocator owns the whole GPU, or a block loop that
must not stall on, or fail in, cudaMalloc) get the same result as the context-based
entry point, computed with the library's fixed scratch array instead of any
allocation.  This file is collected last so a failure here leaves every other test
already run; it needs nothing from them and also passes alone in a fresh process.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")]

import vestra_attn as va  # noqa: E402

MAX_ABS = 2e-2   # the tolerance of the other GPU parity tests
MIN_COS = 0.9999


def _case(heads, n, seed):
    rng = np.random.default_rng(seed)
    q, k, v = (rng.standard_normal((heads, n, 64)).astype(np.float32) for _ in range(3))
    g = (1 + 0.1 * rng.standard_normal(64)).astype(np.float32)
    b = (0.1 * rng.standard_normal(64)).astype(np.float32)
    pos = np.stack([rng.integers(0, 40, n), rng.integers(0, 40, n)], 1).astype(np.float32)
    return q, k, v, g, b, pos


def test_noalloc_matches_context_entry_point_on_two_calls_in_a_row():
    ctx = va.Context(va.default_config(max_rows=1024), 0)
    try:
        # Two different shapes back to back: the second call runs on scratch the
        # first one left behind.
        for heads, n, seed in ((12, 866, 1), (3, 197, 2)):
            q, k, v, g, b, pos = _case(heads, n, seed)
            tq, tk, tv = (torch.from_numpy(x).cuda() for x in (q, k, v))
            tg, tb = torch.from_numpy(g).cuda(), torch.from_numpy(b).cuda()
            kg, kb = torch.flip(tg, [0]).contiguous(), torch.flip(tb, [0]).contiguous()
            ref = torch.empty_like(tq)
            ctx.op_attention(tq, tk, tv, ref, qnorm=(tg, tb), knorm=(kg, kb), rope=(pos, 100.0))
            torch.cuda.synchronize()
            ctx.check_device()
            got = torch.full_like(tq, float("nan"))
            rc = va.op_attention_noalloc(tq, tk, tv, got, qnorm=(tg, tb), knorm=(kg, kb),
                                         pos_yx_dev=torch.from_numpy(pos).cuda(), freq=100.0)
            assert rc == va.VA_OK
            a, r = got.cpu().numpy().astype(np.float64), ref.cpu().numpy().astype(np.float64)
            assert np.isfinite(a).all()
            err = np.abs(a - r).max()
            cos = (a.ravel() @ r.ravel()) / (np.linalg.norm(a) * np.linalg.norm(r))
            assert err <= MAX_ABS and cos >= MIN_COS, (heads, n, err, cos)
    finally:
        ctx.close()


def test_noalloc_rejects_requests_beyond_its_scratch():
    heads, n = 16, va.NOALLOC_MAX_ELEMS // (16 * 64) + 1
    t = torch.empty(1, device="cuda")
    assert va.load_library().va_op_attention_noalloc(
        t.data_ptr(), t.data_ptr(), t.data_ptr(), heads, n, 64, None, None, None, None, 1e-5,
        None, 100.0, 0, t.data_ptr(), None) == va.VA_ERR_CAPACITY
