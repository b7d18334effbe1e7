"""Parity against the reference's own dumps and a real DA3 model, when they exist.

The reference gates its real-weight and kernel parity on files it does not ship: a
dump GGUF (`dumps/reference.gguf`) with a `manifest.json` of tolerances
(da-parity/src/lib.rs:14-135), and a DA3 model file.  Its tests skip with a message
when those are absent (crates/da-engine/tests/kernel_rope_parity.rs:5-18,
backbone_parity.rs:183-235).  This file does the same:

  VA_DUMPS=<dir>      the dump directory (reference.gguf + manifest.json)
  VA_DA3_GGUF=<file>  a DA3 model file (e.g. da3-base-f16.gguf)
  VA_ROPE_PAIRING=0|1 the RoPE pairing the library is configured with (default 0)

* rope2d: the dump's rope_in / rope_pos / rope_out (1 head, 4 tokens, head_dim 64,
  base 100) through the CPU restatement and, on a GPU, through Op::Attention.  This
  is the check that pins the pairing inside each half, the one convention no test
  in the reference checkout fixes; a failure says whether the other pairing fits.
* backbone: input_image -> tokens -> 12 blocks on the GPU, the captures of layers
  5/7/9/11 against feat_{5,7,9,11} and cam_token_{5,7,9,11}.

Tolerances: the CPU restatement uses the manifest's atol/rtol, as the reference's
assert_parity does (|got - ref| <= atol + rtol |ref| elementwise).  The GPU path
computes in bf16 with F32 accumulation, so it is held to the attention gates
(max-abs <= 2e-2, cosine >= 0.9999) for one op, and for the captures of a 12-block
stack to cosine >= 0.999 per capture with the max-abs reported.
"""
import json
import os

import numpy as np
import pytest

import vestra_attn as va  # noqa: E402

MODEL = os.environ.get("VA_DA3_GGUF")
PAIRING = int(os.environ.get("VA_ROPE_PAIRING", "0"))


def _dumps():
    DUMPS = os.environ.get("VA_DUMPS")
    if not DUMPS or not os.path.exists(os.path.join(DUMPS, "reference.gguf")):
        pytest.skip("[skip] no dumps (set VA_DUMPS to a directory with reference.gguf and manifest.json)")
    from gguf import GgufFile  # oracle/gguf.py: the restated reader (test infrastructure)

    g = GgufFile.open(os.path.join(DUMPS, "reference.gguf"))
    atol = rtol = 2e-3  # da-parity's defaults
    mpath = os.path.join(DUMPS, "manifest.json")
    if os.path.exists(mpath):
        with open(mpath) as f:
            m = json.load(f)
        atol, rtol = float(m.get("atol", atol)), float(m.get("rtol", rtol))
    return g, atol, rtol


def _parity(got, ref, atol, rtol):
    """da-parity's compare: ok when every |got - ref| <= atol + rtol |ref|."""
    got, ref = np.asarray(got, np.float64).ravel(), np.asarray(ref, np.float64).ravel()
    assert got.shape == ref.shape, (got.shape, ref.shape)
    d = np.abs(got - ref)
    return bool((d <= atol + rtol * np.abs(ref)).all()), float(d.max())


def _rope_tensors(g):
    _, rin = g.tensor_f32("rope_in")     # (1, 1, 4, 64): heads 1, 4 tokens, head_dim 64
    _, rpos = g.tensor_f32("rope_pos")   # (1, 4, 2): (y, x) as F32
    _, rout = g.tensor_f32("rope_out")
    n = rpos.size // 2
    return rin.reshape(1, n, 64), rpos.reshape(n, 2), rout.reshape(1, n, 64)


def test_rope2d_matches_reference_dump(oracle_mod):
    g, atol, rtol = _dumps()
    rin, rpos, rout = _rope_tensors(g)
    ok, err = _parity(oracle_mod.rope2d(rin, rpos, 100.0, pairing=PAIRING), rout, atol, rtol)
    if not ok:
        other_ok, other_err = _parity(oracle_mod.rope2d(rin, rpos, 100.0, pairing=1 - PAIRING), rout, atol, rtol)
        pytest.fail(f"rope2d pairing {PAIRING}: max|d| {err:.3e}; pairing {1 - PAIRING} "
                    f"{'matches' if other_ok else 'does not match either'} (max|d| {other_err:.3e})")


@pytest.mark.gpu
def test_rope2d_dump_through_gpu_op_attention(oracle_mod):
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    g, _, _ = _dumps()
    rin, rpos, rout = _rope_tensors(g)
    v = np.random.default_rng(0).standard_normal(rin.shape).astype(np.float32)
    # The GPU rotates q and k itself; the oracle attends over the dump's rotated rows.
    ref = oracle_mod.op_attention(rout, rout, v)
    ctx = va.Context(va.default_config(max_rows=1024, rope_pairing=PAIRING), 0)
    try:
        dev = [torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in (rin, rin, v)]
        out = torch.empty_like(dev[0])
        ctx.op_attention(*dev, out, rope=(rpos, 100.0))
        torch.cuda.synchronize()
        ctx.check_device()
        got = out.cpu().numpy()
    finally:
        ctx.close()
    a, b = got.astype(np.float64).ravel(), ref.astype(np.float64).ravel()
    err = float(np.abs(a - b).max())
    cos = float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))
    assert err <= 2e-2 and cos >= 0.9999, f"GPU rope via Op::Attention: max-abs {err:.3e} cos {cos:.7f}"


@pytest.mark.gpu
def test_backbone_captures_match_reference_dumps():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    if not MODEL or not os.path.exists(MODEL):
        pytest.skip("[skip] no DA3 model file (set VA_DA3_GGUF)")
    g, _, _ = _dumps()
    shape, img = g.tensor_f32("input_image")  # [3, H, W], preprocessed
    _, h, w = shape
    with va.GgufFile(MODEL) as mf:
        cfg = va.ModelConfig.from_gguf(mf)
        mc = mf.model_config()
        p = cfg.patch_size
        gh, gw = h // p, w // p
        n = 1 + cfg.num_register + gh * gw
        ctx = va.Context(cfg.to_va(max_rows=max(n, 1024), rope_pairing=PAIRING), 0)
        try:
            ctx.load_gguf(mf)
            cam_shape, cam = mf.tensor_f32("vit.camera_token")
            tokens = torch.empty(n, cfg.embed_dim, device="cuda")
            ctx.prepare_tokens_device(torch.from_numpy(img.reshape(1, 3, h, w)).cuda(), 1, h, w, tokens)
            out_layers = (5, 7, 9, 11)
            caps = ctx.backbone_device(tokens, gh, gw, 1, 0, cfg.depth, cfg.alt_start,
                                       camera_dev=torch.from_numpy(cam).cuda(), out_layers=out_layers,
                                       cat_token=bool(mc["cat_token"]))
            torch.cuda.synchronize()
            ctx.check_device()
            for layer in out_layers:
                for name, got in ((f"feat_{layer}", caps[layer][0]), (f"cam_token_{layer}", caps[layer][1])):
                    _, ref = g.tensor_f32(name)
                    a = got.cpu().numpy().astype(np.float64).ravel()
                    b = ref.astype(np.float64).ravel()
                    assert a.shape == b.shape, (name, a.shape, b.shape)
                    cos = float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))
                    err = float(np.abs(a - b).max())
                    assert cos >= 0.999, f"{name}: cos {cos:.6f} max-abs {err:.3e}"
        finally:
            ctx.close()


def _fabricated_dump(tmp_path, oracle_mod, pairing):
    """A dump directory in the reference's layout whose rope_out was made by the CPU
    restatement with the given pairing (exercises the harness; pins nothing)."""
    import synthetic as syn

    rng = np.random.default_rng(3)
    rin = rng.standard_normal((1, 4, 64)).astype(np.float32)
    rpos = np.array([[0, 0], [1, 1], [1, 2], [3, 5]], np.float32)
    rout = oracle_mod.rope2d(rin, rpos, 100.0, pairing=pairing)
    w = syn.GgufWriter()
    w.tensor("rope_in", rin.reshape(1, 1, 4, 64))
    w.tensor("rope_pos", rpos.reshape(1, 4, 2))
    w.tensor("rope_out", rout.reshape(1, 1, 4, 64))
    (tmp_path / "reference.gguf").write_bytes(w.to_bytes())
    (tmp_path / "manifest.json").write_text(json.dumps({"atol": 1e-5, "rtol": 1e-5}))
    return str(tmp_path)


@pytest.mark.parametrize("pairing", [0, 1])
def test_harness_on_a_fabricated_dump(tmp_path, monkeypatch, oracle_mod, pairing):
    monkeypatch.setenv("VA_DUMPS", _fabricated_dump(tmp_path, oracle_mod, pairing))
    if pairing == PAIRING:
        test_rope2d_matches_reference_dump(oracle_mod)
    else:
        with pytest.raises(pytest.fail.Exception, match=f"pairing {pairing} matches"):
            test_rope2d_matches_reference_dump(oracle_mod)


def test_harness_skips_without_dumps(monkeypatch, oracle_mod):
    monkeypatch.delenv("VA_DUMPS", raising=False)
    with pytest.raises(pytest.skip.Exception, match="no dumps"):
        test_rope2d_matches_reference_dump(oracle_mod)
