"""GPU parity of the GGUF model-file path: the device conversion of stored tensor
bytes (F32, F16, Q8_0; rank-2 transposed or not) against the oracle's host decoding,
bit for bit (Q8_0 and F16 values are exact in F32), and va_load_model_gguf against
the host route the reference takes (weights_from_gguf to F32, then the per-set
loads): the loaded weights must give bitwise-equal block and token outputs.
Every call goes through the C ABI."""
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")]

import gguf  # noqa: E402
import synthetic as syn  # noqa: E402
import vestra_attn as va  # noqa: E402


def _file(tmp_path, data, name="m.gguf"):
    p = tmp_path / name
    p.write_bytes(data)
    return str(p)


@pytest.fixture(scope="module")
def tensors_file(tmp_path_factory):
    r = np.random.default_rng(17)
    w = syn.GgufWriter(alignment=64)
    cases = {}
    for dt in ("f32", "f16", "q8_0"):
        for name, shape in (("m", (96, 64)), ("odd2d", (32, 7)), ("r3", (2, 4, 32)), ("big", (4096, 1024)),
                            ("row", (1, 768))):
            if dt == "q8_0" and int(np.prod(shape)) % 32:
                continue
            a = (r.standard_normal(shape) * (10.0 if name == "odd2d" else 1.0)).astype(np.float32)
            w.tensor(f"{dt}.{name}", a, dt)
            cases[f"{dt}.{name}"] = shape
        if dt != "q8_0":
            w.tensor(f"{dt}.ragged", r.standard_normal(13).astype(np.float32), dt)
            cases[f"{dt}.ragged"] = (13,)
    data = w.to_bytes()
    path = tmp_path_factory.mktemp("gguf") / "t.gguf"
    path.write_bytes(data)
    return str(path), gguf.GgufFile(data), cases


@pytest.mark.parametrize("transpose", [False, True])
def test_tensor_f32_bitwise(tensors_file, transpose):
    path, o, cases = tensors_file
    with va.GgufFile(path) as g:
        for name, shape in cases.items():
            oshape, ref = o.tensor_f32(name)
            if transpose and len(oshape) == 2:
                ref = ref.reshape(oshape).T.reshape(-1)
            gshape, got = g.tensor_f32(name, transpose2d=transpose)
            assert gshape == oshape == list(shape)
            assert got.view(np.uint32).tobytes() == ref.view(np.uint32).tobytes(), name


def test_tensor_device_unaligned_output(tensors_file):
    path, o, _ = tensors_file
    with va.GgufFile(path) as g:
        for name in ("q8_0.m", "f16.ragged", "f32.r3"):
            _, ref = o.tensor_f32(name)
            buf = torch.full((ref.size + 3,), float("nan"), device="cuda")
            g.tensor_device(name, buf[1:1 + ref.size])  # 4-byte aligned only: the scalar store path
            got = buf.cpu().numpy()
            assert np.isnan(got[0]) and np.isnan(got[-2:]).all()
            assert got[1:1 + ref.size].view(np.uint32).tobytes() == ref.view(np.uint32).tobytes(), name


def _host_route(ctx, weights, depth, embed, num_register):
    """weights_from_gguf content -> the per-set host loads (vit_block.rs:239-318)."""
    for i in range(depth):
        if va.wname(i, "attn_qkv.weight") not in weights:
            continue
        ctx.load_layer(i, va.layer_params_from_weights(weights, i))
        ctx.load_mlp(i, va.mlp_params_from_weights(weights, i))
    ctx.load_patch_embed(weights[va.PATCH_EMBED_WEIGHT].reshape(embed, 3, 14, 14), weights[va.PATCH_EMBED_BIAS],
                         weights[va.CLS_TOKEN_WEIGHT], weights[va.POS_EMBED_WEIGHT],
                         weights.get(va.REGISTER_TOKENS_WEIGHT) if num_register else None)
    ctx.load_vit_norm(weights["vit.norm.weight"], weights["vit.norm.bias"])


@pytest.mark.parametrize("dtype,layout", [("q8_0", "rank2"), ("f16", "rank2"), ("f32", "flat"), ("q8_0", "flat")])
def test_load_model_gguf_equals_host_route(tmp_path, dtype, layout):
    embed, heads, depth, nreg = 768, 12, 6, 2
    data = syn.gguf_model(embed=embed, depth=depth, heads=heads, num_register=nreg, grid=6, dtype=dtype,
                          layout=layout, layers=[4, 5], seed=3)
    path = _file(tmp_path, data)
    with va.GgufFile(path) as g:
        mc = va.ModelConfig.from_gguf(g)
        assert (mc.embed_dim, mc.num_heads, mc.depth, mc.num_register, mc.alt_start) == (embed, heads, depth, nreg, 4)
        a = va.Context(mc.to_va(4 * 300), 0)
        sent = a.load_gguf(g)
    assert sent == sum(len(gguf.GgufFile(data).tensor_check(n)[3]) for n in gguf.GgufFile(data).tensor_names())
    b = va.Context(mc.to_va(4 * 300), 0)
    _host_route(b, gguf.weights_from_gguf(gguf.GgufFile(data)), depth, embed, nreg)

    h, w_, views = 140, 196, 3
    img = syn.images(views, h, w_, seed=4)
    ta, tb = a.prepare_tokens_host(img, h, w_), b.prepare_tokens_host(img, h, w_)
    assert ta.tobytes() == tb.tobytes()
    gh, gw = h // 14, w_ // 14
    x = ta.reshape(-1, embed)
    for layer, global_ in ((4, False), (5, True)):
        ya = a.run_tail(layer, x, gh, gw, views, global_)
        yb = b.run_tail(layer, x, gh, gw, views, global_)
        assert np.isfinite(ya).all() and ya.tobytes() == yb.tobytes(), layer
    a.close()
    b.close()


def test_executor_from_gguf(tmp_path):
    data = syn.gguf_model(embed=768, depth=6, heads=12, grid=4, dtype="q8_0", layers=[5], seed=9)
    path = _file(tmp_path, data)
    ex = va.CudaTransformerTailExecutor.from_gguf(path, max_rows=2 * 200)
    ref = va.CudaTransformerTailExecutor(ex.cfg, gguf.weights_from_gguf(gguf.GgufFile(data)), max_rows=2 * 200)
    x = syn.hidden_states(2 * (1 + 8 * 8), 768, seed=2)
    ya = ex.run_tail(5, x, None, x.shape[0], 8, 8, True, 2)
    yb = ref.run_tail(5, x, None, x.shape[0], 8, 8, True, 2)
    assert ya.tobytes() == yb.tobytes()


def test_load_model_gguf_errors(tmp_path):
    data = syn.gguf_model(embed=768, depth=2, heads=12, grid=4, dtype="q8_0", layers=[1], patch_embed=False)
    path = _file(tmp_path, data)
    with va.GgufFile(path) as g:
        c = va.Context(va.default_config(embed_dim=1024, num_heads=16, depth=2, max_rows=256), 0)
        with pytest.raises(va.VestraError) as e:
            c.load_gguf(g)
        assert e.value.code == va.VA_ERR_INVALID and "attn_qkv.weight" in str(e.value)
        c.close()
    # a file whose block lacks its required qkv bias
    w = syn.GgufWriter()
    syn.model_metadata(w, 768, 1, 12, 3072)
    r = np.random.default_rng(0)
    w.tensor("vit.blk.0.attn_qkv.weight", r.standard_normal((2304, 768)).astype(np.float32), "q8_0")
    path2 = _file(tmp_path, w.to_bytes(), "nobias.gguf")
    with va.GgufFile(path2) as g:
        c = va.Context(va.default_config(depth=1, max_rows=256), 0)
        with pytest.raises(va.VestraError) as e:
            c.load_gguf(g)
        assert e.value.code == va.VA_ERR_NOT_FOUND and "vit.blk.0.attn_qkv.bias" in str(e.value)
        c.close()


def test_reload_and_mixed_ownership(tmp_path):
    """A second model file replaces the first (its weight arena is released); a host
    load over a block that came from the file owns its own buffers; both routes give
    the same block output."""
    data = syn.gguf_model(embed=768, depth=6, heads=12, grid=4, dtype="q8_0", layers=[4, 5], seed=5)
    path = _file(tmp_path, data)
    x = syn.hidden_states(2 * (1 + 8 * 8), 768, seed=1)
    with va.GgufFile(path) as g:
        c = va.Context(va.ModelConfig.from_gguf(g).to_va(256), 0)
        c.load_gguf(g)
        y0 = c.run_tail(5, x, 8, 8, 2, True)
        weights = gguf.weights_from_gguf(gguf.GgufFile(data))
        c.load_layer(5, va.layer_params_from_weights(weights, 5))
        c.load_mlp(5, va.mlp_params_from_weights(weights, 5))
        y1 = c.run_tail(5, x, 8, 8, 2, True)
        c.load_gguf(g)
        y2 = c.run_tail(5, x, 8, 8, 2, True)
        y3 = c.run_tail(4, x, 8, 8, 2, False)
        c.close()
    assert np.isfinite(y0).all() and np.isfinite(y3).all()
    assert y0.tobytes() == y1.tobytes() == y2.tobytes()
