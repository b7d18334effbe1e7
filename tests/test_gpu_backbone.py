"""GPU parity of the multi-view device route (va_backbone_device) against the CPU
restatement applied block by block, following forward_multi_view_with_persistent_
cuda_tail (backbone.rs:885-1137): global blocks at odd layers >= alt_start
(backbone.rs:459-460), camera slots before block alt_start (:746-768), the local
snapshot before a global block, and the out-layer captures of :1139-1179.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")]

import synthetic as syn  # noqa: E402
import vestra_attn as va  # noqa: E402

E, HEADS = 768, 12
ALT, QK_START, ROPE_START = 4, 4, 4


def _is_global(layer):
    return ALT >= 0 and layer >= ALT and layer % 2 == 1


def _capture(x, local, views, n, n_special, norm_w, norm_b, oracle_mod):
    feats, cams = [], []
    for v in range(views):
        xv, lv = x[v * n:(v + 1) * n], local[v * n:(v + 1) * n]
        normed = oracle_mod.layernorm(xv[n_special:], norm_w, norm_b, 1e-6)
        feats.append(np.concatenate([lv[n_special:], normed], axis=1))
        cams.append(np.concatenate([lv[0], xv[0]]))
    return np.stack(feats), np.stack(cams)


def _close(got, ref, what):
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    err = float(np.abs(got - ref).max())
    cos = float(got.ravel() @ ref.ravel() / (np.linalg.norm(got) * np.linalg.norm(ref)))
    assert err <= 2e-2 and cos >= 0.9999, f"{what}: max-abs {err:.3e} cos {cos:.7f}"


def test_backbone_route_matches_blockwise_oracle(oracle_mod):
    wl = syn.CONFIGS["cfg2_s2_global"]
    views, n_special = wl.views, wl.n_special
    n = wl.rows // views
    first, last, out_layers = 2, 8, (4, 5, 7)
    c = va.Context(va.default_config(max_rows=wl.rows, num_register=n_special - 1, depth=12,
                                     rope_start=ROPE_START, qknorm_start=QK_START), 0)
    try:
        params = {}
        for layer in range(first, last):
            p = syn.layer_weights(E, seed=30, layer=layer, bias=True, norm1=True, perturb_norm=True,
                                  ls1=True, mlp=True, ls2=True)
            c.load_layer(layer, p)
            c.load_mlp(layer, p)
            params[layer] = p
        r = np.random.default_rng(31)
        norm_w = (1.0 + 0.1 * r.standard_normal(E)).astype(np.float32)
        norm_b = (0.1 * r.standard_normal(E)).astype(np.float32)
        c.load_vit_norm(norm_w, norm_b)
        camera = syn.camera_tokens(E, seed=31)
        x0 = syn.hidden_states(wl.rows, E, seed=31)

        t = torch.from_numpy(x0.copy()).cuda()
        caps = c.backbone_device(t, wl.gh, wl.gw, views, first, last, ALT,
                                 camera_dev=torch.from_numpy(camera).cuda(), out_layers=out_layers)
        torch.cuda.synchronize()
        c.check_device()

        x = x0.copy()
        snap = None
        ref_caps = {}
        for layer in range(first, last):
            glob = _is_global(layer)
            if layer == ALT:
                for v in range(views):
                    x[v * n] = camera[:E] if v == 0 else camera[E:]
            pos = va.positions_yx(wl.rows, views, n_special, wl.gh, wl.gw, glob) if layer >= ROPE_START else None
            x = oracle_mod.block(x, params[layer], HEADS, pos_yx=pos, seg_len=0 if glob else n,
                                 use_qknorm=layer >= QK_START)
            if layer in out_layers:
                ref_caps[layer] = _capture(x, snap if glob else x, views, n, n_special, norm_w, norm_b, oracle_mod)
            if not glob and layer + 1 < last and _is_global(layer + 1):
                snap = x.copy()
        _close(t.cpu().numpy(), x, "tokens after blocks 2..7")
        for layer in out_layers:
            _close(caps[layer][0].cpu().numpy(), ref_caps[layer][0], f"feat capture {layer}")
            _close(caps[layer][1].cpu().numpy(), ref_caps[layer][1], f"cam capture {layer}")
    finally:
        c.close()


def test_backbone_route_replays_from_a_cuda_graph():
    """The device route issues only stream-ordered work once its position tables are
    built, so a whole layer range can be captured into a CUDA graph and replayed:
    the replay gives the eager result bit for bit."""
    wl = syn.CONFIGS["cfg2_s2_global"]
    views, n_special = wl.views, wl.n_special
    first, last = 2, 8
    c = va.Context(va.default_config(max_rows=wl.rows, num_register=n_special - 1, depth=12,
                                     rope_start=ROPE_START, qknorm_start=QK_START), 0)
    try:
        for layer in range(first, last):
            p = syn.layer_weights(E, seed=40, layer=layer, bias=True, norm1=True, perturb_norm=True,
                                  ls1=True, mlp=True, ls2=True)
            c.load_layer(layer, p)
            c.load_mlp(layer, p)
        x0 = torch.from_numpy(syn.hidden_states(wl.rows, E, seed=41)).cuda()
        camera = torch.from_numpy(syn.camera_tokens(E, seed=41)).cuda()
        side = torch.cuda.Stream()
        t = x0.clone()
        with torch.cuda.stream(side):  # eager run (also builds the cached tables)
            c.backbone_device(t, wl.gh, wl.gw, views, first, last, ALT, camera_dev=camera,
                              stream=side.cuda_stream)
        torch.cuda.synchronize()
        c.check_device()
        eager = t.clone()

        tg = x0.clone()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=side):
            c.backbone_device(tg, wl.gh, wl.gw, views, first, last, ALT, camera_dev=camera,
                              stream=side.cuda_stream)
        for _ in range(2):
            tg.copy_(x0)
            g.replay()
        torch.cuda.synchronize()
        c.check_device()
        assert torch.equal(tg, eager), float((tg - eager).abs().max())
        del g
    finally:
        c.close()
