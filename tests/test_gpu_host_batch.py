"""va_attention_host_batch: several independent same-shape host inputs through one
pipelined call give exactly the outputs of one va_attention_host call each (global
and local blocks).  Every call goes through the C ABI."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")]

import synthetic as syn  # noqa: E402
import vestra_attn as va  # noqa: E402


@pytest.mark.parametrize("name", ["cfg2_s2_global", "cfg3_s12_global", "cfg4_s12_local"])
def test_batch_equals_separate_calls(name):
    wl = syn.CONFIGS[name]
    ctx = va.Context(va.default_config(max_rows=wl.rows, num_register=wl.n_special - 1), 0)
    try:
        ctx.load_layer(5, syn.layer_weights(wl.embed, seed=4, layer=5, ls1=True, perturb_norm=True, bias=True))
        xs = [torch.from_numpy(syn.hidden_states(wl.rows, wl.embed, seed=10 + s)).pin_memory() for s in range(3)]
        outs = [torch.full_like(x, float("nan")).pin_memory() for x in xs]
        ctx.attention_host_batch(5, xs, outs, wl.gh, wl.gw, wl.views, wl.global_)
        for x, y in zip(xs, outs):
            ref = ctx.attention_host(5, x.numpy(), wl.gh, wl.gw, wl.views, wl.global_)
            assert np.isfinite(ref).all()
            assert y.numpy().tobytes() == ref.tobytes()
        ctx.attention_host_batch(5, xs[:1], outs[:1], wl.gh, wl.gw, wl.views, wl.global_)  # one step
        ctx.check_device()
    finally:
        ctx.close()
