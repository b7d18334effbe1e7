"""Query-sharded global attention on N GPUs (va_attention_device_sharded).

One child process per GPU; rank 0 creates the NCCL unique id and hands it to the
others through a multiprocessing queue, every rank then projects K'/V for its own
equal token slice, all-gathers them in place and attends its queries to the whole
window.  K'/V travel by copy-engine pushes with per-peer flags (the default when
every rank can map every peer's window and write its flags), by direct peer stores
from the QKV epilogue (VA_KV_EXCHANGE=sm), or by an NCCL all-gather
(VA_KV_EXCHANGE=nccl); all must give the same result.  The concatenated rank
outputs must match the single-GPU sub-block (same kernels; only the split of the
single launch's last wave rounds differently) and meet the oracle gates on a row
sample.
Skipped when fewer GPUs than ranks are visible.
"""
import multiprocessing as mp
import os
import queue

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")]

import synthetic as syn  # noqa: E402
import vestra_attn as va  # noqa: E402

LAYER = 5
WORKLOAD = "cfg3_s12_global"
TIMEOUT_S = 240


def _config(wl):
    return va.default_config(embed_dim=wl.embed, num_heads=wl.heads, num_register=wl.n_special - 1,
                             max_rows=wl.rows, depth=12, rope_start=4, qknorm_start=4)


def _rank_main(rank, nranks, exchange, ids, results):
    try:
        if exchange in ("nccl", "sm"):
            os.environ["VA_KV_EXCHANGE"] = exchange
        elif exchange == "ce":  # copy-engine push for every slice size
            os.environ["VA_KV_EXCHANGE"] = "ce"
        elif exchange == "parallel":  # copy-engine push, one stream per peer
            os.environ["VA_KV_EXCHANGE"] = "ce"
            os.environ["VA_PUSH_ORDER"] = "parallel"
        elif exchange.startswith("chunks"):  # copy-engine push in that many chunks per peer
            os.environ["VA_KV_EXCHANGE"] = "ce"
            os.environ["VA_PUSH_CHUNKS"] = exchange[len("chunks"):]
        torch.cuda.set_device(rank)
        wl = syn.CONFIGS[WORKLOAD]
        row0, local = va.shard_rows(wl.rows, nranks, rank)
        ctx = va.Context(_config(wl), rank)
        ctx.load_layer(LAYER, syn.layer_weights(wl.embed, seed=3, layer=LAYER, bias=True, perturb_norm=True))
        if rank == 0:
            uid = va.comm_unique_id()
            for _ in range(nranks - 1):
                ids.put(uid)
        else:
            uid = ids.get(timeout=TIMEOUT_S / 2)
        ctx.comm_init(uid, nranks, rank)
        mode = ctx.exchange_mode()
        x = syn.hidden_states(wl.rows, wl.embed, seed=3)[row0:row0 + local]
        ln1 = torch.from_numpy(np.ascontiguousarray(x)).cuda()
        out = torch.empty_like(ln1)
        # Three calls: the direct exchange alternates between two window pairs, so the
        # third call reuses the first call's pair on every rank.
        outs = []
        for _ in range(3):
            ctx.attention_device_sharded(LAYER, ln1, out, wl.gh, wl.gw, wl.views, True, stream=0)
            torch.cuda.synchronize()
            outs.append(out.cpu().numpy())
        ctx.check_device()
        same = all(np.array_equal(outs[0], o) for o in outs[1:])
        # The host-buffer entry (chunked copies, same exchange) gives the same rows.
        host = ctx.attention_host_sharded(LAYER, np.ascontiguousarray(x), wl.gh, wl.gw, wl.views, True)
        host_diff = float(np.abs(host - outs[-1]).max())
        status = "ok" if same and host_diff <= 2e-3 else f"calls differ (host {host_diff:.2e}, same {same})"
        results.put((rank, status, (mode, outs[-1])))
        ctx.close()
    except Exception as e:  # reported to the parent, which fails the test
        results.put((rank, f"error: {e!r}", None))


# "default": the copy-engine push (one stream, peers in reading order) where every
# rank can write a peer's flag by a stream memory operation and a peer gets 12 MB or
# more, else the epilogue's peer stores; "ce": the push for every size; "parallel" /
# "chunks1" / "chunks5": the push on one stream per peer / in 1 or 5 chunks per
# peer; "sm": forced epilogue stores + flag kernel; "nccl": forced all-gather.
EXPECTED_MODE = {"default": ("direct-ce", "direct"), "ce": ("direct-ce", "direct"),
                 "parallel": ("direct-ce", "direct"), "chunks1": ("direct-ce", "direct"),
                 "chunks5": ("direct-ce", "direct"), "sm": ("direct",), "nccl": ("nccl",)}


@pytest.mark.parametrize("exchange", ["default", "ce", "parallel", "chunks1", "chunks5", "sm", "nccl"])
@pytest.mark.parametrize("nranks", [2, 4, 8])
def test_sharded_global_attention_matches_single_gpu(oracle_mod, nranks, exchange):
    if torch.cuda.device_count() < nranks:
        pytest.skip(f"needs {nranks} GPUs")
    wl = syn.CONFIGS[WORKLOAD]
    mpc = mp.get_context("spawn")
    ids, results = mpc.Queue(), mpc.Queue()
    procs = [mpc.Process(target=_rank_main, args=(r, nranks, exchange, ids, results)) for r in range(nranks)]
    for p in procs:
        p.start()
    outs = {}
    try:
        for _ in range(nranks):
            rank, status, payload = results.get(timeout=TIMEOUT_S)
            assert status == "ok", f"rank {rank}: {status}"
            mode, outs[rank] = payload
            assert mode in EXPECTED_MODE[exchange], f"rank {rank} exchanged K'/V by {mode}"

    except queue.Empty:
        pytest.fail("a rank did not report within the time limit")
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    sharded = np.concatenate([outs[r] for r in range(nranks)], axis=0)

    # Single GPU, same inputs and weights.
    ctx = va.Context(_config(wl), 0)
    p = syn.layer_weights(wl.embed, seed=3, layer=LAYER, bias=True, perturb_norm=True)
    ctx.load_layer(LAYER, p)
    x = syn.hidden_states(wl.rows, wl.embed, seed=3)
    single = ctx.attention_host(LAYER, x, wl.gh, wl.gw, wl.views, True)
    ctx.close()
    # A rank's query slice is attended in one launch without a split key range; the
    # single-GPU launch splits the key range of its partial last wave, so the two
    # agree to rounding (bitwise wherever neither splits).
    assert float(np.abs(sharded - single).max()) <= 2e-3, float(np.abs(sharded - single).max())

    rows = np.sort(np.random.default_rng(nranks).choice(wl.rows, 96, replace=False)).astype(np.int64)
    pos = va.positions_yx(wl.rows, wl.views, wl.n_special, wl.gh, wl.gw, True)
    ref = oracle_mod.attention_block(x, p, wl.heads, pos_yx=pos, seg_len=0, q_rows=rows)
    got = sharded[rows]
    err = float(np.abs(got - ref).max())
    a, b = got.astype(np.float64).ravel(), ref.astype(np.float64).ravel()
    cos = float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))
    assert err <= 2e-2 and cos >= 0.9999, (err, cos)


def _block_rank_main(rank, nranks, ids, results):
    try:
        torch.cuda.set_device(rank)
        wl = syn.CONFIGS[WORKLOAD]
        row0, local = va.shard_rows(wl.rows, nranks, rank)
        ctx = va.Context(_config(wl), rank)
        p = syn.layer_weights(wl.embed, seed=8, layer=LAYER, norm1=True, mlp=True, ls1=True, ls2=True)
        ctx.load_layer(LAYER, p)
        ctx.load_mlp(LAYER, p)
        if rank == 0:
            uid = va.comm_unique_id()
            for _ in range(nranks - 1):
                ids.put(uid)
        else:
            uid = ids.get(timeout=TIMEOUT_S / 2)
        ctx.comm_init(uid, nranks, rank)
        x = syn.hidden_states(wl.rows, wl.embed, seed=8)[row0:row0 + local]
        t = torch.from_numpy(np.ascontiguousarray(x)).cuda()
        ctx.block_device_sharded(LAYER, t, wl.gh, wl.gw, wl.views, True, stream=0)
        torch.cuda.synchronize()
        ctx.check_device()
        results.put((rank, "ok", t.cpu().numpy()))
        ctx.close()
    except Exception as e:  # reported to the parent, which fails the test
        results.put((rank, f"error: {e!r}", None))


def test_sharded_whole_block_matches_single_gpu():
    # The device-resident tail over a query-sharded window: attention with the K'/V
    # exchange, then the token-local LN2/MLP on every rank's slice.
    nranks = 2
    if torch.cuda.device_count() < nranks:
        pytest.skip(f"needs {nranks} GPUs")
    wl = syn.CONFIGS[WORKLOAD]
    mpc = mp.get_context("spawn")
    ids, results = mpc.Queue(), mpc.Queue()
    procs = [mpc.Process(target=_block_rank_main, args=(r, nranks, ids, results)) for r in range(nranks)]
    for pr in procs:
        pr.start()
    outs = {}
    try:
        for _ in range(nranks):
            rank, status, arr = results.get(timeout=TIMEOUT_S)
            assert status == "ok", f"rank {rank}: {status}"
            outs[rank] = arr
    except queue.Empty:
        pytest.fail("a rank did not report within the time limit")
    finally:
        for pr in procs:
            pr.join(timeout=60)
            if pr.is_alive():
                pr.kill()
    sharded = np.concatenate([outs[r] for r in range(nranks)], axis=0)
    ctx = va.Context(_config(wl), 0)
    p = syn.layer_weights(wl.embed, seed=8, layer=LAYER, norm1=True, mlp=True, ls1=True, ls2=True)
    ctx.load_layer(LAYER, p)
    ctx.load_mlp(LAYER, p)
    t = torch.from_numpy(syn.hidden_states(wl.rows, wl.embed, seed=8)).cuda()
    ctx.block_device(LAYER, t, wl.gh, wl.gw, wl.views, True)
    torch.cuda.synchronize()
    single = t.cpu().numpy()
    ctx.close()
    assert float(np.abs(sharded - single).max()) <= 2e-3, float(np.abs(sharded - single).max())


def _route_rank_main(rank, nranks, ids, results):
    try:
        torch.cuda.set_device(rank)
        wl = syn.Workload("s3_global", 768, 12, 3, 36, 24, 2, True)
        n = wl.rows // wl.views
        row0, local = va.shard_views(wl.views, n, nranks, rank)
        ctx = va.Context(_config(wl), rank)
        for layer in range(3, 7):
            p = syn.layer_weights(wl.embed, seed=9, layer=layer, norm1=True, mlp=True)
            ctx.load_layer(layer, p)
            ctx.load_mlp(layer, p)
        ctx.load_vit_norm(np.ones(wl.embed, np.float32), np.zeros(wl.embed, np.float32))
        if rank == 0:
            uid = va.comm_unique_id()
            for _ in range(nranks - 1):
                ids.put(uid)
        else:
            uid = ids.get(timeout=TIMEOUT_S / 2)
        ctx.comm_init(uid, nranks, rank)
        x = syn.hidden_states(wl.rows, wl.embed, seed=9)[row0:row0 + local]
        t = torch.from_numpy(np.ascontiguousarray(x)).cuda()
        cam = torch.from_numpy(syn.camera_tokens(wl.embed, seed=9)).cuda()
        caps = ctx.backbone_device_sharded(t, row0, wl.rows, wl.gh, wl.gw, wl.views, 3, 7, 4, camera_dev=cam,
                                           out_layers=(4, 5))
        torch.cuda.synchronize()
        ctx.check_device()
        results.put((rank, "ok", (t.cpu().numpy(), {k: (v[0].cpu().numpy(), v[1].cpu().numpy())
                                                    for k, v in caps.items()})))
        ctx.close()
    except Exception as e:  # reported to the parent, which fails the test
        results.put((rank, f"error: {e!r}", None))


def test_sharded_backbone_route_uneven_views_matches_single_gpu():
    # Three views on two GPUs (2 + 1 whole views): local blocks run on each rank's
    # own views, the global block exchanges K'/V between uneven slices.
    nranks = 2
    if torch.cuda.device_count() < nranks:
        pytest.skip(f"needs {nranks} GPUs")
    wl = syn.Workload("s3_global", 768, 12, 3, 36, 24, 2, True)
    mpc = mp.get_context("spawn")
    ids, results = mpc.Queue(), mpc.Queue()
    procs = [mpc.Process(target=_route_rank_main, args=(r, nranks, ids, results)) for r in range(nranks)]
    for pr in procs:
        pr.start()
    outs = {}
    try:
        for _ in range(nranks):
            rank, status, payload = results.get(timeout=TIMEOUT_S)
            assert status == "ok", f"rank {rank}: {status}"
            outs[rank] = payload
    except queue.Empty:
        pytest.fail("a rank did not report within the time limit")
    finally:
        for pr in procs:
            pr.join(timeout=60)
            if pr.is_alive():
                pr.kill()
    ctx = va.Context(_config(wl), 0)
    for layer in range(3, 7):
        p = syn.layer_weights(wl.embed, seed=9, layer=layer, norm1=True, mlp=True)
        ctx.load_layer(layer, p)
        ctx.load_mlp(layer, p)
    ctx.load_vit_norm(np.ones(wl.embed, np.float32), np.zeros(wl.embed, np.float32))
    t = torch.from_numpy(syn.hidden_states(wl.rows, wl.embed, seed=9)).cuda()
    cam = torch.from_numpy(syn.camera_tokens(wl.embed, seed=9)).cuda()
    caps = ctx.backbone_device(t, wl.gh, wl.gw, wl.views, 3, 7, 4, camera_dev=cam, out_layers=(4, 5))
    torch.cuda.synchronize()
    single = t.cpu().numpy()
    sharded = np.concatenate([outs[r][0] for r in range(nranks)], axis=0)

    # Rank 0's attention launches split their last wave over key ranges and the
    # single launch does not, so the two agree to rounding that four blocks carry
    # forward: the parity gates apply (a wrong slot or view order would be O(1)).
    def gate(got, ref, what):
        got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
        err = float(np.abs(got - ref).max())
        cos = float(got.ravel() @ ref.ravel() / (np.linalg.norm(got) * np.linalg.norm(ref)))
        assert err <= 2e-2 and cos >= 0.9999, f"{what}: max-abs {err:.3e} cos {cos:.7f}"

    gate(sharded, single, "tokens")
    for layer in (4, 5):
        for i, what in enumerate(("feat", "cam")):
            got = np.concatenate([outs[r][1][layer][i] for r in range(nranks)], axis=0)
            gate(got, caps[layer][i].cpu().numpy(), f"{what} capture {layer}")
    ctx.close()
