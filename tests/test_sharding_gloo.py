"""Query-sharded global attention, decomposition checked on CPU ranks (gloo).

The sharded path (va_attention_device_sharded) gives each rank an equal,
contiguous token slice of the window (shard_rows); a rank projects Q'/K'/V for its
own rows, all-gathers K'/V in rank order and attends its queries to the whole
window.  Two gloo ranks replay exactly that decomposition with the CPU
restatement's pieces and must reproduce the one-process attention sub-block.
No GPU is touched.
"""
import multiprocessing as mp
import os
import queue
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")

import synthetic as syn  # noqa: E402
import vestra_attn as va  # noqa: E402

WL = syn.Workload("gloo_s2", 256, 4, 2, 4, 6, 2, True)  # 2 views x 26 tokens, 4 heads x 64
NRANKS = 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _heads(t, rows):
    return np.ascontiguousarray(t.reshape(rows, WL.heads, 64).transpose(1, 0, 2))


def _rank_main(rank, port, results):
    import torch.distributed as dist
    from datetime import timedelta
    import oracle

    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=NRANKS, timeout=timedelta(seconds=60))
        E = WL.embed
        row0, local = va.shard_rows(WL.rows, NRANKS, rank)
        p = syn.layer_weights(E, seed=4, layer=6, bias=True, ls1=True, perturb_norm=True)
        x = syn.hidden_states(WL.rows, E, seed=4)[row0:row0 + local]
        pos = va.positions_yx(WL.rows, WL.views, WL.n_special, WL.gh, WL.gw, True)[row0:row0 + local]
        qkv = oracle.linear(x, p["qkv_w"], p["qkv_b"])
        q = oracle.rope2d(oracle.layernorm(_heads(qkv[:, :E], local), p["q_g"], p["q_b"], 1e-5), pos)
        k = oracle.rope2d(oracle.layernorm(_heads(qkv[:, E:2 * E], local), p["k_g"], p["k_b"], 1e-5), pos)
        v = _heads(qkv[:, 2 * E:], local)
        # K'/V all-gather in rank order -> the whole window, [heads, rows, 64].
        kg = [torch.empty_like(torch.from_numpy(k)) for _ in range(NRANKS)]
        vg = [torch.empty_like(torch.from_numpy(v)) for _ in range(NRANKS)]
        dist.all_gather(kg, torch.from_numpy(k))
        dist.all_gather(vg, torch.from_numpy(v))
        kw = torch.cat(kg, dim=1).double().numpy()
        vw = torch.cat(vg, dim=1).double().numpy()
        s = np.einsum("hqd,hkd->hqk", q.astype(np.float64), kw) / 8.0
        s = np.exp(s - s.max(-1, keepdims=True))
        a = np.einsum("hqk,hkd->hqd", s / s.sum(-1, keepdims=True), vw)
        attn = a.transpose(1, 0, 2).reshape(local, E).astype(np.float32)
        out = oracle.linear(attn, p["proj_w"], p["proj_b"], scale=p["ls1"])
        og = [torch.empty(local, E) for _ in range(NRANKS)]
        dist.all_gather(og, torch.from_numpy(out))
        results.put((rank, "ok", torch.cat(og).numpy()))
        dist.destroy_process_group()
    except Exception as e:  # reported to the parent, which fails the test
        results.put((rank, f"error: {e!r}", None))


def test_two_rank_decomposition_matches_single_process(oracle_mod):
    mpc = mp.get_context("spawn")
    results = mpc.Queue()
    port = _free_port()
    procs = [mpc.Process(target=_rank_main, args=(r, port, results)) for r in range(NRANKS)]
    for pr in procs:
        pr.start()
    outs = {}
    try:
        for _ in range(NRANKS):
            rank, status, arr = results.get(timeout=180)
            assert status == "ok", f"rank {rank}: {status}"
            outs[rank] = arr
    except queue.Empty:
        pytest.fail("a gloo rank did not report within the time limit")
    finally:
        for pr in procs:
            pr.join(timeout=60)
            if pr.is_alive():
                pr.kill()
    p = syn.layer_weights(WL.embed, seed=4, layer=6, bias=True, ls1=True, perturb_norm=True)
    x = syn.hidden_states(WL.rows, WL.embed, seed=4)
    pos = va.positions_yx(WL.rows, WL.views, WL.n_special, WL.gh, WL.gw, True)
    ref = oracle_mod.attention_block(x, p, WL.heads, pos_yx=pos, seg_len=0)
    for r in range(NRANKS):  # every rank ends with the same gathered window output
        assert np.abs(outs[r] - ref).max() <= 1e-5, (r, float(np.abs(outs[r] - ref).max()))
    assert np.array_equal(outs[0], outs[1])


def test_shard_rows_refuses_unequal_slices():
    with pytest.raises(ValueError):
        va.shard_rows(10392, 5, 0)
    spans = [va.shard_rows(10392, 8, r) for r in range(8)]
    assert [s[0] for s in spans] == [1299 * r for r in range(8)] and all(s[1] == 1299 for s in spans)
