"""The bench's multi-GPU parity check on two CPU ranks (gloo): every rank holds its
slice of the window's output, a seeded sample of rows is gathered from all ranks
and compared with the oracle on rank 0, and every rank gets the same verdict.  A
wrong row on one rank must fail the check everywhere.  No GPU is touched."""
import multiprocessing as mp
import os
import queue
import socket
import sys

import numpy as np
import pytest

torch = pytest.importorskip("torch")

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import synthetic as syn  # noqa: E402

WL = syn.Workload("gloo_s2", 256, 4, 2, 4, 6, 2, True)  # 2 views x 26 tokens, 4 heads x 64
NRANKS = 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, port, plant, results):
    import torch.distributed as dist
    from datetime import timedelta

    import bench
    import oracle
    import vestra_attn as va

    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=NRANKS, timeout=timedelta(seconds=60))
        p = syn.layer_weights(WL.embed, seed=5, layer=5, perturb_norm=True)
        x = syn.hidden_states(WL.rows, WL.embed, seed=5)
        pos = va.positions_yx(WL.rows, WL.views, WL.n_special, WL.gh, WL.gw, True)
        full = oracle.attention_block(x, p, WL.heads, pos_yx=pos, seg_len=0)
        row0, local = va.shard_rows(WL.rows, NRANKS, rank)
        mine = torch.from_numpy(full[row0:row0 + local].copy())
        if plant and rank == 1:
            mine[3] += 0.5  # a wrong output row on one rank only
        res = bench.parity_check(WL, p, x, mine, row0, np.arange(WL.rows, dtype=np.int64), NRANKS, rank)
        results.put((rank, res))
        dist.destroy_process_group()
    except Exception as e:  # noqa: BLE001
        results.put((rank, repr(e)))


@pytest.mark.parametrize("plant", [False, True])
def test_parity_check_gathers_rows_from_every_rank(plant):
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, port, plant, results)) for r in range(NRANKS)]
    for pr in procs:
        pr.start()
    got = {}
    try:
        for _ in range(NRANKS):
            r, res = results.get(timeout=180)
            got[r] = res
    except queue.Empty:
        pytest.fail("a rank did not report")
    finally:
        for pr in procs:
            pr.join(timeout=30)
            if pr.is_alive():
                pr.kill()
    for r in range(NRANKS):
        assert isinstance(got[r], dict), got[r]
    assert got[0] == got[1]  # one verdict on every rank
    assert got[0]["rows"] == WL.rows
    if plant:
        assert not got[0]["ok"] and got[0]["max_abs"] >= 0.4
    else:
        assert got[0]["ok"] and got[0]["max_abs"] == 0.0 and got[0]["cos"] >= 0.99999999
