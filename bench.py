#!/usr/bin/env python
"""Benchmark of the B200 attention path of the DA3 ViT backbone (Vestra Engine).

Metric: global-attention TFLOP/s at S=12 views (504x336, 866 tokens
per view, 10,392-token window, E=768, 12 heads x 64), FLOPs = 4 * N^2 * d * heads.
A step is one global attention sub-block over the whole window: LN1 output (F32,
resident in HBM) -> QKV UMMA with QK-norm/RoPE epilogue -> fused flash attention ->
output projection (F32).  With --gpus N > 1 the window's queries are split into N
equal token slices (one process per GPU); each rank's K'/V rows reach the peers'
windows over NVLink by copy engines, and the attention kernel waits on per-peer flags
(epilogue peer stores, or an NCCL all-gather, where that is unavailable).
The line also reports one whole block (attention + LN2/MLP) under "block", the
12-block window under "window", the token input side (patch projection and
position/CLS assembly of every view) under "tokens", and the load of a Q8_0 model
file into the device operands under "gguf".

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints one JSON line on rank 0.  `value` is device-timed (CUDA events around each
step on the launching stream, L2 flushed between steps, max over ranks); `e2e`
goes through the public host API with pinned host buffers and the H2D/D2H copies
inside the timed region.  `--impl reference` times the CPU F32 restatement of the
reference attention (oracle/, the reference itself cannot be built here) on the
host cores, on the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "vestra-engine_b200"))

import synthetic as syn  # noqa: E402

LAYER = 5           # a global block of the DA3-BASE schedule (alt_start 4: globals 5,7,9,11)
L2_FLUSH_BYTES = 256 << 20
# dram__bytes_read.sum + dram__bytes_write.sum of one launch of the default
# fixed-offset attention kernel (flash_fwd_d64_ks_kernel<72, split, quadratic>) on
# the cfg3 window at one GPU, from one ncu capture of that kernel (47.95 MB read:
# Q + K + V once; 2.87 MB written, O mostly still in L2 when the launch ends; the
# capture is `ncu ... -k regex:flash_fwd_d64_ks python bench.py --ncu-case flash`).  Used
# for the roofline's `traffic` at N = 1; a rank's launch at N > 1 reads the whole
# key window but only its own queries, so the figure does not carry over.
FLASH_DRAM_BYTES_PER_LAUNCH = {"cfg3_s12_global": 50.82e6}
PARITY_ROWS = 256   # seeded output rows checked against the oracle at every N
MAX_ABS, MIN_COS = 2e-2, 0.9999


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="cfg3_s12_global", choices=sorted(syn.CONFIGS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--variants", action="store_true",
                    help="also time the attention kernel's exponential-split and f16-P variants")
    ap.add_argument("--no-large", action="store_true", help="skip the DA3-LARGE S=32 window section")
    ap.add_argument("--ncu-case", choices=NCU_CASES, default=None,
                    help="run one small case of a kernel family a few times and exit (for a profiler)")
    return ap.parse_args()


def cpu_threads():
    """Host threads this process may run on (the oracle is given this count
    explicitly, so a launcher's OMP_NUM_THREADS=1 does not apply)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


NCU_CASES = ("subblock", "block", "fc2", "tokens", "capture", "gguf", "flash", "flash_slice8", "flash_local")


def run_ncu_case(name):
    """One small case of a kernel family on cuda:0 at the cfg3 shapes, run a few times
    (the profiler skips the first launches): subblock / block (LN1, QKV, attention,
    proj / + LN2, fc1, fc2), fc2 (the K3 GEMM at fc2's K = 3072, residual in place as in
    a block), tokens (patchify +
    patch projection), capture (two capture launches), gguf (device decoding of a
    2-block Q8_0 file), flash (the default fixed-offset attention launch over the
    window), flash_slice8 (one rank's 1,299 queries of 8 against the window) and
    flash_local (local attention over the window's 12 views of 866 tokens)."""
    import numpy as np
    import torch
    import vestra_attn as va

    wl = syn.CONFIGS["cfg3_s12_global"]
    E = wl.embed
    ctx = va.Context(va.default_config(max_rows=wl.rows, depth=12, rope_start=4, qknorm_start=4,
                                       num_register=1), 0)
    x = torch.from_numpy(syn.hidden_states(wl.rows, E, seed=0)).cuda()
    if name in ("subblock", "block", "capture"):
        for layer in (4, LAYER):
            p = syn.layer_weights(E, seed=0, layer=layer, norm1=True, mlp=True)
            ctx.load_layer(layer, p)
            ctx.load_mlp(layer, p)
        if name == "capture":
            ctx.load_vit_norm(np.ones(E, np.float32), np.zeros(E, np.float32))
            ctx.backbone_device(x.clone(), wl.gh, wl.gw, wl.views, 4, 6, 4, out_layers=(4, 5), cat_token=True)
        else:
            out = torch.empty_like(x)
            for _ in range(3):
                if name == "subblock":
                    ctx.attention_device(LAYER, x, out, wl.gh, wl.gw, wl.views, True)
                else:
                    ctx.block_device(LAYER, x.clone(), wl.gh, wl.gw, wl.views, True)
    elif name == "fc2":
        h = torch.randn(wl.rows, 4 * E, device="cuda").to(torch.bfloat16)
        w = (0.02 * torch.randn(E, 4 * E, device="cuda")).to(torch.bfloat16)
        out = x.clone()
        for _ in range(3):
            ctx.linear_bf16(h, w, out, bias=torch.zeros(E, device="cuda"), residual=out)
    elif name == "tokens":
        pw = syn.patch_embed_weights(E, 14, 37, 1, seed=0)
        ctx.load_patch_embed(pw["weight"], pw["bias"], pw["cls"], pw["pos_embed"], pw["registers"], 14)
        imgs = torch.from_numpy(syn.images(wl.views, wl.gh * 14, wl.gw * 14, seed=0)).cuda()
        tk = torch.empty(wl.rows, E, device="cuda")
        for _ in range(3):
            ctx.prepare_tokens_device(imgs, wl.views, wl.gh * 14, wl.gw * 14, tk)
    elif name == "gguf":
        data = syn.gguf_model(embed=E, depth=2, heads=wl.heads, grid=37, dtype="q8_0", seed=0)
        with tempfile.TemporaryDirectory() as d:
            path = os.path.join(d, "m.gguf")
            with open(path, "wb") as f:
                f.write(data)
            with va.GgufFile(path) as g:
                c2 = va.Context(va.default_config(embed_dim=E, num_heads=wl.heads, depth=2, max_rows=1024), 0)
                c2.load_gguf(g)
                c2.close()
    else:
        g = torch.Generator(device="cuda").manual_seed(0)

        def hn(t):
            return torch.nn.functional.layer_norm(t.view(t.shape[0], wl.heads, 64), (64,)).view(t.shape[0], -1)

        local = wl.rows // 8 if name == "flash_slice8" else wl.rows
        seg = wl.rows // wl.views if name == "flash_local" else 0
        q = hn(torch.randn(local, E, device="cuda", generator=g)).to(torch.bfloat16)
        k = hn(torch.randn(wl.rows, E, device="cuda", generator=g)).to(torch.bfloat16)
        v = torch.randn(wl.rows, E, device="cuda", generator=g).to(torch.bfloat16)
        o = torch.empty_like(q)
        for _ in range(3):
            ctx.flash_bf16(q, k, v, wl.heads, o, q_offset=wl.rows - local, seg_len=seg, variant=511)
    torch.cuda.synchronize()
    ctx.check_device()
    ctx.close()
    return 0


def dist_env():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return p["bf16_tflops"], p.get("hbm_gbs"), "measured"
    return 1590.0, 6650.0, "fallback"


def cpu_info():
    """Model name, logical CPU count and AVX-512 feature flags of the host."""
    model, flags = "", []
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name") and not model:
                    model = line.split(":", 1)[1].strip()
                elif line.startswith("flags") and not flags:
                    flags = sorted(x for x in line.split(":", 1)[1].split() if x.startswith("avx512"))
    except OSError:
        pass
    return f"{model}; nproc {os.cpu_count()}; {' '.join(flags) or 'no avx512'}"


# --------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi sampled every 200 ms while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.dev = device_index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(prefix="va_clocks_", suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.dev), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if self.proc is None or not self.path or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9 and parts[1].isdigit():
                    rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [int(r[1]) for r in rows]
        mx = max(int(r[2]) for r in rows)
        loaded = [s for s, r in zip(sm, rows) if float(r[3] or 0) > 200.0] or sm
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": int(statistics.median(loaded)), "sm_max_mhz": mx, "reasons": reasons,
                "samples": len(rows), "power_w_max": max(float(r[3] or 0) for r in rows)}


# --------------------------------------------------------------------------- CPU baseline
def cpu_attention_full(wl, reps, threads, warmup=1):
    """Times the CPU F32 restatement (oracle/) of the attention sub-block over the
    whole window (every query row, no extrapolation) on `threads` host threads;
    returns the per-run seconds."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    import vestra_attn as va

    oracle.build()
    x = syn.hidden_states(wl.rows, wl.embed, seed=0)
    p = syn.layer_weights(wl.embed, seed=0, layer=LAYER)
    pos = va.positions_yx(wl.rows, wl.views, wl.n_special, wl.gh, wl.gw, wl.global_)
    seg = 0 if wl.global_ else wl.seg_len
    for _ in range(warmup):
        oracle.attention_block(x, p, wl.heads, pos_yx=pos, seg_len=seg, threads=threads)
    times = []
    for _ in range(reps):
        t = time.perf_counter()
        oracle.attention_block(x, p, wl.heads, pos_yx=pos, seg_len=seg, threads=threads)
        times.append(time.perf_counter() - t)
    return times


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    wl = syn.CONFIGS[args.workload]
    threads = cpu_threads()
    # Every step is the whole window: each query row, the full K/V projection, the
    # output projection, on all host threads (about half a second at cfg3).
    times = cpu_attention_full(wl, args.steps, threads, warmup=args.warmup)
    total = sum(times)
    value = wl.attention_flops() / (total / args.steps) / 1e12
    sample = f"the full window ({wl.rows} query rows) every step, {threads} threads"
    line = {
        "impl": "reference", "metric": "global-attention TFLOP/s", "value": round(value, 4),
        "unit": "TFLOP/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(total / args.steps * 1e3, 3),
        "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded N(0,1) tokens, N(0,0.02) weights)",
        "config": workload_config(wl, args.gpus),
        "cpu_baseline": {"value": round(value, 4), "unit": "TFLOP/s", "cores": threads, "kind": "port",
                         "sample": sample, "cpu": cpu_info()},
        "e2e": {"value": round(value, 4), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "CPU F32 restatement of the reference attention (vestra-kernels is un-vendored and no Rust "
                "toolchain exists, so the reference binary cannot be built); rank 0 alone runs it",
    }
    print(json.dumps(line), file=JSON_OUT, flush=True)
    return 0


def workload_config(wl, n_gpus):
    return {
        "workload": wl.name, "views": wl.views, "tokens_per_view": wl.tokens_per_view, "window_tokens": wl.rows,
        "embed": wl.embed, "heads": wl.heads, "head_dim": 64, "global": wl.global_,
        "step": "one attention sub-block: LN1 out -> QKV (+QK-norm, 2D RoPE) -> flash attention -> proj",
        "flops_per_step": wl.attention_flops(),
        "l2": f"flushed between timed steps ({L2_FLUSH_BYTES >> 20} MiB write)",
        "parallelism": "single GPU" if n_gpus == 1 else
        f"query-sharded window over {n_gpus} GPUs; K'/V rows exchanged directly over NVLink (copy-engine "
        "push with per-peer flags, or QKV-epilogue peer stores), NCCL all-gather as the fallback",
    }


# --------------------------------------------------------------------------- parity
def parity_rows(rows, n, seed):
    """Seeded sorted sample of n window rows (every row when the window is smaller)."""
    import numpy as np
    if n >= rows:
        return np.arange(rows, dtype=np.int64)
    return np.sort(np.random.default_rng(seed).choice(rows, n, replace=False)).astype(np.int64)


def parity_check(wl, p, x_all, out_local, row0, sel, world, rank, seg_len=0):
    """Compares a seeded sample of output rows, gathered from every rank, with the
    oracle (CPU F32 restatement) on rank 0.  Collective; returns the same dict on
    every rank: {rows, max_abs, cos, ok}."""
    import numpy as np
    import torch
    import torch.distributed as dist

    local = out_local.shape[0]
    mine = sel[(sel >= row0) & (sel < row0 + local)]
    got = out_local[torch.from_numpy(mine - row0).to(out_local.device)].float().cpu().numpy()
    parts = [(mine, got)]
    if world > 1:
        parts = [None] * world
        dist.all_gather_object(parts, (mine, got))
    res = None
    if rank == 0:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle
        import vestra_attn as va

        oracle.build()
        idx = np.concatenate([a for a, _ in parts])
        val = np.concatenate([b for _, b in parts])
        order = np.argsort(idx)
        idx, val = idx[order], val[order]
        pos = va.positions_yx(wl.rows, wl.views, wl.n_special, wl.gh, wl.gw, wl.global_)
        ref = oracle.attention_block(x_all, p, wl.heads, pos_yx=pos, seg_len=seg_len, q_rows=idx,
                                     threads=cpu_threads())
        a, b = val.astype(np.float64), ref.astype(np.float64)
        err = float(np.abs(a - b).max()) if np.isfinite(a).all() else float("inf")
        cos = float((a.ravel() @ b.ravel()) / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-300))
        res = {"rows": int(len(idx)), "max_abs": err, "cos": round(cos, 8),
               "ok": bool(len(idx) == len(sel) and err <= MAX_ABS and cos >= MIN_COS)}
    if world > 1:
        box = [res]
        dist.broadcast_object_list(box, src=0)
        res = box[0]
    return res


# --------------------------------------------------------------------------- cfg5
def run_large(args, world, rank, local_rank, barrier, max_over_ranks, flush_buf, stream):
    """The DA3-LARGE S=32 window (E=1024, 16 heads, 110,656 tokens): one global
    attention sub-block, query-sharded over the run's GPUs with the same exchange as
    the metric's window, timed with CUDA events (max over ranks), and an oracle
    check of a seeded row sample."""
    import numpy as np
    import torch
    import torch.distributed as dist
    import vestra_attn as va

    wl = syn.CONFIGS["cfg5_large_s32_global"]
    row0, local = va.shard_rows(wl.rows, world, rank)
    cfg = va.default_config(embed_dim=wl.embed, num_heads=wl.heads, num_register=wl.n_special - 1,
                            max_rows=wl.rows, depth=24, rope_start=4, qknorm_start=4)
    ctx = va.Context(cfg, local_rank)
    p = syn.layer_weights(wl.embed, seed=0, layer=LAYER)
    ctx.load_layer(LAYER, p)
    if world > 1:
        obj = [va.comm_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        ctx.comm_init(obj[0], world, rank)
    x_all = syn.hidden_states(wl.rows, wl.embed, seed=0)
    ln1 = torch.from_numpy(np.ascontiguousarray(x_all[row0:row0 + local])).cuda()
    out = torch.empty_like(ln1)
    sp = stream.cuda_stream

    def step():
        if world == 1:
            ctx.attention_device(LAYER, ln1, out, wl.gh, wl.gw, wl.views, True, stream=sp)
        else:
            ctx.attention_device_sharded(LAYER, ln1, out, wl.gh, wl.gw, wl.views, True, stream=sp)

    for _ in range(2):
        step()
    barrier()
    ctx.check_device()
    evs = []
    for _ in range(3):
        flush_buf.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        step()
        b.record(stream)
        evs.append((a, b))
    barrier()
    ctx.check_device()
    ms = max_over_ranks(statistics.mean(a.elapsed_time(b) for a, b in evs))
    ctx.set_phase_profile(True)
    flush_buf.zero_()
    step()
    core = ctx.phase_times()["core"]
    ctx.set_phase_profile(False)
    barrier()
    flops = wl.attention_flops()
    peak, _, kind = load_peaks()
    my_flops = 4.0 * local * wl.rows * 64 * wl.heads
    par = parity_check(wl, p, x_all, out, row0, parity_rows(wl.rows, 64, 9), world, rank)
    ctx.close()
    tf = flops / (ms * 1e-3) / 1e12
    return {"workload": wl.name, "window_tokens": wl.rows, "embed": wl.embed, "heads": wl.heads,
            "attention_flops": flops, "ms": round(ms, 3), "tflops": round(tf, 1),
            "frac_of_n_peaks": round(tf / (world * peak), 4),
            "core_ms_rank0": round(core, 3), "kernel_tflops_rank0": round(my_flops / (core * 1e-3) / 1e12, 1),
            "parity": par,
            "what": "one global attention sub-block of the S=32 DA3-LARGE window (LN1 out -> QKV -> attention "
                    f"-> proj), query-sharded over {world} GPU(s); frac against {world} x the measured bf16 "
                    f"peak ({kind})"}


# --------------------------------------------------------------------------- ours
def run_ours(args):
    import numpy as np
    import torch
    import torch.distributed as dist
    import vestra_attn as va

    rank, world, local_rank = dist_env()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE {world}")
    torch.cuda.set_device(local_rank)
    if world > 1:
        from datetime import timedelta
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=timedelta(seconds=180),
                                device_id=torch.device("cuda", local_rank))
    wl = syn.CONFIGS[args.workload]
    if not wl.global_ and world > 1:
        raise SystemExit("the benchmark shards global blocks only")
    row0, local = va.shard_rows(wl.rows, world, rank)
    cfg = va.default_config(embed_dim=wl.embed, num_heads=wl.heads, num_register=wl.n_special - 1,
                            max_rows=wl.rows, depth=12, rope_start=4, qknorm_start=4)
    ctx = va.Context(cfg, local_rank)
    ctx.load_layer(LAYER, syn.layer_weights(wl.embed, seed=0, layer=LAYER))
    if world > 1:
        obj = [va.comm_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        ctx.comm_init(obj[0], world, rank)

    x_all = syn.hidden_states(wl.rows, wl.embed, seed=0)
    x_local = np.ascontiguousarray(x_all[row0:row0 + local])
    ln1 = torch.from_numpy(x_local).cuda()
    out = torch.empty_like(ln1)
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream
    flush_buf = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device="cuda")

    def step():
        if world == 1:
            ctx.attention_device(LAYER, ln1, out, wl.gh, wl.gw, wl.views, wl.global_, stream=sp)
        else:
            ctx.attention_device_sharded(LAYER, ln1, out, wl.gh, wl.gw, wl.views, wl.global_, stream=sp)

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(args.warmup):
        flush_buf.zero_()
        step()
    barrier()
    ctx.check_device()

    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    with ClockSampler(local_rank) as clocks:
        barrier()
        for i in range(args.steps):
            flush_buf.zero_()
            starts[i].record(stream)
            step()
            ends[i].record(stream)
        barrier()
    ctx.check_device()
    step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    total_ms = max_over_ranks(sum(step_ms))
    ms_per_step = total_ms / args.steps
    flops = wl.attention_flops()
    value = flops / (ms_per_step * 1e-3) / 1e12

    # ---- per-phase times of the same step (CUDA events between its launches),
    # the reference's phase names; outside the timed region above.
    ctx.set_phase_profile(True)
    phase_runs, xchg_runs = [], []
    mode = ctx.exchange_mode() if world > 1 else "single GPU"
    for _ in range(max(3, min(args.steps, 10))):
        flush_buf.zero_()
        step()
        phase_runs.append(ctx.phase_times())
        if world > 1:
            xchg_runs.append((ctx.last_exchange(), ctx.exchange_times()))
    ctx.set_phase_profile(False)
    barrier()
    phases = {k: round(statistics.median(r[k] for r in phase_runs), 4) for k in phase_runs[0]}
    local_rows = local
    gemm_tflops = {
        "qkv": round(2.0 * local_rows * wl.embed * 3 * wl.embed / (phases["qkv"] * 1e-3) / 1e12, 1),
        "proj": round(2.0 * local_rows * wl.embed * wl.embed / (phases["proj"] * 1e-3) / 1e12, 1),
    }
    ln_gbs = round(local_rows * wl.embed * 6 / (phases["ln"] * 1e-3) / 1e9, 1)  # F32 read + bf16 write
    exchange = None
    if world > 1:
        used = xchg_runs[-1][0]
        exchange = {"mode": mode, "path": {"direct": "QKV-epilogue peer stores + per-peer flags",
                                           "direct-ce": "copy-engine push + per-peer flags",
                                           "nccl": "NCCL all-gather"}.get(used, used)}
        pushes = [r[1] for r in xchg_runs if r[1][0]]
        if pushes:
            npeer = len(pushes[0][0])
            per_peer = [statistics.median(r[0][i] for r in pushes) for i in range(npeer)]
            nbytes = pushes[0][1]
            exchange.update({
                "bytes_per_peer": nbytes,
                "per_peer_ms": [round(v, 4) for v in per_peer],
                "per_peer_gbs": [round(nbytes / (v * 1e-3) / 1e9, 1) for v in per_peer],
                "push_ms": round(max(per_peer), 4),
                "out_gbs": round(nbytes * npeer / (max(per_peer) * 1e-3) / 1e9, 1),
                "what": "this rank's K'/V rows pushed to every peer by copy engines: CUDA events around each "
                        "peer's copies and flag writes on its copy stream, median of the profiled steps "
                        "(rank 0's view); out_gbs = all bytes sent / the slowest peer's push"})

    # ---- parity of this N's output against the oracle: a seeded sample of output
    # rows gathered from every rank, outside the timed region.  Exits non-zero (after
    # the line is printed) when the gates fail.
    p_metric = syn.layer_weights(wl.embed, seed=0, layer=LAYER)
    parity = parity_check(wl, p_metric, x_all, out, row0, parity_rows(wl.rows, PARITY_ROWS, 7), world, rank)
    parity["gate"] = f"max-abs <= {MAX_ABS}, cos >= {MIN_COS}"
    parity["vs"] = "oracle (CPU F32 restatement), rows gathered from every rank"

    # ---- one whole block (device-resident tail: attention + LN2/MLP, residuals),
    # reported beside the metric; tokens restored from a copy before every run.
    pb = syn.layer_weights(wl.embed, seed=0, layer=LAYER, norm1=True, mlp=True)
    ctx.load_layer(LAYER, pb)
    ctx.load_mlp(LAYER, pb)
    tok0 = ln1.clone()
    tok = torch.empty_like(tok0)
    block_ms = []
    for i in range(args.warmup + args.steps):
        flush_buf.zero_()
        tok.copy_(tok0)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        if world == 1:
            ctx.block_device(LAYER, tok, wl.gh, wl.gw, wl.views, wl.global_, stream=sp)
        else:
            ctx.block_device_sharded(LAYER, tok, wl.gh, wl.gw, wl.views, wl.global_, stream=sp)
        b.record(stream)
        if i >= args.warmup:
            block_ms.append((a, b))
    barrier()
    ctx.check_device()
    block_ms = max_over_ranks(statistics.mean(a.elapsed_time(b) for a, b in block_ms))
    mlp_flops = 16.0 * wl.rows * wl.embed * wl.embed
    block = {"ms": round(block_ms, 4), "mlp_flops": mlp_flops,
             "tflops_incl_mlp": round((flops + mlp_flops) / (block_ms * 1e-3) / 1e12, 1),
             "what": "x += attention(LN1 x); x += fc2(GELU(fc1(LN2 x))) on device, one block"}
    # ---- the whole 12-block stack of one window (DA3-BASE schedule: alt_start 4,
    # global blocks 5/7/9/11, the others local).  With N GPUs every rank holds whole
    # views (12 on 8: 2,2,2,2,1,1,1,1): local blocks need no communication, global
    # blocks exchange K'/V between the uneven slices.
    window = None
    n_tok = wl.rows // wl.views
    if wl.views >= world and (world == 1 or ctx.exchange_mode().startswith("direct")):
        for layer in range(12):
            pl = syn.layer_weights(wl.embed, seed=0, layer=layer, norm1=True, mlp=True)
            ctx.load_layer(layer, pl)
            ctx.load_mlp(layer, pl)
        v0, vrows = va.shard_views(wl.views, n_tok, world, rank)
        xw = torch.from_numpy(np.ascontiguousarray(x_all[v0:v0 + vrows])).cuda()
        tw = torch.empty_like(xw)
        win_ms = []
        for i in range(max(3, args.warmup) + max(3, args.steps // 2)):
            flush_buf.zero_()
            tw.copy_(xw)
            barrier()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            ctx.backbone_device_sharded(tw, v0, wl.rows, wl.gh, wl.gw, wl.views, 0, 12, 4, stream=sp)
            b.record(stream)
            if i >= max(3, args.warmup):
                win_ms.append((a, b))
        barrier()
        ctx.check_device()
        win_ms = max_over_ranks(statistics.mean(a.elapsed_time(b) for a, b in win_ms))
        attn_win = 4 * flops + 8 * 4.0 * wl.views * n_tok * n_tok * 64 * wl.heads
        window = {"ms": round(win_ms, 3), "blocks": 12, "global_blocks": [5, 7, 9, 11],
                  "attention_flops": attn_win, "attention_tflops": round(attn_win / (win_ms * 1e-3) / 1e12, 1),
                  "views_per_rank": [va.shard_views(wl.views, n_tok, world, r)[1] // n_tok for r in range(world)],
                  "what": f"12 whole blocks (attention + MLP) of the S={wl.views} window on device, "
                          "va_backbone_device_sharded (max over ranks)"}
        if world == 1:
            # The same window captured once into a CUDA graph and replayed: what the
            # route costs without host-side launch work.
            gs = torch.cuda.Stream()
            gs.wait_stream(stream)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=gs):
                ctx.backbone_device_sharded(tw, v0, wl.rows, wl.gh, wl.gw, wl.views, 0, 12, 4,
                                            stream=gs.cuda_stream)
            graph_ms = []
            for i in range(3 + max(3, args.steps // 2)):
                flush_buf.zero_()
                tw.copy_(xw)
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                graph.replay()
                b.record(stream)
                if i >= 3:
                    graph_ms.append((a, b))
            torch.cuda.synchronize()
            ctx.check_device()
            window["graph_ms"] = round(statistics.mean(a.elapsed_time(b) for a, b in graph_ms), 3)
            del graph
    ctx.load_layer(LAYER, syn.layer_weights(wl.embed, seed=0, layer=LAYER))  # back to the metric's weights

    # ---- local blocks (cfg4: the same 12 views, each attending to itself): this
    # rank's whole views, no communication; the attention kernel's time from the
    # phase profile.
    local_section = None
    n_tok = wl.rows // wl.views
    if wl.views >= world:
        v0, vrows = va.shard_views(wl.views, n_tok, world, rank)
        lv = vrows // n_tok
        xl = torch.from_numpy(np.ascontiguousarray(x_all[v0:v0 + vrows])).cuda()
        ol = torch.empty_like(xl)

        def lstep():
            ctx.attention_device(LAYER, xl, ol, wl.gh, wl.gw, lv, False, stream=sp)

        for _ in range(3):
            lstep()
        barrier()
        lms, lcore = [], []
        ctx.set_phase_profile(True)
        for _ in range(max(3, args.steps // 2)):
            flush_buf.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            lstep()
            b.record(stream)
            lms.append((a, b))
            lcore.append(ctx.phase_times()["core"])
        ctx.set_phase_profile(False)
        barrier()
        ctx.check_device()
        l_ms = max_over_ranks(statistics.mean(a.elapsed_time(b) for a, b in lms))
        l_core = max_over_ranks(statistics.median(lcore))
        l_flops = 4.0 * wl.views * n_tok * n_tok * 64 * wl.heads
        my_flops = 4.0 * lv * n_tok * n_tok * 64 * wl.heads
        peak_t, _, _ = load_peaks()
        wl_local = syn.CONFIGS["cfg4_s12_local"]  # the same views with per-view positions
        lpar = parity_check(wl_local, p_metric, x_all, ol, v0, parity_rows(wl.rows, PARITY_ROWS, 8), world, rank,
                            seg_len=n_tok)
        local_section = {
            "workload": "cfg4 local blocks (12 x 866-token views, block-diagonal attention)",
            "ms": round(l_ms, 4), "attention_flops": l_flops,
            "tflops": round(l_flops / (l_ms * 1e-3) / 1e12, 1),
            "core_ms_rank0": round(statistics.median(lcore), 4),
            "kernel_tflops_rank0": round(my_flops / (statistics.median(lcore) * 1e-3) / 1e12, 1),
            "kernel_frac_rank0": round(my_flops / (statistics.median(lcore) * 1e-3) / 1e12 / peak_t, 4),
            "views_per_rank": [va.shard_views(wl.views, n_tok, world, r)[1] // n_tok for r in range(world)],
            "parity": lpar,
            "what": "one local attention sub-block over this rank's whole views (max over ranks); kernel = "
                    "the attention launch alone (phase profile), rank 0's views"}
        del xl, ol

    # ---- the DA3-LARGE S=32 window (cfg5: E=1024, 16 heads, 110,656 tokens),
    # query-sharded over the run's GPUs exactly like the metric's window.
    large = None
    if not args.no_large:
        large = run_large(args, world, rank, local_rank, barrier, max_over_ranks, flush_buf, stream)

    # ---- token input side: this rank's views of 504x336 images -> tokens (patch
    # projection GEMM + position/CLS/register assembly), no communication.
    pw = syn.patch_embed_weights(wl.embed, 14, 37, wl.n_special - 1, seed=0)
    ctx.load_patch_embed(pw["weight"], pw["bias"], pw["cls"], pw["pos_embed"], pw["registers"], 14)
    v0, vrows = va.shard_views(wl.views, n_tok, world, rank)
    my_views = vrows // n_tok
    img_h, img_w = wl.gh * 14, wl.gw * 14
    imgs = torch.from_numpy(syn.images(my_views, img_h, img_w, seed=rank)).cuda()
    tk_out = torch.empty(vrows, wl.embed, device="cuda")
    ctx.prepare_tokens_device(imgs, my_views, img_h, img_w, tk_out, stream=sp)  # builds the cached table
    tok_ms = []
    for i in range(args.warmup + args.steps):
        flush_buf.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        ctx.prepare_tokens_device(imgs, my_views, img_h, img_w, tk_out, stream=sp)
        b.record(stream)
        if i >= args.warmup:
            tok_ms.append((a, b))
    barrier()
    ctx.check_device()
    tok_ms = max_over_ranks(statistics.mean(a.elapsed_time(b) for a, b in tok_ms))
    patches = wl.views * wl.gh * wl.gw
    # image F32 read + token F32 write (+ the bf16 patch rows written and read back)
    tok_bytes = wl.views * 3 * img_h * img_w * 4 + wl.rows * wl.embed * 4 + 2 * patches * 640 * 2
    tokens = {"ms": round(tok_ms, 4), "bytes": tok_bytes,
              "gbs": round(tok_bytes / (tok_ms * 1e-3) / 1e9, 1),
              "gemm_tflops": round(2.0 * patches * 588 * wl.embed / (tok_ms * 1e-3) / 1e12, 1),
              "what": "prepare_tokens of every view on device: patchify -> tcgen05 projection with "
                      "bias + position epilogue -> CLS/register rows (max over ranks)"}

    # ---- dominant kernel alone (K2), same shapes, CUDA events on its stream
    # Q/K: every 64-wide head row LayerNormed (gamma 1, beta 0), as the QK-norm leaves
    # them, so |q|, |k| <= 8 and |q.k| / 8 * log2(e) <= 11.6: the kernel runs with the
    # fixed exponent offset the layer path selects for such rows (variant + 256); the
    # row-max form is timed beside it.  V bf16 (production path).
    g = torch.Generator(device="cuda").manual_seed(rank)

    def head_norm(x):
        x = x.view(x.shape[0], wl.heads, 64)
        return torch.nn.functional.layer_norm(x, (64,), eps=1e-5).view(x.shape[0], -1)

    q = head_norm(torch.randn(local, wl.embed, device="cuda", generator=g)).to(torch.bfloat16)
    kw = head_norm(torch.randn(wl.rows, wl.embed, device="cuda", generator=g)).to(torch.bfloat16)
    vw = (0.5 * torch.randn(wl.rows, wl.embed, device="cuda", generator=g)).to(torch.bfloat16)
    FIXED = 511  # fixed exponent offset with the library's default layout (see va_flash_attention_bf16)
    o = torch.empty(local, wl.embed, device="cuda", dtype=torch.bfloat16)

    def time_flash(v_tensor, poly=-1):
        for _ in range(3):
            ctx.flash_bf16(q, kw, v_tensor, wl.heads, o, q_offset=row0, stream=sp, variant=poly)
        evs = []
        barrier()
        for _ in range(args.steps):
            flush_buf.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            ctx.flash_bf16(q, kw, v_tensor, wl.heads, o, q_offset=row0, stream=sp, variant=poly)
            b.record(stream)
            evs.append((a, b))
        barrier()
        ctx.check_device()
        return statistics.mean(a.elapsed_time(b) for a, b in evs)

    flash_flops = 4.0 * local * wl.rows * 64 * wl.heads
    flash_ms = time_flash(vw, FIXED)
    rowmax_ms = time_flash(vw)
    w20_fixed_ms = time_flash(vw, 256 + 24)  # the four-threads-per-row layout with the fixed offset
    variants = {}
    if args.variants:
        to_tf = lambda ms: round(flash_flops / (ms * 1e-3) / 1e12, 2)  # noqa: E731
        for form in (0, 2, 3, 5, 6, 7):
            for p in range(3):
                name = {3: f"w20_poly{p}", 5: f"w20ord_poly{p}", 6: f"w20nosplit_poly{p}",
                        7: f"w20splitp_poly{p}"}.get(form, f"form{form}_poly{p}")
                variants[name] = to_tf(time_flash(vw, p + 8 * form))
        for p in range(3):
            variants[f"w20fixed_poly{p}"] = to_tf(time_flash(vw, 256 + 24 + p))
            variants[f"w20fixed_nosplit_poly{p}"] = to_tf(time_flash(vw, 256 + 48 + p))
        variants["w20half_poly0"] = to_tf(time_flash(vw, 64))
        for form, name in ((9, "ks_cubic"), (10, "ks_quad"), (11, "ks_cubic_turns"), (12, "ks_quad_turns")):
            for i in range(5):
                variants[f"{name}_ka{64 + 8 * i}"] = to_tf(time_flash(vw, 256 + 8 * form + i))
        variants["f16_p"] = to_tf(time_flash(vw.to(torch.float16)))
    peak_tflops, _, peak_kind = load_peaks()
    achieved = flash_flops / (flash_ms * 1e-3) / 1e12

    # ---- end to end through the public API, pinned host buffers, copies timed
    h_in = torch.from_numpy(x_local).pin_memory()
    h_out = torch.empty_like(h_in).pin_memory()
    if world == 1:
        def e2e_step():
            ctx.attention_host(LAYER, h_in, wl.gh, wl.gw, wl.views, wl.global_, out=h_out)
    else:
        def e2e_step():
            ctx.attention_host_sharded(LAYER, h_in, wl.gh, wl.gw, wl.views, wl.global_, out=h_out)
    for _ in range(max(1, args.warmup)):
        e2e_step()
    barrier()
    e2e_s = 0.0
    for _ in range(args.steps):
        flush_buf.zero_()
        torch.cuda.synchronize()
        t = time.perf_counter()
        e2e_step()
        e2e_s += time.perf_counter() - t
    barrier()
    e2e_s = max_over_ranks(e2e_s)
    # The same bytes over PCIe with nothing else running: the H2D of the step's input
    # and the D2H of its output, one after the other (a global block's outputs all
    # depend on its last input row, so this sum bounds e2e from below).
    d_in = torch.empty(h_in.shape, dtype=h_in.dtype, device="cuda")
    h_tmp = torch.empty_like(h_in).pin_memory()  # h_out keeps the e2e result checked below
    copy_ms = []
    for _ in range(3 + args.steps):
        ca, cb, cc = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        ca.record(stream)
        d_in.copy_(h_in, non_blocking=True)
        cb.record(stream)
        h_tmp.copy_(d_in, non_blocking=True)
        cc.record(stream)
        cc.synchronize()
        copy_ms.append((ca.elapsed_time(cb), cb.elapsed_time(cc)))
    copy_ms = copy_ms[3:]
    h2d_ms = max_over_ranks(statistics.median(c[0] for c in copy_ms))
    d2h_ms = max_over_ranks(statistics.median(c[1] for c in copy_ms))
    # Both directions at once (the floor of a pipelined batch): one step's input in
    # and another buffer's output back on two streams, timed from a common start.
    d_out = torch.empty_like(d_in)
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
    duplex = []
    for _ in range(3 + args.steps):
        ca, cb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ca.record(stream)
        s_in.wait_stream(stream)
        s_out.wait_stream(stream)
        with torch.cuda.stream(s_in):
            d_in.copy_(h_in, non_blocking=True)
        with torch.cuda.stream(s_out):
            h_tmp.copy_(d_out, non_blocking=True)
        stream.wait_stream(s_in)
        stream.wait_stream(s_out)
        cb.record(stream)
        cb.synchronize()
        duplex.append(ca.elapsed_time(cb))
    duplex_ms = max_over_ranks(statistics.median(duplex[3:]))
    del d_in, h_tmp, d_out
    e2e_value = flops / (e2e_s / args.steps) / 1e12
    # parity of the host path against the device path on this input.  The host path
    # attends its queries in wave-sized chunks, the device path in one launch whose
    # partial last wave is split over key ranges, so the two agree to rounding.
    # The difference is reduced over ranks first, so every rank takes the same exit.
    e2e_diff = float(np.abs(out.cpu().numpy() - h_out.numpy()).max())
    e2e_diff = max_over_ranks(e2e_diff if np.isfinite(e2e_diff) else 1e30)
    if e2e_diff > 2e-2:
        raise SystemExit(f"e2e output differs from the device-path output (max abs {e2e_diff})")
    # The same steps as independent requests through va_attention_host_batch: step
    # s+1's copy in runs beside step s's attention and copy out (both PCIe directions
    # at once).  One GPU; two pinned input and output buffers, alternating.
    pipelined = None
    if world == 1:
        h_ins = [h_in, torch.from_numpy(x_local.copy()).pin_memory()]
        h_outs = [torch.empty_like(h_in).pin_memory() for _ in range(2)]
        ins = [h_ins[s % 2] for s in range(args.steps)]
        outs = [h_outs[s % 2] for s in range(args.steps)]
        ctx.attention_host_batch(LAYER, ins[:2], outs[:2], wl.gh, wl.gw, wl.views, wl.global_)  # warm-up
        flush_buf.zero_()
        torch.cuda.synchronize()
        t = time.perf_counter()
        ctx.attention_host_batch(LAYER, ins, outs, wl.gh, wl.gw, wl.views, wl.global_)
        pipe_s = time.perf_counter() - t
        pipe_diff = max(float(np.abs(o.numpy() - h_out.numpy()).max()) for o in h_outs)
        if not pipe_diff == 0.0:
            raise SystemExit(f"pipelined host batch differs from va_attention_host (max abs {pipe_diff})")
        pipelined = {"value": round(flops / (pipe_s / args.steps) / 1e12, 3), "unit": "TFLOP/s",
                     "ms_per_step": round(pipe_s / args.steps * 1e3, 4),
                     "h2d_bytes_per_step": int(wl.rows * wl.embed * 4),
                     "d2h_bytes_per_step": int(wl.rows * wl.embed * 4),
                     "path": "va_attention_host_batch (C ABI, K independent steps in one call, pinned host "
                             "in/out; outputs bitwise equal to va_attention_host)"}
        del h_ins, h_outs, ins, outs

    # ---- model file: a 12-block DA3 GGUF of this width (Q8_0 linear weights, F32
    # vectors, the patch embedding) read and converted into a fresh context's device
    # operands by va_load_model_gguf (host wall clock, median; one GPU only).
    gguf_section = None
    if world == 1:
        import tempfile
        data = syn.gguf_model(embed=wl.embed, depth=12, heads=wl.heads, grid=37, dtype="q8_0", seed=0)
        gctx = va.Context(va.default_config(embed_dim=wl.embed, num_heads=wl.heads, depth=12, max_rows=1024), 0)
        with tempfile.TemporaryDirectory() as d:
            path = os.path.join(d, "model.gguf")
            with open(path, "wb") as f:
                f.write(data)
            load_ms, sent = [], 0
            with va.GgufFile(path) as gf:
                for _ in range(4):
                    t0 = time.perf_counter()
                    sent = gctx.load_gguf(gf)
                    load_ms.append((time.perf_counter() - t0) * 1e3)
        gctx.close()
        load_ms = statistics.median(load_ms[1:])
        gguf_section = {"ms": round(load_ms, 2), "file_bytes": len(data), "stored_bytes": sent,
                        "gbs": round(sent / (load_ms * 1e-3) / 1e9, 2),
                        "what": "va_load_model_gguf of a 12-block Q8_0 model file of this width (page-cache "
                                "resident): stored bytes -> pinned staging -> H2D -> device decode into the "
                                "bf16/F32 operands; host wall clock, median of 3 after one warm-up"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = cpu_threads()
        times = cpu_attention_full(wl, 3, threads)
        cpu = {"value": round(wl.attention_flops() / statistics.median(times) / 1e12, 4), "unit": "TFLOP/s",
               "cores": threads, "kind": "port", "ms_per_step": round(statistics.median(times) * 1e3, 1),
               "sample": f"the full window ({wl.rows} query rows), median of 3 after one warm-up",
               "cpu": cpu_info()}

    # The kernel this rank's launch ran, from the library's own launch plan.
    sms = torch.cuda.get_device_properties(local_rank).multi_processor_count
    flash_kernel = va.flash_plan(local, wl.rows, wl.heads, q_offset=row0, sms=sms)["kernel"]
    if rank == 0:
        line = {
            "metric": "global-attention TFLOP/s", "value": round(value, 3), "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
            "ms_per_window_layer": round(ms_per_step, 4),
            "pct_of_bf16_peak": round(100.0 * value / peak_tflops, 2),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic (seeded N(0,1) tokens, N(0,0.02) weights, QK-norm gamma 1 beta 0)",
            "config": workload_config(wl, world),
            "roofline": {"bound": "tensor", "kernel": flash_kernel, "achieved": round(achieved, 2),
                         "peak": peak_tflops, "unit": "TFLOP/s", "frac": round(achieved / peak_tflops, 4),
                         "peak_kind": f"bf16 burst ({peak_kind})", "flops_per_launch": flash_flops,
                         "ms_per_launch": round(flash_ms, 4),
                         "softmax": "fixed exponent offset (scores bounded by the QK-norm); keys split between "
                                    "MUFU and FMA-pipe warps (72 of every 128 on MUFU)",
                         "rowmax_tflops": round(flash_flops / (rowmax_ms * 1e-3) / 1e12, 2),
                         "w20_fixed_tflops": round(flash_flops / (w20_fixed_ms * 1e-3) / 1e12, 2),
                         **({"variants_tflops": variants} if variants else {}),
                         "traffic": FLASH_DRAM_BYTES_PER_LAUNCH.get(args.workload) if world == 1 else None},
            "e2e": {"value": round(e2e_value, 3), "unit": "TFLOP/s", "ms_per_step": round(e2e_s / args.steps * 1e3, 4),
                    "h2d_bytes_per_step": int(wl.rows * wl.embed * 4), "d2h_bytes_per_step": int(wl.rows * wl.embed * 4),
                    "path": "va_attention_host (C ABI, pinned host in/out)" if world == 1 else
                    "va_attention_host_sharded (C ABI, pinned host in/out, per rank)",
                    "max_abs_vs_device_path": e2e_diff,
                    "pcie_floor_ms": {"h2d": round(h2d_ms, 4), "d2h": round(d2h_ms, 4),
                                      "sum": round(h2d_ms + d2h_ms, 4),
                                      "duplex": round(duplex_ms, 4),
                                      "h2d_gbs": round(h_in.numel() * 4 / (h2d_ms * 1e-3) / 1e9, 1),
                                      "d2h_gbs": round(h_in.numel() * 4 / (d2h_ms * 1e-3) / 1e9, 1),
                                      "what": "the step's input H2D then its output D2H alone, per rank "
                                              "(median); a global block's outputs need its last input row; "
                                              "duplex: both copies at once on two streams (the floor of the "
                                              "pipelined batch)"},
                    "pipelined": pipelined},
            "phases_ms": phases, "gemm_tflops": gemm_tflops, "ln_cast_gbs": ln_gbs, "block": block, "window": window, "tokens": tokens,
            "gguf": gguf_section,
            "gpu_launches": (5 if world > 1 and xchg_runs[-1][0] == "direct" else 4) * args.steps,
            "parity": parity, "exchange": exchange, "local": local_section, "large": large,
            "clocks": clocks.summary(),
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), file=JSON_OUT, flush=True)
    ctx.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    failed = [n for n, sec in (("metric", parity), ("local", (local_section or {}).get("parity")),
                               ("large", (large or {}).get("parity"))) if sec is not None and not sec["ok"]]
    if failed:
        print(f"parity gates failed: {failed}", file=sys.stderr)
        return 1
    return 0


JSON_OUT = sys.stdout


def main():
    global JSON_OUT
    args = parse_args()
    # The result line is the only thing on the process's stdout: file descriptor 1
    # is pointed at stderr for everything else (NCCL's version banner, any print of
    # the libraries), and the line goes to a duplicate of the original stdout.
    sys.stdout.flush()
    JSON_OUT = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    if args.ncu_case:
        return run_ncu_case(args.ncu_case)
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
