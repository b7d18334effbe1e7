"""ctypes front end of the CPU F32 restatement in oracle.cpp.

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py, always as the checker or the timed CPU baseline.
The product path (vestra-engine_b200/) never imports this module.

Each function names the reference code it restates (paths are inside the
vestra-engine project).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "liboracle.so")
_lib = None

_f32p = ctypes.POINTER(ctypes.c_float)
_f64p = ctypes.POINTER(ctypes.c_double)
_i64p = ctypes.POINTER(ctypes.c_int64)


def build() -> str:
    """Compiles oracle.cpp with the Makefile beside it (idempotent)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def _load():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(_LIB_PATH):
        build()
    lib = ctypes.CDLL(_LIB_PATH)
    c_i64, c_int, c_float = ctypes.c_int64, ctypes.c_int, ctypes.c_float
    lib.oracle_has_avx512.restype = c_int
    lib.oracle_positions.argtypes = [c_i64, c_int, c_int, c_int, c_int, c_int, _f32p]
    lib.oracle_layernorm.argtypes = [_f32p, c_i64, c_int, _f32p, _f32p, c_float, c_int]
    lib.oracle_rope2d.argtypes = [_f32p, c_int, c_i64, c_int, _f32p, c_float, c_int, c_int]
    lib.oracle_linear.argtypes = [_f32p, c_i64, c_int, _f32p, c_int, _f32p, _f32p, _f32p, c_int]
    lib.oracle_attention_core.argtypes = [_f32p, _f32p, _f32p, c_int, c_i64, c_int, c_i64, _f32p, c_int]
    lib.oracle_op_attention.argtypes = [_f32p, _f32p, _f32p, c_int, c_i64, c_int, _f32p, _f32p, _f32p,
                                        _f32p, c_float, _f32p, c_float, c_int, _f32p, c_int]
    lib.oracle_attention_block.argtypes = [_f32p, c_i64, c_int, c_int, c_int, _f32p, _f32p, _f32p, _f32p,
                                           _f32p, _f32p, c_float, _f32p, c_float, c_int, c_i64, _f32p,
                                           _f32p, _f32p, _i64p, c_i64, _f32p, c_int]
    lib.oracle_attention_block.restype = c_int
    lib.oracle_attention_naive_f64.argtypes = [_f64p, _f64p, _f64p, c_int, c_i64, c_int, c_i64, _f64p]
    lib.oracle_mlp_block.argtypes = [_f32p, c_i64, c_int, c_int, _f32p, _f32p, c_float, _f32p, _f32p,
                                     _f32p, _f32p, _f32p, _f32p, c_int]
    _lib = lib
    return lib


def _p(a):
    if a is None:
        return None
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(_f32p)


def _f32(a):
    return None if a is None else np.ascontiguousarray(a, dtype=np.float32)


def has_avx512() -> bool:
    return bool(_load().oracle_has_avx512())


def positions(rows, view_count, n_special, gh, gw, global_):
    """RoPE position table, vit_block.rs:841-881."""
    out = np.zeros((rows, 2), np.float32)
    _load().oracle_positions(rows, view_count, n_special, gh, gw, int(bool(global_)), _p(out))
    return out


def layernorm(x, gamma, beta, eps, threads=0):
    """Row LayerNorm (torch semantics), vit_block.rs:696-714."""
    x = np.array(x, dtype=np.float32, order="C", copy=True)
    rows, cols = x.reshape(-1, x.shape[-1]).shape
    _load().oracle_layernorm(_p(x), rows, cols, _p(_f32(gamma)), _p(_f32(beta)), eps, threads)
    return x


def rope2d(x, pos_yx, freq=100.0, pairing=0, threads=0):
    """2D RoPE on [heads, n, d] in a copy (vestra_kernels::rope2d, vit_block.rs:944-948)."""
    x = np.array(x, dtype=np.float32, order="C", copy=True)
    heads, n, d = x.shape
    _load().oracle_rope2d(_p(x), heads, n, d, _p(_f32(pos_yx)), freq, pairing, threads)
    return x


def linear(a, w, bias=None, scale=None, threads=0):
    """a[M,K] @ w[K,N] + bias, * scale (run_linear, vit_block.rs:721-761)."""
    a, w = _f32(a), _f32(w)
    m, k = a.shape
    n = w.shape[1]
    out = np.zeros((m, n), np.float32)
    _load().oracle_linear(_p(a), m, k, _p(w), n, _p(_f32(bias)), _p(_f32(scale)), _p(out), threads)
    return out


def attention_core(q, k, v, seg_len=0, threads=0):
    """softmax(q k^T / sqrt(d)) v per head over segments of seg_len tokens."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    heads, n, d = q.shape
    out = np.zeros_like(q)
    _load().oracle_attention_core(_p(q), _p(k), _p(v), heads, n, d, seg_len, _p(out), threads)
    return out


def op_attention(q, k, v, qnorm=None, knorm=None, qk_norm_eps=1e-5, rope=None, pairing=0, threads=0):
    """Op::Attention (graph.rs:67-105, cpu_backend.rs:198-298).

    qnorm/knorm: (gamma, beta) or None.  rope: (pos_yx [n,2], freq) or None.
    """
    q, k, v = _f32(q), _f32(k), _f32(v)
    heads, n, d = q.shape
    out = np.zeros_like(q)
    qg, qb = (None, None) if qnorm is None else (_f32(qnorm[0]), _f32(qnorm[1]))
    kg, kb = (None, None) if knorm is None else (_f32(knorm[0]), _f32(knorm[1]))
    pos, freq = (None, 100.0) if rope is None else (_f32(rope[0]), float(rope[1]))
    _load().oracle_op_attention(_p(q), _p(k), _p(v), heads, n, d, _p(qg), _p(qb), _p(kg), _p(kb),
                                qk_norm_eps, _p(pos), freq, pairing, _p(out), threads)
    return out


def attention_block(ln1, layer, heads, pos_yx=None, seg_len=0, rope_freq=100.0, qk_norm_eps=1e-5,
                    use_qknorm=True, pairing=0, q_rows=None, threads=0):
    """Attention sub-block of one ViT block (vit_block.rs:772-992) -> [rows, E] branch.

    layer: dict with qkv_w [E,3E], qkv_b [3E], q_g, q_b, k_g, k_b [d], proj_w [E,E],
    proj_b [E], optional ls1 [E] (the reference's [in,out] orientation).
    """
    ln1 = _f32(ln1)
    rows, e = ln1.shape
    d = e // heads
    nq = rows if q_rows is None else len(q_rows)
    out = np.zeros((nq, e), np.float32)
    qr = None if q_rows is None else np.ascontiguousarray(q_rows, dtype=np.int64)
    g = (lambda name: _f32(layer.get(name))) if use_qknorm else (lambda name: None)
    rc = _load().oracle_attention_block(
        _p(ln1), rows, e, heads, d, _p(_f32(layer["qkv_w"])), _p(_f32(layer["qkv_b"])),
        _p(g("q_g")), _p(g("q_b")), _p(g("k_g")), _p(g("k_b")), qk_norm_eps,
        _p(_f32(pos_yx)), rope_freq, pairing, seg_len,
        _p(_f32(layer["proj_w"])), _p(_f32(layer["proj_b"])), _p(_f32(layer.get("ls1"))),
        None if qr is None else qr.ctypes.data_as(_i64p), nq, _p(out), threads)
    if rc != 0:
        raise ValueError("oracle_attention_block: shape error")
    return out


def mlp_block(x, layer, ln_eps=1e-6, threads=0):
    """MLP sub-block + residual (vit_block.rs:1092-1129): x + (GELU_erf(LN2(x) fc1) fc2) * ls2.

    layer: dict with norm2_w, norm2_b [E], fc1_w [E,H], fc1_b [H], fc2_w [H,E], fc2_b [E],
    optional ls2 [E] ([in,out] orientation)."""
    x = _f32(x)
    rows, E = x.shape
    hidden = layer["fc1_w"].shape[1]
    out = np.zeros_like(x)
    _load().oracle_mlp_block(_p(x), rows, E, hidden, _p(_f32(layer["norm2_w"])), _p(_f32(layer["norm2_b"])),
                             ln_eps, _p(_f32(layer["fc1_w"])), _p(_f32(layer["fc1_b"])), _p(_f32(layer["fc2_w"])),
                             _p(_f32(layer["fc2_b"])), _p(_f32(layer.get("ls2"))), _p(out), threads)
    return out


def block(x, layer, heads, pos_yx=None, seg_len=0, ln_eps=1e-6, rope_freq=100.0, qk_norm_eps=1e-5,
          use_qknorm=True, pairing=0, threads=0):
    """One whole ViT block (vit_block.rs:1019-1139): x += attention(LN1(x)); x += MLP(x)."""
    x = _f32(x)
    ln1 = layernorm(x, layer["norm1_w"], layer["norm1_b"], ln_eps, threads)
    x1 = x + attention_block(ln1, layer, heads, pos_yx=pos_yx, seg_len=seg_len, rope_freq=rope_freq,
                             qk_norm_eps=qk_norm_eps, use_qknorm=use_qknorm, pairing=pairing, threads=threads)
    return mlp_block(x1, layer, ln_eps, threads)


def attention_naive_f64(q, k, v, seg_len=0):
    q, k, v = (np.ascontiguousarray(a, dtype=np.float64) for a in (q, k, v))
    heads, n, d = q.shape
    out = np.zeros_like(q)
    _load().oracle_attention_naive_f64(q.ctypes.data_as(_f64p), k.ctypes.data_as(_f64p),
                                       v.ctypes.data_as(_f64p), heads, n, d, seg_len,
                                       out.ctypes.data_as(_f64p))
    return out
