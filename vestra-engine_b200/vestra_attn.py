"""Host-side mirror of the reference's attention executor seams over libvestra_attn.so.

The reference (Rust) plugs device attention into its block loop through traits in
crates/da-engine/src/vit_block.rs; this module offers the same shapes of calls to
Python callers (tests, bench, smoke) through the C ABI in include/vestra_attn.h:

  CudaAttentionExecutor.run_attention   AttentionExecutor::run_attention (vit_block.rs:95-105)
  CudaAttentionExecutor.run_attention_views  run_attention with closed-form positions
                                        (vit_block.rs:841-881) for local/global blocks
  op_attention                          Op::Attention / GraphBuilder::attention_full
                                        (graph.rs:67-105, 394-422)
  select_reference_view_saddle, reference_first_order, restore_original_view_order
                                        backbone.rs:133-224, engine.rs:198-205

There is no CPU fallback: a missing library or a failing call raises.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_build", "libvestra_attn.so")

(VA_OK, VA_ERR_INVALID, VA_ERR_CUDA, VA_ERR_DEVICE, VA_ERR_STATE, VA_ERR_NCCL, VA_ERR_CAPACITY, VA_ERR_IO,
 VA_ERR_FORMAT, VA_ERR_NOT_FOUND, VA_ERR_DTYPE) = range(11)
# va_gguf metadata kinds (the MetaValue variants) and GGML tensor types
(META_U32, META_I32, META_F32, META_U64, META_BOOL, META_STR, META_ARR_U32, META_ARR_I32, META_ARR_F32,
 META_ARR_STR) = range(10)
GGML_F32, GGML_F16, GGML_Q8_0 = 0, 1, 8
NOALLOC_MAX_ELEMS = 1 << 21  # heads * n * 64 limit of va_op_attention_noalloc

# Every symbol include/vestra_attn.h declares (checked by tests/test_abi.py).
EXPORTED = [
    "va_version", "va_default_config", "va_create", "va_destroy", "va_last_error", "va_load_layer",
    "va_layer_flags", "va_run_attention", "va_attention_host", "va_attention_device",
    "va_block_attention_device", "va_op_attention_device", "va_flash_attention_bf16",
    "va_linear_bf16", "va_flash_plan", "va_select_reference_view_saddle", "va_reference_first_order",
    "va_restore_order", "va_camera_inject_device", "va_permute_views_device", "va_check_device",
    "va_selftest_bounded_wait", "va_set_phase_profile", "va_phase_times", "va_exchange_times", "va_last_exchange",
    "va_load_mlp", "va_block_device", "va_block_device_sharded", "va_run_tail_host",
    "va_load_vit_norm", "va_backbone_device", "va_backbone_device_sharded",
    "va_comm_unique_id", "va_comm_init", "va_comm_exchange_mode", "va_attention_device_sharded",
    "va_attention_host_sharded", "va_attention_host_batch",
    "va_op_attention_noalloc",
    "va_load_patch_embed", "va_prepare_tokens_device", "va_prepare_tokens_host", "va_pos_embed_device",
    "va_selftest_peer_wait",
    "va_gguf_open", "va_gguf_close", "va_gguf_last_error", "va_gguf_version", "va_gguf_meta_count",
    "va_gguf_meta_entry", "va_gguf_meta_u32", "va_gguf_meta_i32", "va_gguf_meta_f32", "va_gguf_meta_u64",
    "va_gguf_meta_bool", "va_gguf_meta_str", "va_gguf_meta_arr_u32", "va_gguf_meta_arr_i32",
    "va_gguf_meta_arr_f32", "va_gguf_meta_arr_str", "va_gguf_tensor_count", "va_gguf_tensor_name",
    "va_gguf_tensor_info", "va_gguf_tensor_check", "va_gguf_tensor_device", "va_gguf_tensor_f32",
    "va_gguf_model_config", "va_load_model_gguf",
]


class VestraError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"vestra_attn error {code}: {msg}")
        self.code = code


class VaConfig(ctypes.Structure):
    """va_config: the ModelConfig fields the attention path reads (config.rs:146)."""

    _fields_ = [
        ("embed_dim", ctypes.c_int32), ("num_heads", ctypes.c_int32), ("head_dim", ctypes.c_int32),
        ("depth", ctypes.c_int32), ("num_register", ctypes.c_int32), ("rope_start", ctypes.c_int32),
        ("qknorm_start", ctypes.c_int32), ("rope_freq", ctypes.c_float), ("ln_eps", ctypes.c_float),
        ("qk_norm_eps", ctypes.c_float), ("rope_pairing", ctypes.c_int32), ("max_rows", ctypes.c_int32),
    ]


class VaModelConfig(ctypes.Structure):
    """va_model_config: ModelConfig as ModelConfig::from_gguf reads it (config.rs:146-264)."""

    _fields_ = [
        ("arch", ctypes.c_char * 32),
        ("patch_size", ctypes.c_uint32), ("image_size", ctypes.c_uint32), ("embed_dim", ctypes.c_uint32),
        ("depth", ctypes.c_uint32), ("num_heads", ctypes.c_uint32), ("head_dim", ctypes.c_uint32),
        ("mlp_hidden", ctypes.c_uint32), ("num_register", ctypes.c_uint32),
        ("rope_start", ctypes.c_int32), ("qknorm_start", ctypes.c_int32),
        ("rope_freq", ctypes.c_float), ("ln_eps", ctypes.c_float),
        ("out_layers", ctypes.c_int32 * 16), ("n_out_layers", ctypes.c_int32),
        ("ffn_type", ctypes.c_char * 16),
        ("alt_start", ctypes.c_int32), ("cat_token", ctypes.c_int32),
        ("head_features", ctypes.c_uint32), ("head_max_depth", ctypes.c_float), ("head_pos_embed", ctypes.c_int32),
        ("img_mean", ctypes.c_float * 3), ("img_std", ctypes.c_float * 3),
        ("img_resize_mode", ctypes.c_char * 32),
        ("cam_dim_in", ctypes.c_uint32),
    ]


_lib = None
_vp = ctypes.c_void_p
_f32p = ctypes.POINTER(ctypes.c_float)
_i32p = ctypes.POINTER(ctypes.c_int)


def load_library(path: str = LIB_PATH):
    """Loads libvestra_attn.so.  Raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise RuntimeError(f"{path} is missing: build it with vestra-engine_b200/build.py")
    lib = ctypes.CDLL(path)
    i64, c_int, c_float = ctypes.c_int64, ctypes.c_int, ctypes.c_float
    sig = {
        "va_version": ([], ctypes.c_char_p),
        "va_default_config": ([ctypes.POINTER(VaConfig)], None),
        "va_create": ([ctypes.POINTER(VaConfig), c_int, ctypes.POINTER(_vp)], c_int),
        "va_destroy": ([_vp], None),
        "va_last_error": ([_vp], ctypes.c_char_p),
        "va_load_layer": ([_vp, c_int] + [_vp] * 11, c_int),
        "va_layer_flags": ([_vp, c_int, _i32p, _i32p], c_int),
        "va_run_attention": ([_vp, c_int, _vp, i64, c_int, c_int, _vp, _vp], c_int),
        "va_attention_host": ([_vp, c_int, _vp, i64, c_int, c_int, c_int, c_int, _vp], c_int),
        "va_attention_host_batch": ([_vp, c_int, _vp, _vp, c_int, i64, c_int, c_int, c_int, c_int], c_int),
        "va_attention_device": ([_vp, c_int, _vp, _vp, i64, c_int, c_int, c_int, c_int, _vp], c_int),
        "va_block_attention_device": ([_vp, c_int, _vp, i64, c_int, c_int, c_int, c_int, _vp], c_int),
        "va_op_attention_device": ([_vp, _vp, _vp, _vp, c_int, i64, c_int, _vp, _vp, _vp, _vp, c_float,
                                    _vp, c_float, _vp, _vp], c_int),
        "va_flash_attention_bf16": ([_vp, _vp, _vp, _vp, i64, i64, i64, c_int, i64, c_int, c_int, _vp, _vp],
                                    c_int),
        "va_comm_unique_id": ([_vp], c_int),
        "va_comm_init": ([_vp, _vp, c_int, c_int], c_int),
        "va_comm_exchange_mode": ([_vp], c_int),
        "va_attention_host_sharded": ([_vp, c_int, _vp, _vp, i64, c_int, c_int, c_int, c_int], c_int),
        "va_attention_device_sharded": ([_vp, c_int, _vp, _vp, i64, c_int, c_int, c_int, c_int, _vp], c_int),
        "va_op_attention_noalloc": ([_vp, _vp, _vp, c_int, i64, c_int, _vp, _vp, _vp, _vp, c_float, _vp, c_float,
                                     c_int, _vp, _vp], c_int),
        "va_linear_bf16": ([_vp, _vp, _vp, _vp, _vp, _vp, _vp, i64, c_int, c_int, _vp], c_int),
        "va_flash_plan": ([i64, i64, i64, c_int, i64, c_int, c_int, c_int, _i32p], c_int),
        "va_select_reference_view_saddle": ([_vp, c_int, c_int, _i32p], c_int),
        "va_reference_first_order": ([c_int, c_int, _i32p], c_int),
        "va_restore_order": ([c_int, c_int, _i32p], c_int),
        "va_camera_inject_device": ([_vp, _vp, c_int, i64, c_int, _vp], c_int),
        "va_permute_views_device": ([_vp, _vp, _i32p, c_int, i64, _vp], c_int),
        "va_check_device": ([_vp], c_int),
        "va_selftest_bounded_wait": ([_vp, ctypes.c_int64], c_int),
        "va_set_phase_profile": ([_vp, c_int], c_int),
        "va_load_mlp": ([_vp, c_int, c_int] + [_vp] * 7, c_int),
        "va_load_vit_norm": ([_vp, _vp, _vp], c_int),
        "va_backbone_device": ([_vp, _vp, i64, c_int, c_int, c_int, c_int, c_int, c_int, c_int, _vp, c_int,
                                _vp, _vp, _vp, _vp], c_int),
        "va_backbone_device_sharded": ([_vp, _vp, i64, i64, i64, c_int, c_int, c_int, c_int, c_int, c_int, c_int,
                                        _vp, c_int, _vp, _vp, _vp, _vp], c_int),
        "va_block_device": ([_vp, c_int, _vp, i64, c_int, c_int, c_int, c_int, _vp], c_int),
        "va_block_device_sharded": ([_vp, c_int, _vp, i64, c_int, c_int, c_int, c_int, _vp], c_int),
        "va_run_tail_host": ([_vp, c_int, _vp, i64, c_int, c_int, c_int, c_int, _vp], c_int),
        "va_phase_times": ([_vp, _vp], c_int),
        "va_exchange_times": ([_vp, _vp, _vp, _vp], c_int),
        "va_last_exchange": ([_vp], c_int),
        "va_load_patch_embed": ([_vp, _vp, _vp, _vp, _vp, i64, _vp, c_int, c_int, c_float], c_int),
        "va_prepare_tokens_device": ([_vp, _vp, c_int, c_int, c_int, _vp, _vp, _vp], c_int),
        "va_prepare_tokens_host": ([_vp, _vp, c_int, c_int, c_int, _vp, _vp], c_int),
        "va_pos_embed_device": ([_vp, c_int, c_int, _vp, _vp], c_int),
        "va_selftest_peer_wait": ([_vp, c_int, _f32p], c_int),
        "va_gguf_open": ([ctypes.c_char_p, ctypes.POINTER(_vp)], c_int),
        "va_gguf_close": ([_vp], None),
        "va_gguf_last_error": ([], ctypes.c_char_p),
        "va_gguf_version": ([_vp, ctypes.POINTER(ctypes.c_uint32)], c_int),
        "va_gguf_meta_count": ([_vp, ctypes.POINTER(i64)], c_int),
        "va_gguf_meta_entry": ([_vp, i64, ctypes.POINTER(_vp), ctypes.POINTER(i64), _i32p], c_int),
        "va_gguf_meta_u32": ([_vp, ctypes.c_char_p, ctypes.POINTER(ctypes.c_uint32)], c_int),
        "va_gguf_meta_i32": ([_vp, ctypes.c_char_p, ctypes.POINTER(ctypes.c_int32)], c_int),
        "va_gguf_meta_f32": ([_vp, ctypes.c_char_p, _f32p], c_int),
        "va_gguf_meta_u64": ([_vp, ctypes.c_char_p, ctypes.POINTER(ctypes.c_uint64)], c_int),
        "va_gguf_meta_bool": ([_vp, ctypes.c_char_p, _i32p], c_int),
        "va_gguf_meta_str": ([_vp, ctypes.c_char_p, ctypes.POINTER(_vp), ctypes.POINTER(i64)], c_int),
        "va_gguf_meta_arr_u32": ([_vp, ctypes.c_char_p, _vp, i64, ctypes.POINTER(i64)], c_int),
        "va_gguf_meta_arr_i32": ([_vp, ctypes.c_char_p, _vp, i64, ctypes.POINTER(i64)], c_int),
        "va_gguf_meta_arr_f32": ([_vp, ctypes.c_char_p, _vp, i64, ctypes.POINTER(i64)], c_int),
        "va_gguf_meta_arr_str": ([_vp, ctypes.c_char_p, i64, ctypes.POINTER(_vp), ctypes.POINTER(i64),
                                  ctypes.POINTER(i64)], c_int),
        "va_gguf_tensor_count": ([_vp, ctypes.POINTER(i64)], c_int),
        "va_gguf_tensor_name": ([_vp, i64, ctypes.POINTER(_vp), ctypes.POINTER(i64)], c_int),
        "va_gguf_tensor_info": ([_vp, ctypes.c_char_p, _i32p, _i32p, ctypes.POINTER(i64), c_int,
                                 ctypes.POINTER(ctypes.c_uint64)], c_int),
        "va_gguf_tensor_check": ([_vp, ctypes.c_char_p, ctypes.POINTER(i64), ctypes.POINTER(_vp),
                                  ctypes.POINTER(i64)], c_int),
        "va_gguf_tensor_device": ([_vp, ctypes.c_char_p, c_int, _vp, _vp], c_int),
        "va_gguf_tensor_f32": ([_vp, ctypes.c_char_p, c_int, _vp, i64], c_int),
        "va_gguf_model_config": ([_vp, ctypes.POINTER(VaModelConfig)], c_int),
        "va_load_model_gguf": ([_vp, _vp, ctypes.POINTER(i64)], c_int),
    }
    for name, (args, res) in sig.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    _lib = lib
    return lib


def _ptr(x):
    """Device/host address of a torch tensor, numpy array, int or None."""
    if x is None:
        return None
    if isinstance(x, int):
        return x
    if isinstance(x, np.ndarray):
        assert x.flags.c_contiguous
        return x.ctypes.data
    if hasattr(x, "data_ptr"):
        assert x.is_contiguous()
        return x.data_ptr()
    raise TypeError(type(x))


def _f32(a):
    return None if a is None else np.ascontiguousarray(a, dtype=np.float32)


def default_config(**overrides) -> VaConfig:
    cfg = VaConfig()
    load_library().va_default_config(ctypes.byref(cfg))
    for k, v in overrides.items():
        setattr(cfg, k, v)
    return cfg


def wname(layer_idx: int, suffix: str) -> str:
    """Weight tensor names, vit_block.rs:30-53 / :688-690."""
    return f"vit.blk.{layer_idx}.{suffix}"


@dataclass
class ModelConfig:
    """The ModelConfig fields of the attention path (config.rs:146-...)."""

    embed_dim: int = 768
    num_heads: int = 12
    head_dim: int = 64
    depth: int = 12
    num_register: int = 0
    rope_start: int = 4
    qknorm_start: int = 4
    rope_freq: float = 100.0
    ln_eps: float = 1e-6
    alt_start: int = 4
    patch_size: int = 14

    def to_va(self, max_rows: int, qk_norm_eps: float = 1e-5, rope_pairing: int = 0) -> VaConfig:
        return default_config(embed_dim=self.embed_dim, num_heads=self.num_heads, head_dim=self.head_dim,
                              depth=self.depth, num_register=self.num_register, rope_start=self.rope_start,
                              qknorm_start=self.qknorm_start, rope_freq=self.rope_freq, ln_eps=self.ln_eps,
                              qk_norm_eps=qk_norm_eps, rope_pairing=rope_pairing, max_rows=max_rows)

    @classmethod
    def from_gguf(cls, g: "GgufFile") -> "ModelConfig":
        """ModelConfig::from_gguf (config.rs:219-264), the fields of this path."""
        m = g.model_config()
        return cls(embed_dim=m["embed_dim"], num_heads=m["num_heads"], head_dim=m["head_dim"], depth=m["depth"],
                   num_register=m["num_register"], rope_start=m["rope_start"], qknorm_start=m["qknorm_start"],
                   rope_freq=m["rope_freq"], ln_eps=m["ln_eps"], alt_start=m["alt_start"],
                   patch_size=m["patch_size"])

    def is_global(self, layer_idx: int) -> bool:
        """backbone.rs:459-460 / :770-771."""
        return self.alt_start >= 0 and layer_idx >= self.alt_start and layer_idx % 2 == 1


class Context:
    """Owns one va_ctx (one device, serial calls)."""

    def __init__(self, cfg: VaConfig, device: int = 0):
        self.lib = load_library()
        self.cfg = cfg
        h = _vp()
        rc = self.lib.va_create(ctypes.byref(cfg), device, ctypes.byref(h))
        if rc != VA_OK:
            raise VestraError(rc, "va_create failed")
        self.h = h

    def close(self):
        if getattr(self, "h", None):
            self.lib.va_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def check(self, rc: int):
        if rc != VA_OK:
            raise VestraError(rc, self.lib.va_last_error(self.h).decode())

    def load_layer(self, layer: int, p: dict):
        """p: qkv_w [E,3E], qkv_b, proj_w [E,E], proj_b, optional norm1_w/b, q_g/q_b/k_g/k_b, ls1."""
        keep = {k: _f32(v) for k, v in p.items() if v is not None}
        g = lambda k: _ptr(keep.get(k))  # noqa: E731
        self.check(self.lib.va_load_layer(self.h, layer, g("norm1_w"), g("norm1_b"), g("qkv_w"), g("qkv_b"),
                                          g("q_g"), g("q_b"), g("k_g"), g("k_b"), g("proj_w"), g("proj_b"),
                                          g("ls1")))

    def load_mlp(self, layer: int, p: dict):
        """p: norm2_w/b [E], fc1_w [E,H], fc1_b [H], fc2_w [H,E], fc2_b [E], optional ls2 [E]."""
        keep = {k: _f32(v) for k, v in p.items() if v is not None}
        g = lambda k: _ptr(keep.get(k))  # noqa: E731
        hidden = keep["fc1_w"].size // self.cfg.embed_dim  # [E, hidden], or flat as the reference's Weights
        self.check(self.lib.va_load_mlp(self.h, layer, hidden, g("norm2_w"), g("norm2_b"), g("fc1_w"),
                                        g("fc1_b"), g("fc2_w"), g("fc2_b"), g("ls2")))

    def block_device(self, layer, tokens_dev, gh, gw, view_count, global_, stream=0):
        """One whole block in place on device tokens (run_tail_device, vit_block.rs:489-583)."""
        self.check(self.lib.va_block_device(self.h, layer, _ptr(tokens_dev), tokens_dev.shape[0], gh, gw,
                                            view_count, int(bool(global_)), stream))

    def block_device_sharded(self, layer, tokens_local, gh, gw, view_count, global_, stream=0):
        self.check(self.lib.va_block_device_sharded(self.h, layer, _ptr(tokens_local), tokens_local.shape[0],
                                                    gh, gw, view_count, int(bool(global_)), stream))

    def run_tail(self, layer, tokens, gh, gw, view_count, global_, out=None):
        """TransformerTailExecutor::run_tail (vit_block.rs:110-129) on host tokens."""
        tokens = _f32(tokens)
        out = np.empty_like(tokens) if out is None else out
        self.check(self.lib.va_run_tail_host(self.h, layer, _ptr(tokens), tokens.shape[0], gh, gw, view_count,
                                             int(bool(global_)), _ptr(out)))
        return out

    def load_vit_norm(self, w, b):
        w, b = _f32(w), _f32(b)
        self.check(self.lib.va_load_vit_norm(self.h, _ptr(w), _ptr(b)))

    def load_gguf(self, g: "GgufFile") -> int:
        """Every block / patch-embedding / final-norm tensor of an open model file
        straight into the device operands (va_load_model_gguf).  Returns the stored
        bytes uploaded."""
        n = ctypes.c_int64(0)
        self.check(self.lib.va_load_model_gguf(self.h, g.h, ctypes.byref(n)))
        if PATCH_EMBED_WEIGHT in g.tensor_names():
            _, shape, _ = g.tensor_info(PATCH_EMBED_WEIGHT)
            self._patch = int(round((int(np.prod(shape)) // self.cfg.embed_dim // 3) ** 0.5))
        return n.value

    def backbone_device(self, tokens_dev, gh, gw, view_count, first_layer, last_layer, alt_start,
                        camera_dev=None, out_layers=(), cat_token=True, stream=0):
        """Blocks [first_layer, last_layer) in place on view-major device tokens
        (backbone.rs:885-1137).  Returns {layer: (feat, cam)} device tensors of the
        captures at out_layers."""
        return self.backbone_device_sharded(tokens_dev, 0, tokens_dev.shape[0], gh, gw, view_count, first_layer,
                                            last_layer, alt_start, camera_dev, out_layers, cat_token, stream)

    def backbone_device_sharded(self, tokens_local, row_offset, window_rows, gh, gw, view_count, first_layer,
                                last_layer, alt_start, camera_dev=None, out_layers=(), cat_token=True, stream=0):
        """This rank's whole views [row_offset, row_offset + rows) of a window_rows window
        (collective when the range holds a global block).  Captures cover the rank's views."""
        import torch
        E = tokens_local.shape[1]
        n = window_rows // view_count
        local_views = tokens_local.shape[0] // n
        n_special = n - gh * gw
        width = 2 * E if cat_token else E
        caps = {l: (torch.empty(local_views, n - n_special, width, device=tokens_local.device),
                    torch.empty(local_views, width, device=tokens_local.device)) for l in out_layers}
        layers = (ctypes.c_int * max(1, len(out_layers)))(*out_layers)
        feats = (ctypes.c_void_p * max(1, len(out_layers)))(*[caps[l][0].data_ptr() for l in out_layers])
        cams = (ctypes.c_void_p * max(1, len(out_layers)))(*[caps[l][1].data_ptr() for l in out_layers])
        self.check(self.lib.va_backbone_device_sharded(
            self.h, _ptr(tokens_local), tokens_local.shape[0], row_offset, window_rows, gh, gw, view_count,
            first_layer, last_layer, alt_start, int(bool(cat_token)), _ptr(camera_dev), len(out_layers), layers,
            feats, cams, stream))
        return caps

    def layer_flags(self, layer: int):
        a, b = ctypes.c_int(), ctypes.c_int()
        self.check(self.lib.va_layer_flags(self.h, layer, ctypes.byref(a), ctypes.byref(b)))
        return bool(a.value), bool(b.value)

    def attention_host(self, layer, ln1, gh, gw, view_count, global_, out=None):
        ln1 = ln1 if hasattr(ln1, "data_ptr") else _f32(ln1)
        rows = ln1.shape[0]
        if out is None:
            out = np.empty_like(ln1) if isinstance(ln1, np.ndarray) else ln1.new_empty(ln1.shape)
        self.check(self.lib.va_attention_host(self.h, layer, _ptr(ln1), rows, gh, gw, view_count,
                                              int(bool(global_)), _ptr(out)))
        return out

    def attention_host_batch(self, layer, inputs, outputs, gh, gw, view_count, global_):
        """va_attention_host over independent same-shape host inputs, pipelined."""
        n = len(inputs)
        assert len(outputs) == n and n > 0
        rows = inputs[0].shape[0]
        ins = (ctypes.c_void_p * n)(*[_ptr(x) for x in inputs])
        outs = (ctypes.c_void_p * n)(*[_ptr(y) for y in outputs])
        self.check(self.lib.va_attention_host_batch(self.h, layer, ins, outs, n, rows, gh, gw, view_count,
                                                    int(bool(global_))))
        return outputs

    def attention_device(self, layer, ln1_dev, out_dev, gh, gw, view_count, global_, stream=0):
        self.check(self.lib.va_attention_device(self.h, layer, _ptr(ln1_dev), _ptr(out_dev), ln1_dev.shape[0],
                                                gh, gw, view_count, int(bool(global_)), stream))

    def block_attention_device(self, layer, tokens_dev, gh, gw, view_count, global_, stream=0):
        self.check(self.lib.va_block_attention_device(self.h, layer, _ptr(tokens_dev), tokens_dev.shape[0],
                                                      gh, gw, view_count, int(bool(global_)), stream))

    def run_attention(self, layer, inp, rows, heads, head_dim, positions_yx):
        inp = _f32(inp)
        out = np.empty_like(inp)
        pos = _f32(positions_yx)
        self.check(self.lib.va_run_attention(self.h, layer, _ptr(inp), rows, heads, head_dim, _ptr(pos),
                                             _ptr(out)))
        return out

    def flash_bf16(self, q, k, v, heads, out, seg_len=0, q_offset=0, stream=0, variant=-1):
        """q [q_count, heads*64], k [kv_rows, heads*64] bf16 token-major; v bf16 (production)
        or f16 (torch dtype decides); seg_len 0 = global; variant = poly + 8 * form of the
        softmax (< 0 = library default)."""
        v_f16 = int(str(getattr(v, "dtype", "")) == "torch.float16")
        self.check(self.lib.va_flash_attention_bf16(self.h, _ptr(q), _ptr(k), _ptr(v), q.shape[0], q_offset,
                                                    k.shape[0], heads, seg_len, v_f16, variant, _ptr(out),
                                                    stream))

    def comm_init(self, comm_id: bytes, nranks: int, rank: int):
        buf = ctypes.create_string_buffer(bytes(comm_id), 128)
        self.check(self.lib.va_comm_init(self.h, buf, nranks, rank))

    def attention_host_sharded(self, layer, ln1_local, gh, gw, view_count, global_, out=None):
        """This rank's slice of a query-sharded window, host buffers (collective)."""
        ln1_local = ln1_local if hasattr(ln1_local, "data_ptr") else _f32(ln1_local)
        if out is None:
            out = (np.empty_like(ln1_local) if isinstance(ln1_local, np.ndarray)
                   else ln1_local.new_empty(ln1_local.shape))
        self.check(self.lib.va_attention_host_sharded(self.h, layer, _ptr(ln1_local), _ptr(out),
                                                      ln1_local.shape[0], gh, gw, view_count,
                                                      int(bool(global_))))
        return out

    def exchange_mode(self) -> str:
        """How K'/V reach the other ranks: "none", "nccl", "direct" (the QKV epilogue
        stores into the peers' windows) or "direct-ce" (copy engines push each rank's
        rows, the attention kernel waits on per-peer flags)."""
        return ("none", "nccl", "direct", "direct-ce")[self.lib.va_comm_exchange_mode(self.h)]

    def attention_device_sharded(self, layer, ln1_local, out_local, gh, gw, view_count, global_, stream=0):
        self.check(self.lib.va_attention_device_sharded(self.h, layer, _ptr(ln1_local), _ptr(out_local),
                                                        ln1_local.shape[0], gh, gw, view_count,
                                                        int(bool(global_)), stream))

    def linear_bf16(self, a, w_t, out, bias=None, scale=None, residual=None, stream=0):
        m, k = a.shape
        n = w_t.shape[0]
        self.check(self.lib.va_linear_bf16(self.h, _ptr(a), _ptr(w_t), _ptr(bias), _ptr(scale), _ptr(residual),
                                           _ptr(out), m, n, k, stream))

    def op_attention(self, q, k, v, out, qnorm=None, knorm=None, qk_norm_eps=1e-5, rope=None, stream=0):
        heads, n, d = q.shape
        pos = None if rope is None else _f32(rope[0])
        freq = 100.0 if rope is None else float(rope[1])
        qg, qb = (None, None) if qnorm is None else qnorm
        kg, kb = (None, None) if knorm is None else knorm
        self.check(self.lib.va_op_attention_device(self.h, _ptr(q), _ptr(k), _ptr(v), heads, n, d, _ptr(qg),
                                                   _ptr(qb), _ptr(kg), _ptr(kb), qk_norm_eps, _ptr(pos), freq,
                                                   _ptr(out), stream))

    def check_device(self):
        self.check(self.lib.va_check_device(self.h))

    PHASES = ("ln", "qkv", "allgather", "core", "proj")

    def set_phase_profile(self, enable: bool):
        self.check(self.lib.va_set_phase_profile(self.h, int(bool(enable))))

    def phase_times(self) -> dict:
        """Durations (ms) of the last profiled device-path call, by phase name."""
        ms = np.zeros(len(self.PHASES), np.float32)
        self.check(self.lib.va_phase_times(self.h, _ptr(ms)))
        return dict(zip(self.PHASES, (float(v) for v in ms)))

    def last_exchange(self) -> str:
        """The K'/V path the last sharded call took (names as exchange_mode)."""
        return ("none", "nccl", "direct", "direct-ce")[self.lib.va_last_exchange(self.h)]

    def exchange_times(self):
        """Per-peer copy-engine push of the last profiled sharded call: (ms per peer,
        bytes sent to each peer)."""
        ms = np.zeros(8, np.float32)
        n = ctypes.c_int()
        nb = ctypes.c_int64()
        self.check(self.lib.va_exchange_times(self.h, _ptr(ms), ctypes.byref(n), ctypes.byref(nb)))
        return [float(v) for v in ms[:n.value]], int(nb.value)

    def selftest_bounded_wait(self, limit_us: int) -> int:
        """Runs the failure-detection self-test; returns the raw status (VA_ERR_DEVICE
        when the bounded wait gave up as designed)."""
        return self.lib.va_selftest_bounded_wait(self.h, int(limit_us))

    def selftest_peer_wait(self, peer_flag: int):
        """The attention kernel's wait for peer rows on one GPU (see the header):
        returns (raw status, max |difference| to the launch without a peer)."""
        m = ctypes.c_float(-1.0)
        rc = self.lib.va_selftest_peer_wait(self.h, int(peer_flag), ctypes.byref(m))
        return rc, m.value

    def load_patch_embed(self, weight_oihw, bias, cls_token, pos_embed, register_tokens=None, patch=14,
                         interp_offset=0.1):
        """Patch filter [E, 3, p, p], bias [E], CLS [E], learned positions [M*M + 1, E],
        register tokens [num_register, E] (pos_embed.rs:23-39, patch_embed.rs:33-36)."""
        w, b, c = _f32(weight_oihw), _f32(bias), _f32(cls_token)
        pe = _f32(pos_embed).reshape(-1, self.cfg.embed_dim)
        regs = None if register_tokens is None else _f32(register_tokens).reshape(-1, self.cfg.embed_dim)
        nreg = 0 if regs is None else regs.shape[0]
        self.check(self.lib.va_load_patch_embed(self.h, _ptr(w), _ptr(b), _ptr(c), _ptr(pe), pe.shape[0],
                                                None if regs is None else _ptr(regs), nreg, patch,
                                                float(interp_offset)))
        self._patch = patch

    def prepare_tokens_device(self, image_dev, views, height, width, tokens_dev, position_dev=None, stream=0):
        """prepare_tokens for `views` NCHW images on the device -> view-major tokens
        [views * (1 + num_register + gh*gw), E] (pos_embed.rs:236-300)."""
        self.check(self.lib.va_prepare_tokens_device(self.h, _ptr(image_dev), views, height, width,
                                                     None if position_dev is None else _ptr(position_dev),
                                                     _ptr(tokens_dev), stream))

    def prepare_tokens_host(self, images, height, width, position=None):
        """Host images [views, 3, H, W] (or one [3, H, W]) -> tokens [views, n, E]."""
        img = _f32(images).reshape(-1, 3, height, width)
        views = img.shape[0]
        patch = self._patch
        n = 1 + self.cfg.num_register + (height // patch) * (width // patch)
        out = np.empty((views, n, self.cfg.embed_dim), np.float32)
        pos = None if position is None else _f32(position)
        self.check(self.lib.va_prepare_tokens_host(self.h, _ptr(img), views, height, width,
                                                   None if pos is None else _ptr(pos), _ptr(out)))
        return out

    def pos_embed_device(self, gh, gw, out_dev, stream=0):
        """The interpolated position table [(1 + gh*gw), E] (PosEmbedCache::get_or_build)."""
        self.check(self.lib.va_pos_embed_device(self.h, gh, gw, _ptr(out_dev), stream))

    def last_error(self) -> str:
        return self.lib.va_last_error(self.h).decode()


class _FromGguf:
    """Engine::load's route (engine.rs:110-126, :323) for the executor classes."""

    @classmethod
    def from_gguf(cls, path, device: int = 0, max_rows: int = 12 * 866):
        """The config and every tensor the context holds, from a model file,
        converted on the device (va_load_model_gguf)."""
        with GgufFile(path) as g:
            self = cls.__new__(cls)
            self.cfg = ModelConfig.from_gguf(g)
            self.ctx = Context(self.cfg.to_va(max_rows), device)
            self.ctx.load_gguf(g)
        return self


class CudaAttentionExecutor(_FromGguf):
    """AttentionExecutor (vit_block.rs:95-105) backed by the sm_100a path.

    Built from the reference's `Weights` naming (dict name -> F32 array, linear
    weights [in, out]); uploads every layer once, like CudaAttentionExecutor::new
    (vit_block.rs:239-318).  run_attention raises instead of returning None: the
    reference's silent CPU fallback does not exist here.
    """

    def __init__(self, cfg: ModelConfig, weights: dict, device: int = 0, max_rows: int = 12 * 866):
        self.cfg = cfg
        self.ctx = Context(cfg.to_va(max_rows), device)
        for i in range(cfg.depth):
            if weights.get(wname(i, "attn_qkv.weight")) is None:
                continue
            self.ctx.load_layer(i, layer_params_from_weights(weights, i))

    def run_attention(self, layer_idx, input, rows, heads, head_dim, positions_yx):
        return self.ctx.run_attention(layer_idx, input, rows, heads, head_dim, positions_yx)

    def run_attention_views(self, layer_idx, ln1, gh, gw, view_count, global_):
        return self.ctx.attention_host(layer_idx, ln1, gh, gw, view_count, global_)


class CudaTransformerTailExecutor(_FromGguf):
    """TransformerTailExecutor (vit_block.rs:110-129) backed by the sm_100a path.

    Uploads every block's attention and MLP weights once from the reference's
    `Weights` naming (vit_block.rs:30-53: norm1/2, attn_*, mlp_fc1/2, ls1/ls2).
    run_tail returns the updated tokens of one block; the reference's `ln1`
    argument is accepted for signature parity and not used (LN1 is recomputed on
    the device from `tokens`).  No CPU fallback: failures raise.
    """

    def __init__(self, cfg: ModelConfig, weights: dict, device: int = 0, max_rows: int = 12 * 866):
        self.cfg = cfg
        self.ctx = Context(cfg.to_va(max_rows), device)
        for i in range(cfg.depth):
            if weights.get(wname(i, "attn_qkv.weight")) is None:
                continue
            self.ctx.load_layer(i, layer_params_from_weights(weights, i))
            if weights.get(wname(i, "mlp_fc1.weight")) is not None:
                self.ctx.load_mlp(i, mlp_params_from_weights(weights, i))

    def run_tail(self, layer_idx, tokens, ln1, rows, gh, gw, global_, view_count, cfg=None):
        del ln1, cfg
        t = np.asarray(tokens, np.float32).reshape(rows, self.cfg.embed_dim)
        return self.ctx.run_tail(layer_idx, t, gh, gw, view_count, global_)


PATCH_EMBED_WEIGHT = "vit.patch_embed.weight"
PATCH_EMBED_BIAS = "vit.patch_embed.bias"
POS_EMBED_WEIGHT = "vit.pos_embed"
CLS_TOKEN_WEIGHT = "vit.cls_token"
REGISTER_TOKENS_WEIGHT = "vit.register_tokens"


class CudaPatchEmbedExecutor(_FromGguf):
    """CudaPatchEmbedExecutor (patch_embed.rs:140-245) backed by the sm_100a path.

    Uploads the patch filter, bias, CLS token, learned positions and (when the
    model has them) register tokens once from the reference's `Weights` naming.
    run() is the reference's run(image_nchw, height, width, position) for one
    image: returns (gh, gw, tokens [1 + num_register + gh*gw, E]); position may be
    None, in which case the interpolated table is built on the device and cached.
    run_views() does several views in one call.  Errors raise.
    """

    def __init__(self, cfg: ModelConfig, weights: dict, device: int = 0, max_rows: int = 12 * 866):
        self.cfg = cfg
        self.ctx = Context(cfg.to_va(max_rows), device)
        regs = weights.get(REGISTER_TOKENS_WEIGHT)
        self.ctx.load_patch_embed(weights[PATCH_EMBED_WEIGHT], weights[PATCH_EMBED_BIAS],
                                  weights[CLS_TOKEN_WEIGHT], weights[POS_EMBED_WEIGHT], regs, cfg.patch_size)

    def run(self, image_nchw, height, width, position=None):
        tokens = self.ctx.prepare_tokens_host(image_nchw, height, width, position)[0]
        p = self.cfg.patch_size
        return height // p, width // p, tokens

    def run_views(self, images, height, width):
        return self.ctx.prepare_tokens_host(images, height, width)


class GgufFile:
    """GgufFile (crates/da-gguf reader.rs / meta.rs) over the library's va_gguf_*.

    The header, metadata and tensor infos are parsed on the host over a read-only
    mapping of the file; tensor values are converted on the GPU (tensor_f32).
    Getters return None where the reference's return Option::None (absent key or
    another kind).  Errors raise VestraError with the reference's GgufError text.
    """

    def __init__(self, path):
        self.lib = load_library()
        h = _vp()
        rc = self.lib.va_gguf_open(os.fsencode(path), ctypes.byref(h))
        if rc != VA_OK:
            raise VestraError(rc, self.lib.va_gguf_last_error().decode())
        self.h = h
        self.path = path

    open = classmethod(lambda cls, path: cls(path))

    def close(self):
        if getattr(self, "h", None):
            self.lib.va_gguf_close(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _raise(self, rc):
        raise VestraError(rc, self.lib.va_gguf_last_error().decode())

    @property
    def version(self) -> int:
        v = ctypes.c_uint32()
        self.lib.va_gguf_version(self.h, ctypes.byref(v))
        return v.value

    # ---- metadata (meta.rs:14-92)
    def _scalar(self, fn, ctype, key):
        v = ctype()
        rc = fn(self.h, key.encode(), ctypes.byref(v))
        if rc == VA_ERR_NOT_FOUND:
            return None
        if rc:
            self._raise(rc)
        return v.value

    def meta_u32(self, key):
        return self._scalar(self.lib.va_gguf_meta_u32, ctypes.c_uint32, key)

    def meta_i32(self, key):
        return self._scalar(self.lib.va_gguf_meta_i32, ctypes.c_int32, key)

    def meta_f32(self, key):
        return self._scalar(self.lib.va_gguf_meta_f32, ctypes.c_float, key)

    def meta_u64(self, key):
        return self._scalar(self.lib.va_gguf_meta_u64, ctypes.c_uint64, key)

    def meta_bool(self, key):
        v = self._scalar(self.lib.va_gguf_meta_bool, ctypes.c_int, key)
        return None if v is None else bool(v)

    def meta_str(self, key):
        s, n = _vp(), ctypes.c_int64()
        rc = self.lib.va_gguf_meta_str(self.h, key.encode(), ctypes.byref(s), ctypes.byref(n))
        if rc == VA_ERR_NOT_FOUND:
            return None
        if rc:
            self._raise(rc)
        return ctypes.string_at(s.value, n.value).decode()

    def _arr(self, fn, dtype, key):
        n = ctypes.c_int64()
        rc = fn(self.h, key.encode(), None, 0, ctypes.byref(n))
        if rc == VA_ERR_NOT_FOUND:
            return None
        if rc:
            self._raise(rc)
        out = np.zeros(n.value, dtype)
        if n.value:
            rc = fn(self.h, key.encode(), out.ctypes.data, n.value, ctypes.byref(n))
            if rc:
                self._raise(rc)
        return out.tolist()

    def meta_arr_u32(self, key):
        return self._arr(self.lib.va_gguf_meta_arr_u32, np.uint32, key)

    def meta_arr_i32(self, key):
        return self._arr(self.lib.va_gguf_meta_arr_i32, np.int32, key)

    def meta_arr_f32(self, key):
        return self._arr(self.lib.va_gguf_meta_arr_f32, np.float32, key)

    def meta_arr_str(self, key):
        n = ctypes.c_int64()
        rc = self.lib.va_gguf_meta_arr_str(self.h, key.encode(), 0, None, None, ctypes.byref(n))
        if rc == VA_ERR_NOT_FOUND:
            return None
        if rc:
            self._raise(rc)
        out = []
        for i in range(n.value):
            s, ln = _vp(), ctypes.c_int64()
            self.lib.va_gguf_meta_arr_str(self.h, key.encode(), i, ctypes.byref(s), ctypes.byref(ln), None)
            out.append(ctypes.string_at(s.value, ln.value).decode())
        return out

    _GETTER = {META_U32: "meta_u32", META_I32: "meta_i32", META_F32: "meta_f32", META_U64: "meta_u64",
               META_BOOL: "meta_bool", META_STR: "meta_str", META_ARR_U32: "meta_arr_u32",
               META_ARR_I32: "meta_arr_i32", META_ARR_F32: "meta_arr_f32", META_ARR_STR: "meta_arr_str"}

    @property
    def kv(self):
        """[(key, kind, value)] in file order (GgufFile::kv)."""
        n = ctypes.c_int64()
        self.lib.va_gguf_meta_count(self.h, ctypes.byref(n))
        out = []
        for i in range(n.value):
            k, ln, kind = _vp(), ctypes.c_int64(), ctypes.c_int()
            self.lib.va_gguf_meta_entry(self.h, i, ctypes.byref(k), ctypes.byref(ln), ctypes.byref(kind))
            out.append((ctypes.string_at(k.value, ln.value).decode(), kind.value))
        # a repeated key answers with its first entry (meta.rs:16-18); a key holding a
        # NUL byte cannot be looked up by name and lists None
        return [(k, kind, None if "\0" in k else getattr(self, self._GETTER[kind])(k)) for k, kind in out]

    # ---- tensors
    def tensor_names(self):
        n = ctypes.c_int64()
        self.lib.va_gguf_tensor_count(self.h, ctypes.byref(n))
        names = []
        for i in range(n.value):
            s, ln = _vp(), ctypes.c_int64()
            self.lib.va_gguf_tensor_name(self.h, i, ctypes.byref(s), ctypes.byref(ln))
            names.append(ctypes.string_at(s.value, ln.value).decode())
        return names

    def tensor_info(self, name):
        """(dtype, shape outer -> inner, offset)."""
        dt, nd, off = ctypes.c_int(), ctypes.c_int(), ctypes.c_uint64()
        shape = (ctypes.c_int64 * 16)()
        rc = self.lib.va_gguf_tensor_info(self.h, name.encode(), ctypes.byref(dt), ctypes.byref(nd), shape, 16,
                                          ctypes.byref(off))
        if rc:
            self._raise(rc)
        return dt.value, list(shape[:nd.value]), off.value

    def tensor_bytes(self, name) -> bytes:
        """The stored bytes after tensor_f32's checks."""
        n, data, nb = ctypes.c_int64(), _vp(), ctypes.c_int64()
        rc = self.lib.va_gguf_tensor_check(self.h, name.encode(), ctypes.byref(n), ctypes.byref(data),
                                           ctypes.byref(nb))
        if rc:
            self._raise(rc)
        return ctypes.string_at(data.value, nb.value) if nb.value else b""

    def tensor_q8_0(self, name):
        """tensor_q8_0 (reader.rs:351-376) for a Q8_0 tensor: (shape, scales f16
        [blocks], quants int8 [blocks, 32])."""
        dtype, shape, _ = self.tensor_info(name)
        if dtype != GGML_Q8_0:
            raise VestraError(VA_ERR_DTYPE, f"tensor '{name}' is not Q8_0 (dtype {dtype})")
        blk = np.frombuffer(self.tensor_bytes(name), np.uint8).reshape(-1, 34)
        return shape, blk[:, :2].copy().view("<f2").reshape(-1), blk[:, 2:].copy().view(np.int8)

    def tensor_f32(self, name, transpose2d: bool = False):
        """tensor_f32 (reader.rs:279-349) converted on the GPU: (shape, F32 values
        flat).  transpose2d: a rank-2 tensor comes back transposed (weights_from_gguf)."""
        dtype, shape, _ = self.tensor_info(name)
        n = int(np.prod(shape, dtype=np.int64))
        out = np.empty(n, np.float32)
        rc = self.lib.va_gguf_tensor_f32(self.h, name.encode(), int(transpose2d), out.ctypes.data, n)
        if rc:
            self._raise(rc)
        return shape, out

    def tensor_device(self, name, out_dev, transpose2d: bool = False, stream=0):
        """tensor_f32 into a device buffer (numel floats)."""
        rc = self.lib.va_gguf_tensor_device(self.h, name.encode(), int(transpose2d), _ptr(out_dev), _ptr(stream))
        if rc:
            self._raise(rc)

    def model_config(self) -> dict:
        """ModelConfig::from_gguf (config.rs:219-264), every field."""
        c = VaModelConfig()
        rc = self.lib.va_gguf_model_config(self.h, ctypes.byref(c))
        if rc:
            self._raise(rc)
        d = {f: getattr(c, f) for f, _ in VaModelConfig._fields_}
        for f in ("arch", "ffn_type", "img_resize_mode"):
            d[f] = d[f].decode()
        d["out_layers"] = list(c.out_layers[:c.n_out_layers])
        del d["n_out_layers"]
        d["img_mean"], d["img_std"] = list(c.img_mean), list(c.img_std)
        d["cat_token"], d["head_pos_embed"] = bool(c.cat_token), bool(c.head_pos_embed)
        return d


def weights_from_gguf(g: GgufFile) -> dict:
    """weights_from_gguf (engine.rs:110-126): name -> F32 values, rank-2 tensors
    transposed to [in, out]; converted on the GPU."""
    return {name: g.tensor_f32(name, transpose2d=True)[1] for name in g.tensor_names()}


def mlp_params_from_weights(weights: dict, i: int) -> dict:
    g = lambda s: weights.get(wname(i, s))  # noqa: E731
    return {"norm2_w": g("norm2.weight"), "norm2_b": g("norm2.bias"), "fc1_w": g("mlp_fc1.weight"),
            "fc1_b": g("mlp_fc1.bias"), "fc2_w": g("mlp_fc2.weight"), "fc2_b": g("mlp_fc2.bias"), "ls2": g("ls2")}


def layer_params_from_weights(weights: dict, i: int) -> dict:
    g = lambda s: weights.get(wname(i, s))  # noqa: E731
    return {"norm1_w": g("norm1.weight"), "norm1_b": g("norm1.bias"), "qkv_w": g("attn_qkv.weight"),
            "qkv_b": g("attn_qkv.bias"), "q_g": g("attn_qnorm.weight"), "q_b": g("attn_qnorm.bias"),
            "k_g": g("attn_knorm.weight"), "k_b": g("attn_knorm.bias"), "proj_w": g("attn_proj.weight"),
            "proj_b": g("attn_proj.bias"), "ls1": g("ls1")}


def positions_yx(rows: int, view_count: int, n_special: int, gh: int, gw: int, global_: bool) -> np.ndarray:
    """RoPE position table of run_attention (vit_block.rs:841-881), [rows, 2] F32."""
    per_view = n_special + gh * gw
    if view_count <= 0 or per_view * view_count != rows:
        raise ValueError("token count must equal tokens_per_view * view_count")
    p = np.zeros((view_count, per_view, 2), np.float32)
    if global_:
        p[:, n_special:, :] = 1.0
    else:
        idx = np.arange(gh * gw)
        p[:, n_special:, 0] = idx // gw + 1
        p[:, n_special:, 1] = idx % gw + 1
    return p.reshape(rows, 2)


def op_attention_noalloc(q, k, v, out, qnorm=None, knorm=None, qk_norm_eps=1e-5, pos_yx_dev=None,
                         freq=100.0, rope_pairing=0, stream=0) -> int:
    """Op::Attention without any device allocation (for callers that cannot call
    cudaMalloc); all arguments are device tensors.  Returns the raw status code."""
    heads, n, d = q.shape
    qg, qb = (None, None) if qnorm is None else qnorm
    kg, kb = (None, None) if knorm is None else knorm
    return load_library().va_op_attention_noalloc(_ptr(q), _ptr(k), _ptr(v), heads, n, d, _ptr(qg), _ptr(qb),
                                                  _ptr(kg), _ptr(kb), qk_norm_eps, _ptr(pos_yx_dev), freq,
                                                  rope_pairing, _ptr(out), stream)


def comm_unique_id() -> bytes:
    """128-byte communicator id, made on rank 0 and shared with the other ranks."""
    buf = ctypes.create_string_buffer(128)
    rc = load_library().va_comm_unique_id(buf)
    if rc != VA_OK:
        raise VestraError(rc, "va_comm_unique_id failed (NCCL unavailable?)")
    return buf.raw


def shard_views(view_count: int, tokens_per_view: int, nranks: int, rank: int) -> tuple[int, int]:
    """(row_offset, local_rows) of a rank's whole views: view_count views split as
    evenly as possible, the first ranks taking one more (12 on 8: 2,2,2,2,1,1,1,1)."""
    if view_count < nranks:
        raise ValueError(f"{view_count} views cannot give every one of {nranks} ranks a view")
    base, extra = divmod(view_count, nranks)
    first = rank * base + min(rank, extra)
    count = base + (1 if rank < extra else 0)
    return first * tokens_per_view, count * tokens_per_view


def shard_rows(window_rows: int, nranks: int, rank: int) -> tuple[int, int]:
    """(row_offset, local_rows) of a rank's equal contiguous slice of the window."""
    if window_rows % nranks:
        raise ValueError(f"window of {window_rows} tokens does not split into {nranks} equal slices")
    local = window_rows // nranks
    return rank * local, local


FLASH_KERNELS = {15: "flash_fwd_d64_ks1_kernel", 14: "flash_fwd_d64_ksp_kernel"}


def flash_plan(q_count: int, kv_rows: int, heads: int, seg_len: int = 0, q_offset: int = 0,
               fixed_offset: bool = True, variant: int = -1, sms: int = 148) -> dict:
    """The attention launch plan the library makes for these shapes (va_flash_plan; no
    GPU needed): variant form/poly, the kernel, units, key split and grid."""
    out = (ctypes.c_int * 9)()
    rc = load_library().va_flash_plan(q_count, q_offset, kv_rows, heads, seg_len, int(fixed_offset), variant,
                                      sms, out)
    if rc != VA_OK:
        raise VestraError(rc, "flash_plan")
    form, poly, unit_rows, per_sm, n_full, splits, gx, gy, gz = list(out)
    if form in FLASH_KERNELS:
        kernel = FLASH_KERNELS[form]
    elif form >= 9:
        kernel = "flash_fwd_d64_ks_kernel"
    elif form == 3 or form >= 5:
        kernel = "flash_fwd_d64_w20_kernel"
    else:
        kernel = "flash_fwd_d64_kernel"
    return {"form": form, "poly": poly, "kernel": kernel, "unit_rows": unit_rows, "per_sm": per_sm,
            "n_full": n_full, "splits": splits, "grid": (gx, gy, gz)}


def select_reference_view_saddle(cls) -> int:
    cls = _f32(cls)
    out = ctypes.c_int()
    rc = load_library().va_select_reference_view_saddle(_ptr(cls), cls.shape[0], cls.shape[1], ctypes.byref(out))
    if rc != VA_OK:
        raise VestraError(rc, "select_reference_view_saddle")
    return out.value


def reference_first_order(view_count: int, reference: int) -> list[int]:
    buf = (ctypes.c_int * view_count)()
    rc = load_library().va_reference_first_order(view_count, reference, buf)
    if rc != VA_OK:
        raise VestraError(rc, "reference_first_order")
    return list(buf)


def restore_original_view_order(ordered: list, reference_view_index: int) -> list:
    """engine.rs:198-205: caller order from reference-first order."""
    n = len(ordered)
    buf = (ctypes.c_int * n)()
    rc = load_library().va_restore_order(n, reference_view_index, buf)
    if rc != VA_OK:
        raise VestraError(rc, "restore_order")
    return [ordered[i] for i in buf]


def camera_inject_device(tokens_dev, camera_dev, views, tokens_per_view, embed, stream=0):
    rc = load_library().va_camera_inject_device(_ptr(tokens_dev), _ptr(camera_dev), views, tokens_per_view,
                                                embed, stream)
    if rc != VA_OK:
        raise VestraError(rc, "camera_inject_device")


def permute_views_device(src_dev, dst_dev, order, views, view_elems, stream=0):
    buf = (ctypes.c_int * views)(*order)
    rc = load_library().va_permute_views_device(_ptr(src_dev), _ptr(dst_dev), buf, views, view_elems, stream)
    if rc != VA_OK:
        raise VestraError(rc, "permute_views_device")
