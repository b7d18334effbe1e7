"""Pure-Python / NumPy restatement of the reference's GGUF model-file reader.

TEST INFRASTRUCTURE ONLY: imported by tests/ as the checker of the library's
GGUF reader and device dequantisation.  The product path (vestra-engine_b200/)
never imports this module.

Restated from the vestra-engine project (paths inside it):
  crates/da-gguf/src/reader.rs   GgufFile::open (:213-266), read_kv_value (:86-208),
                                 tensor_f32 (:279-349), tensor_q8_0 (:351-376)
  crates/da-gguf/src/meta.rs     MetaValue (:1-12) and the typed getters (:14-92)
  crates/da-gguf/src/q8_0.rs     dequantize_q8_0 (:24-33), read_blocks (:36-51)
  crates/da-engine/src/engine.rs weights_from_gguf (:110-126): rank-2 tensors
                                 transposed, every other rank kept as stored
  crates/da-engine/src/config.rs ModelConfig::from_gguf (:219-264), req_* (:187-212)
The container format and the Q8_0 block (an IEEE half scale then 32 int8 quants)
are ggml's (rev eced84c8, as the reference pins it).
"""
from __future__ import annotations

import struct

import numpy as np

GGML_F32, GGML_F16, GGML_Q8_0 = 0, 1, 8  # reader.rs:52-55
QK8_0 = 32
Q8_0_BLOCK_BYTES = 34

# MetaValue variants (meta.rs:1-12), numbered like the C ABI's VA_META_* codes.
U32, I32, F32, U64, BOOL, STR, ARR_U32, ARR_I32, ARR_F32, ARR_STR = range(10)


class GgufError(Exception):
    """GgufError (reader.rs:15-29); `kind` is one of io, bad_magic, version,
    not_found, dtype, malformed; str(e) is the reference's Display text."""

    def __init__(self, kind: str, msg: str):
        super().__init__(msg)
        self.kind = kind


def _malformed(what):
    return GgufError("malformed", f"malformed: {what}")


class _Cursor:
    """reader.rs:56-84."""

    def __init__(self, b: bytes):
        self.b, self.p = b, 0

    def take(self, n: int) -> bytes:
        if n > len(self.b) - self.p:
            raise _malformed("eof")
        s = self.b[self.p:self.p + n]
        self.p += n
        return s

    def u32(self) -> int:
        return struct.unpack("<I", self.take(4))[0]

    def u64(self) -> int:
        return struct.unpack("<Q", self.take(8))[0]

    def string(self) -> str:
        n = self.u64()
        return self.take(n).decode("utf-8", errors="replace")  # from_utf8_lossy


def read_kv_value(c: _Cursor, vtype: int):
    """read_kv_value (reader.rs:86-208): (kind, value), or None for the spec-valid
    array element types the reader skips."""
    if vtype == 0:
        return U32, c.take(1)[0]
    if vtype == 1:
        return I32, c.take(1)[0]  # `u8 as i32`: zero-extended, not sign-extended
    if vtype == 2:
        return U32, struct.unpack("<H", c.take(2))[0]
    if vtype == 3:
        return I32, struct.unpack("<h", c.take(2))[0]
    if vtype == 4:
        return U32, c.u32()
    if vtype == 5:
        return I32, struct.unpack("<i", c.take(4))[0]
    if vtype == 6:
        return F32, float(np.frombuffer(c.take(4), "<f4")[0])
    if vtype == 7:
        return BOOL, c.take(1)[0] != 0
    if vtype == 8:
        return STR, c.string()
    if vtype == 10:
        return U64, c.u64()
    if vtype == 11:
        return U64, c.u64()  # `i64 as u64`: the bit pattern
    if vtype == 12:
        with np.errstate(over="ignore"):  # `as f32` saturates to +-inf
            return F32, float(np.float32(struct.unpack("<d", c.take(8))[0]))
    if vtype == 9:
        elem = c.u32()
        n = c.u64()
        if elem in (4, 5, 6):
            if n > (len(c.b) - c.p) // 4:
                raise _malformed("eof")
            raw = c.take(4 * n)
            if elem == 4:
                return ARR_U32, [int(x) for x in np.frombuffer(raw, "<u4")]
            if elem == 5:
                return ARR_I32, [int(x) for x in np.frombuffer(raw, "<i4")]
            return ARR_F32, [float(x) for x in np.frombuffer(raw, "<f4")]
        if elem == 8:
            return ARR_STR, [c.string() for _ in range(n)]
        if elem in (0, 1, 2, 3, 7, 10, 11, 12):
            width = 1 if elem in (0, 1, 7) else 2 if elem in (2, 3) else 8
            if n > (len(c.b) - c.p) // width:
                raise _malformed("eof")
            c.take(n * width)
            return None
        raise _malformed(f"array element type {elem}")
    raise _malformed(f"kv type {vtype}")


class GgufFile:
    """GgufFile::open (reader.rs:213-266) over the file's bytes."""

    def __init__(self, data: bytes):
        self.raw = bytes(data)
        c = _Cursor(self.raw)
        if c.take(4) != b"GGUF":
            raise GgufError("bad_magic", "bad magic")
        self.version = c.u32()
        if self.version not in (2, 3):
            raise GgufError("version", f"unsupported gguf version {self.version}")
        tensor_count = c.u64()
        kv_count = c.u64()
        alignment = 32
        self.kv = []  # [(key, kind, value)] in file order
        for _ in range(kv_count):
            key = c.string()
            vtype = c.u32()
            if key == "general.alignment" and vtype == 4:
                alignment = c.u32()
                if alignment == 0:
                    raise _malformed("general.alignment is 0")
                self.kv.append((key, U32, alignment))
                continue
            v = read_kv_value(c, vtype)
            if v is not None:
                self.kv.append((key, v[0], v[1]))
        self.tensors = []  # [(name, dims innermost first, dtype, offset)]
        for _ in range(tensor_count):
            name = c.string()
            n_dims = c.u32()
            if n_dims > (len(self.raw) - c.p) // 8:
                raise _malformed("eof")
            dims = [c.u64() for _ in range(n_dims)]
            dtype = c.u32()
            offset = c.u64()
            self.tensors.append((name, dims, dtype, offset))
        self.alignment = alignment
        self.data_start = c.p + (alignment - c.p % alignment) % alignment

    @classmethod
    def open(cls, path):
        with open(path, "rb") as f:
            return cls(f.read())

    # ---- meta.rs:14-92
    def meta(self, key):
        for k, kind, v in self.kv:
            if k == key:
                return kind, v
        return None

    def _typed(self, key, kinds):
        m = self.meta(key)
        return m[1] if m is not None and m[0] in kinds else None

    def meta_u32(self, key):
        v = self._typed(key, (U32, I32))
        return None if v is None else v & 0xFFFFFFFF

    def meta_i32(self, key):
        v = self._typed(key, (U32, I32))
        return None if v is None else (v & 0xFFFFFFFF) - ((v & 0x80000000) << 1)

    def meta_f32(self, key):
        return self._typed(key, (F32,))

    def meta_u64(self, key):
        return self._typed(key, (U64,))

    def meta_str(self, key):
        return self._typed(key, (STR,))

    def meta_bool(self, key):
        return self._typed(key, (BOOL,))

    def meta_arr_u32(self, key):
        return self._typed(key, (ARR_U32,))

    def meta_arr_i32(self, key):
        m = self.meta(key)
        if m is None:
            return None
        if m[0] == ARR_I32:
            return list(m[1])
        if m[0] == ARR_U32:
            return [(v & 0xFFFFFFFF) - ((v & 0x80000000) << 1) for v in m[1]]
        return None

    def meta_arr_f32(self, key):
        return self._typed(key, (ARR_F32,))

    def meta_arr_str(self, key):
        return self._typed(key, (ARR_STR,))

    def tensor_names(self):
        return [t[0] for t in self.tensors]

    def _info(self, name):
        for t in self.tensors:
            if t[0] == name:
                return t
        raise GgufError("not_found", f"tensor not found: {name}")

    def tensor_shape(self, name):
        return [int(d) for d in reversed(self._info(name)[1])]

    def tensor_check(self, name):
        """The checks of tensor_f32 (reader.rs:279-349) in its order; returns
        (shape outer->inner, dtype, element count, stored bytes)."""
        name_, dims, dtype, offset = self._info(name)
        n = _wrapping_product(dims)
        base = self.data_start + offset
        if dtype == GGML_F32:
            nbytes = 4 * n
        elif dtype == GGML_F16:
            nbytes = 2 * n
        elif dtype == GGML_Q8_0:
            if n % QK8_0:
                raise _malformed(f"tensor '{name}' has {n} elements, not a multiple of block size {QK8_0} (QK8_0)")
            nbytes = n // QK8_0 * Q8_0_BLOCK_BYTES
        else:
            raise GgufError("dtype", f"unsupported dtype {dtype}")
        end = base + nbytes
        if end > len(self.raw):
            raise _malformed(_out_of_bounds(name, base, nbytes, len(self.raw)))
        return [int(d) for d in reversed(dims)], dtype, n, self.raw[base:end]

    def tensor_f32(self, name):
        """tensor_f32 (reader.rs:279-349): (shape, F32 values flat)."""
        shape, dtype, n, raw = self.tensor_check(name)
        if dtype == GGML_F32:
            return shape, np.frombuffer(raw, "<f4").astype(np.float32)
        if dtype == GGML_F16:
            return shape, np.frombuffer(raw, "<f2").astype(np.float32)
        d, qs = read_blocks(raw, n)
        return shape, dequantize_q8_0(d, qs)

    def tensor_q8_0(self, name):
        """tensor_q8_0 (reader.rs:351-376): (shape, scales f16 [nblocks], quants
        int8 [nblocks, 32]).  Like the reference it does not look at the dtype: the
        stored bytes are read as Q8_0 blocks whatever the tensor's type."""
        _, dims, _, offset = self._info(name)
        n = _wrapping_product(dims)
        if n % QK8_0:
            raise _malformed(f"tensor '{name}' has {n} elements, not a multiple of block size {QK8_0} (QK8_0)")
        base = self.data_start + offset
        end = base + n // QK8_0 * Q8_0_BLOCK_BYTES
        if end > len(self.raw):
            raise _malformed(_out_of_bounds(name, base, n // QK8_0 * Q8_0_BLOCK_BYTES, len(self.raw)))
        d, qs = read_blocks(self.raw[base:end], n)
        return [int(x) for x in reversed(dims)], d, qs


def _wrapping_product(dims) -> int:
    """The element count as the reference's release build computes it: the product
    of the dims as usize, wrapping at 2^64."""
    n = 1
    for d in dims:
        n = (n * d) % (1 << 64)
    return n


def _out_of_bounds(name, base, nbytes, size):
    """The out-of-bounds message; a base or end at or past 2^64 prints the wrapped
    base and "overflow" for the end (a 64-bit reader cannot form them)."""
    end = base + nbytes
    ok = base < (1 << 64) and nbytes < (1 << 64) and end < (1 << 64)
    return (f"tensor '{name}' data out of bounds: [{base % (1 << 64)}, {end if ok else 'overflow'}) "
            f"exceeds file size {size}")


def read_blocks(raw: bytes, n: int):
    """read_blocks (q8_0.rs:36-51): densely packed 34-byte blocks."""
    nb = n // QK8_0
    blk = np.frombuffer(raw[:nb * Q8_0_BLOCK_BYTES], np.uint8).reshape(nb, Q8_0_BLOCK_BYTES)
    d = blk[:, :2].copy().view("<f2").reshape(nb)
    qs = blk[:, 2:].copy().view(np.int8)
    return d, qs


def dequantize_q8_0(d, qs):
    """dequantize_q8_0 (q8_0.rs:24-33): out[32*b + j] = f32(d[b]) * f32(qs[b][j])."""
    return (d.astype(np.float32)[:, None] * qs.astype(np.float32)).reshape(-1).astype(np.float32)


def weights_from_gguf(f: GgufFile) -> dict:
    """weights_from_gguf (engine.rs:110-126): every tensor as F32; a rank-2 tensor
    [rows, cols] is transposed to [cols, rows] (GGUF [out, in] -> [in, out])."""
    out = {}
    for name in f.tensor_names():
        shape, data = f.tensor_f32(name)
        if len(shape) == 2:
            data = data.reshape(shape[0], shape[1]).T.reshape(-1)
        out[name] = np.ascontiguousarray(data, np.float32)
    return out


class ConfigError(Exception):
    """EngineError variants of ModelConfig::from_gguf (config.rs:98-104)."""

    def __init__(self, kind: str, msg: str):
        super().__init__(msg)
        self.kind = kind


def model_config(f: GgufFile) -> dict:
    """ModelConfig::from_gguf (config.rs:219-264) with req_* (:187-212)."""
    p = "depthanything3."
    arch = f.meta_str(p + "arch")
    if arch != "depthanything3":
        found = "None" if arch is None else f'Some("{arch}")'
        raise ConfigError("unsupported", f"unsupported model architecture: expected 'depthanything3', found {found}")

    def req(getter, key):
        v = getter(p + key)
        if v is None:
            raise ConfigError("missing", f"missing required gguf metadata key: {p + key}")
        return v

    def vec3(key):
        v = req(f.meta_arr_f32, key)
        if len(v) != 3:
            raise ConfigError("malformed", f"malformed gguf metadata for key {p + key}: expected 3 elements, got {len(v)}")
        return list(v)

    cfg = {"arch": arch}
    cfg["patch_size"] = req(f.meta_u32, "patch_size")
    image_size = f.meta_u32(p + "img.resize_target")
    if image_size is None:
        image_size = f.meta_u32(p + "image_size")
    if image_size is None:
        raise ConfigError("missing", f"missing required gguf metadata key: {p}img.resize_target")
    cfg["image_size"] = image_size
    for field, key in (("embed_dim", "vit.embed_dim"), ("depth", "vit.depth"), ("num_heads", "vit.num_heads"),
                       ("head_dim", "vit.head_dim"), ("mlp_hidden", "vit.mlp_hidden"),
                       ("num_register", "vit.num_register_tokens")):
        cfg[field] = req(f.meta_u32, key)
    cfg["rope_start"] = req(f.meta_i32, "vit.rope_start")
    cfg["qknorm_start"] = req(f.meta_i32, "vit.qknorm_start")
    cfg["rope_freq"] = req(f.meta_f32, "vit.rope_freq")
    cfg["ln_eps"] = req(f.meta_f32, "vit.ln_eps")
    cfg["out_layers"] = req(f.meta_arr_i32, "vit.out_layers")
    ffn = f.meta_str(p + "vit.ffn_type")
    cfg["ffn_type"] = "mlp" if ffn is None else ffn
    alt = f.meta_i32(p + "vit.alt_start")
    cfg["alt_start"] = -1 if alt is None else alt
    cat = f.meta_bool(p + "vit.cat_token")
    cfg["cat_token"] = True if cat is None else cat
    cfg["head_features"] = req(f.meta_u32, "head.features")
    md = f.meta_f32(p + "head.max_depth")
    cfg["head_max_depth"] = 0.0 if md is None else md
    hp = f.meta_bool(p + "head.pos_embed")
    cfg["head_pos_embed"] = True if hp is None else hp
    cfg["img_mean"] = vec3("img.mean")
    cfg["img_std"] = vec3("img.std")
    cfg["img_resize_mode"] = req(f.meta_str, "img.resize_mode")
    cfg["cam_dim_in"] = req(f.meta_u32, "cam.dim_in")
    return cfg
