"""The library's GGUF reader (va_gguf_*, host code) against the oracle: the
reference's own known answers, every truncation of a small model file, and seeded
byte corruptions must give the same metadata, tensor table, checks and error text.
No device calls (CPU only)."""
import json
import os

import numpy as np
import pytest

import gguf
import synthetic as syn
import vestra_attn as va

HERE = os.path.dirname(os.path.abspath(__file__))
with open(os.path.join(HERE, "golden", "gguf_vectors.json")) as f:
    VEC = json.load(f)

CODE = {"io": va.VA_ERR_IO, "bad_magic": va.VA_ERR_FORMAT, "version": va.VA_ERR_FORMAT,
        "malformed": va.VA_ERR_FORMAT, "not_found": va.VA_ERR_NOT_FOUND, "dtype": va.VA_ERR_DTYPE}
GETTER = {gguf.U32: "meta_u32", gguf.I32: "meta_i32", gguf.F32: "meta_f32", gguf.U64: "meta_u64",
          gguf.BOOL: "meta_bool", gguf.STR: "meta_str", gguf.ARR_U32: "meta_arr_u32", gguf.ARR_I32: "meta_arr_i32",
          gguf.ARR_F32: "meta_arr_f32", gguf.ARR_STR: "meta_arr_str"}


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(va.LIB_PATH):
        import __graft_entry__
        __graft_entry__.build()
    return va.load_library()


def write(tmp_path, data: bytes, name="m.gguf"):
    p = tmp_path / name
    p.write_bytes(data)
    return str(p)


def outcome_oracle(data: bytes):
    try:
        o = gguf.GgufFile(data)
    except gguf.GgufError as e:
        return ("error", CODE[e.kind], str(e))
    keys = [(k, kind) for k, kind, _ in o.kv]
    # names are looked up as C strings: one holding a NUL byte is reachable by enumeration only
    vals = [None if "\0" in k else getattr(o, GETTER[kind])(k) for k, kind in keys]
    tensors = []
    for name in o.tensor_names():
        if "\0" in name:
            tensors.append((name, "unreachable"))
            continue
        try:
            shape, dtype, n, raw = o.tensor_check(name)
            tensors.append((name, "ok", shape, dtype, n, raw))
        except gguf.GgufError as e:
            tensors.append((name, "error", CODE[e.kind], str(e)))
    return ("ok", o.version, keys, vals, tensors)


def outcome_lib(path):
    try:
        g = va.GgufFile(path)
    except va.VestraError as e:
        return ("error", e.code, str(e).split(": ", 1)[1])
    with g:
        kv = g.kv
        keys = [(k, kind) for k, kind, _ in kv]
        vals = [v for _, _, v in kv]
        tensors = []
        for name in g.tensor_names():
            if "\0" in name:
                tensors.append((name, "unreachable"))
                continue
            try:
                dtype, shape, _ = g.tensor_info(name)
                raw = g.tensor_bytes(name)
                tensors.append((name, "ok", shape, dtype, int(np.prod(shape, dtype=np.int64)), raw))
            except va.VestraError as e:
                tensors.append((name, "error", e.code, str(e).split(": ", 1)[1]))
        return ("ok", g.version, keys, vals, tensors)


def small_model() -> bytes:
    w = syn.GgufWriter(version=3)
    w.kv_str("depthanything3.arch", "depthanything3")
    w.kv_u8("x.u8", 7)
    w.kv_i8("x.i8", -3)
    w.kv_i16("x.i16", -300)
    w.kv_f64("x.f64", 1.0 / 3.0)
    w.kv_i64("x.i64", -9)
    w.kv_bool("x.b", False)
    w.kv_arr("x.strs", 8, ["ab", "c"])
    w.kv_arr("x.skip", 11, [1, 2])
    w.kv_arr("x.f", 6, [1.25, -2.5])
    r = np.random.default_rng(0)
    w.tensor("t.f32", r.standard_normal((3, 5)).astype(np.float32))
    w.tensor("t.f16", r.standard_normal(12).astype(np.float32), "f16")
    w.tensor("t.q8", r.standard_normal((2, 64)).astype(np.float32), "q8_0")
    return w.to_bytes()


def test_golden_metadata_and_config(lib, tmp_path):
    for case in ("bool_array_skip", "u16_array_skip"):
        v = VEC[case]
        with va.GgufFile(write(tmp_path, bytes.fromhex(v["file_hex"]))) as g:
            kind = {"u32": va.META_U32, "i32": va.META_I32}
            assert g.kv == [(e[0], kind[e[1]], e[2]) for e in v["expect_kv"]]
    for case in ("config_full", "config_alt4", "config_cat_off", "e2e_tiny"):
        v = VEC[case]
        with va.GgufFile(write(tmp_path, bytes.fromhex(v["file_hex"]))) as g:
            assert g.model_config() == v["expect"], case
    for case, code in (("config_no_arch", va.VA_ERR_INVALID), ("config_missing_heads", va.VA_ERR_NOT_FOUND)):
        v = VEC[case]
        with va.GgufFile(write(tmp_path, bytes.fromhex(v["file_hex"]))) as g:
            with pytest.raises(va.VestraError) as e:
                g.model_config()
            assert e.value.code == code and str(e.value).endswith(v["expect_message"])


def test_golden_misaligned_q8_0(lib, tmp_path):
    v = VEC["misaligned_q8_0"]
    with va.GgufFile(write(tmp_path, bytes.fromhex(v["file_hex"]))) as g:
        with pytest.raises(va.VestraError) as e:
            g.tensor_bytes(v["tensor"])
        assert e.value.code == va.VA_ERR_FORMAT and v["expect_message_contains"] in str(e.value)


def test_golden_e2e_tiny_tensor_bytes(lib, tmp_path):
    v = VEC["e2e_tiny"]
    with va.GgufFile(write(tmp_path, bytes.fromhex(v["file_hex"]))) as g:
        for name, t in v["tensors"].items():
            assert g.tensor_info(name)[:2] == (va.GGML_F32, t["shape"])
            np.testing.assert_array_equal(np.frombuffer(g.tensor_bytes(name), "<f4"), np.asarray(t["f32"], np.float32))


def test_open_errors(lib, tmp_path):
    with pytest.raises(va.VestraError) as e:
        va.GgufFile(str(tmp_path / "absent.gguf"))
    assert e.value.code == va.VA_ERR_IO
    for data, code, msg in ((b"", va.VA_ERR_FORMAT, "malformed: eof"),
                            (b"GGUX" + bytes(20), va.VA_ERR_FORMAT, "bad magic"),
                            (b"GGUF" + np.uint32(1).tobytes() + bytes(16), va.VA_ERR_FORMAT,
                             "unsupported gguf version 1")):
        with pytest.raises(va.VestraError) as e:
            va.GgufFile(write(tmp_path, data))
        assert e.value.code == code and str(e.value).endswith(msg)


def test_model_file_matches_oracle(lib, tmp_path):
    data = syn.gguf_model(embed=256, depth=2, heads=4, grid=4, num_register=2, dtype="q8_0")
    assert outcome_lib(write(tmp_path, data)) == outcome_oracle(data)


def test_every_truncation_matches_oracle(lib, tmp_path):
    data = small_model()
    for n in range(len(data) + 1):
        cut = data[:n]
        assert outcome_lib(write(tmp_path, cut)) == outcome_oracle(cut), n


def test_seeded_corruptions_match_oracle(lib, tmp_path):
    data = small_model()
    r = np.random.default_rng(1234)
    header_end = gguf.GgufFile(data).data_start
    for trial in range(400):
        b = bytearray(data)
        for _ in range(int(r.integers(1, 4))):
            i = int(r.integers(0, header_end))  # the parsed region
            b[i] = int(r.integers(0, 256)) if r.random() < 0.7 else b[i] ^ (1 << int(r.integers(0, 8)))
        b = bytes(b)
        assert outcome_lib(write(tmp_path, b)) == outcome_oracle(b), trial


def test_meta_getter_coercions(lib, tmp_path):
    w = syn.GgufWriter()
    w.kv_i32("k.i32", -5)
    w.kv_u32("k.u32", 0x80000001)
    w.kv_arr("k.au32", 4, [0xFFFFFFFF, 3])
    w.kv_u32("k.i32", 1)  # repeated: the first entry answers
    with va.GgufFile(write(tmp_path, w.to_bytes())) as g:
        assert g.meta_i32("k.i32") == -5 and g.meta_u32("k.i32") == 2 ** 32 - 5
        assert g.meta_i32("k.u32") == -(2 ** 31) + 1
        assert g.meta_arr_i32("k.au32") == [-1, 3] and g.meta_arr_u32("k.au32") == [0xFFFFFFFF, 3]
        assert g.meta_f32("k.i32") is None and g.meta_str("absent") is None
        assert g.meta_arr_f32("k.au32") is None
