"""The GGUF oracle (oracle/gguf.py) against the known answers of the reference's
own tests (tests/golden/gguf_vectors.json), and the test-side writer
(synthetic.GgufWriter) against the oracle.  CPU only."""
import json
import os
import struct

import numpy as np
import pytest

import gguf
import synthetic as syn

HERE = os.path.dirname(os.path.abspath(__file__))
with open(os.path.join(HERE, "golden", "gguf_vectors.json")) as f:
    VEC = json.load(f)

KIND = {"u32": gguf.U32, "i32": gguf.I32}


def test_q8_0_block_matches_scale_times_quants():
    v = VEC["q8_0_block"]
    d, qs = gguf.read_blocks(bytes.fromhex(v["block_hex"]), 32)
    out = gguf.dequantize_q8_0(d, qs)
    np.testing.assert_array_equal(out, np.asarray(v["expect_f32"], np.float32))


@pytest.mark.parametrize("case", ["bool_array_skip", "u16_array_skip"])
def test_unmodeled_array_is_skipped_and_the_cursor_lands_on_the_sentinel(case):
    v = VEC[case]
    kv = bytes.fromhex(v["kv_hex"])
    c = gguf._Cursor(kv)
    c.string()
    assert gguf.read_kv_value(c, c.u32()) is None
    key = c.string()
    kind, val = gguf.read_kv_value(c, c.u32())
    assert [key, kind, val] == [v["expect_kv"][0][0], KIND[v["expect_kv"][0][1]], v["expect_kv"][0][2]]
    assert c.p == len(kv)
    f = gguf.GgufFile(bytes.fromhex(v["file_hex"]))
    assert [(k, kind, val) for k, kind, val in f.kv] == [(e[0], KIND[e[1]], e[2]) for e in v["expect_kv"]]


def test_misaligned_q8_0_tensor_is_rejected():
    v = VEC["misaligned_q8_0"]
    f = gguf.GgufFile(bytes.fromhex(v["file_hex"]))
    with pytest.raises(gguf.GgufError) as e:
        f.tensor_f32(v["tensor"])
    assert e.value.kind == v["expect_error"] and v["expect_message_contains"] in str(e.value)
    with pytest.raises(gguf.GgufError):
        f.tensor_q8_0(v["tensor"])


@pytest.mark.parametrize("case", ["config_full", "config_alt4", "config_cat_off", "e2e_tiny"])
def test_model_config_known_answers(case):
    v = VEC[case]
    cfg = gguf.model_config(gguf.GgufFile(bytes.fromhex(v["file_hex"])))
    assert cfg == v["expect"]


@pytest.mark.parametrize("case", ["config_no_arch", "config_missing_heads"])
def test_model_config_errors(case):
    v = VEC[case]
    with pytest.raises(gguf.ConfigError) as e:
        gguf.model_config(gguf.GgufFile(bytes.fromhex(v["file_hex"])))
    assert e.value.kind == v["expect_error"] and str(e.value) == v["expect_message"]


def test_e2e_tiny_tensors_are_flat_f32_and_not_transposed():
    v = VEC["e2e_tiny"]
    f = gguf.GgufFile(bytes.fromhex(v["file_hex"]))
    w = gguf.weights_from_gguf(f)
    assert f.tensor_names() == list(v["tensors"])
    for name, t in v["tensors"].items():
        assert f.tensor_shape(name) == t["shape"]
        np.testing.assert_array_equal(w[name], np.asarray(t["f32"], np.float32))


def test_header_errors():
    with pytest.raises(gguf.GgufError) as e:
        gguf.GgufFile(b"GGUX" + bytes(20))
    assert e.value.kind == "bad_magic" and str(e.value) == "bad magic"
    with pytest.raises(gguf.GgufError) as e:
        gguf.GgufFile(b"GGUF" + struct.pack("<IQQ", 4, 0, 0))
    assert str(e.value) == "unsupported gguf version 4"
    for n in range(0, 24):  # every truncation of a valid empty header
        with pytest.raises(gguf.GgufError) as e:
            gguf.GgufFile((b"GGUF" + struct.pack("<IQQ", 3, 0, 0))[:n])
        assert str(e.value) == "malformed: eof"


def test_writer_round_trip_every_value_type():
    w = syn.GgufWriter(version=2, alignment=64)
    w.kv_u8("a.u8", 200)
    w.kv_i8("a.i8", -1)        # read back zero-extended: 255 (`u8 as i32`)
    w.kv_u16("a.u16", 65535)
    w.kv_i16("a.i16", -2)
    w.kv_u32("a.u32", 0xFFFFFFFF)
    w.kv_i32("a.i32", -7)
    w.kv_f32("a.f32", 1.5)
    w.kv_bool("a.bool", True)
    w.kv_str("a.str", "héllo")
    w.kv_u64("a.u64", 2 ** 63 + 5)
    w.kv_i64("a.i64", -3)
    w.kv_f64("a.f64", 0.1)
    w.kv_arr("a.arr_u32", 4, [1, 2, 3])
    w.kv_arr("a.arr_i32", 5, [-1, 2])
    w.kv_arr("a.arr_f32", 6, [0.5, -0.25])
    w.kv_arr("a.arr_str", 8, ["x", "yz", ""])
    w.kv_arr("a.arr_f64", 12, [1.0, 2.0])   # skipped
    w.kv_arr("a.arr_bool", 7, [1, 0, 1])    # skipped
    w.kv_u32("a.u32", 9)                    # repeated key: the first entry answers
    f = gguf.GgufFile(w.to_bytes())
    assert f.version == 2 and f.alignment == 64
    assert f.meta_u32("a.u8") == 200 and f.meta_i32("a.i8") == 255
    assert f.meta_u32("a.u16") == 65535 and f.meta_i32("a.i16") == -2
    assert f.meta_u32("a.u32") == 0xFFFFFFFF and f.meta_i32("a.u32") == -1
    assert f.meta_i32("a.i32") == -7 and f.meta_u32("a.i32") == 2 ** 32 - 7
    assert f.meta_f32("a.f32") == 1.5 and f.meta_u32("a.f32") is None
    assert f.meta_bool("a.bool") is True and f.meta_str("a.str") == "héllo"
    assert f.meta_u64("a.u64") == 2 ** 63 + 5 and f.meta_u64("a.i64") == 2 ** 64 - 3
    assert f.meta_f32("a.f64") == float(np.float32(0.1))
    assert f.meta_arr_u32("a.arr_u32") == [1, 2, 3] and f.meta_arr_i32("a.arr_u32") == [1, 2, 3]
    assert f.meta_arr_i32("a.arr_i32") == [-1, 2] and f.meta_arr_u32("a.arr_i32") is None
    assert f.meta_arr_f32("a.arr_f32") == [0.5, -0.25]
    assert f.meta_arr_str("a.arr_str") == ["x", "yz", ""]
    assert f.meta("a.arr_f64") is None and f.meta("a.arr_bool") is None
    assert f.meta("missing") is None


def test_lossy_utf8_keys_and_strings():
    w = syn.GgufWriter()
    w.kv_raw(b"k\xff\xfe", 8, struct.pack("<Q", 4) + b"a\xe2\x82b")
    f = gguf.GgufFile(w.to_bytes())
    assert f.kv[0][0] == "k��" and f.kv[0][2] == "a�b"


@pytest.mark.parametrize("dtype", ["f32", "f16", "q8_0"])
def test_writer_tensors_and_weights_from_gguf(dtype):
    r = np.random.default_rng(3)
    m = r.standard_normal((96, 64)).astype(np.float32)  # [out, in]
    v = r.standard_normal(40).astype(np.float32)
    w = syn.GgufWriter()
    w.tensor("m", m, dtype)
    w.tensor("v3", v[:32].reshape(1, 4, 8), dtype)
    w.tensor("v", v, "f32")
    f = gguf.GgufFile(w.to_bytes())
    shape, got = f.tensor_f32("m")
    assert shape == [96, 64]
    if dtype == "f32":
        np.testing.assert_array_equal(got, m.reshape(-1))
    elif dtype == "f16":
        np.testing.assert_array_equal(got, m.astype(np.float16).astype(np.float32).reshape(-1))
    else:
        # Q8_0: |error| <= d/2 + 127 |d16 - d| per block, d = max|x| / 127 rounded to f16 as d16
        d = np.abs(m.reshape(-1, 32)).max(axis=1, keepdims=True) / np.float32(127)
        d16 = d.astype(np.float16).astype(np.float32)
        assert np.all(np.abs(got.reshape(-1, 32) - m.reshape(-1, 32)) <= d * 0.5 + 127 * np.abs(d16 - d) + 1e-7)
        _, dd, qs = f.tensor_q8_0("m")
        np.testing.assert_array_equal(gguf.dequantize_q8_0(dd, qs), got)
    wts = gguf.weights_from_gguf(f)
    np.testing.assert_array_equal(wts["m"], got.reshape(96, 64).T.reshape(-1))  # rank 2: transposed
    np.testing.assert_array_equal(wts["v3"], f.tensor_f32("v3")[1])              # rank 3: as stored
    np.testing.assert_array_equal(wts["v"], v)
    # every tensor starts at an aligned offset
    assert all((f.data_start + t[3]) % 32 == 0 for t in f.tensors)


def test_tensor_errors():
    w = syn.GgufWriter()
    w.tensor("ok", np.zeros(32, np.float32))
    w.tensor_raw("bf16", bytes(64), 30, [32])
    w.tensor_raw("past_end", bytes(16), 0, [1000])
    f = gguf.GgufFile(w.to_bytes())
    with pytest.raises(gguf.GgufError) as e:
        f.tensor_f32("nope")
    assert e.value.kind == "not_found" and str(e.value) == "tensor not found: nope"
    with pytest.raises(gguf.GgufError) as e:
        f.tensor_f32("bf16")
    assert e.value.kind == "dtype" and str(e.value) == "unsupported dtype 30"
    with pytest.raises(gguf.GgufError) as e:
        f.tensor_f32("past_end")
    assert e.value.kind == "malformed" and "data out of bounds" in str(e.value)
