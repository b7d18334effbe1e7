"""The C ABI library: loads without a GPU, exports every declared symbol, and its
host-only logic (view scheduling, config validation) matches the reference's
known answers.  No compute calls (CPU only)."""
import ctypes
import json
import os
import re
import subprocess

import numpy as np
import pytest

import vestra_attn as va

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER_DIR = os.path.join(ROOT, "include")


def declared_symbols():
    names = set()
    for fn in os.listdir(HEADER_DIR):
        if fn.endswith(".h"):
            with open(os.path.join(HEADER_DIR, fn)) as f:
                text = re.sub(r"/\*.*?\*/", "", f.read(), flags=re.S)
            names |= set(re.findall(r"\b(va_[a-z0-9_]+)\s*\(", text))
    return names


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(va.LIB_PATH):
        import __graft_entry__  # noqa: F401
        __graft_entry__.build()
    return va.load_library()


def test_every_declared_symbol_is_exported(lib):
    out = subprocess.run(["nm", "-D", "--defined-only", va.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    declared = declared_symbols()
    assert declared, "no declarations found"
    missing = declared - exported
    assert not missing, f"declared but not exported: {sorted(missing)}"
    assert set(va.EXPORTED) == declared, "python mirror and header disagree"
    for name in declared:
        getattr(lib, name)


def test_version_and_defaults(lib):
    assert b"sm_100a" in lib.va_version()
    cfg = va.default_config()
    assert (cfg.embed_dim, cfg.num_heads, cfg.head_dim) == (768, 12, 64)
    assert abs(cfg.qk_norm_eps - 1e-5) < 1e-12 and abs(cfg.rope_freq - 100.0) < 1e-6
    assert cfg.rope_start == 4 and cfg.qknorm_start == 4


def test_unsupported_config_is_rejected_before_touching_a_device(lib):
    h = ctypes.c_void_p()
    for bad in (dict(head_dim=32), dict(embed_dim=640, num_heads=10), dict(max_rows=0), dict(rope_pairing=2)):
        cfg = va.default_config(**bad)
        assert lib.va_create(ctypes.byref(cfg), 0, ctypes.byref(h)) == va.VA_ERR_INVALID
        assert not h.value


def test_view_scheduling_matches_reference_vectors(lib):
    with open(os.path.join(ROOT, "tests", "golden", "reference_vectors.json")) as f:
        v = json.load(f)
    assert va.select_reference_view_saddle(np.array(v["saddle"]["cls"], np.float32)) == v["saddle"]["reference"]
    for case in v["reference_first_order"]:
        assert va.reference_first_order(case["views"], case["reference"]) == case["order"]
    r = v["restore"]
    assert va.restore_original_view_order(r["ordered"], r["reference"]) == r["restored"]


def test_restore_inverts_reference_first_order(lib):
    for views in range(1, 9):
        for ref in range(views):
            order = va.reference_first_order(views, ref)
            assert sorted(order) == list(range(views))
            assert va.restore_original_view_order([order[i] for i in range(views)], ref) == list(range(views))


def test_saddle_selection_is_deterministic_and_keeps_earliest_tie(lib):
    cls = np.tile(np.array([[0.3, -0.2, 0.5, 0.1]], np.float32), (4, 1))
    assert va.select_reference_view_saddle(cls) == 0
    assert va.select_reference_view_saddle(np.ones((1, 8), np.float32)) == 0


def test_host_entry_points_reject_bad_arguments(lib):
    buf = (ctypes.c_int * 4)()
    assert lib.va_reference_first_order(4, 4, buf) == va.VA_ERR_INVALID
    assert lib.va_reference_first_order(0, 0, buf) == va.VA_ERR_INVALID
    out = ctypes.c_int()
    assert lib.va_select_reference_view_saddle(None, 3, 4, ctypes.byref(out)) == va.VA_ERR_INVALID


def test_positions_mirror(lib):
    p = va.positions_yx(2 * 8, 2, 2, 2, 3, False)
    assert p.shape == (16, 2)
    np.testing.assert_array_equal(p[2], [1, 1])
    np.testing.assert_array_equal(p[7], [2, 3])
    with pytest.raises(ValueError):
        va.positions_yx(15, 2, 2, 2, 3, False)


def test_shard_rows():
    assert va.shard_rows(10392, 8, 3) == (3 * 1299, 1299)
    assert va.shard_rows(10392, 1, 0) == (0, 10392)
    with pytest.raises(ValueError):
        va.shard_rows(10392, 5, 0)


def test_shard_views_splits_whole_views_evenly():
    # 12 views on 8 GPUs: 2,2,2,2,1,1,1,1 whole views, contiguous and in order.
    spans = [va.shard_views(12, 866, 8, r) for r in range(8)]
    assert [s[1] // 866 for s in spans] == [2, 2, 2, 2, 1, 1, 1, 1]
    assert [s[0] for s in spans] == [0, 1732, 3464, 5196, 6928, 7794, 8660, 9526]
    assert spans[-1][0] + spans[-1][1] == 12 * 866
    with pytest.raises(ValueError):
        va.shard_views(3, 866, 4, 0)
