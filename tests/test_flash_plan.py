"""The attention launch plan (va_flash_plan): which kernel form, units, key split and
grid the library picks for a call, computed on the host without a GPU.  The cases
are the bench's workloads on a 148-SM B200: the S=12 window (10,392 tokens, 12
heads) whole, sliced over 2, 4 and 8 ranks, and in local mode (12 views of 866)."""
import os

import pytest

import vestra_attn as va

SMS = 148
ROWS, HEADS = 10392, 12


@pytest.fixture(scope="module", autouse=True)
def lib():
    if not os.path.exists(va.LIB_PATH):
        import __graft_entry__  # noqa: F401
        __graft_entry__.build()
    return va.load_library()


def plan(q, **kw):
    kw.setdefault("sms", SMS)
    return va.flash_plan(q, ROWS, HEADS, **kw)


def test_local_views_take_the_one_tile_form():
    p = plan(ROWS, seg_len=866)
    assert (p["form"], p["poly"], p["kernel"]) == (15, 1, "flash_fwd_d64_ks1_kernel")
    # 7 query tiles of 128 per 866-token view (896 slots), every head, every view
    assert p["unit_rows"] == 128 and p["grid"] == (7, HEADS, 12) and p["splits"] == 1


def test_full_window_takes_the_two_tile_form_with_a_split_tail():
    p = plan(ROWS)
    assert (p["form"], p["poly"], p["kernel"]) == (10, 1, "flash_fwd_d64_ks_kernel")
    # 41 query pairs x 12 heads = 492 units: 444 whole (3 waves) and the last 48 cut
    # into 3 key ranges (one third of a wave each)
    assert p["unit_rows"] == 256 and p["n_full"] == 444 and p["splits"] == 3 and p["grid"] == (588, 1, 1)


@pytest.mark.parametrize("rank", [0, 1])
def test_half_window_slice_takes_the_one_tile_form(rank):
    p = plan(ROWS // 2, q_offset=rank * ROWS // 2)
    assert p["form"] == 15 and p["per_sm"] == 2
    # 492 one-tile units on 296 slots: 296 whole, the other 196 cut into 3 key ranges
    assert p["n_full"] == 296 and p["splits"] == 3 and p["grid"] == (884, 1, 1)


def test_quarter_and_eighth_slices_keep_the_two_tile_form():
    q4 = plan(ROWS // 4)
    assert q4["form"] == 10 and q4["splits"] == 1 and q4["grid"] == (132, 1, 1)  # one wave, no split pays
    q8 = plan(1299)
    assert q8["form"] == 10 and q8["n_full"] == 0 and q8["splits"] == 2 and q8["grid"] == (144, 1, 1)


def test_row_max_layers_take_the_w20_layout():
    p = plan(ROWS, fixed_offset=False)
    assert (p["form"], p["kernel"]) == (3, "flash_fwd_d64_w20_kernel") and p["grid"] == (588, 1, 1)


def test_persistent_form_walks_one_cta_per_sm():
    p = plan(ROWS, variant=256 + 8 * 14 + 1)
    assert p["kernel"] == "flash_fwd_d64_ksp_kernel" and p["grid"] == (SMS, 1, 1)


def test_explicit_variants_and_the_default_marker():
    assert plan(ROWS, variant=511) == plan(ROWS)  # 511: the fixed offset, library default
    assert plan(ROWS, variant=256 + 8 * 15 + 2)["form"] == 15
    assert plan(ROWS, seg_len=866, variant=256 + 8 * 10 + 1)["grid"] == (4, HEADS, 12)  # pairs: 1,024 slots


@pytest.mark.parametrize("kw", [dict(variant=256 + 8 * 15 + 3),           # form 15 has KA <= 80
                                dict(variant=8 * 10 + 1, fixed_offset=False),  # key split needs the offset
                                dict(seg_len=865),                           # views must tile the rows
                                dict(sms=0)])
def test_rejected_plans(kw):
    with pytest.raises(va.VestraError):
        plan(ROWS, **kw)
