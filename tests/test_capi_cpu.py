"""CPU-only checks of the C-ABI library: it loads, exports every symbol the
header declares, computes the reference's blob layout, and rejects bad
arguments with a status code before touching the GPU."""

from __future__ import annotations

import ctypes as C

import pytest

from conftest import GOLDEN


def test_library_exports_every_declared_symbol(q3):
    lib = q3._lib.lib()
    declared = q3._lib.declared_symbols()
    assert len(declared) >= 20
    missing = [s for s in declared if not hasattr(lib, s)]
    assert not missing, missing


def test_layout_matches_reference_pqwf():
    """tools/pqwf.py Layout().compute().header_text(), written by gen_golden.py."""
    import q3b200.model as M
    assert M.header_text(M.Dims()) == (GOLDEN / "layout_default.h").read_text()
    assert M.header_text(M.Dims(layers=1, vocab=1024)) == (GOLDEN / "layout_cfg1.h").read_text()


def test_layout_weight_offsets_match_checked_in_header():
    """The weights part of config/model_big.h (offsets up to kHS) is
    reproduced; the activation scratch and KV-scale sizes of the checked-in
    header predate the per-group/per-head scales of pqwf.py, whose layout is
    the authoritative one (test above)."""
    import q3b200.model as M
    _, off = M.layout(M.Dims())
    expected = {"kEMB": 132112, "kLM": 156322320, "kCOS": 312516624,
                "kLAYERW_STRIDE": 15777792, "kLO": 316858384, "kLD_SCALE": 328421392,
                "kLAYERN_BASE": 754425872, "kN2": 754430992, "kLOGITS": 754683920,
                "kH": 774176768, "kH8": 774307840, "kHS": 774340608}
    for k, v in expected.items():
        assert off[k] == v, k


def _null_view():
    from q3b200._lib import View
    return View(None, 0, 0, 0, 0, 0)


def test_bad_arguments_return_status(q3):
    lib = q3._lib.lib()
    from q3b200._lib import View
    v = _null_view()
    # null views -> Q3_ERR_NULL, nothing launched (no GPU needed)
    assert lib.q3_rmsnorm_rows(C.byref(v), C.byref(v), C.byref(v), 1.0, None) == 1
    assert lib.q3_quant_rows_heads(C.byref(v), C.byref(v), C.byref(v), 256, None) == 1
    # wrong dtype on a non-null view -> Q3_ERR_DTYPE
    bogus = View(0x1000, 4096, 4, 1, 1024, 0)   # dtype i8 where f32 is required
    assert lib.q3_rmsnorm_rows(C.byref(bogus), C.byref(bogus), C.byref(bogus), 1.0, None) == 4
    # K not a multiple of the group -> Q3_ERR_SHAPE
    a = View(0x1000, 1000, 1, 4, 1000, 0)
    asc = View(0x2000, 16, 4, 4, 4, 4)
    b = View(0x3000, 1024, 1, 128, 1024, 0)
    bs = View(0x4000, 4, 4, 128, 1, 4)
    out = View(0x5000, 512, 4, 4, 128, 4)
    rc = lib.q3_gemm_nt_group_store(C.byref(a), C.byref(asc), C.byref(b), C.byref(bs),
                                    C.byref(out), 256, None, None, None, None, None, None,
                                    0.0, None)
    assert rc in (3, 5)
    # head_dim other than 128 -> Q3_ERR_SHAPE
    q = View(0x1000, 2048, 1, 1, 2048, 0)
    qs = View(0x2000, 64, 4, 1, 16, 4)
    from q3b200._lib import PagedKV
    kv = PagedKV(0x10000, 0x20000, 0x30000, 0x40000, 0x50000, 32, 32768, 1024, 1024, 32)
    assert lib.q3_attention_heads_gqa_tokscale_paged(C.byref(q), C.byref(qs), C.byref(kv), 8,
                                                     C.byref(q), C.byref(qs), 16, 8, 64, 1,
                                                     0.125, None) == 3


def test_generate_rejects_bad_workspace(q3):
    import q3b200.model as M
    lib = q3._lib.lib()
    L, _ = M.layout(M.Dims(layers=1, vocab=1024))
    assert lib.q3_generate(C.c_void_p(0x1000), C.byref(L), None, 0, None) == 1
    assert lib.q3_generate(C.c_void_p(0x1000), C.byref(L), C.c_void_p(0x100000), 8, None) == 7
