"""Operator parity on the GPU, through the C ABI: every operator of the
reference's API against the oracle and the golden vectors made by the
reference's own numpy mirror.  Integer/int8 results and float32 results are
compared bit for bit (the path's floats are rounded exactly as the
reference's), which is stricter than the 1e-3 relative tolerance allowed for f32 stages."""

from __future__ import annotations

import numpy as np
import pytest

from conftest import load_golden

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
F = np.float32


@pytest.fixture(scope="module")
def ops(q3):
    assert torch.cuda.is_available(), "GPU tests need CUDA"
    return q3.ops


@pytest.fixture(scope="module")
def gold():
    return load_golden("ops_cr.npz")


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def same_bits(a, b):
    a, b = np.asarray(a), np.asarray(b)
    assert a.shape == b.shape, (a.shape, b.shape)
    if a.dtype == np.float32:
        bad = np.count_nonzero(a.view(np.uint32) != np.asarray(b, F).view(np.uint32))
    else:
        bad = np.count_nonzero(a != b)
    assert bad == 0, f"{bad}/{a.size} elements differ"


from oracle import q3_oracle as O  # noqa: E402


# ---------------------------------------------------------------- GEMM family
@pytest.mark.parametrize("tag,group", [("g256", 256), ("g128", 128), ("m1", 256)])
def test_gemm_store_golden(ops, gold, tag, group):
    a, as_, w, ws = (gold[f"gemm_{tag}_{k}"] for k in ("a", "as", "w", "ws"))
    out = torch.zeros(a.shape[0], w.shape[0], dtype=torch.float32, device="cuda")
    ops.gemm_nt_group_store(dev(a), dev(as_), dev(w), dev(ws), out, group)
    same_bits(host(out), gold[f"gemm_{tag}_out"])


def _rand_gemm(rng, m, k, n, g):
    a = rng.integers(-127, 128, (m, k)).astype(np.int8)
    w = rng.integers(-127, 128, (n, k)).astype(np.int8)
    as_ = rng.uniform(1e-3, 1e-2, (m, k // g)).astype(F)
    ws = rng.uniform(1e-3, 1e-2, n).astype(F)
    return a, as_, w, ws


@pytest.mark.parametrize("m,k,n,g", [(1, 1024, 2048, 256), (32, 2048, 1024, 128),
                                     (7, 3072, 1024, 256), (64, 1024, 6144, 256),
                                     (33, 1024, 256, 128)])
def test_gemm_store_add_random(ops, m, k, n, g):
    rng = np.random.default_rng(m * 7 + n)
    a, as_, w, ws = _rand_gemm(rng, m, k, n, g)
    ref = O.gemm_group(a, as_, w, ws, g)
    out = torch.zeros(m, n, dtype=torch.float32, device="cuda")
    ops.gemm_nt_group_store(dev(a), dev(as_), dev(w), dev(ws), out, g)
    same_bits(host(out), ref)
    x0 = rng.standard_normal((m, n)).astype(F)
    x = dev(x0)
    ops.gemm_nt_group_store(dev(a), dev(as_), dev(w), dev(ws), None, g, add=x)
    same_bits(host(x), (x0 + ref).astype(F))


def test_gemm_quant_epilogue(ops):
    rng = np.random.default_rng(5)
    m, k, n = 9, 1024, 1024
    a, as_, w, ws = _rand_gemm(rng, m, k, n, 256)
    ref8, refs = O.quant_groups(O.gemm_group(a, as_, w, ws, 256), 128)
    q8 = torch.zeros(m, n, dtype=torch.int8, device="cuda")
    qs = torch.zeros(m, n // 128, dtype=torch.float32, device="cuda")
    ops.gemm_nt_group_store(dev(a), dev(as_), dev(w), dev(ws), None, 256, q8=q8, qs=qs)
    same_bits(host(q8), ref8)
    same_bits(host(qs), refs)


@pytest.mark.parametrize("m,n,pos", [(32, 1024, 0), (8, 2048, 32), (1, 1024, 200)])
def test_gemm_norm_rope_quant_epilogue(ops, m, n, pos):
    from oracle import synth
    rng = np.random.default_rng(n + m)
    a, as_, w, ws = _rand_gemm(rng, m, 1024, n, 256)
    nw = (1 + 0.05 * rng.standard_normal(128)).astype(F)
    cos, sin = synth.rope_tables(256, 128)
    y = O.gemm_group(a, as_, w, ws, 256)
    _, ref8, refs = O.qk_norm_rope_quant(y, nw, cos[pos:pos + m], sin[pos:pos + m], n // 128, 128)
    q8 = torch.zeros(m, n, dtype=torch.int8, device="cuda")
    qs = torch.zeros(m, n // 128, dtype=torch.float32, device="cuda")
    ops.gemm_nt_group_store(dev(a), dev(as_), dev(w), dev(ws), None, 256, q8=q8, qs=qs,
                            nw=dev(nw), cos=dev(cos[pos:pos + m]), sin=dev(sin[pos:pos + m]),
                            inv_hd=float(F(1) / F(128)))
    same_bits(host(q8), ref8)
    same_bits(host(qs), refs)


def test_gate_up_swiglu_quant_guest_fixture(ops, gold):
    a, as_ = gold["guest_gu_a"], gold["guest_gu_as"]
    s8 = torch.zeros(32, 256, dtype=torch.int8, device="cuda")
    ss = torch.zeros(32, 1, dtype=torch.float32, device="cuda")
    ops.gemm_gate_up_swiglu_quant(dev(a), dev(as_), dev(gold["guest_gu_wg"]),
                                  dev(gold["guest_gu_wgs"]), dev(gold["guest_gu_wu"]),
                                  dev(gold["guest_gu_wus"]), s8, ss, 256)
    same_bits(host(s8), gold["guest_gu_s8"])
    same_bits(host(ss), gold["guest_gu_ss"])


@pytest.mark.parametrize("m", [1, 5, 32, 64])
def test_gate_up_swiglu_quant_random(ops, m):
    rng = np.random.default_rng(m)
    a, as_, wg, wgs = _rand_gemm(rng, m, 1024, 3072, 256)
    wu = rng.integers(-127, 128, (3072, 1024)).astype(np.int8)
    wus = rng.uniform(1e-3, 1e-2, 3072).astype(F)
    g = O.gemm_group(a, as_, wg, wgs, 256)
    u = O.gemm_group(a, as_, wu, wus, 256)
    ref8, refs = O.quant_groups(O.swiglu(g, u), 256)
    s8 = torch.zeros(m, 3072, dtype=torch.int8, device="cuda")
    ss = torch.zeros(m, 12, dtype=torch.float32, device="cuda")
    ops.gemm_gate_up_swiglu_quant(dev(a), dev(as_), dev(wg), dev(wgs), dev(wu), dev(wus), s8, ss,
                                  256)
    same_bits(host(s8), ref8)
    same_bits(host(ss), refs)


def test_guest_group_gemm_fixture(ops, gold):
    out = torch.zeros(32, 128, dtype=torch.float32, device="cuda")
    ops.gemm_nt_group_store(dev(gold["guest_gg_a"]), dev(np.ones((32, 2), F)),
                            dev(gold["guest_gg_b"]), dev(np.ones(128, F)), out, 128)
    same_bits(host(out), gold["guest_gg_out"])


@pytest.mark.parametrize("m", [1, 3, 40])
def test_lm_head_argmax(ops, m):
    rng = np.random.default_rng(11 + m)
    a, as_, w, ws = _rand_gemm(rng, m, 1024, 4096, 256)
    w[1234] = w[77]                       # duplicate rows -> tied maxima
    ws[1234] = ws[77]
    logits = O.gemm_group(a, as_, w, ws, 256)
    best = dev(np.full(m, -3.0e38, F))
    bidx = dev(np.zeros(m, np.int32))
    ops.gemm_nt_group_argmax(dev(a), dev(as_), dev(w), dev(ws), best, bidx, 256)
    gb, gi = host(best), host(bidx)
    for r in range(m):
        assert gi[r] == int(np.argmax(logits[r]))
        same_bits(gb[r:r + 1], logits[r].max(keepdims=True))


# ---- the per-group GEMM microbench shapes (prefill-size GEMMs) ------------------
# M beyond 64 takes the wide token tiles; 700 leaves a ragged last tile; from
# 1024 rows the CTA-pair kernel runs (1100: a ragged last 256-token tile).
@pytest.mark.parametrize("m", [512, 700, 1100, 4096])
@pytest.mark.parametrize("k,n,g", [(1024, 2048, 256), (2048, 1024, 128), (3072, 1024, 256)])
def test_gemm_config2_store_add(ops, m, k, n, g):
    rng = np.random.default_rng(m + k + n)
    a, as_, w, ws = _rand_gemm(rng, m, k, n, g)
    ref = O.gemm_group(a, as_, w, ws, g)
    out = torch.zeros(m, n, dtype=torch.float32, device="cuda")
    ops.gemm_nt_group_store(dev(a), dev(as_), dev(w), dev(ws), out, g)
    same_bits(host(out), ref)
    x0 = rng.standard_normal((m, n)).astype(F)
    x = dev(x0)
    ops.gemm_nt_group_store(dev(a), dev(as_), dev(w), dev(ws), None, g, add=x)
    same_bits(host(x), (x0 + ref).astype(F))


# The CTA-pair kernel's residual shapes of the tensor-parallel prefill (the O and
# down GEMMs of one rank at 2 and 4 GPUs: 512 or 256 output columns, one or two
# pair tiles) and a token count one past a 192-token tile boundary.
@pytest.mark.parametrize("m,k,n,g", [(1025, 2048, 256, 128), (1151, 3072, 512, 256),
                                     (1344, 2048, 512, 128)])
def test_gemm_pair_residual_shapes(ops, m, k, n, g):
    rng = np.random.default_rng(m + 3 * n)
    a, as_, w, ws = _rand_gemm(rng, m, k, n, g)
    ref = O.gemm_group(a, as_, w, ws, g)
    x0 = rng.standard_normal((m, n)).astype(F)
    x = dev(x0)
    ops.gemm_nt_group_store(dev(a), dev(as_), dev(w), dev(ws), None, g, add=x)
    same_bits(host(x), (x0 + ref).astype(F))


@pytest.mark.parametrize("m", [512, 700, 1100, 4096])
def test_gate_up_swiglu_config2(ops, m):
    rng = np.random.default_rng(100 + m)
    a, as_, wg, wgs = _rand_gemm(rng, m, 1024, 3072, 256)
    wu = rng.integers(-127, 128, (3072, 1024)).astype(np.int8)
    wus = rng.uniform(1e-3, 1e-2, 3072).astype(F)
    ref8, refs = O.quant_groups(O.swiglu(O.gemm_group(a, as_, wg, wgs, 256),
                                         O.gemm_group(a, as_, wu, wus, 256)), 256)
    s8 = torch.zeros(m, 3072, dtype=torch.int8, device="cuda")
    ss = torch.zeros(m, 12, dtype=torch.float32, device="cuda")
    ops.gemm_gate_up_swiglu_quant(dev(a), dev(as_), dev(wg), dev(wgs), dev(wu), dev(wus), s8, ss,
                                  256)
    same_bits(host(s8), ref8)
    same_bits(host(ss), refs)


@pytest.mark.parametrize("m", [200, 700, 1100, 2048])
def test_gemm_head_epilogues_wide_tiles(ops, m):
    from oracle import synth
    rng = np.random.default_rng(200 + m)
    a, as_, w, ws = _rand_gemm(rng, m, 1024, 2048, 256)
    y = O.gemm_group(a, as_, w, ws, 256)
    q8 = torch.zeros(m, 2048, dtype=torch.int8, device="cuda")
    qs = torch.zeros(m, 16, dtype=torch.float32, device="cuda")
    ops.gemm_nt_group_store(dev(a), dev(as_), dev(w), dev(ws), None, 256, q8=q8, qs=qs)
    ref8, refs = O.quant_groups(y, 128)
    same_bits(host(q8), ref8)
    same_bits(host(qs), refs)
    nw = (1 + 0.05 * rng.standard_normal(128)).astype(F)
    cos, sin = synth.rope_tables(m + 8, 128)
    cos, sin = cos[8:8 + m], sin[8:8 + m]
    _, ref8, refs = O.qk_norm_rope_quant(y, nw, cos, sin, 16, 128)
    ops.gemm_nt_group_store(dev(a), dev(as_), dev(w), dev(ws), None, 256, q8=q8, qs=qs,
                            nw=dev(nw), cos=dev(np.ascontiguousarray(cos)),
                            sin=dev(np.ascontiguousarray(sin)), inv_hd=float(F(1) / F(128)))
    same_bits(host(q8), ref8)
    same_bits(host(qs), refs)


@pytest.mark.parametrize("m", [1, 32])
def test_lm_head_argmax_config2(ops, m):
    rng = np.random.default_rng(300 + m)
    a, as_, w, ws = _rand_gemm(rng, m, 1024, 151936, 256)
    logits = O.gemm_group(a, as_, w, ws, 256)
    best = dev(np.full(m, -3.0e38, F))
    bidx = dev(np.zeros(m, np.int32))
    ops.gemm_nt_group_argmax(dev(a), dev(as_), dev(w), dev(ws), best, bidx, 256)
    gb, gi = host(best), host(bidx)
    for r in range(m):
        assert gi[r] == int(np.argmax(logits[r]))
        same_bits(gb[r:r + 1], logits[r].max(keepdims=True))


def test_argmax_logits_golden(ops, gold):
    out = dev(np.zeros(1, np.int32))
    ops.argmax_logits(dev(gold["argmax_logits"]), out)
    assert int(host(out)[0]) == int(gold["argmax_idx"])


# ---------------------------------------------------------------- row ops
@pytest.mark.parametrize("group", [256, 128])
def test_quant_rows_heads_golden(ops, gold, group):
    x = gold["quant_x"]
    q = torch.zeros(x.shape, dtype=torch.int8, device="cuda")
    s = torch.zeros(x.shape[0], x.shape[1] // group, dtype=torch.float32, device="cuda")
    ops.quant_rows_heads(dev(x), q, s, group)
    same_bits(host(q), gold[f"quant_q{group}"])
    same_bits(host(s), gold[f"quant_s{group}"])


def _near_tie_rows(seed=77):
    """Rows of 256 whose first column fixes the group's absmax A (so the scale
    is RN(A / 127 ...)) and whose other columns sit within 3 ulps of (k + 1/2)
    times that scale: the quotients land on or next to the rounding ties of
    the int8 quantisation.  Magnitudes from subnormal to 1e30, plus a zero row
    (scale 0: every quotient is NaN -> 0)."""
    rng = np.random.default_rng(seed)
    rows = []
    for a in [1.0, 3.7e-3, 1234.5, 2.0 ** -120, 1e30, 0.5, 2.0 ** -140, 9.99e-8]:
        a = F(a)
        scale = F(a * O.INV127)
        k = rng.integers(-126, 127, 255).astype(np.float64)
        x = ((k + 0.5) * np.float64(scale)).astype(F)
        for i, n in enumerate(rng.integers(-3, 4, 255)):
            for _ in range(abs(int(n))):
                x[i] = np.nextafter(x[i], F(np.inf) if n > 0 else F(-np.inf))
        x = np.clip(x, -a, a)
        rows.append(np.concatenate([[a], x]).astype(F))
    rows.append(np.zeros(256, F))
    return np.stack(rows)


def test_quant_near_rounding_ties(ops):
    """The requantisation rounds from a reciprocal and falls back to the exact
    division near half-integers; it must match RN(x / scale) rounded to even
    everywhere (ref_qwen3.py:69-76)."""
    x = _near_tie_rows()
    ref8, refs = O.quant_groups(x, 256)
    q = torch.zeros(x.shape, dtype=torch.int8, device="cuda")
    s = torch.zeros(x.shape[0], 1, dtype=torch.float32, device="cuda")
    ops.quant_rows_heads(dev(x), q, s, 256)
    same_bits(host(s), refs)
    same_bits(host(q), ref8)


def test_rmsnorm_golden(ops, gold):
    for xk, wk, ok, inv in (("rms_x", "rms_w", "rms_out", F(1) / F(1024)),
                            ("rmsh_x", "rmsh_w", "rmsh_out", F(1) / F(128))):
        x = gold[xk]
        out = torch.zeros(x.shape, dtype=torch.float32, device="cuda")
        ops.rmsnorm_rows(dev(x), dev(gold[wk]), out, float(inv))
        same_bits(host(out), gold[ok])
        xin = dev(x)                         # in place (out aliases x)
        ops.rmsnorm_rows(xin, dev(gold[wk]), xin, float(inv))
        same_bits(host(xin), gold[ok])


def test_embedding_rmsnorm_golden(ops, gold):
    ids = gold["emb_ids"]
    x = torch.zeros(len(ids), 1024, dtype=torch.float32, device="cuda")
    h = torch.zeros_like(x)
    ops.embedding_rmsnorm_rows(dev(gold["emb_t"]), dev(gold["emb_s"]), dev(ids), x,
                               dev(gold["emb_w"]), h, float(F(1) / F(1024)))
    same_bits(host(x), gold["emb_x"])
    same_bits(host(h), gold["emb_h"])


def test_exp_correctly_rounded(ops):
    from oracle.exp2 import exp2_cr
    import re
    from pathlib import Path
    inc = (Path(__file__).resolve().parent.parent / "qwen3-tile-ops_b200" / "csrc" /
           "exp2_hard_table.inc").read_text()
    xs = re.search(r"HARD_X_INIT \{(.*?)\}", inc, re.S).group(1)
    hard = np.array([int(v, 16) for v in re.findall(r"0x([0-9a-f]+)u", xs)], np.uint32).view(F)
    rng = np.random.default_rng(0)
    pts = [hard, np.array([0.0, -0.0, 1.0, -1.0, 127.99, 128.0, -149.0, -150.0, -151.0,
                           np.inf, -np.inf, 1e-30, -1e-30, 88.0, -88.0], F),
           (rng.standard_normal(1 << 20) * 30).astype(F),
           rng.uniform(-150, 128, 1 << 20).astype(F),
           (rng.standard_normal(1 << 18) * 1e-6).astype(F)]
    x = np.concatenate(pts)
    x = np.concatenate([x, np.zeros((-x.size) % 64, F)]).reshape(-1, 64)
    y = torch.zeros(x.shape, dtype=torch.float32, device="cuda")
    ops.exp2_rows(dev(x), y)
    same_bits(host(y), exp2_cr(x))
    ops.exp_rows(dev(x), y)
    with np.errstate(over="ignore"):
        same_bits(host(y), O.exp_f32(x))


def test_exp2_short_evaluation_exhaustive(q3):
    """The short evaluation of the correctly rounded exp2 that every kernel
    uses (256-entry table, degree-4 polynomial) gives the same bits as the
    longer double-precision one (itself pinned above and to the mpmath
    hard-case table) on EVERY float32 input in [0, 128) and every negative
    one -- -0, -inf and the negative NaNs included, where the softmax's form
    for non-positive inputs is checked too: about 3.2e9 inputs."""
    lib = q3._lib.lib()
    count = torch.zeros(1, dtype=torch.int64, device="cuda")
    first = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    for lo, hi in ((0x00000000, 0x43000000), (0x80000000, 0xFFFFFFFF)):
        assert lib.q3_exp2_selfcheck(lo, hi, count.data_ptr(), first.data_ptr(), None) == 0
    torch.cuda.synchronize()
    bad = int(count.item())
    assert bad == 0, f"{bad} inputs differ, first bit pattern {int(first.item()) & 0xffffffff:#010x}"


def test_quant_from_reciprocal_exhaustive(q3):
    """The int8 codes the kernels form equal the IEEE quotient rounded by the
    float -> int conversion and saturated (ref_qwen3.py:69-76): the quotient
    rounded in float on EVERY float32 x, and the shared-reciprocal form
    (Markstein's correction, no clamp: the scale is amax / 127 of the values'
    own absolute maximum) on every x with |x| <= amax and NaN -- subnormals and
    the double-rounding ties at half-integers included -- for absolute maxima
    at powers of two, next to them, at and beyond the ends of the reciprocal's
    range, at 127 times a power of two and with seeded random mantissas."""
    lib = q3._lib.lib()
    rng = np.random.default_rng(7)
    amaxes = [0.0] + [2.0 ** e for e in (-94, -93, -40, -7, 0, 5, 40, 106, 108)]
    amaxes += [float(np.nextafter(F(2.0 ** e), F(0))) for e in (-7, 0, 3)]
    amaxes += [float(np.nextafter(F(2.0 ** e), F(np.inf))) for e in (-7, 0, 3)]
    amaxes += [float(F(127) * F(2.0) ** F(e)) for e in (-20, 0, 20)]
    amaxes += [float(F(m) * F(2.0) ** F(e)) for m, e in
               zip(rng.uniform(1.0, 2.0, 10), rng.integers(-80, 100, 10))]
    amaxes += [float(F(v)) for v in rng.uniform(1e-4, 1.0, 6)]
    count = torch.zeros(1, dtype=torch.int64, device="cuda")
    first = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    for am in amaxes:
        for lo, hi in ((0x00000000, 0x80000000), (0x80000000, 0xFFFFFFFF)):
            assert lib.q3_quant_selfcheck(lo, hi, am, count.data_ptr(), first.data_ptr(), None) == 0
    torch.cuda.synchronize()
    bad = int(count.item())
    assert bad == 0, f"{bad} codes differ, first bit pattern {int(first.item()) & 0xffffffff:#010x}"


# ---------------------------------------------------------------- attention
def _pool_from_contiguous(k8, ks, v8, vs, kv_heads, table):
    """Scatter contiguous K/V [T][kv_heads*128] into pages following `table`."""
    T, kw = k8.shape
    pages = max(table) + 1
    pk = np.zeros((pages, 32, kw), np.int8)
    pv = np.zeros((pages, 32, kw), np.int8)
    pks = np.zeros((pages, 32, kv_heads), F)
    pvs = np.zeros((pages, 32, kv_heads), F)
    for t in range(T):
        p, s = table[t // 32], t % 32
        pk[p, s], pv[p, s], pks[p, s], pvs[p, s] = k8[t], v8[t], ks[t], vs[t]
    return [dev(a) for a in (pk, pv, pks, pvs)] + [dev(np.asarray(table, np.uint16).view(np.int16))]


def _run_attn(ops, q8, qs, k8, ks, v8, vs, heads, kvh, table):
    pk, pv, pks, pvs, tab = _pool_from_contiguous(k8, ks, v8, vs, kvh, table)
    kv = ops.paged_kv(pk, pv, pks, pvs, tab, kvh)
    R = q8.shape[0]
    o8 = torch.zeros(R, heads * 128, dtype=torch.int8, device="cuda")
    os_ = torch.zeros(R, heads, dtype=torch.float32, device="cuda")
    ops.attention_heads_gqa_tokscale_paged(dev(q8), dev(qs), kv, k8.shape[0], o8, os_, heads, kvh,
                                           128, True, float(F(1.0 / np.sqrt(128.0))))
    keep = (pk, pv, pks, pvs, tab)
    return host(o8), host(os_), keep


@pytest.mark.parametrize("tag,heads,kvh", [("prefill40", 16, 8), ("decode", 16, 8),
                                            ("guestlike", 4, 2), ("first32", 16, 8)])
def test_attention_paged_golden(ops, gold, tag, heads, kvh):
    g = {k: gold[f"attn_{tag}_{k}"] for k in ("q8", "k8", "v8", "qs", "ks", "vs", "out")}
    T = g["k8"].shape[0]
    npages = (T + 31) // 32
    table = list(np.random.default_rng(T).permutation(npages + 2)[:npages])
    o8, os_, _ = _run_attn(ops, g["q8"], g["qs"], g["k8"], g["ks"], g["v8"], g["vs"], heads, kvh,
                           table)
    ref8, refs = O.quant_groups(g["out"], 128)
    same_bits(o8, ref8)
    same_bits(os_, refs)


def test_attention_guest_paged_fixture(ops, gold):
    """tests/guest/paged_attn.cpp: 4 q rows, 80 keys, table {2,0,1}."""
    p = {k: gold[f"guest_pa_{k}"] for k in ("q", "k", "v", "qs", "ks", "vs", "o8", "os")}
    o8, os_, _ = _run_attn(ops, p["q"], p["qs"], p["k"], p["ks"], p["v"], p["vs"], 4, 2, [2, 0, 1])
    same_bits(o8, p["o8"])
    same_bits(os_, p["os"])


@pytest.mark.parametrize("rows,T", [(64, 64), (100, 300), (1, 2049), (33, 95)])
def test_attention_paged_random(ops, rows, T):
    rng = np.random.default_rng(rows * 1000 + T)
    heads, kvh = 16, 8
    q8 = rng.integers(-127, 128, (rows, heads * 128)).astype(np.int8)
    k8 = rng.integers(-127, 128, (T, kvh * 128)).astype(np.int8)
    v8 = rng.integers(-127, 128, (T, kvh * 128)).astype(np.int8)
    qs = rng.uniform(1e-3, 1e-2, (rows, heads)).astype(F)
    ks = rng.uniform(1e-3, 1e-2, (T, kvh)).astype(F)
    vs = rng.uniform(1e-3, 1e-2, (T, kvh)).astype(F)
    npages = (T + 31) // 32
    table = list(rng.permutation(npages))
    o8, os_, _ = _run_attn(ops, q8, qs, k8, ks, v8, vs, heads, kvh, table)
    ref = O.attention(q8, qs, k8, ks, v8, vs, np.arange(T - rows, T), heads, kvh, 128,
                      F(1.0 / np.sqrt(128.0)))
    ref8, refs = O.quant_groups(ref, 128)
    same_bits(o8, ref8)
    same_bits(os_, refs)


def test_attention_two_requests_share_pool(ops):
    """tests/guest/paged_attn_multi.cpp: two requests (4q/80kv, 8q/48kv) in one
    page pool, each with its own table, each equal to its contiguous result."""
    rng = np.random.default_rng(9)
    heads, kvh = 4, 2
    reqs = [(4, 80, [3, 0, 4]), (8, 48, [1, 2])]
    pk = np.zeros((5, 32, 256), np.int8)
    pv = np.zeros((5, 32, 256), np.int8)
    pks = np.zeros((5, 32, 2), F)
    pvs = np.zeros((5, 32, 2), F)
    data = []
    for R, T, table in reqs:
        q8 = rng.integers(-3, 4, (R, 512)).astype(np.int8)
        k8 = rng.integers(-2, 3, (T, 256)).astype(np.int8)
        v8 = rng.integers(-3, 4, (T, 256)).astype(np.int8)
        qs = rng.choice(np.array([1, .5, .25, .75], F), (R, heads))
        ks = rng.choice(np.array([1, .5, .25, .75], F), (T, kvh))
        vs = rng.choice(np.array([1, .5, .25, .75], F), (T, kvh))
        for t in range(T):
            p, s = table[t // 32], t % 32
            pk[p, s], pv[p, s], pks[p, s], pvs[p, s] = k8[t], v8[t], ks[t], vs[t]
        data.append((q8, qs, k8, ks, v8, vs))
    dpk, dpv, dpks, dpvs = dev(pk), dev(pv), dev(pks), dev(pvs)
    for (R, T, table), (q8, qs, k8, ks, v8, vs) in zip(reqs, data):
        tab = dev(np.asarray(table, np.uint16).view(np.int16))
        kv = ops.paged_kv(dpk, dpv, dpks, dpvs, tab, kvh)
        o8 = torch.zeros(R, 512, dtype=torch.int8, device="cuda")
        os_ = torch.zeros(R, heads, dtype=torch.float32, device="cuda")
        ops.attention_heads_gqa_tokscale_paged(dev(q8), dev(qs), kv, T, o8, os_, heads, kvh, 128,
                                               True, float(F(0.08838834764831845)))
        ref = O.attention(q8, qs, k8, ks, v8, vs, np.arange(T - R, T), heads, kvh, 128,
                          F(0.08838834764831845))
        ref8, refs = O.quant_groups(ref, 128)
        same_bits(host(o8), ref8)
        same_bits(host(os_), refs)


# ---------------------------------------------------------------- KV scatter
def test_paged_kv_scatter_and_batch(ops):
    """tests/guest/paged_kv_batch.cpp: two decode rows, distinct tables."""
    kvd, kvh = 256, 2
    k = np.array([[(t * 7 + d * 3 + 1) % 7 - 3 for d in range(kvd)] for t in range(2)], np.int8)
    v = np.array([[(t * 5 + d * 2 + 2) % 5 - 2 for d in range(kvd)] for t in range(2)], np.int8)
    sb = np.array([1.0, 0.5, 0.25, 0.75], F)
    ks = np.array([[sb[(t + h) % 4] for h in range(kvh)] for t in range(2)], F)
    vs = np.array([[sb[(t * 3 + h) % 4] for h in range(kvh)] for t in range(2)], F)
    pk = torch.zeros(2, 32, kvd, dtype=torch.int8, device="cuda")
    pv = torch.zeros_like(pk)
    pks = torch.zeros(2, 32, kvh, dtype=torch.float32, device="cuda")
    pvs = torch.zeros_like(pks)
    t0 = dev(np.array([1, 0], np.int16))
    t1 = dev(np.array([0], np.int16))
    kv0 = ops.paged_kv(pk, pv, pks, pvs, t0, kvh)
    kv1 = ops.paged_kv(pk, pv, pks, pvs, t1, kvh)
    ops.paged_kv_scatter_batch(dev(k), dev(v), dev(ks), dev(vs), [kv0, kv1], [0, 0], 2, kvd, kvh)
    hk, hv, hks, hvs = host(pk), host(pv), host(pks), host(pvs)
    for t, page in ((0, 1), (1, 0)):
        assert np.array_equal(hk[page, 0], k[t]) and np.array_equal(hv[page, 0], v[t])
        same_bits(hks[page, 0], ks[t])
        same_bits(hvs[page, 0], vs[t])
    # single-request scatter of 40 rows through a shuffled table
    rng = np.random.default_rng(3)
    K = rng.integers(-127, 128, (40, kvd)).astype(np.int8)
    Vv = rng.integers(-127, 128, (40, kvd)).astype(np.int8)
    KS = rng.uniform(0, 1, (40, kvh)).astype(F)
    VS = rng.uniform(0, 1, (40, kvh)).astype(F)
    pk.zero_(); pv.zero_(); pks.zero_(); pvs.zero_()
    tab = dev(np.array([1, 0], np.int16))
    kv = ops.paged_kv(pk, pv, pks, pvs, tab, kvh)
    ops.paged_kv_scatter(dev(K), dev(Vv), dev(KS), dev(VS), kv, 0, 40, kvd, kvh)
    hk = host(pk)
    assert np.array_equal(hk[1], K[:32]) and np.array_equal(hk[0, :8], K[32:])
    same_bits(host(pvs)[0, :8], VS[32:])


# ---------------------------------------------------------------- decode batch
@pytest.mark.parametrize("lens", [[1, 31, 32, 33, 100], [2049, 300, 64, 4100, 5],
                                  [2112] * 8, [1, 200, 520, 700, 33],
                                  [2112] * 16, [2100 + 3 * i for i in range(32)],
                                  [2112] * 40])
def test_attention_decode_batch(ops, q3, lens):
    """One decode row per sequence over a shared pool with shuffled per-sequence
    tables.  Few (sequence, head) pairs with more than 4 key groups take the
    key-split kernel: [2112] * 8 runs clusters of 5 CTAs (the carry-in and the
    recurrence chain), the fourth case clusters of 2 in which short sequences
    leave CTAs without keys; 4100 keys exceed the split form and the first
    case needs no split: both take the single-CTA kernel, and so do the
    128-, 256- (the TP-2 shape) and 320-pair cases."""
    rng = np.random.default_rng(sum(lens))
    heads, kvh, kw = 16, 8, 1024
    B = len(lens)
    max_pages = max((n + 31) // 32 for n in lens) + 1
    pages = B * max_pages + 3
    perm = rng.permutation(pages)[:B * max_pages].reshape(B, max_pages).astype(np.uint16)
    pk = rng.integers(-127, 128, (pages, 32, kw)).astype(np.int8)
    pv = rng.integers(-127, 128, (pages, 32, kw)).astype(np.int8)
    pks = rng.uniform(1e-3, 1e-2, (pages, 32, kvh)).astype(F)
    pvs = rng.uniform(1e-3, 1e-2, (pages, 32, kvh)).astype(F)
    pks[:, 20:] = np.nan          # garbage past the end of a partial page must not leak
    pvs[:, 20:] = np.inf
    q8 = rng.integers(-127, 128, (B, heads * 128)).astype(np.int8)
    qs = rng.uniform(1e-3, 1e-2, (B, heads)).astype(F)
    for s, n in enumerate(lens):   # the valid part of every page holds finite scales
        for t in range(n):
            p, sl = perm[s, t // 32], t % 32
            pks[p, sl] = rng.uniform(1e-3, 1e-2, kvh)
            pvs[p, sl] = rng.uniform(1e-3, 1e-2, kvh)
    d = [dev(a) for a in (pk, pv, pks, pvs)]
    kv = ops.paged_kv(*d, dev(np.zeros(1, np.int16)), kvh)
    o8 = torch.zeros(B, heads * 128, dtype=torch.int8, device="cuda")
    os_ = torch.zeros(B, heads, dtype=torch.float32, device="cuda")
    qk = float(F(1.0 / np.sqrt(128.0)))
    ops.attention_decode_batch(dev(q8), dev(qs), kv, pages, dev(perm.view(np.int16)), max_pages,
                               dev(np.asarray(lens, np.int32)), B, o8, os_, heads, kvh, qk)
    got8, gots = host(o8), host(os_)
    assert q3._lib.lib().q3_device_status() == 0
    for s, n in enumerate(lens):
        rows = [perm[s, t // 32] for t in range(n)]
        sl = [t % 32 for t in range(n)]
        k8 = pk[rows, sl]
        v8 = pv[rows, sl]
        ks = pks[rows, sl]
        vs = pvs[rows, sl]
        ref = O.attention(q8[s:s + 1], qs[s:s + 1], k8, ks, v8, vs, np.array([n - 1]), heads,
                          kvh, 128, F(qk))
        r8, rs = O.quant_groups(ref, 128)
        same_bits(got8[s:s + 1], r8)
        same_bits(gots[s:s + 1], rs)
