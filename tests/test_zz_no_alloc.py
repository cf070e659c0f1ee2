"""The lm_head + argmax entry point that allocates nothing.

Some callers of this library cannot call cudaMalloc: a host that only owns one
fixed device buffer planned up front, or a serving loop that keeps
allocation calls (which can synchronize the device) off its hot path.
``q3_gemm_nt_group_argmax_noalloc`` serves them with a built-in device scratch
array instead of a caller workspace.  This test drives it through the C ABI,
three times in a row on different inputs (the array keeps the previous call's
contents; the last call has more rows and smaller maxima than the
first), and requires exactly the (best, bidx) of the workspace entry point
``q3_gemm_nt_group_argmax`` — the same bit-exact bar the other argmax tests use.
It also checks that a call beyond the array's row limit is refused.

The file name makes pytest collect it last, so a run that stops at the first
failure has run every other test before it.
"""

from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
F = np.float32


def _case(rng, m, k=1024, n=4096, g=256, a_scale=1.0):
    a = rng.integers(-127, 128, (m, k)).astype(np.int8)
    w = rng.integers(-127, 128, (n, k)).astype(np.int8)
    w[n - 5] = w[3]                    # a tied maximum candidate
    a_s = (rng.uniform(1e-3, 1e-2, (m, k // g)) * a_scale).astype(F)
    w_s = rng.uniform(1e-3, 1e-2, n).astype(F)
    w_s[n - 5] = w_s[3]
    return [torch.from_numpy(x).cuda() for x in (a, a_s, w, w_s)]


def _views(q3, tensors):
    return [q3.ops.MatrixView.of(t).c() for t in tensors]


def _run(q3, tensors, noalloc: bool):
    lib = q3._lib.lib()
    a, a_s, w, w_s = _views(q3, tensors)
    m = tensors[0].shape[0]
    best = torch.full((m,), -3.0e38, dtype=torch.float32, device="cuda")
    bidx = torch.zeros(m, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    if noalloc:
        rc = lib.q3_gemm_nt_group_argmax_noalloc(C.byref(a), C.byref(a_s), C.byref(w),
                                                  C.byref(w_s), best.data_ptr(), bidx.data_ptr(),
                                                  256, stream)
    else:
        wsb = lib.q3_gemm_nt_group_argmax_workspace_bytes(m)
        ws = torch.zeros(wsb, dtype=torch.uint8, device="cuda")
        rc = lib.q3_gemm_nt_group_argmax(C.byref(a), C.byref(a_s), C.byref(w), C.byref(w_s),
                                         best.data_ptr(), bidx.data_ptr(), 256, ws.data_ptr(),
                                         wsb, stream)
    assert rc == 0, q3._lib.STATUS.get(rc, rc)
    torch.cuda.synchronize()
    return best.cpu().numpy(), bidx.cpu().numpy()


def test_noalloc_argmax_matches_workspace_entry_twice(q3):
    assert torch.cuda.is_available()
    rng = np.random.default_rng(2024)
    # 40 rows, then 3, then 64 rows whose maxima are 1000x smaller than the
    # first call's: keys the first call left in the array would win their rows
    # unless each call clears every row it reads
    for m, a_scale in ((40, 1.0), (3, 1.0), (64, 1e-3)):
        tensors = _case(rng, m, a_scale=a_scale)
        want_best, want_idx = _run(q3, tensors, noalloc=False)
        got_best, got_idx = _run(q3, tensors, noalloc=True)
        assert np.array_equal(got_idx, want_idx)
        assert np.array_equal(got_best.view(np.uint32), want_best.view(np.uint32))


def test_noalloc_argmax_rejects_too_many_rows(q3):
    lib = q3._lib.lib()
    limit = 4096                      # Q3_NOALLOC_ARGMAX_MAX_ROWS
    a = q3._lib.View(0x1000, 1024, 1, limit + 1, 1024, 0)
    rc = lib.q3_gemm_nt_group_argmax_noalloc(C.byref(a), None, None, None, None, None, 256, None)
    assert rc == 7                    # Q3_ERR_CAPACITY, nothing launched
    assert b"4097 rows exceed" in lib.q3_last_cuda_error()
