"""Host-side mirror of the reference's operator API (``kernels/*.h``).

Each function has the reference operator's name and argument meaning and
takes ``MatrixView`` s over CUDA memory (torch tensors or raw device
pointers).  Work is enqueued on the current torch CUDA stream (or the
``stream=`` given).  Where the reference returns silently on an unsupported
shape, these raise ``Q3Error``.
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, replace

import torch

from ._lib import (DT_F32, DT_I8, DT_I32, DT_U32, DT_U8, PagedKV, SampleRow, View, check, lib)

_TORCH_DT = {torch.int8: DT_I8, torch.uint8: DT_U8, torch.int32: DT_I32, torch.float32: DT_F32}
_ESIZE = {DT_I8: 1, DT_U8: 1, DT_I32: 4, DT_U32: 4, DT_F32: 4}


@dataclass(frozen=True)
class MatrixView:
    """kernels/matrix.h:27-34: base address, byte strides, logical shape, dtype."""
    data: int
    row_bytes: int
    col_bytes: int
    rows: int
    cols: int
    dtype: int
    owner: object = None    # keeps the backing tensor alive

    @classmethod
    def of(cls, t: torch.Tensor, dtype: int | None = None) -> "MatrixView":
        """A view of a 1-D ([n] -> [n][1]) or 2-D CUDA tensor."""
        if not t.is_cuda:
            raise ValueError("MatrixView needs CUDA memory")
        dt = dtype if dtype is not None else _TORCH_DT[t.dtype]
        es = t.element_size()
        if t.dim() == 1:
            return cls(t.data_ptr(), t.stride(0) * es, es, t.shape[0], 1, dt, t)
        if t.dim() != 2:
            raise ValueError("MatrixView needs a 1-D or 2-D tensor")
        return cls(t.data_ptr(), t.stride(0) * es, t.stride(1) * es, t.shape[0], t.shape[1], dt, t)

    # matrix.h:46-120
    def sub_view(self, r0: int, c0: int, rows: int, cols: int) -> "MatrixView":
        return replace(self, data=self.data + r0 * self.row_bytes + c0 * self.col_bytes,
                       rows=rows, cols=cols)

    def rows_of(self, r0: int, n: int) -> "MatrixView":
        return self.sub_view(r0, 0, n, self.cols)

    def cols_of(self, c0: int, n: int) -> "MatrixView":
        return self.sub_view(0, c0, self.rows, n)

    def c(self) -> View:
        return View(self.data, self.row_bytes, self.col_bytes, self.rows, self.cols, self.dtype)


def _v(x):
    if x is None:
        return None
    if isinstance(x, torch.Tensor):
        x = MatrixView.of(x)
    return C.byref(x.c())


def _s(stream) -> int:
    if stream is None:
        return torch.cuda.current_stream().cuda_stream
    return stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream)


def rmsnorm_rows(x, w, out, inv: float, stream=None) -> None:
    check("q3_rmsnorm_rows", lib().q3_rmsnorm_rows(_v(x), _v(w), _v(out), inv, _s(stream)))


def quant_rows_heads(x, qi8, scale, group_cols: int, stream=None) -> None:
    check("q3_quant_rows_heads",
          lib().q3_quant_rows_heads(_v(x), _v(qi8), _v(scale), group_cols, _s(stream)))


def embedding_rmsnorm_rows(table, scale, ids, tmp, w, out, inv: float, stream=None) -> None:
    check("q3_embedding_rmsnorm_rows",
          lib().q3_embedding_rmsnorm_rows(_v(table), _v(scale), _v(ids), _v(tmp), _v(w), _v(out),
                                          inv, _s(stream)))


def gemm_nt_group_store(a, a_scale, b, b_scale, out, group_k: int = 128, add=None, q8=None,
                        qs=None, nw=None, cos=None, sin=None, inv_hd: float = 0.0,
                        stream=None) -> None:
    check("q3_gemm_nt_group_store",
          lib().q3_gemm_nt_group_store(_v(a), _v(a_scale), _v(b), _v(b_scale), _v(out), group_k,
                                       _v(add), _v(q8), _v(qs), _v(nw), _v(cos), _v(sin), inv_hd,
                                       _s(stream)))


def gemm_gate_up_swiglu_quant(a, a_scale, wg, wgs, wu, wus, s8, ss, group_k: int = 256,
                              stream=None) -> None:
    check("q3_gemm_gate_up_swiglu_quant",
          lib().q3_gemm_gate_up_swiglu_quant(_v(a), _v(a_scale), _v(wg), _v(wgs), _v(wu), _v(wus),
                                             _v(s8), _v(ss), group_k, _s(stream)))


def paged_kv(k: torch.Tensor, v: torch.Tensor, ks: torch.Tensor, vs: torch.Tensor,
             table: torch.Tensor, kv_heads: int, head_dim: int = 128,
             page_tokens: int = 32) -> PagedKV:
    """kernels/kv_pages.h:13-24 over [pages][page_tokens][kv_heads*head_dim] tensors."""
    row = kv_heads * head_dim
    return PagedKV(k.data_ptr(), v.data_ptr(), ks.data_ptr(), vs.data_ptr(), table.data_ptr(),
                   page_tokens, page_tokens * row, row, page_tokens * kv_heads * 4, kv_heads * 4)


def attention_heads_gqa_tokscale_paged(q8, q_scale, kv: PagedKV, kv_len: int, o8, os, heads: int,
                                       kv_heads: int, head_dim: int, causal: bool,
                                       qk_scale: float, stream=None) -> None:
    check("q3_attention_heads_gqa_tokscale_paged",
          lib().q3_attention_heads_gqa_tokscale_paged(_v(q8), _v(q_scale), C.byref(kv), kv_len,
                                                      _v(o8), _v(os), heads, kv_heads, head_dim,
                                                      1 if causal else 0, qk_scale, _s(stream)))


def attention_decode_batch(q8, q_scale, kv: PagedKV, num_pages: int, tables: torch.Tensor,
                           max_pages: int, kv_len: torch.Tensor, n_seqs: int, o8, os,
                           heads: int, kv_heads: int, qk_scale: float, stream=None) -> None:
    """One decode row per sequence over a shared page pool (per-sequence tables)."""
    check("q3_attention_decode_batch",
          lib().q3_attention_decode_batch(_v(q8), _v(q_scale), C.byref(kv), num_pages,
                                          tables.data_ptr(), max_pages, kv_len.data_ptr(),
                                          n_seqs, _v(o8), _v(os), heads, kv_heads, qk_scale,
                                          _s(stream)))


def paged_kv_scatter(k, v, ks, vs, kv: PagedKV, start_token: int, rows: int, kv_dim: int,
                     kv_heads: int, stream=None) -> None:
    check("q3_paged_kv_scatter",
          lib().q3_paged_kv_scatter(_v(k), _v(v), _v(ks), _v(vs), C.byref(kv), start_token, rows,
                                    kv_dim, kv_heads, _s(stream)))


def paged_kv_scatter_batch(k, v, ks, vs, tables: list, tokens: list, rows: int, kv_dim: int,
                           kv_heads: int, stream=None) -> None:
    arr = (PagedKV * len(tables))(*tables)
    tok = (C.c_uint32 * len(tokens))(*tokens)
    check("q3_paged_kv_scatter_batch",
          lib().q3_paged_kv_scatter_batch(_v(k), _v(v), _v(ks), _v(vs), arr, tok, rows, kv_dim,
                                          kv_heads, _s(stream)))


def gemm_nt_group_argmax(a, a_scale, b, b_scale, best: torch.Tensor, bidx: torch.Tensor,
                         group_k: int = 128, workspace: torch.Tensor | None = None,
                         stream=None) -> None:
    """kernels/lm_argmax.h:72-182; best/bidx are per-row in/out device tensors."""
    rows = (a.rows if isinstance(a, MatrixView) else a.shape[0])
    need = lib().q3_gemm_nt_group_argmax_workspace_bytes(rows)
    if workspace is None:
        workspace = torch.empty(max(need, 8), dtype=torch.uint8, device=best.device)
    check("q3_gemm_nt_group_argmax",
          lib().q3_gemm_nt_group_argmax(_v(a), _v(a_scale), _v(b), _v(b_scale), best.data_ptr(),
                                        bidx.data_ptr(), group_k, workspace.data_ptr(),
                                        workspace.numel(), _s(stream)))


def argmax_logits(logits, out_id: torch.Tensor, stream=None) -> None:
    check("q3_argmax_logits", lib().q3_argmax_logits(_v(logits), out_id.data_ptr(), _s(stream)))


def sample_logits(logits, params, generated=None, stream=None) -> torch.Tensor:
    """tools/engine.py:118-149 (Sampler.sample) for every row of ``logits``
    (rows x vocab float32, CUDA) on the device.  ``params``: one dict per row
    with ``temperature``, ``top_k``, ``top_p``, ``repetition_penalty`` and the
    draw ``u`` (the request's next ``default_rng(seed).random()``);
    ``generated``: per row, the ids the repetition penalty applies to.
    Returns the picked ids (int32, on the device)."""
    lv = MatrixView.of(logits) if isinstance(logits, torch.Tensor) else logits
    rows = len(params)
    gen_all, spec = [], (SampleRow * max(rows, 1))()
    for r, p in enumerate(params):
        g = list(generated[r]) if generated is not None else []
        spec[r] = SampleRow(float(p.get("temperature", 0.0)), float(p.get("top_p", 1.0)),
                            float(p.get("repetition_penalty", 1.0)), float(p.get("u", 0.0)),
                            int(p.get("top_k", 0)), len(gen_all), len(g), 0)
        gen_all += g
    dev = torch.device("cuda", torch.cuda.current_device()) if stream is None else stream.device
    sp = torch.frombuffer(bytearray(spec), dtype=torch.uint8).to(dev)
    gen = torch.tensor(gen_all or [0], dtype=torch.int32, device=dev)
    out = torch.empty(max(rows, 1), dtype=torch.int32, device=dev)
    ws = torch.empty(max(int(lib().q3_sample_workspace_bytes(rows, lv.cols)), 8), dtype=torch.uint8,
                     device=dev)
    check("q3_sample_logits", lib().q3_sample_logits(_v(lv.rows_of(0, rows)), sp.data_ptr(),
                                                     gen.data_ptr(), out.data_ptr(), ws.data_ptr(),
                                                     ws.numel(), _s(stream)))
    return out[:rows]


def exp_rows(x, out, stream=None) -> None:
    """Element-wise exp as the path computes it: exp2(f32(x*log2e)), correctly rounded."""
    check("q3_exp_rows", lib().q3_exp_rows(_v(x), _v(out), _s(stream)))


def exp2_rows(x, out, stream=None) -> None:
    """Element-wise correctly rounded float32 exp2."""
    check("q3_exp2_rows", lib().q3_exp2_rows(_v(x), _v(out), _s(stream)))
