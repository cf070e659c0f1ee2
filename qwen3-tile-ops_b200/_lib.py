"""ctypes binding of ``include/q3_ops.h`` (the C ABI of ``libq3b200.so``).

The library is loaded from this package's directory; nothing falls back to a
CPU implementation — a missing library raises at import of the operators.
"""

from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libq3b200.so"

DT_I8, DT_U8, DT_I32, DT_U32, DT_F32 = 0, 1, 2, 3, 4

STATUS = {0: "OK", 1: "NULL", 2: "MODE", 3: "SHAPE", 4: "DTYPE", 5: "ALIGN", 6: "CUDA",
          7: "CAPACITY", 8: "ARCH"}

# offset indices of q3_layout.off (enum order of include/q3_ops.h)
OFF_NAMES = [
    "kIDS", "kCTRL", "kX", "kEMB", "kLM", "kNF", "kCOS", "kSIN", "kLAYERW_BASE",
    "kLAYERW_STRIDE", "kLQ", "kLQ_SCALE", "kLK", "kLK_SCALE", "kLV", "kLV_SCALE", "kLO",
    "kLO_SCALE", "kLG", "kLG_SCALE", "kLU", "kLU_SCALE", "kLD", "kLD_SCALE",
    "kLAYERN_BASE", "kLAYERN_STRIDE", "kN1", "kNQ", "kNK", "kN2", "kLOGITS", "kBLOCK_END",
    "kH", "kH8", "kHS", "kQ", "kK", "kV", "kQ8", "kK8", "kV8", "kQS", "kKS", "kVS", "kATTN",
    "kO", "kO8", "kOS", "kG", "kU", "kSW", "kS8", "kSS", "kARGF", "kARGI", "kKV_BASE",
    "kKV_STRIDE", "kKV_VOFF", "kKV_SOFF", "kSCRATCH_END",
]


class Q3Error(RuntimeError):
    def __init__(self, fn: str, code: int, detail: str = ""):
        super().__init__(f"{fn} failed: {STATUS.get(code, code)} ({code}){' ' + detail if detail else ''}")
        self.code = code


class View(C.Structure):
    _fields_ = [("data", C.c_void_p), ("row_bytes", C.c_int32), ("col_bytes", C.c_int32),
                ("rows", C.c_uint32), ("cols", C.c_uint32), ("dtype", C.c_uint8)]


class SampleRow(C.Structure):
    _fields_ = [("temperature", C.c_double), ("top_p", C.c_double),
                ("repetition_penalty", C.c_double), ("u", C.c_double), ("top_k", C.c_int32),
                ("gen_offset", C.c_uint32), ("gen_count", C.c_uint32), ("pad", C.c_uint32)]


class PagedKV(C.Structure):
    _fields_ = [("k", C.c_void_p), ("v", C.c_void_p), ("ks", C.c_void_p), ("vs", C.c_void_p),
                ("table", C.c_void_p), ("page_tokens", C.c_uint32), ("page_bytes", C.c_uint32),
                ("row_bytes", C.c_uint32), ("scale_page_bytes", C.c_uint32),
                ("scale_row_bytes", C.c_uint32)]


class Layout(C.Structure):
    _fields_ = [("hidden", C.c_uint32), ("layers", C.c_uint32), ("heads", C.c_uint32),
                ("kv_heads", C.c_uint32), ("head_dim", C.c_uint32), ("inter", C.c_uint32),
                ("vocab", C.c_uint32), ("seq", C.c_uint32), ("max_seq", C.c_uint32),
                ("off", C.c_int64 * len(OFF_NAMES))]


class KVPool(C.Structure):
    _fields_ = [("k", C.c_void_p), ("v", C.c_void_p), ("ks", C.c_void_p), ("vs", C.c_void_p),
                ("layer_stride", C.c_uint64), ("scale_layer_stride", C.c_uint64),
                ("num_pages", C.c_uint32)]


VP = C.POINTER(View)
SIGS = {
    "q3_rmsnorm_rows": [VP, VP, VP, C.c_float, C.c_void_p],
    "q3_quant_rows_heads": [VP, VP, VP, C.c_uint32, C.c_void_p],
    "q3_embedding_rmsnorm_rows": [VP, VP, VP, VP, VP, VP, C.c_float, C.c_void_p],
    "q3_gemm_nt_group_store": [VP, VP, VP, VP, VP, C.c_uint32, VP, VP, VP, VP, VP, VP, C.c_float,
                               C.c_void_p],
    "q3_gemm_gate_up_swiglu_quant": [VP, VP, VP, VP, VP, VP, VP, VP, C.c_uint32, C.c_void_p],
    "q3_attention_heads_gqa_tokscale_paged": [VP, VP, C.POINTER(PagedKV), C.c_uint32, VP, VP,
                                              C.c_int, C.c_int, C.c_int, C.c_int, C.c_float,
                                              C.c_void_p],
    "q3_attention_decode_batch": [VP, VP, C.POINTER(PagedKV), C.c_uint32, C.c_void_p, C.c_uint32,
                                  C.c_void_p, C.c_uint32, VP, VP, C.c_int, C.c_int, C.c_float,
                                  C.c_void_p],
    "q3_paged_kv_scatter": [VP, VP, VP, VP, C.POINTER(PagedKV), C.c_uint32, C.c_uint32,
                            C.c_uint32, C.c_uint32, C.c_void_p],
    "q3_paged_kv_scatter_batch": [VP, VP, VP, VP, C.POINTER(PagedKV), C.POINTER(C.c_uint32),
                                  C.c_uint32, C.c_uint32, C.c_uint32, C.c_void_p],
    "q3_gemm_nt_group_argmax_workspace_bytes": [C.c_uint32],
    "q3_gemm_nt_group_argmax": [VP, VP, VP, VP, C.c_void_p, C.c_void_p, C.c_uint32, C.c_void_p,
                                C.c_size_t, C.c_void_p],
    "q3_gemm_nt_group_argmax_noalloc": [VP, VP, VP, VP, C.c_void_p, C.c_void_p, C.c_uint32,
                                        C.c_void_p],
    "q3_argmax_logits": [VP, C.c_void_p, C.c_void_p],
    "q3_layout_compute": [C.POINTER(Layout)],
    "q3_forward_workspace_bytes": [C.POINTER(Layout)],
    "q3_blob_from_safetensors": [C.c_char_p, C.POINTER(Layout), C.c_double, C.c_uint32,
                                 C.c_void_p, C.c_void_p],
    "q3_safetensors_tensor": [C.c_char_p, C.c_char_p, C.POINTER(C.c_int32),
                              C.POINTER(C.c_uint64), C.POINTER(C.c_int32)],
    "q3_forward_chunk": [C.c_void_p, C.POINTER(Layout), C.c_uint32, C.c_uint32, C.c_int, C.c_int,
                         C.c_void_p, C.c_size_t, C.c_void_p],
    "q3_generate": [C.c_void_p, C.POINTER(Layout), C.c_void_p, C.c_size_t, C.c_void_p],
    "q3_decode_workspace_bytes": [C.POINTER(Layout), C.c_uint32],
    "q3_decode_step_batch": [C.c_void_p, C.POINTER(Layout), C.POINTER(KVPool), C.c_void_p,
                             C.c_uint32, C.c_void_p, C.c_void_p, C.c_uint32, C.c_void_p,
                             C.c_void_p, C.c_size_t, C.c_void_p],
    "q3_prefill_workspace_bytes": [C.POINTER(Layout), C.c_uint32, C.c_uint32],
    "q3_prefill_batch": [C.c_void_p, C.POINTER(Layout), C.POINTER(KVPool), C.c_void_p, C.c_uint32,
                         C.c_void_p, C.c_uint32, C.c_uint32, C.c_void_p, C.c_void_p, C.c_size_t,
                         C.c_void_p],
    "q3_sample_workspace_bytes": [C.c_uint32, C.c_uint32],
    "q3_sample_logits": [VP, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t,
                         C.c_void_p],
    "q3_rng_uniforms": [C.c_uint64, C.c_uint32, C.POINTER(C.c_double)],
    "q3_tokenizer_load": [C.c_char_p, C.POINTER(C.c_void_p)],
    "q3_tokenizer_encode": [C.c_void_p, C.c_char_p, C.c_size_t, C.POINTER(C.c_int32), C.c_uint32,
                            C.POINTER(C.c_uint32)],
    "q3_tokenizer_decode": [C.c_void_p, C.POINTER(C.c_int32), C.c_uint32, C.c_char_p, C.c_size_t,
                            C.POINTER(C.c_size_t)],
    "q3_tokenizer_eos_id": [C.c_void_p],
    "q3_tokenizer_destroy": [C.c_void_p],
    "q3_exp_rows": [VP, VP, C.c_void_p],
    "q3_exp2_rows": [VP, VP, C.c_void_p],
    "q3_exp2_selfcheck": [C.c_uint32, C.c_uint32, C.c_void_p, C.c_void_p, C.c_void_p],
    "q3_quant_selfcheck": [C.c_uint32, C.c_uint32, C.c_float, C.c_void_p, C.c_void_p, C.c_void_p],
    "q3_last_cuda_error": [],
    "q3_device_check": [],
    "q3_launch_count": [],
    "q3_device_status": [],
    "q3_timer_attach": [C.c_char_p, C.POINTER(C.c_void_p), C.POINTER(C.c_void_p), C.c_int],
    "q3_timer_detach": [],
}
RESTYPE = {"q3_gemm_nt_group_argmax_workspace_bytes": C.c_size_t,
           "q3_sample_workspace_bytes": C.c_size_t, "q3_tokenizer_eos_id": C.c_int32,
           "q3_forward_workspace_bytes": C.c_size_t, "q3_decode_workspace_bytes": C.c_size_t,
           "q3_prefill_workspace_bytes": C.c_size_t,
           "q3_last_cuda_error": C.c_char_p, "q3_launch_count": C.c_uint64}

_lib = None


def lib() -> C.CDLL:
    """The loaded library (raises if it was never built)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise FileNotFoundError(f"{LIB_PATH} is missing: run qwen3-tile-ops_b200/build.py")
        handle = C.CDLL(str(LIB_PATH))
        for name, args in SIGS.items():
            fn = getattr(handle, name)
            fn.argtypes = args
            fn.restype = RESTYPE.get(name, C.c_int)
        _lib = handle
    return _lib


def check(fn: str, code: int) -> None:
    if code != 0:
        detail = ""
        if code == 6:
            detail = (lib().q3_last_cuda_error() or b"").decode()
        raise Q3Error(fn, code, detail)


def declared_symbols() -> list[str]:
    """Every function name declared in include/q3_ops.h."""
    import re
    hdr = (Path(__file__).resolve().parent.parent / "include" / "q3_ops.h").read_text()
    body = re.sub(r"/\*.*?\*/", "", hdr, flags=re.S)
    return sorted(set(re.findall(r"\b(q3_[a-z0-9_]+)\s*\(", body)))
