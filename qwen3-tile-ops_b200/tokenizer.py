"""tools/tokenizer.py's ``Tokenizer`` (byte-level BPE from an HF
``tokenizer.json``) over the native implementation (``q3_tokenizer_*``):
same constructor argument, ``encode(text) -> ids``, ``decode(ids) -> text``
and ``eos_id``."""

from __future__ import annotations

import ctypes as C

from ._lib import check, lib


class Tokenizer:
    def __init__(self, path) -> None:
        h = C.c_void_p()
        check("q3_tokenizer_load", lib().q3_tokenizer_load(str(path).encode(), C.byref(h)))
        self._h = h
        self.eos_id = int(lib().q3_tokenizer_eos_id(h))

    def encode(self, text: str) -> list[int]:
        raw = text.encode("utf-8")
        n = C.c_uint32()
        cap = len(raw) + 16
        while True:
            buf = (C.c_int32 * cap)()
            rc = lib().q3_tokenizer_encode(self._h, raw, len(raw), buf, cap, C.byref(n))
            if rc == 7 and n.value > cap:
                cap = n.value
                continue
            check("q3_tokenizer_encode", rc)
            return list(buf[:n.value])

    def decode(self, ids) -> str:
        arr = (C.c_int32 * max(len(ids), 1))(*ids)
        n = C.c_size_t()
        cap = 8 * len(ids) + 16
        while True:
            buf = C.create_string_buffer(cap)
            rc = lib().q3_tokenizer_decode(self._h, arr, len(ids), buf, cap, C.byref(n))
            if rc == 7 and n.value > cap:
                cap = n.value
                continue
            check("q3_tokenizer_decode", rc)
            return buf.raw[:n.value].decode("utf-8")

    def close(self) -> None:
        if self._h:
            lib().q3_tokenizer_destroy(self._h)
            self._h = None

    def __del__(self) -> None:
        try:
            self.close()
        except Exception:
            pass
