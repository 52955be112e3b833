"""ctypes binding of libhakm_tok (include/hakm_tok.h): Qwen2 byte-level BPE
with the full Qwen2 pretokenizer, over the MLF2 tokenizer blob.

Mirrors the reference tokenizer's interface (src/bpe.h of mithraeums/hako):
`Tokenizer.from_mlf2(path)` is tok_new, `encode` tok_encode, `decode_id`
tok_decode_id, `token_id` tok_id, `eos` tok_eos. Raises at load if the
library is not built: there is no fallback.
"""
from __future__ import annotations

import ctypes as C
import os
import struct

HERE = os.path.dirname(os.path.abspath(__file__))
TOK_LIB_PATH = os.path.join(HERE, "_lib", "libhakm_tok.so")

_vp, _i, _sz = C.c_void_p, C.c_int, C.c_size_t
SIGNATURES = {
    "hakm_bpe_new": (_vp, [C.c_char_p, _sz, _i]),
    "hakm_bpe_free": (None, [_vp]),
    "hakm_bpe_vocab": (_i, [_vp]),
    "hakm_bpe_eos": (_i, [_vp]),
    "hakm_bpe_token_id": (_i, [_vp, C.c_char_p, _sz]),
    "hakm_bpe_encode": (_i, [_vp, C.c_char_p, _sz, C.POINTER(C.c_int), _i]),
    "hakm_bpe_decode_id": (_i, [_vp, _i, C.c_char_p, _i]),
    "hakm_pretok_split": (_i, [C.c_char_p, _sz, C.POINTER(C.c_size_t), _i]),
}

_LIB = None


def lib() -> C.CDLL:
    global _LIB
    if _LIB is None:
        if not os.path.exists(TOK_LIB_PATH):
            raise ImportError(f"{TOK_LIB_PATH} is missing: build it with `python -m hako_b200.build`")
        L = C.CDLL(TOK_LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = L
    return _LIB


def _bytes(text: str | bytes) -> bytes:
    return text.encode("utf-8") if isinstance(text, str) else bytes(text)


def pretokenize(text: str | bytes) -> list[bytes]:
    """The Qwen2 pretokenizer's pieces of text (hakm_pretok_split)."""
    b = _bytes(text)
    ends = (C.c_size_t * max(len(b), 1))()
    k = lib().hakm_pretok_split(b, len(b), ends, len(b))
    if k < 0:
        raise RuntimeError("hakm_pretok_split overflow")
    out, start = [], 0
    for e in ends[:k]:
        out.append(b[start:e])
        start = e
    return out


class Tokenizer:
    """One tokenizer over an MLF2 tokenizer blob (a private copy is kept)."""

    def __init__(self, blob: bytes, eos_id: int):
        self._h = lib().hakm_bpe_new(blob, len(blob), eos_id)
        self._buf = C.create_string_buffer(1 << 16)
        if not self._h:
            raise ValueError("malformed tokenizer blob")

    @classmethod
    def from_mlf2(cls, path: str) -> "Tokenizer":
        """The tokenizer of an MLF2 model file (header fields per
        include/mlf2.h:55-78 of the reference: tokenizer_off at byte 68,
        data_off at 76, eos_id at 88; the blob ends where the tensor directory
        or the data begins, whichever follows it)."""
        with open(path, "rb") as f:
            head = f.read(128)
            if head[:4] != b"MLF2":
                raise ValueError(f"{path}: not an MLF2 file")
            tensors_off, tok_off, data_off = struct.unpack_from("<QQQ", head, 60)
            eos = struct.unpack_from("<I", head, 88)[0]
            after = [o for o in (tensors_off, data_off, os.path.getsize(path)) if o > tok_off]
            f.seek(tok_off)
            blob = f.read(min(after) - tok_off)
        return cls(blob, eos)

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().hakm_bpe_free(self._h)
            self._h = None

    def __del__(self):
        self.close()

    @property
    def vocab_size(self) -> int:
        return lib().hakm_bpe_vocab(self._h)

    @property
    def eos(self) -> int:
        return lib().hakm_bpe_eos(self._h)

    def token_id(self, literal: str | bytes) -> int:
        b = _bytes(literal)
        return lib().hakm_bpe_token_id(self._h, b, len(b))

    def encode(self, text: str | bytes, max_ids: int | None = None) -> list[int]:
        """Token ids of text; raises if more than max_ids (default: no limit,
        which is at most one id per byte)."""
        b = _bytes(text)
        cap = max(len(b), 1) if max_ids is None else max_ids
        out = (C.c_int * max(cap, 1))()
        k = lib().hakm_bpe_encode(self._h, b, len(b), out, cap)
        if k < 0:
            raise OverflowError(f"more than {cap} ids, or a symbol outside the vocabulary")
        return list(out[:k])

    def decode_id(self, token: int) -> bytes:
        n = lib().hakm_bpe_decode_id(self._h, token, self._buf, len(self._buf))
        return C.string_at(self._buf, n)

    def decode(self, ids) -> bytes:
        return b"".join(self.decode_id(int(t)) for t in ids)
