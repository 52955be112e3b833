"""Host-side mirror of the reference engine's model interface (src/model.h:29-37
of mithraeums/hako) over libhakm_cuda.

    ctx = HakmCtx("model.mlf2", max_seq=2048)   # hakm_ctx_new
    logits = ctx.forward(token)                 # hakm_forward
    ctx.reset()                                 # hakm_reset
    ctx.close()                                 # hakm_ctx_free

Like the reference, construction returns an error (here: raises) on a
malformed file or a missing tensor, forward() advances the position by one,
and the logits belong to the step that produced them.
"""
from __future__ import annotations

import ctypes as C
import mmap
import os

import numpy as np

from ._lib import check, last_error, lib


class HakmCtx:
    def __init__(self, path_or_image, max_seq: int = 2048, max_batch: int = 1, device: int = 0):
        self._mm = None
        if isinstance(path_or_image, (bytes, bytearray, memoryview, np.ndarray)):
            buf = np.frombuffer(path_or_image, dtype=np.uint8)
            self._keep = buf
            ptr, size = buf.ctypes.data, buf.nbytes
        else:
            f = open(path_or_image, "rb")
            self._mm = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ)
            f.close()
            arr = np.frombuffer(self._mm, dtype=np.uint8)
            self._keep = arr
            ptr, size = arr.ctypes.data, arr.nbytes
        h = lib.hakmc_create(C.c_void_p(ptr), size, max_seq, max_batch, device)
        if not h:
            err = last_error()
            self._release_image()
            raise RuntimeError(f"hakmc_create failed: {err}")
        self._h = C.c_void_p(h)
        # the device holds its own copy: the mapping is no longer needed
        self._release_image()
        self.max_seq = max_seq
        self.vocab = lib.hakmc_vocab(self._h)
        self.d_model = lib.hakmc_dim(self._h)
        self.n_layers = lib.hakmc_n_layers(self._h)

    def _release_image(self):
        self._keep = None
        if self._mm is not None:
            try:
                self._mm.close()
            except BufferError:
                pass
            self._mm = None

    # -- hakm_ctx_free
    def close(self):
        if getattr(self, "_h", None):
            lib.hakmc_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    @property
    def pos(self) -> int:
        return lib.hakmc_pos(self._h)

    def reset(self):
        lib.hakmc_reset(self._h)

    def set_pos(self, pos: int):
        check(lib.hakmc_set_pos(self._h, pos), "set_pos")

    def forward(self, token: int, want_logits: bool = True):
        """One decode step. Returns (logits or None, greedy argmax)."""
        am = C.c_int(-1)
        logits = np.empty(self.vocab, dtype=np.float32) if want_logits else None
        check(lib.hakmc_forward(self._h, int(token),
                                C.c_void_p(logits.ctypes.data) if want_logits else None,
                                C.byref(am)), "forward")
        return logits, am.value

    # -- tensor parallelism (hakmc_tp_*)
    def tp_export(self) -> bytes:
        """This rank's exchange handle, to be gathered by every rank."""
        buf = C.create_string_buffer(lib.hakmc_tp_handle_bytes())
        check(lib.hakmc_tp_export(self._h, buf), "tp_export")
        return buf.raw

    def tp_connect(self, rank: int, handles) -> None:
        """Join the group: `handles` are all ranks' tp_export() bytes in rank order."""
        blob = b"".join(handles)
        check(lib.hakmc_tp_connect(self._h, rank, len(handles), blob), "tp_connect")

    def prefill(self, tokens, want_logits: bool = True):
        """Feed a prompt in one device launch (hakmc_prefill); returns the
        last position's (logits or None, argmax)."""
        t = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32))
        logits = np.empty(self.vocab, np.float32) if want_logits else None
        am = C.c_int(0)
        check(lib.hakmc_prefill(self._h, C.c_void_p(t.ctypes.data), len(t),
                                C.c_void_p(logits.ctypes.data) if want_logits else None, C.byref(am)), "prefill")
        return logits, int(am.value)

    def prefill_batched(self, tokens, want_logits: bool = True, chunk_rows: int = 0):
        """Feed a prompt with its positions batched through each layer
        (hakmc_prefill_batched, chunks of chunk_rows positions; 0: default);
        returns the last position's (logits or None, argmax)."""
        t = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32))
        logits = np.empty(self.vocab, np.float32) if want_logits else None
        am = C.c_int(0)
        check(lib.hakmc_prefill_batched(self._h, C.c_void_p(t.ctypes.data), len(t), int(chunk_rows),
                                        C.c_void_p(logits.ctypes.data) if want_logits else None, C.byref(am)),
              "prefill_batched")
        return logits, int(am.value)

    def generate(self, prompt, n_gen: int) -> list[int]:
        """Greedy: feed the prompt one position at a time, then n_gen tokens."""
        p = np.ascontiguousarray(np.asarray(prompt, dtype=np.int32))
        out = np.zeros(max(n_gen, 1), dtype=np.int32)
        check(lib.hakmc_generate(self._h, C.c_void_p(p.ctypes.data), len(p), n_gen,
                                 C.c_void_p(out.ctypes.data)), "generate")
        return out[:n_gen].tolist()

    def set_layers(self, n: int):
        check(lib.hakmc_set_layers(self._h, n), "set_layers")

    def hidden(self, seq: int = 0) -> np.ndarray:
        out = np.empty(self.d_model, dtype=np.float32)
        check(lib.hakmc_hidden(self._h, seq, C.c_void_p(out.ctypes.data)), "hidden")
        return out

    def fill_kv(self, k: np.ndarray, v: np.ndarray, seq: int = 0):
        k = np.ascontiguousarray(k, dtype=np.float32)
        v = np.ascontiguousarray(v, dtype=np.float32)
        n_pos = k.shape[1]
        check(lib.hakmc_fill_kv(self._h, seq, C.c_void_p(k.ctypes.data), C.c_void_p(v.ctypes.data),
                                n_pos), "fill_kv")

    def fill_kv_normal(self, n_pos: int, seq: int = 0, seed: int = 0):
        """Seeded N(0, 1) K/V for positions [0, n_pos) of slot `seq`, on the device."""
        check(lib.hakmc_fill_kv_normal(self._h, seq, n_pos, seed), "fill_kv_normal")

    def forward_batch(self, tokens, pos, want_logits: bool = False):
        t = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32))
        p = np.ascontiguousarray(np.asarray(pos, dtype=np.int32))
        am = np.zeros(len(t), dtype=np.int32)
        logits = np.empty((len(t), self.vocab), dtype=np.float32) if want_logits else None
        check(lib.hakmc_forward_batch(self._h, C.c_void_p(t.ctypes.data), C.c_void_p(p.ctypes.data), len(t),
                                      C.c_void_p(logits.ctypes.data) if want_logits else None,
                                      C.c_void_p(am.ctypes.data)), "forward_batch")
        return logits, am

    @property
    def last_device_ms(self) -> float:
        return lib.hakmc_last_device_ms(self._h)
