"""Python binding of the test-side checkers. TEST INFRASTRUCTURE ONLY.

- ``Oracle``: the C restatement (oracle/hakm_oracle.c ->
  oracle/_build/libhakm_oracle.so).
- ``Reference``: mithraeums/hako's own sources compiled by oracle/Makefile into
  oracle/_ref/libhakm_ref.so, driven through oracle/ref_driver.c.

Only the tests, the smoke check and bench.py's CPU-baseline leg import this.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "libhakm_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "libhakm_ref.so")
REF_CLI = os.path.join(HERE, "_ref", "hakm")
DROPIN_CLI = os.path.join(HERE, "_ref", "hakm_cuda")  # the same CLI over the CUDA drop-in
# the reference checkout: HAKM_REF_SRC, by default one beside this repository
REF_SRC = os.environ.get("HAKM_REF_SRC", os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference"))

_vp, _i, _f = C.c_void_p, C.c_int, C.c_float


def build(ref: bool = True) -> None:
    """Compile the restatement, and the reference too when its sources exist
    (its tokenizer on its own, and the reference CLI relinked over the CUDA
    drop-in and the Qwen2 tokenizer once libhakm_cuda and libhakm_tok are
    built)."""
    targets = ["all"]
    if ref and os.path.isdir(os.path.join(REF_SRC, "src")):
        targets += ["ref", "reftok"]
        lib = os.path.join(os.path.dirname(HERE), "hako_b200", "_lib")
        if all(os.path.exists(os.path.join(lib, f)) for f in ("libhakm_cuda.so", "libhakm_tok.so")):
            targets.append("dropin")
    subprocess.run(["make", "-s", "-C", HERE, *targets, f"REF={REF_SRC}"], check=True)


def _p(a: np.ndarray):
    return C.c_void_p(a.ctypes.data)


class Oracle:
    def __init__(self):
        if not os.path.exists(ORACLE_SO):
            build(ref=False)
        L = C.CDLL(ORACLE_SO)
        sig = {
            "orc_f16_to_f32": (_f, [C.c_uint16]),
            "orc_f32_to_f16": (C.c_uint16, [_f]),
            "orc_dequant_q4k": (None, [_vp, _vp, _i]),
            "orc_dequant_q6k": (None, [_vp, _vp, _i]),
            "orc_quantize_q8_32": (None, [_vp, _i, _vp, _vp]),
            "orc_q4k_subsums": (None, [_vp, _i, _vp, _vp, _vp]),
            "orc_q4k_dot": (_f, [_vp, _i, _vp, _vp]),
            "orc_q6k_dot": (_f, [_vp, _i, _vp]),
            "orc_rmsnorm": (None, [_vp, _vp, _vp, _i, _f]),
            "orc_softmax": (None, [_vp, _i]),
            "orc_silu": (_f, [_f]),
            "orc_rope_neox": (None, [_vp, _i, _i, _f]),
            "orc_matmul": (_i, [_vp, _vp, _i, _vp, _vp, _i, _i]),
            "orc_model_new": (_vp, [_vp, C.c_size_t, _i]),
            "orc_model_free": (None, [_vp]),
            "orc_model_reset": (None, [_vp]),
            "orc_model_vocab": (_i, [_vp]),
            "orc_model_dim": (_i, [_vp]),
            "orc_model_set_layers": (None, [_vp, _i]),
            "orc_forward": (C.POINTER(C.c_float), [_vp, _i]),
            "orc_hidden": (C.POINTER(C.c_float), [_vp]),
            "orc_argmax": (_i, [_vp, _i]),
            "orc_attention": (None, [_vp, _vp, _vp, _vp, _i, _i, _i, _i]),
            "orc_expf": (_f, [_f]),
            "orc_expf_v8": (_f, [_f]),
            "orc_expf_v4": (_f, [_f]),
        }
        for n, (r, a) in sig.items():
            fn = getattr(L, n)
            fn.restype, fn.argtypes = r, a
        self.L = L

    def quantize_q8_32(self, x: np.ndarray):
        x = np.ascontiguousarray(x, dtype=np.float32)
        xq = np.empty(x.size, np.int8)
        xs = np.empty(x.size // 32, np.float32)
        self.L.orc_quantize_q8_32(_p(x), x.size, _p(xq), _p(xs))
        return xq, xs

    def dequant(self, blocks: np.ndarray, type_: int, nelem: int) -> np.ndarray:
        out = np.empty(nelem, np.float32)
        fn = self.L.orc_dequant_q4k if type_ == 12 else self.L.orc_dequant_q6k
        fn(_p(np.ascontiguousarray(blocks)), _p(out), nelem)
        return out

    def q4k_subsums(self, w: np.ndarray, n_out: int, n_in: int, xq: np.ndarray):
        iqx = np.empty(n_out * n_in // 32, np.int32)
        ix = np.empty_like(iqx)
        rb = n_in // 256 * 144
        for r in range(n_out):
            self.L.orc_q4k_subsums(C.c_void_p(w.ctypes.data + r * rb), n_in, _p(xq),
                                   C.c_void_p(iqx.ctypes.data + 4 * r * (n_in // 32)),
                                   C.c_void_p(ix.ctypes.data + 4 * r * (n_in // 32)))
        return iqx, ix

    def matmul(self, w: np.ndarray, type_: int, x: np.ndarray, n_out: int, n_in: int, bias=None):
        out = np.empty(n_out, np.float32)
        x = np.ascontiguousarray(x, dtype=np.float32)
        b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
        rc = self.L.orc_matmul(_p(out), _p(x), type_, _p(np.ascontiguousarray(w)),
                               None if b is None else _p(b), n_out, n_in)
        assert rc == 0
        return out

    def rmsnorm(self, x, w, eps):
        x = np.ascontiguousarray(x, np.float32)
        y = np.empty_like(x)
        self.L.orc_rmsnorm(_p(y), _p(x), _p(np.ascontiguousarray(w, np.float32)), x.size, eps)
        return y

    def rope(self, x, head_dim, pos, theta):
        x = np.array(x, dtype=np.float32, copy=True)
        for h in range(x.size // head_dim):
            self.L.orc_rope_neox(C.c_void_p(x.ctypes.data + 4 * h * head_dim), head_dim, pos, theta)
        return x

    def attention(self, q, kc, vc, pos, H, KVH, hd):
        """kc / vc: [>= pos + 1][KVH * hd] float32."""
        out = np.empty(H * hd, np.float32)
        q = np.ascontiguousarray(q, np.float32)
        kc = np.ascontiguousarray(kc, np.float32)
        vc = np.ascontiguousarray(vc, np.float32)
        self.L.orc_attention(_p(out), _p(q), _p(kc), _p(vc), pos, H, KVH, hd)
        return out


class OracleModel:
    """The restated forward pass over an MLF2 file (src/model.c:93-165)."""

    def __init__(self, path: str, max_seq: int):
        self.o = Oracle()
        self.img = np.fromfile(path, dtype=np.uint8)
        self.h = self.o.L.orc_model_new(_p(self.img), self.img.nbytes, max_seq)
        if not self.h:
            raise RuntimeError("orc_model_new failed")
        self.vocab = self.o.L.orc_model_vocab(self.h)
        self.dim = self.o.L.orc_model_dim(self.h)

    def forward(self, token: int) -> np.ndarray:
        p = self.o.L.orc_forward(self.h, token)
        return np.ctypeslib.as_array(p, (self.vocab,)).copy()

    def hidden(self) -> np.ndarray:
        return np.ctypeslib.as_array(self.o.L.orc_hidden(self.h), (self.dim,)).copy()

    def set_layers(self, n: int):
        self.o.L.orc_model_set_layers(self.h, n)

    def reset(self):
        self.o.L.orc_model_reset(self.h)

    def close(self):
        if self.h:
            self.o.L.orc_model_free(self.h)
            self.h = None


class Reference:
    """The reference engine's own compiled code (oracle/_ref/libhakm_ref.so)."""

    def __init__(self):
        if not os.path.exists(REF_SO):
            raise FileNotFoundError(f"{REF_SO} not built (needs the reference sources: make -C oracle ref)")
        L = C.CDLL(REF_SO)
        sig = {
            "refd_open": (_vp, [C.c_char_p, _i]),
            "refd_close": (None, [_vp]),
            "refd_reset": (None, [_vp]),
            "refd_vocab": (_i, [_vp]),
            "refd_dim": (_i, [_vp]),
            "refd_pos": (_i, [_vp]),
            "refd_n_layers": (_i, [_vp]),
            "refd_set_layers": (None, [_vp, _i]),
            "refd_hidden": (C.POINTER(C.c_float), [_vp]),
            "refd_forward": (_i, [_vp, _i, _vp, _vp]),
            "refd_greedy": (_i, [_vp, _vp, _i, _i, _vp, _vp]),
            "refd_matmul_raw": (_i, [_vp, _vp, _i, _vp, _vp, _i, _i]),
            "refd_read_kv": (_i, [_vp, _vp, _vp, _i]),
            "refd_set_pos": (None, [_vp, _i]),
            "refd_write_kv": (_i, [_vp, _vp, _vp, _i]),
            "quantize_row_q8_32": (None, [_vp, _i, _vp, _vp]),
            "q4k_vec_dot": (_f, [_vp, _i, _vp, _vp]),
            "dequant_q4_K": (None, [_vp, _vp, _i]),
            "dequant_q6_K": (None, [_vp, _vp, _i]),
            "f16_to_f32": (_f, [C.c_uint16]),
            "rmsnorm": (None, [_vp, _vp, _vp, _i, _f]),
            "rope_neox": (None, [_vp, _i, _i, _f]),
            "softmax": (None, [_vp, _i]),
            "silu_f": (_f, [_f]),
        }
        for n, (r, a) in sig.items():
            fn = getattr(L, n)
            fn.restype, fn.argtypes = r, a
        self.L = L

    # kernel level
    def quantize_q8_32(self, x):
        x = np.ascontiguousarray(x, dtype=np.float32)
        xq = np.empty(x.size, np.int8)
        xs = np.empty(x.size // 32, np.float32)
        self.L.quantize_row_q8_32(_p(x), x.size, _p(xq), _p(xs))
        return xq, xs

    def q4k_vec_dot(self, row: np.ndarray, n_in: int, xq, xs) -> float:
        return self.L.q4k_vec_dot(_p(np.ascontiguousarray(row)), n_in, _p(xq), _p(xs))

    def dequant(self, blocks, type_, nelem):
        out = np.empty(nelem, np.float32)
        fn = self.L.dequant_q4_K if type_ == 12 else self.L.dequant_q6_K
        fn(_p(np.ascontiguousarray(blocks)), _p(out), nelem)
        return out

    def matmul(self, w, type_, x, n_out, n_in, bias=None):
        out = np.empty(n_out, np.float32)
        x = np.ascontiguousarray(x, dtype=np.float32)
        b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
        self.L.refd_matmul_raw(_p(out), _p(x), type_, _p(np.ascontiguousarray(w)),
                               None if b is None else _p(b), n_out, n_in)
        return out

    def rmsnorm(self, x, w, eps):
        x = np.ascontiguousarray(x, np.float32)
        y = np.empty_like(x)
        self.L.rmsnorm(_p(y), _p(x), _p(np.ascontiguousarray(w, np.float32)), x.size, eps)
        return y

    def rope(self, x, head_dim, pos, theta):
        x = np.array(x, dtype=np.float32, copy=True)
        for h in range(x.size // head_dim):
            self.L.rope_neox(C.c_void_p(x.ctypes.data + 4 * h * head_dim), head_dim, pos, theta)
        return x


class RefModel:
    """hakm_ctx over an MLF2 file, driven by token id (oracle/ref_driver.c)."""

    def __init__(self, path: str, max_seq: int):
        self.r = Reference()
        self.h = self.r.L.refd_open(path.encode(), max_seq)
        if not self.h:
            raise RuntimeError("hakm_ctx_new failed")
        self.vocab = self.r.L.refd_vocab(self.h)
        self.dim = self.r.L.refd_dim(self.h)

    def forward(self, token: int, want_logits=True):
        am = C.c_int(-1)
        lg = np.empty(self.vocab, np.float32) if want_logits else None
        rc = self.r.L.refd_forward(self.h, token, _p(lg) if want_logits else None, C.byref(am))
        assert rc == 0
        return lg, am.value

    def greedy(self, prompt, n_gen):
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros(n_gen, np.int32)
        gaps = np.zeros(n_gen, np.float32)
        rc = self.r.L.refd_greedy(self.h, _p(p), len(p), n_gen, _p(out), _p(gaps))
        assert rc == 0
        return out.tolist(), gaps

    def hidden(self):
        return np.ctypeslib.as_array(self.r.L.refd_hidden(self.h), (self.dim,)).copy()

    def read_kv(self, n_layers: int, kv_dim: int, n_pos: int):
        k = np.empty((n_layers, n_pos, kv_dim), np.float32)
        v = np.empty_like(k)
        assert self.r.L.refd_read_kv(self.h, _p(k), _p(v), n_pos) == 0
        return k, v

    def set_pos(self, pos: int):
        self.r.L.refd_set_pos(self.h, pos)

    def write_kv(self, k: np.ndarray, v: np.ndarray):
        """k, v: [n_layers][n_pos][kv_dim] float32; sets pos = n_pos."""
        k = np.ascontiguousarray(k, np.float32)
        v = np.ascontiguousarray(v, np.float32)
        assert self.r.L.refd_write_kv(self.h, _p(k), _p(v), k.shape[1]) == 0

    def set_layers(self, n):
        self.r.L.refd_set_layers(self.h, n)

    def reset(self):
        self.r.L.refd_reset(self.h)

    @property
    def pos(self):
        return self.r.L.refd_pos(self.h)

    def close(self):
        if self.h:
            self.r.L.refd_close(self.h)
            self.h = None
