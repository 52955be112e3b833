"""Seeded synthetic workloads: random-init Qwen2-shaped MLF2 models and random
k-quant blocks (binding of synth/mlf2_synth.c).

The model presets follow the benchmark configurations: weights fp32
N(0, 0.02) from seed 0, round-to-nearest quantized; Q4_K for attn_q/k/output
and ffn_gate/up, Q6_K for attn_v, ffn_down and token_embd (and output.weight
when untied); norm weights 1.0; biases N(0, 0.02).
"""
from __future__ import annotations

import ctypes as C
import dataclasses
import hashlib
import os

import numpy as np

# no import of ._lib here: the workload generator must not map the CUDA library
LIB_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_lib")
SYNTH_LIB_PATH = os.path.join(LIB_DIR, "libhakm_synth.so")
SYNTH_EXE_PATH = os.path.join(LIB_DIR, "hakm_synth")


class _Cfg(C.Structure):
    _fields_ = [("n_layers", C.c_int), ("d_model", C.c_int), ("n_heads", C.c_int),
                ("n_kv_heads", C.c_int), ("head_dim", C.c_int), ("ffn_dim", C.c_int),
                ("vocab", C.c_int), ("ctx", C.c_int), ("rope_theta", C.c_float),
                ("rms_eps", C.c_float), ("tied", C.c_int), ("qkv_bias", C.c_int),
                ("seed", C.c_uint64), ("wstd", C.c_float)]


@dataclasses.dataclass(frozen=True)
class ModelConfig:
    name: str
    n_layers: int
    d_model: int
    n_heads: int
    n_kv_heads: int
    ffn_dim: int
    vocab: int
    tied: bool
    head_dim: int = 128
    ctx: int = 32768
    rope_theta: float = 1.0e6
    rms_eps: float = 1.0e-6
    qkv_bias: bool = True
    seed: int = 0
    wstd: float = 0.02

    def _c(self) -> _Cfg:
        return _Cfg(self.n_layers, self.d_model, self.n_heads, self.n_kv_heads, self.head_dim,
                    self.ffn_dim, self.vocab, self.ctx, self.rope_theta, self.rms_eps,
                    int(self.tied), int(self.qkv_bias), self.seed, self.wstd)

    @property
    def kv_dim(self) -> int:
        return self.n_kv_heads * self.head_dim

    def weight_bytes_per_token(self) -> int:
        """Algorithmic bytes one decode step streams: every matrix once (lm_head
        included) plus the f32 norms and biases and one embedding row."""
        D, F, KV, V = self.d_model, self.ffn_dim, self.kv_dim, self.vocab
        q4 = lambda r, k: r * (k // 256) * 144
        q6 = lambda r, k: r * (k // 256) * 210
        layer = (q4(D, D) + q4(KV, D) + q6(KV, D) + q4(D, D) + 2 * q4(F, D) + q6(D, F)
                 + 2 * D * 4 + (D + 2 * KV) * 4 * int(self.qkv_bias))
        return self.n_layers * layer + q6(V, D) + D * 4 + (D // 256) * 210

    def kv_bytes_per_token(self, pos: int) -> int:
        """K and V cache bytes read by attention at position `pos`."""
        return 2 * self.n_layers * self.kv_dim * 4 * (pos + 1)


PRESETS = {
    # Qwen2 3B shape
    "3b": ModelConfig("3b", 36, 2048, 16, 2, 11008, 151936, tied=True),
    # Qwen2 7B shape
    "7b": ModelConfig("7b", 28, 3584, 28, 4, 18944, 152064, tied=False),
    # small shapes for CPU-checkable parity tests
    "tiny": ModelConfig("tiny", 2, 256, 4, 2, 512, 1024, tied=True, head_dim=64, ctx=2048),
    "small": ModelConfig("small", 3, 512, 8, 2, 1536, 4096, tied=False, head_dim=64, ctx=4096),
    "mid": ModelConfig("mid", 2, 1024, 8, 2, 2816, 8192, tied=True, head_dim=128, ctx=4096),
}


def _load() -> C.CDLL:
    if not os.path.exists(SYNTH_LIB_PATH):
        raise ImportError(f"{SYNTH_LIB_PATH} missing: run `python -m hako_b200.build`")
    lib = C.CDLL(SYNTH_LIB_PATH)
    lib.synth_write_model.restype = C.c_int
    lib.synth_write_model.argtypes = [C.c_char_p, C.POINTER(_Cfg), C.c_int]
    lib.synth_model_size.restype = C.c_uint64
    lib.synth_model_size.argtypes = [C.POINTER(_Cfg)]
    for n in ("synth_random_q4k", "synth_random_q6k"):
        getattr(lib, n).restype = None
        getattr(lib, n).argtypes = [C.c_void_p, C.c_long, C.c_long, C.c_uint64]
    lib.synth_normal.restype = None
    lib.synth_normal.argtypes = [C.c_void_p, C.c_long, C.c_uint64, C.c_float]
    for n in ("synth_quantize_q4k_block", "synth_quantize_q6k_block"):
        getattr(lib, n).restype = None
        getattr(lib, n).argtypes = [C.c_void_p, C.c_void_p]
    return lib


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        _lib = _load()
    return _lib


def _exe_args(cfg: ModelConfig) -> list[str]:
    return [str(v) for v in (cfg.n_layers, cfg.d_model, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.ffn_dim,
                             cfg.vocab, cfg.ctx, repr(float(cfg.rope_theta)), repr(float(cfg.rms_eps)),
                             int(cfg.tied), int(cfg.qkv_bias), cfg.seed, repr(float(cfg.wstd)))]


def model_size(cfg: ModelConfig, via_exe: bool = False) -> int:
    if via_exe:
        import subprocess
        r = subprocess.run([SYNTH_EXE_PATH, "size", *_exe_args(cfg)], capture_output=True, text=True, check=True)
        return int(r.stdout.strip())
    c = cfg._c()
    return int(lib().synth_model_size(C.byref(c)))


def write_model(path: str, cfg: ModelConfig, threads: int = 0, via_exe: bool = False) -> str:
    if via_exe:
        import subprocess
        subprocess.run([SYNTH_EXE_PATH, "write", path, *_exe_args(cfg)], check=True)
        return path
    c = cfg._c()
    rc = lib().synth_write_model(path.encode(), C.byref(c), threads)
    if rc != 0:
        raise RuntimeError(f"synth_write_model({path}) failed: {rc}")
    return path


def cached_model(cfg: ModelConfig, directory: str | None = None, via_exe: bool = False) -> str:
    """Write the model once per machine (under /dev/shm when it has room) and
    return its path; the file name carries the full config. via_exe: use the
    stand-alone writer (hakm_synth) so this process maps no library of this
    package."""
    d = directory or ("/dev/shm" if os.path.isdir("/dev/shm") else "/tmp")
    tag = hashlib.sha1(repr(dataclasses.astuple(cfg)).encode()).hexdigest()[:12]
    path = os.path.join(d, f"hakm_synth_{cfg.name}_{tag}.mlf2")
    size = model_size(cfg, via_exe)
    if os.path.exists(path) and os.path.getsize(path) == size:
        return path
    import fcntl
    # one writer per machine: concurrent callers (e.g. the ranks of a
    # multi-GPU job) wait for it instead of writing the same file
    with open(path + ".lock", "w") as lk:
        fcntl.flock(lk, fcntl.LOCK_EX)
        if not os.path.exists(path) or os.path.getsize(path) != size:
            tmp = path + f".{os.getpid()}.part"
            write_model(tmp, cfg, via_exe=via_exe)
            os.replace(tmp, path)
    return path


def random_q4k(rows: int, k: int, seed: int) -> np.ndarray:
    out = np.empty(rows * (k // 256) * 144, dtype=np.uint8)
    lib().synth_random_q4k(out.ctypes.data, rows, k, seed)
    return out


def random_q6k(rows: int, k: int, seed: int) -> np.ndarray:
    out = np.empty(rows * (k // 256) * 210, dtype=np.uint8)
    lib().synth_random_q6k(out.ctypes.data, rows, k, seed)
    return out


def normal(n: int, seed: int, std: float = 1.0) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    lib().synth_normal(out.ctypes.data, n, seed, std)
    return out


def file_sha256(path: str) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        while True:
            b = f.read(1 << 24)
            if not b:
                break
            h.update(b)
    return h.hexdigest()
