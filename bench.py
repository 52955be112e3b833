#!/usr/bin/env python3
"""bench.py — batch-1 greedy decode throughput of the hako decode path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--model 3b|7b]

Workload at N = 1 (config 0 of the benchmark spec): random-init Qwen2
3B-shaped model in MLF2 (Q4_K + Q6_K, seed 0), 16 seeded prompt ids, then
greedy decode (default 64 steps). At N > 1 (config 3): the 7B-shaped model,
32 seeded prompt ids, greedy decode (default 128 steps). One step = one
decoded token at batch 1. The prompt and W warm-up tokens run untimed;
exactly K decode steps are timed with CUDA events, bracketed by a barrier
and a device synchronize. Weights (2.03 GB / 5.07 GB) exceed the 126 MB L2,
so every step streams them from HBM.

- value: K / device time of one hakmc_decode call, which runs all K steps
  in one launch of the persistent step kernel (CUDA events on its stream).
- e2e: the same K steps through the reference-facing per-token call
  (hakmc_forward: host token in, host argmax out, synchronous), wall clock.
- stream_match: the W + K ids decoded against the reference engine's own
  greedy stream for the same prompt (tests/golden/3b.json, 7b.json).
- roofline: that step-kernel launch (the only kernel of the decode path):
  algorithmic bytes = every step's weights + its K/V reads at that
  position, over the launch's device time.
- cpu_baseline: the reference engine's own compiled decode (oracle/_ref) on
  this host's cores, on a bounded sample of the same workload.
- config3_7b_1gpu (N = 1): config 3 on the one GPU, the N = 1 point of the
  7B series the N > 1 runs measure.
- prefill / batched_decode (one GPU; --no-next-rows skips them): short samples
  of configs 4a and 4b on the 7B shapes, whose full lines come from
  --workload prefill and --workload batch.

N > 1 (torchrun): one tensor-parallel group over the N GPUs (hakmc_tp_*):
every GEMV phase's rows split over all GPUs' CTAs, outputs all-gathered by
peer stores inside the step kernel; one sequence, so scaling is "strong" and
value = its tokens / the slowest rank's device time.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

PROMPT_LEN = 16
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return d, "measured"
    except OSError:
        return PEAKS_FALLBACK, "fallback"


def prompt_ids(model: str):
    if model == "7b":
        return np.random.default_rng(3).integers(0, 151643, 32).tolist()
    return np.random.default_rng(0).integers(0, 151643, PROMPT_LEN).tolist()


class ClockSampler:
    """SM clock, power and clock-event (throttle) reasons sampled during the
    timed region: an NVML polling thread (about one sample per millisecond,
    so even a region of a few tens of milliseconds gets many samples), with
    nvidia-smi as the fallback when NVML is unavailable."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    # NVML clock-event reason bits
    BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40}

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.p = None
        self.rows = []
        self.nv = None
        self.out = ""

    def _poll(self):
        nv, h = self.nv, self.h
        while not self.stop:
            try:
                sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                rs = nv.nvmlDeviceGetCurrentClocksThrottleReasons(h)
                self.rows.append((float(sm), int(rs)))
            except Exception:
                pass
            time.sleep(0.001)

    def __enter__(self):
        self.stop = False
        try:
            import threading
            import pynvml as nv
            nv.nvmlInit()
            self.h = nv.nvmlDeviceGetHandleByIndex(self.idx)
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(self.h, nv.NVML_CLOCK_SM))
            self.nv = nv
            self.th = threading.Thread(target=self._poll, daemon=True)
            self.th.start()
            time.sleep(0.003)  # first samples in before the region starts
            return self
        except Exception:
            self.nv = None
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                       "-lms", "100", "-i", str(self.idx)],
                                      stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.p = None
        return self

    def __exit__(self, *a):
        if self.nv is not None:
            self.stop = True
            self.th.join(timeout=2)
            return
        if self.p:
            self.p.terminate()
            try:
                self.out, _ = self.p.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.p.kill()
                self.out = ""

    def summary(self):
        if self.nv is not None and self.rows:
            sm = [r[0] for r in self.rows]
            mx = self.max_mhz
            reasons = sorted({n for r in self.rows for n, b in self.BITS.items() if r[1] & b})
            loaded = [x for x in sm if x > 0.5 * mx] or sm
            return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": mx, "reasons": reasons,
                    "samples": len(self.rows), "source": "nvml"}
        rows = [r.split(",") for r in self.out.strip().splitlines() if r.count(",") >= 8]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [float(r[1]) for r in rows]
        mx = float(rows[0][2])
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.strip().lower() == "active"})
        loaded = [s for s in sm if s > 0.5 * mx] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": mx, "reasons": reasons,
                "samples": len(rows), "source": "nvidia-smi"}


def dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    pg = None
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300))
        pg = dist
    return world, rank, local, pg


def reduce_max(pg, v: float, device):
    if pg is None:
        return v
    import torch
    t = torch.tensor([v], dtype=torch.float64, device=device)
    pg.all_reduce(t, op=pg.ReduceOp.MAX)
    return float(t.item())


def barrier(pg, device):
    import torch
    torch.cuda.synchronize(device)
    if pg is not None:
        pg.barrier()
        torch.cuda.synchronize(device)


def cpu_reference_decode(path: str, model: str, n_decode: int, max_seq: int):
    """The reference's own hakm_forward (oracle/_ref) on all host cores:
    prompt untimed, then n_decode timed greedy steps. Returns tok/s, cores."""
    cores = min(os.cpu_count() or 1, 16)  # the reference pool caps at 16 (src/nn.c:61)
    os.environ["HAKM_THREADS"] = str(cores)
    from oracle.oracle import RefModel
    m = RefModel(path, max_seq)
    am = 0
    for t in prompt_ids(model):
        _, am = m.forward(t, want_logits=False)
    t0 = time.perf_counter()
    for _ in range(n_decode):
        _, am = m.forward(am, want_logits=False)
    dt = time.perf_counter() - t0
    m.close()
    return n_decode / dt, cores


def run_reference_arm(args):
    world, rank, local, pg = int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")), 0, None
    if rank != 0:
        return 0
    # the model file through the stand-alone writer: this process maps no
    # library of the package, only the reference's own build (oracle/_ref)
    from hako_b200 import synth
    cfg = synth.PRESETS[args.model]
    path = synth.cached_model(cfg, via_exe=True)
    max_seq = len(prompt_ids(args.model)) + args.warmup + args.steps + 8
    cores = min(os.cpu_count() or 1, 16)
    os.environ["HAKM_THREADS"] = str(cores)
    from oracle.oracle import RefModel
    m = RefModel(path, max_seq)
    am = 0
    for t in prompt_ids(args.model):
        _, am = m.forward(t, want_logits=False)
    for _ in range(args.warmup):
        _, am = m.forward(am, want_logits=False)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        _, am = m.forward(am, want_logits=False)
    dt = time.perf_counter() - t0
    m.close()
    v = args.steps / dt
    line = {"impl": "reference", "metric": "decode tok/s (batch 1)", "value": v, "unit": "tok/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * dt / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8/fp32",
            "data": "synthetic (seeded random-init weights, seeded prompt ids)",
            "config": config_block(args, world),
            "cpu_baseline": {"value": v, "unit": "tok/s", "cores": cores, "kind": "reference",
                             "sample": f"{args.steps} greedy decode steps after a {len(prompt_ids(args.model))}-id prompt"},
            "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "libraries_mapped": repo_libraries_mapped()}
    print(json.dumps(line), flush=True)
    return 0


def repo_libraries_mapped():
    """Shared libraries under this repository that this process has mapped
    (the reference arm must show only oracle/_ref's build of the reference)."""
    seen = set()
    try:
        with open("/proc/self/maps") as f:
            for ln in f:
                p = ln.split()[-1] if ln.strip() else ""
                if p.startswith(ROOT) and ".so" in os.path.basename(p):
                    seen.add(os.path.relpath(p, ROOT))
    except OSError:
        pass
    return sorted(seen)


GEMV_SHAPES = [(2048, 2048), (256, 2048), (11008, 2048), (2048, 11008), (18944, 3584), (3584, 18944)]
GEMV_BATCHES = (1, 4, 16, 64)
LMHEAD_SHAPES = [(151936, 2048), (152064, 3584)]


def _graph_us(torch, stream, launch, reps):
    """Per-launch device time of `reps` back-to-back launches captured in one
    CUDA graph (no host launch cost), replayed 3 times between CUDA events."""
    with torch.cuda.stream(stream):
        for i in range(3):
            launch(i)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for i in range(reps):
            launch(i)
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    with torch.cuda.stream(stream):
        for _ in range(3):
            g.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) / (3 * reps) * 1e3
    del g
    return us


def gemv_sweep(device, hbm_gbs):
    """Config 1 (batched Q4_K x q8_32 matmul) and config 2 (Q6_K lm_head +
    greedy argmax): achieved HBM GB/s of the C-ABI kernels. Algorithmic bytes
    = rows*(K/256)*144 + N*(K + 4K/32) + N*rows*4 (Q4_K) and the Q6_K rows +
    the activation (lm_head). Each launch reads a different weight copy
    (copies together > 300 MB, beyond the 126 MB L2)."""
    import ctypes as C
    import torch
    from hako_b200 import check, lib, synth
    P = lambda t: C.c_void_p(t.data_ptr())
    s = torch.cuda.Stream(device)
    sp = C.c_void_p(s.cuda_stream)
    rows_out = []
    for rows, k in GEMV_SHAPES:
        wb = rows * (k // 256) * 144
        ncopy = max(2, -(-300_000_000 // wb))
        w0 = torch.from_numpy(synth.random_q4k(rows, k, rows + k)).to(device)
        ws = [w0] + [w0.clone() for _ in range(ncopy - 1)]
        for n in GEMV_BATCHES:
            g = torch.Generator(device="cpu").manual_seed(n)
            xq = torch.randint(-127, 128, (n, k), dtype=torch.int8, generator=g).to(device)
            xs = (torch.rand((n, k // 32), generator=g) * 0.01).to(device)
            out = torch.empty((n, rows), dtype=torch.float32, device=device)
            nbytes = lib.hakmc_gemv_q4k_q8_batch_scratch(rows, k, n)
            sc = torch.zeros(nbytes, dtype=torch.uint8, device=device)
            launch = lambda i: check(lib.hakmc_gemv_q4k_q8_batch(P(out), P(ws[i % ncopy]), P(xq), P(xs), None,
                                                                 rows, k, n, P(sc), nbytes, sp))
            us = _graph_us(torch, s, launch, max(ncopy, 20))
            byt = wb + n * (k + 4 * k // 32) + n * rows * 4
            rows_out.append({"shape": f"{rows}x{k}", "batch": n, "us": round(us, 2),
                             "gbs": round(byt / us / 1e3, 1), "frac": round(byt / us / 1e3 / hbm_gbs, 3)})
        del ws, w0
        torch.cuda.empty_cache()
    lm = []
    for rows, k in LMHEAD_SHAPES:
        w = synth.random_q6k(rows, k, rows + k)
        src = torch.from_numpy(w).to(device)
        packed = torch.empty(lib.hakmc_q6k_packed_bytes(rows, k), dtype=torch.uint8, device=device)
        check(lib.hakmc_q6k_pack(P(packed), P(src), rows, k, None))
        del src, w
        x = torch.from_numpy(synth.normal(k, 9)).to(device)
        logits = torch.empty(rows, dtype=torch.float32, device=device)
        am = torch.empty(1, dtype=torch.int32, device=device)
        launch = lambda i: check(lib.hakmc_lmhead_argmax(P(logits), P(am), P(packed), P(x), None, 0.0,
                                                         rows, k, sp))
        us = _graph_us(torch, s, launch, 10)
        byt = rows * (k // 256) * 210 + 4 * k + 4 * rows
        lm.append({"shape": f"{rows}x{k}", "us": round(us, 2), "gbs": round(byt / us / 1e3, 1),
                   "frac": round(byt / us / 1e3 / hbm_gbs, 3)})
        del packed
        torch.cuda.empty_cache()
    return {"kernel": "hakmc_gemv_q4k_q8_batch: q4k_batch_kernel (dp4a) for N <= 16, q4k_mma_kernel "
                      "(tcgen05 kind::i8) above; lm_head: stream_kernel (hakmc_lmhead_argmax)",
            "unit": "GB/s", "peak": hbm_gbs,
            "timing": "per launch, CUDA graph of back-to-back launches (programmatic dependent launch), "
                      "each on a different weight copy beyond L2",
            "q4k": rows_out, "lmhead_q6k_argmax": lm}


def gemv_one(rows, k, n):
    """Three launches of the batched Q4_K matmul on one shape (seeded data)."""
    import ctypes as C
    import torch
    from hako_b200 import check, lib, synth
    P = lambda t: C.c_void_p(t.data_ptr())
    dev = torch.device("cuda:0")
    w = torch.from_numpy(synth.random_q4k(rows, k, rows + k)).to(dev)
    g = torch.Generator(device="cpu").manual_seed(n)
    xq = torch.randint(-127, 128, (n, k), dtype=torch.int8, generator=g).to(dev)
    xs = (torch.rand((n, k // 32), generator=g) * 0.01).to(dev)
    out = torch.empty((n, rows), dtype=torch.float32, device=dev)
    nbytes = lib.hakmc_gemv_q4k_q8_batch_scratch(rows, k, n)
    sc = torch.zeros(max(nbytes, 16), dtype=torch.uint8, device=dev)
    for _ in range(3):
        check(lib.hakmc_gemv_q4k_q8_batch(P(out), P(w), P(xq), P(xs), None, rows, k, n, P(sc), nbytes, None))
    torch.cuda.synchronize()
    return 0


def step_profile(model):
    """The step-kernel launches a profiler summary is taken from: launch 1 =
    a 4-id prompt plus 2 greedy ids (one launch), launches 2 and 3 = one
    decode step each."""
    import ctypes as C
    from hako_b200 import HakmCtx, check, lib, synth
    ctx = HakmCtx(synth.cached_model(synth.PRESETS[model]), max_seq=128)
    ctx.generate(list(range(100, 104)), 2)
    out = np.zeros(1, np.int32)
    for _ in range(2):
        check(lib.hakmc_decode(ctx._h, 1, C.c_void_p(out.ctypes.data)))
    ctx.close()
    return 0


def golden_stream(model: str):
    """The reference's greedy stream for the bench prompt (tests/golden/,
    made by the reference engine itself: tests/golden/make_golden.py)."""
    p = os.path.join(ROOT, "tests", "golden", f"{model}.json")
    try:
        with open(p) as f:
            g = json.load(f)
    except OSError:
        return None
    return g["tokens"] if g.get("prompt") == prompt_ids(model) else None


def measure_decode(model: str, steps: int, warmup: int, world: int, local: int, pg, device):
    """Batch-1 greedy decode of `model` after its seeded prompt: the prompt
    and `warmup` steps untimed, then `steps` steps in one hakmc_decode call
    (device time, max over ranks), the same steps again through the
    per-token hakmc_forward (wall clock), and the stream's agreement with
    the reference's golden stream."""
    import ctypes as C
    from hako_b200 import HakmCtx, lib, synth
    cfg = synth.PRESETS[model]
    prompt = prompt_ids(model)
    max_seq = len(prompt) + 2 * (warmup + steps) + 16
    ctx = HakmCtx(synth.cached_model(cfg), max_seq=max_seq, device=local)
    if world > 1:
        from hako_b200 import tp
        tp.connect(ctx)
    for t in prompt:
        ctx.forward(t, want_logits=False)
    toks = np.zeros(warmup, np.int32)
    lib.hakmc_decode(ctx._h, warmup, C.c_void_p(toks.ctypes.data))
    pos0 = ctx.pos
    barrier(pg, device)
    with ClockSampler(local) as clk:
        barrier(pg, device)
        t0 = time.perf_counter()
        out = np.zeros(steps, np.int32)
        rc = lib.hakmc_decode(ctx._h, steps, C.c_void_p(out.ctypes.data))
        barrier(pg, device)
        wall = time.perf_counter() - t0
    if rc != 0:
        raise RuntimeError(f"hakmc_decode failed: {rc}")
    dev_ms = float(ctx.last_device_ms)
    max_ms = reduce_max(pg, dev_ms, device)
    # e2e: the same steps through the per-token host call
    ctx.set_pos(pos0)
    am = int(out[0])
    barrier(pg, device)
    t0 = time.perf_counter()
    for _ in range(steps):
        _, am = ctx.forward(am, want_logits=False)
    e2e_s = reduce_max(pg, time.perf_counter() - t0, device)
    ctx.close()
    stream = toks.tolist() + out.tolist()
    gold = golden_stream(model)
    if gold is None:
        match = {"golden": None}
    else:
        n = min(len(gold), len(stream))
        first_bad = next((i for i in range(n) if stream[i] != gold[i]), None)
        match = {"golden": f"tests/golden/{model}.json", "compared": n,
                 "matched": n if first_bad is None else first_bad, "identical": first_bad is None}
    # roofline: the step-kernel launch of the timed region; per GPU, with
    # tensor parallelism each GPU streams 1/world of the weights
    pk, pk_kind = peaks()
    alg_bytes = sum(cfg.weight_bytes_per_token() + cfg.kv_bytes_per_token(pos0 + i) for i in range(steps)) / world
    achieved = alg_bytes / (max_ms / 1e3) / 1e9
    traffic = None
    tpath = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tpath):
        with open(tpath) as f:
            per_tok = json.load(f).get(f"step_kernel_{model}_bytes_per_token")
        if per_tok:
            traffic = per_tok * steps / world  # per GPU, like bytes_per_launch
    tok_bytes = cfg.weight_bytes_per_token() + cfg.kv_bytes_per_token(pos0 + steps // 2)
    roof = {"bound": "hbm", "kernel": "step_kernel (whole decode steps, one launch)",
            "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s",
            "frac": achieved / pk["hbm_gbs"], "peak_source": pk_kind, "traffic": traffic,
            "bytes_per_launch": alg_bytes, "launch_ms": dev_ms,
            "roofline_tok_s": world * pk["hbm_gbs"] * 1e9 / tok_bytes}
    return {"value": steps / (max_ms / 1e3), "max_ms": max_ms, "e2e": steps / e2e_s, "wall": wall,
            "roofline": roof, "stream_match": match, "clocks": clk.summary()}


def config_block(args, world):
    from hako_b200 import synth
    cfg = synth.PRESETS[args.model]
    return {"workload": f"config {'0' if args.model == '3b' else '3'}: Qwen2 {args.model.upper()}-shaped "
                        f"Q4_K_M greedy decode, batch 1",
            "model": f"qwen2-{args.model}-synthetic", "layers": cfg.n_layers, "d_model": cfg.d_model,
            "heads": f"{cfg.n_heads}/{cfg.n_kv_heads}", "ffn": cfg.ffn_dim, "vocab": cfg.vocab,
            "prompt_len": len(prompt_ids(args.model)), "global_batch": 1, "seq_len": None,
            "parallelism": f"tp{world} (rows of every phase over all GPUs, peer-store all-gather)" if world > 1 else "single",
            "l2": f"weights stream from HBM every step ({cfg.weight_bytes_per_token() / 1e9:.2f} GB > 126 MB L2)"}


INT8_TOPS_NOMINAL = 4500.0  # dense int8 tensor peak of a B200 (NVIDIA's figure; no measured one on this pool)
FP32_TFLOPS_NOMINAL = 148 * 128 * 2 * 1.965e9 / 1e12  # fp32 FMA issue peak of 148 SMs at the max clock, TFLOP/s


def _event_us(torch, fn, reps=5):
    """Mean device time of `reps` launches of fn (after two warm-up calls)."""
    for _ in range(2):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps * 1e3


def row_kernel_times(cfg, M: int, attn_rows: int, attn_pos0: int, attn_row_pos: int):
    """CUDA-event times of the row-batched pass's kernels on its own shapes
    (seeded data; weights > L2 for the large matrices): the tensor-core Q4_K
    matmuls and the Q6_K row matmuls at M activation rows, and the attention
    of attn_rows rows (prompt rows at attn_pos0.., or decode rows at
    attn_row_pos each with its own cache). Per launch, with the work each
    launch does, so each kernel's roofline fraction follows."""
    import ctypes as C
    import torch
    from hako_b200 import check, lib, synth
    P = lambda t: C.c_void_p(t.data_ptr())
    dev = torch.device("cuda:0")
    D, F, KV, H, KVH = cfg.d_model, cfg.ffn_dim, cfg.kv_dim, cfg.n_heads, cfg.n_kv_heads
    hd = D // H
    g = torch.Generator(device="cpu").manual_seed(M)
    xq = torch.randint(-127, 128, (M, max(D, F)), dtype=torch.int8, generator=g).to(dev)
    xs = (torch.rand((M, max(D, F) // 32), generator=g) * 0.01).to(dev)
    x = torch.randn((M, max(D, F)), generator=g).to(dev)
    res = {}
    for name, rows, k in (("wqk", D + KV, D), ("wo", D, D), ("wgu", 2 * F, D)):
        w = torch.from_numpy(synth.random_q4k(rows, k, rows + k)).to(dev)
        out = torch.empty((M, rows), device=dev)
        us = _event_us(torch, lambda: check(lib.hakmc_gemm_q4k_q8(P(out), P(w), P(xq), P(xs), None, rows, k, M,
                                                                   None, 0, None)))
        res[f"q4k_{name}"] = {"us": us, "ops": 2 * rows * k * M}
        del w
    for name, rows, k in (("wv", KV, D), ("down", D, F)):
        src = torch.from_numpy(synth.random_q6k(rows, k, rows + k)).to(dev)
        w = torch.empty(lib.hakmc_q6k_packed_bytes(rows, k), dtype=torch.uint8, device=dev)
        check(lib.hakmc_q6k_pack(P(w), P(src), rows, k, None))
        del src
        out = torch.empty((M, rows), device=dev)
        us = _event_us(torch, lambda: check(lib.hakmc_gemm_q6k(P(out), P(w), P(x), None, rows, k, M, 0, None)))
        res[f"q6k_{name}"] = {"us": us, "ops": 2 * rows * k * M}
        del w
    if attn_row_pos is None:
        # prompt rows: row r reads positions 0 .. attn_pos0 + r (from L2
        # after the first rows: the bound is the score arithmetic)
        n = attn_pos0 + attn_rows
        kc = torch.randn((n, KV), generator=g).to(dev)
        vc = torch.randn((n, KV), generator=g).to(dev)
        q = torch.randn((attn_rows, D), generator=g).to(dev)
        out = torch.empty((attn_rows, D), device=dev)
        us = _event_us(torch, lambda: check(lib.hakmc_attention_rows(P(out), P(q), P(kc), P(vc), attn_rows, attn_pos0,
                                                                      None, n - 1, 0, H, KVH, hd, None)))
        kv_bytes = sum(2 * (attn_pos0 + r + 1) * KV * 4 for r in range(attn_rows))
    else:
        cap = attn_row_pos + 1
        kc = torch.randn((attn_rows, cap, KV), generator=g).to(dev)
        vc = torch.randn((attn_rows, cap, KV), generator=g).to(dev)
        q = torch.randn((attn_rows, D), generator=g).to(dev)
        out = torch.empty((attn_rows, D), device=dev)
        rp = torch.full((attn_rows,), attn_row_pos, dtype=torch.int32, device=dev)
        us = _event_us(torch, lambda: check(lib.hakmc_attention_rows(P(out), P(q), P(kc), P(vc), attn_rows, 0, P(rp),
                                                                      attn_row_pos, cap * KV, H, KVH, hd, None)))
        kv_bytes = attn_rows * 2 * cap * KV * 4
    res["attention"] = {"us": us, "kv_bytes": kv_bytes}
    return res


def cpu_reference_rows(model: str, n_prompt: int, n_decode: int, cache_pos: int):
    """The reference's own hakm_forward (oracle/_ref) on the host cores: a
    bounded sample of the row-batched workloads, which the reference runs
    one position (or one sequence) at a time. n_prompt prompt positions
    (prefill rate) or, after writing cache_pos seeded cache positions,
    n_decode decode steps of one sequence (decode rate at that context)."""
    cores = min(os.cpu_count() or 1, 16)
    os.environ["HAKM_THREADS"] = str(cores)
    from hako_b200 import synth
    from oracle.oracle import RefModel
    cfg = synth.PRESETS[model]
    path = synth.cached_model(cfg)
    if n_prompt:
        m = RefModel(path, n_prompt + 8)
        ids = np.random.default_rng(41).integers(0, 151643, n_prompt).tolist()
        t0 = time.perf_counter()
        for i, t in enumerate(ids):
            m.forward(t, want_logits=i == n_prompt - 1)
        dt = time.perf_counter() - t0
        m.close()
        return n_prompt / dt, cores
    m = RefModel(path, cache_pos + n_decode + 8)
    rng = np.random.default_rng(7)
    m.write_kv(rng.standard_normal((cfg.n_layers, cache_pos, cfg.kv_dim), dtype=np.float32),
               rng.standard_normal((cfg.n_layers, cache_pos, cfg.kv_dim), dtype=np.float32))
    am = 11
    t0 = time.perf_counter()
    for _ in range(n_decode):
        _, am = m.forward(am, want_logits=False)
    dt = time.perf_counter() - t0
    m.close()
    return n_decode / dt, cores


def rows_rooflines(times, pk):
    """Roofline objects for the row kernels: the tensor-core Q4_K matmul
    (int8 tensor pipe), the Q6_K row matmul (fp32 issue) and the attention
    (HBM: K/V bytes)."""
    q4 = max((v for k, v in times.items() if k.startswith("q4k_")), key=lambda v: v["us"])
    q6 = max((v for k, v in times.items() if k.startswith("q6k_")), key=lambda v: v["us"])
    at = times["attention"]
    a4 = q4["ops"] / q4["us"] / 1e6
    a6 = q6["ops"] / q6["us"] / 1e6
    aa = at["kv_bytes"] / at["us"] / 1e3
    return {
        "tensor": {"bound": "tensor", "kernel": "q4k_mma_kernel (largest Q4_K matmul)", "achieved": a4,
                   "peak": INT8_TOPS_NOMINAL, "unit": "TOP/s", "frac": a4 / INT8_TOPS_NOMINAL,
                   "peak_source": "nominal dense int8 (no measured int8 peak on this pool)", "traffic": None,
                   "launch_us": q4["us"]},
        "fp32": {"bound": "fp32", "kernel": "rx_q6k_gemm_kernel (largest Q6_K matmul)", "achieved": a6,
                 "peak": FP32_TFLOPS_NOMINAL, "unit": "TFLOP/s", "frac": a6 / FP32_TFLOPS_NOMINAL,
                 "peak_source": "nominal fp32 FMA issue rate (the exact chains use a rounded product and a "
                                "separate add: at most half of it)", "traffic": None, "launch_us": q6["us"]},
        "hbm": {"bound": "hbm", "kernel": "rx_attention_gqa_kernel (K/V bytes every row reads)", "achieved": aa,
                "peak": pk["hbm_gbs"],
                "unit": "GB/s", "frac": aa / pk["hbm_gbs"], "peak_source": "measured", "traffic": None,
                "launch_us": at["us"]}}


def run_prefill(args, emit: bool = True):
    """Config 4a: a seeded 2048-id prompt through hakmc_prefill_batched (each
    call restarts the sequence, so every step is the whole prompt)."""
    from hako_b200 import HakmCtx, synth
    n = 2048
    cfg = synth.PRESETS[args.model]
    prompt = np.random.default_rng(41).integers(0, 151643, n).tolist()
    ctx = HakmCtx(synth.cached_model(cfg), max_seq=n + 8)
    for _ in range(args.warmup):
        ctx.reset()
        ctx.prefill_batched(prompt, want_logits=False)
    dev = []
    with ClockSampler(0) as clk:
        t0 = time.perf_counter()
        for _ in range(args.steps):
            ctx.reset()
            ctx.prefill_batched(prompt, want_logits=True)  # ids in, last logits out
            dev.append(float(ctx.last_device_ms))
        wall = time.perf_counter() - t0
    # per-position prompt feed (the reference's loop, one launch) on a 256-id slice
    ctx.reset()
    ctx.prefill(prompt[:256], want_logits=False)
    per_pos = 256 / (ctx.last_device_ms / 1e3)
    ctx.close()
    ms = sum(dev) / len(dev)
    line = {"metric": "prefill tok/s (2048-id prompt)", "value": n / (ms / 1e3), "unit": "tok/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8 x int4 (tensor cores), fp32 x int6, fp32 attention",
            "data": "synthetic (seeded random-init weights, seeded prompt ids)",
            "config": {"workload": f"config 4a: Qwen2 {args.model.upper()}-shaped, prefill of a 2048-id prompt "
                                   "(positions batched through each layer, causal attention)",
                       "model": f"qwen2-{args.model}-synthetic", "prompt_len": n, "chunk_rows": 1024},
            "e2e": {"value": args.steps * n / wall, "unit": "tok/s", "h2d_bytes_per_step": 4 * n,
                    "d2h_bytes_per_step": 4 * cfg.vocab},
            "per_position_prefill_tok_s": per_pos, "clocks": clk.summary()}
    if emit:
        # the dominant kernels timed alone on this workload's shapes
        # (1024-row chunks; attention of the second chunk's rows)
        times = row_kernel_times(cfg, 1024, 1024, 1024, None)
        roofs = rows_rooflines(times, peaks()[0])
        line["roofline"] = roofs["fp32"]
        line["roofline_tensor"] = roofs["tensor"]
        line["roofline_attention"] = roofs["hbm"]
        line["kernel_us"] = {k: v["us"] for k, v in times.items()}
        if not getattr(args, "no_cpu_baseline", False):
            v, cores = cpu_reference_rows(args.model, 16, 0, 0)
            line["cpu_baseline"] = {"value": v, "unit": "tok/s", "cores": cores, "kind": "reference",
                                    "sample": "the reference's hakm_forward feed of the first 16 prompt ids "
                                              "(oracle/_ref)"}
    if not emit:
        return line
    print(json.dumps(line), flush=True)
    return 0


def run_batch(args, emit: bool = True):
    """Config 4b: 64 independent sequences, each with a 4096-position KV cache
    of seeded N(0, 1) values, decoded together (hakmc_forward_batch, one row
    per sequence); a step = one new token for every sequence. N > 1: each GPU
    runs its own 64 sequences (replicas, no collective on the data path)."""
    import torch
    world, rank, local, pg = dist_setup(args.gpus)
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    from hako_b200 import HakmCtx, synth
    n_seq, ctx_len = 64, 4096
    cfg = synth.PRESETS[args.model]
    ctx = HakmCtx(synth.cached_model(cfg), max_seq=ctx_len + args.warmup + args.steps + 1, max_batch=n_seq,
                  device=local)
    for i in range(n_seq):
        ctx.fill_kv_normal(ctx_len, seq=i, seed=1000 * rank + i)
    toks = np.random.default_rng(5 + rank).integers(0, 151643, n_seq).tolist()
    pos = ctx_len
    for _ in range(args.warmup):
        _, am = ctx.forward_batch(toks, [pos] * n_seq)
        toks = [int(a) for a in am]
        pos += 1
    barrier(pg, device)
    dev = 0.0
    with ClockSampler(local) as clk:
        t0 = time.perf_counter()
        for _ in range(args.steps):
            _, am = ctx.forward_batch(toks, [pos] * n_seq)  # ids in, picks out
            toks = [int(a) for a in am]
            pos += 1
            dev += float(ctx.last_device_ms)
        barrier(pg, device)
        wall = time.perf_counter() - t0
    ctx.close()
    max_ms = reduce_max(pg, dev, device)
    e2e_s = reduce_max(pg, wall, device)
    line = {"metric": "batched decode tok/s (64 sequences, 4096-position caches)",
            "value": world * n_seq * args.steps / (max_ms / 1e3), "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": max_ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8 x int4 (tensor cores), fp32 x int6, fp32 attention",
            "data": "synthetic (seeded random-init weights, seeded N(0,1) K/V caches, seeded first ids)",
            "config": {"workload": f"config 4b: Qwen2 {args.model.upper()}-shaped, {n_seq} sequences x "
                                   f"{ctx_len}-position caches, one new token each per step",
                       "model": f"qwen2-{args.model}-synthetic", "global_batch": world * n_seq,
                       "seq_len": ctx_len, "parallelism": f"replicas x{world}" if world > 1 else "single",
                       "l2": f"K/V read per step {2 * cfg.n_layers * cfg.kv_dim * 4 * ctx_len * n_seq / 1e9:.1f} GB > L2"},
            "e2e": {"value": world * n_seq * args.steps / e2e_s, "unit": "tok/s", "h2d_bytes_per_step": 8 * n_seq,
                    "d2h_bytes_per_step": 4 * n_seq},
            "clocks": clk.summary()}
    if emit and rank == 0:
        times = row_kernel_times(cfg, n_seq, n_seq, 0, ctx_len)
        roofs = rows_rooflines(times, peaks()[0])
        line["roofline"] = roofs["hbm"]
        line["roofline_fp32"] = roofs["fp32"]
        line["roofline_tensor"] = roofs["tensor"]
        line["kernel_us"] = {k: v["us"] for k, v in times.items()}
        if world == 1 and not getattr(args, "no_cpu_baseline", False):
            v, cores = cpu_reference_rows(args.model, 0, 4, ctx_len)
            line["cpu_baseline"] = {"value": v, "unit": "tok/s", "cores": cores, "kind": "reference",
                                    "sample": f"4 decode steps of one sequence after {ctx_len} seeded cache positions "
                                              "(the reference decodes its sequences one at a time; oracle/_ref)"}
    if not emit:
        return line
    if rank == 0:
        print(json.dumps(line), flush=True)
    if pg is not None:
        pg.destroy_process_group()
    return 0


def prefill_summary(steps: int, warmup: int, model: str = "7b"):
    """Config 4a in brief for the decode line: run_prefill's measurement."""
    ns = argparse.Namespace(model=model, steps=steps, warmup=warmup)
    d = run_prefill(ns, emit=False)
    return {k: d[k] for k in ("metric", "value", "unit", "ms_per_step", "steps", "per_position_prefill_tok_s")} | \
        {"workload": d["config"]["workload"], "e2e_tok_s": d["e2e"]["value"]}


def batch_summary(steps: int, warmup: int, model: str = "7b"):
    """Config 4b in brief for the decode line (one GPU): run_batch's measurement."""
    ns = argparse.Namespace(model=model, steps=steps, warmup=warmup, gpus=1)
    d = run_batch(ns, emit=False)
    return {k: d[k] for k in ("metric", "value", "unit", "ms_per_step", "steps")} | \
        {"workload": d["config"]["workload"], "e2e_tok_s": d["e2e"]["value"]}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None,
                    help="default: 64 (3B decode), 128 (7B decode), 32 (batch), 8 (prefill)")
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--model", default=None, choices=["3b", "7b"],
                    help="default: 3b for decode on one GPU (config 0), 7b for decode on several GPUs "
                         "(config 3) and for the prefill and batch workloads (config 4)")
    ap.add_argument("--workload", default="decode", choices=["decode", "prefill", "batch"],
                    help="decode: batch-1 greedy decode (the headline); prefill: config 4a; batch: config 4b")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-gemv-sweep", action="store_true")
    ap.add_argument("--no-next-rows", action="store_true",
                    help="skip the short config 4a / 4b samples added to the decode line")
    ap.add_argument("--step-profile", action="store_true",
                    help="only a 4-id prompt, 2 generated ids, then two one-step hakmc_decode launches "
                         "(the last is the one a profiler captures: -k step_kernel -s 2 -c 1)")
    ap.add_argument("--gemv-shape", default=None,
                    help="ROWSxKxN: only run three launches of hakmc_gemv_q4k_q8_batch on that shape "
                         "(a small case for a profiler), print nothing else")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.model is None:
        # decode: config 0 (3B) on one GPU, config 3 (7B) across several
        args.model = "3b" if args.workload == "decode" and args.gpus == 1 else "7b"
    if args.steps is None:
        args.steps = {"prefill": 8, "batch": 32}.get(args.workload, 64 if args.model == "3b" else 128)
    if args.impl == "ours" and args.workload == "prefill":
        return run_prefill(args)
    if args.impl == "ours" and args.workload == "batch":
        return run_batch(args)
    if args.gemv_shape:
        return gemv_one(*(int(v) for v in args.gemv_shape.split("x")))
    if args.step_profile:
        return step_profile(args.model)
    if args.impl == "reference":
        return run_reference_arm(args)

    import torch
    world, rank, local, pg = dist_setup(args.gpus)
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    from hako_b200 import synth
    cfg = synth.PRESETS[args.model]
    path = synth.cached_model(cfg)
    prompt = prompt_ids(args.model)
    d = measure_decode(args.model, args.steps, args.warmup, world, local, pg, device)
    max_ms = d["max_ms"]
    line = {"metric": "decode tok/s (batch 1)", "value": d["value"], "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": max_ms / args.steps,
            "higher_is_better": True, "scaling": "strong" if world > 1 else "weak", "vs_baseline": None,
            "dtype": "int8 x int4/int6 dot, fp32 accumulate", "data": "synthetic (seeded random-init weights, seeded prompt ids)",
            "config": config_block(args, world),
            "e2e": {"value": d["e2e"], "unit": "tok/s", "h2d_bytes_per_step": 4, "d2h_bytes_per_step": 4},
            "gpu_launches": 1, "roofline": d["roofline"], "stream_match": d["stream_match"],
            "clocks": d["clocks"], "wall_s": d["wall"]}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        n_cpu = 96 if args.model == "3b" else 48
        v, cores = cpu_reference_decode(path, args.model, n_cpu, len(prompt) + n_cpu + 8)
        line["cpu_baseline"] = {"value": v, "unit": "tok/s", "cores": cores, "kind": "reference",
                                "sample": f"{n_cpu} greedy decode steps after the {len(prompt)}-id prompt "
                                          "(reference hakm_forward, oracle/_ref)"}
    if rank == 0 and world == 1 and args.model == "3b" and not args.no_next_rows:
        # config 3 (7B, 32-id prompt, 128 tokens) on this one GPU: the N = 1
        # point of the 7B series that --gpus N > 1 measures
        d7 = measure_decode("7b", 128, args.warmup, 1, local, None, device)
        line["config3_7b_1gpu"] = {"value": d7["value"], "unit": "tok/s", "steps": 128,
                                   "ms_per_step": d7["max_ms"] / 128, "e2e_tok_s": d7["e2e"],
                                   "roofline_frac": d7["roofline"]["frac"], "stream_match": d7["stream_match"]}
    if rank == 0 and world == 1 and not args.no_gemv_sweep:
        line["gemv_sweep"] = gemv_sweep(device, peaks()[0]["hbm_gbs"])
    if rank == 0 and world == 1 and not args.no_next_rows:
        # the survey's next rows, short samples (their own lines: --workload prefill / batch)
        line["prefill"] = prefill_summary(steps=2, warmup=2)
        line["batched_decode"] = batch_summary(steps=8, warmup=3)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if pg is not None:
        pg.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
