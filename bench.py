#!/usr/bin/env python3
"""Benchmark of the Mamba-130M lockstep decode step on B200 (one JSON line on stdout).

Workload: Mamba-130M, Q8 weight-only (group 64, the reference recipe),
32 lockstep streams per GPU, each a seeded Zipf(1.1) token window; a step advances every stream
by one token.  Weights are seeded random (no checkpoint is available); tokens are synthetic.

  value  tokens/s of the whole job, inputs resident in HBM (device entry point, CUDA-graph replay)
  e2e    the same through the plugin C ABI with host buffers: H2D of slots/tokens and D2H of the
         logits inside the timed region
Extra keys: per-kernel CUDA-event times, the roofline of the dominant kernel, the batch sweep
(1/128/1024 streams, Q8 and F32) at N=1 plus RWKV-7 0.1B W8A8 at 1/32/256 streams,
and the CPU baseline (the reference CPU path restated in C, oracle/, timed on this host's cores).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
Multi-GPU: launch under torch.distributed.run; each rank owns its own windows (weak scaling, no
collective on the data path); times are the max over ranks.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from redukt_b200 import rbin  # noqa: E402
from redukt_b200 import rwkv7_rbin  # noqa: E402
from redukt_b200.shard import max_over_ranks as shard_max  # noqa: E402
from redukt_b200.workload import ZIPF_SEED_BASE, zipf_tokens  # noqa: E402

WINDOW = 2700          # tokens per stream window (configs[0-1])
STREAMS = 32           # lockstep streams per GPU
L2_BYTES = 126 * 2**20
METRIC = "Mamba-130M decode tok/s (Q8, 32 lockstep streams per GPU)"
SWEEP_N = (1, 32, 128, 1024)
FUSED_MAX_N = 32       # Q8 batches up to this size run the fused step kernel (rk_fused.cuh)
RWKV_N = (1, 32, 256)  # configs[3] is 256 lockstep streams of uniform byte tokens


# ---------------------------------------------------------------------------------------------
# Algorithmic bytes (weights read once per step + per-stream compulsory traffic)
# ---------------------------------------------------------------------------------------------

def dims_bytes(dims: rbin.MambaDims, profile: str):
    d, di, xr, dr, V, L = dims.d_model, dims.d_inner, dims.xr, dims.dt_rank, dims.vocab, dims.n_layer
    q8 = profile != "f32"

    def mat(rows, cols):
        return rows * cols + rows * (cols // 64) * 4 if q8 else rows * cols * 4
    small = (d + 4 * di + di + xr * di + di * dr + di + 16 * di + di) * 4
    layer = mat(2 * di, d) + mat(d, di) + small
    weights = L * layer + mat(V, d) + d * 4
    emb_row = (d + (d // 64) * 4) if q8 else d * 4
    per_stream = 2 * dims.state_bytes() + V * 4 + emb_row
    return weights, per_stream


def rwkv7_bytes(d: rwkv7_rbin.Rwkv7Dims):
    """RWKV-7 W8A8 step: (weight bytes read once per step, compulsory bytes per stream)."""
    D, F, V, R = d.d_model, d.d_ffn, d.vocab, d.lora_w + d.lora_a + d.lora_v + d.lora_g
    w8 = lambda rows, cols: rows * cols + rows * 4  # int8 + one f32 scale per row
    layer = 4 * w8(D, D) + w8(F, D) + w8(D, F) + 2 * R * D * 4 + 19 * D * 4
    weights = d.n_layer * layer + w8(V, D) + 2 * D * 4
    state = d.state_floats() * 4
    per_stream = 2 * state + V * 4 + D * 4  # state read + write, logits, embedding row
    return weights, per_stream


def kernel_bytes(cls: str, n: int, dims: rbin.MambaDims, profile: str, conv_in_xproj: bool = True) -> int:
    """Algorithmic bytes of ONE launch of a kernel class for n streams.  The conv1d state (read and
    written) and the conv output belong to x_proj when it runs the conv (option conv_defer, the
    default), else to in_proj's epilogue."""
    d, di, xr, dr, V = dims.d_model, dims.d_inner, dims.xr, dims.dt_rank, dims.vocab
    q8 = profile != "f32"
    act = (lambda K: n * (3 * K + (K // 64) * 4)) if q8 else (lambda K: n * K * 4)
    mat = (lambda r, c: r * c + r * (c // 64) * 4) if q8 else (lambda r, c: r * c * 4)
    if cls == "scan":
        return (n * di * 16 * 4 * 2 + (di * dr + di + 16 * di + di) * 4 + n * (xr + 2 * di) * 4 + act(di))
    conv = n * di * 3 * 4 * 2 + 5 * di * 4 + n * di * 4  # state R/W, taps + bias, one [n][di] pass
    if cls == "in_proj":
        return mat(2 * di, d) + act(d) + n * 2 * di * 4 + (0 if conv_in_xproj else conv)
    if cls == "out_proj":
        return mat(d, di) + act(di) + n * d * 4 * 2
    if cls == "head":
        return mat(V, d) + act(d) + n * V * 4
    if cls == "x_proj":
        return xr * di * 4 + n * di * 4 + n * xr * 4 + (conv if conv_in_xproj else 0)
    if cls == "norm":
        return n * d * 4 + d * 4 + act(d)
    if cls == "embed":
        return n * ((d + (d // 64) * 4) if q8 else d * 4) + n * d * 4
    if cls == "step":  # the fused small-batch step: every layer's weights once, each stream's state in and out
        w, _ = dims_bytes(dims, profile)
        return w - mat(V, d) - d * 4 + n * 2 * dims.state_bytes()
    return 0


# ---------------------------------------------------------------------------------------------
# Environment helpers
# ---------------------------------------------------------------------------------------------

def model_paths(rank: int, world: int, barrier):
    cache = os.environ.get("REDUKT_B200_MODEL_CACHE", os.path.join(tempfile.gettempdir(), "redukt_b200_models"))
    os.makedirs(cache, exist_ok=True)
    f32 = os.path.join(cache, "mamba130m.rbin")
    q8 = os.path.join(cache, "mamba130m.q8.rbin")
    if rank == 0:
        rbin.ensure_model(f32, rbin.MAMBA_130M, kind="gaussian")
        rbin.with_flags(f32, q8, rbin.FLAG_Q8)
    barrier()
    return f32, q8


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled every 200 ms while running (read-only queries).

    The GPU is selected by its UUID (the CUDA-visible index need not be nvidia-smi's index).  If the
    full query is refused (an unknown field on this driver), the sampler retries with only the
    clocks; nvidia-smi's stderr is kept and reported when no sample was taken."""

    FULL = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
            "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
            "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    BASIC = "index,clocks.sm,clocks.max.sm"

    def __init__(self, local: int):
        self.sel = str(local)
        try:
            import torch
            u = str(torch.cuda.get_device_properties(local).uuid)
            self.sel = u if u.startswith("GPU-") else f"GPU-{u}"
        except Exception:
            pass
        self.query = self.FULL
        self.p = self._start(self.FULL)
        if self.p is not None:
            time.sleep(0.3)
            if self.p.poll() is not None:  # exited at once: the query was refused
                self.p = self._start(self.BASIC)
                self.query = self.BASIC

    def _start(self, q):
        self.path = tempfile.mktemp(suffix=".csv")
        self.err = tempfile.mktemp(suffix=".err")
        try:
            return subprocess.Popen(["nvidia-smi", f"--id={self.sel}", f"--query-gpu={q}",
                                     "--format=csv,noheader,nounits", "-lms", "200"],
                                    stdout=open(self.path, "w"), stderr=open(self.err, "w"))
        except OSError:
            return None

    def stop(self) -> dict:
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "samples": 0, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.p.kill()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 3:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        err = open(self.err).read().strip() if os.path.exists(self.err) else ""
        for f in (self.path, self.err):
            if os.path.exists(f):
                os.unlink(f)
        out = {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
               "samples": len(sm), "reasons": sorted(reasons), "gpu": self.sel}
        if self.query != self.FULL:
            out["note"] = "throttle-reason fields refused by nvidia-smi; clocks only"
        if not sm and err:
            out["nvidia_smi_stderr"] = err[-300:]
        return out


def load_peaks() -> dict:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            j = json.load(f)
        return {"hbm_gbs": float(j["hbm_gbs"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


def load_traffic() -> dict:
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f)
    return {}


# ---------------------------------------------------------------------------------------------
# CPU baseline: the reference CPU path (restated in C, oracle/) on this host's cores
# ---------------------------------------------------------------------------------------------

def cpu_model() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_time(path: str, profile: str, n: int, budget_s: float, min_steps: int = 2, reset_every: int = 4096):
    """tok/s of the C restatement of the reference CPU path (oracle/) on all host threads: n lockstep
    streams of Zipf(1.1) windows, timed for about budget_s after one warm-up step."""
    from oracle import oracle as O
    m = O.Model(path, O.PROFILE_Q8 if profile == "q8" else O.PROFILE_F32, 64)
    toks = zipf_tokens(n, WINDOW, vocab=m.vocab)
    states = [m.new_state(reset_every) for _ in range(n)]
    m.forward_multi(toks[:, 0].tolist(), states)  # warm-up (page in weights, start the pool)
    t0 = time.perf_counter()
    steps = 0
    while steps < min_steps or time.perf_counter() - t0 < budget_s:
        m.forward_multi(toks[:, (1 + steps) % WINDOW].tolist(), states)
        steps += 1
    dt = time.perf_counter() - t0
    m.close()
    return n * steps / dt, steps, dt, O.get_threads()


def cpu_baseline(q8_path: str, n: int, budget_s: float, min_steps: int = 2):
    v, steps, dt, thr = cpu_time(q8_path, "q8", n, budget_s, min_steps)
    return {"value": round(v, 2), "unit": "tok/s", "cores": thr, "kind": "port",
            "sample": f"{steps} lockstep steps x {n} streams (Q8 group 64, Mamba-130M, {dt:.1f} s), "
                      f"C restatement of the reference CPU path (oracle/mamba_oracle.c, AVX2 lane order), "
                      f"{thr} threads on {os.cpu_count()} host CPUs ({cpu_model()})"}


def cpu_rows(f32_path: str, q8_path: str, budget_s: float) -> dict:
    """The reference CPU path's rows of the north star's baseline plan: F32 and Q8 single stream,
    lockstep N=32 in Q8 and F32, each on all host threads."""
    out = {"cpu_model": cpu_model(), "nproc": os.cpu_count(),
           "impl": "C restatement of the reference CPU path (oracle/mamba_oracle.c, AVX2 lane order)"}
    for prof, path in (("f32", f32_path), ("q8", q8_path)):
        for n in (1, 32):
            v, steps, dt, thr = cpu_time(path, prof, n, budget_s)
            out[f"{prof}_n{n}"] = {"tok_s": round(v, 2), "steps": steps, "seconds": round(dt, 2), "threads": thr}
    return out


# ---------------------------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------------------------

def run_b200(args, rank, world, local, dist):
    import torch
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)

    def barrier():
        if dist is not None:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        return shard_max(x, dist, dev)

    from redukt_b200.plugin import PluginBackend
    f32_path, q8_path = model_paths(rank, world, barrier)
    dims = rbin.MAMBA_130M
    n, K, W = args.streams, args.steps, args.warmup
    b = PluginBackend(q8_path, device_id=local)
    b.batch_init(n)
    b.set_reset_every(4096)
    V = b.vocab_size
    windows = zipf_tokens(n, WINDOW, vocab=V, seed_base=ZIPF_SEED_BASE + rank * n)
    d_windows = torch.from_numpy(windows.T.copy().astype(np.int32)).to(dev)  # [T, n]
    d_slots = torch.arange(n, dtype=torch.int32, device=dev)
    d_tok = torch.empty(n, dtype=torch.int32, device=dev)
    d_out = torch.empty((n, V), dtype=torch.float32, device=dev)
    stream = torch.cuda.Stream(dev)  # a real stream: handle 0 would select the library's own stream
    sh = stream.cuda_stream
    torch.cuda.set_stream(stream)

    def dev_step(t):
        d_tok.copy_(d_windows[t % WINDOW])
        b.forward_batch_device(n, d_slots.data_ptr(), d_tok.data_ptr(), d_out.data_ptr(), stream=sh)

    t = 0
    for _ in range(W):
        dev_step(t)
        t += 1
    torch.cuda.synchronize()
    clocks = ClockSampler(local)

    def roll(seconds):
        """Untimed steps of the same workload around the timed region, so the clock sampler (one
        sample per 200 ms) sees the clocks under this load even when the timed region is short."""
        nonlocal t
        t0 = time.perf_counter()
        while time.perf_counter() - t0 < seconds:
            for _ in range(32):
                dev_step(t)
                t += 1
            torch.cuda.synchronize()
    roll(0.8)
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(K):
        dev_step(t)
        t += 1
    e1.record(stream)
    torch.cuda.synchronize()
    dev_ms = e0.elapsed_time(e1)
    roll(0.8)
    clk = clocks.stop()
    barrier()
    torch.cuda.synchronize()
    dev_ms = max_over_ranks(dev_ms)
    launches_per_step = b.info_words()["launches_per_step"]

    # per-kernel device times: each class's launches of one step replayed in isolation (CUDA graph,
    # L2 flushed before each replay), timed with CUDA events
    # (batches of up to 32 streams run every layer in one persistent kernel, class "step")
    fused = n <= FUSED_MAX_N
    classes = ("embed", "step", "head") if fused else ("embed", "norm", "in_proj", "x_proj", "scan", "out_proj", "head")
    kt = {c: b.time_kernel(c, n, reps=5) for c in classes}
    per_step_launches = {"embed": 1, "norm": dims.n_layer + 1, "in_proj": dims.n_layer, "x_proj": dims.n_layer,
                         "scan": dims.n_layer, "out_proj": dims.n_layer, "head": 1, "step": 1}

    # e2e through the C ABI with host buffers (pinned output)
    h_out = torch.empty((n, V), dtype=torch.float32, pin_memory=True).numpy()
    slots = list(range(n))
    for i in range(W):
        b.forward_batch(slots, windows[:, t % WINDOW], out=h_out)
        t += 1
    torch.cuda.synchronize()
    barrier()
    t0 = time.perf_counter()
    for i in range(K):
        b.forward_batch(slots, windows[:, t % WINDOW], out=h_out)
        t += 1
    e2e_s = max_over_ranks(time.perf_counter() - t0)

    wbytes, per_stream = dims_bytes(dims, "q8")
    step_bytes = wbytes + n * per_stream
    peaks = load_peaks()
    ms_step = dev_ms / K
    value = world * n * K / (dev_ms / 1e3)
    res = {
        "metric": METRIC, "value": round(value, 1), "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": round(ms_step, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int8 weights x f32 activations (exact int8 digit products), f32 state", "data": "synthetic",
        "config": {"workload": "configs[1]: Mamba-130M Q8 (group 64) lockstep decode", "model": "Mamba-130M",
                   "streams_per_gpu": n, "global_batch": n * world, "window_tokens": WINDOW,
                   "reset_every": 4096, "parallelism": f"windows sharded over {world} GPU(s), no collective",
                   "l2": f"working set {step_bytes / 1e6:.0f} MB per step > {L2_BYTES / 2**20:.0f} MiB L2 (no flush)"},
        "clocks": clk,
        "gpu_launches": launches_per_step * K,
        "e2e": {"value": round(world * n * K / e2e_s, 1), "unit": "tok/s", "h2d_bytes_per_step": n * 8,
                "d2h_bytes_per_step": n * V * 4},
        "step_roofline": {"bound": "hbm", "algorithmic_bytes": step_bytes,
                          "achieved_gbs": round(step_bytes / (ms_step / 1e3) / 1e9, 1), "peak_gbs": peaks["hbm_gbs"],
                          "frac": round(step_bytes / (ms_step / 1e3) / 1e9 / peaks["hbm_gbs"], 4),
                          "peak_source": peaks["source"]},
    }
    # dominant kernel
    kernels = {}
    for cls, ms in kt.items():
        nl = per_step_launches[cls]
        by = kernel_bytes(cls, n, dims, "q8")
        avg_us = ms * 1e3
        kernels[cls] = {"launches_per_step": nl, "avg_us": round(avg_us, 3), "step_us": round(avg_us * nl, 2),
                        "bytes_per_launch": by, "gbs": round(by / (avg_us / 1e6) / 1e9, 1)}
    tot = sum(k["step_us"] for k in kernels.values()) or 1.0
    for k in kernels.values():
        k["share"] = round(k["step_us"] / tot, 4)
    top = max(kernels, key=lambda c: kernels[c]["step_us"])
    tr = load_traffic().get(f"q8_n{n}", {}).get(top)
    kd = kernels[top]
    res["roofline"] = {"kernel": top, "bound": "hbm", "achieved": kd["gbs"], "peak": peaks["hbm_gbs"], "unit": "GB/s",
                       "frac": round(kd["gbs"] / peaks["hbm_gbs"], 4), "traffic": tr,
                       "algorithmic_bytes_per_launch": kd["bytes_per_launch"], "peak_source": peaks["source"]}
    res["kernels"] = kernels

    if world == 1 and not args.no_cdf:   # before the sweep, which replaces the loaded model
        res["coder_cdf"] = coder_cdf(b.libobj, n, V, dev, with_cpu=rank == 0 and not args.no_cpu_baseline,
                                     backend=b, windows=windows)
    res["archive_batch"] = archive_batch(b, rank, world, dev, stream, max_over_ranks, barrier, K, W)
    if not args.no_archive:
        res["archive"] = archive_run(b, rank, world, args.archive_windows, max_over_ranks, barrier)
    res["determinism"] = determinism(b, rank, world, n, dev, dist)
    with_cpu = rank == 0 and world == 1 and not args.no_cpu_baseline
    if world == 1 and not args.no_sweep:
        res["sweep"] = sweep(b, f32_path, q8_path, dims, args, dev, peaks, with_cpu)
    else:
        b.close()
    if with_cpu:
        res["cpu_baseline"] = cpu_baseline(q8_path, n, args.cpu_seconds)
        res["cpu_baselines"] = cpu_rows(f32_path, q8_path, args.cpu_seconds / 4)
    return res


def archive_batch(b, rank, world, dev, stream, max_over_ranks, barrier, K, W) -> dict:
    """configs[4]'s per-GPU batch: 512 lockstep streams per GPU (device-resident step, CUDA-graph
    replay), timed with CUDA events and taken as the max over ranks; whole-job tok/s."""
    import torch
    n = 512
    V = b.vocab_size
    b.batch_init(n)
    b.set_reset_every(4096)
    toks = torch.from_numpy(zipf_tokens(n, W + K, vocab=V, seed_base=ZIPF_SEED_BASE + 7 * 4096 + rank * n).T.copy()
                            .astype(np.int32)).to(dev)
    slots = torch.arange(n, dtype=torch.int32, device=dev)
    tok = torch.empty(n, dtype=torch.int32, device=dev)
    o = torch.empty((n, V), dtype=torch.float32, device=dev)

    def step(i):
        tok.copy_(toks[i])
        b.forward_batch_device(n, slots.data_ptr(), tok.data_ptr(), o.data_ptr(), stream=stream.cuda_stream)
    for i in range(W):
        step(i)
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(K):
        step(W + i)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1)) / K
    b.set_reset_every(0)
    if b.device_error():
        raise RuntimeError("archive batch: device error word set")
    del o, toks
    return {"streams_per_gpu": n, "n_gpus": world, "ms_per_step": round(ms, 4),
            "tok_s": round(world * n / ms * 1e3, 1), "steps": K, "scaling": "weak"}


def archive_run(b, rank, world, n, max_over_ranks, barrier) -> dict:
    """configs[4] on this rank's share: n windows of 10 KB of the synthetic order-3 Markov text
    (global windows rank*n .. rank*n + n - 1), Mamba-130M Q8, reset every 4096 forwards, compressed
    in lockstep (device step + coder CDF per token, native range coder, RDKT v5 + CRC-32) and
    decompressed in lockstep on the GPU; every window must come back byte-exact with its CRC-32
    passing.  Times are wall clock around each pass (the host coder is part of it), max over ranks."""
    from redukt_b200 import archive as A
    from redukt_b200.workload import archive_tokenizer, archive_windows
    cache = os.environ.get("REDUKT_B200_MODEL_CACHE", os.path.join(tempfile.gettempdir(), "redukt_b200_models"))
    tok = archive_tokenizer(b.vocab_size, cache)
    wins = archive_windows(n, first=rank * n)
    tokens = sum(len(tok.encode(w)) for w in wins)
    b.batch_init(n)
    barrier()
    t0 = time.perf_counter()
    arcs = A.compress_windows(b, wins, tok)
    t_enc = max_over_ranks(time.perf_counter() - t0)
    barrier()
    t0 = time.perf_counter()
    back = A.decompress_windows(b, arcs, tok)
    t_dec = max_over_ranks(time.perf_counter() - t0)
    ok = sum(1 for x, w in zip(back, wins) if x == w)
    raw = sum(len(w) for w in wins)
    comp = sum(len(a) for a in arcs)
    return {"windows_per_gpu": n, "window_bytes": len(wins[0]) if wins else 0, "n_gpus": world,
            "tokens_per_gpu": tokens, "bytes_per_token": round(raw / max(1, tokens), 3),
            "compress_tok_s": round(world * tokens / t_enc, 1), "decompress_tok_s": round(world * tokens / t_dec, 1),
            "compress_s": round(t_enc, 2), "decompress_s": round(t_dec, 2),
            "round_trip_exact_windows": ok, "crc_checked": True,
            "bits_per_byte": round(8.0 * comp / max(1, raw), 4),
            "what": "lockstep archive: redukt_b200_forward_batch_cdf per token + native range coder "
                    "(libredukt_archive.so), RDKT v5 with CRC-32; no CM ensemble"}


def window_hash(b, window: int, steps: int = 8) -> str:
    """sha256 (first 16 hex digits) of the logits of global window `window` (its Zipf seed), run as
    the only stream of slot 0 from zero state for `steps` tokens."""
    import hashlib
    toks = zipf_tokens(1, steps, vocab=b.vocab_size, seed_base=ZIPF_SEED_BASE + window)
    b.batch_reset([0])
    h = hashlib.sha256()
    for t in range(steps):
        h.update(b.forward_batch([0], toks[:, t]).tobytes())
    return h.hexdigest()[:16]


def determinism(b, rank, world, n, dev, dist) -> dict:
    """Same window, same bits on every GPU and for every GPU count.  Rank r owns global windows
    r*n .. r*n+n-1; it hashes the logits of its first window.  Rank 0 gathers the hashes and
    recomputes every rank's window on its own GPU; the single-GPU line carries the hashes of the
    first windows of the ranks of an 8-GPU run, so lines of different GPU counts can be compared."""
    import torch
    b.batch_init(max(n, 1))
    mine = window_hash(b, rank * n)
    got = {rank * n: mine}
    if dist is not None:
        t = torch.tensor([int(mine, 16) >> 1], dtype=torch.int64, device=dev)  # 63 bits
        allv = [torch.zeros_like(t) for _ in range(world)]
        dist.all_gather(allv, t)
        got = {r * n: format(int(v.item()) << 1, "016x") for r, v in enumerate(allv)}
    if rank != 0:
        return {}
    want = {w: window_hash(b, w) for w in sorted(set(list(got) + [r * n for r in range(8)]))}
    match = all((int(got[w], 16) >> 1) == (int(want[w], 16) >> 1) for w in got)
    return {"steps": 8, "window_hashes": want, "ranks_agree_with_rank0": match,
            "what": "sha256 prefix of 8 steps of logits of one window (slot 0, fresh state)"}


def sweep(b, f32_path, q8_path, dims, args, dev, peaks, with_cpu: bool):
    """device tok/s at 1/32/128/1024 streams, Q8 and F32.  Each stream runs a Zipf(1.1)
    window with the device-side reset every 4,096 tokens; the slots' reset counters are set so the
    timed steps are the window positions around 4,096 and one reset falls inside the timed region.
    Q8 at 128 and 1024 streams also gets the per-kernel breakdown (each class replayed in isolation
    after an L2 flush).  With with_cpu, the reference CPU path (C restatement, all host threads) is
    timed on a bounded sample of the same configuration beside it."""
    import torch
    from redukt_b200.plugin import PluginBackend
    out = {}
    classes = ("embed", "norm", "in_proj", "x_proj", "scan", "out_proj", "head")
    per_step = {"embed": 1, "norm": dims.n_layer + 1, "in_proj": dims.n_layer, "x_proj": dims.n_layer,
                "scan": dims.n_layer, "out_proj": dims.n_layer, "head": 1}
    for prof, path in (("q8", q8_path), ("f32", f32_path)):
        if prof == "f32":
            b.close()
            b = PluginBackend(path, device_id=dev.index)
        for n in SWEEP_N:
            W = max(3, args.warmup)
            K = max(6, min(args.steps, int(2000 / max(1, n))))
            first = 4096 - W - K // 2          # window position of the first warm-up step
            win = zipf_tokens(n, first + W + K, vocab=b.vocab_size)
            toks = torch.from_numpy(win[:, first:].T.copy().astype(np.int32)).to(dev)
            b.batch_init(n)
            b.set_reset_every(4096)
            b.set_option("reset_counters", first)
            slots = torch.arange(n, dtype=torch.int32, device=dev)
            tok = torch.empty(n, dtype=torch.int32, device=dev)
            o = torch.empty((n, b.vocab_size), dtype=torch.float32, device=dev)
            sh = torch.cuda.current_stream(dev).cuda_stream
            assert sh != 0, "the sweep must run on a non-default stream"

            def step(i):
                tok.copy_(toks[i])
                b.forward_batch_device(n, slots.data_ptr(), tok.data_ptr(), o.data_ptr(), stream=sh)
            for i in range(W):
                step(i)
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(torch.cuda.current_stream(dev))
            for i in range(K):
                step(W + i)
            e1.record(torch.cuda.current_stream(dev))
            torch.cuda.synchronize()
            if b.device_error():
                raise RuntimeError(f"sweep {prof} n={n}: device error word set")
            b.set_reset_every(0)
            ms = e0.elapsed_time(e1) / K
            wb, ps = dims_bytes(dims, prof)
            by = wb + n * ps
            e = {"tok_s": round(n / ms * 1e3, 1), "ms_per_step": round(ms, 4), "steps": K,
                 "positions": f"{first + W}-{first + W + K - 1} of a 4,352-token window (reset before 4,096)",
                 "bytes_per_step": by, "hbm_frac": round(by / (ms / 1e3) / 1e9 / peaks["hbm_gbs"], 4)}
            if prof == "q8" and n in (128, 1024):
                ks = {}
                for c in classes:
                    us = b.time_kernel(c, n, reps=3) * 1e3
                    kb = kernel_bytes(c, n, dims, prof)
                    ks[c] = {"avg_us": round(us, 2), "step_us": round(us * per_step[c], 1),
                             "gbs": round(kb / (us / 1e6) / 1e9, 1)}
                e["kernels"] = ks
            if with_cpu:
                v, st, dt, thr = cpu_time(path, prof, n, budget_s=1.5, min_steps=1)
                e["cpu_tok_s"] = round(v, 2)
                e["cpu_sample"] = f"{st} steps x {n} streams, {thr} threads, {dt:.1f} s"
                e["vs_cpu"] = round(e["tok_s"] / v, 1)
            out[f"{prof}_n{n}"] = e
            del o, toks
    b.close()
    out.update(sweep_rwkv7(args, dev, peaks))
    return out


def sweep_rwkv7(args, dev, peaks):
    """RWKV-7 0.1B (W8A8, the reference's default quantisation) decode tok/s at 256
    lockstep streams of uniform byte tokens (and at 1 and 32), device-resident inputs."""
    import torch
    from redukt_b200.plugin import PluginBackend
    cache = os.environ.get("REDUKT_B200_MODEL_CACHE", os.path.join(tempfile.gettempdir(), "redukt_b200_models"))
    path = rwkv7_rbin.ensure_model(os.path.join(cache, "rwkv7_0_1b.rbin"), rwkv7_rbin.RWKV7_0_1B)
    dims = rwkv7_rbin.RWKV7_0_1B
    wb, ps = rwkv7_bytes(dims)
    b = PluginBackend(path, device_id=dev.index)
    out = {}
    for n in RWKV_N:
        b.batch_init(n)
        toks = torch.from_numpy(rwkv7_rbin.byte_tokens(n, 64).T.copy().astype(np.int32)).to(dev)
        slots = torch.arange(n, dtype=torch.int32, device=dev)
        tok = torch.empty(n, dtype=torch.int32, device=dev)
        o = torch.empty((n, b.vocab_size), dtype=torch.float32, device=dev)
        sh = torch.cuda.current_stream(dev).cuda_stream
        assert sh != 0, "the sweep must run on a non-default stream"

        def step(i):
            tok.copy_(toks[i % 64])
            b.forward_batch_device(n, slots.data_ptr(), tok.data_ptr(), o.data_ptr(), stream=sh)
        for i in range(max(3, args.warmup)):
            step(i)
        torch.cuda.synchronize()
        K = max(5, min(args.steps, int(4000 / max(1, n)) + 5))
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(torch.cuda.current_stream(dev))
        for i in range(K):
            step(i)
        e1.record(torch.cuda.current_stream(dev))
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / K
        by = wb + n * ps
        out[f"rwkv7_w8a8_n{n}"] = {"tok_s": round(n / ms * 1e3, 1), "ms_per_step": round(ms, 4), "steps": K,
                                   "hbm_frac": round(by / (ms / 1e3) / 1e9 / peaks["hbm_gbs"], 4),
                                   "bytes_per_step": by}
        if b.device_error():
            raise RuntimeError("RWKV-7 sweep: device error word set")
        del o, toks
    b.close()
    return out


# ---------------------------------------------------------------------------------------------
# Reference arm: the reference CPU path (C restatement) on this host's cores
# ---------------------------------------------------------------------------------------------

def run_reference(args, rank, world):
    if rank != 0:
        return None
    from oracle import oracle as O
    f32, q8 = model_paths(0, 1, lambda: None)
    m = O.Model(q8, O.PROFILE_Q8, 64)
    n = args.streams
    toks = zipf_tokens(n, WINDOW, vocab=m.vocab)
    states = [m.new_state(4096) for _ in range(n)]
    t = 0
    # bound the whole run to about two minutes: shrink the streams per step if needed
    t0 = time.perf_counter()
    m.forward_multi(toks[:, t].tolist(), states)
    t += 1
    per_step = time.perf_counter() - t0
    ns = n
    if per_step * (args.steps + args.warmup) > 120.0:
        ns = max(1, int(n * 120.0 / (per_step * (args.steps + args.warmup))))
        states = states[:ns]
    for _ in range(args.warmup):
        m.forward_multi(toks[:ns, t % WINDOW].tolist(), states)
        t += 1
    t0 = time.perf_counter()
    for _ in range(args.steps):
        m.forward_multi(toks[:ns, t % WINDOW].tolist(), states)
        t += 1
    dt = time.perf_counter() - t0
    v = ns * args.steps / dt
    sample = (f"{args.steps} lockstep steps x {ns} streams (of {n}) of Mamba-130M Q8 group 64; "
              f"C restatement of the reference CPU path (oracle/mamba_oracle.c), {O.get_threads()} threads")
    return {"impl": "reference", "metric": METRIC, "value": round(v, 2), "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8 weights x f32",
            "data": "synthetic",
            "config": {"workload": "configs[1]: Mamba-130M Q8 (group 64) lockstep decode", "model": "Mamba-130M",
                       "streams_per_gpu": n, "window_tokens": WINDOW, "parallelism": "host CPU, rank 0 only"},
            "cpu_baseline": {"value": round(v, 2), "unit": "tok/s", "cores": O.get_threads(), "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(v, 2), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def coder_cdf(lib, n: int, vocab: int, dev, with_cpu: bool, reps: int = 20, backend=None, windows=None) -> dict:
    """The coder's 24-bit CDF for the step's n rows (redukt_b200_cdf_device), the reference's
    cdf_from_logits_with(.., FmathV1) + Cdf::from_probs: device time of the kernel (CUDA events, L2
    flushed before each launch), end to end through the host-buffer C ABI in encoder mode (logits in,
    {symbol, low, high} out), a bit-exactness check against the C oracle, and the oracle on all host
    cores.  Seeded synthetic logits N(0, 3^2), the spread of a trained LM's logits."""
    import torch
    from redukt_b200.plugin import BackendResult
    rng = np.random.default_rng(2024)
    x = (rng.standard_normal((n, vocab)) * 3).astype(np.float32)
    d_x = torch.from_numpy(x).to(dev)
    d_c = torch.empty((n, vocab + 1), dtype=torch.int32, device=dev)
    flush = torch.empty(2 * L2_BYTES, dtype=torch.uint8, device=dev)
    st = torch.cuda.current_stream(dev)

    def call():
        rc = lib.cdf_device(d_x.data_ptr(), n, vocab, vocab, d_c.data_ptr(), vocab + 1, stream=st.cuda_stream)
        assert rc == BackendResult.OK, lib.last_error()
    for _ in range(3):
        call()
    torch.cuda.synchronize()
    evs = []
    for _ in range(reps):
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        call()
        e1.record(st)
        evs.append((e0, e1))
    torch.cuda.synchronize()
    ms = sorted(a.elapsed_time(b) for a, b in evs)[reps // 2]
    from oracle import oracle as O
    got = d_c.cpu().numpy().view(np.uint32)
    k = min(n, 4)
    exact = bool(np.array_equal(got[:k], O.cdf_from_logits(x[:k])))

    sym = rng.integers(0, vocab, n).astype(np.uint32)
    for _ in range(3):
        lib.cdf(x, symbols=sym, want_cdf=False)
    t0 = time.perf_counter()
    for _ in range(reps):
        _, q = lib.cdf(x, symbols=sym, want_cdf=False)
    e2e_s = (time.perf_counter() - t0) / reps
    bytes_per_row = vocab * 4 + (vocab + 1) * 4
    step_cdf = None
    if backend is not None:
        # the coder's view of a step: redukt_b200_forward_batch_cdf in encoder mode (tokens and next
        # symbols in, {symbol, low, high} out: the step and the CDF on the device, 12 bytes per stream back)
        slots = list(range(n))
        T = windows.shape[1]
        for i in range(3):
            backend.forward_batch_cdf(slots, windows[:, i % T], symbols=windows[:, (i + 1) % T])
        t0 = time.perf_counter()
        for i in range(reps):
            backend.forward_batch_cdf(slots, windows[:, (3 + i) % T], symbols=windows[:, (4 + i) % T])
        dt = (time.perf_counter() - t0) / reps
        step_cdf = {"value": round(n / dt, 1), "unit": "tok/s", "ms_per_step": round(dt * 1e3, 4),
                    "h2d_bytes_per_step": n * 12, "d2h_bytes_per_step": n * 12,
                    "what": "redukt_b200_forward_batch_cdf: step + coder CDF on the device, encoder queries back"}
    out = {"rows": n, "vocab": vocab, "kernel_ms": round(ms, 4), "rows_per_s": round(n / (ms / 1e3), 1),
           "e2e_rows_per_s": round(n / e2e_s, 1), "e2e": "host logits in, {symbol, cdf[symbol], cdf[symbol+1]} out",
           "h2d_bytes_per_call": n * vocab * 4 + n * 4, "d2h_bytes_per_call": n * 12,
           "gpu_launches_per_call": 1, "bit_exact_vs_oracle_rows": k if exact else -1,
           "bound": "latency: two exact binary64 index-order sums per row as binade-blocked scan rounds",
           "algorithmic_bytes": n * bytes_per_row,
           "achieved_gbs": round(n * bytes_per_row / (ms / 1e3) / 1e9, 1)}
    if step_cdf is not None:
        out["e2e_step_and_cdf"] = step_cdf
    if with_cpu:
        thr = os.cpu_count() or 1
        rows = min(max(n, 2 * thr), 512)
        xs = np.resize(x, (rows, vocab))
        O.cdf_from_logits(xs[:thr], threads=thr)
        t0 = time.perf_counter()
        calls = 0
        while calls < 2 or time.perf_counter() - t0 < 3.0:
            O.cdf_from_logits(xs, threads=thr)
            calls += 1
        dt = time.perf_counter() - t0
        out["cpu_baseline"] = {"value": round(rows * calls / dt, 1), "unit": "rows/s", "cores": thr, "kind": "port",
                               "sample": f"{calls} x {rows} rows of {vocab} logits ({dt:.1f} s), "
                                         f"oracle/cdf_oracle.c (scalar, one row per thread)"}
    return out


def run_profile_cdf(n: int) -> None:
    """Small case for ncu captures of the CDF kernel: two launches over n rows of 50,280 logits."""
    import torch
    from redukt_b200.plugin import BackendResult, PluginLibrary
    lib = PluginLibrary()
    V = rbin.MAMBA_130M.vocab
    x = (torch.randn((n, V), generator=torch.Generator().manual_seed(1)) * 3).cuda()
    c = torch.empty((n, V + 1), dtype=torch.int32, device="cuda")
    for _ in range(2):
        assert lib.cdf_device(x.data_ptr(), n, V, V, c.data_ptr(), V + 1) == BackendResult.OK, lib.last_error()
    torch.cuda.synchronize()
    print(json.dumps({"profile_cdf": n, "vocab": V, "launches": 2}))


def run_profile_case(n: int, quant: str = "q8", fused: int = 1) -> None:
    """Small case for ncu captures: two eager (graph-free) steps of n streams through the C ABI.
    quant "rwkv7" runs the RWKV-7 0.1B W8A8 model instead of Mamba-130M; fused 0 runs the Mamba
    per-kernel step even where the fused step kernel would (Q8, n <= 32)."""
    from redukt_b200.plugin import PluginBackend
    if quant == "rwkv7":
        cache = os.environ.get("REDUKT_B200_MODEL_CACHE", os.path.join(tempfile.gettempdir(), "redukt_b200_models"))
        path = rwkv7_rbin.ensure_model(os.path.join(cache, "rwkv7_0_1b.rbin"), rwkv7_rbin.RWKV7_0_1B)
        b = PluginBackend(path)
        b.set_option("graphs", 0)
        b.batch_init(n)
        toks = rwkv7_rbin.byte_tokens(n, 2)
        for t in range(2):
            b.forward_batch(list(range(n)), toks[:, t])
        b.close()
        print(json.dumps({"profile_case": n, "quant": quant, "steps": 2}))
        return
    f32_path, q8_path = model_paths(0, 1, lambda: None)
    b = PluginBackend(q8_path if quant == "q8" else f32_path)
    b.set_option("graphs", 0)
    b.set_option("fused", fused)
    b.batch_init(n)
    toks = zipf_tokens(n, 2, vocab=b.vocab_size)
    for t in range(2):
        b.forward_batch(list(range(n)), toks[:, t])
    b.close()
    print(json.dumps({"profile_case": n, "quant": quant, "steps": 2}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--streams", type=int, default=STREAMS)
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--profile-case", type=int, default=0,
                    help="run two eager steps of N streams and exit (small case for ncu captures)")
    ap.add_argument("--profile-quant", default="q8", choices=["q8", "f32", "rwkv7"])
    ap.add_argument("--profile-fused", type=int, default=1, choices=[0, 1],
                    help="0: the per-kernel Mamba step even at n <= 32")
    ap.add_argument("--no-cdf", action="store_true", help="skip the coder-CDF measurement")
    ap.add_argument("--no-archive", action="store_true", help="skip the configs[4] archive round trip")
    ap.add_argument("--archive-windows", type=int, default=512, help="10 KB windows per GPU for the archive")
    ap.add_argument("--profile-cdf", type=int, default=0,
                    help="run two launches of the CDF kernel over N rows and exit (small case for ncu)")
    args = ap.parse_args()
    if args.profile_cdf:
        run_profile_cdf(args.profile_cdf)
        return
    if args.profile_case:
        run_profile_case(args.profile_case, args.profile_quant, args.profile_fused)
        return
    args.warmup = max(3, args.warmup)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        res = run_reference(args, rank, world)
        if res is not None:
            print(json.dumps(res), flush=True)
        return
    dist = None
    if world > 1:
        import datetime

        import torch
        import torch.distributed as D
        torch.cuda.set_device(local)
        D.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                             device_id=torch.device("cuda", local))
        dist = D
    try:
        res = run_b200(args, rank, world, local, dist)
    finally:
        if dist is not None:
            dist.barrier()
            dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
