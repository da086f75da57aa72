#!/usr/bin/env python3
"""Benchmark: Whisper-large-v3 Q4_0 batched transcription on B200.

Workload: 64 synthetic 30 s clips per GPU; encoder
forward, then a 4-token prefix and a 128-token teacher-forced decode through
the paged Q8_0 self-attention KV cache and the Q8_0 cross-attention store.
One "step" = that whole pass for one batch of 64 utterances. With N GPUs
(torchrun) every rank processes its own batch (utterances shard by request;
weak scaling, no collective on the hot path).

Prints one JSON line (rank 0). `value` = audio-seconds per second with the
log-mels already in HBM; `e2e` = the same metric with the log-mels copied
from pinned host memory and the greedy ids read back every step.

`--impl reference` times the reference's CPU algorithm (the C++ restatement
in oracle/, the Rust reference cannot be built here) on a bounded sample of
the same workload and extrapolates to the metric's unit.
"""
from __future__ import annotations

import argparse
import dataclasses
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

# The arithmetic of each --precision mode, as the JSON lines' "dtype" states it.
PREC_DTYPE = {"split": "f16 hi+lo tensor-core operands, fp32 accumulate (Q4_0 weights, Q8_0 KV)",
              "enc_f16": "encoder: f16 tensor-core operands, fp32 accumulate; decoder: f16 hi+lo "
                         "operands, fp32 accumulate (Q4_0 weights, Q8_0 KV)",
              "f16": "f16 (Q4_0 weights, Q8_0 KV)"}

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CLIP_SECONDS = 30.0
PREFIX = 4
METRIC = "audio-s/s + decode tok/s, Whisper-large-v3 Q4_0 @1/2/4/8 B200; % of roofline"


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p["hbm_gbs"], p["bf16_tflops"], p.get("bf16_tflops_sustained", p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, 1400.0, "fallback"


class ClockSampler:
    """Samples nvidia-smi SM clocks and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu_index = gpu_index
        self.rows = []
        self._stop = threading.Event()
        self._t = None

    def _run(self):
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", "-i", str(self.gpu_index), f"--query-gpu={self.FIELDS}",
                                      "--format=csv,noheader,nounits"], capture_output=True, text=True, timeout=5)
                for line in out.stdout.strip().splitlines():
                    self.rows.append([c.strip() for c in line.split(",")])
            except Exception:
                pass
            self._stop.wait(0.2)

    def __enter__(self):
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        self._t.join(timeout=10)

    def summary(self):
        def num(x):
            try:
                return float(x)
            except ValueError:
                return None
        sm = [v for v in (num(r[1]) for r in self.rows if len(r) > 2) if v is not None]
        mx = [v for v in (num(r[2]) for r in self.rows if len(r) > 2) if v is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for r in self.rows:
            for i, n in enumerate(names):
                if len(r) > 5 + i and r[5 + i].lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(self.rows)}


def model_path(name: str) -> str:
    d = os.environ.get("VKB_BENCH_CACHE", "/tmp/vkb_bench")
    os.makedirs(d, exist_ok=True)
    return os.path.join(d, f"whisper_{name}_seed0.gguf")


def ensure_model(path: str, arch, qtag: int):
    from vokra_b200 import synth
    if not os.path.exists(path):
        tmp = path + f".tmp{os.getpid()}"
        synth.write_synthetic_whisper(tmp, arch, qtag, seed=0)
        os.replace(tmp, path)
    return path


def synthetic_pcm(n: int, seed: int, n_samples: int = 480000, sr: int = 16000) -> np.ndarray:
    """n clips of 16 kHz PCM: white noise at RMS 0.1 plus three tones (f ~ U(100, 4000) Hz,
    phase ~ U(0, 2 pi), amplitude 0.05), clipped to +-1; clip i from rng(seed + i)."""
    t = np.arange(n_samples, dtype=np.float64) / sr
    out = np.empty((n, n_samples), np.float32)
    for i in range(n):
        rng = np.random.default_rng(seed + i)
        x = 0.1 * rng.standard_normal(n_samples)
        for f, ph in zip(rng.uniform(100.0, 4000.0, 3), rng.uniform(0.0, 2 * np.pi, 3)):
            x += 0.05 * np.sin(2 * np.pi * f * t + ph)
        out[i] = np.clip(x, -1.0, 1.0)
    return out


def synthetic_logmels(n: int, n_mels: int, n_frames: int, seed: int) -> np.ndarray:
    """Seeded stand-in for the frontend output, in Whisper's normalised log-mel range."""
    rng = np.random.default_rng(seed)
    base = rng.uniform(-0.8, 0.2, (n, n_mels, 1)).astype(np.float32)
    x = base + rng.standard_normal((n, n_mels, n_frames)).astype(np.float32) * np.float32(0.25)
    return np.clip(x, -1.0, 1.5).astype(np.float32)


# ---------------------------------------------------------------------------
# Multi-rank host logic (one process per GPU; utterances shard by request, no
# collective on the data path). Kept free of CUDA so it runs under gloo on CPU.
# ---------------------------------------------------------------------------
def rank_input_seed(rank: int) -> int:
    """Each rank decodes its own clips: distinct seeded inputs per rank."""
    return 1000 + rank


def init_process_group(world: int, local_rank: int, backend: str, timeout_s: float | None = None):
    """Joins the job's process group (torchrun's env:// rendezvous on 127.0.0.1). With
    timeout_s, a collective that a dead rank never joins fails after that long."""
    import datetime
    import torch
    import torch.distributed as dist
    if world <= 1:
        return None
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    kw = {"timeout": datetime.timedelta(seconds=timeout_s)} if timeout_s else {}
    if backend == "nccl":
        dist.init_process_group("nccl", device_id=torch.device(f"cuda:{local_rank}"), **kw)
    else:
        dist.init_process_group(backend, **kw)
    return dist


def max_over_ranks(ms: float, dist, device) -> float:
    """The job's time is the slowest rank's device time."""
    if dist is None:
        return ms
    import torch
    t = torch.tensor([ms], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def job_throughput(world: int, clips: int, steps: int, tokens: int, ms: float):
    """Whole-job audio-seconds/s and decode tokens/s: every rank's clips over the max-over-ranks time."""
    audio = world * clips * CLIP_SECONDS * steps
    return audio / (ms / 1e3), world * clips * tokens * steps / (ms / 1e3)


# ---------------------------------------------------------------------------
# CPU leg: the oracle (reference algorithm restated in C++) on a bounded sample
# ---------------------------------------------------------------------------
def cpu_sample(arch, qtag, qname, n_tokens: int, threads: int):
    """Times 1 clip on a 2+2-layer model of the same dims and extrapolates to the full depth.

    The decoder keeps the reference's own caches: a dense f32 self-attention KvCache and f32
    cross K/V (crates/vokra-models/src/whisper/decoder.rs:183-216, 455-470). Returns the
    extrapolated full-depth rates and the measured wall time of the sample itself."""
    from oracle import py as o, whisper_ref
    o.lib().orc_set_threads(threads)
    small = dataclasses.replace(arch, n_audio_layer=2, n_text_layer=2)
    path = ensure_model(model_path(f"sample_{qname}_e2d2"), small, qtag)
    ref = whisper_ref.RefWhisper(path)
    pcm = synthetic_pcm(1, 123)[0]
    t_sample0 = time.perf_counter()
    t0 = time.perf_counter()
    lm = o.log_mel(pcm, arch.n_mels)
    t_front = time.perf_counter() - t0
    ref.n_audio_layer = 0
    t0 = time.perf_counter()
    ref.encode(lm)
    t_conv = time.perf_counter() - t0
    ref.n_audio_layer = 2
    t0 = time.perf_counter()
    enc = ref.encode(lm)
    t_enc2 = time.perf_counter() - t0
    t0 = time.perf_counter()
    dec = ref.decoder(enc, kv_mode="f32", cross_mode="f32")
    t_cross2 = time.perf_counter() - t0
    dec.step(list(arch.start_ids))
    steps = 3
    t0 = time.perf_counter()
    for i in range(steps):
        dec.step([100 + i])
    t_step2 = (time.perf_counter() - t0) / steps
    x = np.zeros((1, arch.d_model), np.float32)
    t0 = time.perf_counter()
    o.gemm_kn(x, ref.emb_t)
    t_head = time.perf_counter() - t0
    t_sample = time.perf_counter() - t_sample0
    L_e, L_d = arch.n_audio_layer, arch.n_text_layer
    t_enc = t_conv + (t_enc2 - t_conv) * L_e / 2
    t_cross = t_cross2 * L_d / 2
    t_step = t_head + max(0.0, t_step2 - t_head) * L_d / 2
    t_clip = t_front + t_enc + t_cross + n_tokens * t_step
    sample = (f"1 clip on a 2+2-layer {qname} model of the same dims, dense f32 self-KV and f32 cross K/V as the "
              f"reference decoder keeps them (log-mel {t_front:.2f}s, conv {t_conv:.2f}s, 2 enc layers "
              f"{t_enc2 - t_conv:.2f}s, cross K/V {t_cross2:.2f}s, decode step {t_step2 * 1e3:.1f}ms; "
              f"{t_sample:.1f}s wall per sample), extrapolated linearly to {L_e}+{L_d} layers and {n_tokens} "
              f"tokens = {t_clip:.1f}s per clip; the reference CPU algorithm restated in C++ (oracle/)")
    return {"audio_s_per_s": CLIP_SECONDS / t_clip, "tok_s": n_tokens / (t_cross + n_tokens * t_step),
            "sample": sample, "sample_wall_s": t_sample, "clip_s": t_clip}


def run_reference(args, rank):
    """The reference arm: the reference's CPU algorithm (oracle/, the Rust crate cannot be
    built here) on the host cores. Only numpy, the GGUF writer and the oracle's C++ library
    are loaded; nothing of libvkb200 runs in this process."""
    if rank != 0:
        return
    from vokra_b200 import synth
    arch = synth.WHISPER_LARGE_V3
    threads = os.cpu_count() or 1
    vals = []
    for i in range(args.warmup + args.steps):
        r = cpu_sample(arch, synth.Q4_0, "q4_0", args.tokens, threads)
        if i >= args.warmup:
            vals.append(r)
    v = float(np.median([r["audio_s_per_s"] for r in vals]))
    tok = float(np.median([r["tok_s"] for r in vals]))
    step_ms = 1000.0 * float(np.median([r["sample_wall_s"] for r in vals]))
    line = {
        "metric": METRIC, "impl": "reference", "value": v, "unit": "audio-s/s", "decode_tok_s": tok,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(step_ms, 1), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "configs[3]: whisper-large-v3 q4_0, log-mel frontend + encoder + 4-token prefix + "
                               "128 teacher-forced tokens, f32 self-KV and f32 cross K/V",
                   "step": "one sampled utterance on a 2+2-layer model of the same dims (ms_per_step is its "
                           "measured wall time); value extrapolates the sample's per-layer times to 32+32 "
                           "layers and 128 tokens (clip_s_extrapolated)",
                   "clip_s_extrapolated": round(float(np.median([r["clip_s"] for r in vals])), 2)},
        "cpu_baseline": {"value": v, "unit": "audio-s/s", "cores": threads, "kind": "port",
                         "sample": vals[-1]["sample"]},
        "e2e": {"value": v, "unit": "audio-s/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_kernel_only(args):
    """One kernel alone, for ncu: the encoder fc1 GEMM, or the decode cross-attention."""
    import ctypes as C
    import torch
    from vokra_b200 import _lib, ops, synth
    ctx = ops.Context(0)
    if args.kernel == "encoder":
        from vokra_b200 import whisper
        big = synth.WHISPER_LARGE_V3
        arch = dataclasses.replace(big, n_audio_layer=1, n_text_layer=1, n_vocab=1000, eot=999,
                                   start_ids=(1, 2, 3, 4))
        path = ensure_model(model_path("large_v3_dims_e1d1_q4_0"), arch, synth.Q4_0)
        prec = {"split": _lib.PREC_SPLIT, "f16": _lib.PREC_F16, "enc_f16": _lib.PREC_ENCODER_F16}[args.precision]
        _lib.check(_lib.load().vkb_context_set_precision(ctx.h, prec))
        model = whisper.WhisperModel(ctx, path)
        B = args.clips
        sess = whisper.Session(model, max_streams=B, max_clips=B, cross_kv_q8=True)
        lm = torch.from_numpy(synthetic_logmels(B, arch.n_mels, 2 * arch.n_audio_ctx, 5)).cuda()
        for _ in range(3):
            sess.encode(lm, list(range(B)))
        torch.cuda.synchronize()
        print(json.dumps({"kernel": args.kernel, "clips": B, "frames": arch.n_audio_ctx, "ok": True}))
        return
    if args.kernel == "xattn":
        B, T, H, D = args.clips, 1500, 20, 64
        W = H * D
        g = torch.Generator(device="cuda").manual_seed(3)
        kq = torch.empty((B * T, W), dtype=torch.int8, device="cuda")
        vq = torch.empty_like(kq)
        kd = torch.empty((B * T, W // 32), dtype=torch.float16, device="cuda")
        vd = torch.empty_like(kd)
        for q8, dd in ((kq, kd), (vq, vd)):
            ops.quantize_rows_q8_0(ctx, torch.randn((B * T, W), device="cuda", generator=g), q8, dd)
        q = torch.randn((B, W), device="cuda", generator=g) * 0.125
        seq = torch.arange(B, dtype=torch.int32, device="cuda")
        out = torch.empty((B, W), device="cuda")
        for _ in range(3):
            ops.attention_dense(ctx, q, seq, kq, vq, T, H, D, out, k_scale=kd, v_scale=vd)
        torch.cuda.synchronize()
        print(json.dumps({"kernel": args.kernel, "streams": B, "keys": T, "width": W, "ok": True}))
        return
    if args.kernel == "paged_decode":
        run_paged_decode(ctx, args)
        return
    if args.kernel == "decode_step":
        # one 64-stream decode step of the bench model at position ~100, alone between
        # cudaProfilerStart/Stop (for ncu --profile-from-start off)
        import torch
        from vokra_b200 import whisper
        arch = synth.WHISPER_LARGE_V3
        path = ensure_model(model_path("large_v3_q4_0"), arch, synth.Q4_0)
        model = whisper.WhisperModel(ctx, path)
        B = args.clips
        sess = whisper.Session(model, max_streams=B, max_step_tokens=B * PREFIX, max_clips=B, cross_kv_q8=True)
        st = np.arange(B, dtype=np.int32)
        sess.encode(torch.from_numpy(synthetic_logmels(B, arch.n_mels, 2 * arch.n_audio_ctx, 5)).cuda(), st)
        sess.step(np.repeat(st, PREFIX), np.tile(np.arange(PREFIX, dtype=np.int32), B),
                  np.tile(np.array(arch.start_ids[:PREFIX], np.int32), B))
        ids = torch.zeros(B, dtype=torch.int32, device="cuda")
        pos = PREFIX
        for _ in range(96):
            sess.step(st, np.full(B, pos, np.int32), np.full(B, 7, np.int32), ids_dev=ids)
            pos += 1
        torch.cuda.synchronize()
        torch.cuda.profiler.start()
        sess.step(st, np.full(B, pos, np.int32), np.full(B, 7, np.int32), ids_dev=ids)
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
        print(json.dumps({"kernel": args.kernel, "streams": B, "position": pos, "ok": True}))
        return
    if args.precision == "f16":
        _lib.check(_lib.load().vkb_context_set_precision(ctx.h, _lib.PREC_F16))
    M = 1500 if args.kernel == "fc1_m1500" else args.clips * 1500
    N, K = 5120, 1280
    wq = synth.quantize(synth.Q4_0, np.random.default_rng(7).standard_normal(N * K).astype(np.float32) * 0.02)
    w = ops.Weight(ctx, synth.Q4_0, N, K, wq)
    planes = 2 if args.precision == "split" else 1
    a = (torch.randn((planes * M, K), device="cuda") * 0.5).half()
    out = torch.empty((M, N), device="cuda", dtype=torch.float16)
    def fc1():
        _lib.check(_lib.load().vkb_linear(ctx.h, w.h, M, C.c_void_p(a.data_ptr()),
                                          _lib.DT_F16X2 if planes == 2 else _lib.DT_F16, None,
                                          C.c_void_p(out.data_ptr()), _lib.DT_F16, _lib.EPI_NONE, None,
                                          C.c_float(1.0)))
    for _ in range(3):
        fc1()
    torch.cuda.synchronize()
    # under a profiler only the three launches above run (ncu -s 2 -c 1 takes the last one)
    ms = None
    if not os.environ.get("VKB_BENCH_NO_TIMING"):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 10
        e0.record()
        for _ in range(reps):
            fc1()
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / reps
    print(json.dumps({"kernel": args.kernel, "M": M, "N": N, "K": K, "ok": True,
                      "ms_per_launch": ms, "tflops": None if ms is None else 2.0 * M * N * K / ms / 1e9}))


def run_paged_decode(ctx, args):
    """the decode step's fused append + self-attention over the paged
    Q8_0 cache (vkb_kv_append_attention, the kernel the session runs): 256 sequences, 20
    heads x 64, lengths U[16, 448] in 16-token pages scattered by a seeded permutation,
    Q/K/V N(0, 1). Prints one JSON line with the kernel's HBM roofline fraction."""
    import torch
    from vokra_b200 import _lib, ops
    n_seq, H, D, T, bs = 256, 20, 64, 448, 16
    W = H * D
    rng = np.random.default_rng(2024)
    pool = ops.QuantizedPagedKvCache(ctx, ops.KvDims(1, H, D, n_seq, 1, T), bs, _lib.KV_Q8_0,
                                     _lib.KV_LAYOUT_SEQUENCE)
    pool.set_page_table(rng.permutation(n_seq * (T // bs)).astype(np.int32))
    lengths = rng.integers(16, T + 1, n_seq)
    g = torch.Generator(device="cuda").manual_seed(3)
    s0 = 0
    while s0 < n_seq:
        s1, n_tok = s0, 0
        while s1 < n_seq and n_tok + int(lengths[s1]) - 1 <= 2048:
            n_tok += int(lengths[s1]) - 1
            s1 += 1
        seqs = np.concatenate([np.full(int(lengths[s]) - 1, s) for s in range(s0, s1)])
        poss = np.concatenate([np.arange(int(lengths[s]) - 1) for s in range(s0, s1)])
        pool.begin_step(seqs, poss)
        pool.append(0, torch.randn((len(seqs), W), device="cuda", generator=g),
                    torch.randn((len(seqs), W), device="cuda", generator=g))
        s0 = s1
    pool.begin_step(np.arange(n_seq), lengths - 1)
    assert pool.decode_fused()
    qkv = torch.randn((n_seq, 3 * W), device="cuda", generator=g)
    qkv[:, :W] *= D ** -0.5
    out = torch.empty((n_seq, W), device="cuda")
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")  # > L2: every launch reads the pages from HBM
    for _ in range(3):
        pool.append_attention(0, qkv, out)
    reps, ms = 20, 0.0
    stream = torch.cuda.current_stream()
    for _ in range(reps):
        flush.fill_(1)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        pool.append_attention(0, qkv, out)
        e1.record(stream)
        torch.cuda.synchronize()
        ms += e0.elapsed_time(e1) / reps
    keys = int(lengths.sum())
    # K and V int8 quants + one f16 scale per 32 channels of every key, the q|k|v rows in, the context out
    alg = keys * 2 * (W + W // 16) + n_seq * 3 * W * 4 + n_seq * W * 4
    hbm, _, _, peak_kind = _peaks()
    gbs = alg / (ms / 1e3) / 1e9
    print(json.dumps({"kernel": "paged_decode_kernel (vkb_kv_append_attention)",
                      "workload": "configs[2]: 256 sequences, 20 heads x 64, lengths U[16, 448], 16-token Q8_0 "
                                  "pages, seeded page permutation; L2 flushed before every launch",
                      "keys": keys, "algorithmic_bytes": alg, "us_per_launch": round(ms * 1e3, 2),
                      "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm, "unit": "GB/s",
                                   "frac": round(gbs / hbm, 4), "peak_kind": peak_kind}}), flush=True)
    # the cross-attention half of configs[2]: one query per sequence over its dense 1500 x 1280 K/V,
    # in the Q8_0 store the session keeps (the bench default) and in the f16 store
    del pool, flush
    n_ctx = 1500
    seq = torch.arange(n_seq, dtype=torch.int32, device="cuda")
    q = torch.randn((n_seq, W), device="cuda", generator=g) * D ** -0.5
    for store in ("q8_0", "f16"):
        if store == "q8_0":
            kq = torch.empty((n_seq * n_ctx, W), dtype=torch.int8, device="cuda")
            vq = torch.empty_like(kq)
            kd = torch.empty((n_seq * n_ctx, W // 32), dtype=torch.float16, device="cuda")
            vd = torch.empty_like(kd)
            for q8, dd in ((kq, kd), (vq, vd)):
                for r0 in range(0, n_seq * n_ctx, 96000):
                    r1 = min(n_seq * n_ctx, r0 + 96000)
                    ops.quantize_rows_q8_0(ctx, torch.randn((r1 - r0, W), device="cuda", generator=g), q8[r0:r1],
                                           dd[r0:r1])
            call = lambda: ops.attention_dense(ctx, q, seq, kq, vq, n_ctx, H, D, out, k_scale=kd, v_scale=vd)
            kv_bytes = n_seq * n_ctx * 2 * (W + W // 16)
        else:
            kq = torch.randn((n_seq * n_ctx, W), device="cuda", generator=g).half()
            vq = torch.randn((n_seq * n_ctx, W), device="cuda", generator=g).half()
            call = lambda: ops.attention_dense(ctx, q, seq, kq, vq, n_ctx, H, D, out)
            kv_bytes = n_seq * n_ctx * 2 * W * 2
        for _ in range(3):
            call()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 10
        e0.record(stream)
        for _ in range(reps):
            call()
        e1.record(stream)
        torch.cuda.synchronize()
        ms_x = e0.elapsed_time(e1) / reps
        alg_x = kv_bytes + 2 * n_seq * W * 4
        gbs_x = alg_x / (ms_x / 1e3) / 1e9
        print(json.dumps({"kernel": f"cross-attention over the dense {store} store (vkb_attention_dense)",
                          "workload": f"configs[2] cross half: 256 sequences x 1500 keys, 20 heads x 64, {store} "
                                      "K/V (> L2, read once per launch)",
                          "algorithmic_bytes": alg_x, "us_per_launch": round(ms_x * 1e3, 2),
                          "roofline": {"bound": "hbm", "achieved": round(gbs_x, 1), "peak": hbm, "unit": "GB/s",
                                       "frac": round(gbs_x / hbm, 4), "peak_kind": peak_kind}}), flush=True)
        del kq, vq


SWEEP_SHAPES = [(1280, 1280), (1280, 5120), (5120, 1280), (1280, 51866)]  # (K, N)
SWEEP_M = [1, 8, 64, 256, 1500, 12000]


def run_sweep(args):
    """the quantized Linear alone over K x N in SWEEP_SHAPES, Q8_0 / Q4_0 /
    Q4_K weights (seeded N(0, 0.02), quantized by the GGUF quantizers), M tokens in SWEEP_M.

    Timing: C copies of the weight (C x bytes > 300 MB, so no launch finds its weight in the
    126 MB L2) are launched back to back through vkb_linear, the C launches recorded once as a
    CUDA graph; the graph is replayed and timed with CUDA events, per launch = time / C. This
    is the steady state a decode step sees (launch latencies overlap through programmatic
    dependent launch). f32 activations for M <= 8, f16 hi+lo planes above (what the producing
    kernels hand the tensor-core GEMM), f32 output. One JSON line per point with the achieved
    HBM GB/s (algorithmic bytes: N*K*b_w + M*K*4 + M*N*4) and tensor TFLOP/s (2*M*N*K)."""
    import ctypes as C
    import torch
    from vokra_b200 import _lib, ops, synth
    ctx = ops.Context(0)
    L = _lib.load()
    hbm, bf16, _, peak_kind = _peaks()
    fmts = {"q8_0": (synth.Q8_0, 34 / 32), "q4_0": (synth.Q4_0, 18 / 32), "q4_k": (synth.Q4_K, 144 / 256)}
    only = set(args.sweep_formats.split(",")) if args.sweep_formats else set(fmts)
    ms_list = [int(x) for x in args.sweep_m.split(",")] if args.sweep_m else SWEEP_M
    for fname, (tag, bw) in fmts.items():
        if fname not in only:
            continue
        shapes = ([tuple(int(v) for v in x.split("x")) for x in args.sweep_shapes.split(",")]
                  if args.sweep_shapes else SWEEP_SHAPES)
        for (K, N) in shapes:
            rng = np.random.default_rng(K * 7 + N)
            wq = synth.quantize(tag, rng.standard_normal(N * K, dtype=np.float32) * np.float32(0.02))
            copies = int(min(200, max(2, np.ceil(300e6 / (N * K * bw)))))
            ws = [ops.Weight(ctx, tag, N, K, wq) for _ in range(copies)]
            for M in ms_list:
                if M <= 8:
                    a = torch.randn((M, K), device="cuda")
                    a_dt = _lib.DT_F32
                else:
                    a = (torch.randn((2 * M, K), device="cuda") * 0.5).half()
                    a_dt = _lib.DT_F16X2
                out = torch.empty((M, N), device="cuda")

                def launch(w):
                    _lib.check(L.vkb_linear(ctx.h, w.h, M, C.c_void_p(a.data_ptr()), a_dt, None,
                                            C.c_void_p(out.data_ptr()), _lib.DT_F32, _lib.EPI_NONE, None,
                                            C.c_float(1.0)))
                for w in ws[:3]:
                    launch(w)  # plans, workspace, attributes
                torch.cuda.synchronize()
                g = torch.cuda.CUDAGraph()
                side = torch.cuda.Stream()
                with torch.cuda.stream(side):
                    ctx.set_stream(side.cuda_stream)
                    with torch.cuda.graph(g, stream=side):
                        for w in ws:
                            launch(w)
                ctx.set_stream(torch.cuda.current_stream().cuda_stream or 1)
                g.replay()
                torch.cuda.synchronize()
                times = []
                for _ in range(3):
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    e0.record()
                    g.replay()
                    e1.record()
                    torch.cuda.synchronize()
                    times.append(e0.elapsed_time(e1) / copies)
                ms = float(np.median(times))
                alg = N * K * bw + M * K * 4 + M * N * 4
                gbs = alg / (ms / 1e3) / 1e9
                tfl = 2.0 * M * N * K / (ms / 1e3) / 1e12
                print(json.dumps({"sweep": "configs[1]", "format": fname, "K": K, "N": N, "M": M,
                                  "us": round(ms * 1e3, 2), "algorithmic_bytes": int(alg), "GB_s": round(gbs, 1),
                                  "hbm_frac": round(gbs / hbm, 4), "TFLOP_s": round(tfl, 2),
                                  "tensor_frac": round(tfl / bf16, 4), "peak_kind": peak_kind,
                                  "launches_per_graph": copies}), flush=True)
                del g
            for w in ws:
                w.close()


def run_base(args):
    """Whisper-base (6+6 layers, d 512, 51865-token vocabulary) in Q8_0,
    one 30 s clip at batch 1: log-mel frontend, encoder, the 4-token prefix and 64
    teacher-forced tokens, every kernel on the device (the decode steps replay CUDA graphs).
    Timed over --steps passes with CUDA events after --warmup passes (the clip's PCM is
    resident; e2e adds its H2D copy and the ids' D2H read). cpu_baseline: the same pass
    through the oracle (the reference CPU algorithm, f32 caches) on the host cores."""
    import torch
    from vokra_b200 import ops, synth, whisper
    arch = synth.WHISPER_BASE
    path = ensure_model(model_path("base_q8_0"), arch, synth.Q8_0)
    ctx = ops.Context(0)
    model = whisper.WhisperModel(ctx, path)
    sess = whisper.Session(model, max_streams=1, max_step_tokens=8, max_clips=1, cross_kv_q8=True)
    NT = 64
    pcm_host = torch.from_numpy(synthetic_pcm(1, 7)).pin_memory()
    pcm_dev = pcm_host.cuda()
    lm = torch.empty((1, arch.n_mels, 3000), device="cuda")
    toks = np.random.default_rng(3).integers(0, arch.n_vocab, NT).astype(np.int32)
    ids_dev = torch.zeros(NT, dtype=torch.int32, device="cuda")
    ids_host = torch.zeros(NT, dtype=torch.int32).pin_memory()
    pre = list(arch.start_ids[:PREFIX])
    stream = torch.cuda.current_stream()

    def one(e2e):
        if e2e:
            pcm_dev.copy_(pcm_host, non_blocking=True)
        ops.log_mel(ctx, pcm_dev, arch.n_mels, out=lm)
        sess.encode(lm, [0])
        sess.step([0] * PREFIX, list(range(PREFIX)), pre)
        for t in range(NT):
            sess.step([0], [PREFIX + t], [int(toks[t])], ids_dev=ids_dev[t:t + 1])
        if e2e:
            ids_host.copy_(ids_dev, non_blocking=True)
        sess.release(0)

    for _ in range(max(3, args.warmup)):
        one(False)
    torch.cuda.synchronize()
    res = {}
    for e2e in (False, True):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            one(e2e)
        e1.record(stream)
        torch.cuda.synchronize()
        res[e2e] = e0.elapsed_time(e1) / args.steps
    cpu = None
    if not args.no_cpu_baseline:
        from oracle import py as o, whisper_ref
        threads = os.cpu_count() or 1
        o.lib().orc_set_threads(threads)
        ref = whisper_ref.RefWhisper(path)
        t0 = time.perf_counter()
        dec = ref.decoder(ref.encode(o.log_mel(pcm_host.numpy()[0], arch.n_mels)), "f32", "f32")
        dec.step(pre)
        for t in range(NT):
            dec.step([int(toks[t])])
        cpu_s = time.perf_counter() - t0
        cpu = {"value": round(CLIP_SECONDS / cpu_s, 3), "unit": "audio-s/s", "cores": threads, "kind": "port",
               "sample": "the whole configs[0] pass (1 clip, 64 tokens) through the oracle, f32 self-KV and cross K/V"}
    print(json.dumps({
        "metric": "audio-s/s, Whisper-base Q8_0 batch 1 (configs[0])", "value": round(CLIP_SECONDS / (res[False] / 1e3), 2),
        "unit": "audio-s/s", "decode_tok_s": None, "ms_per_step": round(res[False], 3), "n_gpus": 1,
        "steps": args.steps, "warmup": max(3, args.warmup), "higher_is_better": True,
        "dtype": "f16 hi+lo tensor-core operands / fp32 GEMV (Q8_0 weights, Q8_0 KV)", "data": "synthetic",
        "config": {"workload": "configs[0]: whisper-base q8_0, 1 clip x 30 s, log-mel + encoder + 4-token prefix + 64 "
                               "teacher-forced tokens, batch 1"},
        "e2e": {"value": round(CLIP_SECONDS / (res[True] / 1e3), 2), "unit": "audio-s/s",
                "h2d_bytes_per_step": int(pcm_host.numel() * 4), "d2h_bytes_per_step": NT * 4},
        "cpu_baseline": cpu}), flush=True)


def throughput_utterances(n: int, rank: int, pool: int):
    """configs[4] workload of one rank: clip lengths U[5, 30] s (padded to 30 s by the
    frontend), decode lengths U[32, 224]; clip i reads row i % pool of the PCM pool."""
    from vokra_b200.batching import Utterance
    rng = np.random.default_rng(50 + rank)
    secs = rng.uniform(5.0, 30.0, n)
    toks = rng.integers(32, 225, n)
    return [Utterance(i % pool, int(secs[i] * 16000), int(toks[i])) for i in range(n)], float(secs.sum())


def run_throughput(args, world, rank, local_rank):
    """continuous batching of up to 128 streams per GPU over the whole
    utterance list of this rank; audio-s/s counts each clip's own length."""
    import torch
    from vokra_b200 import ops, synth, whisper
    from vokra_b200.batching import ContinuousBatcher
    torch.cuda.set_device(local_rank)
    dist = init_process_group(world, local_rank, "nccl")
    arch = synth.WHISPER_LARGE_V3
    path = model_path("large_v3_q4_0")
    if rank == 0:
        ensure_model(path, arch, synth.Q4_0)
    if dist is not None:
        dist.barrier()
    ctx = ops.Context(local_rank)
    from vokra_b200 import _lib
    prec = {"split": _lib.PREC_SPLIT, "f16": _lib.PREC_F16, "enc_f16": _lib.PREC_ENCODER_F16}[args.precision]
    _lib.check(_lib.load().vkb_context_set_precision(ctx.h, prec))
    model = whisper.WhisperModel(ctx, path)
    SLOTS, ENC, POOL = 128, 32, 64
    sess = whisper.Session(model, max_streams=SLOTS, max_step_tokens=4 * SLOTS, max_clips=ENC, cross_kv_q8=True)
    dev = f"cuda:{local_rank}"
    pcm = torch.from_numpy(synthetic_pcm(POOL, rank_input_seed(rank))).to(dev)
    n_rank = max(1, args.utterances // world)
    warm, _ = throughput_utterances(min(n_rank, 2 * SLOTS), rank + 1000, POOL)
    ContinuousBatcher(ctx, sess, SLOTS, ENC, arch.start_ids[:PREFIX], arch.n_mels).run(warm, pcm)
    utts, audio = throughput_utterances(n_rank, rank, POOL)
    batcher = ContinuousBatcher(ctx, sess, SLOTS, ENC, arch.start_ids[:PREFIX], arch.n_mels)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    l0 = ctx.launch_count
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    batcher.run(utts, pcm)
    e1.record()
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1), dist, dev)
    tokens = float(batcher.tokens)
    if dist is not None:
        t = torch.tensor([audio, tokens], dtype=torch.float64, device=dev)
        dist.all_reduce(t)
        audio, tokens = float(t[0]), float(t[1])
    if rank == 0:
        print(json.dumps({
            "metric": METRIC, "value": round(audio / (ms / 1e3), 2), "unit": "audio-s/s",
            "decode_tok_s": round(tokens / (ms / 1e3), 1), "n_gpus": world, "steps": 1, "warmup": 1,
            "ms_per_step": round(ms, 1), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": PREC_DTYPE[args.precision], "data": "synthetic",
            "config": {"workload": f"configs[4]: {n_rank * world} utterances of whisper-large-v3 q4_0 ({n_rank} per "
                                   f"GPU), clip lengths U[5, 30] s padded to 30 s, greedy decode lengths U[32, 224]; "
                                   f"continuous batching of up to {SLOTS} streams per GPU, clips encoded {ENC} at a "
                                   f"time as slots free up; PCM rows drawn from a pool of {POOL} seeded synthetic "
                                   f"clips, each utterance with its own length",
                       "decode_steps": batcher.steps, "parallelism": f"dp{world} (utterances sharded by request)"},
            "gpu_launches": int(ctx.launch_count - l0),
        }), flush=True)
    if dist is not None:
        dist.destroy_process_group()


# ---------------------------------------------------------------------------
# GPU leg
# ---------------------------------------------------------------------------
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="vkb", choices=["vkb", "reference"])
    ap.add_argument("--clips", type=int, default=64)
    ap.add_argument("--tokens", type=int, default=128)
    ap.add_argument("--precision", default="enc_f16", choices=["split", "f16", "enc_f16"],
                    help="split: hi+lo f16 operands everywhere; enc_f16: single-f16 operands in the encoder "
                         "(VKB_PREC_ENCODER_F16), split in the decoder; f16: single f16 everywhere")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--kernel", default=None, choices=["fc1", "fc1_m1500", "xattn", "encoder", "paged_decode", "decode_step"],
                    help="run only one kernel three times, for ncu: the encoder fc1 GEMM (M = clips x 1500, or "
                         "1500), the decode cross-attention over the Q8_0 store (clips streams x 1500 keys), or "
                         "the encoder of a one-layer model with large-v3's dimensions on 8 clips, or the fused decode "
                         "self-attention over configs[2] (prints its own JSON line with the HBM roofline), or one "
                         "64-stream decode step at position 100 between profiler start/stop")
    ap.add_argument("--sweep-formats", default="", help="sweep: comma-separated subset of q8_0,q4_0,q4_k")
    ap.add_argument("--sweep-m", default="", help="sweep: comma-separated M values")
    ap.add_argument("--sweep-shapes", default="", help="sweep: comma-separated KxN shapes, e.g. 1280x51866")
    ap.add_argument("--config", default="batch", choices=["batch", "throughput", "sweep", "base"],
                    help="batch: configs[3] (the default bench line); throughput: configs[4], continuous batching "
                         "of --utterances utterances per job; sweep: configs[1], the quantized Linear alone; base: configs[0] (extra "
                         "measurements, not the driver's line)")
    ap.add_argument("--utterances", type=int, default=2048)
    args = ap.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        run_reference(args, rank)
        return
    if args.kernel:
        run_kernel_only(args)
        return
    if args.config == "throughput":
        run_throughput(args, world, rank, local_rank)
        return
    if args.config == "base":
        run_base(args)
        return
    if args.config == "sweep":
        run_sweep(args)
        return

    import torch
    torch.cuda.set_device(local_rank)
    dist = init_process_group(world, local_rank, "nccl")

    def barrier():
        if dist is not None:
            dist.barrier()

    from vokra_b200 import _lib, ops, synth, whisper
    arch = synth.WHISPER_LARGE_V3
    path = model_path("large_v3_q4_0")
    if rank == 0:
        ensure_model(path, arch, synth.Q4_0)
    barrier()

    ctx = ops.Context(local_rank)
    prec = {"split": _lib.PREC_SPLIT, "f16": _lib.PREC_F16, "enc_f16": _lib.PREC_ENCODER_F16}[args.precision]
    _lib.check(_lib.load().vkb_context_set_precision(ctx.h, prec))
    model = whisper.WhisperModel(ctx, path)
    B, NT = args.clips, args.tokens
    sess = whisper.Session(model, max_streams=B, max_step_tokens=B * PREFIX, max_clips=B, cross_kv_q8=True)
    dev = f"cuda:{local_rank}"
    pcm_host = torch.from_numpy(synthetic_pcm(B, rank_input_seed(rank))).pin_memory()
    pcm_dev = pcm_host.to(dev)
    logmel_dev = torch.empty((B, arch.n_mels, 2 * arch.n_audio_ctx), dtype=torch.float32, device=dev)
    rng = np.random.default_rng(2 + rank)
    toks = rng.integers(0, arch.n_vocab, (NT, B)).astype(np.int32)
    streams = np.arange(B, dtype=np.int32)
    pre_streams = np.repeat(streams, PREFIX)
    pre_pos = np.tile(np.arange(PREFIX, dtype=np.int32), B)
    pre_tok = np.tile(np.array(arch.start_ids[:PREFIX], np.int32), B)
    positions = [np.full(B, PREFIX + t, np.int32) for t in range(NT)]
    ids_dev = torch.zeros((NT, B), dtype=torch.int32, device=dev)
    ids_host = torch.zeros((NT, B), dtype=torch.int32).pin_memory()
    stream = torch.cuda.current_stream()

    dec_events = []  # (start, end) of the decode loop of each timed device-resident step

    def one_step(e2e: bool, mark: bool = False):
        if e2e:
            pcm_dev.copy_(pcm_host, non_blocking=True)
        ops.log_mel(ctx, pcm_dev, arch.n_mels, out=logmel_dev)
        sess.encode(logmel_dev, streams)
        sess.step(pre_streams, pre_pos, pre_tok)
        if mark:
            d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            d0.record(stream)
        for t in range(NT):
            sess.step(streams, positions[t], toks[t], ids_dev=ids_dev[t])
        if mark:
            d1.record(stream)
            dec_events.append((d0, d1))
        if e2e:
            ids_host.copy_(ids_dev, non_blocking=True)
        for s in range(B):
            sess.release(s)

    for _ in range(args.warmup):
        one_step(False)
    torch.cuda.synchronize()

    def timed(e2e: bool):
        barrier()
        torch.cuda.synchronize()
        l0 = ctx.launch_count
        ev0 = torch.cuda.Event(enable_timing=True)
        ev1 = torch.cuda.Event(enable_timing=True)
        ev0.record(stream)
        for _ in range(args.steps):
            one_step(e2e, mark=not e2e)
        ev1.record(stream)
        torch.cuda.synchronize()
        barrier()
        ms = max_over_ranks(ev0.elapsed_time(ev1), dist, dev)
        return ms, ctx.launch_count - l0

    phys = local_rank
    cvd = os.environ.get("CUDA_VISIBLE_DEVICES")
    if cvd:
        try:
            phys = int(cvd.split(",")[local_rank])
        except Exception:
            pass
    with ClockSampler(phys) as clk:
        ms, launches = timed(False)
    ms_e2e, _ = timed(True)

    value, tok_s = job_throughput(world, B, args.steps, NT, ms)
    e2e_value, _ = job_throughput(world, B, args.steps, NT, ms_e2e)

    # Dominant kernel: the encoder MLP fc1 GEMM (Q4_0, M = 64 x 1500 tokens, N = 5120, K = 1280,
    # f16 hi+lo activations in the default precision), timed alone with CUDA events.
    hbm, bf16, bf16_sus, peak_kind = _peaks()
    M, N, K = B * arch.n_audio_ctx, arch.ffn_dim, arch.d_model
    wq = synth.quantize(synth.Q4_0, np.random.default_rng(7).standard_normal(N * K).astype(np.float32) * 0.02)
    w = ops.Weight(ctx, synth.Q4_0, N, K, wq)
    planes = 2 if args.precision == "split" else 1
    a = (torch.randn((planes * M, K), device=dev) * 0.5).half()
    out = torch.empty((M, N), device=dev, dtype=torch.float16)
    a_dt = _lib.DT_F16X2 if planes == 2 else _lib.DT_F16
    L = _lib.load()
    import ctypes as C

    def fc1():
        _lib.check(L.vkb_linear(ctx.h, w.h, M, C.c_void_p(a.data_ptr()), a_dt, None, C.c_void_p(out.data_ptr()),
                                _lib.DT_F16, _lib.EPI_NONE, None, C.c_float(1.0)))
    for _ in range(3):
        fc1()
    reps = 10
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        fc1()
    e1.record(stream)
    torch.cuda.synchronize()
    k_ms = e0.elapsed_time(e1) / reps
    mma_factor = 3 if planes == 2 else 1
    tflops = 2.0 * M * N * K / (k_ms / 1e3) / 1e12
    roofline = {"bound": "tensor", "achieved": round(tflops, 1), "peak": bf16, "unit": "TFLOP/s",
                "frac": round(tflops / bf16, 4), "traffic": None,
                "kernel": ("tc_gemm_persist_kernel (persistent, double-buffered accumulator, weights dequantized "
                           "into tensor memory)" if planes == 2 else
                           "tc_gemm_pair_kernel (persistent, CTA pairs with one cta_group::2 MMA per 256x256 tile, "
                           "both operands by TMA from shared memory; the time includes dequant_plane_kernel, the "
                           "once-per-call f16 weight plane)")
                          + f" Q4_0 encoder fc1 M={M} N={N} K={K}, "
                          f"{'split f16 (3 MMAs per step)' if planes == 2 else 'f16'}",
                "algorithmic_flops": 2 * M * N * K, "mma_flops_issued": 2 * M * N * K * mma_factor,
                "ms_per_launch": round(k_ms, 4), "peak_kind": f"{peak_kind} bf16 dense burst"}
    prof = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(prof):
        try:
            key = "tc_gemm_fc1_bytes_per_launch" if planes == 2 else "tc_gemm_fc1_f16_bytes_per_launch"
            roofline["traffic"] = json.load(open(prof)).get(key)
        except Exception:
            pass

    # The decode loop (128 one-token steps of 64 streams, events inside the timed steps):
    # algorithmic bytes per token step = the decoder's Q4_0 Linear weights incl. the
    # embedding-tied logits head, the Q8_0 cross K/V store of every stream and layer,
    # the Q8_0 self-KV of every key each stream attends to (34/32 bytes per element).
    dec_ms = float(np.mean([a.elapsed_time(b) for a, b in dec_events])) / NT
    d_, f_, Ld, V_, T_ = arch.d_model, arch.ffn_dim, arch.n_text_layer, arch.n_vocab, arch.n_audio_ctx
    w_bytes = (Ld * (4 * d_ * d_ + 2 * d_ * d_ + 2 * d_ * f_) + V_ * d_) * 18 / 32
    cross_bytes = Ld * B * T_ * 2 * d_ * 34 / 32
    self_bytes = np.mean([Ld * B * (PREFIX + t + 1) * 2 * d_ * 34 / 32 for t in range(NT)])
    dec_alg = w_bytes + cross_bytes + self_bytes
    dec_gbs = dec_alg / (dec_ms / 1e3) / 1e9
    roofline_decode = {"bound": "hbm", "achieved": round(dec_gbs, 1), "peak": hbm, "unit": "GB/s",
                       "frac": round(dec_gbs / hbm, 4), "traffic": None,
                       "kernel": "whole decode step (64 streams, 32 layers, CUDA-graph replay), mean over 128 "
                                 "token steps",
                       "ms_per_token_step": round(dec_ms, 4), "algorithmic_bytes_per_step": int(dec_alg),
                       "bytes_split": {"weights": int(w_bytes), "cross_kv": int(cross_bytes),
                                       "self_kv_mean": int(self_bytes)},
                       "peak_kind": f"{peak_kind} HBM copy"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            r = cpu_sample(arch, synth.Q4_0, "q4_0", NT, os.cpu_count() or 1)
            cpu = {"value": r["audio_s_per_s"], "unit": "audio-s/s", "cores": os.cpu_count() or 1, "kind": "port",
                   "sample": r["sample"], "decode_tok_s": r["tok_s"]}
        except Exception as e:  # the baseline is reported, never required
            cpu = {"value": None, "unit": "audio-s/s", "cores": os.cpu_count() or 1, "kind": "port",
                   "sample": f"failed: {e}"}

    if rank == 0:
        h2d = int(pcm_host.numel() * 4 + (PREFIX * B * 3 + NT * B * 3) * 4)
        d2h = int(ids_host.numel() * 4)
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "audio-s/s", "decode_tok_s": round(tok_s, 1),
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms / args.steps, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None,
            "dtype": PREC_DTYPE[args.precision],
            "data": "synthetic",
            "config": {"workload": "configs[3]: whisper-large-v3 q4_0, 64 clips x 30 s per GPU, log-mel frontend + "
                                   "encoder + 4-token "
                                   "prefix + 128 teacher-forced tokens through the paged Q8_0 KV",
                       "global_batch": world * B, "seq_len": arch.n_audio_ctx, "decode_tokens": NT,
                       "parallelism": f"dp{world} (utterances sharded by request)",
                       "l2": "inputs larger than L2 (96000x1280 activations per layer)",
                       "inputs": "seeded synthetic 30 s PCM per clip (noise + tones); every step runs the "
                                 "log-mel frontend (vkb_log_mel), the encoder and the decoder"},
            "e2e": {"value": round(e2e_value, 2), "unit": "audio-s/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "gpu_launches": int(launches),
            "roofline": roofline,
            "roofline_decode": roofline_decode,
            "cpu_baseline": cpu,
            "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
