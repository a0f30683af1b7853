"""Benchmark of the quantized dual-AR decode step on B200.

Workload: Qwen3-4B-shaped slow AR (36 layers, d 2560, 32/8 heads,
hd 128, QK-norm, SwiGLU 9728, vocab 151936+4096) + fast AR (4 layers, 10 codebooks x
4096), Q8_0 weights from seeded N(0, 0.02)-like values (synthetic, no checkpoint), batch 1,
512-token prompt (82 text ids + 430 reference-voice positions), greedy frames with the stop
id masked so every step produces a frame. One step = one frame: semantic head + argmax,
10 fast-AR steps, MCF embed, 36-layer slow step. Weights (4.8 GB) exceed L2 (126 MB), so
every step streams them from HBM; no L2 flush is needed.

  python bench.py [--gpus N --steps K --warmup W] [--impl reference]
  torchrun --nproc-per-node N bench.py --tp N --steps 1024   (config 5, tensor parallel)

Multi-GPU: one process per GPU (torchrun); utterances are independent, each rank decodes
its own (weak scaling, no collective on the data path); timing is the max over ranks.
The reference arm (--impl reference) times the CPU restatement of the reference path
(oracle/, the Rust/Candle reference cannot be built here) on the host cores.
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

PROMPT_T = 512
PROMPT_SEMANTIC = 430
SEED = 2
METRIC = "semantic frames/s/GPU, 4B-shape Q8_0 dual-AR decode b1/b8; % of HBM roofline"
# DRAM bytes (read + write) of one launch of the dominant kernel, the batch-1 w1|w3 GEMV
# (k_gemv_q8<1>), from one `ncu --set full` capture (python -m syrinx_b200.profile --what
# gemv --kind 2 --layers 8 --launches 16): 52.97 MB read + 0.11 MB written against 52.92 MB
# algorithmic.
W13_DRAM_BYTES = 53085184


def peak_bf16():
    """(bf16 dense TFLOP/s burst, "measured" | "fallback")."""
    try:
        with open(os.path.join(os.path.dirname(os.path.abspath(__file__)), "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops"]), "measured"
    except (OSError, KeyError, ValueError):
        return 1590.0, "fallback"


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class Clocks:
    """nvidia-smi clock / throttle sampling during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        self.lines = []
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                out = ""
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in getattr(self, "lines", []):
            f = [x.strip() for x in l.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def kernels_per_frame(cfg, stack: bool = True) -> int:
    """Kernel launches in one greedy frame graph (mirrors the sequence in model.cu). A Q8_0
    GEMV is two launches: k_gemv_q8 and its k_merge_q8, except the decode wqkv GEMV, whose
    partials the attention kernel adds (one launch, unless SYRINX_QKV_MERGE=1), and the
    one-token w1|w3 GEMV, whose partials the w2 GEMV adds (unless SYRINX_GLU_MERGE=1). With the
    persistent decode kernel a whole stack (36 slow layers, or the 4 fast layers of one
    codebook step) is one launch."""
    gemv = 2
    qkv = 2 if os.environ.get("SYRINX_QKV_MERGE", "0") == "1" else 1
    w13 = 2 if os.environ.get("SYRINX_GLU_MERGE", "0") == "1" else 1
    per_layer = qkv + w13 + 2 * gemv + 1  # wqkv, w1|w3, wo, w2 + attention
    n = gemv + 1  # semantic head, take_semantic
    if cfg.has_fast:
        C = cfg.num_codebooks
        n += C * (1 if stack else cfg.fast.n_layer * per_layer)  # fast steps 0..C-1
        n += 1  # code-0 embedding (take_code)
        n += (C - 1) * (gemv + 1)  # fast head + take_code
    n += 1 + (1 if stack else cfg.slow.n_layer * per_layer) + 1  # embed, slow stack, advance
    return n


def bench_device(args):
    import torch
    import syrinx_b200 as sx
    from syrinx_b200 import dp
    from syrinx_b200.configs import SX_DTYPE_Q8_0, frame_bytes
    from syrinx_b200.workloads import dual_ar_prompt

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600))
    cfg = sx.QWEN3_4B
    t0 = time.time()
    blob = sx.synth_blob(cfg, SX_DTYPE_Q8_0, seed=SEED)
    model = sx.Model(cfg, blob, device=local)
    t_load = time.time() - t0
    K, W = args.steps, args.warmup
    max_ctx = PROMPT_T + 2 * (K + W) + 16
    be = sx.B200DualAr(model, max_ctx=max_ctx)
    stream = torch.cuda.Stream()
    be.set_stream(stream.cuda_stream)
    # each rank decodes its own utterance (independent prompts: seed + rank)
    prompt = dual_ar_prompt(cfg, PROMPT_T, PROMPT_SEMANTIC, seed=dp.rank_seed(SEED, rank))
    t_pf = time.time()
    be.prefill(prompt)
    t_prefill = time.time() - t_pf

    def barrier():
        if dist:
            dist.barrier()

    # ---- value: device-resident greedy loop (one CUDA graph per frame) ----
    be.decode_greedy(W, mask_stop=True)  # warm-up (captures the frame graph)
    ctx_start = be.seq_len()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    with Clocks(local) as clk:
        with torch.cuda.stream(stream):
            start.record(stream)
            frames = be.decode_greedy(K, mask_stop=True)
            end.record(stream)
        torch.cuda.synchronize()
    barrier()
    ms = start.elapsed_time(end)
    assert frames.shape[0] == K, frames.shape
    ms_all = dp.max_over_ranks(ms, dist, device="cuda")
    mean_ctx = ctx_start + (K - 1) / 2.0
    fb_sem = frame_bytes(cfg, SX_DTYPE_Q8_0, ctx=mean_ctx, semantic_head=True, kv_elem=4)
    # the algorithmic bytes as defined for the path count the KV cache at bf16
    fb_bf16 = frame_bytes(cfg, SX_DTYPE_Q8_0, ctx=mean_ctx, semantic_head=True, kv_elem=2)

    # ---- roofline of the dominant kernel: the batch-1 Q8_0 GEMV, timed alone live ----
    peak, peak_kind = peaks()
    n_prof = 4 * cfg.slow.n_layer
    d, F = cfg.slow.dim, cfg.slow.intermediate_size
    # kinds: 0 wqkv, 1 wo, 2 w1|w3 + its SwiGLU merge, 3 w2, 4 w1|w3 alone as the one-token
    # chain runs it (its SwiGLU is formed by the w2 GEMV)
    kinds = {0: cfg.slow.qkv_rows * d, 1: d * cfg.slow.n_head * cfg.slow.head_dim, 2: 2 * F * d, 3: d * F}
    if os.environ.get("SYRINX_GLU_MERGE", "0") != "1":
        kinds[4] = 2 * F * d
    gemv = {}
    for kind, nw in kinds.items():
        be.profile_gemv(kind, cfg.slow.n_layer)  # warm
        s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        s2.record(stream)
        be.profile_gemv(kind, n_prof)
        e2.record(stream)
        torch.cuda.synchronize()
        per = s2.elapsed_time(e2) / n_prof
        gemv[kind] = (nw * 34 / 32, per)
    # the largest per-layer matrix (w1|w3, 52.9 MB) is the dominant kernel of the step
    dom = 4 if 4 in gemv else 2
    bytes_w13, ms_w13 = gemv[dom]
    achieved = bytes_w13 / (ms_w13 * 1e-3) / 1e9
    dom_name = ("k_gemv_q8<1>: Q8_0 w1|w3 at M=1, partials only, as the one-token chain runs it (its SwiGLU "
                "merge is formed by the w2 GEMV)" if dom == 4 else
                "k_gemv_q8<1> + k_merge_q8<1,SwiGLU>: Q8_0 w1|w3 at M=1 (timed as the pair)")

    # ---- e2e: the per-frame public call with host buffers (H2D frame in, D2H frame out) ----
    pin_in = torch.empty(cfg.frame_width, dtype=torch.int32, pin_memory=True).numpy().view(np.uint32)
    pin_out = torch.empty(cfg.frame_width, dtype=torch.int32, pin_memory=True).numpy().view(np.uint32)
    pin_in[:] = frames[-1]
    for _ in range(3):
        be.frame_step_greedy(pin_in, mask_stop=True)
    K_e2e = max(8, min(K, 64))
    s3, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    s3.record(stream)
    for _ in range(K_e2e):
        out, _ = be.frame_step_greedy(pin_in, mask_stop=True)
        pin_out[:] = out
        pin_in[:] = pin_out
    e3.record(stream)
    torch.cuda.synchronize()
    ms_e2e = dp.max_over_ranks(s3.elapsed_time(e3), dist, device="cuda")

    # ---- the device-sampled loop (reference Sampler defaults, seed per rank), same session ----
    K_s = max(0, min(64, be.max_ctx - be.seq_len() - 1))
    sampled = None
    if K_s > 0:
        s4, e4 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        s4.record(stream)
        got = be.decode_sample(K_s, seed=dp.rank_seed(SEED, rank), sampling=sx.SamplingParams())
        e4.record(stream)
        torch.cuda.synchronize()
        ms_s = s4.elapsed_time(e4)
        if got.shape[0] > 0:
            sampled = {"value": round(got.shape[0] / (ms_s * 1e-3), 2), "unit": "frames/s", "frames": int(got.shape[0]),
                       "api": "sx_decode_sample (device sampler: top-p 0.9, top-k 30, RAS; timed with CUDA events)"}

    frames_total = K * world
    value = frames_total / (ms_all * 1e-3)
    res = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "frames/s",
        "n_gpus": world,
        "steps": K,
        "warmup": W,
        "ms_per_step": round(ms_all / K, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "q8_0 weights, f32 activations/accumulation, f32 KV",
        "data": "synthetic (seeded N(0,0.02)-like weights quantized to Q8_0; random prompt ids)",
        "config": {"workload": "config3 qwen3-4b-shaped dual-AR Q8_0 b1: prompt 512 (430 semantic), "
                               "greedy frames, stop masked", "global_batch": world, "seq_len": PROMPT_T,
                   "ctx_mean": mean_ctx, "parallelism": f"dp{world} (independent utterances, no collective)",
                   "l2": "inputs larger than L2 (4.8 GB of weights; 8.4 GB streamed per frame)"},
        "hbm_roofline": {"bytes_per_frame": fb_sem["total"], "frac_of_peak": round(
            fb_sem["total"] * value / world / (peak * 1e9), 4), "peak_gbs": peak, "peak_kind": peak_kind,
            "bytes_per_frame_kv_bf16": fb_bf16["total"],
            "frac_of_peak_kv_bf16": round(fb_bf16["total"] * value / world / (peak * 1e9), 4),
            "note": "semantic-only head (4097 rows) counted, as streamed; the session's KV cache is f32 "
                    "(bytes_per_frame), the kv_bf16 figures count the same KV at bf16"},
        "roofline": {"bound": "hbm", "kernel": dom_name,
                     "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": W13_DRAM_BYTES,
                     "traffic_unit": "bytes per launch (ncu dram__bytes_read.sum + dram__bytes_write.sum)",
                     "algorithmic_bytes": int(bytes_w13),
                     "per_kind_ms": {k: round(v[1], 5) for k, v in gemv.items()},
                     "pair_with_merge_frac": round(gemv[2][0] / (gemv[2][1] * 1e-3) / 1e9 / peak, 4),
                     "peak_source": peak_kind + " (MEASURED_PEAKS.json hbm_gbs)"},
        "e2e": {"value": round(K_e2e * world / (ms_e2e * 1e-3), 2), "unit": "frames/s",
                "h2d_bytes_per_step": int(cfg.frame_width * 4), "d2h_bytes_per_step": int(cfg.frame_width * 4),
                "api": "sx_frame_step_greedy (host frame in, host frame out, per frame)"},
        "gpu_launches": kernels_per_frame(cfg, os.environ.get("SYRINX_STACK", "0") == "1") * K,
        "clocks": clk.summary(),
        "load_s": round(t_load, 1),
        "prefill_s": round(t_prefill, 3),
        "sampled": sampled,
    }
    be.close()
    model.close()
    if not args.no_b8:
        res["b8"] = bench_b8(args, local, stream, dist, world, peak, peak_kind)
    if not args.no_codec:
        res["codec"] = bench_codec(args, local, stream, dist, world, rank)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:  # the host-core baseline is an N=1 figure
        res["cpu_baseline"] = cpu_baseline(cfg, budget_s=args.cpu_budget)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(res), flush=True)


def bench_b8(args, local, stream, dist, world, peak, peak_kind):
    """Config 4 on each GPU: the Qwen3-4B-shaped dual-AR in Q4_K, 8 utterances (prompts 256-1024
    tokens, seeded) prefilled into one paged cache and decoded as one greedy batch of 8 (every
    batched step streams the weights once for all 8 frames). frames/s counts every
    utterance's frames; the roofline counts the weights once per step plus each utterance's
    KV read (f32 cache, and at bf16 as the path defines it)."""
    import torch
    import syrinx_b200 as sx
    from syrinx_b200 import dp
    from syrinx_b200.configs import SX_DTYPE_Q4_K, frame_bytes
    from syrinx_b200.workloads import config4_prompts

    cfg = sx.QWEN3_4B
    K, W = min(args.steps, 64), max(3, min(args.warmup, 8))
    model = sx.Model(cfg, sx.synth_blob(cfg, SX_DTYPE_Q4_K, seed=SEED), device=local)
    prompts = config4_prompts(cfg, 8)
    lens = [p.shape[1] for p in prompts]
    be = sx.B200DualAr(model, max_ctx=max(lens) + K + W + 8, max_batch=8)
    be.set_stream(stream.cuda_stream)
    t0 = time.time()
    be.prefill_batch(prompts)
    t_prefill = time.time() - t0
    be.decode_greedy_batch(8, W, mask_stop=True)
    s1, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        s1.record(stream)
        got = be.decode_greedy_batch(8, K, mask_stop=True)
        e1.record(stream)
    torch.cuda.synchronize()
    ms = dp.max_over_ranks(s1.elapsed_time(e1), dist, device="cuda")
    assert len(got) == 8 and all(g.shape[0] == K for g in got), [g.shape for g in got]
    ctx_mean = [T + W + (K - 1) / 2.0 for T in lens]
    w_bytes = frame_bytes(cfg, SX_DTYPE_Q4_K, ctx=0, semantic_head=True)["total"]
    kv_f32 = sum(frame_bytes(cfg, SX_DTYPE_Q4_K, ctx=c, kv_elem=4)["kv"] for c in ctx_mean)
    kv_bf16 = sum(frame_bytes(cfg, SX_DTYPE_Q4_K, ctx=c, kv_elem=2)["kv"] for c in ctx_mean)
    steps_per_s = K / (ms * 1e-3)
    be.close()
    model.close()
    return {"value": round(8 * K * world / (ms * 1e-3), 2), "unit": "frames/s", "per_gpu_batch": 8,
            "ms_per_batched_step": round(ms / K, 4), "steps": K, "warmup": W,
            "workload": "config4 qwen3-4b-shaped dual-AR Q4_K, 8 utterances per GPU batched (prompts " +
                        "/".join(str(t) for t in lens) + "), greedy, stop masked",
            "prefill_batch_s": round(t_prefill, 3),
            "hbm_roofline": {"bytes_per_step": w_bytes + kv_f32, "frac_of_peak": round(
                (w_bytes + kv_f32) * steps_per_s / (peak * 1e9), 4), "bytes_per_step_kv_bf16": w_bytes + kv_bf16,
                "frac_of_peak_kv_bf16": round((w_bytes + kv_bf16) * steps_per_s / (peak * 1e9), 4),
                "peak_gbs": peak, "peak_kind": peak_kind}}


CODEC_FRAMES = 256  # 11.9 s of 44.1 kHz audio per decode


def bench_codec(args, local, stream, dist, world, rank):
    """Row f2 on each GPU: the s2 causal-DAC codec decode (codes [10, 256] -> 524,288
    samples) with seeded synthetic weights of the s2 shape. Device time over K decodes with
    inputs resident; e2e through sx_codec_decode (host codes in, host waveform out). The
    weights (0.74 GB) and activations exceed L2, so no flush is needed between decodes."""
    import torch
    from syrinx_b200 import dp
    from syrinx_b200.codec import S2_CODEC, RvqCodec, decode_flops, decode_launches, synth_codec_weights, synth_codes

    T = CODEC_FRAMES
    K, W = min(args.steps, 8), 3
    weights = synth_codec_weights(S2_CODEC, seed=SEED)
    codec = RvqCodec(weights, device=local)
    codec.reserve(T)
    codes = synth_codes(S2_CODEC, T, seed=SEED)
    dcodes = torch.from_numpy(codes.astype(np.int32)).cuda()
    wav = torch.empty(T * codec.hop, dtype=torch.float32, device="cuda")
    codec.set_stream(stream.cuda_stream)
    for _ in range(W):
        codec.decode_device(dcodes.data_ptr(), codes.shape[0], T, wav.data_ptr())
    s1, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    s1.record(stream)
    for _ in range(K):
        codec.decode_device(dcodes.data_ptr(), codes.shape[0], T, wav.data_ptr())
    e1.record(stream)
    torch.cuda.synchronize()
    ms = dp.max_over_ranks(s1.elapsed_time(e1), dist, device="cuda") / K
    host_wav = codec.decode(codes)  # e2e warm-up
    t0 = time.perf_counter()
    for _ in range(K):
        host_wav = codec.decode(codes)
    ms_e2e = dp.max_over_ranks((time.perf_counter() - t0) * 1e3, dist, device="cuda") / K
    assert host_wav.shape == (T * codec.hop,) and np.isfinite(host_wav).all()
    assert np.array_equal(host_wav, wav.cpu().numpy())
    flops = decode_flops(S2_CODEC, T)
    tflops = flops / (ms * 1e-3) / 1e12
    if os.environ.get("SYRINX_CODEC_TC", "1") == "0":
        bound, cpeak = "fp32", 148 * 128 * 2 * 1.965e9 / 1e12
        psrc = ("nominal FP32 CUDA-core rate at clocks.max.sm (148 SMs x 128 lanes x 2 x 1965 MHz); "
                "not in MEASURED_PEAKS.json")
    else:
        bf16, kind = peak_bf16()
        bound, cpeak = "tensor", bf16 / 2 / 3
        psrc = (f"{kind} bf16 dense {bf16} TFLOP/s (MEASURED_PEAKS.json) / 2 (kind::tf32 runs at half the "
                "bf16 rate) / 3 (three tf32 products per f32 product): the useful-f32 ceiling of the split")
    out = {"value": round(T * world / (ms * 1e-3), 1), "unit": "codec frames/s",
           "audio_s_per_s": round(T * codec.hop / 44100 * world / (ms * 1e-3), 1),
           "ms_per_decode": round(ms, 3), "steps": K, "warmup": W,
           "gpu_launches": decode_launches(S2_CODEC) * K,
           "workload": f"s2 codec decode, {T} frames x 10 codebooks -> {T * codec.hop} samples, "
                       "synthetic weights of the s2 shape (seed %d)" % SEED,
           "dtype": "f32 (products: tf32 three-term split on tcgen05, f32 sums)" if bound == "tensor" else "f32",
           "roofline": {"bound": bound, "achieved": round(tflops, 2), "unit": "TFLOP/s",
                        "flops_per_decode": flops, "peak": round(cpeak, 1),
                        "frac": round(tflops / cpeak, 4), "peak_source": psrc},
           "e2e": {"value": round(T * world / (ms_e2e * 1e-3), 1), "unit": "codec frames/s",
                   "h2d_bytes_per_step": int(codes.size * 4), "d2h_bytes_per_step": int(T * codec.hop * 4),
                   "api": "sx_codec_decode (host codes in, host waveform out)"}}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import codec_oracle
        n = 8
        t0 = time.perf_counter()
        codec_oracle.decode(weights, codes[:, :n])
        secs = time.perf_counter() - t0
        out["cpu_baseline"] = {"value": round(n / secs, 3), "unit": "codec frames/s",
                               "cores": os.cpu_count(), "kind": "port",
                               "sample": f"the first {n} frames of the same codes on the float64 numpy "
                                         f"oracle ({secs:.1f} s)"}
    codec.close()
    return out


TP_METRIC = "semantic frames/s per tensor-parallel group, config 5 (4B-shape Q8_0 dual-AR b1, KV grown to 8192)"


def bench_tp(args):
    """--tp N (config 5): one utterance decoded by a tensor-parallel group of N GPUs (one
    process per GPU under torchrun). The cache is brought to args.tp_ctx - steps - warmup
    positions: all but the last 64 hold seeded synthetic K/V (sx_session_fill_kv_synthetic;
    a 7K-token prefill at 8 tokens per GEMV launch would stream every weight ~900 times),
    the last 64 are a real prompt prefilled on top of them. Then `warmup` untimed and
    `steps` timed greedy frames attend over the whole cache (which ends near args.tp_ctx).
    value = frames/s of the group (strong scaling: the work per frame is fixed); the timing
    is the max over ranks of the CUDA-event time of the timed frames."""
    import datetime

    import torch
    import torch.distributed as dist
    import syrinx_b200 as sx
    from syrinx_b200 import dp, tp
    from syrinx_b200.configs import SX_DTYPE_Q8_0, frame_bytes
    from syrinx_b200.workloads import dual_ar_prompt

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.tp:
        raise SystemExit(f"--tp {args.tp} needs {args.tp} processes (torchrun --nproc-per-node {args.tp})")
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600))
    cfg = sx.QWEN3_4B
    K, W = args.steps, args.warmup
    T = args.tp_ctx - K - W
    blob = sx.synth_blob(cfg, SX_DTYPE_Q8_0, seed=3)
    model = sx.Model(cfg, blob, device=local, tp_rank=rank, tp_size=world)
    from syrinx_b200.configs import SX_DTYPE_BF16, SX_DTYPE_F32
    kv_bf16 = args.tp_kv == "bf16"
    be = sx.B200DualAr(model, max_ctx=args.tp_ctx + 16, kv_dtype=SX_DTYPE_BF16 if kv_bf16 else SX_DTYPE_F32)
    stream = torch.cuda.Stream()
    be.set_stream(stream.cuda_stream)
    if world > 1:
        tp.connect(be, dist)
    tail = 64
    prompt = dual_ar_prompt(cfg, tail, 54, seed=3)
    t0 = time.time()
    be.fill_kv_synthetic(T - tail, seed=3)
    be.prefill(prompt)
    t_prefill = time.time() - t0
    be.decode_greedy(W, mask_stop=True)
    ctx_start = be.seq_len()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with Clocks(local) as clk:
        with torch.cuda.stream(stream):
            start.record(stream)
            frames = be.decode_greedy(K, mask_stop=True)
            end.record(stream)
        torch.cuda.synchronize()
    ms = dp.max_over_ranks(start.elapsed_time(end), dist if world > 1 else None, device="cuda")
    assert frames.shape[0] == K, frames.shape
    peak, peak_kind = peaks()
    mean_ctx = ctx_start + (K - 1) / 2.0
    fb = frame_bytes(cfg, SX_DTYPE_Q8_0, ctx=mean_ctx, semantic_head=True, kv_elem=2 if kv_bf16 else 4)
    # per GPU: layers and KV split over the ranks; the heads are replicated
    fast_out = (cfg.num_codebooks - 1) * cfg.codebook_size * cfg.fast.dim * 34 / 32
    per_gpu = (fb["slow"] + fb["fast"] - fast_out + fb["kv"]) / world + fb["head"] + fast_out
    value = K / (ms * 1e-3)
    res = {
        "metric": TP_METRIC, "value": round(value, 2), "unit": "frames/s", "n_gpus": world, "steps": K,
        "warmup": W, "ms_per_step": round(ms / K, 4), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None,
        "dtype": "q8_0 weights, f32 activations/accumulation, " + ("bf16 KV (paged)" if kv_bf16 else "f32 KV"),
        "data": "synthetic (seed 3)",
        "config": {"workload": f"config5 qwen3-4b-shaped dual-AR Q8_0 b1, tp{world}: {T - tail} synthetic KV "
                               f"positions + {tail}-token prompt, {W}+{K} greedy frames, KV to {args.tp_ctx}",
                   "ctx_mean": mean_ctx, "parallelism": f"tp{world}",
                   "exchange": "residual rows after wo and w2 over NVLink in the merge kernel (no NCCL call)"},
        "hbm_roofline": {"bytes_per_frame_per_gpu": per_gpu, "frac_of_peak": round(per_gpu * value / (peak * 1e9), 4),
                         "peak_gbs": peak, "peak_kind": peak_kind,
                         "note": "layers and KV divided over the ranks; semantic head and fast_output replicated"},
        "gpu_launches": kernels_per_frame(cfg, world == 1 and os.environ.get("SYRINX_STACK", "0") == "1") * K,
        "clocks": clk.summary(), "prefill_s": round(t_prefill, 2),
    }
    if world > 1:
        tp.close(be, model, dist)
        dist.destroy_process_group()
    else:
        be.close()
        model.close()
    if rank == 0:
        print(json.dumps(res), flush=True)


def cpu_decoder(cfg, seed: int):
    """The oracle (CPU restatement of the reference path) on all host cores, prefilled with
    the GPU arm's 512-token prompt (untimed). Its weights come from the oracle library's copy
    of the seeded writer, so this arm never loads the product library."""
    from oracle import oracle as oc
    from syrinx_b200.configs import SX_DTYPE_Q8_0
    from syrinx_b200.workloads import dual_ar_prompt

    # all host cores, whatever OMP_NUM_THREADS a launcher (torchrun sets 1) left behind
    oc.set_num_threads(len(os.sched_getaffinity(0)))
    blob = oc.synth_blob(cfg, SX_DTYPE_Q8_0, seed)
    om = oc.OracleModel(cfg, blob)
    sess = oc.OracleSession(om, max_ctx=PROMPT_T + 1024, kv_bf16=False)
    prompt = dual_ar_prompt(cfg, PROMPT_T, PROMPT_SEMANTIC, seed=seed)
    t0 = time.perf_counter()
    logits, hidden = sess.prefill(prompt)
    state = {"om": om, "sess": sess, "logits": logits, "hidden": hidden, "blob": blob,
             "prefill_s": time.perf_counter() - t0, "cores": oc.num_threads()}

    def frame():
        tok, _ = om.greedy_semantic(state["logits"], mask_stop=True)
        codes, _ = sess.fast_expand_greedy(state["hidden"], om.first_code(tok))
        state["logits"], state["hidden"] = sess.slow_step(np.concatenate([[tok], codes]).astype(np.uint32))

    return frame, state


def cpu_baseline(cfg, budget_s: float) -> dict:
    """A bounded sample of the bench workload on the CPU oracle: greedy frames after the same
    512-token prompt, timed until the budget is spent (prefill excluded)."""
    frame, st = cpu_decoder(cfg, SEED)
    n, t_total = 0, 0.0
    while t_total < budget_s and n < 1000:
        t0 = time.perf_counter()
        frame()
        t_total += time.perf_counter() - t0
        n += 1
    return {"value": round(n / t_total, 4), "unit": "frames/s", "cores": st["cores"], "kind": "port",
            "sample": f"config3 Q8_0 weights, the same 512-token prompt (prefill {st['prefill_s']:.1f} s, "
                      f"excluded), {n} greedy frames decoded on the CPU oracle ({t_total:.1f} s)"}


def bench_reference(args):
    """--impl reference: the reference path on the host cores (the CPU restatement: the
    Rust/Candle reference cannot be built here). Same workload as the GPU arm: config 3 after
    the 512-token prompt (prefill untimed), `warmup` untimed frames, then `steps` timed frames."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from syrinx_b200.configs import QWEN3_4B

    cfg = QWEN3_4B
    frame, st = cpu_decoder(cfg, SEED)
    for _ in range(args.warmup):
        frame()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        frame()
    secs = time.perf_counter() - t0
    value = args.steps / secs
    sample = (f"config3 Q8_0 weights, the GPU arm's 512-token prompt (prefill {st['prefill_s']:.1f} s, untimed), "
              f"{args.warmup} warm-up + {args.steps} timed greedy frames on the CPU oracle ({secs:.1f} s)")
    res = {
        "metric": METRIC, "value": round(value, 4), "unit": "frames/s", "n_gpus": 0, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(1000.0 * secs / args.steps, 2),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "impl": "reference",
        "dtype": "q8_0 weights, f32 activations, f32 KV", "data": "synthetic (same seeded weights and prompt)",
        "config": {"workload": "config3 qwen3-4b-shaped dual-AR Q8_0 b1: prompt 512 (430 semantic), "
                               "greedy frames, stop masked", "global_batch": 1, "seq_len": PROMPT_T,
                   "same_config": True},
        "cpu_baseline": {"value": round(value, 4), "unit": "frames/s", "cores": st["cores"], "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(value, 4), "unit": "frames/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "Rust/Candle reference cannot be built here (no cargo/rustc, candle not vendored); "
                "timed arm is the oracle/ CPU restatement of the same path",
    }
    print(json.dumps(res), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-b8", action="store_true", help="skip the config-4 batch-8 Q4_K measurement")
    ap.add_argument("--no-codec", action="store_true", help="skip the codec decode measurement")
    ap.add_argument("--cpu-budget", type=float, default=15.0)
    ap.add_argument("--tp", type=int, default=0, help="config 5: tensor-parallel group of N GPUs")
    ap.add_argument("--tp-ctx", type=int, default=8192)
    ap.add_argument("--tp-kv", default="f32", choices=["f32", "bf16"],
                    help="config 5 KV cache element: f32 (default: measured faster, 183 vs 134 frames/s "
                         "at TP1) or the workload's paged bf16")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.tp:
        bench_tp(args)
    elif args.impl == "reference":
        bench_reference(args)
    else:
        bench_device(args)


if __name__ == "__main__":
    main()
