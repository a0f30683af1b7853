"""Profiling driver: runs the batch-1 decode GEMV (or a few greedy frames) of the
Qwen3-4B-shaped model with fewer layers, so an `ncu --set full` capture stays small
(the weights still exceed L2, so DRAM counters are meaningful).

  python -m syrinx_b200.profile --what gemv --kind 2 --layers 8 --launches 16
  python -m syrinx_b200.profile --what frames --layers 8 --frames 4 --prompt 512
  python -m syrinx_b200.profile --what stack --layers 36 --prompt 512   (phase timing, printed)
  python -m syrinx_b200.profile --what prefill --layers 36 --prompt 512  (prefill time, printed)
  python -m syrinx_b200.profile --what batch --layers 8 --q4k --frames 4   (8 utterances batched)
  python -m syrinx_b200.profile --what codec --frames 32 --launches 2   (s2 codec decodes, timed)
  python -m syrinx_b200.profile --what sample --layers 8 --frames 4 --prompt 512  (sampled frames)
"""
from __future__ import annotations

import argparse
import time

from . import QWEN3_4B, B200DualAr, Model, shrink, synth_blob
from .configs import SX_DTYPE_Q4_K, SX_DTYPE_Q8_0
from .workloads import dual_ar_prompt


def codec_run(frames: int, n: int):
    """`n` decodes of `frames` frames through the s2-shaped codec, each timed on the host
    after a synchronisation (the first one includes nothing but the decode)."""
    import numpy as np

    from .codec import S2_CODEC, RvqCodec, synth_codec_weights, synth_codes

    codec = RvqCodec(synth_codec_weights(S2_CODEC, seed=2))
    codes = synth_codes(S2_CODEC, frames, seed=2)
    codec.reserve(frames)
    for i in range(n):
        t0 = time.perf_counter()
        wav = codec.decode(codes)
        print(f"decode {i}: {frames} frames in {1e3 * (time.perf_counter() - t0):.2f} ms")
    assert np.isfinite(wav).all()
    codec.close()
    print("profile run ok")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--what", choices=["gemv", "frames", "stack", "prefill", "batch", "codec", "sample"], default="gemv")
    ap.add_argument("--kind", type=int, default=2,
                    help="0 wqkv, 1 wo, 2 w1|w3 + SwiGLU merge, 3 w2, 4 w1|w3 alone (as the one-token chain runs it)")
    ap.add_argument("--layers", type=int, default=8)
    ap.add_argument("--launches", type=int, default=16)
    ap.add_argument("--frames", type=int, default=4)
    ap.add_argument("--q4k", action="store_true")
    ap.add_argument("--prompt", type=int, default=8, help="prompt positions prefilled before the run")
    args = ap.parse_args()
    if args.what == "codec":
        codec_run(args.frames, args.launches)
        return
    cfg = shrink(QWEN3_4B, args.layers, min(4, args.layers))
    wtype = SX_DTYPE_Q4_K if args.q4k else SX_DTYPE_Q8_0
    model = Model(cfg, synth_blob(cfg, wtype, seed=2))
    if args.what == "batch":  # 8 utterances of args.prompt .. args.prompt + 7 tokens, decoded batched
        be = B200DualAr(model, max_ctx=args.prompt + 16 + args.frames, max_batch=8)
        be.prefill_batch([dual_ar_prompt(cfg, args.prompt + i, (args.prompt + i) * 3 // 4, seed=20 + i)
                          for i in range(8)])
        be.decode_greedy_batch(8, args.frames, mask_stop=True)
        be.close()
        model.close()
        print("profile run ok")
        return
    be = B200DualAr(model, max_ctx=args.prompt + 64 + args.frames)
    prompt = dual_ar_prompt(cfg, args.prompt, max(1, args.prompt * 3 // 4), seed=2)
    t0 = time.perf_counter()
    be.prefill(prompt)
    t_prefill = time.perf_counter() - t0
    if args.what == "prefill":
        for _ in range(2):
            be.reset()
            t0 = time.perf_counter()
            be.prefill(prompt)
            t_prefill = min(t_prefill, time.perf_counter() - t0)
        print(f"prefill of {args.prompt} tokens, {args.layers} layers: {t_prefill * 1e3:.2f} ms")
    elif args.what == "stack":
        for fast in (False, True):
            be.profile_stack(fast)  # warm
            r = be.profile_stack(fast)
            print(("fast" if fast else "slow") + f" stack: total {r['total']:.1f} us, setup {r['setup']:.2f}, "
                  f"final {r['final']:.2f}")
            for k in ("wqkv", "attention", "wo", "w13", "w2", "attention_cta0"):
                print(f"  {k}: " + ", ".join(f"{n} {v:.2f}" for n, v in r[k].items()))
        be.decode_greedy(args.frames, mask_stop=True)
    elif args.what == "gemv":
        be.profile_gemv(args.kind, args.launches)  # close() below synchronizes the stream
    elif args.what == "sample":  # the reference's default sampling (temperature, top-p, RAS)
        from . import SamplingParams
        be.decode_sample(args.frames, seed=7, sampling=SamplingParams())
    else:
        be.decode_greedy(args.frames, mask_stop=True)
    be.close()
    model.close()
    print("profile run ok")


if __name__ == "__main__":
    main()
