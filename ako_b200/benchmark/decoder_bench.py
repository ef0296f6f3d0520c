"""Decoder throughput: prefill and decode tokens per second.

4-layer LLaMA-style stack (d 4096, 32 heads / 8 KV heads, head_dim 128, FFN
11008, eps 1e-5, theta 1e4, vocab 32000), bf16, random N(0, 0.02) weights.
Prefill: batch 8 x 2048 random ids into an empty KV cache, logits of the
last position. Decode: batch 32, 128 greedy steps (argmax on the device, fed
back) from a 2048-token cache. Both backends share the weights: ``b200``
runs RMSNorm, RoPE and SwiGLU on the sm_100a kernels, ``torch`` on the
unfused reference math; GEMMs and attention are torch's in both. Times are
CUDA events on the current stream; the cache is reset to its starting
length before every timed repetition.

    python -m ako_b200.benchmark.decoder_bench [--out FILE] [--layers 4]
"""

from __future__ import annotations

import argparse
import json
import statistics
from pathlib import Path

import torch

from ako_b200.decoder import ModelConfig, build_decoder


def _events_ms(fn, reps: int) -> list[float]:
    out = []
    for _ in range(reps):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        out.append(s.elapsed_time(e))
    return out


def run(args) -> dict:
    dev = torch.device("cuda", 0)
    cfg = ModelConfig(n_layers=args.layers, max_seq_len=8192)
    g = torch.Generator(device=dev).manual_seed(1)
    prefill_ids = torch.randint(0, cfg.vocab_size, (args.prefill_batch, args.prefill_len), generator=g, device=dev)
    ctx_ids = torch.randint(0, cfg.vocab_size, (args.decode_batch, args.context), generator=g, device=dev)
    result: dict = {"config": {**cfg.__dict__, "prefill": [args.prefill_batch, args.prefill_len],
                               "decode": [args.decode_batch, args.decode_steps, args.context], "dtype": "bf16"}}
    logits_by_backend = {}
    tokens_by_backend = {}
    for backend in ("b200", "torch"):
        model = build_decoder(cfg, backend=backend, device=dev, seed=0)
        with torch.inference_mode():
            # prefill
            cache = model.new_cache(args.prefill_batch, args.prefill_len)

            def prefill():
                cache.length = 0
                return model(prefill_ids, cache)

            logits_by_backend[backend] = prefill().float()
            for _ in range(args.warmup):
                prefill()
            pms = _events_ms(prefill, args.reps)
            del cache
            # decode
            dcache = model.new_cache(args.decode_batch, args.context + args.decode_steps)
            model(ctx_ids, dcache)  # fill the cache with the context
            first = model.lm_head.weight.new_zeros(0)  # placeholder to keep names short
            start_tok = ctx_ids[:, -1:].clone()

            def decode():
                dcache.length = args.context
                tok = start_tok
                toks = []
                for _ in range(args.decode_steps):
                    tok = model(tok, dcache).argmax(-1, keepdim=True)
                    toks.append(tok)
                return torch.cat(toks, dim=1)

            tokens_by_backend[backend] = decode()
            for _ in range(args.warmup):
                decode()
            dms = _events_ms(decode, args.reps)
            del dcache, first
        p_ms, d_ms = statistics.median(pms), statistics.median(dms)
        result[backend] = {
            "prefill_ms": round(p_ms, 3),
            "prefill_tok_s": round(args.prefill_batch * args.prefill_len / p_ms * 1e3, 1),
            "decode_ms_per_step": round(d_ms / args.decode_steps, 4),
            "decode_tok_s": round(args.decode_batch * args.decode_steps / d_ms * 1e3, 1),
        }
        del model
        torch.cuda.empty_cache()
    a, b = logits_by_backend["b200"], logits_by_backend["torch"]
    result["parity"] = {
        "prefill_logits_max_abs_diff": round((a - b).abs().max().item(), 5),
        "prefill_logits_max_abs": round(b.abs().max().item(), 5),
        "prefill_top1_agreement": round((a.argmax(-1) == b.argmax(-1)).float().mean().item(), 4),
        "decode_greedy_token_agreement": round(
            (tokens_by_backend["b200"] == tokens_by_backend["torch"]).float().mean().item(), 4),
    }
    result["speedup"] = {
        "prefill": round(result["torch"]["prefill_ms"] / result["b200"]["prefill_ms"], 3),
        "decode": round(result["torch"]["decode_ms_per_step"] / result["b200"]["decode_ms_per_step"], 3),
    }
    return result


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--prefill-batch", type=int, default=8)
    ap.add_argument("--prefill-len", type=int, default=2048)
    ap.add_argument("--decode-batch", type=int, default=32)
    ap.add_argument("--decode-steps", type=int, default=128)
    ap.add_argument("--context", type=int, default=2048)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--reps", type=int, default=5)
    ap.add_argument("--out", default=None)
    args = ap.parse_args()
    res = run(args)
    line = json.dumps(res)
    print(line, flush=True)
    if args.out:
        Path(args.out).write_text(json.dumps(res, indent=1))


if __name__ == "__main__":
    main()
