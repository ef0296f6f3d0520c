"""Decoder throughput, benchmark configuration 5: prefill and decode tokens per second.

4-layer LLaMA-style stack (d 4096, 32 heads / 8 KV heads, head_dim 128, FFN
11008, eps 1e-5, theta 1e4, vocab 32000), bf16, random N(0, 0.02) weights.
Prefill: batch 8 x 2048 random ids into an empty KV cache, logits of the
last position. Decode: batch 32, 128 greedy steps (argmax on the device, fed
back) from a 2048-token cache, eagerly and with each whole step replayed
from one CUDA graph. Both backends share the weights: ``b200`` runs RMSNorm,
RoPE and SwiGLU on the sm_100a kernels, ``torch`` on the unfused reference
math; GEMMs and attention are torch's in both. Accuracy: both are compared
with an fp32 evaluation of the same weights on the same tokens (decode
teacher-forced). Times are CUDA events on the current stream; the cache is
reset to its starting length before every timed repetition.

    python -m ako_b200.benchmark.decoder_bench [--out FILE] [--layers 4]
"""

from __future__ import annotations

import argparse
import json
import statistics
from pathlib import Path

import torch

from ako_b200.decoder import GraphDecoder, ModelConfig, build_decoder


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
    forced = torch.randint(0, cfg.vocab_size, (args.decode_batch, 8), generator=g, device=dev)
    result: dict = {"config": {**cfg.__dict__, "prefill": [args.prefill_batch, args.prefill_len],
                               "decode": [args.decode_batch, args.decode_steps, args.context], "dtype": "bf16",
                               "weights": "N(0, 0.02), seed 0"}}
    prefill_logits, forced_logits = {}, {}
    for backend in ("b200", "torch", "fp32"):
        dtype = torch.float32 if backend == "fp32" else torch.bfloat16
        model = build_decoder(cfg, backend="torch" if backend == "fp32" else backend, device=dev, seed=0)
        if backend == "fp32":
            model = model.float()  # the same bf16 weights, evaluated in fp32: the accuracy yardstick
        with torch.inference_mode():
            cache = model.new_cache(args.prefill_batch, args.prefill_len)

            def prefill():
                cache.length = 0
                return model(prefill_ids, cache)

            prefill_logits[backend] = prefill().float()
            # teacher-forced decode logits: every backend is fed the same tokens
            small = model.new_cache(args.decode_batch, args.context + 8)
            model(ctx_ids, small)
            forced_logits[backend] = torch.stack([model(forced[:, i:i + 1], small).float() for i in range(8)], 1)
            del small
            if backend == "fp32":
                del cache, model
                torch.cuda.empty_cache()
                continue
            for _ in range(args.warmup):
                prefill()
            pms = _events_ms(prefill, args.reps)
            del cache
            dcache = model.new_cache(args.decode_batch, args.context + args.decode_steps)
            model(ctx_ids, dcache)  # the context fills the cache
            start_tok = ctx_ids[:, -1:].clone()

            def decode_eager():
                dcache.length = args.context
                tok = start_tok
                for _ in range(args.decode_steps):
                    tok = model(tok, dcache).argmax(-1, keepdim=True)
                return tok

            for _ in range(args.warmup):
                decode_eager()
            dms = _events_ms(decode_eager, args.reps)
            dcache.length = args.context
            gd = GraphDecoder(model, dcache, start_tok, args.decode_steps)
            gd.capture()
            for _ in range(args.warmup):
                gd.run(start_tok)
            gms = _events_ms(lambda: gd.run(start_tok), args.reps)
            del gd, dcache
        p_ms, d_ms, g_ms = statistics.median(pms), statistics.median(dms), statistics.median(gms)
        n_dec = args.decode_batch * args.decode_steps
        result[backend] = {
            "prefill_ms": round(p_ms, 3),
            "prefill_tok_s": round(args.prefill_batch * args.prefill_len / p_ms * 1e3, 1),
            "decode_ms_per_step": round(d_ms / args.decode_steps, 4),
            "decode_tok_s": round(n_dec / d_ms * 1e3, 1),
            "decode_graph_ms_per_step": round(g_ms / args.decode_steps, 4),
            "decode_graph_tok_s": round(n_dec / g_ms * 1e3, 1),
        }
        del model
        torch.cuda.empty_cache()
    truth_p, truth_d = prefill_logits["fp32"], forced_logits["fp32"]
    result["parity"] = {
        "note": "max |logit - fp32 logit| of each bf16 backend, same weights and tokens (decode teacher-forced)",
        "logit_scale": round(truth_p.abs().max().item(), 4),
        **{f"{b}_prefill_vs_fp32": round((prefill_logits[b] - truth_p).abs().max().item(), 5) for b in ("b200", "torch")},
        **{f"{b}_decode_vs_fp32": round((forced_logits[b] - truth_d).abs().max().item(), 5) for b in ("b200", "torch")},
        "b200_vs_torch_prefill": round((prefill_logits["b200"] - prefill_logits["torch"]).abs().max().item(), 5),
    }
    result["speedup_vs_reference_math"] = {
        "prefill": round(result["torch"]["prefill_ms"] / result["b200"]["prefill_ms"], 3),
        "decode": round(result["torch"]["decode_ms_per_step"] / result["b200"]["decode_ms_per_step"], 3),
        "decode_graph": round(result["torch"]["decode_graph_ms_per_step"] / result["b200"]["decode_graph_ms_per_step"], 3),
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
