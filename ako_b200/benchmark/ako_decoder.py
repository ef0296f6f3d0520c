"""AKO's own decoder stack (``ako.models.decoder``), benchmark configuration 5,
run through AKO's dispatcher with and without the sm_100a candidates.

The stack is the reference's unmodified ``DecoderStack`` (4 layers, d 4096,
32 heads / 8 KV heads, FFN 11008, eps 1e-5, theta 1e4, neox RoPE) in bf16 with
its seeded random weights, plus the embedding (vocab 32000) and LM head that
the reference leaves out, as plain torch modules outside it. Three modes, each
in a fresh process with its own ``AKO_CACHE_PATH`` so that every selection is
made from scratch:

* ``torch``: ``backend="torch"``, the reference's eager path;
* ``ako``: ``backend="ako"``, AKO's selector over its own candidates;
* ``ako+b200``: the same after ``ako_b200.register(b200_timing=True)``, so
  the sm_100a kernels compete in AKO's validate-then-benchmark selection,
  with every candidate timed from a cold B200 L2.

Prefill: batch 8 x 2048 ids into an empty ``KVCache``, logits of the last
position. Decode: batch 32, 128 greedy steps (argmax fed back) from a
2048-token cache grown by the reference's ``torch.cat``. The first pass of
each phase is untimed: it makes the selector's decisions (autotuning). Times
are CUDA events on the current stream, median of the repetitions. The record
lists, per op and shape, the kernel AKO's selector chose and its speed-up
over the pytorch reference as the selector measured it.

    python -m ako_b200.benchmark.ako_decoder [--out FILE] [--modes torch,ako,ako+b200]

Needs the reference package (``ako_b200.reference``).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
from pathlib import Path

MODES = ("torch", "ako", "ako+b200")


def _events_ms(fn, reps: int, before=None) -> list[float]:
    import torch

    out = []
    for _ in range(reps):
        if before is not None:
            before()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        out.append(s.elapsed_time(e))
    return out


def _selections(cache_path: Path) -> list[dict]:
    if not cache_path.exists():
        return []
    entries = json.loads(cache_path.read_text()).get("entries", {})
    rows = []
    for per_gpu in entries.values():
        for op, shapes in per_gpu.items():
            for key, rec in shapes.items():
                rec = rec if isinstance(rec, dict) else {"kernel": rec}
                rows.append({"op": op, "key": key, "kernel": rec.get("kernel"),
                             "latency_ms": rec.get("latency_p50_ms"), "baseline_ms": rec.get("baseline_ms"),
                             "speedup": rec.get("speedup"),
                             "best_baseline_kernel": rec.get("best_baseline_kernel"),
                             "speedup_vs_best_baseline": rec.get("speedup_vs_best_baseline")})
    return sorted(rows, key=lambda r: (r["op"], r["key"]))


def run_mode(mode: str, args) -> dict:
    """One mode in this process (the caller gave it a fresh ``AKO_CACHE_PATH``)."""
    from ako_b200.reference import ako

    ako()
    import torch
    from ako.models.decoder import ModelConfig, build_stack

    if mode == "ako+b200":
        import ako_b200

        ako_b200.register(b200_timing=True)
    dev = torch.device("cuda", 0)
    cfg = ModelConfig(hidden_dim=4096, n_layers=args.layers, n_heads=32, n_kv_heads=8, intermediate_dim=11008,
                      max_seq_len=8192, rope_base=1e4, rope_style="neox", eps=1e-5)
    stack = build_stack(cfg, backend="torch" if mode == "torch" else "ako", device=dev, dtype=torch.bfloat16,
                        seed=0)
    torch.manual_seed(1)
    embed = torch.nn.Embedding(args.vocab, cfg.hidden_dim).to(dev, torch.bfloat16)
    head = torch.nn.Linear(cfg.hidden_dim, args.vocab, bias=False).to(dev, torch.bfloat16)
    g = torch.Generator(device=dev).manual_seed(2)
    prefill_ids = torch.randint(0, args.vocab, (args.prefill_batch, args.prefill_len), generator=g, device=dev)
    ctx_ids = torch.randint(0, args.vocab, (args.decode_batch, args.context), generator=g, device=dev)

    state: dict = {}

    def prefill():
        cache = stack.new_kv_cache()
        h = stack(embed(prefill_ids), kv_cache=cache)
        state["prefill_logits"] = head(h[:, -1])

    def fill_context():
        cache = stack.new_kv_cache()
        h = stack(embed(ctx_ids), kv_cache=cache)
        state["cache"] = cache
        state["next"] = head(h[:, -1]).argmax(-1, keepdim=True)
        del h
        torch.cuda.synchronize()

    def decode():
        cache, tok = state["cache"], state["next"]
        toks = []
        for _ in range(args.decode_steps):
            h = stack(embed(tok), kv_cache=cache)
            tok = head(h[:, -1]).argmax(-1, keepdim=True)
            toks.append(tok)
        state["tokens"] = torch.cat(toks, dim=1)

    with torch.inference_mode():
        prefill()  # selection for the prefill shapes
        torch.cuda.synchronize()
        pre_ms = _events_ms(prefill, args.reps)
        fill_context()
        decode()  # selection for the decode shapes
        dec_ms = _events_ms(decode, args.reps, before=fill_context)
        tokens = state["tokens"].cpu().tolist()
        logits = state["prefill_logits"].float().cpu()
    pre, dec = statistics.median(pre_ms), statistics.median(dec_ms)
    return {
        "mode": mode,
        "prefill_ms": round(pre, 3), "prefill_ms_all": [round(v, 3) for v in pre_ms],
        "prefill_tok_s": round(args.prefill_batch * args.prefill_len / pre * 1e3, 1),
        "decode_ms_per_step": round(dec / args.decode_steps, 4),
        "decode_ms_all": [round(v, 3) for v in dec_ms],
        "decode_tok_s": round(args.decode_batch * args.decode_steps / dec * 1e3, 1),
        "prefill_logits_checksum": round(float(logits.double().sum()), 3),
        "decode_tokens_head": tokens[0][:16],
        "decode_tokens": tokens,
        "selections": _selections(Path(os.environ["AKO_CACHE_PATH"])),
    }


def _agreement(a: list[list[int]], b: list[list[int]]) -> float:
    same = sum(x == y for ra, rb in zip(a, b) for x, y in zip(ra, rb))
    return same / max(1, sum(len(r) for r in a))


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--modes", default=",".join(MODES))
    ap.add_argument("--mode", default=None, help=argparse.SUPPRESS)
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--vocab", type=int, default=32000)
    ap.add_argument("--prefill-batch", type=int, default=8)
    ap.add_argument("--prefill-len", type=int, default=2048)
    ap.add_argument("--decode-batch", type=int, default=32)
    ap.add_argument("--decode-steps", type=int, default=128)
    ap.add_argument("--context", type=int, default=2048)
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--out", default=None)
    args = ap.parse_args()
    if args.mode is not None:
        print(json.dumps(run_mode(args.mode, args)))
        return
    from ako_b200.reference import ako

    ako()  # fails here, naming where it looked, when the reference package is missing
    results = []
    child = [f"--{k.replace('_', '-')}={v}" for k, v in vars(args).items() if k not in ("modes", "mode", "out")]
    for mode in args.modes.split(","):
        with tempfile.TemporaryDirectory() as tmp:
            env = dict(os.environ, AKO_CACHE_PATH=str(Path(tmp) / "kernel_cache.json"))
            proc = subprocess.run([sys.executable, "-m", "ako_b200.benchmark.ako_decoder", "--mode", mode, *child],
                                  env=env, capture_output=True, text=True, check=False)
        if proc.returncode != 0:
            sys.stderr.write(proc.stderr)
            raise SystemExit(f"mode {mode} failed with status {proc.returncode}")
        res = json.loads(proc.stdout.strip().splitlines()[-1])
        results.append(res)
        print(f"{mode:9s} prefill {res['prefill_ms']:8.2f} ms ({res['prefill_tok_s']:9.0f} tok/s)  "
              f"decode {res['decode_ms_per_step']:7.3f} ms/step ({res['decode_tok_s']:8.0f} tok/s)", flush=True)
        for sel in res["selections"]:
            print(f"    {sel['op']:17s} {sel['key'][:60]:60s} -> {sel['kernel']} (x{sel['speedup']})", flush=True)
    base = next((r for r in results if r["mode"] == "torch"), None)
    if base is not None:
        for r in results:
            r["decode_token_agreement_with_torch"] = round(_agreement(base["decode_tokens"], r["decode_tokens"]), 4)
            print(f"{r['mode']:9s} greedy tokens equal to the torch mode's: {r['decode_token_agreement_with_torch']:.4f}")
    for r in results:
        r.pop("decode_tokens")
    if args.out:
        Path(args.out).write_text(json.dumps({"config": vars(args), "results": results}, indent=1))


if __name__ == "__main__":
    main()
