"""A decode run sized for profilers: one seeded engine, a short prompt, then
one chained launch of the persistent decode kernel.

    python -m infernt_b200.profile_case --layers 4 --steps 8

The TinyLlama-1.1B shape (or, with `--shape llama3-8b`, the Llama-3-8B
shape) with `--layers` decoder layers (the per-layer matrices keep their
full size; `--vocab` shrinks the embedding and LM head), seeded N(0, 0.02)
weights.
Launch order on the device: `--prompt` single-step launches (the prompt),
then one warm-up chain and one measured chain of `--steps` steps, so a
profiler that skips `--prompt + 1` launches of the decode kernel captures
the measured chain.

    python -m infernt_b200.profile_case --batched 64 --layers 2

runs the batched engine instead (bf16, `--batched` sequences with contexts
uniform in [512, 2048], numpy seed 1234, seeded KV rows): `--steps` timed
steps, then one more step between cudaProfilerStart and cudaProfilerStop,
for a profiler started with `--profile-from-start off`.

    python -m infernt_b200.profile_case --prefill 4096 --start 28672 --layers 1 --shape llama3-8b

runs the batched engine's prompt prefill (bf16, one sequence): the first
`--start` KV rows seeded, then a prompt of `--prefill` seeded tokens at
positions [start, start + prefill) in chunks of `--chunk`, twice (a warm-up
prefill, then the measured one).  Per chunk and layer the launch order is
pgemm (Q|K|V), pf_qkv_rope, pf_attn, pgemm (O), bt_resid_norm, pgemm
(gate/up), bt_swiglu, pgemm (down), bt_resid_norm."""
import argparse
import sys

import infernt_b200 as ib


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--steps", type=int, default=8)
    ap.add_argument("--prompt", type=int, default=2)
    ap.add_argument("--bf16", action="store_true", help="bf16 weights (FP32 activations)")
    ap.add_argument("--shape", choices=["tinyllama", "llama3-8b"], default="tinyllama")
    ap.add_argument("--vocab", type=int, default=0, help="vocabulary size (0: the shape's own)")
    ap.add_argument("--batched", type=int, default=0, help="sequences of a batched-engine run (0: b=1 decode)")
    ap.add_argument("--prefill", type=int, default=0, help="prompt tokens of a prefill run (0: decode)")
    ap.add_argument("--start", type=int, default=0, help="prefill: seeded KV rows before the prompt")
    ap.add_argument("--chunk", type=int, default=4096, help="prefill: tokens per chunk")
    args = ap.parse_args(argv)
    if args.prefill:
        return prefill(args)
    if args.batched:
        return batched(args)
    base = ib.TINYLLAMA if args.shape == "tinyllama" else ib.LLAMA3_8B.with_(max_seq_len=1024)
    cfg = base.with_(num_layers=args.layers)
    if args.vocab:
        cfg = cfg.with_(vocab_size=args.vocab)
    if args.bf16:
        cfg = cfg.with_(weight_dtype=ib.DTYPE_BF16)
    eng = ib.Engine(cfg, seed=0)
    t = 5
    for pos in range(args.prompt):
        t = eng.forward_token(t, pos)
    eng.decode_chain(t, args.prompt, args.steps)
    toks, ms = eng.decode_chain(t, args.prompt, args.steps)
    wbytes = cfg.weight_params * (2 if args.bf16 else 4)
    print("layers=%d steps=%d mode=%d: %.4f ms/step, %.0f tok/s, weights %.3f GB -> %.1f GB/s"
          % (args.layers, args.steps, eng.mode, ms / args.steps, args.steps * 1e3 / ms, wbytes / 1e9,
             wbytes / (ms / args.steps / 1e3) / 1e9))
    eng.close()
    return 0


def batched(args):
    import numpy as np
    import torch
    T = args.batched
    base = ib.TINYLLAMA if args.shape == "tinyllama" else ib.LLAMA3_8B
    cfg = base.with_(num_layers=args.layers, weight_dtype=ib.DTYPE_BF16, max_seq_len=2048 + 2 * args.steps + 8)
    if args.vocab:
        cfg = cfg.with_(vocab_size=args.vocab)
    eng = ib.BatchEngine(cfg, T, seed=0)
    ctx = np.random.default_rng(1234).integers(512, 2049, size=T)
    for b in range(T):
        eng.fill_kv(b, 1000 + b, int(ctx[b]))
    tokens = [5 + b for b in range(T)]
    pos = [int(c) for c in ctx]
    toks, _ = eng.decode(tokens, pos, args.steps)
    tokens, pos = [int(t) for t in toks[-1]], [p + args.steps for p in pos]
    toks, ms = eng.decode(tokens, pos, args.steps)
    tokens, pos = [int(t) for t in toks[-1]], [p + args.steps for p in pos]
    print("batched T=%d layers=%d: %.4f ms/step, %.0f tok/s, splits %s"
          % (T, args.layers, ms / args.steps, T * args.steps * 1e3 / ms, eng.splits()))
    torch.cuda.synchronize()
    torch.cuda.cudart().cudaProfilerStart()
    eng.step(tokens, pos)
    torch.cuda.synchronize()
    torch.cuda.cudart().cudaProfilerStop()
    eng.close()
    return 0


def prefill(args):
    import oracle as O
    base = ib.TINYLLAMA if args.shape == "tinyllama" else ib.LLAMA3_8B
    cfg = base.with_(num_layers=args.layers, weight_dtype=ib.DTYPE_BF16, max_seq_len=args.start + args.prefill + 8)
    if args.vocab:
        cfg = cfg.with_(vocab_size=args.vocab)
    eng = ib.BatchEngine(cfg, 1, seed=1)
    if args.start:
        eng.fill_kv(0, 77, args.start)
    prompt = O.prompt(args.prefill, 1000, 3, cfg.vocab_size)
    eng.prefill(0, prompt, start_pos=args.start, chunk=args.chunk)
    nxt, _, ms = eng.prefill(0, prompt, start_pos=args.start, chunk=args.chunk)
    print("prefill tokens=%d start=%d layers=%d chunk=%d: %.3f ms, %.0f tok/s, next token %d"
          % (args.prefill, args.start, args.layers, args.chunk, ms, args.prefill * 1e3 / ms, nxt))
    eng.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
