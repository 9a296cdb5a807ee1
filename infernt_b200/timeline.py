"""Phase timeline of the persistent decode kernel.

Captures a traced decode chain (infernt_plan_set_trace: every CTA records
%globaltimer marks and wait counters per step and phase) and summarises the
critical path of each phase kind of a layer (Q|K|V, attention, O, gate/up,
down) and of the LM head:

    python -m infernt_b200.timeline --shape tinyllama --position 40 --steps 8
    python -m infernt_b200.timeline --shape llama3-8b --position 28 --steps 6

The engine is a one-rank TPEngine with the benchmarks' seeded weights
(N(0, 0.02); seed 0 TinyLlama, seed 1 the 8B shape), fed a seeded prompt of
`--prompt` tokens, then an untraced warm-up chain, then the traced chain of
`--steps` steps from `--position`.  `--save` keeps the raw trace
([cta][step][phase][field] int64) and `--load` summarises a saved one.

Per phase (times in microseconds, averaged over layers and steps 1..S-1):
  crit      last CTA's work done minus the previous phase's last work done:
            the phase's share of the step
  inputs    median CTA's input words current (GEMV phases: thread 0's
            tagged reads, field 7) after the previous phase's last work done
  work      median CTA's work done minus its input loaded (fields 2 - 1)
  spread    last CTA's work done minus the median CTA's
  cwait     median CTA's consumer warp 0 wait for full slots (field 5, SM
            cycles at --sm-mhz)
  issued    median CTA's producer issued the phase's last slot (field 4),
            after the previous phase's last work done
Attention phases: the CTAs that own (KV head, split) items, their inputs
landed (1), RoPE and append done (7), first tile's softmax (8), partial
stored (4), merge start / end (5, 6), done (2), median and last.
"""
import argparse
import sys

import numpy as np

KINDS = ["qkv", "attention", "o", "gate_up", "down"]


def summarize(tr, num_layers, sm_mhz=1965.0):
    """Per-phase-kind figures (microseconds) of a trace array
    [cta][step][phase][field] with 5 num_layers + 1 phases per step."""
    tr = np.asarray(tr, dtype=np.float64)
    C, S, P, F = tr.shape
    assert P == 5 * num_layers + 1 and S >= 2, (tr.shape, num_layers)
    out = {}
    for kind in KINDS + ["lm_head"]:
        phases = [P - 1] if kind == "lm_head" else list(range(KINDS.index(kind), P - 1, 5))
        rows = []
        for s in range(1, S):
            for p in phases:
                t = tr[:, s, p, :]
                prev = tr[:, s, p - 1, 2] if p > 0 else tr[:, s - 1, P - 1, 2]
                base = prev.max()
                done = t[:, 2]
                has_in = t[:, 1] > 0  # attention: only the CTAs that own items mark their inputs
                r = {"crit": done.max() - base,
                     "work": np.median(done[has_in] - t[has_in, 1]) if has_in.any() else np.nan,
                     "spread": done.max() - np.median(done),
                     "cwait": np.median(t[:, 5]) * 1e3 / sm_mhz}  # ns, as the marks
                if kind == "attention":
                    own = t[:, 4] > 0
                    r["items"] = float(own.sum())
                    for f, name in ((1, "landed"), (7, "rope_append"), (8, "first_tile"), (4, "partial"),
                                    (5, "merge_start"), (6, "merge_end"), (2, "done")):
                        v = t[own, f]
                        v = v[v > 0]
                        if len(v):
                            r[name] = np.median(v) - base
                            r[name + "_last"] = v.max() - base
                else:
                    cur = t[:, 7] > 0
                    r["inputs"] = np.median(t[cur, 7]) - base if cur.any() else np.nan
                    r["issued"] = np.median(t[:, 4]) - base
                rows.append(r)
        keys = sorted(set().union(*[r.keys() for r in rows]))
        summ = {}
        for k in keys:
            vals = [r[k] for r in rows if k in r and np.isfinite(r[k])]
            if vals:
                # every field is in ns (cwait converted from cycles) but the item count
                summ[k] = float(np.mean(vals)) * (1.0 if k == "items" else 1e-3)
        out[kind] = summ
    steps = [(tr[:, s, P - 1, 2].max() - tr[:, s - 1, P - 1, 2].max()) * 1e-3 for s in range(1, S)]
    out["step_us"] = float(np.mean(steps))
    return out


def format_summary(summ, num_layers):
    cols = ["crit", "inputs", "work", "spread", "cwait", "issued"]
    lines = ["| phase | " + " | ".join(cols) + " |", "|---" * (len(cols) + 1) + "|"]
    layer = 0.0
    for kind in KINDS + ["lm_head"]:
        s = summ[kind]
        if kind != "lm_head":
            layer += s["crit"]
        lines.append("| %s | " % kind + " | ".join("%.2f" % s[c] if c in s else "-" for c in cols) + " |")
    a = summ["attention"]
    att = ["landed", "rope_append", "first_tile", "partial", "merge_start", "merge_end", "done"]
    lines.append("")
    lines.append("attention items per phase: %.1f CTAs; median / last after Q|K|V done:" % a.get("items", 0))
    lines.append("  " + ", ".join("%s %.2f / %.2f" % (k, a[k], a[k + "_last"]) for k in att if k in a))
    lines.append("")
    lines.append("layer critical path %.2f us x %d layers + LM head %.2f = %.1f us; measured step %.1f us"
                 % (layer, num_layers, summ["lm_head"]["crit"], layer * num_layers + summ["lm_head"]["crit"],
                    summ["step_us"]))
    return "\n".join(lines)


def capture(shape, position, steps, prompt_len):
    import infernt_b200 as ib
    if shape == "tinyllama":
        cfg, seed = ib.TINYLLAMA, 0
    else:
        cfg, seed = ib.LLAMA3_8B.with_(max_seq_len=max(600, position + steps + 16)), 1
    eng = ib.TPEngine(cfg, 0, 1, seed=seed, std=0.02)
    try:
        t = None
        for pos, tok in enumerate(ib.prompt(prompt_len, seed, 3, cfg.vocab_size)):
            t = eng.forward_token(tok, pos)
        warm, _ = eng.decode_chain(t, prompt_len, max(1, position - prompt_len))
        tok = warm[-1]
        toks, ms = eng.decode_chain(tok, position, steps)
        tr = eng.trace_chain(tok, position, steps)
        toks2, _ = eng.decode_chain(tok, position, steps)
        assert toks == toks2, "traced chain changed the tokens"
    finally:
        eng.close()
    return cfg, tr, ms / steps


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--shape", choices=["tinyllama", "llama3-8b"], default="tinyllama")
    ap.add_argument("--position", type=int, default=40)
    ap.add_argument("--steps", type=int, default=8)
    ap.add_argument("--prompt", type=int, default=32)
    ap.add_argument("--sm-mhz", type=float, default=1965.0)
    ap.add_argument("--save", default="")
    ap.add_argument("--load", default="")
    a = ap.parse_args(argv)
    if a.load:
        import infernt_b200 as ib
        cfg = ib.TINYLLAMA if a.shape == "tinyllama" else ib.LLAMA3_8B
        tr = np.load(a.load)
    else:
        if a.prompt >= a.position:
            ap.error("--prompt must be below --position")
        cfg, tr, ms = capture(a.shape, a.position, a.steps, a.prompt)
        print("untraced chain: %.4f ms per step" % ms)
        if a.save:
            np.save(a.save, tr)
    print(format_summary(summarize(tr, cfg.num_layers, a.sm_mhz), cfg.num_layers))
    return 0


if __name__ == "__main__":
    sys.exit(main())
