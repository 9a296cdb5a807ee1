"""Writes tests/golden/ref_forward_*.npz: logits and greedy tokens produced
by the reference's own build (INFERNT sources compiled unchanged for sm_100
into oracle/_ref/libinfernt_ref.so, cuBLAS FP32) on seeded weights, driven
through launch_embedding_lookup + LlamaArchitecture::forward + launch_argmax
(the reference's forward_token sequence, src/engine.cpp:53-76).

Needs a GPU and the prebuilt runner:  python tests/golden/make_ref_fixtures.py [outdir]
The CPU test tests/test_oracle_golden.py::test_oracle_matches_reference_build
checks the oracle against these files.
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

import infernt_b200 as ib  # noqa: E402  (configuration presets only)
import oracle as O  # noqa: E402

CASES = [
    # name, config, seed, steps, logit rows kept (None = all)
    ("gen_h128", ib.ModelConfig(vocab_size=500, hidden_size=128, num_layers=3, num_attention_heads=8,
                                num_key_value_heads=2, intermediate_size=256, max_seq_len=64,
                                rms_norm_eps=1e-6, rope_theta=50000.0), 3, 12, None),
    ("gen_h512", ib.ModelConfig(vocab_size=1000, hidden_size=512, num_layers=2, num_attention_heads=8,
                                num_key_value_heads=2, intermediate_size=1536, max_seq_len=128), 5, 12, None),
    ("tinyllama", ib.TINYLLAMA, 0, 3, np.arange(0, 32000, 37)),
]


def main(outdir):
    os.makedirs(outdir, exist_ok=True)
    for name, cfg, seed, steps, rows in CASES:
        ref = O.RefArch(cfg, seed=seed, std=0.02)
        prompt = O.prompt(steps, seed, 3, cfg.vocab_size)
        logits_all, nexts = [], []
        for pos in range(steps):
            t, logits = ref.decode(int(prompt[pos]), pos)
            logits_all.append(logits if rows is None else logits[rows])
            nexts.append(t)
        ref.close()
        path = os.path.join(outdir, "ref_forward_%s.npz" % name)
        np.savez_compressed(path, cfg_ints=np.array(cfg.ints(), dtype=np.int64),
                            eps=np.float32(cfg.rms_norm_eps), theta=np.float32(cfg.rope_theta),
                            seed=np.int64(seed), std=np.float32(0.02), tokens=prompt.astype(np.int32),
                            logits=np.stack(logits_all).astype(np.float32),
                            next=np.array(nexts, dtype=np.int32),
                            logit_rows=(np.array([], dtype=np.int64) if rows is None else rows))
        print("wrote", path)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.path.dirname(os.path.abspath(__file__)))
