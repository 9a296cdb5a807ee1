"""Batched decode on the tensor cores (infernt_batch_engine_*) against the
CPU oracle, sequence by sequence.

The oracle runs the same seeded model with bf16-rounded weights in its
batched-decode variant (act_bf16: activations rounded to bf16 where they
enter a projection, K/V rows rounded to bf16), so both sides round the same
quantities.  Their sums differ only in order (FP32 tensor-core sums over K
splits against double sums): the logits then agree to about 1e-6 of the
largest |logit|, except where a value lands within that difference of a bf16
rounding tie and the two sides round it to neighbouring bf16 values (one
bf16 step, 2^-8 relative); such a flip moves the logits by up to a few
1e-3.  How many cases flip depends on the inputs (sums with heavy
cancellation have the largest relative differences): a third to two thirds
of the cases of these small configurations show a flip.  The test therefore requires:
every (step, sequence) within 1e-2 of the largest |logit| and at least one
within 1e-5; the kernels themselves are held to FP32 rounding by the
batched attention and projection tests;
greedy tokens identical unless the oracle's top-2 gap is below twice the
step's error."""
import numpy as np
import pytest

import infernt_b200 as ib
import oracle as O

pytestmark = pytest.mark.gpu

CFG = ib.ModelConfig(vocab_size=1024, hidden_size=512, num_layers=2, num_attention_heads=8,
                     num_key_value_heads=2, intermediate_size=1024, max_seq_len=256, rms_norm_eps=1e-5,
                     rope_theta=10000.0, weight_dtype=ib.DTYPE_BF16)
CFG_D128 = CFG.with_(hidden_size=1024, num_attention_heads=8, num_key_value_heads=4, head_dim=128,
                     intermediate_size=1536, num_layers=1)


def top2_gap(x):
    s = np.sort(x)
    return float(s[-1] - s[-2])


def check_batch(cfg, n_pos, steps=3, seed=5, attn_splits=0, attention=None):
    T = len(n_pos)
    eng = ib.BatchEngine(cfg, T, seed=seed, attn_splits=attn_splits)
    if attention:
        eng.set_attention(*attention)
    orcs = []
    for b, p in enumerate(n_pos):
        eng.fill_kv(b, 100 + b, p)
        o = O.LlamaOracle(cfg, seed=seed, round_bf16=True, act_bf16=True)
        o.fill_kv(100 + b, p)
        orcs.append(o)
    tokens = [int(t) for t in O.prompt(T, seed, 3, cfg.vocab_size)]
    positions = list(n_pos)
    rel = []
    for step in range(steps):
        nxt = eng.step(tokens, positions)
        logits = eng.logits()
        for b in range(T):
            want_tok, want = orcs[b].decode_token(tokens[b], positions[b])
            err = float(np.abs(logits[b] - want).max())
            scale = float(np.abs(want).max())
            rel.append(err / scale)
            assert err <= 1e-2 * scale, (step, b, err, scale)
            if nxt[b] != want_tok:
                assert top2_gap(want) < 2 * err, (step, b, nxt[b], want_tok)
        tokens = nxt
        positions = [p + 1 for p in positions]
    eng.close()
    assert min(rel) <= 1e-5, rel


def test_batch_matches_oracle_mixed_contexts():
    """Five sequences at contexts 0..130 (one or three attention splits)."""
    check_batch(CFG, [0, 3, 40, 65, 130])


def test_batch_single_split_and_many_splits():
    check_batch(CFG, [7, 100], attn_splits=1)
    check_batch(CFG, [7, 100], attn_splits=16)


def test_batch_head_dim_128():
    check_batch(CFG_D128, [2, 70, 129])


def test_batch_attention_work_splits():
    """(splits, least chunk, copy stages) change the work split only:
    chunks of 32 positions with 5 splits (ragged last tiles), one split of
    everything, deep and shallow copy rings."""
    check_batch(CFG, [0, 33, 200], attention=(5, 32, 4))
    check_batch(CFG, [0, 33, 200], attention=(2, 512, 2))
    check_batch(CFG_D128, [1, 95], attention=(3, 32, 2))


def test_batch_group_of_16_heads():
    """16 query heads per KV head (the CUDA-core partials)."""
    cfg = CFG.with_(hidden_size=1024, num_attention_heads=16, num_key_value_heads=1, intermediate_size=1024)
    check_batch(cfg, [0, 50, 140])


def test_batch_decode_chain_equals_steps():
    T = 4
    eng = ib.BatchEngine(CFG, T, seed=9)
    for b in range(T):
        eng.fill_kv(b, 200 + b, 10 * b)
    tokens = [5, 6, 7, 8]
    positions = [0, 10, 20, 30]
    chain, _ = eng.decode(tokens, positions, 4)
    eng.close()
    eng = ib.BatchEngine(CFG, T, seed=9)
    for b in range(T):
        eng.fill_kv(b, 200 + b, 10 * b)
    toks, pos = list(tokens), list(positions)
    for s in range(4):
        toks = eng.step(toks, pos)
        pos = [p + 1 for p in pos]
        assert list(chain[s]) == toks, s
    eng.close()
