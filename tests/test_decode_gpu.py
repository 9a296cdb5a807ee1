"""Decode-step parity on the GPU: the fused plan (through the C++
InferenceEngine's C entry points) against the CPU oracle on the same
seeded weights and prompts.

FP32 tolerance (the stated bar for the FP32 path): logits within max-abs
1e-3 and max-abs / max|logit| 1e-4 at every step; greedy tokens identical
unless the oracle's top-2 gap is below 1e-4 (a logged near-tie).
bf16-weight variant: the oracle runs on the same bf16-rounded weights with
FP32 arithmetic; the same tolerance applies (both sides accumulate in FP32)."""
import numpy as np
import pytest

import infernt_b200 as ib
import oracle as O

pytestmark = pytest.mark.gpu

SMALL_FAST = ib.ModelConfig(vocab_size=1000, hidden_size=512, num_layers=2, num_attention_heads=8,
                            num_key_value_heads=2, intermediate_size=1536, max_seq_len=128,
                            rms_norm_eps=1e-5, rope_theta=10000.0)
SMALL_PLAIN = ib.ModelConfig(vocab_size=500, hidden_size=128, num_layers=3, num_attention_heads=8,
                             num_key_value_heads=2, intermediate_size=256, max_seq_len=64,
                             rms_norm_eps=1e-6, rope_theta=50000.0)


def check_logits(got, want, where):
    err = float(np.abs(got - want).max())
    scale = float(np.abs(want).max())
    assert err <= 1e-3 and err / scale <= 1e-4, (where, err, scale)


def top2_gap(logits):
    s = np.sort(logits)
    return float(s[-1] - s[-2])


def run_parity(cfg, seed, steps, bf16=False, start_tokens=4, mode=None, expect_mode=None):
    eng = ib.Engine(cfg, seed=seed)
    if mode is not None:
        eng.set_mode(mode)
    orc = O.LlamaOracle(cfg, seed=seed, round_bf16=bf16)
    prompt = O.prompt(start_tokens, seed, 3, cfg.vocab_size)
    near_ties = []
    tok = None
    for pos in range(start_tokens + steps):
        t_in = int(prompt[pos]) if pos < start_tokens else tok
        mine = eng.forward_token(t_in, pos)
        want_tok, want_logits = orc.decode_token(t_in, pos)
        check_logits(eng.logits(), want_logits, (cfg, pos))
        if mine != want_tok:
            assert top2_gap(want_logits) < 1e-4, (pos, mine, want_tok)
            near_ties.append(pos)
        tok = want_tok  # follow the oracle's path
    if expect_mode is not None:
        assert eng.mode == expect_mode
    eng.close()
    return near_ties


@pytest.mark.parametrize("cfg,mode,expect", [
    (SMALL_FAST, ib.MODE_PERSISTENT, ib.MODE_PERSISTENT),
    (SMALL_FAST, ib.MODE_GRAPH, ib.MODE_GRAPH),
    (SMALL_FAST, ib.MODE_EAGER, ib.MODE_EAGER),
    (SMALL_PLAIN, ib.MODE_PERSISTENT, ib.MODE_GRAPH),  # h=128: falls back to the kernel sequence
], ids=["persistent", "graph_tma", "eager_tma", "graph_plain"])
def test_decode_matches_oracle(cfg, mode, expect):
    run_parity(cfg, seed=5, steps=20, mode=mode, expect_mode=expect)


@pytest.mark.parametrize("mode", [ib.MODE_PERSISTENT, ib.MODE_GRAPH], ids=["persistent", "graph"])
def test_decode_bf16_matches_oracle_on_rounded_weights(mode):
    run_parity(SMALL_FAST.with_(weight_dtype=ib.DTYPE_BF16), seed=6, steps=12, bf16=True, mode=mode,
               expect_mode=mode)


def test_persistent_split_groups_match_oracle():
    """Shapes whose row-group counts are not multiples of the CTA count
    (uneven group ranges per CTA, a ragged last group in the LM head)."""
    cfg = ib.ModelConfig(vocab_size=3001, hidden_size=1024, num_layers=2, num_attention_heads=16,
                         num_key_value_heads=4, intermediate_size=2560, max_seq_len=96)
    run_parity(cfg, seed=12, steps=10, mode=ib.MODE_PERSISTENT, expect_mode=ib.MODE_PERSISTENT)


@pytest.mark.parametrize("mode", [ib.MODE_PERSISTENT, ib.MODE_GRAPH], ids=["persistent", "graph"])
def test_chain_equals_stepwise(mode):
    """Device-chained decode produces the same tokens as host-driven steps."""
    cfg = SMALL_FAST
    eng = ib.Engine(cfg, seed=7)
    eng.set_mode(mode)
    toks = []
    t = 11
    for pos in range(30):
        t = eng.forward_token(t, pos)
        toks.append(t)
    eng.reset()
    chain, ms = eng.decode_chain(11, 0, 30)
    assert chain == toks
    assert ms > 0
    eng.close()


def test_sample_next_token_greedy_is_last_token():
    eng = ib.Engine(SMALL_FAST, seed=8)
    t = eng.forward_token(5, 0)
    assert eng.sample_next_token(0.0) == t
    assert eng.sample_next_token(0.0) == t
    assert 0 <= eng.sample_next_token(0.7) < SMALL_FAST.vocab_size
    eng.close()


def test_bad_position_and_token_are_rejected():
    cfg = SMALL_FAST
    eng = ib.Engine(cfg, seed=9)
    with pytest.raises(ib.InferntError):
        eng.forward_token(1, cfg.max_seq_len)
    with pytest.raises(ib.InferntError):
        eng.forward_token(cfg.vocab_size, 0)
    with pytest.raises(ib.InferntError):
        eng.decode_chain(1, cfg.max_seq_len - 2, 5)
    # the engine stays usable after rejected calls
    assert 0 <= eng.forward_token(1, 0) < cfg.vocab_size
    eng.close()


def test_tinyllama_first_steps_match_oracle():
    """TinyLlama-1.1B shape, FP32, seed 0: the first decode steps of the
    32-token prompt (positions 0..5) against the oracle."""
    O.set_threads(8)
    cfg = ib.TINYLLAMA
    eng = ib.Engine(cfg, seed=0)
    orc = O.LlamaOracle(cfg, seed=0)
    prompt = O.prompt(32, 0, 3, cfg.vocab_size)
    for pos in range(6):
        mine = eng.forward_token(int(prompt[pos]), pos)
        want_tok, want_logits = orc.decode_token(int(prompt[pos]), pos)
        check_logits(eng.logits(), want_logits, pos)
        assert mine == want_tok or top2_gap(want_logits) < 1e-4
    eng.close()


@pytest.mark.parametrize("mode", [ib.MODE_PERSISTENT, ib.MODE_GRAPH], ids=["persistent", "graph"])
def test_mid_context_positions_match_oracle(mode):
    """One layer at the TinyLlama shape, KV prefilled up to each position:
    1 to 10 key splits per KV head, tile edges (31, 32, 33, 64) and the
    bench's positions (40..296)."""
    cfg = ib.TINYLLAMA.with_(num_layers=1, max_seq_len=512)
    eng = ib.Engine(cfg, seed=2)
    eng.set_mode(mode)
    orc = O.LlamaOracle(cfg, seed=2)
    for pos in (31, 32, 33, 40, 64, 100, 131, 200, 296, 511):
        eng.fill_kv(seed=pos, n_pos=pos, std=1.0)
        orc.fill_kv(seed=pos, n_pos=pos, std=1.0)
        mine = eng.forward_token(77 + pos, pos)
        want_tok, want_logits = orc.decode_token(77 + pos, pos)
        check_logits(eng.logits(), want_logits, pos)
        assert mine == want_tok or top2_gap(want_logits) < 1e-4
    assert eng.mode == mode
    eng.close()


def test_long_context_position_4095_matches_oracle():
    """One layer at the TinyLlama shape, KV prefilled with seeded N(0,1) for
    positions 0..4094, decode at position 4095 (past the reference's 1024-key
    limit, where only the oracle is a valid reference)."""
    cfg = ib.TINYLLAMA.with_(num_layers=1, max_seq_len=4096)
    eng = ib.Engine(cfg, seed=0)
    eng.fill_kv(seed=0, n_pos=4095, std=1.0)
    orc = O.LlamaOracle(cfg, seed=0)
    orc.fill_kv(seed=0, n_pos=4095, std=1.0)
    mine = eng.forward_token(123, 4095)
    want_tok, want_logits = orc.decode_token(123, 4095)
    check_logits(eng.logits(), want_logits, 4095)
    assert mine == want_tok or top2_gap(want_logits) < 1e-4
    eng.close()
