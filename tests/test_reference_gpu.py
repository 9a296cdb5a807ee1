"""The new engine against the reference's own build on the same GPU, the
same seeded weights and the same prompt (logits and greedy tokens).

The reference runner (oracle/_ref/libinfernt_ref.so) is built from the
reference checkout by `make -C oracle ref`; without it these tests skip
and parity rests on the oracle (itself pinned to fixtures the reference
build produced)."""
import numpy as np
import pytest

import infernt_b200 as ib
import oracle as O

pytestmark = pytest.mark.gpu

CFG = ib.ModelConfig(vocab_size=1000, hidden_size=512, num_layers=2, num_attention_heads=8,
                     num_key_value_heads=2, intermediate_size=1536, max_seq_len=128)


def _need_ref():
    if not O.ref_available():
        pytest.skip("reference runner not built")


@pytest.mark.parametrize("cfg,steps", [(CFG, 16), (ib.TINYLLAMA, 4)], ids=["h512", "tinyllama"])
def test_logits_and_tokens_match_reference_build(cfg, steps):
    _need_ref()
    ref = O.RefArch(cfg, seed=4)
    eng = ib.Engine(cfg, seed=4)
    prompt = O.prompt(steps, 4, 3, cfg.vocab_size)
    for pos in range(steps):
        t_ref, l_ref = ref.decode(int(prompt[pos]), pos)
        t_me = eng.forward_token(int(prompt[pos]), pos)
        l_me = eng.logits()
        err = float(np.abs(l_me - l_ref).max())
        assert err <= 1e-3 and err / float(np.abs(l_ref).max()) <= 1e-4, (pos, err)
        s = np.sort(l_ref)
        if s[-1] - s[-2] >= 1e-4:
            assert t_me == t_ref, pos
    ref.close()
    eng.close()


def test_reference_engine_loop_runs():
    """The benchmark's reference arm: InferenceEngine::forward_token +
    sample_next_token, timed with CUDA events."""
    _need_ref()
    eng = O.RefEngine(CFG, seed=2)
    toks, ms = eng.decode_loop(5, 0, 8)
    assert len(toks) == 8 and ms > 0
    eng.close()
