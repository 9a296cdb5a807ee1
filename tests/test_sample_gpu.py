"""Temperature sampling on the GPU (infernt_sample_tokens, Gumbel-max)
against the distribution the reference samples on the host,
softmax(logits / T) (src/engine.cpp:78-104).  The reference's draws come
from a host mt19937, so parity is statistical: the counts of many
independent rows must pass a chi-square test against softmax(logits / T)
computed in float64 (p-value above 1e-6), and the greedy path (T <= 0) is
the exact argmax with the lowest index among equal maxima."""
import numpy as np
import pytest

import infernt_b200 as ib

pytestmark = pytest.mark.gpu


def sample(cuda, logits, rows, temperature, seed=1, counter=0, ld=0):
    torch = cuda
    lg = torch.as_tensor(np.asarray(logits, dtype=np.float32), device="cuda").contiguous()
    V = lg.shape[-1]
    out = torch.full((rows,), -1, dtype=torch.int32, device="cuda")
    ws = torch.zeros(int(ib.lib().infernt_sample_workspace_bytes(rows)), dtype=torch.uint8, device="cuda")
    ib.call("infernt_sample_tokens", lg.data_ptr(), ld, rows, V, temperature, seed, counter, out.data_ptr(),
            ws.data_ptr(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return out.cpu().numpy()


def chi2_pvalue(counts, probs, n):
    from scipy.stats import chi2
    exp = probs * n
    keep = exp >= 5
    c = np.append(counts[keep], counts[~keep].sum())
    e = np.append(exp[keep], exp[~keep].sum())
    if e[-1] == 0:
        c, e = c[:-1], e[:-1]
    stat = float(((c - e) ** 2 / e).sum())
    return float(chi2.sf(stat, len(c) - 1))


@pytest.mark.parametrize("temperature", [1.0, 0.5, 2.0])
def test_sampling_follows_softmax(cuda, temperature):
    rng = np.random.default_rng(5)
    logits = (rng.standard_normal(16) * 2.0).astype(np.float32)
    n = 60000
    toks = sample(cuda, logits, n, temperature, seed=42)
    assert toks.min() >= 0 and toks.max() < 16
    z = logits.astype(np.float64) / temperature
    p = np.exp(z - z.max())
    p /= p.sum()
    counts = np.bincount(toks, minlength=16).astype(np.float64)
    assert chi2_pvalue(counts, p, n) > 1e-6


def test_sampling_large_vocabulary(cuda):
    rng = np.random.default_rng(6)
    V = 32000
    logits = rng.standard_normal(V).astype(np.float32)
    logits[[17, 4000, 31999]] = [9.0, 8.5, 8.0]  # a few likely tokens at the edges of the slices
    n = 30000
    toks = sample(cuda, logits, n, 1.0, seed=7)
    z = logits.astype(np.float64)
    p = np.exp(z - z.max())
    p /= p.sum()
    for t in (17, 4000, 31999):
        c = int((toks == t).sum())
        sd = np.sqrt(n * p[t] * (1 - p[t]))
        assert abs(c - n * p[t]) < 6 * sd, (t, c, n * p[t])


def test_greedy_ties_and_nan(cuda):
    logits = np.zeros(4096, dtype=np.float32)
    logits[[3000, 700, 2500]] = 5.0
    logits[100] = np.nan
    toks = sample(cuda, logits, 4, 0.0)
    assert list(toks) == [700] * 4


def test_reproducible_per_seed_and_counter(cuda):
    logits = np.linspace(0, 1, 64, dtype=np.float32)
    a = sample(cuda, logits, 500, 1.0, seed=3, counter=10)
    b = sample(cuda, logits, 500, 1.0, seed=3, counter=10)
    c = sample(cuda, logits, 500, 1.0, seed=4, counter=10)
    d = sample(cuda, logits, 490, 1.0, seed=3, counter=20)
    assert np.array_equal(a, b)
    assert (a != c).mean() > 0.5
    assert np.array_equal(a[10:], d[:490])  # row r draws with counter + r


def test_rows_with_their_own_logits(cuda):
    V, rows = 1000, 300
    logits = np.full((rows, V), -1e30, dtype=np.float32)
    want = (np.arange(rows) * 7) % V
    logits[np.arange(rows), want] = 0.0
    toks = sample(cuda, logits, rows, 0.8, ld=V)
    assert np.array_equal(toks, want)


def test_batched_engine_sampling_matches_the_sampler(cuda):
    """Temperature sampling fused into the batched engine's argmax
    (infernt_batch_engine_set_sampling) draws, for every sequence and step,
    exactly the token infernt_sample_tokens draws from the same logits row
    with counter = the sequence's position; temperature 0 is greedy again."""
    cfg = ib.ModelConfig(vocab_size=1024, hidden_size=512, num_layers=2, num_attention_heads=8,
                         num_key_value_heads=2, intermediate_size=1024, max_seq_len=256,
                         weight_dtype=ib.DTYPE_BF16)
    eng = ib.BatchEngine(cfg, 4, seed=3)
    positions = [0, 10, 40, 100]
    for b, p in enumerate(positions):
        eng.fill_kv(b, 50 + b, p)
    tokens = [5, 6, 7, 8]
    temp, seed = 0.8, 21
    eng.set_sampling(temp, seed)
    differs = 0
    for _ in range(4):
        nxt = eng.step(tokens, positions)
        logits = eng.logits()
        for b in range(4):
            want = int(sample(cuda, logits[b], 1, temp, seed=seed, counter=positions[b])[0])
            assert nxt[b] == want, (b, nxt[b], want)
            differs += int(nxt[b] != int(np.argmax(logits[b])))
        tokens, positions = nxt, [p + 1 for p in positions]
    assert differs > 0  # at this temperature some draws are not the greedy token
    eng.set_sampling(0.0)
    nxt = eng.step(tokens, positions)
    logits = eng.logits()
    assert nxt == [int(np.argmax(logits[b])) for b in range(4)]
    eng.close()


STEP_CFG = ib.ModelConfig(vocab_size=1000, hidden_size=512, num_layers=2, num_attention_heads=8,
                          num_key_value_heads=2, intermediate_size=1536, max_seq_len=128)


@pytest.mark.parametrize("temperature", [0.5, 1.0, 2.0])
def test_step_sampling_inside_the_decode_kernel(cuda, temperature):
    """With a step temperature, the persistent decode kernel's LM-head phase
    draws the token itself (Gumbel-max over the logits it computes): the
    token forward_token returns equals infernt_sample_tokens on the same
    logits with (seed 1337, counter = position), and sample_next_token at
    that temperature returns it without another kernel.  The logits are the
    raw values; at temperature 0 the step is greedy again."""
    eng = ib.Engine(STEP_CFG, seed=31)
    assert eng.mode == ib.MODE_PERSISTENT
    eng.set_step_temperature(temperature)
    tok, drawn = 7, 0
    for pos in range(12):
        got = eng.forward_token(tok, pos)
        logits = eng.logits()
        want = int(sample(cuda, logits, 1, temperature, seed=1337, counter=pos)[0])
        assert got == want, (pos, got, want)
        assert eng.sample_next_token(temperature) == got
        drawn += int(got != int(np.argmax(logits)))
        tok = got
    assert drawn > 0  # some steps drew a token other than the argmax
    eng.set_step_temperature(0.0)
    got = eng.forward_token(tok, 12)
    assert got == int(np.argmax(eng.logits()))
    eng.close()


def test_sample_next_token_draws_on_the_gpu_by_default(cuda):
    """Without a step temperature the step is greedy and sample_next_token(T)
    draws with one kernel over the step's logits (seed 1337, counter =
    position); sample_next_token(0) is the greedy token."""
    eng = ib.Engine(STEP_CFG, seed=32)
    greedy = eng.forward_token(11, 0)
    logits = eng.logits()
    assert greedy == int(np.argmax(logits))
    assert eng.sample_next_token(0.0) == greedy
    assert eng.sample_next_token(1.5) == int(sample(cuda, logits, 1, 1.5, seed=1337, counter=0)[0])
    eng.set_step_temperature(1.5)
    drawn = eng.forward_token(11, 0)
    assert eng.sample_next_token(0.0) == greedy  # greedy from the same logits
    assert drawn == int(sample(cuda, eng.logits(), 1, 1.5, seed=1337, counter=0)[0])
    eng.close()
