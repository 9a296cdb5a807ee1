"""Paged KV caches and continuous batching on the GPU.

The paged engine (infernt_batch_engine_create_paged) runs the batched
engine's kernels with every cache row addressed through a block table, so
against the contiguous engine of the same seed its logits, tokens and cache
rows are equal bit for bit, whatever pages a sequence holds (shuffled pool
order, page sizes that do not divide the attention's 32-position tiles).
Empty slots (position -1) leave the other sequences' results and their own
pages untouched.

The server (infernt_server_*) is checked two ways: a request's tokens equal
those of the same request served alone (bit for bit: the decode step's rows
do not interact, and prefill is per sequence) unless it was preempted and
recomputed; and every token is checked teacher-forced against the CPU oracle
(bf16-rounded weights and activations): the oracle's greedy token given the
request's previous tokens, unless the oracle's top-2 gap is below 1e-2 of
its largest |logit| (the batched tests' bound on the logit error)."""
import random

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


def pools(cfg, T, page_size, spare=3, seed=0):
    """Shuffled disjoint pages covering every sequence's whole max_seq_len."""
    mp = -(-cfg.max_seq_len // page_size)
    n = T * mp + spare
    perm = list(range(n))
    random.Random(seed + page_size).shuffle(perm)
    return n, [perm[t * mp:(t + 1) * mp] for t in range(T)]


@pytest.mark.parametrize("cfg,page_size", [(CFG, 16), (CFG, 32), (CFG, 48), (CFG, 1), (CFG, 256),
                                           (CFG_D128, 32), (CFG_D128, 80)])
def test_paged_decode_equals_contiguous(cfg, page_size):
    n_pos = [0, 3, 40, 65, 130]
    T, steps = len(n_pos), 4
    n_pages, tables = pools(cfg, T, page_size)
    flat = ib.BatchEngine(cfg, T, seed=5)
    paged = ib.BatchEngine(cfg, T, seed=5, pages=(page_size, n_pages))
    assert paged.paging() == (page_size, n_pages, -(-cfg.max_seq_len // page_size))
    for t in range(T):
        paged.set_pages(t, tables[t])
        flat.fill_kv(t, 100 + t, n_pos[t])
        paged.fill_kv(t, 100 + t, n_pos[t])
    tokens = [int(x) for x in O.prompt(T, 5, 3, cfg.vocab_size)]
    positions = list(n_pos)
    for _ in range(steps):
        a = flat.step(tokens, positions)
        b = paged.step(tokens, positions)
        assert a == b
        assert np.array_equal(flat.logits(), paged.logits())
        tokens = a
        positions = [p + 1 for p in positions]
    for t in range(T):
        for layer in range(cfg.num_layers):
            k1, v1 = flat.read_kv(t, layer, positions[t])
            k2, v2 = paged.read_kv(t, layer, positions[t])
            assert np.array_equal(k1, k2) and np.array_equal(v1, v2), (t, layer)
    # chained steps on the device
    toks1, _ = flat.decode(tokens, positions, 3)
    toks2, _ = paged.decode(tokens, positions, 3)
    assert np.array_equal(toks1, toks2)
    flat.close()
    paged.close()


def test_empty_slots_leave_the_others_unchanged():
    n_pos = [10, 50, 90, 130]
    T, P = len(n_pos), 32
    n_pages, tables = pools(CFG, T, P)
    full = ib.BatchEngine(CFG, T, seed=7, pages=(P, n_pages))
    part = ib.BatchEngine(CFG, T, seed=7, pages=(P, n_pages))
    for e in (full, part):
        for t in range(T):
            e.set_pages(t, tables[t])
            e.fill_kv(t, 200 + t, n_pos[t])
    tokens = [int(x) for x in O.prompt(T, 7, 3, CFG.vocab_size)]
    before = [part.read_kv(t, 0, n_pos[t] + 2) for t in (1, 3)]
    positions = list(n_pos)
    empty = [n_pos[0], -1, n_pos[2], -1]
    for _ in range(2):
        a = full.step(tokens, positions)
        b = part.step(tokens, empty)
        la, lb = full.logits(), part.logits()
        for t in (0, 2):
            assert a[t] == b[t]
            assert np.array_equal(la[t], lb[t])
        tokens = a
        positions = [p + 1 for p in positions]
        empty = [p + 1 if p >= 0 else -1 for p in empty]
    after = [part.read_kv(t, 0, n_pos[t] + 2) for t in (1, 3)]
    for (k0, v0), (k1, v1) in zip(before, after):
        assert np.array_equal(k0, k1) and np.array_equal(v0, v1)
    full.close()
    part.close()


def test_step_without_a_page_is_refused_on_the_host():
    P = 16
    e = ib.BatchEngine(CFG, 2, seed=1, pages=(P, 8))
    e.set_pages(0, [3])
    e.set_pages(1, [5, 6])
    e.fill_kv(0, 1, 10)
    e.fill_kv(1, 1, 20)
    e.step([1, 2], [10, 20])  # positions 10 and 20 have pages
    with pytest.raises(ib.InferntError):
        e.step([1, 2], [P, 20])  # position 16 of sequence 0 has none
    with pytest.raises(ib.InferntError):
        e.set_pages(0, [8])  # outside the pool
    e.step([1, 2], [-1, 21])
    e.close()


@pytest.mark.parametrize("page_size", [16, 24])
def test_paged_prefill_equals_contiguous(page_size):
    T = 3
    n_pages, tables = pools(CFG, T, page_size)
    flat = ib.BatchEngine(CFG, T, seed=9)
    paged = ib.BatchEngine(CFG, T, seed=9, pages=(page_size, n_pages))
    for t in range(T):
        paged.set_pages(t, tables[t])
    toks = [int(x) for x in O.prompt(70, 9, 3, CFG.vocab_size)]
    # a whole prompt, and a prompt continued from position 33
    for e in (flat, paged):
        e.fill_kv(0, 11, 0)
    a = flat.prefill(1, toks, want_logits=True)
    b = paged.prefill(1, toks, want_logits=True)
    assert a[0] == b[0] and np.array_equal(a[1], b[1])
    a0 = flat.prefill(2, toks[:33], chunk=16)
    b0 = paged.prefill(2, toks[:33], chunk=16)
    assert a0[0] == b0[0]
    a1 = flat.prefill(2, toks[33:], start_pos=33, chunk=16, want_logits=True)
    b1 = paged.prefill(2, toks[33:], start_pos=33, chunk=16, want_logits=True)
    assert a1[0] == b1[0] and np.array_equal(a1[1], b1[1])
    for t, n in ((1, 70), (2, 70)):
        for layer in range(CFG.num_layers):
            k1, v1 = flat.read_kv(t, layer, n)
            k2, v2 = paged.read_kv(t, layer, n)
            assert np.array_equal(k1, k2) and np.array_equal(v1, v2), (t, layer)
    # decode after the prefill
    tokens, positions = [0, a[0], a1[0]], [-1, 70, 70]
    flat_pos = [0, 70, 70]
    x = flat.step(tokens, flat_pos)
    y = paged.step(tokens, positions)
    assert x[1:] == y[1:]
    assert np.array_equal(flat.logits()[1:], paged.logits()[1:])
    flat.close()
    paged.close()


def top2_gap(x):
    s = np.sort(x)
    return float(s[-1] - s[-2])


def teacher_forced(cfg, seed, prompt, out):
    """Each generated token against the oracle's greedy token after the
    request's own previous tokens (near ties allowed)."""
    o = O.LlamaOracle(cfg, seed=seed, round_bf16=True, act_bf16=True)
    ctx = list(prompt)
    for pos, tok in enumerate(ctx[:-1]):
        o.decode_token(tok, pos)
    for i, got in enumerate(out):
        want, logits = o.decode_token(ctx[-1], len(ctx) - 1)
        if got != want:
            assert top2_gap(logits) < 1e-2 * float(np.abs(logits).max()), (i, got, want)
        ctx.append(got)


def requests(n, seed, vocab):
    rng = random.Random(seed)
    out = []
    for _ in range(n):
        plen = rng.randint(3, 60)
        out.append(([rng.randrange(3, vocab) for _ in range(plen)], rng.randint(4, 24)))
    return out


def test_server_continuous_batching_matches_solo_and_oracle():
    seed, slots, P = 5, 4, 16
    reqs = requests(10, 1, CFG.vocab_size)
    srv = ib.Server(CFG, slots, P, 9, seed=seed)  # 9 pages: four running requests overflow them
    ids = [srv.submit(p, n) for p, n in reqs]
    srv.run()
    st = srv.stats()
    assert st["finished"] == len(reqs) and st["free_pages"] == 9
    assert st["preemptions"] > 0
    results = [srv.result(r) for r in ids]
    srv.close()
    solo = ib.Server(CFG, slots, P, 64, seed=seed)
    for (p, n), (out, state, pre) in zip(reqs, results):
        assert state == "finished" and len(out) == n
        rid = solo.submit(p, n)
        solo.run()
        alone, _, _ = solo.result(rid)
        if pre == 0:
            assert out == alone, (p, out, alone)
        teacher_forced(CFG, seed, p, out)
    solo.close()


def test_server_eos_and_sampling_keys_per_request():
    srv = ib.Server(CFG, 3, 16, 32, seed=2)
    p = [int(x) for x in O.prompt(12, 3, 3, CFG.vocab_size)]
    rid = srv.submit(p, 16)
    srv.run()
    greedy, _, _ = srv.result(rid)
    eos = greedy[5]
    rid = srv.submit(p, 16, eos)
    srv.run()
    out, _, _ = srv.result(rid)
    assert out == greedy[:greedy.index(eos) + 1]
    # temperature draws: the same prompt in two slots draws independent
    # tokens (keys carry the request id), and a new server repeats them
    srv.set_sampling(1.0, seed=11)
    a, b = srv.submit(p, 16), srv.submit(p, 16)
    srv.run()
    ta, tb = srv.result(a)[0], srv.result(b)[0]
    assert ta != tb
    srv.close()
    again = ib.Server(CFG, 3, 16, 32, seed=2)
    for _ in range(2):
        again.submit(p, 1)
    again.run()
    again.set_sampling(1.0, seed=11)
    a2, b2 = again.submit(p, 16), again.submit(p, 16)
    again.run()
    # request ids 3 and 4 on both servers
    assert (a2, b2) == (a, b)
    assert again.result(a2)[0] == ta and again.result(b2)[0] == tb
    again.close()
