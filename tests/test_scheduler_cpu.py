"""Continuous-batching scheduler (infernt_scheduler_*, host logic) driven by a
fake paged model on the host.

The fake model keeps a page pool [num_pages][page_size] of token values and
writes every fed token at (its slot's page for the position, row position
mod page_size), exactly where the paged engine writes K/V rows; its next
token is a hash of the whole context READ BACK THROUGH THE BLOCK TABLE.  A
scheduler that hands out a page twice, frees a live page, loses rows on
preemption or feeds a wrong token or position therefore changes the
outputs, which are compared with each request decoded alone (greedy over
the same hash: the reference's generate loop, src/engine.cpp:106-170, one
request at a time)."""
import random

import numpy as np
import pytest

import infernt_b200 as ib

V = 97


def next_token(context):
    h = 0
    for i, t in enumerate(context):
        h = (h * 31 + int(t) * (i + 7) + 3) % 1000003
    return h % V


def solo(prompt, max_new, eos=-1):
    ctx = list(prompt)
    out = []
    while len(out) < max_new:
        t = next_token(ctx)
        out.append(t)
        ctx.append(t)
        if t == eos:
            break
    return out


class FakePagedModel:
    def __init__(self, slots, page_size, num_pages):
        self.P = page_size
        self.pool = np.full((num_pages, page_size), -1, dtype=np.int64)
        self.table = [[] for _ in range(slots)]

    def apply(self, plan):
        for s in plan["changed"]:
            self.table[s] = list(plan["pages"][s])

    def write(self, slot, pos, tok):
        self.pool[self.table[slot][pos // self.P], pos % self.P] = tok

    def context(self, slot, n):
        return [self.pool[self.table[slot][p // self.P], p % self.P] for p in range(n)]

    def prefill(self, slot, tokens):
        for p, t in enumerate(tokens):
            self.write(slot, p, t)
        return next_token(self.context(slot, len(tokens)))

    def decode(self, slot, tok, pos):
        self.write(slot, pos, tok)
        return next_token(self.context(slot, pos + 1))


def check_plan(plan, num_pages, page_size):
    live = [pg for s, pages in enumerate(plan["pages"]) for pg in pages]
    assert len(live) == len(set(live)), "a page is held by two slots"
    assert all(0 <= pg < num_pages for pg in live)
    prefill_slots = {s for s, _ in plan["prefill"]}
    for s, pos in enumerate(plan["positions"]):
        if pos >= 0:
            assert s not in prefill_slots
            assert len(plan["pages"][s]) > pos // page_size, "decode position without a page"
    for s, toks in plan["prefill"]:
        assert len(plan["pages"][s]) > len(toks) // page_size


def drive(sched, model, num_pages, page_size, max_steps=10000):
    for _ in range(max_steps):
        st = sched.stats()
        if st["waiting"] == 0 and st["running"] == 0:
            return
        plan = sched.plan()
        check_plan(plan, num_pages, page_size)
        model.apply(plan)
        pf = [model.prefill(s, toks) for s, toks in plan["prefill"]]
        nxt = [0] * sched.slots
        for s, (tok, pos) in enumerate(zip(plan["tokens"], plan["positions"])):
            if pos >= 0:
                nxt[s] = model.decode(s, tok, pos)
        sched.commit(pf, nxt)
    raise AssertionError("requests did not finish")


def workload(seed, n, max_len, max_total):
    rng = random.Random(seed)
    reqs = []
    for _ in range(n):
        plen = rng.randint(1, max_len)
        new = rng.randint(1, max(1, min(max_len, max_total - plen)))
        eos = rng.randrange(V) if rng.random() < 0.3 else -1
        reqs.append(([rng.randrange(V) for _ in range(plen)], new, eos))
    return reqs


@pytest.mark.parametrize("slots,page_size,num_pages", [(3, 4, 10), (4, 1, 40), (2, 16, 4), (5, 3, 64)])
def test_outputs_match_solo_runs(slots, page_size, num_pages):
    max_seq = 64
    most = num_pages * page_size  # positions the pool can hold
    reqs = workload(slots * 100 + page_size, 14, 20, min(max_seq, most))
    sched = ib.Scheduler(slots, page_size, num_pages, max_seq)
    model = FakePagedModel(slots, page_size, num_pages)
    ids = [sched.submit(p, n, eos) for p, n, eos in reqs]
    drive(sched, model, num_pages, page_size)
    for rid, (p, n, eos) in zip(ids, reqs):
        out, state, _ = sched.result(rid)
        assert state == "finished"
        assert out == solo(p, n, eos), rid
    st = sched.stats()
    assert st["free_pages"] == num_pages and st["finished"] == len(reqs)
    # every token comes from a decode position or a prefill (one per
    # admission: the first, and one after each preemption)
    assert st["decode_tokens"] + len(reqs) + st["preemptions"] == sum(len(sched.result(r)[0]) for r in ids)


def test_preemption_recomputes_and_keeps_outputs():
    """A pool too small for every running request: the youngest are
    preempted (their generated tokens kept) and finish after recomputation."""
    slots, P, pages = 4, 4, 12
    reqs = [([(7 * i + j) % V for j in range(10)], 30, -1) for i in range(6)]
    sched = ib.Scheduler(slots, P, pages, 64)
    model = FakePagedModel(slots, P, pages)
    ids = [sched.submit(p, n, eos) for p, n, eos in reqs]
    drive(sched, model, pages, P)
    st = sched.stats()
    assert st["preemptions"] > 0
    pre = [sched.result(r)[2] for r in ids]
    assert pre[0] == 0, "the oldest request is never preempted"
    assert sum(pre) == st["preemptions"]
    for rid, (p, n, eos) in zip(ids, reqs):
        assert sched.result(rid)[0] == solo(p, n, eos)
    # recomputation re-prefills prompt + generated tokens
    assert st["prefill_tokens"] > sum(len(p) for p, _, _ in reqs)


def test_first_come_first_served():
    sched = ib.Scheduler(1, 8, 8, 64)
    model = FakePagedModel(1, 8, 8)
    ids = [sched.submit([i + 1, i + 2], 3) for i in range(4)]
    order = []
    for _ in range(100):
        if sched.stats()["running"] == 0 and sched.stats()["waiting"] == 0:
            break
        plan = sched.plan()
        model.apply(plan)
        for s, toks in plan["prefill"]:
            order.append(toks[:2])
        pf = [model.prefill(s, toks) for s, toks in plan["prefill"]]
        nxt = [model.decode(s, t, p) if p >= 0 else 0
               for s, (t, p) in enumerate(zip(plan["tokens"], plan["positions"]))]
        sched.commit(pf, nxt)
    assert order == [[i + 1, i + 2] for i in range(4)]
    assert all(sched.result(r)[1] == "finished" for r in ids)


def test_eos_finishes_early_and_is_included():
    p = [3, 1, 4, 1, 5]
    ref = solo(p, 20)
    eos = ref[4]
    want = solo(p, 20, eos)
    assert want[-1] == eos and len(want) <= 5
    sched = ib.Scheduler(2, 4, 16, 64)
    rid = sched.submit(p, 20, eos)
    drive(sched, FakePagedModel(2, 4, 16), 16, 4)
    assert sched.result(rid)[0] == want


def test_cancel_frees_pages():
    sched = ib.Scheduler(2, 4, 8, 64)
    model = FakePagedModel(2, 4, 8)
    a = sched.submit([1, 2, 3], 10)
    b = sched.submit([4, 5, 6], 10)
    c = sched.submit([7, 8, 9], 10)
    plan = sched.plan()
    model.apply(plan)
    sched.commit([model.prefill(s, t) for s, t in plan["prefill"]], [0, 0])
    sched.cancel(a)  # running
    sched.cancel(c)  # waiting
    assert sched.result(a)[1] == "cancelled" and sched.result(c)[1] == "cancelled"
    drive(sched, model, 8, 4)
    assert sched.result(b)[0] == solo([4, 5, 6], 10)
    assert sched.stats()["free_pages"] == 8
    sched.release(a)
    with pytest.raises(ib.InferntError):
        sched.result(a)


def test_bad_requests_and_call_order():
    sched = ib.Scheduler(2, 4, 4, 32)
    with pytest.raises(ib.InferntError):
        sched.submit([1] * 30, 3)  # passes max_seq_len
    with pytest.raises(ib.InferntError):
        sched.submit([1] * 14, 4)  # 17 positions need 5 pages of 4; the pool has 4
    with pytest.raises(ib.InferntError):
        sched.submit([1, 2], 0)
    with pytest.raises(ib.InferntError):
        sched.submit([1, -2], 3)
    rid = sched.submit([1, 2], 3)
    sched.plan()
    with pytest.raises(ib.InferntError):
        sched.plan()  # the plan awaits its commit
    with pytest.raises(ib.InferntError):
        sched.release(rid)  # still running
