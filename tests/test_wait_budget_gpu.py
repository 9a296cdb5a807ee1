"""Failure detection inside the persistent decode kernel, without a GPU
fault: every wait in the kernel has a time budget, after which it sets the
wait-timeout bit of the plan's error word and the launch returns.

Rank 0 of a two-rank tensor-parallel plan runs alone on one GPU: the other
rank's exchange region is a zeroed buffer that nothing ever writes, so the
first phase that needs the other rank's partial rows (the gate/up input
after the O all-reduce) waits for words that never arrive.  With a 20 ms
budget the call must report INFERNT_ERR_DEVICE quickly, and the CUDA
context must stay usable: a single-GPU engine then decodes like the
oracle."""
import time

import numpy as np
import pytest

import infernt_b200 as ib
import oracle as O

pytestmark = pytest.mark.gpu

CFG = ib.ModelConfig(vocab_size=1000, hidden_size=1024, num_layers=2, num_attention_heads=8,
                     num_key_value_heads=2, intermediate_size=2048, max_seq_len=64)


def test_missing_tp_peer_times_out_within_budget_and_context_survives(cuda):
    torch = cuda
    eng = ib.TPEngine(CFG, 0, 2, seed=3)
    own, nbytes = eng.xchg_region()
    # the absent rank's region: nothing ever writes it, so its tags never match
    absent = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    eng.set_peer_regions([own, absent.data_ptr()])
    eng.set_wait_budget(20000)
    t0 = time.perf_counter()
    with pytest.raises(ib.InferntError) as info:
        eng.forward_token(5, 0)
    elapsed = time.perf_counter() - t0
    assert info.value.status == 5, info.value  # INFERNT_ERR_DEVICE
    assert "wait timeout" in str(info.value) or "0x1" in str(info.value)
    assert elapsed < 5.0, elapsed
    # the error word was cleared by the report: the same failure reports again
    with pytest.raises(ib.InferntError):
        eng.forward_token(5, 1)
    eng.close()
    del absent
    torch.cuda.synchronize()

    # a fresh single-GPU engine on the same context decodes like the oracle
    e1 = ib.Engine(CFG, seed=4)
    orc = O.LlamaOracle(CFG, seed=4)
    tok = 17
    for pos in range(3):
        mine = e1.forward_token(tok, pos)
        want, logits = orc.decode_token(tok, pos)
        err = float(np.abs(e1.logits() - logits).max())
        assert err <= 1e-3 and err / float(np.abs(logits).max()) <= 1e-4, (pos, err)
        assert mine == want
        tok = want
    e1.close()


def test_wait_budget_is_validated():
    eng = ib.TPEngine(CFG, 0, 1, seed=3)
    with pytest.raises(ib.InferntError):
        eng.set_wait_budget(0)
    eng.close()


def test_stream_depth_changes_no_result():
    """The in-flight limit of the weight stream only reorders bulk copies in
    time: every setting decodes the same tokens and the same logits bits."""
    eng = ib.TPEngine(CFG, 0, 1, seed=5)
    depth, ring = eng.stream_depth()
    assert 1 <= depth <= ring
    runs = []
    for d in (0, 1, 3, ring):
        eng.set_stream_depth(d)
        assert eng.stream_depth()[0] == (ring if d == 0 else d)
        toks, _ = eng.decode_chain(7, 0, 12)
        runs.append((toks, eng.logits().tobytes()))
    assert all(r == runs[0] for r in runs), [r[0] for r in runs]
    with pytest.raises(ib.InferntError):
        eng.set_stream_depth(-1)
    eng.close()
