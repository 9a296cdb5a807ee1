"""Tensor-parallel batched decode (infernt_batch_engine_create_tp) against
the CPU oracle.

Each rank is a process on its own GPU (one process per GPU, as torchrun
starts them); rank 0 makes the NCCL unique id and a gloo process group
hands it to the others.  Every rank must return the same greedy tokens at
every step.  The ranks' logits slices, put together in rank order, are held
to the batched decode's own tolerance against the oracle's batched-decode
variant (test_batch_gpu.py): every (step, sequence) within 1e-2 of the
largest |logit|, tokens identical unless the oracle's top-2 gap is below
twice the error.  The shapes cover both head dims and a vocabulary whose
rank slices need zero-padded LM-head rows (1152 over 2 ranks: 576 rows,
padded to 640).  The ranks' O and down sums cross by the peer-memory
exchange (the default; every rank adds them in rank order) and by
ncclAllReduce (the baseline); both are held to the same tolerance."""
import os
import socket

import numpy as np
import pytest

import infernt_b200 as ib
import oracle as O

pytestmark = pytest.mark.gpu

CFG = ib.ModelConfig(vocab_size=1024, hidden_size=512, num_layers=2, num_attention_heads=8,
                     num_key_value_heads=2, intermediate_size=1024, max_seq_len=256, rms_norm_eps=1e-5,
                     rope_theta=10000.0, weight_dtype=ib.DTYPE_BF16)
CFG_D128 = CFG.with_(hidden_size=1024, num_attention_heads=8, num_key_value_heads=4, head_dim=128,
                     intermediate_size=1536, num_layers=1, vocab_size=1152)
N_POS, STEPS, SEED = [0, 40, 130], 3, 7


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, cfg, out, peer=True):
    import datetime
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    try:
        obj = [ib.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        T = len(N_POS)
        eng = ib.BatchEngine(cfg, T, seed=SEED, rank=rank, world=world, nccl_id=obj[0])
        if world > 1:
            eng.set_tp_exchange(peer)
        for b, p in enumerate(N_POS):
            eng.fill_kv(b, 100 + b, p)
        tokens = [int(t) for t in O.prompt(T, SEED, 3, cfg.vocab_size)]
        positions = list(N_POS)
        toks, logits = [], []
        for _ in range(STEPS):
            tokens = eng.step(tokens, positions)
            positions = [p + 1 for p in positions]
            toks.append(tokens)
            logits.append(eng.logits())
        rng = eng.vocab_range
        eng.close()
        out[rank] = (toks, logits, rng)
    finally:
        dist.destroy_process_group()


def run_tp(cfg, world, peer=True):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        out = mgr.dict()
        port = _free_port()
        procs = [ctx.Process(target=_rank, args=(r, world, port, cfg, out, peer)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(600)
        codes = [p.exitcode for p in procs]
        assert codes == [0] * world, codes
        return dict(out)


def top2_gap(x):
    s = np.sort(x)
    return float(s[-1] - s[-2])


def check_against_oracle(cfg, world, peer=True):
    res = run_tp(cfg, world, peer)
    toks = [res[r][0] for r in range(world)]
    assert all(t == toks[0] for t in toks), "ranks disagree on the greedy tokens"
    ranges = [res[r][2] for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == cfg.vocab_size
    assert all(ranges[r][1] == ranges[r + 1][0] for r in range(world - 1))
    T = len(N_POS)
    orcs = []
    for b, p in enumerate(N_POS):
        o = O.LlamaOracle(cfg, seed=SEED, round_bf16=True, act_bf16=True)
        o.fill_kv(100 + b, p)
        orcs.append(o)
    tokens = [int(t) for t in O.prompt(T, SEED, 3, cfg.vocab_size)]
    positions = list(N_POS)
    for step in range(STEPS):
        full = np.concatenate([res[r][1][step] for r in range(world)], axis=1)
        for b in range(T):
            want_tok, want = orcs[b].decode_token(tokens[b], positions[b])
            err = float(np.abs(full[b] - want).max())
            scale = float(np.abs(want).max())
            assert err <= 1e-2 * scale, (step, b, err, scale)
            got_tok = toks[0][step][b]
            assert got_tok == int(np.argmax(full[b])) or full[b][got_tok] == full[b].max(), (step, b)
            if got_tok != want_tok:
                assert top2_gap(want) < 2 * err, (step, b, got_tok, want_tok)
        tokens = toks[0][step]  # both sides follow the engine's tokens
        positions = [p + 1 for p in positions]


def _gpus():
    import torch
    return torch.cuda.device_count()


def test_batch_tp1_matches_oracle():
    """One rank through the tensor-parallel constructor: no collective."""
    check_against_oracle(CFG, 1)


@pytest.mark.skipif("_gpus() < 2", reason="needs two GPUs")
@pytest.mark.parametrize("peer", [True, False], ids=["peer-exchange", "nccl"])
def test_batch_tp2_matches_oracle(peer):
    check_against_oracle(CFG, 2, peer)


@pytest.mark.skipif("_gpus() < 2", reason="needs two GPUs")
def test_batch_tp2_head_dim_128_padded_vocab():
    check_against_oracle(CFG_D128, 2)


PF_PROMPT, PF_CHUNK, PF_STEPS = 40, 16, 3


def _prefill_rank(rank, world, port, cfg, out):
    import datetime
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    try:
        obj = [ib.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        prompt = [int(t) for t in O.prompt(PF_PROMPT, SEED + 1, 3, cfg.vocab_size)]

        def run(eng):
            tok, logits, _ = eng.prefill(0, prompt, 0, chunk=PF_CHUNK, want_logits=True)
            kv = [eng.read_kv(0, l, PF_PROMPT) for l in range(cfg.num_layers)]
            tokens, positions, toks = [tok, 11], [PF_PROMPT, 0], []
            for _ in range(PF_STEPS):
                tokens = eng.step(tokens, positions)
                positions = [p + 1 for p in positions]
                toks.append(tokens)
            return tok, logits, kv, toks

        eng = ib.BatchEngine(cfg, 2, seed=SEED, rank=rank, world=world, nccl_id=obj[0])
        res = run(eng) + (eng.vocab_range,)
        eng.close()
        dist.barrier()
        if rank == 0:
            one = ib.BatchEngine(cfg, 2, seed=SEED)
            out["one"] = run(one)
            one.close()
        out[rank] = res
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif("_gpus() < 2", reason="needs two GPUs")
@pytest.mark.parametrize("cfg", [CFG, CFG_D128], ids=["d64", "d128-padded-vocab"])
def test_batch_tp2_prefill_matches_one_gpu(cfg):
    """Prompt prefill on a two-rank engine (ncclAllReduce of each chunk's O
    and down rows) against the one-GPU engine with the same seeded weights:
    both ranks return the same next token, the ranks' logits slices and KV
    heads put together match the one-GPU prefill (layer 0's K/V rows exactly:
    no sum over ranks precedes them; later layers within the batched
    tolerance), and the decode steps that follow agree."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        out = mgr.dict()
        port = _free_port()
        procs = [ctx.Process(target=_prefill_rank, args=(r, 2, port, cfg, out)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(600)
        assert [p.exitcode for p in procs] == [0, 0]
        res = dict(out)
    tok1, logits1, kv1, toks1 = res["one"]
    assert res[0][0] == res[1][0], "ranks disagree on the prefill token"
    full = np.concatenate([res[0][1], res[1][1]])
    assert full.shape == logits1.shape
    err = float(np.abs(full - logits1).max())
    scale = float(np.abs(logits1).max())
    assert err <= 1e-2 * scale, (err, scale)
    if res[0][0] != tok1:
        assert top2_gap(logits1) < 2 * err, (res[0][0], tok1)
    nkv_l = cfg.num_key_value_heads // 2
    for l in range(cfg.num_layers):
        for which in (0, 1):  # K, V
            mine = np.concatenate([res[r][2][l][which] for r in range(2)])
            want = kv1[l][which]
            if l == 0:
                np.testing.assert_array_equal(mine, want)
            else:
                assert float(np.abs(mine - want).max()) <= 2e-2 * float(np.abs(want).max()), (l, which)
        assert res[0][2][l][0].shape[0] == nkv_l
    assert res[0][3] == res[1][3], "ranks disagree on the decode tokens"
    agree = sum(a == b for s, t in zip(res[0][3], toks1) for a, b in zip(s, t))
    assert agree >= len(toks1) * 2 - 1, (res[0][3], toks1)
