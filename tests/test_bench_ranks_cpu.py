"""The N > 1 host logic of bench.py on CPU: two gloo ranks (one process
each, as torchrun starts them) report different step times; every rank gets
the slowest rank's time, and the job throughput counts every rank's tokens
over that time."""
import os
import socket

import pytest
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out):
    import datetime
    import torch
    import torch.distributed as dist
    import bench
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        ms = 10.0 + 5.0 * rank  # rank 1 is the slow one
        ms_max = bench.max_over_ranks(torch, ms, "cpu")
        out[rank] = (ms_max, bench.job_tokens_per_s(world, 64, ms_max))
    finally:
        dist.destroy_process_group()


def test_max_over_ranks_and_job_throughput_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        out = mgr.dict()
        port = _free_port()
        procs = [ctx.Process(target=_rank, args=(r, 2, port, out)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(120)
            assert p.exitcode == 0
        res = dict(out)
    for r in range(2):
        ms_max, value = res[r]
        assert ms_max == 15.0
        assert value == pytest.approx(2 * 64 / 0.015)


def test_single_process_is_identity():
    import torch
    import bench
    assert bench.max_over_ranks(torch, 3.5, "cpu") == 3.5
    assert bench.job_tokens_per_s(1, 100, 250.0) == pytest.approx(400.0)


def test_prefill_flops_counts_projections_attention_and_lm_head():
    """The prefill bench's algorithmic FLOPs: 2 per weight element per token
    for every projection, 4 * Nq * D per (query, visible key) for the causal
    attention of every layer, and the LM head of the last token; checked
    against a direct count over tokens and keys."""
    import bench
    import infernt_b200 as ib
    cfg = ib.ModelConfig(vocab_size=96, hidden_size=64, num_layers=3, num_attention_heads=4,
                         num_key_value_heads=2, intermediate_size=80, max_seq_len=64)
    for n, start in ((1, 0), (7, 0), (5, 11)):
        total, proj, attn = bench.prefill_flops(cfg, n, start)
        H, D, I, L = 64, 16, 80, 3
        per_token = 0
        for (rows, cols) in ((4 * D + 2 * 2 * D, H), (H, 4 * D), (2 * I, H), (H, I)):
            per_token += 2 * rows * cols
        want_proj = n * L * per_token
        want_attn = sum(4 * 4 * D * (start + t + 1) * L for t in range(n))
        assert proj == want_proj and attn == want_attn
        assert total == want_proj + want_attn + 2 * 96 * H
