"""Attention of a batch of decoding sequences over bf16 KV caches
(infernt_batch_attention: the batched engine's partial and merge kernels)
against a float64 PyTorch restatement of cuda/attention.cu:9-42 (scores
q.k / sqrt(D) over positions [0, pos], softmax, weighted sum of values) on
the same bf16 cache values and FP32 queries.

The tensor-core partials take the FP32 queries and probabilities as three
bf16 terms (24 mantissa bits) and accumulate in FP32, so the FP32 output
must agree with float64 to FP32 rounding: max-abs error <= 1e-5 of the
largest |output|.  The bf16 output must be the round-to-nearest-even of
the FP32 output, bit for bit."""
import math

import numpy as np
import pytest

import infernt_b200 as ib

pytestmark = pytest.mark.gpu


def _torch():
    import torch
    return torch


def run_attention(positions, nq, nkv, D, max_seq, splits, min_chunk, stages, q_scale=1.0, seed=0):
    torch = _torch()
    T = len(positions)
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn(T, nq, D, device="cuda", generator=g) * q_scale
    kc = torch.randn(T, nkv, max_seq, D, device="cuda", generator=g).to(torch.bfloat16)
    vc = torch.randn(T, nkv, max_seq, D, device="cuda", generator=g).to(torch.bfloat16)
    pos = torch.tensor(positions, dtype=torch.int32, device="cuda")
    G = nq // nkv
    part = torch.full((T * nkv * splits * G * (D + 2),), float("nan"), device="cuda")
    attn = torch.zeros(T, nq, D, dtype=torch.bfloat16, device="cuda")
    attn32 = torch.full((T, nq, D), float("nan"), device="cuda")
    ib.call("infernt_batch_attention", q.data_ptr(), kc.data_ptr(), vc.data_ptr(), pos.data_ptr(), T, nq, nkv, D,
            max_seq, splits, min_chunk, stages, part.data_ptr(), attn.data_ptr(), attn32.data_ptr(),
            torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    want = torch.empty(T, nq, D, dtype=torch.float64, device="cuda")
    for t, p in enumerate(positions):
        k = kc[t, :, :p + 1].double()                      # [nkv][n][D]
        v = vc[t, :, :p + 1].double()
        qq = q[t].double().view(nkv, G, D)
        s = torch.einsum("hgd,hnd->hgn", qq, k) / math.sqrt(D)
        w = torch.softmax(s, dim=-1)
        want[t] = torch.einsum("hgn,hnd->hgd", w, v).reshape(nq, D)
    return attn, attn32, want


def check(positions, nq, nkv, D, splits, min_chunk, stages, max_seq=2112, q_scale=1.0):
    attn, attn32, want = run_attention(positions, nq, nkv, D, max_seq, splits, min_chunk, stages, q_scale)
    err = float((attn32.double() - want).abs().max())
    scale = float(want.abs().max())
    assert err <= 1e-5 * scale, (err, scale)
    assert bool(attn.eq(attn32.to(_torch().bfloat16)).all())


RAGGED = [0, 1, 30, 31, 32, 33, 63, 64, 65, 127, 128, 129, 200, 511]


@pytest.mark.parametrize("splits,min_chunk,stages", [
    (1, 64, 2), (2, 64, 3), (3, 64, 4), (5, 32, 4), (8, 256, 2), (64, 1, 3),
])
def test_tinyllama_heads(splits, min_chunk, stages):
    """32 query heads on 4 KV heads, D = 64: ragged contexts around the
    32-position tiles and several work splits."""
    check(RAGGED, 32, 4, 64, splits, min_chunk, stages)


def test_long_contexts_tinyllama_heads():
    rng = np.random.default_rng(7)
    check([int(x) for x in rng.integers(512, 2049, size=12)], 32, 4, 64, 2, 64, 3)


@pytest.mark.parametrize("stages", [2, 3])
def test_head_dim_128(stages):
    """The 8B layout: 32 query heads on 8 KV heads, D = 128."""
    check(RAGGED[:10] + [1000, 2047], 32, 8, 128, 3, 64, stages)


@pytest.mark.parametrize("nq,nkv", [(8, 8), (8, 4), (12, 4), (16, 4), (32, 2)])
def test_group_sizes(nq, nkv):
    """1, 2, 3, 4 and 16 query heads per KV head (16: the CUDA-core
    partials)."""
    check([0, 40, 97, 300], nq, nkv, 64, 3, 64, 3)


@pytest.mark.parametrize("splits,stages", [(1, 2), (4, 3)])
def test_long_contexts_8b_heads(splits, stages):
    """The long-context decode layout: 32 query heads on 8 KV heads, D = 128,
    contexts up to the 32768-position cache."""
    check([32767, 20000, 5], 32, 8, 128, splits, 64, stages, max_seq=32768)


def test_peaked_scores():
    """Queries scaled by 8: scores spread over about +-60, so the softmax is
    dominated by a few positions and the running maxima change often."""
    check(RAGGED, 32, 4, 64, 3, 64, 3, q_scale=8.0)


def test_rejects_bad_arguments():
    torch = _torch()
    z = torch.zeros(4096, device="cuda")
    zi = torch.zeros(4, dtype=torch.int32, device="cuda")
    for args in [(1, 32, 4, 64, 0, 64, 3),     # no splits
                 (1, 32, 4, 64, 2, 64, 5),     # too many stages at D = 64
                 (1, 32, 4, 96, 2, 64, 3),     # head_dim 96
                 (1, 48, 4, 64, 2, 64, 3)]:    # 12 query heads per KV head
        T, nq, nkv, D, S, mc, st = args
        with pytest.raises(ib.InferntError):
            ib.call("infernt_batch_attention", z.data_ptr(), z.data_ptr(), z.data_ptr(), zi.data_ptr(), T, nq, nkv, D,
                    16, S, mc, st, z.data_ptr(), z.data_ptr(), None, None)
