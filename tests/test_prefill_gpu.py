"""Prompt prefill on the tensor cores: the chunk projections
(infernt_pgemm_bf16), the causal attention of a chunk
(infernt_prefill_attention) and the batched engine's prefill
(infernt_batch_engine_prefill), which replaces the reference's sequential
single-token forwards over the prompt (src/engine.cpp:124-126).

Tolerances, stated per check:
- pgemm against a PyTorch FP32 matmul of the same bf16 operands: one FP32
  accumulation over K per element in another order, so max-abs error <=
  2e-5 of the largest |Y| plus 1e-6.
- prefill attention against a float64 restatement of causal GQA attention on
  the same bf16 q, K and V: the probabilities enter the tensor cores as bf16
  (each within 2^-9 relative, moving the output by at most 2^-9 of the
  largest |V| of the head) and the output is rounded to bf16 (2^-9 of |O| <=
  the largest |V|), so max-abs error <= 2^-8 of the largest |V| of the head.
- the engine's prefill against the CPU oracle's batched-decode variant
  (bf16-rounded weights, activations into projections and K/V rows) run
  token by token over the same prompt.  On top of the bf16 rounding flips
  that the batched decode test allows (within 1e-2 of the largest |logit|),
  the prefill rounds queries and probabilities to bf16 inside the
  attention; the same bounds hold: last-token logits within 1e-2 of the
  largest |logit|, the greedy token identical unless the oracle's top-2 gap
  is below twice the error, every layer's K and V rows within 2e-2 of their
  largest magnitude; then decode steps from the prefilled caches as in
  test_batch_gpu.py."""
import math

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
CFG_G8 = CFG.with_(hidden_size=1024, num_attention_heads=16, num_key_value_heads=2, head_dim=64)


def _torch():
    import torch
    return torch


def _stream():
    return _torch().cuda.current_stream().cuda_stream


@pytest.mark.parametrize("N,K,T,ldy", [
    (128, 64, 1, 128),        # one tile, one stage, one token
    (256, 512, 37, 256),      # token tile of 48
    (384, 1024, 300, 384),    # two token tiles, the second ragged
    (640, 512, 513, 640),     # three token tiles, one token in the last
    (1024, 2048, 1000, 1024),
    (256, 512, 100, 384),     # padded output rows: columns past N untouched
])
def test_pgemm_matches_torch(N, K, T, ldy):
    torch = _torch()
    g = torch.Generator(device="cuda").manual_seed(N + K + T)
    W = (torch.randn(N, K, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    X = torch.randn(T, K, device="cuda", generator=g).to(torch.bfloat16)
    Y = torch.full((T, ldy), float("nan"), device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    ib.call("infernt_pgemm_bf16", W.data_ptr(), N, K, X.data_ptr(), T, Y.data_ptr(), ldy, err.data_ptr(), _stream())
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    want = X.float() @ W.float().t()
    e = float((Y[:, :N] - want).abs().max())
    scale = float(want.abs().max())
    assert e <= 2e-5 * scale + 1e-6, (e, scale)
    if ldy > N:
        assert bool(torch.isnan(Y[:, N:]).all())


@pytest.mark.parametrize("I,K,T", [
    (128, 64, 1),
    (256, 512, 300),     # two token tiles, the second ragged
    (384, 2048, 513),
])
def test_pgemm_swiglu_matches_torch(I, K, T):
    """silu(g) u rounded to bf16 against PyTorch on the same bf16 operands:
    g and u differ from the FP32 matmul by summation order only (2e-5
    relative), so each output is within one bf16 step (2^-7 relative) of
    the reference value, plus 1e-6 of the largest."""
    torch = _torch()
    g = torch.Generator(device="cuda").manual_seed(I + K + T)
    W = (torch.randn(2 * I, K, device="cuda", generator=g) * 0.05).to(torch.bfloat16)
    X = torch.randn(T, K, device="cuda", generator=g).to(torch.bfloat16)
    act = torch.zeros(T, I, dtype=torch.bfloat16, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    ib.call("infernt_pgemm_swiglu_bf16", W.data_ptr(), I, K, X.data_ptr(), T, act.data_ptr(), I, err.data_ptr(),
            _stream())
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    gu = X.float() @ W.float().t()
    gt, up = gu[:, :I], gu[:, I:]
    want = gt / (1.0 + torch.exp(-gt)) * up
    got = act.float()
    tol = 2.0 ** -7 * want.abs() + 1e-6 * float(want.abs().max())
    assert bool(((got - want).abs() <= tol).all()), float((got - want).abs().max())


def test_pgemm_rejects_bad_shapes():
    torch = _torch()
    W = torch.zeros(128, 64, dtype=torch.bfloat16, device="cuda")
    X = torch.zeros(1, 64, dtype=torch.bfloat16, device="cuda")
    Y = torch.zeros(1, 128, device="cuda")
    for n, k, t, ldy in [(100, 64, 1, 128), (128, 60, 1, 128), (128, 64, 0, 128), (128, 64, 1, 64)]:
        with pytest.raises(ib.InferntError):
            ib.call("infernt_pgemm_bf16", W.data_ptr(), n, k, X.data_ptr(), t, Y.data_ptr(), ldy, None, None)


def ref_causal_attention(q, k, v, p0):
    """float64 causal GQA attention: q [C][nq][D], caches [nkv][S][D]."""
    torch = _torch()
    C, nq, D = q.shape
    nkv = k.shape[0]
    G = nq // nkv
    n = p0 + C
    out = torch.empty((C, nq, D), dtype=torch.float64, device=q.device)
    keys = torch.arange(n, device=q.device)
    pos = p0 + torch.arange(C, device=q.device)
    mask = keys[None, :] > pos[:, None]
    for h in range(nq):
        kh = h // G
        s = (q[:, h, :] @ k[kh, :n, :].t()) / math.sqrt(D)
        s = s.masked_fill(mask, float("-inf"))
        out[:, h, :] = torch.softmax(s, dim=-1) @ v[kh, :n, :]
    return out


@pytest.mark.parametrize("D,nq,nkv,C,p0,tc", [
    (64, 8, 1, 1, 0, 0),         # one token, one key
    (64, 8, 1, 100, 37, 0),      # groups of 8 (TinyLlama), ragged blocks
    (64, 4, 2, 130, 0, 0),       # groups of 2, the chunk starts the sequence
    (128, 8, 2, 65, 200, 0),     # groups of 4 (8B shape)
    (128, 4, 4, 33, 64, 0),      # one query head per KV head
    (128, 32, 8, 300, 1000, 0),  # 8B head layout, a chunk after 1000 positions
    (64, 32, 4, 257, 0, 0),      # TinyLlama head layout
    # the tensor-core kernel
    (64, 8, 1, 1, 0, 1),         # head_dim 64: one token, one key
    (64, 8, 1, 100, 37, 1),      # groups of 8 (TinyLlama), ragged blocks
    (64, 32, 4, 257, 0, 1),      # TinyLlama head layout
    (64, 4, 2, 700, 300, 1),     # groups of 2, several key tiles, diagonal tiles
    (128, 8, 2, 1, 0, 1),        # one token, one key
    (128, 8, 2, 65, 200, 1),     # groups of 4, partial last block, keys past one 128-key tile
    (128, 4, 4, 33, 64, 1),      # one query head per KV head
    (128, 8, 1, 100, 37, 1),     # groups of 8
    (128, 4, 2, 130, 0, 1),      # groups of 2, the chunk starts the sequence
    (128, 32, 8, 300, 1000, 1),  # 8B head layout, a chunk after 1000 positions
    (128, 32, 8, 1024, 3000, 1),  # many tiles per block, diagonal tiles, rows that grow late
])
def test_prefill_attention_matches_float64(D, nq, nkv, C, p0, tc):
    torch = _torch()
    S = p0 + C + 5
    g = torch.Generator(device="cuda").manual_seed(D * 7 + C + p0)
    q = torch.randn(C, nq, D, device="cuda", generator=g).to(torch.bfloat16)
    k = torch.randn(nkv, S, D, device="cuda", generator=g).to(torch.bfloat16)
    v = torch.randn(nkv, S, D, device="cuda", generator=g).to(torch.bfloat16)
    # rows past the chunk's last position must not be read
    k[:, p0 + C:, :] = float("nan")
    v[:, p0 + C:, :] = float("nan")
    attn = torch.full((C, nq, D), float("nan"), dtype=torch.bfloat16, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    ib.call("infernt_prefill_attention", q.data_ptr(), k.data_ptr(), v.data_ptr(), C, p0, nq, nkv, D, S,
            attn.data_ptr(), err.data_ptr(), tc, _stream())
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    want = ref_causal_attention(q.double(), k.double(), v.double(), p0)
    got = attn.double()
    assert not bool(torch.isnan(got).any())
    G = nq // nkv
    for h in range(nq):
        vmax = float(v[h // G, :p0 + C].double().abs().max())
        e = float((got[:, h] - want[:, h]).abs().max())
        assert e <= 2.0 ** -8 * vmax, (h, e, vmax)


def top2_gap(x):
    s = np.sort(x)
    return float(s[-1] - s[-2])


def check_prefill(cfg, n, chunk, start=0, seed=5, steps=3):
    eng = ib.BatchEngine(cfg, 1, seed=seed)
    orc = O.LlamaOracle(cfg, seed=seed, round_bf16=True, act_bf16=True)
    if start:
        eng.fill_kv(0, 77, start)
        orc.fill_kv(77, start)
    prompt = [int(t) for t in O.prompt(n, seed + n, 3, cfg.vocab_size)]
    nxt, logits, _ = eng.prefill(0, prompt, start_pos=start, chunk=chunk, want_logits=True)
    for i, tok in enumerate(prompt):
        want_tok, want = orc.decode_token(tok, start + i)
    err = float(np.abs(logits - want).max())
    scale = float(np.abs(want).max())
    assert err <= 1e-2 * scale, ("logits", err, scale)
    if nxt != want_tok:
        assert top2_gap(want) < 2 * err, ("token", nxt, want_tok)
    L, nkv, S, D = cfg.num_layers, cfg.num_key_value_heads, cfg.max_seq_len, cfg.head_dim
    ok_k = orc.kv_k.reshape(L, nkv, S, D)
    ok_v = orc.kv_v.reshape(L, nkv, S, D)
    end = start + n
    for l in range(L):
        k, v = eng.read_kv(0, l, end)
        for name, got, ref in (("K", k, ok_k[l, :, :end]), ("V", v, ok_v[l, :, :end])):
            e = float(np.abs(got - ref).max())
            assert e <= 2e-2 * float(np.abs(ref).max()), (name, l, e)
    # decode from the prefilled caches, both sides fed the engine's tokens
    tok, pos = nxt, end
    for step in range(steps):
        got_tok = eng.step([tok], [pos])[0]
        got = eng.logits()[0]
        want_tok, want = orc.decode_token(tok, pos)
        err = float(np.abs(got - want).max())
        scale = float(np.abs(want).max())
        assert err <= 1e-2 * scale, ("decode", step, err, scale)
        if got_tok != want_tok:
            assert top2_gap(want) < 2 * err, ("decode token", step)
        tok, pos = got_tok, pos + 1
    eng.close()


@pytest.mark.parametrize("n,chunk,start", [
    (40, 0, 0),     # one chunk
    (40, 16, 0),    # three chunks, the last ragged
    (37, 7, 20),    # after 20 seeded positions, chunks of 7
    (150, 64, 0),   # chunks past one 64-key tile
])
def test_prefill_matches_oracle(n, chunk, start):
    check_prefill(CFG, n, chunk, start)


def test_prefill_head_dim_128():
    check_prefill(CFG_D128, 70, 32, 5)


def test_prefill_group_of_8():
    check_prefill(CFG_G8, 45, 20)


def test_prefill_rejects_bad_arguments():
    eng = ib.BatchEngine(CFG, 2, seed=1)
    for args in [(2, [5], 0, 0), (0, [], 0, 0), (0, [5], 256, 0), (0, [5] * 10, 250, 0), (0, [5000], 0, 0),
                 (0, [5], 0, -1)]:
        with pytest.raises(ib.InferntError):
            eng.prefill(*args)
    eng.close()
