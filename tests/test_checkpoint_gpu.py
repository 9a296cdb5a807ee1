"""A model loaded from an INFT v1 checkpoint (infernt_checkpoint_load onto
the device) decodes through the plan (infernt_plan_create / _decode) like
the CPU oracle holding the same weights: the oracle's seeded model is
written as config.json + model.bin, loaded, and decoded for a short prompt
and greedy continuation.  Tolerances are the decode tests': logits max-abs
1e-3 and 1e-4 of the largest |logit|, greedy tokens identical unless the
oracle's top-2 gap is below 1e-4; the bf16 option against the oracle on the
same bf16-rounded weights."""
import ctypes

import numpy as np
import pytest

import infernt_b200 as ib
import oracle as O
from inft_file import LAYER_NAMES, write_config, write_inft

pytestmark = pytest.mark.gpu

CFG = ib.ModelConfig(vocab_size=1000, hidden_size=512, num_layers=2, num_attention_heads=8, num_key_value_heads=2,
                     intermediate_size=1536, max_seq_len=64)


def oracle_tensors(orc, cfg):
    H, V, I = cfg.hidden_size, cfg.vocab_size, cfg.intermediate_size
    qs, kvs = cfg.num_attention_heads * cfg.head_dim, cfg.num_key_value_heads * cfg.head_dim
    shapes = [(H,), (qs, H), (kvs, H), (kvs, H), (H, qs), (H,), (I, H), (I, H), (H, I)]
    named = [("model.embed_tokens.weight", orc.emb.reshape(V, H))]
    for l, lw in enumerate(orc.layers):
        named += [("model.layers.%d.%s" % (l, n), w.reshape(s)) for n, w, s in zip(LAYER_NAMES, lw, shapes)]
    named += [("model.norm.weight", orc.final_norm), ("lm_head.weight", orc.lm_head.reshape(V, H))]
    return named


def run(tmp_path, cuda, bf16):
    torch = cuda
    orc = O.LlamaOracle(CFG, seed=3)  # FP32 weights are what the checkpoint holds
    cj, mb = str(tmp_path / "config.json"), str(tmp_path / "model.bin")
    write_config(cj, CFG, weight_dtype="bf16" if bf16 else "fp32")
    write_inft(mb, oracle_tensors(orc, CFG))
    cfg = ib.Checkpoint.read_config(cj)
    assert cfg.weight_dtype == (ib.DTYPE_BF16 if bf16 else ib.DTYPE_F32)
    ck = ib.Checkpoint(mb, cfg, device=1)
    want_orc = O.LlamaOracle(CFG, seed=3, round_bf16=bf16)
    L, nkv, S, D = cfg.num_layers, cfg.num_key_value_heads, cfg.max_seq_len, cfg.head_dim
    kc = [torch.zeros(nkv * S * D, device="cuda") for _ in range(L)]
    vc = [torch.zeros(nkv * S * D, device="cuda") for _ in range(L)]
    P = ctypes.c_void_p
    wp = (P * len(ck.ptrs))(*ck.ptrs)
    kp = (P * L)(*[t.data_ptr() for t in kc])
    vp = (P * L)(*[t.data_ptr() for t in vc])
    c = cfg.c()
    h = P()
    ib.call("infernt_plan_create", ctypes.byref(c), wp, kp, vp, ib.MODE_PERSISTENT, ctypes.byref(h))
    logits = torch.empty(cfg.vocab_size, device="cuda")
    prompt = O.prompt(4, 3, 3, cfg.vocab_size)
    tok = None
    try:
        for pos in range(12):
            t_in = int(prompt[pos]) if pos < len(prompt) else tok
            ib.call("infernt_plan_decode", h, t_in, pos, logits.data_ptr(), None)
            got_tok = ctypes.c_int()
            ib.call("infernt_plan_read_token", h, ctypes.byref(got_tok), None)
            want_tok, want = want_orc.decode_token(t_in, pos)
            got = logits.cpu().numpy()
            err = float(np.abs(got - want).max())
            assert err <= 1e-3 and err / float(np.abs(want).max()) <= 1e-4, (pos, err)
            if got_tok.value != want_tok:
                s = np.sort(want)
                assert s[-1] - s[-2] < 1e-4, (pos, got_tok.value, want_tok)
            tok = got_tok.value
    finally:
        ib.lib().infernt_plan_destroy(h)
        ck.close()


def test_checkpoint_fp32_decodes_like_oracle(tmp_path, cuda):
    run(tmp_path, cuda, bf16=False)


def test_checkpoint_bf16_option_decodes_like_oracle(tmp_path, cuda):
    run(tmp_path, cuda, bf16=True)


def write_tokenizer(path, n):
    """tokenizer.bin as the engine's Tokenizer::load reads it: uint32 count,
    uint32 longest piece, then per piece float score, int32 length, bytes."""
    import struct
    pieces = [("t%d" % i).encode() for i in range(n)]
    with open(path, "wb") as f:
        f.write(struct.pack("II", n, max(len(p) for p in pieces)))
        for i, p in enumerate(pieces):
            f.write(struct.pack("fi", -float(i), len(p)))
            f.write(p)


def test_engine_load_model_and_device_sampling(tmp_path, cuda):
    """InferenceEngine::load_model of a checkpoint directory decodes like the
    oracle; with device sampling on, sample_next_token(T) draws from
    softmax(logits / T) of the last step (the top token's frequency within
    6 standard deviations of its probability over 3000 draws)."""
    orc = O.LlamaOracle(CFG, seed=4)
    d = str(tmp_path)
    write_config(d + "/config.json", CFG)
    write_inft(d + "/model.bin", oracle_tensors(orc, CFG))
    write_tokenizer(d + "/tokenizer.bin", CFG.vocab_size)
    eng = ib.Engine.load_model(d)
    prompt = O.prompt(4, 4, 3, CFG.vocab_size)
    tok = None
    for pos in range(8):
        t_in = int(prompt[pos]) if pos < len(prompt) else tok
        got_tok = eng.forward_token(t_in, pos)
        want_tok, want = orc.decode_token(t_in, pos)
        got = eng.logits()
        err = float(np.abs(got - want).max())
        assert err <= 1e-3 and err / float(np.abs(want).max()) <= 1e-4, (pos, err)
        if got_tok != want_tok:
            s = np.sort(want)
            assert s[-1] - s[-2] < 1e-4, pos
        tok = got_tok
    eng.set_device_sampling(True, seed=9)
    T = 0.05
    z = want.astype(np.float64) / T
    p = np.exp(z - z.max())
    p /= p.sum()
    top = int(np.argmax(p))
    n = 3000
    draws = np.array([eng.sample_next_token(T) for _ in range(n)])
    assert draws.min() >= 0 and draws.max() < CFG.vocab_size
    c = int((draws == top).sum())
    sd = np.sqrt(n * p[top] * (1 - p[top])) + 1e-9
    assert abs(c - n * p[top]) <= 6 * sd + 1, (c, n * p[top])
    assert eng.sample_next_token(0.0) == tok
    eng.close()
