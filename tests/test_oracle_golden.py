"""The CPU oracle against the reference's own known answers (CPU only).

Per-op cases come from the reference's self-test suite (src/main.cpp, via
tests/golden/kat.json); full-forward logits come from the reference's own
CUDA build (tests/golden/ref_forward_*.npz, made by
tests/golden/make_ref_fixtures.py on a GPU)."""
import glob
import os

import numpy as np
import pytest

import oracle as O

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def test_gemm(kat):
    g = kat["gemm"]
    C = O.gemm(g["A"], g["B"], g["M"], g["N"], g["K"], trans_a=g["trans_a"], trans_b=g["trans_b"])
    assert np.abs(C - np.array(g["expected"])).max() <= g["tol"]


def test_gemm_transposes_agree():
    rng = np.random.default_rng(0)
    M, N, K = 3, 5, 7
    A = rng.standard_normal((M, K)).astype(np.float32)
    B = rng.standard_normal((N, K)).astype(np.float32)
    ref = (A.astype(np.float64) @ B.T.astype(np.float64)).ravel()
    assert np.allclose(O.gemm(A, B, M, N, K, trans_b=1), ref, atol=1e-5)
    assert np.allclose(O.gemm(A.T.copy(), B, M, N, K, trans_a=1, trans_b=1), ref, atol=1e-5)
    C0 = rng.standard_normal(M * N).astype(np.float32)
    out = O.gemm(A, B, M, N, K, alpha=2.0, beta=0.5, trans_b=1, C=C0)
    assert np.allclose(out, 2.0 * ref + 0.5 * C0, atol=1e-5)


def test_rmsnorm(kat):
    r = kat["rmsnorm"]
    out = O.rmsnorm(r["x"], r["w"], r["batch"], r["hidden"], r["eps"])
    assert np.abs(out - r["expected"]).max() <= r["tol"]


def test_residual(kat):
    r = kat["residual"]
    assert np.abs(O.residual_add(r["a"], r["b"]) - r["expected"]).max() <= r["tol"]


def test_rope(kat):
    r = kat["rope"]
    q, k = O.rope(r["q"], r["k"], r["batch"], r["num_q_heads"], r["num_kv_heads"], r["head_dim"],
                  r["position"], r["theta"])
    assert np.abs(q - r["expected_q"]).max() <= r["tol"]
    assert np.abs(k - r["expected_k"]).max() <= r["tol"]


def test_softmax(kat):
    r = kat["softmax"]
    assert np.abs(O.softmax(r["x"], r["rows"], r["seq_len"]) - r["expected"]).max() <= r["tol"]


def test_softmax_with_mask_zeroes_tail():
    x = np.arange(8, dtype=np.float32)
    out = O.softmax_with_mask(x, 1, 5, 8)
    assert np.all(out[5:] == 0)
    assert np.allclose(out[:5], O.softmax(x[:5], 1, 5))


def test_kv_cache(kat):
    r = kat["kv_cache"]
    n = r["num_kv_heads"] * r["max_seq_len"] * r["head_dim"]
    kc, vc = np.zeros(n, np.float32), np.zeros(n, np.float32)
    for pos in r["positions"]:
        kc, vc = O.kv_cache_append(kc, vc, r["k_new"], r["v_new"], r["num_kv_heads"], r["head_dim"],
                                   r["max_seq_len"], pos)
    assert np.abs(kc - r["expected_k"]).max() <= r["tol"]
    assert np.abs(vc - r["expected_v"]).max() <= r["tol"]


def test_attention_gqa(kat):
    a = kat["attention_gqa"]
    nq, nkv, D, seq, ms = a["num_q_heads"], a["num_kv_heads"], a["head_dim"], a["seq_len"], a["max_seq_len"]
    sc = O.attention_scores(a["q"], a["k_cache"], nq, nkv, D, seq, ms, a["scale"])
    p = O.softmax(sc, nq, seq)
    out = O.attention_values(p, a["v_cache"], nq, nkv, D, seq, ms)
    assert np.abs(out - a["expected"]).max() <= a["tol"]


def test_silu_mul(kat):
    s = kat["silu_mul"]
    assert np.abs(O.silu_mul(s["gate"], s["up"]) - s["expected"]).max() <= s["tol"]


def test_embedding_and_argmax(kat):
    e = kat["embedding_argmax"]
    row = O.embedding_lookup(e["table"], e["token"], e["hidden"])
    assert np.abs(row - e["expected_row"]).max() <= e["tol"]
    assert O.argmax(e["logits"]) == e["expected_argmax"]
    assert O.argmax_ref_order(e["logits"]) == e["expected_argmax"]


def test_argmax_edge_cases():
    # NaN never wins; everything <= -1e30 gives 0 (sampling.cu:8-9, strict '>')
    x = np.array([1.0, np.nan, 3.0, 3.0, 2.0], dtype=np.float32)
    assert O.argmax(x) == 2
    assert O.argmax(np.full(10, -np.inf, dtype=np.float32)) == 0
    assert O.argmax(np.full(10, np.nan, dtype=np.float32)) == 0
    # the reference's thread-stride order can pick a higher index on ties
    y = np.zeros(600, dtype=np.float32)
    y[300] = y[50] = 5.0
    assert O.argmax(y) == 50
    assert O.argmax_ref_order(y) == 300


def test_seeded_generator_properties():
    x = O.fill_normal(1 << 20, 0, 5, 1.0)
    assert abs(float(x.mean())) < 5e-3 and abs(float(x.var()) - 1.0) < 5e-3
    assert np.abs(x).max() <= 6.0
    # deterministic, stream-separated, range == slice of the stream
    assert np.array_equal(x, O.fill_normal(1 << 20, 0, 5, 1.0))
    assert not np.array_equal(x[:100], O.fill_normal(100, 0, 6, 1.0))
    assert np.array_equal(O.fill_normal_range(100, 0, 5, 1.0, 1000), x[1000:1100])
    # scaling by std is one IEEE multiply of the unit deviate
    y = O.fill_normal(1000, 0, 5, 0.02)
    assert np.array_equal(y, (x[:1000] * np.float32(0.02)).astype(np.float32))
    # bf16 rounding keeps the top 16 bits
    b = O.fill_normal(1000, 0, 5, 0.02, round_bf16=True)
    assert np.all((b.view(np.uint32) & 0xFFFF) == 0)
    assert np.abs(b - y).max() <= np.abs(y).max() * 2 ** -8


def test_prompt_ids_in_range():
    p = O.prompt(32, 0, 3, 32000)
    assert p.min() >= 3 and p.max() < 32000
    assert np.array_equal(p, O.prompt(32, 0, 3, 32000))


def _small_cfg(**kw):
    from infernt_b200 import ModelConfig
    base = dict(vocab_size=500, hidden_size=128, num_layers=3, num_attention_heads=8,
                num_key_value_heads=2, intermediate_size=256, max_seq_len=64, rms_norm_eps=1e-6,
                rope_theta=50000.0)
    base.update(kw)
    return ModelConfig(**base)


def test_oracle_decode_is_self_consistent():
    """forward == layers + final norm + head; decode == embedding + forward."""
    cfg = _small_cfg()
    m = O.LlamaOracle(cfg, seed=3)
    emb = m.emb.reshape(cfg.vocab_size, cfg.hidden_size)[7]
    logits = m.forward(emb, 0)
    m.reset()
    tok, logits2 = m.decode_token(7, 0)
    assert np.array_equal(logits, logits2)
    assert tok == int(np.argmax(logits))


def _ref_fixtures():
    return sorted(glob.glob(os.path.join(GOLDEN, "ref_forward_*.npz")))


@pytest.mark.parametrize("path", _ref_fixtures() or [None])
def test_oracle_matches_reference_build(path):
    """Logits of the reference's own CUDA build (FP32, cuBLAS) on seeded
    weights vs the oracle on the same weights, step by step."""
    if path is None:
        pytest.skip("no reference fixtures generated yet")
    from infernt_b200 import ModelConfig
    z = np.load(path)
    cfg = ModelConfig(*[int(v) for v in z["cfg_ints"]], rms_norm_eps=float(z["eps"]),
                      rope_theta=float(z["theta"]))
    m = O.LlamaOracle(cfg, seed=int(z["seed"]), std=float(z["std"]))
    tokens, ref_logits, ref_next = z["tokens"], z["logits"], z["next"]
    rows = z["logit_rows"]
    for i, t in enumerate(tokens):
        nxt, logits = m.decode_token(int(t), i)
        sel = logits[rows] if rows.size else logits
        ref = ref_logits[i]
        err = np.abs(sel - ref).max()
        scale = max(np.abs(ref).max(), 1e-6)
        assert err <= 1e-3 and err / scale <= 1e-4, (path, i, err)
        top2 = np.sort(logits)[-2:]
        if top2[1] - top2[0] >= 1e-4:
            assert nxt == int(ref_next[i]), (path, i)
