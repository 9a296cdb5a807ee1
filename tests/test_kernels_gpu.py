"""Per-op parity on the GPU: every kernels.h entry point and every fused
decode op, through the C ABI, against the reference's known answers
(tests/golden/kat.json) and the CPU oracle on seeded inputs.

Tolerances: the reference's own test tolerances for the known answers;
1e-5 relative (to the row's max magnitude) for FP32 ops on random inputs
(only summation order differs); bf16 weights are compared with the oracle on
the same bf16-rounded weights at 1e-5 relative as well (accumulation is FP32
on both sides)."""
import numpy as np
import pytest

import infernt_b200 as ib
import oracle as O

pytestmark = pytest.mark.gpu

REL = 1e-5


_KEEP = []  # device buffers stay alive until the test's kernels are done


@pytest.fixture(autouse=True)
def _release_buffers():
    yield
    if _KEEP:
        import torch
        torch.cuda.synchronize()
        _KEEP.clear()


def dev(torch, a, dtype=None):
    t = torch.as_tensor(np.asarray(a, dtype=np.float32)).cuda()
    t = t if dtype is None else t.to(dtype)
    _KEEP.append(t)
    return t


def host(torch, t):
    torch.cuda.synchronize()
    return t.float().cpu().numpy().ravel()


def close(got, want, rel=REL, atol=0.0):
    got, want = np.asarray(got, np.float64).ravel(), np.asarray(want, np.float64).ravel()
    scale = max(np.abs(want).max(), 1e-30)
    err = np.abs(got - want).max()
    assert err <= max(rel * scale, atol), (err, scale)


# ---------------------------------------------------------------- known answers

def test_kat_rmsnorm(cuda, kat):
    r = kat["rmsnorm"]
    x, w = dev(cuda, r["x"]), dev(cuda, r["w"])
    out = cuda.zeros_like(x)
    ib.call("infernt_rmsnorm", out.data_ptr(), x.data_ptr(), w.data_ptr(), 1, r["hidden"], r["eps"], None)
    assert np.abs(host(cuda, out) - r["expected"]).max() <= r["tol"]


def test_kat_residual(cuda, kat):
    r = kat["residual"]
    a, b = dev(cuda, r["a"]), dev(cuda, r["b"])
    out = cuda.zeros_like(a)
    ib.call("infernt_residual_add", out.data_ptr(), a.data_ptr(), b.data_ptr(), r["n"], None)
    assert np.abs(host(cuda, out) - r["expected"]).max() <= r["tol"]


def test_kat_rope(cuda, kat):
    r = kat["rope"]
    q, k = dev(cuda, r["q"]), dev(cuda, r["k"])
    ib.call("infernt_rope", q.data_ptr(), k.data_ptr(), 1, r["num_q_heads"], r["num_kv_heads"],
            r["head_dim"], r["position"], r["theta"], None)
    assert np.abs(host(cuda, q) - r["expected_q"]).max() <= r["tol"]
    assert np.abs(host(cuda, k) - r["expected_k"]).max() <= r["tol"]


def test_kat_softmax(cuda, kat):
    r = kat["softmax"]
    x = dev(cuda, r["x"])
    out = cuda.zeros_like(x)
    ib.call("infernt_softmax", out.data_ptr(), x.data_ptr(), 1, 5, None)
    assert np.abs(host(cuda, out) - r["expected"]).max() <= r["tol"]


def test_kat_kv_cache(cuda, kat):
    r = kat["kv_cache"]
    n = r["num_kv_heads"] * r["max_seq_len"] * r["head_dim"]
    kc, vc = cuda.zeros(n, device="cuda"), cuda.zeros(n, device="cuda")
    kn, vn = dev(cuda, r["k_new"]), dev(cuda, r["v_new"])
    for pos in r["positions"]:
        ib.call("infernt_kv_cache_append", kc.data_ptr(), vc.data_ptr(), kn.data_ptr(), vn.data_ptr(),
                r["num_kv_heads"], r["head_dim"], r["max_seq_len"], pos, None)
    assert np.abs(host(cuda, kc) - r["expected_k"]).max() <= r["tol"]
    assert np.abs(host(cuda, vc) - r["expected_v"]).max() <= r["tol"]


def test_kat_attention_gqa(cuda, kat):
    a = kat["attention_gqa"]
    nq, nkv, D, seq, ms = a["num_q_heads"], a["num_kv_heads"], a["head_dim"], a["seq_len"], a["max_seq_len"]
    q, kc, vc = dev(cuda, a["q"]), dev(cuda, a["k_cache"]), dev(cuda, a["v_cache"])
    sc = cuda.zeros(nq * seq, device="cuda")
    out = cuda.zeros(nq * D, device="cuda")
    ib.call("infernt_attention_scores", sc.data_ptr(), q.data_ptr(), kc.data_ptr(), nq, nkv, D, seq, ms,
            a["scale"], None)
    ib.call("infernt_softmax", sc.data_ptr(), sc.data_ptr(), nq, seq, None)
    ib.call("infernt_attention_values", out.data_ptr(), sc.data_ptr(), vc.data_ptr(), nq, nkv, D, seq, ms, None)
    assert np.abs(host(cuda, out) - a["expected"]).max() <= a["tol"]


def test_kat_silu_mul(cuda, kat):
    s = kat["silu_mul"]
    g, u = dev(cuda, s["gate"]), dev(cuda, s["up"])
    out = cuda.zeros_like(g)
    ib.call("infernt_silu_mul", out.data_ptr(), g.data_ptr(), u.data_ptr(), 4, None)
    assert np.abs(host(cuda, out) - s["expected"]).max() <= s["tol"]


def test_kat_embedding_argmax(cuda, kat):
    e = kat["embedding_argmax"]
    table = dev(cuda, e["table"])
    out = cuda.zeros(e["hidden"], device="cuda")
    ib.call("infernt_embedding_lookup", out.data_ptr(), table.data_ptr(), e["token"], e["hidden"], None)
    assert np.abs(host(cuda, out) - e["expected_row"]).max() <= e["tol"]
    logits = dev(cuda, e["logits"])
    tok = cuda.zeros(1, dtype=cuda.int32, device="cuda")
    ib.call("infernt_argmax", tok.data_ptr(), logits.data_ptr(), len(e["logits"]), None)
    cuda.cuda.synchronize()
    assert int(tok.item()) == e["expected_argmax"]


def test_kat_gemm(cuda, kat):
    g = kat["gemm"]
    A, B = dev(cuda, g["A"]), dev(cuda, g["B"])
    C = cuda.zeros(g["M"] * g["N"], device="cuda")
    ib.call("infernt_gemm_f32", A.data_ptr(), B.data_ptr(), C.data_ptr(), g["M"], g["N"], g["K"], 1.0, 0.0,
            0, 0, None)
    assert np.abs(host(cuda, C) - g["expected"]).max() <= g["tol"]


# ---------------------------------------------------------- seeded random inputs

def rnd(n, stream, std=1.0, seed=11):
    return O.fill_normal(n, seed, stream, std)


@pytest.mark.parametrize("batch,hidden", [(1, 2048), (3, 200), (2, 5632)])
def test_rmsnorm_vs_oracle(cuda, batch, hidden):
    x, w = rnd(batch * hidden, 1), rnd(hidden, 2)
    out = cuda.zeros(batch * hidden, device="cuda")
    ib.call("infernt_rmsnorm", out.data_ptr(), dev(cuda, x).data_ptr(), dev(cuda, w).data_ptr(), batch, hidden,
            1e-5, None)
    close(host(cuda, out), O.rmsnorm(x, w, batch, hidden, 1e-5))


@pytest.mark.parametrize("pos", [0, 7, 4095])
def test_rope_vs_oracle(cuda, pos):
    nq, nkv, D = 32, 4, 64
    q, k = rnd(nq * D, 3), rnd(nkv * D, 4)
    qd, kd = dev(cuda, q), dev(cuda, k)
    ib.call("infernt_rope", qd.data_ptr(), kd.data_ptr(), 1, nq, nkv, D, pos, 10000.0, None)
    qo, ko = O.rope(q, k, 1, nq, nkv, D, pos, 10000.0)
    close(host(cuda, qd), qo, rel=1e-5)
    close(host(cuda, kd), ko, rel=1e-5)


@pytest.mark.parametrize("rows,seq", [(32, 1), (32, 288), (4, 3000)])
def test_softmax_vs_oracle(cuda, rows, seq):
    x = rnd(rows * seq, 5, 3.0)
    out = cuda.zeros(rows * seq, device="cuda")
    ib.call("infernt_softmax", out.data_ptr(), dev(cuda, x).data_ptr(), rows, seq, None)
    close(host(cuda, out), O.softmax(x, rows, seq))


def test_softmax_with_mask_vs_oracle(cuda):
    heads, seq, total = 8, 100, 160
    x = rnd(heads * total, 6, 2.0)
    out = cuda.full((heads * total,), 7.0, device="cuda")
    ib.call("infernt_softmax_with_mask", out.data_ptr(), dev(cuda, x).data_ptr(), heads, seq, total, None)
    close(host(cuda, out), O.softmax_with_mask(x, heads, seq, total))


@pytest.mark.parametrize("seq", [1, 300, 1500])
def test_attention_scores_values_vs_oracle(cuda, seq):
    """Covers seq_len > 1024, where the reference leaves positions unset
    (attention.cu:49); the new kernels compute every position."""
    nq, nkv, D, ms = 32, 4, 64, 2048
    q = rnd(nq * D, 7)
    kc, vc = rnd(nkv * ms * D, 8), rnd(nkv * ms * D, 9)
    scale = 1.0 / np.sqrt(D)
    sc = cuda.zeros(nq * seq, device="cuda")
    ib.call("infernt_attention_scores", sc.data_ptr(), dev(cuda, q).data_ptr(), dev(cuda, kc).data_ptr(), nq,
            nkv, D, seq, ms, scale, None)
    want = O.attention_scores(q, kc, nq, nkv, D, seq, ms, scale)
    close(host(cuda, sc), want)
    p = O.softmax(want, nq, seq)
    out = cuda.zeros(nq * D, device="cuda")
    ib.call("infernt_attention_values", out.data_ptr(), dev(cuda, p).data_ptr(), dev(cuda, vc).data_ptr(), nq,
            nkv, D, seq, ms, None)
    close(host(cuda, out), O.attention_values(p, vc, nq, nkv, D, seq, ms))


def test_argmax_edge_cases(cuda):
    def run(x):
        t = dev(cuda, x)
        tok = cuda.zeros(1, dtype=cuda.int32, device="cuda")
        ib.call("infernt_argmax", tok.data_ptr(), t.data_ptr(), len(x), None)
        cuda.cuda.synchronize()
        return int(tok.item())
    x = rnd(128256, 10)
    assert run(x) == O.argmax(x)
    y = np.zeros(200000, np.float32)
    y[150000] = y[70000] = 5.0  # tie across blocks -> lowest index
    assert run(y) == 70000
    z = np.full(1000, np.nan, np.float32)
    z[999] = 1.0
    assert run(z) == 999
    assert run(np.full(1000, -np.inf, np.float32)) == 0


@pytest.mark.parametrize("M,N,K,ta,tb,alpha,beta", [
    (1, 3072, 2048, 0, 1, 1.0, 0.0),   # the decode projection -> weight-streaming GEMV
    (1, 100, 72, 0, 1, 1.0, 0.0),      # GEMV, plain path
    (5, 70, 33, 0, 1, 1.0, 0.0),
    (17, 9, 65, 1, 0, 0.5, 2.0),
    (64, 128, 256, 1, 1, 1.0, 1.0),
])
def test_gemm_vs_oracle(cuda, M, N, K, ta, tb, alpha, beta):
    A, B, C0 = rnd(M * K, 11), rnd(N * K, 12), rnd(M * N, 13)
    Cd = dev(cuda, C0)
    ib.call("infernt_gemm_f32", dev(cuda, A).data_ptr(), dev(cuda, B).data_ptr(), Cd.data_ptr(), M, N, K, alpha,
            beta, ta, tb, None)
    close(host(cuda, Cd), O.gemm(A, B, M, N, K, alpha, beta, ta, tb, C=C0), rel=1e-5)


# ---------------------------------------------------------------- fused ops

def _w(torch, rows, K, stream, dtype):
    w = O.fill_normal(rows * K, 21, stream, 0.02, round_bf16=(dtype == ib.DTYPE_BF16))
    t = dev(torch, w, torch.bfloat16 if dtype == ib.DTYPE_BF16 else None)
    return w, t


@pytest.mark.parametrize("dtype", [ib.DTYPE_F32, ib.DTYPE_BF16])
@pytest.mark.parametrize("K,n", [(2048, (2048, 256, 256)), (512, (100, 7, 0)), (200, (64, 16, 16))])
def test_rmsnorm_gemv_qkv(cuda, dtype, K, n):
    ws = [_w(cuda, r, K, 30 + i, dtype) if r else (None, None) for i, r in enumerate(n)]
    x, nw = rnd(K, 14), rnd(K, 15)
    y = cuda.zeros(sum(n), device="cuda")
    args = []
    for (w, t), r in zip(ws, n):
        args += [t.data_ptr() if t is not None else None, r]
    ib.call("infernt_rmsnorm_gemv", y.data_ptr(), *args, K, dtype, dev(cuda, x).data_ptr(),
            dev(cuda, nw).data_ptr(), 1e-5, None)
    xn = O.rmsnorm(x, nw, 1, K, 1e-5)
    want = np.concatenate([O.gemm(xn, w, 1, r, K, trans_b=1) for (w, _), r in zip(ws, n) if r])
    close(host(cuda, y), want)


@pytest.mark.parametrize("dtype", [ib.DTYPE_F32, ib.DTYPE_BF16])
@pytest.mark.parametrize("n,K", [(2048, 5632), (2048, 2048), (96, 160)])
def test_gemv_residual(cuda, dtype, n, K):
    w, t = _w(cuda, n, K, 40, dtype)
    x, res = rnd(K, 16), rnd(n, 17)
    out = dev(cuda, res)
    ib.call("infernt_gemv_residual", out.data_ptr(), out.data_ptr(), t.data_ptr(), n, K, dtype,
            dev(cuda, x).data_ptr(), None)
    close(host(cuda, out), res + O.gemm(x, w, 1, n, K, trans_b=1))


@pytest.mark.parametrize("dtype", [ib.DTYPE_F32, ib.DTYPE_BF16])
@pytest.mark.parametrize("n,K", [(5632, 2048), (37, 1024), (50, 96)])
def test_gate_up_silu(cuda, dtype, n, K):
    wg, tg = _w(cuda, n, K, 41, dtype)
    wu, tu = _w(cuda, n, K, 42, dtype)
    x, nw = rnd(K, 18), rnd(K, 19)
    out = cuda.zeros(n, device="cuda")
    ib.call("infernt_rmsnorm_gate_up_silu", out.data_ptr(), tg.data_ptr(), tu.data_ptr(), n, K, dtype,
            dev(cuda, x).data_ptr(), dev(cuda, nw).data_ptr(), 1e-5, None)
    xn = O.rmsnorm(x, nw, 1, K, 1e-5)
    want = O.silu_mul(O.gemm(xn, wg, 1, n, K, trans_b=1), O.gemm(xn, wu, 1, n, K, trans_b=1))
    close(host(cuda, out), want)


@pytest.mark.parametrize("dtype", [ib.DTYPE_F32, ib.DTYPE_BF16])
@pytest.mark.parametrize("V,K", [(32000, 2048), (1000, 96)])
def test_lm_head_argmax(cuda, dtype, V, K):
    w, t = _w(cuda, V, K, 43, dtype)
    x, nw = rnd(K, 20), np.ones(K, np.float32)
    logits = cuda.zeros(V, device="cuda")
    tok = cuda.zeros(1, dtype=cuda.int32, device="cuda")
    ws = cuda.zeros(ib.lib().infernt_lm_head_workspace_bytes(), dtype=cuda.uint8, device="cuda")
    for _ in range(2):  # the workspace counter must be left at zero
        ib.call("infernt_rmsnorm_lm_head_argmax", logits.data_ptr(), tok.data_ptr(), t.data_ptr(), V, K, dtype,
                dev(cuda, x).data_ptr(), dev(cuda, nw).data_ptr(), 1e-5, ws.data_ptr(), None)
        want = O.gemm(O.rmsnorm(x, nw, 1, K, 1e-5), w, 1, V, K, trans_b=1)
        got = host(cuda, logits)
        close(got, want)
        assert int(tok.item()) == int(np.argmax(got))


@pytest.mark.parametrize("nq,nkv,D,pos,splits", [
    (32, 4, 64, 0, 37), (32, 4, 64, 287, 37), (32, 4, 64, 4095, 37), (32, 4, 64, 1500, 1),
    (32, 8, 128, 511, 18), (8, 2, 64, 40, 3), (16, 16, 32, 5, 2),
])
def test_attention_decode_vs_oracle(cuda, nq, nkv, D, pos, splits):
    """RoPE + KV append + split-KV GQA attention against the oracle's
    rope -> append -> scores -> softmax -> values (llama_layer.cpp:25-48)."""
    ms = max(pos + 1, 64)
    qkv = rnd(nq * D + 2 * nkv * D, 22)
    kc, vc = rnd(nkv * ms * D, 23), rnd(nkv * ms * D, 24)
    kd, vd = dev(cuda, kc), dev(cuda, vc)
    out = cuda.zeros(nq * D, device="cuda")
    nbytes = ib.lib().infernt_attention_workspace_bytes(nq, nkv, D, splits)
    ws = cuda.zeros(nbytes, dtype=cuda.uint8, device="cuda")
    theta = 10000.0
    for _ in range(2):
        ib.call("infernt_attention_decode", out.data_ptr(), dev(cuda, qkv).data_ptr(), kd.data_ptr(), vd.data_ptr(),
                nq, nkv, D, ms, pos, theta, splits, ws.data_ptr(), None)
        q, k = O.rope(qkv[:nq * D], qkv[nq * D:nq * D + nkv * D], 1, nq, nkv, D, pos, theta)
        v = qkv[nq * D + nkv * D:]
        kc2, vc2 = O.kv_cache_append(kc, vc, k, v, nkv, D, ms, pos)
        sc = O.attention_scores(q, kc2, nq, nkv, D, pos + 1, ms, 1.0 / np.sqrt(np.float32(D)))
        want = O.attention_values(O.softmax(sc, nq, pos + 1), vc2, nq, nkv, D, pos + 1, ms)
        close(host(cuda, out), want, rel=2e-5)
        # RoPE angle = position * freq: one ulp of freq (powf differs by an ulp
        # between the device and glibc) moves the angle by ~position ulps
        close(host(cuda, kd), kc2, rel=1e-6 + 2e-7 * pos)
        assert np.array_equal(host(cuda, vd), vc2)
