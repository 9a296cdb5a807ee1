"""Writes tests/golden/kat.json: the known-answer cases of INFERNT's built-in
self-test suite, as input/expected-output vectors.

Each case restates one ``test_*`` function of the reference's
``src/main.cpp`` (line ranges below): the same inputs, the same analytic
expected values computed in float32 the way the test computes them, and the
same tolerance.  Run from anywhere:  python tests/golden/make_kat.py
"""
import json
import math
import os

import numpy as np

f32 = np.float32


def kat_gemm():
    # src/main.cpp:108-157 — M=4, N=3, K=5, A[i]=0.1(i+1), B[i]=0.2(i+1), no transpose
    M, N, K = 4, 3, 5
    A = (np.arange(M * K, dtype=f32) + 1) * f32(0.1)
    B = (np.arange(K * N, dtype=f32) + 1) * f32(0.2)
    C = np.zeros(M * N, dtype=f32)
    for i in range(M):
        for j in range(N):
            s = f32(0)
            for k in range(K):
                s = f32(s + f32(A[i * K + k] * B[k * N + j]))
            C[i * N + j] = s
    return dict(M=M, N=N, K=K, trans_a=0, trans_b=0, A=A.tolist(), B=B.tolist(),
                expected=C.tolist(), tol=1e-4, source="src/main.cpp:108-157")


def kat_rmsnorm():
    # src/main.cpp:159-200 — hidden 8, x=0.5(i+1), w=1, eps 1e-5
    h = 8
    x = (np.arange(h, dtype=f32) + 1) * f32(0.5)
    w = np.ones(h, dtype=f32)
    eps = f32(1e-5)
    ss = f32(0)
    for v in x:
        ss = f32(ss + f32(v * v))
    rms = f32(math.sqrt(f32(f32(ss / f32(h)) + eps)))
    exp = (x / rms * w).astype(f32)
    return dict(batch=1, hidden=h, eps=1e-5, x=x.tolist(), w=w.tolist(),
                expected=exp.tolist(), tol=1e-4, source="src/main.cpp:159-200")


def kat_residual():
    # src/main.cpp:202-233 — a=i, b=2i -> 3i
    n = 16
    a = np.arange(n, dtype=f32)
    b = np.arange(n, dtype=f32) * f32(2)
    return dict(n=n, a=a.tolist(), b=b.tolist(), expected=(a * f32(3)).tolist(),
                tol=1e-5, source="src/main.cpp:202-233")


def kat_rope():
    # src/main.cpp:235-296 — 2 heads, D=4, pos=3, theta=1e4, q=k=1
    heads, D, theta, pos = 2, 4, 10000.0, 3
    half = D // 2
    qe = np.zeros(heads * D, dtype=f32)
    for hh in range(heads):
        for d in range(half):
            freq = f32(1.0) / f32(math.pow(f32(theta), f32(2 * d) / f32(D)))
            ang = f32(f32(pos) * freq)
            c, s = f32(math.cos(ang)), f32(math.sin(ang))
            qe[hh * D + d] = f32(c - s)
            qe[hh * D + d + half] = f32(c + s)
    ones = [1.0] * (heads * D)
    return dict(batch=1, num_q_heads=heads, num_kv_heads=heads, head_dim=D, position=pos,
                theta=theta, q=ones, k=ones, expected_q=qe.tolist(), expected_k=qe.tolist(),
                tol=1e-4, source="src/main.cpp:235-296")


def kat_softmax():
    # src/main.cpp:298-333 — [1,2,3,4,5]
    x = np.array([1, 2, 3, 4, 5], dtype=f32)
    e = np.exp(x - f32(5)).astype(f32)
    e = (e / e.sum(dtype=f32)).astype(f32)
    return dict(rows=1, seq_len=5, x=x.tolist(), expected=e.tolist(), tol=1e-5,
                source="src/main.cpp:298-333")


def kat_kv_cache():
    # src/main.cpp:335-380 — Nkv=2, D=4, max_seq=8, k_new=0.1(i+1), v_new=0.2(i+1),
    # appended at positions 0 and 1
    nkv, D, max_seq = 2, 4, 8
    kn = (np.arange(nkv * D, dtype=f32) + 1) * f32(0.1)
    vn = (np.arange(nkv * D, dtype=f32) + 1) * f32(0.2)
    kc = np.zeros((nkv, max_seq, D), dtype=f32)
    vc = np.zeros((nkv, max_seq, D), dtype=f32)
    for pos in (0, 1):
        kc[:, pos, :] = kn.reshape(nkv, D)
        vc[:, pos, :] = vn.reshape(nkv, D)
    return dict(num_kv_heads=nkv, head_dim=D, max_seq_len=max_seq, positions=[0, 1],
                k_new=kn.tolist(), v_new=vn.tolist(), expected_k=kc.ravel().tolist(),
                expected_v=vc.ravel().tolist(), tol=1e-5, source="src/main.cpp:335-380")


def kat_attention_gqa():
    # src/main.cpp:382-446 — Nq=4, Nkv=2, D=4, max_seq=16, seq=3, q=1, K=1,
    # V[s]=s+1; scores -> softmax -> values gives 2.0 everywhere
    nq, nkv, D, max_seq, seq = 4, 2, 4, 16, 3
    kc = np.zeros((nkv, max_seq, D), dtype=f32)
    vc = np.zeros((nkv, max_seq, D), dtype=f32)
    for s in range(seq):
        kc[:, s, :] = 1.0
        vc[:, s, :] = float(s + 1)
    exp = [f32(1.0 / 3.0) * 1 + f32(1.0 / 3.0) * 2 + f32(1.0 / 3.0) * 3] * (nq * D)
    return dict(num_q_heads=nq, num_kv_heads=nkv, head_dim=D, max_seq_len=max_seq,
                seq_len=seq, scale=1.0 / math.sqrt(D), q=[1.0] * (nq * D),
                k_cache=kc.ravel().tolist(), v_cache=vc.ravel().tolist(),
                expected=[float(v) for v in exp], tol=1e-3, source="src/main.cpp:382-446")


def kat_silu():
    # src/main.cpp:448-477 — g = i-1, u = 2
    g = np.arange(4, dtype=f32) - f32(1)
    u = np.full(4, 2.0, dtype=f32)
    exp = (g / (f32(1) + np.exp(-g).astype(f32)) * u).astype(f32)
    return dict(n=4, gate=g.tolist(), up=u.tolist(), expected=exp.tolist(), tol=1e-4,
                source="src/main.cpp:448-477")


def kat_embedding_argmax():
    # src/main.cpp:633-681 — iota table [10,8], token 3; logits 0.01 i with [42]=99
    V, h, tok = 10, 8, 3
    table = np.arange(V * h, dtype=f32)
    logits = (np.arange(100, dtype=f32) * f32(0.01)).astype(f32)
    logits[42] = 99.0
    return dict(vocab_size=V, hidden=h, token=tok, table=table.tolist(),
                expected_row=table[tok * h:(tok + 1) * h].tolist(),
                logits=logits.tolist(), expected_argmax=42, tol=1e-5,
                source="src/main.cpp:633-681")


def kat_config():
    # src/main.cpp:83-106 — TinyLlama dims derive head_dim 64 and 8 kv groups
    return dict(hidden_size=2048, num_attention_heads=32, num_key_value_heads=4,
                expected_head_dim=64, expected_kv_groups=8, source="src/main.cpp:83-106")


def main():
    out = dict(
        gemm=kat_gemm(), rmsnorm=kat_rmsnorm(), residual=kat_residual(), rope=kat_rope(),
        softmax=kat_softmax(), kv_cache=kat_kv_cache(), attention_gqa=kat_attention_gqa(),
        silu_mul=kat_silu(), embedding_argmax=kat_embedding_argmax(), config=kat_config(),
    )
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "kat.json")
    with open(path, "w") as f:
        json.dump(out, f, indent=1)
    print("wrote", path)


if __name__ == "__main__":
    main()
