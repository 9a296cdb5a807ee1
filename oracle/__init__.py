"""CPU oracle of INFERNT's decode step — TEST INFRASTRUCTURE.

ctypes bindings of ``oracle/liboracle.so`` (the scalar C restatement in
oracle.c) and of ``oracle/_ref/libinfernt_ref.so`` (the reference's own
sources compiled unchanged, driven by ref_runner.cpp).  Only the tests, the
smoke check and the benchmark's CPU-baseline / reference legs use this
package; the product library never does.

Parity pins: tests/test_oracle_golden.py checks the per-op functions against
the known-answer cases of the reference's self-test suite
(tests/golden/kat.json) and the full forward against logits that the
reference build produced (tests/golden/ref_forward_*.npz).
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libinfernt_ref.so")

STREAM_EMBEDDING = 1
STREAM_LM_HEAD = 2
STREAM_PROMPT = 7
STREAM_KV_K = 8
STREAM_KV_V = 9
STREAM_LOGITS = 10


def stream_layer(l, m):
    return 100 + 16 * l + m


def build(ref=None):
    """Runs oracle/Makefile (the oracle; the reference runner when the
    reference checkout exists)."""
    target = "all" if ref is None else ("ref" if ref else "oracle")
    subprocess.run(["make", "-s", "-C", HERE, target], check=True)


_olib = None
_F = ctypes.c_float
_I = ctypes.c_int
_P = ctypes.c_void_p


class OracleConfig(ctypes.Structure):
    _fields_ = [("vocab_size", _I), ("hidden_size", _I), ("num_layers", _I),
                ("num_attention_heads", _I), ("num_key_value_heads", _I),
                ("intermediate_size", _I), ("max_seq_len", _I), ("head_dim", _I),
                ("rms_norm_eps", _F), ("rope_theta", _F)]


def olib():
    global _olib
    if _olib is None:
        if not os.path.exists(ORACLE_SO):
            build(ref=False)
        l = ctypes.CDLL(ORACLE_SO)
        l.oracle_set_threads.argtypes = [_I]
        l.oracle_set_act_bf16.argtypes = [_I]
        l.oracle_fill_normal.argtypes = [_P, ctypes.c_size_t, ctypes.c_uint64, ctypes.c_uint64, _F, _I]
        l.oracle_fill_normal_range.argtypes = [_P, ctypes.c_size_t, ctypes.c_uint64, ctypes.c_uint64,
                                               _F, _I, ctypes.c_uint64]
        l.oracle_fill_prompt.argtypes = [_P, _I, ctypes.c_uint64, _I, _I]
        l.oracle_rmsnorm.argtypes = [_P, _P, _P, _I, _I, _F]
        l.oracle_residual_add.argtypes = [_P, _P, _P, _I]
        l.oracle_rope.argtypes = [_P, _P, _I, _I, _I, _I, _I, _F]
        l.oracle_softmax.argtypes = [_P, _P, _I, _I]
        l.oracle_softmax_with_mask.argtypes = [_P, _P, _I, _I, _I]
        l.oracle_kv_cache_append.argtypes = [_P, _P, _P, _P, _I, _I, _I, _I]
        l.oracle_attention_scores.argtypes = [_P, _P, _P, _I, _I, _I, _I, _I, _F]
        l.oracle_attention_values.argtypes = [_P, _P, _P, _I, _I, _I, _I, _I]
        l.oracle_silu_mul.argtypes = [_P, _P, _P, _I]
        l.oracle_embedding_lookup.argtypes = [_P, _P, _I, _I]
        l.oracle_argmax.argtypes = [_P, _I]
        l.oracle_argmax.restype = _I
        l.oracle_argmax_ref_order.argtypes = [_P, _I]
        l.oracle_argmax_ref_order.restype = _I
        l.oracle_gemm.argtypes = [_P, _P, _P, _I, _I, _I, _F, _F, _I, _I]
        l.oracle_llama_forward.argtypes = [ctypes.POINTER(OracleConfig), ctypes.POINTER(_P), _P, _P,
                                           _I, _P, _P]
        l.oracle_decode_token.argtypes = [ctypes.POINTER(OracleConfig), ctypes.POINTER(_P), _P, _P,
                                          _I, _I, _P]
        l.oracle_decode_token.restype = _I
        l.oracle_llama_layers.argtypes = [ctypes.POINTER(OracleConfig), ctypes.POINTER(_P), _P, _P,
                                          _I, _P, _I, _P]
        _olib = l
    return _olib


def set_threads(n):
    olib().oracle_set_threads(int(n))


def _p(a):
    return a.ctypes.data


def f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def fill_normal(n, seed, stream, std, round_bf16=False):
    out = np.empty(int(n), dtype=np.float32)
    olib().oracle_fill_normal(_p(out), out.size, seed, stream, std, int(round_bf16))
    return out


def fill_normal_range(n, seed, stream, std, start, round_bf16=False):
    out = np.empty(int(n), dtype=np.float32)
    olib().oracle_fill_normal_range(_p(out), out.size, seed, stream, std, int(round_bf16), start)
    return out


def prompt(n, seed, lo, hi):
    out = np.empty(n, dtype=np.int32)
    olib().oracle_fill_prompt(_p(out), n, seed, lo, hi)
    return out


# ---- per-op wrappers (numpy in, numpy out) ----

def rmsnorm(x, w, batch, hidden, eps):
    x, w = f32(x), f32(w)
    out = np.empty_like(x)
    olib().oracle_rmsnorm(_p(out), _p(x), _p(w), batch, hidden, eps)
    return out


def residual_add(a, b):
    a, b = f32(a), f32(b)
    out = np.empty_like(a)
    olib().oracle_residual_add(_p(out), _p(a), _p(b), a.size)
    return out


def rope(q, k, batch, nq, nkv, D, pos, theta):
    q, k = f32(q).copy(), f32(k).copy()
    olib().oracle_rope(_p(q), _p(k), batch, nq, nkv, D, pos, theta)
    return q, k


def softmax(x, rows, seq_len):
    x = f32(x)
    out = np.empty_like(x)
    olib().oracle_softmax(_p(out), _p(x), rows, seq_len)
    return out


def softmax_with_mask(x, heads, seq_len, total):
    x = f32(x)
    out = np.empty_like(x)
    olib().oracle_softmax_with_mask(_p(out), _p(x), heads, seq_len, total)
    return out


def kv_cache_append(kc, vc, kn, vn, nkv, D, max_seq, pos):
    kc, vc = f32(kc).copy(), f32(vc).copy()
    kn, vn = f32(kn), f32(vn)
    olib().oracle_kv_cache_append(_p(kc), _p(vc), _p(kn), _p(vn), nkv, D, max_seq, pos)
    return kc, vc


def attention_scores(q, kc, nq, nkv, D, seq, max_seq, scale):
    q, kc = f32(q), f32(kc)
    out = np.empty(nq * seq, dtype=np.float32)
    olib().oracle_attention_scores(_p(out), _p(q), _p(kc), nq, nkv, D, seq, max_seq, scale)
    return out


def attention_values(sc, vc, nq, nkv, D, seq, max_seq):
    sc, vc = f32(sc), f32(vc)
    out = np.empty(nq * D, dtype=np.float32)
    olib().oracle_attention_values(_p(out), _p(sc), _p(vc), nq, nkv, D, seq, max_seq)
    return out


def silu_mul(g, u):
    g, u = f32(g), f32(u)
    out = np.empty_like(g)
    olib().oracle_silu_mul(_p(out), _p(g), _p(u), g.size)
    return out


def embedding_lookup(table, token, hidden):
    table = f32(table)
    out = np.empty(hidden, dtype=np.float32)
    olib().oracle_embedding_lookup(_p(out), _p(table), token, hidden)
    return out


def argmax(logits):
    logits = f32(logits)
    return olib().oracle_argmax(_p(logits), logits.size)


def argmax_ref_order(logits):
    logits = f32(logits)
    return olib().oracle_argmax_ref_order(_p(logits), logits.size)


def gemm(A, B, M, N, K, alpha=1.0, beta=0.0, trans_a=0, trans_b=0, C=None):
    A, B = f32(A), f32(B)
    C = np.zeros(M * N, dtype=np.float32) if C is None else f32(C).copy()
    olib().oracle_gemm(_p(A), _p(B), _p(C), M, N, K, alpha, beta, int(trans_a), int(trans_b))
    return C


def round_bf16(a):
    """Round FP32 values to the nearest bf16 value, ties to even (the same
    arithmetic as infernt_round_bf16 in include/infernt_seed.h)."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32).view(np.float32)
    special = (a.view(np.uint32) & 0x7F800000) == 0x7F800000
    return np.where(special, a, r).astype(np.float32)


class LlamaOracle:
    """Seeded model + KV cache on the host; decode steps through oracle.c.

    `cfg` is an infernt_b200.ModelConfig-like object.  Weights follow the
    stream layout of include/infernt_seed.h; `round_bf16` rounds the
    projection matrices and lm_head to bf16 values (the bf16 variant's
    oracle)."""

    def __init__(self, cfg, seed=0, std=0.02, round_bf16=False, layers=None, act_bf16=False):
        self.cfg = cfg
        # the batched-decode variant: bf16 activations into the projections
        # and bf16 KV rows (oracle_set_act_bf16)
        self.act_bf16 = bool(act_bf16)
        c = cfg
        self.L = c.num_layers if layers is None else layers
        H, I, D = c.hidden_size, c.intermediate_size, c.head_dim
        qs, ks = c.num_attention_heads * D, c.num_key_value_heads * D
        rb = bool(round_bf16)
        self.emb = fill_normal(c.vocab_size * H, seed, STREAM_EMBEDDING, std)
        self.final_norm = np.ones(H, dtype=np.float32)
        self.lm_head = fill_normal(c.vocab_size * H, seed, STREAM_LM_HEAD, std, rb)
        self.layers = []
        for l in range(self.L):
            self.layers.append([
                np.ones(H, dtype=np.float32),
                fill_normal(qs * H, seed, stream_layer(l, 0), std, rb),
                fill_normal(ks * H, seed, stream_layer(l, 1), std, rb),
                fill_normal(ks * H, seed, stream_layer(l, 2), std, rb),
                fill_normal(H * qs, seed, stream_layer(l, 3), std, rb),
                np.ones(H, dtype=np.float32),
                fill_normal(I * H, seed, stream_layer(l, 4), std, rb),
                fill_normal(I * H, seed, stream_layer(l, 5), std, rb),
                fill_normal(H * I, seed, stream_layer(l, 6), std, rb),
            ])
        per = c.num_key_value_heads * c.max_seq_len * D
        self.kv_k = np.zeros(self.L * per, dtype=np.float32)
        self.kv_v = np.zeros(self.L * per, dtype=np.float32)
        ptrs = [self.emb, self.final_norm, self.lm_head] + [t for lw in self.layers for t in lw]
        self._ptrs = (_P * len(ptrs))(*[_p(a) for a in ptrs])
        self._c = OracleConfig(c.vocab_size, H, self.L, c.num_attention_heads,
                               c.num_key_value_heads, I, c.max_seq_len, D, c.rms_norm_eps,
                               c.rope_theta)

    def reset(self):
        self.kv_k[:] = 0
        self.kv_v[:] = 0

    def fill_kv(self, seed, n_pos, std=1.0):
        """Rows [0, n_pos) of every layer's caches: element (l, h, p, d) is element
        ((l*Nkv + h) * 2^20 + p) * D + d of the K / V stream (include/infernt_seed.h)."""
        c = self.cfg
        D, nkv, S = c.head_dim, c.num_key_value_heads, c.max_seq_len
        for which, arr, stream in ((0, self.kv_k, STREAM_KV_K), (1, self.kv_v, STREAM_KV_V)):
            view = arr.reshape(self.L, nkv, S, D)
            view[:] = 0
            for l in range(self.L):
                for h in range(nkv):
                    base = ((l * nkv + h) << 20) * D
                    rows = fill_normal_range(n_pos * D, seed, stream, std, base).reshape(n_pos, D)
                    view[l, h, :n_pos, :] = round_bf16(rows) if self.act_bf16 else rows

    def decode_token(self, token, position):
        logits = np.empty(self.cfg.vocab_size, dtype=np.float32)
        olib().oracle_set_act_bf16(int(self.act_bf16))
        nxt = olib().oracle_decode_token(ctypes.byref(self._c), self._ptrs, _p(self.kv_k),
                                         _p(self.kv_v), token, position, _p(logits))
        return nxt, logits

    def forward(self, input_embedding, position):
        x = f32(input_embedding)
        logits = np.empty(self.cfg.vocab_size, dtype=np.float32)
        olib().oracle_llama_forward(ctypes.byref(self._c), self._ptrs, _p(self.kv_k),
                                    _p(self.kv_v), position, _p(x), _p(logits))
        return logits

    def layers_forward(self, input_embedding, position, n_layers):
        x = f32(input_embedding)
        out = np.empty(self.cfg.hidden_size, dtype=np.float32)
        olib().oracle_llama_layers(ctypes.byref(self._c), self._ptrs, _p(self.kv_k),
                                   _p(self.kv_v), position, _p(x), n_layers, _p(out))
        return out


# ---- the reference's own build (GPU; oracle/_ref) ----

_rlib = None


def ref_available():
    return os.path.exists(REF_SO)


def rlib():
    global _rlib
    if _rlib is None:
        if not os.path.exists(REF_SO):
            raise RuntimeError("reference runner %s not built" % REF_SO)
        l = ctypes.CDLL(REF_SO)
        l.ref_last_error.restype = ctypes.c_char_p
        l.ref_arch_create.argtypes = [ctypes.POINTER(_I), ctypes.POINTER(_F), ctypes.c_ulonglong, _F, _I]
        l.ref_arch_create.restype = _P
        l.ref_arch_destroy.argtypes = [_P]
        l.ref_arch_reset.argtypes = [_P]
        l.ref_arch_decode.argtypes = [_P, _I, _I, _P]
        l.ref_arch_decode.restype = _I
        l.ref_arch_prefill_kv.argtypes = [_P, ctypes.c_ulonglong, _I, _F]
        l.ref_engine_create.argtypes = [ctypes.POINTER(_I), ctypes.POINTER(_F), ctypes.c_ulonglong, _F]
        l.ref_engine_create.restype = _P
        l.ref_engine_destroy.argtypes = [_P]
        l.ref_engine_forward_token.argtypes = [_P, _I, _I]
        l.ref_engine_forward_token.restype = _I
        l.ref_engine_sample_next_token.argtypes = [_P]
        l.ref_engine_sample_next_token.restype = _I
        l.ref_engine_decode_loop.argtypes = [_P, _I, _I, _I, _P]
        l.ref_engine_decode_loop.restype = _F
        _rlib = l
    return _rlib


def _cfg_arrays(cfg):
    ci = (_I * 8)(cfg.vocab_size, cfg.hidden_size, cfg.num_layers, cfg.num_attention_heads,
                  cfg.num_key_value_heads, cfg.intermediate_size, cfg.max_seq_len, cfg.head_dim)
    cf = (_F * 2)(cfg.rms_norm_eps, cfg.rope_theta)
    return ci, cf


class RefArch:
    """The reference's LlamaArchitecture + KVCache with seeded weights (GPU)."""

    def __init__(self, cfg, seed=0, std=0.02, round_bf16=False):
        self.cfg = cfg
        ci, cf = _cfg_arrays(cfg)
        self._h = rlib().ref_arch_create(ci, cf, seed, std, int(round_bf16))
        if not self._h:
            raise RuntimeError("ref_arch_create: " + rlib().ref_last_error().decode())

    def close(self):
        if self._h:
            rlib().ref_arch_destroy(self._h)
            self._h = None

    def reset(self):
        rlib().ref_arch_reset(self._h)

    def prefill_kv(self, seed, n_pos, std=1.0):
        rlib().ref_arch_prefill_kv(self._h, seed, n_pos, std)

    def decode(self, token, position):
        logits = np.empty(self.cfg.vocab_size, dtype=np.float32)
        t = rlib().ref_arch_decode(self._h, token, position, _p(logits))
        if t < 0:
            raise RuntimeError("ref_arch_decode: " + rlib().ref_last_error().decode())
        return t, logits


class RefEngine:
    """The reference's InferenceEngine with seeded weights (GPU)."""

    def __init__(self, cfg, seed=0, std=0.02):
        self.cfg = cfg
        ci, cf = _cfg_arrays(cfg)
        self._h = rlib().ref_engine_create(ci, cf, seed, std)
        if not self._h:
            raise RuntimeError("ref_engine_create: " + rlib().ref_last_error().decode())

    def close(self):
        if self._h:
            rlib().ref_engine_destroy(self._h)
            self._h = None

    def forward_token(self, token, position):
        return rlib().ref_engine_forward_token(self._h, token, position)

    def decode_loop(self, token, position, steps):
        toks = np.zeros(max(steps, 1), dtype=np.int32)
        ms = rlib().ref_engine_decode_loop(self._h, token, position, steps, _p(toks))
        if ms < 0:
            raise RuntimeError("ref_engine_decode_loop: " + rlib().ref_last_error().decode())
        return toks[:steps].tolist(), ms
