"""infernt_b200 — B200-native decode step of INFERNT behind a C ABI.

The product is the shared library ``infernt_b200/lib/libinfernt_b200.so``
(CUDA kernels for sm_100a, the C ABI of ``include/infernt_capi.h`` and the
C++ drop-in classes of ``include/*.h``).  This module binds it with ctypes
for Python callers (tests, the benchmark).  Importing never falls back to
anything: if the library is missing, ``lib()`` raises.

Configurations follow the reference's ``ModelConfig`` (include/config.h).
"""
import ctypes
import os
from dataclasses import dataclass, replace

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libinfernt_b200.so")

DTYPE_F32 = 0
DTYPE_BF16 = 1

# Phase-timeline fields (infernt_plan_set_trace): phase start, input loaded,
# work done, barrier passed, producer issued last tile (ns); consumer wait
# cycles, producer wait cycles; thread 0's input words current, input and
# constants in shared memory (ns).
TRACE_FIELDS = 9

MODE_EAGER = 0
MODE_GRAPH = 1
MODE_PERSISTENT = 2

STATUS = {0: "ok", 1: "invalid argument", 2: "unsupported", 3: "CUDA error",
          4: "out of device memory", 5: "device-side error", 6: "no usable CUDA device"}


class InferntError(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, status, what, detail):
        super().__init__("%s: %s (%s)" % (what, STATUS.get(status, status), detail))
        self.status = status


class LlamaConfig(ctypes.Structure):
    """``infernt_llama_config`` (include/infernt_capi.h)."""
    _fields_ = [("vocab_size", ctypes.c_int), ("hidden_size", ctypes.c_int),
                ("num_layers", ctypes.c_int), ("num_attention_heads", ctypes.c_int),
                ("num_key_value_heads", ctypes.c_int), ("intermediate_size", ctypes.c_int),
                ("max_seq_len", ctypes.c_int), ("head_dim", ctypes.c_int),
                ("rms_norm_eps", ctypes.c_float), ("rope_theta", ctypes.c_float),
                ("weight_dtype", ctypes.c_int)]


@dataclass(frozen=True)
class ModelConfig:
    """Hyper-parameters of a LLaMA-family decoder (reference include/config.h:22-46)."""
    vocab_size: int
    hidden_size: int
    num_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    intermediate_size: int
    max_seq_len: int
    head_dim: int = 0
    rms_norm_eps: float = 1e-5
    rope_theta: float = 10000.0
    weight_dtype: int = DTYPE_F32

    def __post_init__(self):
        if self.head_dim == 0:
            object.__setattr__(self, "head_dim", self.hidden_size // self.num_attention_heads)

    def c(self):
        return LlamaConfig(self.vocab_size, self.hidden_size, self.num_layers,
                           self.num_attention_heads, self.num_key_value_heads,
                           self.intermediate_size, self.max_seq_len, self.head_dim,
                           self.rms_norm_eps, self.rope_theta, self.weight_dtype)

    def ints(self):
        return [self.vocab_size, self.hidden_size, self.num_layers, self.num_attention_heads,
                self.num_key_value_heads, self.intermediate_size, self.max_seq_len, self.head_dim]

    def with_(self, **kw):
        return replace(self, **kw)

    @property
    def weight_params(self):
        """Parameters streamed per decode step (all weights except the embedding table)."""
        H, I, L, V = self.hidden_size, self.intermediate_size, self.num_layers, self.vocab_size
        qs = self.num_attention_heads * self.head_dim
        kvs = self.num_key_value_heads * self.head_dim
        per_layer = H * (qs + 2 * kvs) + qs * H + 3 * H * I
        return L * per_layer + V * H


# TinyLlama-1.1B shape (FP32 batch-1 greedy decode workload)
TINYLLAMA = ModelConfig(vocab_size=32000, hidden_size=2048, num_layers=22, num_attention_heads=32,
                        num_key_value_heads=4, intermediate_size=5632, max_seq_len=2048,
                        rms_norm_eps=1e-5, rope_theta=10000.0)
# Llama-3-8B shape (bf16 decode workload)
LLAMA3_8B = ModelConfig(vocab_size=128256, hidden_size=4096, num_layers=32, num_attention_heads=32,
                        num_key_value_heads=8, intermediate_size=14336, max_seq_len=8192,
                        rms_norm_eps=1e-5, rope_theta=500000.0, weight_dtype=DTYPE_BF16)

_lib = None

_P = ctypes.c_void_p
_I = ctypes.c_int
_F = ctypes.c_float
_S = ctypes.c_size_t
_U64 = ctypes.c_uint64

_SIGS = {
    "infernt_status_string": (ctypes.c_char_p, [_I]),
    "infernt_last_error": (ctypes.c_char_p, []),
    "infernt_version": (_I, []),
    "infernt_rmsnorm": (_I, [_P, _P, _P, _I, _I, _F, _P]),
    "infernt_residual_add": (_I, [_P, _P, _P, _I, _P]),
    "infernt_rope": (_I, [_P, _P, _I, _I, _I, _I, _I, _F, _P]),
    "infernt_softmax": (_I, [_P, _P, _I, _I, _P]),
    "infernt_softmax_with_mask": (_I, [_P, _P, _I, _I, _I, _P]),
    "infernt_kv_cache_append": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _P]),
    "infernt_attention_scores": (_I, [_P, _P, _P, _I, _I, _I, _I, _I, _F, _P]),
    "infernt_attention_values": (_I, [_P, _P, _P, _I, _I, _I, _I, _I, _P]),
    "infernt_silu_mul": (_I, [_P, _P, _P, _I, _P]),
    "infernt_embedding_lookup": (_I, [_P, _P, _I, _I, _P]),
    "infernt_argmax": (_I, [_P, _P, _I, _P]),
    "infernt_gemm_f32": (_I, [_P, _P, _P, _I, _I, _I, _F, _F, _I, _I, _P]),
    "infernt_rmsnorm_gemv": (_I, [_P, _P, _I, _P, _I, _P, _I, _I, _I, _P, _P, _F, _P]),
    "infernt_gemv_residual": (_I, [_P, _P, _P, _I, _I, _I, _P, _P]),
    "infernt_rmsnorm_gate_up_silu": (_I, [_P, _P, _P, _I, _I, _I, _P, _P, _F, _P]),
    "infernt_attention_workspace_bytes": (_S, [_I, _I, _I, _I]),
    "infernt_attention_decode": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _I, _F, _I, _P, _P]),
    "infernt_attention_decode_noalloc": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _I, _F, _I, _P]),
    "infernt_lm_head_workspace_bytes": (_S, []),
    "infernt_rmsnorm_lm_head_argmax": (_I, [_P, _P, _P, _I, _I, _I, _P, _P, _F, _P, _P]),
    "infernt_bgemm_bf16": (_I, [_P, _I, _I, _P, _I, _P, _I, _P, _P]),
    "infernt_batch_engine_create_seeded": (_I, [ctypes.POINTER(LlamaConfig), _I, _U64, _F, _I, ctypes.POINTER(_P)]),
    "infernt_batch_engine_destroy": (_I, [_P]),
    "infernt_batch_engine_fill_kv": (_I, [_P, _I, _U64, _I, _F]),
    "infernt_batch_engine_step": (_I, [_P, _P, _P, _P]),
    "infernt_batch_engine_decode": (_I, [_P, _P, _P, _I, _P, ctypes.POINTER(_F)]),
    "infernt_batch_engine_logits": (_I, [_P, _P, _S]),
    "infernt_batch_engine_splits": (_I, [_P, _P]),
    "infernt_batch_engine_set_attention": (_I, [_P, _I, _I, _I]),
    "infernt_batch_attention": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I, _P, _P, _P, _P]),
    "infernt_batch_engine_prefill": (_I, [_P, _I, _P, _I, _I, _I, _P, _P, _P]),
    "infernt_batch_engine_create_tp": (_I, [_P, _I, ctypes.c_uint64, _F, _I, _I, _I, _P, _P]),
    "infernt_nccl_unique_id": (_I, [_P, ctypes.c_size_t]),
    "infernt_batch_engine_vocab_range": (_I, [_P, _P, _P]),
    "infernt_batch_engine_set_sampling": (_I, [_P, _F, ctypes.c_uint64]),
    "infernt_batch_engine_set_tp_exchange": (_I, [_P, _I]),
    "infernt_sample_workspace_bytes": (_S, [_I]),
    "infernt_engine_set_device_sampling": (_I, [_P, _I, ctypes.c_uint64]),
    "infernt_engine_set_step_temperature": (_I, [_P, _F]),
    "infernt_plan_set_sampling": (_I, [_P, _F, ctypes.c_uint64]),
    "infernt_engine_load_model": (_I, [ctypes.c_char_p, _I, _P]),
    "infernt_sample_tokens": (_I, [_P, ctypes.c_longlong, _I, _I, _F, ctypes.c_uint64, ctypes.c_uint64, _P, _P,
                                   _P]),
    "infernt_checkpoint_read_config": (_I, [ctypes.c_char_p, ctypes.POINTER(LlamaConfig)]),
    "infernt_checkpoint_load": (_I, [ctypes.c_char_p, ctypes.POINTER(LlamaConfig), _I, _P]),
    "infernt_checkpoint_weights": (_I, [_P, ctypes.POINTER(_P), _I]),
    "infernt_checkpoint_free": (_I, [_P]),
    "infernt_batch_engine_read_kv": (_I, [_P, _I, _I, _I, _P, _P]),
    "infernt_batch_engine_create_paged": (_I, [_P, _I, _I, _I, _U64, _F, _I, _P]),
    "infernt_batch_engine_set_pages": (_I, [_P, _I, _P, _I]),
    "infernt_batch_engine_paging": (_I, [_P, _P, _P, _P]),
    "infernt_batch_engine_set_salts": (_I, [_P, _P]),
    "infernt_scheduler_create": (_I, [_I, _I, _I, _I, _P]),
    "infernt_scheduler_destroy": (_I, [_P]),
    "infernt_scheduler_submit": (_I, [_P, _P, _I, _I, _I, _P]),
    "infernt_scheduler_cancel": (_I, [_P, ctypes.c_int64]),
    "infernt_scheduler_plan": (_I, [_P, _P]),
    "infernt_scheduler_commit": (_I, [_P, _P, _P]),
    "infernt_scheduler_result": (_I, [_P, ctypes.c_int64, _P, _I, _P, _P, _P]),
    "infernt_scheduler_release": (_I, [_P, ctypes.c_int64]),
    "infernt_scheduler_stats": (_I, [_P, _P]),
    "infernt_server_create_seeded": (_I, [_P, _I, _I, _I, _U64, _F, _P]),
    "infernt_server_destroy": (_I, [_P]),
    "infernt_server_submit": (_I, [_P, _P, _I, _I, _I, _P]),
    "infernt_server_step": (_I, [_P, _P]),
    "infernt_server_run": (_I, [_P, _P]),
    "infernt_server_result": (_I, [_P, ctypes.c_int64, _P, _I, _P, _P, _P]),
    "infernt_server_stats": (_I, [_P, _P]),
    "infernt_server_set_sampling": (_I, [_P, _F, _U64]),
    "infernt_server_engine": (_I, [_P, _P]),
    "infernt_pgemm_bf16": (_I, [_P, _I, _I, _P, _I, _P, _I, _P, _P]),
    "infernt_pgemm_swiglu_bf16": (_I, [_P, _I, _I, _P, _I, _P, _I, _P, _P]),
    "infernt_prefill_attention": (_I, [_P, _P, _P, _I, _I, _I, _I, _I, _I, _P, _P, _I, _P]),
    "infernt_plan_create": (_I, [ctypes.POINTER(LlamaConfig), ctypes.POINTER(_P),
                                 ctypes.POINTER(_P), ctypes.POINTER(_P), _I, ctypes.POINTER(_P)]),
    "infernt_plan_destroy": (_I, [_P]),
    "infernt_plan_forward": (_I, [_P, _P, _I, _P, _P]),
    "infernt_plan_decode": (_I, [_P, _I, _I, _P, _P]),
    "infernt_plan_decode_chain": (_I, [_P, _I, _I, _I, _P, _P]),
    "infernt_plan_read_token": (_I, [_P, ctypes.POINTER(_I), _P]),
    "infernt_plan_logits": (_P, [_P]),
    "infernt_plan_kernels_per_step": (_I, [_P]),
    "infernt_plan_mode": (_I, [_P]),
    "infernt_plan_trace_entries": (_S, [_P, _I]),
    "infernt_plan_set_trace": (_I, [_P, _P]),
    "infernt_persistent_ctas": (_I, []),
    "infernt_engine_trace_chain": (_I, [_P, _I, _I, _I, _P, _S]),
    "infernt_engine_set_mode": (_I, [_P, _I]),
    "infernt_engine_mode": (_I, [_P, ctypes.POINTER(_I)]),
    "infernt_fill_normal": (_I, [_P, _S, _I, _U64, _U64, _F, _P]),
    "infernt_fill_const": (_I, [_P, _S, _F, _P]),
    "infernt_fill_prompt": (_I, [_P, _I, _U64, _I, _I]),
    "infernt_fill_kv": (_I, [ctypes.POINTER(_P), ctypes.POINTER(_P), _I, _I, _I, _I, _I, _U64, _F, _P]),
    "infernt_engine_create_seeded": (_I, [ctypes.POINTER(LlamaConfig), _U64, _F, ctypes.POINTER(_P)]),
    "infernt_engine_destroy": (_I, [_P]),
    "infernt_engine_reset": (_I, [_P]),
    "infernt_engine_forward_token": (_I, [_P, _I, _I, ctypes.POINTER(_I)]),
    "infernt_engine_sample_next_token": (_I, [_P, _F, ctypes.POINTER(_I)]),
    "infernt_engine_logits": (_I, [_P, _P]),
    "infernt_engine_fill_kv": (_I, [_P, _U64, _I, _F]),
    "infernt_engine_decode_chain": (_I, [_P, _I, _I, _I, _P, ctypes.POINTER(_F)]),
    "infernt_engine_weight_ptrs": (_I, [_P, ctypes.POINTER(_P), _I]),
    "infernt_engine_kv_ptrs": (_I, [_P, ctypes.POINTER(_P), ctypes.POINTER(_P), _I]),
    "infernt_fill_normal_window": (_I, [_P, _I, _I, _I, _U64, _U64, _U64, _I, _U64, _U64, _F, _P]),
    "infernt_tp_shard_dims": (_I, [ctypes.POINTER(LlamaConfig), _I, _I, ctypes.POINTER(_I)]),
    "infernt_plan_create_tp": (_I, [ctypes.POINTER(LlamaConfig), ctypes.POINTER(_P), ctypes.POINTER(_P),
                                    ctypes.POINTER(_P), _I, _I, ctypes.POINTER(_P)]),
    "infernt_plan_xchg_handle": (_I, [_P, _P]),
    "infernt_plan_set_peers": (_I, [_P, _P]),
    "infernt_tp_engine_create_seeded": (_I, [ctypes.POINTER(LlamaConfig), _U64, _F, _I, _I, ctypes.POINTER(_P)]),
    "infernt_tp_engine_destroy": (_I, [_P]),
    "infernt_tp_engine_xchg_handle": (_I, [_P, _P]),
    "infernt_tp_engine_set_peers": (_I, [_P, _P]),
    "infernt_tp_engine_forward_token": (_I, [_P, _I, _I, ctypes.POINTER(_I)]),
    "infernt_tp_engine_decode_chain": (_I, [_P, _I, _I, _I, _P, ctypes.POINTER(_F)]),
    "infernt_tp_engine_logits": (_I, [_P, _P, _I]),
    "infernt_tp_engine_dims": (_I, [_P, ctypes.POINTER(_I)]),
    "infernt_tp_engine_trace_chain": (_I, [_P, _I, _I, _I, _P, _S]),
    "infernt_tp_engine_plan": (_I, [_P, ctypes.POINTER(_P)]),
    "infernt_plan_xchg_bytes": (_I, [_P, ctypes.POINTER(_S)]),
    "infernt_plan_xchg_region": (_P, [_P]),
    "infernt_plan_set_peer_regions": (_I, [_P, ctypes.POINTER(_P)]),
    "infernt_plan_set_wait_budget": (_I, [_P, ctypes.c_longlong]),
    "infernt_plan_set_stream_depth": (_I, [_P, _I]),
    "infernt_plan_stream_depth": (_I, [_P, _P, _P]),
}

IPC_HANDLE_BYTES = 64


def exported_symbols():
    """Names of the C-ABI entry points this module binds."""
    return sorted(_SIGS)


def lib():
    """The loaded product library (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError("%s is missing: run `python -m infernt_b200.build` (or "
                               "__graft_entry__.build())" % LIB_PATH)
        l = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            f = getattr(l, name)
            f.restype = res
            f.argtypes = args
        _lib = l
    return _lib


def check(status, what):
    if status != 0:
        raise InferntError(status, what, lib().infernt_last_error().decode())
    return status


def call(name, *args):
    """Calls a C-ABI entry point and raises InferntError on a non-zero status."""
    return check(getattr(lib(), name)(*args), name)


def _trace(cfg, fn, handle, token, position, steps):
    """Runs a traced decode chain through `fn`; [cta][step][phase][TRACE_FIELDS] int64."""
    import numpy as np
    nph = 5 * cfg.num_layers + 1
    ctas = lib().infernt_persistent_ctas()
    out = np.zeros(ctas * steps * nph * TRACE_FIELDS, dtype=np.uint64)
    call(fn, handle, token, position, steps, out.ctypes.data, out.size)
    return out.reshape(ctas, steps, nph, TRACE_FIELDS).astype(np.int64)


def prompt(n: int, seed: int, lo: int = 3, hi: int = 32000):
    """n seeded token ids uniform in [lo, hi) (infernt_fill_prompt): the
    synthetic prompts of the benchmarks."""
    arr = (ctypes.c_int * max(int(n), 1))()
    call("infernt_fill_prompt", arr, int(n), int(seed), int(lo), int(hi))
    return [arr[i] for i in range(int(n))]


def ptr(t):
    """Device pointer of a torch tensor (or pass an int through)."""
    if t is None:
        return None
    if isinstance(t, int):
        return t
    return t.data_ptr()


class Engine:
    """The C++ InferenceEngine (include/engine.h) through its C entry points,
    with seeded synthetic weights (include/infernt_seed.h)."""

    def __init__(self, cfg: ModelConfig, seed: int = 0, std: float = 0.02):
        self.cfg = cfg
        h = ctypes.c_void_p()
        call("infernt_engine_create_seeded", ctypes.byref(cfg.c()), seed, std, ctypes.byref(h))
        self._h = h

    def close(self):
        if self._h:
            lib().infernt_engine_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def reset(self):
        call("infernt_engine_reset", self._h)

    def set_mode(self, mode: int):
        """MODE_EAGER / MODE_GRAPH / MODE_PERSISTENT for the following steps."""
        call("infernt_engine_set_mode", self._h, mode)

    @property
    def mode(self) -> int:
        out = ctypes.c_int()
        call("infernt_engine_mode", self._h, ctypes.byref(out))
        return out.value

    def forward_token(self, token: int, position: int) -> int:
        out = ctypes.c_int()
        call("infernt_engine_forward_token", self._h, token, position, ctypes.byref(out))
        return out.value

    def sample_next_token(self, temperature: float = 0.0) -> int:
        out = ctypes.c_int()
        call("infernt_engine_sample_next_token", self._h, temperature, ctypes.byref(out))
        return out.value

    def set_device_sampling(self, on: bool = True, seed: int = 1337):
        """Temperature sampling on the GPU (Gumbel-max, the default) or, with
        on=False, the reference's host sampler."""
        call("infernt_engine_set_device_sampling", self._h, int(on), seed)

    def set_step_temperature(self, temperature: float):
        """Following steps draw their token at this temperature inside the
        decode kernel (0: greedy)."""
        call("infernt_engine_set_step_temperature", self._h, float(temperature))

    @classmethod
    def load_model(cls, model_dir: str, weight_dtype: int = -1) -> "Engine":
        """InferenceEngine::load_model of a converted checkpoint directory
        (config.json, model.bin, tokenizer.bin)."""
        cfg = Checkpoint.read_config(model_dir + "/config.json")
        if weight_dtype >= 0:
            cfg = cfg.with_(weight_dtype=weight_dtype)
        e = cls.__new__(cls)
        e.cfg = cfg
        h = ctypes.c_void_p()
        call("infernt_engine_load_model", model_dir.encode(), weight_dtype, ctypes.byref(h))
        e._h = h
        return e

    def logits(self):
        import numpy as np
        out = np.empty(self.cfg.vocab_size, dtype=np.float32)
        call("infernt_engine_logits", self._h, out.ctypes.data)
        return out

    def fill_kv(self, seed: int, n_pos: int, std: float = 1.0):
        call("infernt_engine_fill_kv", self._h, seed, n_pos, std)

    def decode_chain(self, token: int, position: int, steps: int):
        """Device-chained greedy decode; returns (tokens, device ms)."""
        import numpy as np
        toks = np.zeros(max(steps, 1), dtype=np.int32)
        ms = ctypes.c_float()
        call("infernt_engine_decode_chain", self._h, token, position, steps, toks.ctypes.data,
             ctypes.byref(ms))
        return toks[:steps].tolist(), ms.value

    def trace_chain(self, token: int, position: int, steps: int):
        """Device-chained decode with the persistent kernel's phase timeline.
        Returns an int64 array [cta][step][phase][9] over every CTA of the
        launch: %globaltimer ns of phase start, input loaded, work done,
        barrier passed, producer issued the phase's last slot; then the SM
        cycles the CTA's first consumer waited for slots and its producer
        for free ones."""
        return _trace(self.cfg, "infernt_engine_trace_chain", self._h, token, position, steps)

    def weight_ptrs(self):
        n = 3 + 9 * self.cfg.num_layers
        arr = (ctypes.c_void_p * n)()
        call("infernt_engine_weight_ptrs", self._h, arr, n)
        return [arr[i] for i in range(n)]

    def kv_ptrs(self):
        n = self.cfg.num_layers
        k = (ctypes.c_void_p * n)()
        v = (ctypes.c_void_p * n)()
        call("infernt_engine_kv_ptrs", self._h, k, v, n)
        return [k[i] for i in range(n)], [v[i] for i in range(n)]


class BatchEngine:
    """T sequences decoding together on the tensor cores
    (infernt_batch_engine_*): seeded bf16 weights, bf16 KV caches."""

    def __init__(self, cfg: ModelConfig, batch: int, seed: int = 0, std: float = 0.02, attn_splits: int = 0,
                 rank: int = 0, world: int = 1, nccl_id: bytes = None, pages=None, _handle=None):
        """world > 1: one rank of a tensor-parallel engine
        (infernt_batch_engine_create_tp); every rank passes the same nccl_id
        (nccl_unique_id() on one rank) and all ranks call every method in the
        same order.  pages=(page_size, num_pages): paged KV caches
        (infernt_batch_engine_create_paged; set_pages gives each sequence its
        pages)."""
        self.cfg = cfg
        self.T = batch
        self.world = world
        self._c = cfg.c()
        self._owned = _handle is None
        if _handle is not None:
            self._h = _handle
        else:
            h = ctypes.c_void_p()
            if pages is not None:
                call("infernt_batch_engine_create_paged", ctypes.byref(self._c), batch, pages[0], pages[1], seed,
                     std, attn_splits, ctypes.byref(h))
            else:
                idbuf = None
                if nccl_id is not None:
                    idbuf = ctypes.create_string_buffer(bytes(nccl_id), len(nccl_id))
                call("infernt_batch_engine_create_tp", ctypes.byref(self._c), batch, seed, std, attn_splits, rank,
                     world, idbuf, ctypes.byref(h))
            self._h = h
        v0, vl = ctypes.c_int(), ctypes.c_int()
        call("infernt_batch_engine_vocab_range", self._h, ctypes.byref(v0), ctypes.byref(vl))
        self.vocab_range = (v0.value, v0.value + vl.value)

    def close(self):
        if self._h:
            if self._owned:
                lib().infernt_batch_engine_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_pages(self, seq: int, pages):
        """Pages of sequence `seq` for its positions [0, len(pages) x page_size)."""
        arr = (ctypes.c_int * max(1, len(pages)))(*[int(p) for p in pages])
        call("infernt_batch_engine_set_pages", self._h, seq, arr, len(pages))

    def paging(self):
        """(page_size, num_pages, max_pages per sequence); zeros when contiguous."""
        a, b, c = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
        call("infernt_batch_engine_paging", self._h, ctypes.byref(a), ctypes.byref(b), ctypes.byref(c))
        return a.value, b.value, c.value

    def set_salts(self, salts):
        """Per-sequence sampling salts (None: none)."""
        if salts is None:
            call("infernt_batch_engine_set_salts", self._h, None)
            return
        arr = (ctypes.c_uint64 * self.T)(*[int(x) for x in salts])
        call("infernt_batch_engine_set_salts", self._h, arr)

    def fill_kv(self, seq: int, seed: int, n_pos: int, std: float = 1.0):
        call("infernt_batch_engine_fill_kv", self._h, seq, seed, n_pos, std)

    def _ints(self, xs):
        arr = (ctypes.c_int * self.T)(*[int(x) for x in xs])
        return arr

    def step(self, tokens, positions):
        out = (ctypes.c_int * self.T)()
        call("infernt_batch_engine_step", self._h, self._ints(tokens), self._ints(positions), out)
        return list(out)

    def decode(self, tokens, positions, steps: int):
        import numpy as np
        out = np.zeros(steps * self.T, dtype=np.int32)
        ms = ctypes.c_float()
        call("infernt_batch_engine_decode", self._h, self._ints(tokens), self._ints(positions), steps,
             out.ctypes.data, ctypes.byref(ms))
        return out.reshape(steps, self.T), ms.value

    def logits(self):
        """The last step's logits [T][vocabulary rows of this rank]."""
        import numpy as np
        out = np.empty((self.T, self.vocab_range[1] - self.vocab_range[0]), dtype=np.float32)
        call("infernt_batch_engine_logits", self._h, out.ctypes.data, out.size)
        return out

    def prefill(self, seq: int, tokens, start_pos: int = 0, chunk: int = 0, want_logits: bool = False):
        """Prompt prefill of sequence `seq` (infernt_batch_engine_prefill):
        writes its K/V rows of positions [start_pos, start_pos + len(tokens))
        and returns (greedy next token, last token's logits or None, device
        ms).  Tensor-parallel ranks all call it with the same arguments; the
        logits are then this rank's vocabulary rows (vocab_range)."""
        import numpy as np
        toks = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32))
        nxt = ctypes.c_int()
        ms = ctypes.c_float()
        logits = np.empty(self.cfg.vocab_size, dtype=np.float32) if want_logits else None
        call("infernt_batch_engine_prefill", self._h, seq, toks.ctypes.data, toks.size, start_pos, chunk,
             ctypes.byref(nxt), None if logits is None else logits.ctypes.data, ctypes.byref(ms))
        if logits is not None:
            logits = logits[:self.vocab_range[1] - self.vocab_range[0]].copy()
        return nxt.value, logits, ms.value

    def read_kv(self, seq: int, layer: int, n_pos: int):
        """Rows [0, n_pos) of the sequence's K and V caches of one layer as
        float32 arrays [nkv][n_pos][head_dim] (exact bf16 values; a
        tensor-parallel rank's own KV heads)."""
        import numpy as np
        shape = (self.cfg.num_key_value_heads // self.world, n_pos, self.cfg.head_dim)
        k = np.zeros(shape, dtype=np.uint16)
        v = np.zeros(shape, dtype=np.uint16)
        call("infernt_batch_engine_read_kv", self._h, seq, layer, n_pos, k.ctypes.data, v.ctypes.data)
        widen = lambda a: (a.astype(np.uint32) << 16).view(np.float32)
        return widen(k), widen(v)

    def set_sampling(self, temperature: float, seed: int = 0):
        """Temperature sampling (Gumbel-max in the argmax kernels) for the
        following steps; temperature 0 is greedy."""
        call("infernt_batch_engine_set_sampling", self._h, temperature, seed)

    def set_tp_exchange(self, peer: bool):
        """Tensor parallelism: sums cross the ranks by the peer-memory exchange
        (True, the default) or by ncclAllReduce (False)."""
        call("infernt_batch_engine_set_tp_exchange", self._h, 1 if peer else 0)

    def splits(self):
        out = (ctypes.c_int * 6)()
        call("infernt_batch_engine_splits", self._h, out)
        return list(out)

    def set_attention(self, splits: int, min_chunk: int, stages: int):
        """KV splits per (sequence, KV head), least positions per split and
        copy stages per warp of the attention; results do not change."""
        call("infernt_batch_engine_set_attention", self._h, splits, min_chunk, stages)


class SchedPlan(ctypes.Structure):
    """``infernt_sched_plan`` (include/infernt_capi.h)."""
    _fields_ = [("n_prefill", ctypes.c_int), ("prefill_slot", ctypes.POINTER(ctypes.c_int)),
                ("prefill_offset", ctypes.POINTER(ctypes.c_int)), ("prefill_len", ctypes.POINTER(ctypes.c_int)),
                ("prefill_tokens", ctypes.POINTER(ctypes.c_int)), ("n_decode", ctypes.c_int),
                ("tokens", ctypes.POINTER(ctypes.c_int)), ("positions", ctypes.POINTER(ctypes.c_int)),
                ("n_changed", ctypes.c_int), ("changed_slot", ctypes.POINTER(ctypes.c_int)),
                ("pages", ctypes.POINTER(ctypes.c_int)), ("n_pages", ctypes.POINTER(ctypes.c_int)),
                ("max_pages", ctypes.c_int), ("n_preempted", ctypes.c_int)]


class SchedStats(ctypes.Structure):
    """``infernt_sched_stats`` (include/infernt_capi.h)."""
    _fields_ = [("waiting", ctypes.c_int), ("running", ctypes.c_int), ("finished", ctypes.c_int),
                ("free_pages", ctypes.c_int), ("steps", ctypes.c_longlong), ("preemptions", ctypes.c_longlong),
                ("prefill_tokens", ctypes.c_longlong), ("decode_tokens", ctypes.c_longlong)]

    def as_dict(self):
        return {f: getattr(self, f) for f, _ in self._fields_}


REQUEST_STATES = {0: "waiting", 1: "running", 2: "finished", 3: "cancelled"}


def _request_result(fn, handle, rid):
    n, state, pre = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    call(fn, handle, rid, None, 0, ctypes.byref(n), ctypes.byref(state), ctypes.byref(pre))
    buf = (ctypes.c_int * max(1, n.value))()
    call(fn, handle, rid, buf, n.value, ctypes.byref(n), ctypes.byref(state), ctypes.byref(pre))
    return list(buf[:n.value]), REQUEST_STATES[state.value], pre.value


class Scheduler:
    """Iteration-level scheduler over paged KV (infernt_scheduler_*; host
    logic only): plan() gives a step's prefills, decode inputs and page
    tables, commit() takes the step's tokens."""

    def __init__(self, slots: int, page_size: int, num_pages: int, max_seq_len: int):
        h = ctypes.c_void_p()
        call("infernt_scheduler_create", slots, page_size, num_pages, max_seq_len, ctypes.byref(h))
        self._h = h
        self.slots = slots

    def close(self):
        if self._h:
            lib().infernt_scheduler_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def submit(self, prompt, max_new_tokens: int, eos: int = -1) -> int:
        arr = (ctypes.c_int * len(prompt))(*[int(t) for t in prompt])
        rid = ctypes.c_int64()
        call("infernt_scheduler_submit", self._h, arr, len(prompt), max_new_tokens, eos, ctypes.byref(rid))
        return rid.value

    def cancel(self, rid: int):
        call("infernt_scheduler_cancel", self._h, rid)

    def plan(self):
        """The next step as a dict of Python lists."""
        p = SchedPlan()
        call("infernt_scheduler_plan", self._h, ctypes.byref(p))
        S, mp = self.slots, p.max_pages
        ntok = sum(p.prefill_len[i] for i in range(p.n_prefill))
        return {
            "prefill": [(p.prefill_slot[i],
                         [p.prefill_tokens[p.prefill_offset[i] + j] for j in range(p.prefill_len[i])])
                        for i in range(p.n_prefill)],
            "prefill_tokens": ntok,
            "n_decode": p.n_decode,
            "tokens": [p.tokens[i] for i in range(S)],
            "positions": [p.positions[i] for i in range(S)],
            "changed": [p.changed_slot[i] for i in range(p.n_changed)],
            "pages": [[p.pages[i * mp + j] for j in range(p.n_pages[i])] for i in range(S)],
            "max_pages": mp,
            "n_preempted": p.n_preempted,
        }

    def commit(self, prefill_next, decode_next):
        a = (ctypes.c_int * max(1, len(prefill_next)))(*[int(t) for t in prefill_next])
        b = (ctypes.c_int * self.slots)(*[int(t) for t in decode_next])
        call("infernt_scheduler_commit", self._h, a, b)

    def result(self, rid: int):
        """(generated tokens, state name, preemptions)."""
        return _request_result("infernt_scheduler_result", self._h, rid)

    def release(self, rid: int):
        call("infernt_scheduler_release", self._h, rid)

    def stats(self):
        st = SchedStats()
        call("infernt_scheduler_stats", self._h, ctypes.byref(st))
        return st.as_dict()


class Server:
    """Continuous batching on a paged batched engine (infernt_server_*)."""

    def __init__(self, cfg: ModelConfig, slots: int, page_size: int, num_pages: int, seed: int = 0,
                 std: float = 0.02):
        self.cfg = cfg
        self._c = cfg.c()
        h = ctypes.c_void_p()
        call("infernt_server_create_seeded", ctypes.byref(self._c), slots, page_size, num_pages, seed, std,
             ctypes.byref(h))
        self._h = h
        e = ctypes.c_void_p()
        call("infernt_server_engine", self._h, ctypes.byref(e))
        self.engine = BatchEngine(cfg, slots, _handle=e)
        self.slots = slots

    def close(self):
        if self._h:
            self.engine.close()
            lib().infernt_server_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def submit(self, prompt, max_new_tokens: int, eos: int = -1) -> int:
        arr = (ctypes.c_int * len(prompt))(*[int(t) for t in prompt])
        rid = ctypes.c_int64()
        call("infernt_server_submit", self._h, arr, len(prompt), max_new_tokens, eos, ctypes.byref(rid))
        return rid.value

    def step(self) -> int:
        n = ctypes.c_int()
        call("infernt_server_step", self._h, ctypes.byref(n))
        return n.value

    def run(self) -> float:
        """Steps until every request finished; host milliseconds."""
        ms = ctypes.c_double()
        call("infernt_server_run", self._h, ctypes.byref(ms))
        return ms.value

    def result(self, rid: int):
        return _request_result("infernt_server_result", self._h, rid)

    def stats(self):
        st = SchedStats()
        call("infernt_server_stats", self._h, ctypes.byref(st))
        return st.as_dict()

    def set_sampling(self, temperature: float, seed: int = 0):
        call("infernt_server_set_sampling", self._h, temperature, seed)


class Checkpoint:
    """An INFT v1 checkpoint (infernt_checkpoint_*): config.json read into a
    ModelConfig, model.bin into one buffer per tensor on the host (device=0)
    or the current CUDA device (device=1), projections and lm_head in
    cfg.weight_dtype."""

    @staticmethod
    def read_config(path: str) -> "ModelConfig":
        c = LlamaConfig()
        call("infernt_checkpoint_read_config", path.encode(), ctypes.byref(c))
        return ModelConfig(vocab_size=c.vocab_size, hidden_size=c.hidden_size, num_layers=c.num_layers,
                           num_attention_heads=c.num_attention_heads, num_key_value_heads=c.num_key_value_heads,
                           intermediate_size=c.intermediate_size, max_seq_len=c.max_seq_len, head_dim=c.head_dim,
                           rms_norm_eps=c.rms_norm_eps, rope_theta=c.rope_theta, weight_dtype=c.weight_dtype)

    def __init__(self, model_bin: str, cfg: "ModelConfig", device: int = 1):
        self.cfg = cfg
        self._c = cfg.c()
        h = ctypes.c_void_p()
        call("infernt_checkpoint_load", model_bin.encode(), ctypes.byref(self._c), device, ctypes.byref(h))
        self._h = h
        n = 3 + 9 * cfg.num_layers
        arr = (_P * n)()
        call("infernt_checkpoint_weights", self._h, arr, n)
        self.ptrs = [arr[i] for i in range(n)]

    def close(self):
        if self._h:
            lib().infernt_checkpoint_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def nccl_unique_id() -> bytes:
    """A new ncclUniqueId (128 bytes) for BatchEngine(..., world > 1)."""
    buf = ctypes.create_string_buffer(128)
    call("infernt_nccl_unique_id", buf, 128)
    return buf.raw


class TPEngine:
    """One rank of a tensor-parallel decoder (infernt_tp_engine_* in
    include/infernt_capi.h) with seeded synthetic weights: the rank's shards
    of the model Engine(cfg, seed) would hold.  All ranks construct, swap
    xchg_handle() bytes by any host channel, and call set_peers(handles in
    rank order) before decoding; then every call must be made on every rank
    in the same order."""

    def __init__(self, cfg: ModelConfig, rank: int, world: int, seed: int = 0, std: float = 0.02):
        self.cfg, self.rank, self.world = cfg, rank, world
        h = ctypes.c_void_p()
        call("infernt_tp_engine_create_seeded", ctypes.byref(cfg.c()), seed, std, rank, world, ctypes.byref(h))
        self._h = h
        d = (ctypes.c_int * 6)()
        call("infernt_tp_engine_dims", self._h, d)
        self.dims = list(d)
        self.vocab_range = (d[4], d[4] + d[5])

    def close(self):
        if self._h:
            lib().infernt_tp_engine_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def xchg_handle(self) -> bytes:
        buf = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
        call("infernt_tp_engine_xchg_handle", self._h, buf)
        return buf.raw

    def set_peers(self, handles):
        blob = b"".join(handles)
        assert len(blob) == IPC_HANDLE_BYTES * self.world
        buf = ctypes.create_string_buffer(blob, len(blob))
        call("infernt_tp_engine_set_peers", self._h, buf)

    def forward_token(self, token: int, position: int) -> int:
        out = ctypes.c_int()
        call("infernt_tp_engine_forward_token", self._h, token, position, ctypes.byref(out))
        return out.value

    def decode_chain(self, token: int, position: int, steps: int):
        """Device-chained greedy decode; returns (tokens, device ms)."""
        import numpy as np
        toks = np.zeros(steps, dtype=np.int32)
        ms = ctypes.c_float()
        call("infernt_tp_engine_decode_chain", self._h, token, position, steps, toks.ctypes.data, ctypes.byref(ms))
        return toks.tolist(), ms.value

    def logits(self):
        """This rank's vocabulary rows [vocab_range) of the last step's logits."""
        import numpy as np
        out = np.empty(self.dims[5], dtype=np.float32)
        call("infernt_tp_engine_logits", self._h, out.ctypes.data, out.size)
        return out

    def trace_chain(self, token: int, position: int, steps: int):
        """decode_chain with the persistent kernel's phase timeline (as
        Engine.trace_chain)."""
        return _trace(self.cfg, "infernt_tp_engine_trace_chain", self._h, token, position, steps)

    def _plan(self):
        p = ctypes.c_void_p()
        call("infernt_tp_engine_plan", self._h, ctypes.byref(p))
        return p

    def xchg_region(self):
        """(device pointer, bytes) of this rank's exchange region."""
        p = self._plan()
        n = ctypes.c_size_t()
        call("infernt_plan_xchg_bytes", p, ctypes.byref(n))
        return lib().infernt_plan_xchg_region(p), n.value

    def set_peer_regions(self, regions):
        """In place of set_peers: every rank's exchange region as a device
        pointer of this process (own region at this rank's index)."""
        arr = (_P * self.world)(*regions)
        call("infernt_plan_set_peer_regions", self._plan(), arr)

    def set_wait_budget(self, microseconds: int):
        """Time budget of every wait inside the decode kernel."""
        call("infernt_plan_set_wait_budget", self._plan(), int(microseconds))

    def set_stream_depth(self, slots: int):
        """Weight-stream slots the decode kernel keeps in flight per SM
        (infernt_plan_set_stream_depth; 0: the whole ring)."""
        call("infernt_plan_set_stream_depth", self._plan(), int(slots))

    def stream_depth(self):
        """(slots in flight, ring slots) of the decode kernel."""
        a, b = ctypes.c_int(), ctypes.c_int()
        call("infernt_plan_stream_depth", self._plan(), ctypes.byref(a), ctypes.byref(b))
        return a.value, b.value
