"""The C-ABI library on a host without a GPU: it loads, exports every entry
point include/infernt_capi.h declares, and rejects bad arguments with a
status code (no kernel is launched)."""
import ctypes
import os
import re
import subprocess

import pytest

import infernt_b200 as ib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared(header):
    text = open(os.path.join(ROOT, "include", header)).read()
    return sorted(set(re.findall(r"INFERNT_API\s+[\w\s\*]+?\b(infernt_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = ib.lib()
    declared = _declared("infernt_capi.h")
    assert len(declared) >= 40
    missing = [s for s in declared if not hasattr(lib, s)]
    assert not missing, missing
    # the ctypes table covers exactly the declared entry points
    assert sorted(ib.exported_symbols()) == declared


def test_dynamic_symbol_table_has_cxx_dropin_api():
    out = subprocess.run(["nm", "-D", "-C", "--defined-only", ib.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    for sym in ["launch_rmsnorm(", "launch_argmax(", "launch_attention_scores(",
                "LlamaArchitecture::forward(", "InferenceEngine::forward_token(",
                "InferenceEngine::sample_next_token(", "KVCache::allocate(", "Tensor::copy_from(",
                "CublasWrapper::gemm(", "ModelConfig::validate()"]:
        assert sym in out, sym


def test_status_strings():
    lib = ib.lib()
    assert lib.infernt_status_string(0) == b"ok"
    assert lib.infernt_status_string(1) == b"invalid argument"
    assert lib.infernt_status_string(5) == b"device-side error"
    assert lib.infernt_version() >= 100


@pytest.mark.parametrize("call", [
    lambda l: l.infernt_rmsnorm(None, None, None, 1, 8, 1e-5, None),
    lambda l: l.infernt_residual_add(None, None, None, 4, None),
    lambda l: l.infernt_softmax(None, None, 1, 4, None),
    lambda l: l.infernt_argmax(None, None, 10, None),
    lambda l: l.infernt_gemm_f32(None, None, None, 1, 1, 1, 1.0, 0.0, 0, 1, None),
    lambda l: l.infernt_rmsnorm_gemv(None, None, 4, None, 0, None, 0, 512, 0, None, None, 1e-5, None),
    lambda l: l.infernt_rmsnorm_gemv(8, 8, 4, None, 0, None, 0, 512, 7, 8, None, 1e-5, None),
    lambda l: l.infernt_attention_decode(8, 8, 8, 8, 32, 4, 64, 16, 16, 1e4, 4, 8, None),
    lambda l: l.infernt_attention_decode(8, 8, 8, 8, 32, 5, 64, 16, 3, 1e4, 4, 8, None),
    lambda l: l.infernt_attention_decode(8, 8, 8, 8, 32, 4, 47, 16, 3, 1e4, 4, 8, None),
    lambda l: l.infernt_attention_decode(8, 8, 8, 8, 32, 4, 256, 16, 3, 1e4, 4, 8, None),
    lambda l: l.infernt_kv_cache_append(8, 8, 8, 8, 2, 4, 8, 8, None),
])
def test_bad_arguments_are_rejected_without_a_launch(call):
    lib = ib.lib()
    assert call(lib) == 1
    assert lib.infernt_last_error() != b""


def test_plan_rejects_bad_config():
    lib = ib.lib()
    cfg = ib.TINYLLAMA.with_(num_key_value_heads=5).c()
    out = ctypes.c_void_p()
    assert lib.infernt_plan_create(ctypes.byref(cfg), None, None, None, 1, ctypes.byref(out)) == 1
    assert not out.value


def test_workspace_sizes():
    lib = ib.lib()
    n = lib.infernt_attention_workspace_bytes(32, 4, 64, 37)
    assert n >= 4 * 37 * 8 * 66 * 4 and n % 256 == 0
    assert lib.infernt_lm_head_workspace_bytes() >= 1024 * 8


def test_model_shapes():
    assert ib.TINYLLAMA.head_dim == 64
    # streamed parameters per token: every projection matrix and the LM head
    H, I, L, V = 2048, 5632, 22, 32000
    per_layer = H * (2048 + 512) + 2048 * H + 3 * H * I
    assert ib.TINYLLAMA.weight_params == L * per_layer + V * H
    assert ib.LLAMA3_8B.head_dim == 128


def test_prompt_generator_matches_oracle():
    """The product's seeded prompt (infernt_fill_prompt, used by the
    benchmarks) is the oracle's token for token."""
    import infernt_b200 as ib
    import oracle as O
    for n, seed, hi in ((32, 0, 32000), (512, 1, 128256), (7, 99, 50)):
        assert ib.prompt(n, seed, 3, hi) == [int(t) for t in O.prompt(n, seed, 3, hi)]
