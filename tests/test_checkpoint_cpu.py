"""INFT v1 checkpoint loading (infernt_checkpoint_*, CheckpointLoader) on the
host, against the arrays written and against the reference's own
CheckpointLoader (loader/checkpoint_loader.cpp, compiled unchanged into
oracle/_ref) loading the same files on the CPU: FP32 payloads bit-exact,
the bf16 option the exact round-to-nearest-even of each value, the
configuration equal field by field.  Error cases the reference leaves
unchecked (truncation, element counts, missing tensors) must fail cleanly."""
import ctypes
import os

import numpy as np
import pytest

import infernt_b200 as ib
import oracle as O
from inft_file import LAYER_NAMES, model_tensors, write_config, write_inft

CFG = ib.ModelConfig(vocab_size=64, hidden_size=32, num_layers=2, num_attention_heads=4, num_key_value_heads=2,
                     intermediate_size=48, max_seq_len=128, rms_norm_eps=1e-6, rope_theta=500000.0)


def _load_host(path, cfg):
    ck = ib.Checkpoint(path, cfg, device=0)
    out = []
    for p, a in zip(ck.ptrs, _expected_sizes(cfg)):
        n, is_proj = a
        if is_proj and cfg.weight_dtype == ib.DTYPE_BF16:
            buf = (ctypes.c_uint16 * n).from_address(p)
            out.append(np.frombuffer(buf, dtype=np.uint16).copy())
        else:
            buf = (ctypes.c_float * n).from_address(p)
            out.append(np.frombuffer(buf, dtype=np.float32).copy())
    ck.close()
    return out


def _expected_sizes(cfg):
    H, V, I = cfg.hidden_size, cfg.vocab_size, cfg.intermediate_size
    qs, kvs = cfg.num_attention_heads * cfg.head_dim, cfg.num_key_value_heads * cfg.head_dim
    sizes = [(V * H, False), (H, False), (V * H, True)]
    for _ in range(cfg.num_layers):
        sizes += [(H, False), (qs * H, True), (kvs * H, True), (kvs * H, True), (H * qs, True), (H, False),
                  (I * H, True), (I * H, True), (H * I, True)]
    return sizes


def _ref_load(config_json, model_bin, cfg):
    """The reference's CheckpointLoader on the host: (ci, cf, arrays)."""
    l = O.rlib()
    ci = (ctypes.c_int * 8)()
    cf = (ctypes.c_float * 2)()
    sizes = [n for n, _ in _expected_sizes(cfg)]
    arrays = [np.zeros(n, dtype=np.float32) for n in sizes]
    ptrs = (ctypes.c_void_p * len(arrays))(*[a.ctypes.data for a in arrays])
    ns = (ctypes.c_longlong * len(arrays))(*sizes)
    l.ref_checkpoint_load_cpu.restype = ctypes.c_int
    rc = l.ref_checkpoint_load_cpu(config_json.encode(), model_bin.encode() if model_bin else None, ci, cf,
                                   len(arrays), ptrs, ns)
    assert rc == 0, l.ref_last_error()
    return list(ci), list(cf), arrays


def _bf16_bits(a):
    return (O.round_bf16(np.asarray(a, dtype=np.float32)).view(np.uint32) >> 16).astype(np.uint16)


@pytest.fixture
def ckpt(tmp_path):
    rng = np.random.default_rng(11)
    named, order = model_tensors(CFG, rng)
    cj, mb = str(tmp_path / "config.json"), str(tmp_path / "model.bin")
    write_config(cj, CFG)
    write_inft(mb, named)
    return cj, mb, order


def test_config_matches_reference(ckpt):
    cj, _, _ = ckpt
    mine = ib.Checkpoint.read_config(cj)
    assert (mine.vocab_size, mine.hidden_size, mine.num_layers, mine.num_attention_heads,
            mine.num_key_value_heads, mine.intermediate_size, mine.max_seq_len, mine.head_dim) == (
        64, 32, 2, 4, 2, 48, 128, 8)
    assert mine.rms_norm_eps == np.float32(1e-6) and mine.rope_theta == 500000.0
    if O.ref_available():
        ci, cf, _ = _ref_load(cj, None, CFG)
        assert ci == mine.ints()
        assert cf == [np.float32(mine.rms_norm_eps), np.float32(mine.rope_theta)]


def test_config_defaults_and_nested_keys(tmp_path):
    p = str(tmp_path / "config.json")
    with open(p, "w") as f:
        f.write('{"rope_scaling": {"type": "linear", "factor": 2.0, "vocab_size": 5}, "architectures": ["X"],\n'
                ' "vocab_size": 1000, "hidden_size": 256, "num_layers": 3, "num_attention_heads": 8,\n'
                ' "num_key_value_heads": 2, "intermediate_size": 512, "tie": true, "weight_dtype": "bf16"}')
    c = ib.Checkpoint.read_config(p)
    assert (c.vocab_size, c.max_seq_len, c.head_dim, c.weight_dtype) == (1000, 2048, 32, ib.DTYPE_BF16)
    assert c.rms_norm_eps == np.float32(1e-5) and c.rope_theta == 10000.0


def test_fp32_load_is_exact_and_matches_reference(ckpt):
    cj, mb, order = ckpt
    got = _load_host(mb, CFG)
    for i, (g, w) in enumerate(zip(got, order)):
        assert np.array_equal(g, w.ravel()), i
    if O.ref_available():
        _, _, ref = _ref_load(cj, mb, CFG)
        for i, (g, r) in enumerate(zip(got, ref)):
            assert np.array_equal(g, r), i


def test_bf16_option_rounds_projections_only(ckpt):
    _, mb, order = ckpt
    cfg = CFG.with_(weight_dtype=ib.DTYPE_BF16)
    got = _load_host(mb, cfg)
    for i, ((_, proj), g, w) in enumerate(zip(_expected_sizes(cfg), got, order)):
        if proj:
            assert np.array_equal(g, _bf16_bits(w.ravel())), i
        else:
            assert np.array_equal(g, w.ravel()), i


def test_missing_lm_head_copies_embedding(tmp_path):
    rng = np.random.default_rng(12)
    named, order = model_tensors(CFG, rng, with_lm_head=False)
    cj, mb = str(tmp_path / "config.json"), str(tmp_path / "model.bin")
    write_config(cj, CFG)
    # extra tensors the model does not use are skipped; order does not matter
    named = [("model.rotary_emb.inv_freq", np.ones(4, np.float32))] + named[::-1]
    write_inft(mb, named)
    got = _load_host(mb, CFG)
    assert np.array_equal(got[2], order[0].ravel())
    for g, w in zip(got, order):
        assert np.array_equal(g, w.ravel())
    if O.ref_available():
        _, _, ref = _ref_load(cj, mb, CFG)
        assert all(np.array_equal(g, r) for g, r in zip(got, ref))


@pytest.mark.parametrize("case", ["magic", "version", "truncated", "count", "missing", "extra_layer_ok"])
def test_bad_files(tmp_path, case):
    rng = np.random.default_rng(13)
    named, _ = model_tensors(CFG, rng)
    mb = str(tmp_path / "model.bin")
    if case == "magic":
        write_inft(mb, named, magic=0x12345678)
    elif case == "version":
        write_inft(mb, named, version=2)
    elif case == "truncated":
        write_inft(mb, named)
        size = os.path.getsize(mb)
        with open(mb, "r+b") as f:
            f.truncate(size - 100)
    elif case == "count":
        named = [(n, a[:-1] if n.endswith("q_proj.weight") else a) for n, a in named]
        write_inft(mb, named)
    elif case == "missing":
        write_inft(mb, [(n, a) for n, a in named if n != "model.layers.1.mlp.up_proj.weight"])
    else:
        # a layer index past num_layers is not a tensor of this model: skipped
        named.append(("model.layers.7." + LAYER_NAMES[0], np.ones(CFG.hidden_size, np.float32)))
        write_inft(mb, named)
        ib.Checkpoint(mb, CFG, device=0).close()
        return
    with pytest.raises(ib.InferntError):
        ib.Checkpoint(mb, CFG, device=0)
