"""Writes INFT v1 checkpoints for the loader tests, byte for byte in the
layout the reference's converter writes (tools/convert_checkpoint.py:124-145,
README.md:206-215): "III" magic 0x494E4654 / version / tensor count, then per
tensor int32 name length, UTF-8 name, int32 dim count, int32 dims, int64
element count and the FP32 payload; and config.json with the converter's keys
(tools/convert_checkpoint.py:23-34)."""
import json
import struct

import numpy as np

MAGIC = 0x494E4654

LAYER_NAMES = ["input_layernorm.weight", "self_attn.q_proj.weight", "self_attn.k_proj.weight",
               "self_attn.v_proj.weight", "self_attn.o_proj.weight", "post_attention_layernorm.weight",
               "mlp.gate_proj.weight", "mlp.up_proj.weight", "mlp.down_proj.weight"]


def write_config(path, cfg, **extra):
    d = {"architecture": "LlamaForCausalLM", "vocab_size": cfg.vocab_size, "hidden_size": cfg.hidden_size,
         "num_layers": cfg.num_layers, "num_attention_heads": cfg.num_attention_heads,
         "num_key_value_heads": cfg.num_key_value_heads, "intermediate_size": cfg.intermediate_size,
         "max_seq_len": cfg.max_seq_len, "rms_norm_eps": cfg.rms_norm_eps, "rope_theta": cfg.rope_theta}
    d.update(extra)
    with open(path, "w") as f:
        json.dump(d, f, indent=4)


def write_inft(path, tensors, magic=MAGIC, version=1, count=None):
    """tensors: list of (name, array); arrays are written as FP32."""
    with open(path, "wb") as f:
        f.write(struct.pack("III", magic, version, len(tensors) if count is None else count))
        for name, a in tensors:
            a = np.ascontiguousarray(np.asarray(a, dtype=np.float32))
            nb = name.encode("utf-8")
            f.write(struct.pack("i", len(nb)))
            f.write(nb)
            f.write(struct.pack("i", a.ndim))
            for d in a.shape:
                f.write(struct.pack("i", int(d)))
            f.write(struct.pack("q", int(a.size)))
            f.write(a.tobytes())


def model_tensors(cfg, rng, with_lm_head=True):
    """Random tensors of cfg's shapes in the converter's order (embedding,
    layers, final norm, lm_head) and the same arrays in the engine's weight
    order [embedding, final_norm, lm_head, per layer 9]."""
    H, V, I, L = cfg.hidden_size, cfg.vocab_size, cfg.intermediate_size, cfg.num_layers
    qs, kvs = cfg.num_attention_heads * cfg.head_dim, cfg.num_key_value_heads * cfg.head_dim
    r = lambda *s: (rng.standard_normal(s) * 0.02).astype(np.float32)
    emb, norm, lm = r(V, H), (1.0 + r(H)).astype(np.float32), r(V, H)
    named = [("model.embed_tokens.weight", emb)]
    order = [emb, norm, lm if with_lm_head else emb]
    for l in range(L):
        ws = [(1.0 + r(H)).astype(np.float32), r(qs, H), r(kvs, H), r(kvs, H), r(H, qs),
              (1.0 + r(H)).astype(np.float32), r(I, H), r(I, H), r(H, I)]
        named += [("model.layers.%d.%s" % (l, n), w) for n, w in zip(LAYER_NAMES, ws)]
        order += ws
    named.append(("model.norm.weight", norm))
    if with_lm_head:
        named.append(("lm_head.weight", lm))
    return named, order
