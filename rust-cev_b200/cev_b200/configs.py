"""Model shapes the decision forward runs, as HF-style ``config.json`` dicts.

Field names follow the checkpoints the reference loads
(``crates/cev-model/src/qwen3.rs:60-99``, ``qwen35.rs:43-122``,
``lfm2.rs:18-88``).  ``BENCH`` holds the five benchmark shapes; ``tiny_*``
build small models of the same families for parity tests.
"""
from __future__ import annotations

import copy


def qwen3(vocab, hidden, inter, layers, heads, kv, head_dim, theta=1e6, eps=1e-6, tie=False, max_pos=40960):
    return {
        "model_type": "qwen3", "vocab_size": vocab, "hidden_size": hidden, "intermediate_size": inter,
        "num_hidden_layers": layers, "num_attention_heads": heads, "num_key_value_heads": kv,
        "head_dim": head_dim, "rope_theta": theta, "rms_norm_eps": eps, "tie_word_embeddings": tie,
        "max_position_embeddings": max_pos, "attention_bias": False,
    }


def qwen35(vocab, hidden, inter, layers, heads, kv, head_dim, nk, nv, dk, dv, conv=4, theta=1e7,
           partial=0.25, eps=1e-6, every=4, tie=False, max_pos=262144):
    types = ["full_attention" if (i + 1) % every == 0 else "linear_attention" for i in range(layers)]
    return {
        "model_type": "qwen3_5_text", "vocab_size": vocab, "hidden_size": hidden, "intermediate_size": inter,
        "num_hidden_layers": layers, "num_attention_heads": heads, "num_key_value_heads": kv,
        "head_dim": head_dim, "layer_types": types, "linear_conv_kernel_dim": conv,
        "linear_key_head_dim": dk, "linear_value_head_dim": dv, "linear_num_key_heads": nk,
        "linear_num_value_heads": nv, "rms_norm_eps": eps, "max_position_embeddings": max_pos,
        "attn_output_gate": True, "tie_word_embeddings": tie,
        "rope_parameters": {"rope_theta": theta, "partial_rotary_factor": partial,
                            "mrope_section": [11, 11, 10], "mrope_interleaved": True, "rope_type": "default"},
    }


def lfm2(vocab, hidden, inter, layers, heads, kv, attn_layers, kernel=3, theta=1e6, eps=1e-5, max_pos=128000):
    types = ["full_attention" if i in attn_layers else "conv" for i in range(layers)]
    return {
        "model_type": "lfm2", "vocab_size": vocab, "hidden_size": hidden, "intermediate_size": inter,
        "num_hidden_layers": layers, "num_attention_heads": heads, "num_key_value_heads": kv,
        "layer_types": types, "conv_L_cache": kernel, "conv_bias": False, "norm_eps": eps,
        "max_position_embeddings": max_pos, "rope_theta": theta, "block_auto_adjust_ff_dim": False,
        "tie_word_embeddings": True,
    }


# The five benchmark shapes.  cfg4's intermediate size, vocabulary, partial
# rotary factor and theta are not fixed by the benchmark; these are the
# Qwen3.5-family defaults (theta 1e7 and factor 0.25 as in qwen35.rs:39-41,
# 110-113).  cfg5 places its six attention layers like LFM2-1.2B.
BENCH = {
    "cfg1": qwen3(151936, 1024, 3072, 28, 16, 8, 128),
    "cfg3": qwen3(151936, 4096, 12288, 36, 32, 8, 128),
    "cfg4": qwen35(248320, 4096, 12288, 32, 16, 4, 256, 16, 32, 128, 128),
    "cfg5": lfm2(65536, 2048, 8192, 16, 32, 8, {2, 5, 8, 10, 12, 14}),
}


def tiny_qwen3(layers=2, hidden=256, heads=4, kv=2, head_dim=64, inter=512, vocab=1024):
    return qwen3(vocab, hidden, inter, layers, heads, kv, head_dim)


def tiny_qwen35(layers=4, hidden=256, heads=4, kv=2, head_dim=64, inter=512, vocab=1024, nk=2, nv=4, dk=64, dv=64):
    return qwen35(vocab, hidden, inter, layers, heads, kv, head_dim, nk, nv, dk, dv)


def tiny_lfm2(layers=4, hidden=256, heads=4, kv=2, inter=512, vocab=1024):
    return lfm2(vocab, hidden, inter, layers, heads, kv, {1, 3})


def get(name: str) -> dict:
    return copy.deepcopy(BENCH[name])
