"""Generate the golden vectors the oracle is pinned to.

The reference (Rust/candle) cannot run in this image, but its declared
parity target is HF transformers in f32 with eager attention
(``training/parity/dump_qwen35.py``; README "matches HF transformers to
|dp| < 5e-5").  This script builds tiny random-init Qwen3, Qwen3.5 and LFM2
models with ``cev_b200.weights.init_weights`` (seeded, CPU, reproducible),
loads the same tensors into the HF classes, and records HF's final hidden
states for a few random token rows, mirroring the reference's dump format
(``hidden_last``, ``hidden_mid``, ``logits_last`` at probe ids).

Run from the repository root:  python tests/golden/make_golden.py
Output: tests/golden/hf_<family>.safetensors (+ .json with the config).
"""
import json
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "rust-cev_b200"))

from cev_b200 import configs, weights  # noqa: E402

FAMILIES = {
    "qwen3": (configs.tiny_qwen3(), 11),
    "qwen35": (configs.tiny_qwen35(), 12),
    "lfm2": (configs.tiny_lfm2(), 13),
}
ROW_LENS = (37, 90, 150)
PROBE = [5, 17, 123, 400, 999]


def hf_model(name, cfg):
    import transformers as tf
    if name == "qwen3":
        c = tf.Qwen3Config(**{k: v for k, v in cfg.items() if k != "model_type"})
        m = tf.Qwen3ForCausalLM(c)
    elif name == "qwen35":
        kw = {k: v for k, v in cfg.items() if k != "model_type"}
        c = tf.Qwen3_5TextConfig(**kw)
        m = tf.Qwen3_5ForCausalLM(c)
    else:
        kw = {k: v for k, v in cfg.items() if k != "model_type"}
        c = tf.Lfm2Config(**kw)
        m = tf.Lfm2ForCausalLM(c)
    c._attn_implementation = "eager"
    return m.eval()


def main():
    torch.manual_seed(0)
    for name, (cfg, seed) in FAMILIES.items():
        w = weights.init_weights(cfg, seed)
        m = hf_model(name, cfg)
        sd = m.state_dict()
        missing = [k for k in sd if k not in w and not (k == "lm_head.weight" and cfg.get("tie_word_embeddings"))]
        assert not missing, missing
        load = {k: w[k] if k in w else w["model.embed_tokens.weight"] for k in sd}
        m.load_state_dict(load, strict=True)
        gen = torch.Generator().manual_seed(seed + 100)
        out = {}
        for r, n in enumerate(ROW_LENS):
            ids = torch.randint(0, cfg["vocab_size"], (n,), generator=gen)
            with torch.no_grad():
                o = m(input_ids=ids[None], output_hidden_states=True)
            hid = o.hidden_states[-1][0]
            out[f"row{r}.ids"] = ids.to(torch.int32)
            out[f"row{r}.hidden_last"] = hid[n - 1].float().contiguous()
            out[f"row{r}.hidden_mid"] = hid[n // 2].float().contiguous()
            out[f"row{r}.logits_last"] = o.logits[0, n - 1, PROBE].float().contiguous()
        from safetensors.torch import save_file
        save_file(out, os.path.join(HERE, f"hf_{name}.safetensors"))
        with open(os.path.join(HERE, f"hf_{name}.json"), "w") as f:
            json.dump({"config": cfg, "seed": seed, "rows": len(ROW_LENS), "probe_ids": PROBE,
                       "transformers": __import__("transformers").__version__}, f, indent=1)
        print(name, "ok")


if __name__ == "__main__":
    main()
