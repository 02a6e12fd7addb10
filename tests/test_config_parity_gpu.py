"""Served-probability parity at the benchmark configs' own shapes.

cfg3 (Qwen3-8B-shaped), cfg4 (Qwen3.5-shaped GDN hybrid) and cfg5
(LFM2-shaped) run through the GPU engines and through the CPU oracle on the
same seeded weights and token ids, and their served option probabilities
must agree within |dp| < 1e-3 (bf16).  The oracle runs in the model dtype
(bf16 matmuls and stored activations, f32 softmax, GDN core and norm
accumulation), as the reference's candle path does.

Every layer keeps the config's shape (hidden size, heads, head dims, GDN
heads, conv kernels, MLP width, vocabulary) and every request keeps its
full state length, question count and lengths; only the number of layers is
reduced, so that the CPU oracle finishes in about a minute per config.  The
reference's own parity suites check model-level outputs the same way
(``crates/cev-model/tests/parity_models.rs:36-73``,
``parity_qwen35.rs:36-90``).
"""
import pytest
import torch

from cev_b200 import configs, service, weights, workloads
from oracle import engine as oeng
from oracle import hybrid as ohyb
from oracle import qwen3 as oq3
from oracle import service as osvc

pytestmark = pytest.mark.gpu

TOL_BF16 = 1e-3


def to_oracle_q(qs):
    return [osvc.Question(q.head, q.options, q.tail, list(q.order)) for q in qs]


def _weights(cfg, seed):
    """Seeded weights generated on the GPU (fast at these sizes), with one
    host copy for the oracle."""
    w = weights.init_weights(cfg, seed, torch.float32, "cuda")
    return w, {k: v.cpu() for k, v in w.items()}


def _worst(pa, pb):
    return max(abs(a - b) for x, y in zip(pa, pb) for a, b in zip(x, y))


def _oracle_threads():
    import os
    torch.set_num_threads(os.cpu_count() or 1)


def test_cfg3_shape_served_probabilities_match_oracle():
    """cfg3: Qwen3-8B layer shape (hidden 4096, 32 Q / 8 KV heads, head_dim
    128, SwiGLU 12288, vocab 151936), bf16, seed 1, 2 of the 36 layers.
    One request: an 8192-token random-id state (head 7680 prefilled in
    512-token chunks, tail 512 in the packed pass), 32 questions of
    U[48,128] tokens with 4 option codes x 2 rotations, all 64 suffixes and
    the tail in ONE packed pass (engine.rs:242-306)."""
    from cev_b200.engine import Engine
    from cev_b200.qwen3 import Qwen3
    cfg = configs.get("cfg3")
    cfg["num_hidden_layers"] = 2
    w_dev, w_host = _weights(cfg, 1)
    codes = workloads.code_ids(4)
    prefix, qs = workloads.decision_request(10_001, 8192, 32, 48, 128, 4, 151643)
    model = Qwen3(cfg, w_dev, torch.bfloat16, "cuda", arena_rows=8192 + 16384)
    del w_dev
    gpu = Engine(model, codes, prefill_chunk=512, pass_tokens=16384)
    _, p_gpu = service.run_debiased(gpu, prefix, qs, "permute", codes, workloads.SEP_ID, max_permutations=2)
    del gpu, model
    torch.cuda.empty_cache()
    _oracle_threads()
    ref = oeng.Engine(oq3.Qwen3(cfg, w_host, torch.bfloat16), codes, prefill_chunk=512, pass_tokens=16384)
    _, p_ref = osvc.run_debiased(ref, prefix, to_oracle_q(qs), "permute", codes, workloads.SEP_ID,
                                 max_permutations=2)
    assert len(p_gpu) == 32
    worst = _worst(p_gpu, p_ref)
    print(f"cfg3 shape: max |dp| {worst:.2e}")
    assert worst < TOL_BF16, worst


def test_cfg4_shape_served_probabilities_match_oracle():
    """cfg4: Qwen3.5-shaped hybrid at its layer shapes (hidden 4096; GDN
    nk 16 / nv 32, dk = dv = 128, conv kernel 4, chunk 64; gated attention
    16 Q / 4 KV heads, head_dim 256, partial RoPE 64; SwiGLU 12288; vocab
    248320), bf16, seed 2, 4 of the 32 layers (3 GDN + 1 attention, the
    config's pattern).  The 16384-token state runs once as one pass into the
    cached KV + recurrent + conv-tail state; 32 questions of U[32,128]
    tokens (4 codes x 2 rotations = 64 rows) then run as one right-padded
    batch continuing it (hybrid.rs:555-575, 595-617, 697-739)."""
    from cev_b200 import hybrid
    cfg = configs.get("cfg4")
    cfg["num_hidden_layers"] = 4
    cfg["layer_types"] = cfg["layer_types"][:4]
    assert cfg["layer_types"].count("linear_attention") == 3
    w_dev, w_host = _weights(cfg, 2)
    codes = workloads.code_ids(4)
    plen = 16384
    prefix, qs = workloads.decision_request(20_001, plen, 32, 32, 128, 4, cfg["vocab_size"] - 1)
    dec = hybrid.Qwen35(cfg, w_dev, torch.bfloat16, "cuda", max_len=plen + 1024, arena_rows=plen + 8192)
    del w_dev
    gpu = hybrid.HybridEngine(dec, codes, pad_id=0, prefill_chunk=plen, pass_tokens=8192, prefix_cache_tokens=plen)
    _, p_gpu = service.run_debiased(gpu, prefix, qs, "permute", codes, workloads.SEP_ID, max_permutations=2)
    del gpu, dec
    torch.cuda.empty_cache()
    _oracle_threads()
    odec = ohyb.Qwen35(cfg, w_host, torch.bfloat16)
    ref = ohyb.HybridEngine(odec, codes, pad_id=0, prefill_chunk=plen, pass_tokens=8192, prefix_cache_tokens=plen)
    _, p_ref = osvc.run_debiased(ref, prefix, to_oracle_q(qs), "permute", codes, workloads.SEP_ID,
                                 max_permutations=2)
    assert len(p_gpu) == 32
    worst = _worst(p_gpu, p_ref)
    print(f"cfg4 shape: max |dp| {worst:.2e}")
    assert worst < TOL_BF16, worst


def test_cfg5_shape_served_probabilities_match_oracle():
    """cfg5: LFM2 layer shapes (hidden 2048, gated short conv kernel 3, GQA
    32 Q / 8 KV heads, head_dim 64, SwiGLU 8192, vocab 65536), bf16, seed 3,
    3 of the 16 layers (conv, conv, attention).  A single 65536-token state
    is prefilled in 512-token chunks (each chunk's attention reads up to 64k
    cached keys), then 64 questions of 64 tokens run as right-padded rows
    continuing it, 4 option codes, no rotation (hybrid.rs:555-617)."""
    from cev_b200 import hybrid
    cfg = configs.get("cfg5")
    cfg["num_hidden_layers"] = 3
    cfg["layer_types"] = ["conv", "conv", "full_attention"]
    w_dev, w_host = _weights(cfg, 3)
    codes = workloads.code_ids(4)
    plen = 65536
    prefix, qs = workloads.decision_request(30_001, plen, 64, 64, 64, 4, cfg["vocab_size"] - 1)
    dec = hybrid.Lfm2(cfg, w_dev, torch.bfloat16, "cuda", max_len=plen + 1024, arena_rows=plen + 8192)
    del w_dev
    gpu = hybrid.HybridEngine(dec, codes, pad_id=0, prefill_chunk=512, pass_tokens=8192, prefix_cache_tokens=plen)
    _, p_gpu = service.run_debiased(gpu, prefix, qs, "none", codes, workloads.SEP_ID)
    del gpu, dec
    torch.cuda.empty_cache()
    _oracle_threads()
    odec = ohyb.Lfm2(cfg, w_host, torch.bfloat16)
    ref = ohyb.HybridEngine(odec, codes, pad_id=0, prefill_chunk=512, pass_tokens=8192, prefix_cache_tokens=plen)
    _, p_ref = osvc.run_debiased(ref, prefix, to_oracle_q(qs), "none", codes, workloads.SEP_ID)
    assert len(p_gpu) == 64
    worst = _worst(p_gpu, p_ref)
    print(f"cfg5 shape: max |dp| {worst:.2e}")
    assert worst < TOL_BF16, worst
