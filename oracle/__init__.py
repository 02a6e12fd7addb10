"""CPU oracle for cev's one-pass decision forward.

TEST INFRASTRUCTURE ONLY.  This package restates, in plain PyTorch on the CPU,
the arithmetic of the reference implementation (CarterCole/rust-cev, a Rust /
candle 0.11.0 code base) for the hot path the GPU library replaces:

* packed block-masked Qwen3 prefill (``crates/cev-model/src/qwen3.rs``,
  ``crates/cev-model/src/engine.rs``),
* the Qwen3.5 Gated DeltaNet hybrid with right-padded continuation rows
  (``crates/cev-model/src/qwen35.rs``, ``crates/cev-model/src/hybrid.rs``),
* the LFM2 short-conv hybrid (``crates/cev-model/src/lfm2.rs``),
* the debiased served probabilities (``crates/cev-runtime/src/service.rs``,
  ``crates/cev-core/src/math.rs``, ``crates/cev-core/src/compile.rs``).

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` may import it, and only as the checker or the timed CPU
baseline.  The product (``rust-cev_b200/cev_b200``) never imports it.

Pinning: the reference is Rust and cannot be built in this image (no cargo,
no vendored crates), so parity is pinned by (1) reproducing the reference's
own known-answer unit tests bit-for-bit in their inputs
(``qwen35.rs:759-822``, ``compile.rs:463-476``, ``runtime.rs:184-207``) and
(2) golden vectors from HF transformers 5.5.0 -- the reference's declared
parity target -- committed under ``tests/golden/`` with the script that made
them.
"""
