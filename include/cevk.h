/*
 * cevk -- B200 (sm_100a) kernels for cev's one-pass decision forward.
 *
 * A C ABI a Rust/candle host binds through `extern "C"` (see INTEGRATION.md
 * for the binding).  Every entry point:
 *   - takes plain device pointers, sizes and a `cudaStream_t` passed as
 *     `void*` (NULL = legacy default stream), and is stream-ordered: no host
 *     synchronisation, no allocation of device memory;
 *   - returns CEVK_OK (0) or a negative CEVK_E_* status; the message of the
 *     calling thread's last failure is `cevk_last_error()`;
 *   - validates shapes and descriptor ranges on the host before launching
 *     (CEVK_E_SHAPE / CEVK_E_RANGE, the candle-side `bail!` / `InputError`
 *     of the reference).
 * The caller owns every buffer.  Tensors are row-major; "rows" are tokens.
 * `dtype` is CEVK_BF16 or CEVK_F32 and applies to every floating tensor of
 * the call unless a parameter says otherwise.
 *
 * Reference paths below are relative to the CarterCole/rust-cev tree.
 */
#ifndef CEVK_H
#define CEVK_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CEVK_OK 0
#define CEVK_E_SHAPE (-1)       /* bad shape / stride / unsupported head size */
#define CEVK_E_RANGE (-2)       /* a descriptor points outside its buffer    */
#define CEVK_E_CUDA (-3)        /* CUDA launch / runtime failure              */
#define CEVK_E_TIMEOUT (-5)     /* a bounded device wait gave up              */
#define CEVK_E_UNSUPPORTED (-6) /* dtype / feature not built                  */

#define CEVK_BF16 1
#define CEVK_F32 2

/* Message of this thread's last failed call ("" if none). */
const char* cevk_last_error(void);
/* ABI version (major * 100 + minor). */
int cevk_version(void);
/* Reads and clears the device-side error flag raised by bounded waits;
 * synchronises the device.  CEVK_OK or CEVK_E_TIMEOUT. */
int cevk_device_status(void);
/* Failure-detection self-test: launches one thread that waits, through the
 * same bounded wait as the kernels, on a barrier nothing arrives on.  The
 * wait gives up after limit_cycles (1 .. 2^32) SM clock cycles and raises
 * the device error record; the kernel then returns normally, so the next
 * cevk_device_status() returns CEVK_E_TIMEOUT with the record's location
 * and the context stays usable.  No fault, trap or hang is involved. */
int cevk_selftest_wait_timeout(int64_t limit_cycles, void* stream);

/* ------------------------------------------------------------------------
 * Packed block-masked prefill attention.
 *
 * Replaces `Attention::attend` (crates/cev-model/src/qwen3.rs:206-220,
 * qwen35.rs:563-579, lfm2.rs:160-168) together with the additive mask the
 * engine builds on the host (engine.rs:418-442, qwen3.rs:157-169,
 * qwen35.rs:471-479, lfm2.rs:282-290) and the K/V concatenation
 * (qwen3.rs:197-200, engine.rs:375-387).
 *
 * A segment is a run of new tokens (query rows q_start .. q_start+q_len-1)
 * that sees, in full, K/V rows prefix_off .. prefix_off+prefix_len-1 and,
 * causally, its own K/V rows self_off .. self_off+q_len-1 (token i of the
 * segment sees self rows 0..i).  One segment per question suffix, per
 * prefix tail, per prefill chunk or per right-padded row.  No mask is
 * materialised; fully masked key tiles are never loaded.
 * ---------------------------------------------------------------------- */
typedef struct cevk_segment {
  int32_t q_start;
  int32_t q_len;
  int32_t prefix_off;
  int32_t prefix_len;
  int32_t self_off;
  int32_t tile_start; /* first work tile of the segment; set by cevk_attn_schedule */
  int32_t flags;      /* CEVK_SEG_* */
} cevk_segment;

/* Segment flag: every row of the segment sees all q_len of its own rows,
 * not only the earlier ones (Attn::Bidirectional, decoder.rs:109-116: a
 * right-padded row's real tokens as one such segment; its padding never
 * reaches a real token). */
#define CEVK_SEG_BIDIRECTIONAL 1

/* Validates host-side `segs` against the query/KV row counts (every range
 * inside its buffer; CEVK_E_RANGE otherwise), fills their `tile_start` and
 * returns the total tile count in `*n_tiles` (per KV head).  Call on the
 * host, then copy `segs` to the device for cevk_attn_packed_prefill. */
int cevk_attn_schedule(cevk_segment* segs, int32_t n_segs, int32_t n_tokens, int32_t n_kv_rows, int32_t hq,
                       int32_t hkv, int32_t head_dim, int32_t dtype, int32_t* n_tiles);

/* q: [n_tokens, hq, head_dim] with row stride q_row_stride (elements);
 * k, v: [n_kv_rows, hkv, head_dim] with row stride kv_row_stride;
 * o: [n_tokens, hq, head_dim] with row stride o_row_stride.
 * Query head h reads KV head h / (hq / hkv).  scale multiplies q.k
 * (the reference uses 1/sqrt(head_dim)).  segs_dev: device array of
 * n_segs descriptors as filled by cevk_attn_schedule.
 * bf16: head_dim 64, 128 or 256 on tcgen05 tensor cores, hq / hkv dividing
 * 128, q/k/v/o 16-byte aligned and every row stride a multiple of 8
 * (CEVK_E_SHAPE otherwise); f32: any head_dim <= 256 that is a multiple
 * of 32. */
int cevk_attn_packed_prefill(const void* q, const void* k, const void* v, void* o, int32_t n_tokens,
                             int32_t n_kv_rows, int32_t hq, int32_t hkv, int32_t head_dim, int32_t q_row_stride,
                             int32_t kv_row_stride, int32_t o_row_stride, const cevk_segment* segs_dev,
                             int32_t n_segs, int32_t n_tiles, float scale, int32_t dtype, void* stream);

/* Split-KV for calls whose work tiles underfill the GPU (a prefill chunk
 * after a long cached prefix: few tiles, each walking many key blocks).
 * The reference has no counterpart (candle runs one matmul per head); it is
 * a scheduling choice of this library with the same results.
 *
 * cevk_attn_split_plan: from the host-side `segs` as filled by
 * cevk_attn_schedule, returns in *n_split how many CTAs share one tile's
 * key blocks (1 when the tiles already fill n_sms SMs or the prefixes are
 * too short to pay) and in *workspace_bytes the workspace that split needs.
 * bf16 only (f32 plans 1). */
int cevk_attn_split_plan(const cevk_segment* segs, int32_t n_segs, int32_t n_tiles, int32_t hkv, int32_t head_dim,
                         int32_t dtype, int32_t n_sms, int32_t* n_split, int64_t* workspace_bytes);

/* Workspace bytes cevk_attn_packed_prefill_split needs for n_split (0 for
 * n_split <= 1): an f32 partial output row and its log-sum-exp per query
 * row, head and key range. */
int64_t cevk_attn_split_workspace_size(int32_t n_tiles, int32_t hkv, int32_t head_dim, int32_t n_split);

/* cevk_attn_packed_prefill with each work tile's key blocks cut into up to
 * n_split contiguous ranges (each starting inside the segment's prefix; a
 * tile whose prefix has fewer 64-key blocks than n_split uses that many),
 * run by separate CTAs that leave normalised f32 partial rows and their
 * log-sum-exp in `workspace` (16-byte aligned, at least
 * cevk_attn_split_workspace_size bytes); a second kernel on the same stream
 * merges them into o.  Tiles with one range write o directly.  n_split 1
 * (and every f32 call) is cevk_attn_packed_prefill.  The workspace serves
 * one call at a time. */
int cevk_attn_packed_prefill_split(const void* q, const void* k, const void* v, void* o, int32_t n_tokens,
                                   int32_t n_kv_rows, int32_t hq, int32_t hkv, int32_t head_dim, int32_t q_row_stride,
                                   int32_t kv_row_stride, int32_t o_row_stride, const cevk_segment* segs_dev,
                                   int32_t n_segs, int32_t n_tiles, float scale, int32_t n_split, void* workspace,
                                   int64_t workspace_bytes, int32_t dtype, void* stream);

/* ------------------------------------------------------------------------
 * Head all-gather fused into the attention epilogue, over NVLink peer
 * memory.  Replaces the NCCL all-gather of the per-head outputs under the
 * KV-head split of long-prefix attention (lfm2.rs:145-171 per rank, then
 * out_proj on the gathered [T, Hq * D] rows).
 *
 * Setup, once per rank: cevk_ipc_alloc the gathered buffers and an int32
 * flag array of `world` entries (zeroed), export each with cevk_ipc_handle,
 * exchange the handles between the ranks (any host channel), cevk_ipc_open
 * the peers' (peer access is enabled lazily; no multicast objects).
 * Per call (epoch = 1, 2, ... the same on every rank):
 *   cevk_attn_packed_prefill_gather  -- this rank's heads, every output row
 *       stored to each of o_bufs (every rank's gathered buffer, offset to
 *       this rank's head columns; o_row_stride = the gathered row width);
 *   cevk_gather_signal  -- after it on the same stream: flag[rank] = epoch
 *       in every rank's flag array (system-scope release);
 *   cevk_gather_wait    -- then: until every entry of this rank's flag
 *       array reaches epoch (bounded by limit_cycles; a timeout raises the
 *       device error record that cevk_device_status reports).
 * A rank reuses a gathered buffer for epoch e + 2 at the earliest, so two
 * buffers alternating by epoch parity never overwrite rows a peer still
 * reads.
 * ---------------------------------------------------------------------- */
#define CEVK_IPC_HANDLE_BYTES 64
int cevk_ipc_alloc(int64_t bytes, void** dev_ptr);
int cevk_ipc_free(void* dev_ptr);
int cevk_ipc_handle(const void* dev_ptr, void* handle);
int cevk_ipc_open(const void* handle, void** dev_ptr);
int cevk_ipc_close(void* dev_ptr);
/* bf16 only; arguments as cevk_attn_packed_prefill_split plus the 1..8
 * output buffers (16-byte aligned). */
int cevk_attn_packed_prefill_gather(const void* q, const void* k, const void* v, void* const* o_bufs, int32_t n_bufs,
                                    int32_t n_tokens, int32_t n_kv_rows, int32_t hq, int32_t hkv, int32_t head_dim,
                                    int32_t q_row_stride, int32_t kv_row_stride, int32_t o_row_stride,
                                    const cevk_segment* segs_dev, int32_t n_segs, int32_t n_tiles, float scale,
                                    int32_t n_split, void* workspace, int64_t workspace_bytes, void* stream);
int cevk_gather_signal(int32_t* const* flags, int32_t world, int32_t rank, int32_t epoch, void* stream);
int cevk_gather_wait(const int32_t* flags, int32_t world, int32_t epoch, int64_t limit_cycles, void* stream);
/* The same pair with the epoch in device memory (an int32 counter per rank,
 * zeroed with the flags): the signal advances it and publishes the new
 * value, the wait reads it -- so a CUDA graph can replay the calls, each
 * replay a new epoch.  A process uses one form or the other. */
int cevk_gather_signal_dev(int32_t* const* flags, int32_t world, int32_t rank, int32_t* epoch, void* stream);
int cevk_gather_wait_dev(const int32_t* flags, int32_t world, const int32_t* epoch, int64_t limit_cycles,
                         void* stream);
/* `bytes` (a multiple of 16) from src to each of dst[0 .. n_dst) (this
 * rank's and its peers' IPC buffers; 16-byte aligned): the residual
 * stream's all-gather under the token split of the KV-head-split layers,
 * followed by cevk_gather_signal_dev / cevk_gather_wait_dev.  No reference
 * counterpart (the reference runs one process). */
int cevk_rows_to_peers(const void* src, void* const* dst, int32_t n_dst, int64_t bytes, void* stream);
/* cevk_gather_signal_dev + cevk_gather_wait_dev in one launch. */
int cevk_gather_sync_dev(int32_t* const* flags, int32_t world, int32_t rank, int32_t* epoch, const int32_t* own_flags,
                         int64_t limit_cycles, void* stream);
/* cevk_rows_to_peers + cevk_gather_sync_dev in one launch (the last block
 * to finish its copies signals and waits).  `ticket`: a device uint32,
 * zero-initialised, that the launch leaves at zero; one per stream of
 * calls. */
int cevk_rows_gather_dev(const void* src, void* const* dst, int32_t n_dst, int64_t bytes, int32_t* const* flags,
                         int32_t world, int32_t rank, int32_t* epoch, const int32_t* own_flags, int64_t limit_cycles,
                         uint32_t* ticket, void* stream);

/* ------------------------------------------------------------------------
 * Per-head RMSNorm + (partial) RoPE at explicit positions, writing Q and
 * the arena K/V rows.  Replaces q_norm/k_norm + Rotary::apply + the K/V
 * `cat` (qwen3.rs:190-200; qwen35.rs:529-541 incl. the zero-centred `1+w`
 * norm and partial rotary; lfm2.rs:147-156).
 *
 * qkv: [n_tokens, row_stride] holding per token q (hq heads; each
 * q_head_stride elements apart, head_dim used), k (hkv heads, at column
 * k_col) and v (at column v_col).  Outputs: q_out [n_tokens, hq, head_dim];
 * k_arena/v_arena rows kv_rows[t] of [*, hkv, head_dim] (row stride
 * kv_row_stride).  pos: int32 [n_tokens].  The first rotary_dim dims of
 * each head rotate (half-split) with inverse frequencies
 * 1/(theta^(2i/rotary_dim)).  norm_plus_one: scale (1+w) instead of w.
 * ---------------------------------------------------------------------- */
int cevk_qk_norm_rope(const void* qkv, int32_t row_stride, int32_t q_head_stride, int32_t k_col, int32_t v_col,
                      const void* q_norm_w, const void* k_norm_w, float eps, int32_t norm_plus_one,
                      const int32_t* pos, double theta, int32_t rotary_dim, void* q_out, void* k_arena,
                      void* v_arena, int32_t kv_row_stride, const int32_t* kv_rows, int32_t n_tokens, int32_t hq,
                      int32_t hkv, int32_t head_dim, int32_t dtype, void* stream);

/* ------------------------------------------------------------------------
 * Token-wise RMSNorm (candle_nn::ops::rms_norm; qwen3.rs:254-255,
 * qwen35.rs:161-176 with plus_one, lfm2.rs operator/ffn norms).
 * If `residual` is non-NULL it is updated first: residual += add (the
 * decoder's `x = x + h`), then out = norm(residual); with out == NULL only
 * the residual add runs (w may then be NULL).  x/add/out: [n, hidden]
 * contiguous.
 * ---------------------------------------------------------------------- */
int cevk_rms_norm(const void* x, void* residual, const void* add, const void* w, void* out, int32_t n, int32_t hidden,
                  float eps, int32_t plus_one, int32_t dtype, void* stream);

/* out[t, j] = silu(gu[t, j]) * gu[t, inter + j]: the SwiGLU of
 * qwen3.rs:229-233 / lfm2.rs:253-255 on a fused gate|up projection. */
int cevk_swiglu(const void* gu, void* out, int32_t n, int32_t inter, int32_t dtype, void* stream);

/* out[t, :] = table[ids[t], :] (Embedding::index_select, qwen3.rs:288-293). */
int cevk_embed(const void* table, const int32_t* ids, void* out, int32_t n, int32_t hidden, int32_t vocab, int32_t dtype,
               void* stream);

/* out = a * sigmoid(gate) elementwise (qwen35.rs:556-558), in place allowed. */
int cevk_sigmoid_gate(const void* a, const void* gate, int32_t gate_row_stride, int32_t gate_head_stride,
                      void* out, int32_t n, int32_t heads, int32_t head_dim, int32_t dtype, void* stream);

/* ------------------------------------------------------------------------
 * Codes readout: final RMSNorm at the answer rows, then f32 logits against
 * the code rows (engine.rs:463-469, qwen3.rs:399-400, hybrid.rs:619-641).
 * x: residual stream [*, hidden]; rows: int32 [n_rows];
 * code_head: f32 [n_codes, hidden]; hidden_out: f32 [n_rows, hidden];
 * logits_out: f32 [n_rows, n_codes].
 * ---------------------------------------------------------------------- */
int cevk_readout(const void* x, const int32_t* rows, int32_t n_rows, const void* norm_w, float eps,
                 int32_t norm_plus_one, const float* code_head, int32_t n_codes, float* hidden_out,
                 float* logits_out, int32_t hidden, int32_t dtype, void* stream);

/* ------------------------------------------------------------------------
 * Gated DeltaNet (Qwen3.5 linear attention, qwen35.rs:415-453).
 *
 * cevk_gdn_conv: causal depthwise conv (kernel K) over the in_proj_qkv
 * output continuing from a conv tail, then SiLU:
 *   mixed: [B, T, C] rows of mixed_row_stride elements (C = 2*nk*dk + nv*dv),
 *   conv_w: [C, K], tail_in: [B or 1, C, K-1] (tail_batch_stride 0
 *   broadcasts one prefix state; NULL = zeros), tail_out: [B, C, K-1] or
 *   NULL (must not alias tail_in), out: [B, T, C] contiguous.
 * Replaces depthwise_conv1d + silu + the tail bookkeeping
 * (decoder.rs:137-151, qwen35.rs:419-431).
 * ---------------------------------------------------------------------- */
int cevk_gdn_conv(const void* mixed, int32_t mixed_row_stride, const void* conv_w, const void* tail_in,
                  int64_t tail_batch_stride, void* tail_out, void* out, int32_t B, int32_t T, int32_t C, int32_t K,
                  int32_t dtype, void* stream);

/* cevk_gdn_chunk_prefill: the chunked gated delta rule
 * (chunk_gated_delta_rule, qwen35.rs:301-368) in f32 for B rows of T
 * tokens, fused with its prologue (l2norm of q/k, q scale dk^-1/2, k-head
 * repeat nk -> nv, beta = sigmoid(b), g = -exp(A_log) * softplus(a +
 * dt_bias)) and followed by the gated RMSNorm epilogue
 * y = rmsnorm(o) * norm_w * silu(z) (qwen35.rs:443-451).
 *   conv_out: [B, T, C] (q | k | v per token) from cevk_gdn_conv;
 *   ab: per token the in_proj_b outputs (nv) then the in_proj_a outputs
 *     (nv), rows of ab_row_stride elements;
 *   z: [B, T, nv*dv] rows of z_row_stride elements;
 *   a_log, dt_bias: f32 [nv]; norm_w: [dv];
 *   s_in: f32 [B or 1, nv, dk, dv] (s_batch_stride 0 broadcasts one prefix
 *     state to every row; NULL = zero state); s_out: f32 [B, nv, dk, dv]
 *     or NULL (may alias s_in only when s_batch_stride is nv*dk*dv);
 *   y: [B, T, nv*dv].
 * Shapes: nv a multiple of nk, dk a multiple of 32 in [64, 128], dv 64, 128
 * or 256; z, norm_w, y and z's row stride aligned to dv/32 elements.
 * Padding tokens at the end of a row are computed like the reference
 * (causal: they never reach a real token); s_out is the state after all T
 * tokens.  workspace: device scratch of cevk_gdn_workspace_size() bytes:
 * the f32 core output before the norm and, for bf16 with dk = dv = 64 or
 * 128, the per-chunk matrices of the tensor-core path.  A workspace of only
 * B*T*nv*dv*4 bytes (the core output) runs every dtype on the f32 SIMT
 * kernel instead.  A bf16 dk = dv = 128 call with B = 1, s_out given and at
 * least 42 chunks (a state run once through the layer), made outside stream
 * capture, runs in pieces on three streams the library creates per device
 * on first use, forked from and joined back into `stream` (the next
 * piece's prep beside the current piece's scan); such calls must not span
 * a cudaDeviceReset of that device. */
size_t cevk_gdn_workspace_size(int32_t B, int32_t T, int32_t nv, int32_t dk, int32_t dv);
int cevk_gdn_chunk_prefill(const void* conv_out, int32_t C, const void* ab, int32_t ab_row_stride, const void* z,
                           int32_t z_row_stride, const float* a_log, const float* dt_bias, const void* norm_w,
                           float eps, const float* s_in, int64_t s_batch_stride, float* s_out, void* y, int32_t B,
                           int32_t T, int32_t nk, int32_t nv, int32_t dk, int32_t dv, void* workspace,
                           size_t workspace_bytes, int32_t dtype, void* stream);

/* Allocation-free variant of cevk_gdn_chunk_prefill (no counterpart in the
 * reference).  For callers that cannot give this library a workspace: hosts
 * whose device memory belongs to their own fixed pool, or paths where a
 * cudaMalloc is not allowed or would stall.  Same arguments and results as
 * cevk_gdn_chunk_prefill without workspace / workspace_bytes; the f32
 * scratch is a fixed device array inside the library (CEVK_GDN_NOALLOC_MAX_BYTES,
 * held by every GPU that loads the library until exit).
 *   - The array holds cevk_gdn_workspace_size() for small calls (tensor-core
 *     path); larger ones run the f32 SIMT kernel, whose scratch is
 *     B*T*nv*dv*4 bytes.  Calls needing more than that return CEVK_E_SHAPE;
 *     split them or use the workspace entry point.
 *   - The first call on a device looks up the array's device address (once
 *     per device, with that device current); make that first call before
 *     any stream capture.  The address is kept for the life of the process,
 *     so calls must not span a cudaDeviceReset (or any other teardown of
 *     the device's primary context).
 *   - Allocates nothing: no cudaMalloc / cudaFree or allocating library call.
 *   - All calls share the array: calls that overlap on the GPU (other
 *     streams, other host threads on the same device) race.  Nothing in it
 *     needs to start at zero; each call overwrites what it reads. */
#define CEVK_GDN_NOALLOC_MAX_BYTES ((size_t)16 << 20)
int cevk_gdn_chunk_prefill_noalloc(const void* conv_out, int32_t C, const void* ab, int32_t ab_row_stride,
                                   const void* z, int32_t z_row_stride, const float* a_log, const float* dt_bias,
                                   const void* norm_w, float eps, const float* s_in, int64_t s_batch_stride,
                                   float* s_out, void* y, int32_t B, int32_t T, int32_t nk, int32_t nv, int32_t dk,
                                   int32_t dv, int32_t dtype, void* stream);

/* ------------------------------------------------------------------------
 * Served debiased probabilities (run_debiased's answer math,
 * service.rs:288-348 with math::{softmax, log_softmax}, math.rs:7-18), on
 * the device so that only k values per question cross to the host.
 *   logits: [n_variants, ld] f32 code logits of every rotation variant in
 *     display order (readout rows), cf_logits: the same rows of the
 *     content-free calibration twin or NULL;
 *   span: [n_questions + 1] variant ranges of the questions;
 *   n_options: [n_questions] option counts (<= ld <= 32);
 *   order: [n_variants, ld] canonical option shown at each display position;
 *   scores: [n_questions, out_ld] f32, probs: [n_questions, out_ld] f64.
 * score_o = mean over variants of log_softmax(z)[pos] - log_softmax(cf)[pos]
 * at the canonical option o shown at pos, rounded to f32; probs =
 * softmax(score), f64 like the reference.  No counterpart function in the
 * reference (it runs this on the host). */
int cevk_debias(const float* logits, const float* cf_logits, int32_t ld, const int32_t* span,
                const int32_t* n_options, const int32_t* order, int32_t n_questions, float* scores, double* probs,
                int32_t out_ld, void* stream);

/* ------------------------------------------------------------------------
 * LFM2 gated short convolution (ShortConv::forward, lfm2.rs:199-219):
 * y = C (.) conv_K(B (.) X) continuing from a tail of K-1 inputs.
 *   bcx: [B, T, 3*d] in_proj output (b | c | x per token);
 *   conv_w: [d, K]; bias: [d] or NULL;
 *   tail_in: [B or 1, d, K-1] (tail_batch_stride 0 broadcasts; NULL = zeros);
 *   tail_out: [B, d, K-1] or NULL; y: [B, T, d].
 * ---------------------------------------------------------------------- */
int cevk_short_conv(const void* bcx, const void* conv_w, const void* bias, const void* tail_in,
                    int64_t tail_batch_stride, void* tail_out, void* y, int32_t B, int32_t T, int32_t d, int32_t K,
                    int32_t dtype, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* CEVK_H */
