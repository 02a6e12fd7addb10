//! Raw bindings to the C ABI of include/cevk.h (one `extern "C"` item per
//! entry point, same names, argument order and meaning).  Every function
//! returns CEVK_OK or a negative CEVK_E_* status; `cevk_last_error()` gives
//! the calling thread's message.  Device pointers and `cudaStream_t` are
//! passed as raw pointers; the caller owns every buffer.
#![allow(non_camel_case_types)]
use std::ffi::{c_char, c_void};

#[repr(C)]
#[derive(Clone, Copy, Default)]
pub struct cevk_segment {
    pub q_start: i32, pub q_len: i32,
    pub prefix_off: i32, pub prefix_len: i32,
    pub self_off: i32, pub tile_start: i32,
    pub flags: i32,  // CEVK_SEG_BIDIRECTIONAL
}

pub const CEVK_SEG_BIDIRECTIONAL: i32 = 1;

pub const CEVK_BF16: i32 = 1;
pub const CEVK_F32: i32 = 2;

pub const CEVK_OK: i32 = 0;
pub const CEVK_E_SHAPE: i32 = -1;
pub const CEVK_E_RANGE: i32 = -2;
pub const CEVK_E_CUDA: i32 = -3;
pub const CEVK_E_TIMEOUT: i32 = -5;
pub const CEVK_E_UNSUPPORTED: i32 = -6;
pub const CEVK_IPC_HANDLE_BYTES: usize = 64;
pub const CEVK_GDN_NOALLOC_MAX_BYTES: usize = 16 << 20;

// edition 2024: foreign blocks are `unsafe extern`
unsafe extern "C" {
    pub fn cevk_last_error() -> *const c_char;
    pub fn cevk_version() -> i32;
    pub fn cevk_device_status() -> i32;
    pub fn cevk_selftest_wait_timeout(limit_cycles: i64, stream: *mut c_void) -> i32;
    pub fn cevk_attn_schedule(segs: *mut cevk_segment, n_segs: i32, n_tokens: i32, n_kv_rows: i32,
                              hq: i32, hkv: i32, head_dim: i32, dtype: i32, n_tiles: *mut i32) -> i32;
    pub fn cevk_attn_packed_prefill(q: *const c_void, k: *const c_void, v: *const c_void, o: *mut c_void,
                                    n_tokens: i32, n_kv_rows: i32, hq: i32, hkv: i32, head_dim: i32,
                                    q_row_stride: i32, kv_row_stride: i32, o_row_stride: i32,
                                    segs_dev: *const cevk_segment, n_segs: i32, n_tiles: i32,
                                    scale: f32, dtype: i32, stream: *mut c_void) -> i32;
    pub fn cevk_attn_split_plan(segs: *const cevk_segment, n_segs: i32, n_tiles: i32, hkv: i32, head_dim: i32,
                                dtype: i32, n_sms: i32, n_split: *mut i32, workspace_bytes: *mut i64) -> i32;
    pub fn cevk_attn_split_workspace_size(n_tiles: i32, hkv: i32, head_dim: i32, n_split: i32) -> i64;
    pub fn cevk_attn_packed_prefill_split(q: *const c_void, k: *const c_void, v: *const c_void, o: *mut c_void,
                                          n_tokens: i32, n_kv_rows: i32, hq: i32, hkv: i32, head_dim: i32,
                                          q_row_stride: i32, kv_row_stride: i32, o_row_stride: i32,
                                          segs_dev: *const cevk_segment, n_segs: i32, n_tiles: i32,
                                          scale: f32, n_split: i32, workspace: *mut c_void,
                                          workspace_bytes: i64, dtype: i32, stream: *mut c_void) -> i32;
    // the fused head all-gather of the KV-head split
    pub fn cevk_ipc_alloc(bytes: i64, dev_ptr: *mut *mut c_void) -> i32;
    pub fn cevk_ipc_free(dev_ptr: *mut c_void) -> i32;
    pub fn cevk_ipc_handle(dev_ptr: *const c_void, handle: *mut c_void) -> i32;  // 64 bytes out
    pub fn cevk_ipc_open(handle: *const c_void, dev_ptr: *mut *mut c_void) -> i32;
    pub fn cevk_ipc_close(dev_ptr: *mut c_void) -> i32;
    pub fn cevk_attn_packed_prefill_gather(q: *const c_void, k: *const c_void, v: *const c_void,
                                           o_bufs: *const *mut c_void, n_bufs: i32, n_tokens: i32, n_kv_rows: i32,
                                           hq: i32, hkv: i32, head_dim: i32, q_row_stride: i32,
                                           kv_row_stride: i32, o_row_stride: i32, segs_dev: *const cevk_segment,
                                           n_segs: i32, n_tiles: i32, scale: f32, n_split: i32,
                                           workspace: *mut c_void, workspace_bytes: i64, stream: *mut c_void) -> i32;
    pub fn cevk_gather_signal(flags: *const *mut i32, world: i32, rank: i32, epoch: i32, stream: *mut c_void) -> i32;
    pub fn cevk_gather_wait(flags: *const i32, world: i32, epoch: i32, limit_cycles: i64, stream: *mut c_void) -> i32;
    pub fn cevk_gather_signal_dev(flags: *const *mut i32, world: i32, rank: i32, epoch: *mut i32, stream: *mut c_void)
        -> i32;
    pub fn cevk_gather_wait_dev(flags: *const i32, world: i32, epoch: *const i32, limit_cycles: i64,
                                stream: *mut c_void) -> i32;
    pub fn cevk_rows_to_peers(src: *const c_void, dst: *const *mut c_void, n_dst: i32, bytes: i64,
                              stream: *mut c_void) -> i32;
    pub fn cevk_gather_sync_dev(flags: *const *mut i32, world: i32, rank: i32, epoch: *mut i32,
                                own_flags: *const i32, limit_cycles: i64, stream: *mut c_void) -> i32;
    pub fn cevk_rows_gather_dev(src: *const c_void, dst: *const *mut c_void, n_dst: i32, bytes: i64,
                                flags: *const *mut i32, world: i32, rank: i32, epoch: *mut i32, own_flags: *const i32,
                                limit_cycles: i64, ticket: *mut u32, stream: *mut c_void) -> i32;
    pub fn cevk_qk_norm_rope(qkv: *const c_void, row_stride: i32, q_head_stride: i32, k_col: i32, v_col: i32,
                             q_norm_w: *const c_void, k_norm_w: *const c_void, eps: f32, norm_plus_one: i32,
                             pos: *const i32, theta: f64, rotary_dim: i32, q_out: *mut c_void,
                             k_arena: *mut c_void, v_arena: *mut c_void, kv_row_stride: i32,
                             kv_rows: *const i32, n_tokens: i32, hq: i32, hkv: i32, head_dim: i32,
                             dtype: i32, stream: *mut c_void) -> i32;
    pub fn cevk_rms_norm(x: *const c_void, residual: *mut c_void, add: *const c_void, w: *const c_void,
                         out: *mut c_void, n: i32, hidden: i32, eps: f32, plus_one: i32, dtype: i32,
                         stream: *mut c_void) -> i32;
    pub fn cevk_swiglu(gu: *const c_void, out: *mut c_void, n: i32, inter: i32, dtype: i32,
                       stream: *mut c_void) -> i32;
    pub fn cevk_embed(table: *const c_void, ids: *const i32, out: *mut c_void, n: i32, hidden: i32,
                      vocab: i32, dtype: i32, stream: *mut c_void) -> i32;
    pub fn cevk_sigmoid_gate(a: *const c_void, gate: *const c_void, gate_row_stride: i32,
                             gate_head_stride: i32, out: *mut c_void, n: i32, heads: i32, head_dim: i32,
                             dtype: i32, stream: *mut c_void) -> i32;
    pub fn cevk_readout(x: *const c_void, rows: *const i32, n_rows: i32, norm_w: *const c_void, eps: f32,
                        norm_plus_one: i32, code_head: *const f32, n_codes: i32, hidden_out: *mut f32,
                        logits_out: *mut f32, hidden: i32, dtype: i32, stream: *mut c_void) -> i32;
    pub fn cevk_gdn_conv(mixed: *const c_void, mixed_row_stride: i32, conv_w: *const c_void,
                         tail_in: *const c_void, tail_batch_stride: i64, tail_out: *mut c_void,
                         out: *mut c_void, b: i32, t: i32, c: i32, k: i32, dtype: i32,
                         stream: *mut c_void) -> i32;
    pub fn cevk_gdn_workspace_size(b: i32, t: i32, nv: i32, dk: i32, dv: i32) -> usize;
    pub fn cevk_gdn_chunk_prefill(conv_out: *const c_void, c: i32, ab: *const c_void, ab_row_stride: i32,
                                  z: *const c_void, z_row_stride: i32, a_log: *const f32, dt_bias: *const f32,
                                  norm_w: *const c_void, eps: f32, s_in: *const f32, s_batch_stride: i64,
                                  s_out: *mut f32, y: *mut c_void, b: i32, t: i32, nk: i32, nv: i32,
                                  dk: i32, dv: i32, workspace: *mut c_void, workspace_bytes: usize,
                                  dtype: i32, stream: *mut c_void) -> i32;
    // no counterpart in the reference: the GDN call for hosts that cannot
    // hand the library a workspace (scratch in a 16 MiB static device array)
    pub fn cevk_gdn_chunk_prefill_noalloc(conv_out: *const c_void, c: i32, ab: *const c_void, ab_row_stride: i32,
                                          z: *const c_void, z_row_stride: i32, a_log: *const f32,
                                          dt_bias: *const f32, norm_w: *const c_void, eps: f32, s_in: *const f32,
                                          s_batch_stride: i64, s_out: *mut f32, y: *mut c_void, b: i32, t: i32,
                                          nk: i32, nv: i32, dk: i32, dv: i32, dtype: i32,
                                          stream: *mut c_void) -> i32;
    pub fn cevk_short_conv(bcx: *const c_void, conv_w: *const c_void, bias: *const c_void,
                           tail_in: *const c_void, tail_batch_stride: i64, tail_out: *mut c_void,
                           y: *mut c_void, b: i32, t: i32, d: i32, k: i32, dtype: i32,
                           stream: *mut c_void) -> i32;
    pub fn cevk_debias(logits: *const f32, cf_logits: *const f32, ld: i32, span: *const i32,
                       n_options: *const i32, order: *const i32, n_questions: i32, scores: *mut f32,
                       probs: *mut f64, out_ld: i32, stream: *mut c_void) -> i32;
}
