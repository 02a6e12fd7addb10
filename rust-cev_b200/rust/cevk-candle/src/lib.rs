//! candle glue for libcevk, the B200 kernels of cev's decision forward.
//!
//! Where the calls go in the reference (`crates/cev-model/src`):
//! - `Attention::attend` (qwen3.rs:206-220, qwen35.rs:563-579,
//!   lfm2.rs:160-168): [`PackedAttention`] over the K/V arena, one
//!   [`Seg`] per tail / suffix / prefill chunk / padded row instead of the
//!   host-built additive mask (engine.rs:418-442);
//! - the q/k norm + RoPE + K/V `cat` of `Attention::forward`
//!   (qwen3.rs:190-204): [`qk_norm_rope`];
//! - `chunk_gated_delta_rule` + the gated norm of `GatedDeltaNet::forward`
//!   (qwen35.rs:301-368, 443-451): [`gdn_chunk_prefill`];
//! - `ShortConv::forward`'s conv part (lfm2.rs:199-219): [`short_conv`].
//!
//! Every op runs on candle's CUDA stream of the tensors' device and fails
//! on the CPU: there is no CPU fallback.  Ops that write into long-lived
//! buffers (the K/V arena, recurrent states) take them as tensors the
//! engine owns exclusively and write through their device pointers.
use std::ffi::{CStr, c_void};

use candle_core::backend::BackendStorage;
use candle_core::cuda_backend::cudarc::driver::{CudaSlice, DevicePtr, DeviceRepr};
use candle_core::cuda_backend::{CudaDType, WrapErr};
use candle_core::{CpuStorage, CudaDevice, CudaStorage, CustomOp3, DType, Layout, Result, Shape, Storage, Tensor, bail};
use cevk_sys as ffi;

/// Status -> candle error, with the library's message for this thread.
pub fn check(rc: i32) -> Result<()> {
    if rc == ffi::CEVK_OK {
        return Ok(());
    }
    let msg = unsafe { CStr::from_ptr(ffi::cevk_last_error()) }.to_string_lossy().into_owned();
    bail!("cevk status {rc}: {msg}")
}

/// A bounded device wait that gave up (CEVK_E_TIMEOUT) fails the request
/// as an internal error; call once per request after its last kernel.
pub fn device_status() -> Result<()> {
    check(unsafe { ffi::cevk_device_status() })
}

fn dtype_code(dt: DType) -> Result<i32> {
    match dt {
        DType::BF16 => Ok(ffi::CEVK_BF16),
        DType::F32 => Ok(ffi::CEVK_F32),
        other => bail!("cevk: dtype {other:?} not supported"),
    }
}

fn stream(dev: &CudaDevice) -> *mut c_void {
    dev.cuda_stream().cu_stream() as *mut c_void
}

/// Device address of a storage at a layout's start offset.
fn ptr_of<T: CudaDType + DeviceRepr>(s: &CudaStorage, l: &Layout) -> Result<*mut c_void> {
    let slice = s.as_cuda_slice::<T>()?;
    let st = s.device().cuda_stream();
    let (p, _sync) = slice.device_ptr(&st);
    Ok((p as usize + l.start_offset() * std::mem::size_of::<T>()) as *mut c_void)
}

fn dev_ptr(s: &CudaStorage, l: &Layout) -> Result<*mut c_void> {
    match s.dtype() {
        DType::BF16 => ptr_of::<half::bf16>(s, l),
        DType::F32 => ptr_of::<f32>(s, l),
        DType::I64 => ptr_of::<i64>(s, l),
        DType::U32 => ptr_of::<u32>(s, l),
        other => bail!("cevk: dtype {other:?} not supported"),
    }
}

/// Device pointer of a contiguous CUDA tensor (an exclusively owned buffer
/// the op reads or writes), with its candle stream.
fn tensor_ptr(t: &Tensor) -> Result<(*mut c_void, CudaDevice)> {
    if !t.is_contiguous() {
        bail!("cevk: tensor must be contiguous");
    }
    let (st, l) = t.storage_and_layout();
    match &*st {
        Storage::Cuda(s) => Ok((dev_ptr(s, l)?, s.device().clone())),
        _ => bail!("cevk: CUDA tensors only (no CPU fallback)"),
    }
}

fn opt_ptr(t: Option<&Tensor>) -> Result<*mut c_void> {
    Ok(match t {
        Some(t) => tensor_ptr(t)?.0,
        None => std::ptr::null_mut(),
    })
}

/// One attention segment descriptor (`cevk_segment`) in device memory.
#[repr(transparent)]
#[derive(Clone, Copy, Default)]
pub struct Seg(pub ffi::cevk_segment);
unsafe impl DeviceRepr for Seg {}

/// The segments of one pass, validated and tiled on the host
/// (`cevk_attn_schedule`), then uploaded.
pub struct Segments {
    pub dev: CudaSlice<Seg>,
    pub n_segs: i32,
    pub n_tiles: i32,
}

impl Segments {
    pub fn new(device: &CudaDevice, segs: &mut [ffi::cevk_segment], n_tokens: usize, n_kv_rows: usize, hq: usize,
               hkv: usize, head_dim: usize, dtype: DType) -> Result<Self> {
        let mut n_tiles = 0i32;
        check(unsafe {
            ffi::cevk_attn_schedule(segs.as_mut_ptr(), segs.len() as i32, n_tokens as i32, n_kv_rows as i32,
                                    hq as i32, hkv as i32, head_dim as i32, dtype_code(dtype)?, &mut n_tiles)
        })?;
        let host: Vec<Seg> = segs.iter().copied().map(Seg).collect();
        let dev = device.cuda_stream().memcpy_stod(&host).w()?;
        Ok(Self { dev, n_segs: segs.len() as i32, n_tiles })
    }
}

/// Packed block-masked prefill attention (`cevk_attn_packed_prefill`):
/// `q` [T, Hq, D] against the K/V arena `k`, `v` [rows, Hkv, D]; returns
/// o [T, Hq, D].  Masked query-key tiles are skipped, not multiplied.
pub struct PackedAttention<'a> {
    pub segments: &'a Segments,
    pub scale: f32,
}

impl CustomOp3 for PackedAttention<'_> {
    fn name(&self) -> &'static str {
        "cevk-packed-attention"
    }

    fn cpu_fwd(&self, _: &CpuStorage, _: &Layout, _: &CpuStorage, _: &Layout, _: &CpuStorage, _: &Layout)
        -> Result<(CpuStorage, Shape)> {
        bail!("cevk: packed attention runs on CUDA only")
    }

    fn cuda_fwd(&self, q: &CudaStorage, ql: &Layout, k: &CudaStorage, kl: &Layout, v: &CudaStorage, vl: &Layout)
        -> Result<(CudaStorage, Shape)> {
        let (t, hq, d) = ql.shape().dims3()?;
        let (rows, hkv, dk) = kl.shape().dims3()?;
        if dk != d || vl.shape() != kl.shape() || !ql.is_contiguous() || !kl.is_contiguous() || !vl.is_contiguous() {
            bail!("cevk: attention operands must be contiguous [T, Hq, D] / [rows, Hkv, D]");
        }
        let dt = q.dtype();
        let dev = q.device().clone();
        let (o, optr) = match dt {
            DType::BF16 => {
                let o = unsafe { dev.alloc::<half::bf16>(t * hq * d)? };
                let p = o.device_ptr(&dev.cuda_stream()).0 as *mut c_void;
                (CudaStorage::wrap_cuda_slice(o, dev.clone()), p)
            }
            DType::F32 => {
                let o = unsafe { dev.alloc::<f32>(t * hq * d)? };
                let p = o.device_ptr(&dev.cuda_stream()).0 as *mut c_void;
                (CudaStorage::wrap_cuda_slice(o, dev.clone()), p)
            }
            other => bail!("cevk: dtype {other:?} not supported"),
        };
        let segs = self.segments.dev.device_ptr(&dev.cuda_stream()).0 as *const ffi::cevk_segment;
        check(unsafe {
            ffi::cevk_attn_packed_prefill(dev_ptr(q, ql)?, dev_ptr(k, kl)?, dev_ptr(v, vl)?, optr, t as i32,
                                          rows as i32, hq as i32, hkv as i32, d as i32, (hq * d) as i32,
                                          (hkv * d) as i32, (hq * d) as i32, segs, self.segments.n_segs,
                                          self.segments.n_tiles, self.scale, dtype_code(dt)?, stream(&dev))
        })?;
        Ok((o, Shape::from((t, hq, d))))
    }
}

/// Per-head q/k RMSNorm (`w` or `1 + w`) + (partial) RoPE at explicit
/// positions, writing Q to `q_out` and this pass's K/V into the arena rows
/// `kv_rows` (`cevk_qk_norm_rope`): qkv [T, row_stride] holds q (per head
/// `q_head_stride` apart), k at column `k_col`, v at `v_col`.
#[allow(clippy::too_many_arguments)]
pub fn qk_norm_rope(qkv: &Tensor, q_head_stride: usize, k_col: usize, v_col: usize, q_norm: &Tensor,
                    k_norm: &Tensor, eps: f32, plus_one: bool, pos: &Tensor, theta: f64, rotary_dim: usize,
                    q_out: &Tensor, k_arena: &Tensor, v_arena: &Tensor, kv_rows: &Tensor) -> Result<()> {
    let (t, row_stride) = qkv.dims2()?;
    let (_, hq, d) = q_out.dims3()?;
    let (_, hkv, _) = k_arena.dims3()?;
    let (qp, dev) = tensor_ptr(qkv)?;
    check(unsafe {
        ffi::cevk_qk_norm_rope(qp, row_stride as i32, q_head_stride as i32, k_col as i32, v_col as i32,
                               tensor_ptr(q_norm)?.0, tensor_ptr(k_norm)?.0, eps, plus_one as i32,
                               tensor_ptr(pos)?.0 as *const i32, theta, rotary_dim as i32, tensor_ptr(q_out)?.0,
                               tensor_ptr(k_arena)?.0, tensor_ptr(v_arena)?.0, (hkv * d) as i32,
                               tensor_ptr(kv_rows)?.0 as *const i32, t as i32, hq as i32, hkv as i32, d as i32,
                               dtype_code(qkv.dtype())?, stream(&dev))
    })
}

/// The chunked gated delta rule with its prologue and gated-norm epilogue
/// (`cevk_gdn_chunk_prefill`) for B rows of T tokens: returns y
/// [B*T, nv*dv].  `s_in` [B or 1, nv, dk, dv] f32 (one row broadcasts) or
/// None; `s_out` [B, nv, dk, dv] f32 receives the state after T tokens.
/// The workspace comes from candle's allocator.
#[allow(clippy::too_many_arguments)]
pub fn gdn_chunk_prefill(conv_out: &Tensor, ab: &Tensor, z: &Tensor, a_log: &Tensor, dt_bias: &Tensor,
                         norm_w: &Tensor, eps: f32, s_in: Option<&Tensor>, s_out: Option<&Tensor>, b: usize,
                         t: usize, nk: usize, nv: usize, dk: usize, dv: usize) -> Result<Tensor> {
    let (cp, dev) = tensor_ptr(conv_out)?;
    let c = conv_out.dim(1)?;
    let y = Tensor::zeros((b * t, nv * dv), conv_out.dtype(), conv_out.device())?;
    let ws_bytes = unsafe { ffi::cevk_gdn_workspace_size(b as i32, t as i32, nv as i32, dk as i32, dv as i32) };
    let ws = Tensor::zeros(ws_bytes.div_ceil(4), DType::F32, conv_out.device())?;
    let s_bs = match s_in {
        Some(s) if s.dim(0)? > 1 => (nv * dk * dv) as i64,
        _ => 0,
    };
    check(unsafe {
        ffi::cevk_gdn_chunk_prefill(cp, c as i32, tensor_ptr(ab)?.0, ab.dim(1)? as i32, tensor_ptr(z)?.0,
                                    z.dim(1)? as i32, tensor_ptr(a_log)?.0 as *const f32,
                                    tensor_ptr(dt_bias)?.0 as *const f32, tensor_ptr(norm_w)?.0, eps,
                                    opt_ptr(s_in)? as *const f32, s_bs, opt_ptr(s_out)? as *mut f32,
                                    tensor_ptr(&y)?.0, b as i32, t as i32, nk as i32, nv as i32, dk as i32,
                                    dv as i32, tensor_ptr(&ws)?.0, ws_bytes, dtype_code(conv_out.dtype())?,
                                    stream(&dev))
    })?;
    Ok(y)
}

/// LFM2 gated short conv (`cevk_short_conv`): bcx [B*T, 3d] (b | c | x per
/// token) -> y [B*T, d], continuing from `tail_in` [B or 1, d, K-1] and
/// writing the new tail to `tail_out` when given.
#[allow(clippy::too_many_arguments)]
pub fn short_conv(bcx: &Tensor, b: usize, t: usize, d: usize, conv_w: &Tensor, bias: Option<&Tensor>,
                  tail_in: Option<&Tensor>, tail_out: Option<&Tensor>) -> Result<Tensor> {
    let (bp, dev) = tensor_ptr(bcx)?;
    let k = conv_w.dim(1)?;
    let y = Tensor::zeros((b * t, d), bcx.dtype(), bcx.device())?;
    let tbs = match tail_in {
        Some(s) if s.dim(0)? > 1 => (d * (k - 1)) as i64,
        _ => 0,
    };
    check(unsafe {
        ffi::cevk_short_conv(bp, tensor_ptr(conv_w)?.0, opt_ptr(bias)?, opt_ptr(tail_in)?, tbs, opt_ptr(tail_out)?,
                             tensor_ptr(&y)?.0, b as i32, t as i32, d as i32, k as i32, dtype_code(bcx.dtype())?,
                             stream(&dev))
    })?;
    Ok(y)
}
