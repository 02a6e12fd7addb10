// Per-head RMSNorm + (partial) half-split RoPE at explicit positions, with
// Q written densely and K/V written straight into their arena rows: one
// pass over the projection output replaces the reference's q_norm / k_norm,
// Rotary::apply, the head transposes and the K/V concatenation
// (qwen3.rs:190-200, qwen35.rs:529-541, lfm2.rs:147-156).
//
// One block per token (cos/sin computed once per token), one warp per head
// row; the warp holds the row in shared memory so the rotation partner
// (d +- rot/2) can live in any lane.  HBM-bound: each element is read once
// and written once.
#include "common.cuh"

namespace cevk {

template <typename T>
__global__ void __launch_bounds__(256) qk_norm_rope_kernel(
    const T* __restrict__ qkv, int row_stride, int q_head_stride, int k_col, int v_col, const T* __restrict__ qw,
    const T* __restrict__ kw, float eps, int plus_one, const int32_t* __restrict__ pos, double theta, int rot,
    T* __restrict__ q_out, T* __restrict__ k_arena, T* __restrict__ v_arena, int kv_rs, const int32_t* __restrict__ kv_rows,
    int hq, int hkv, int D) {
  // One block per token: cos/sin of its position are computed once and
  // shared by all of its heads.
  extern __shared__ float sm[];
  const int half = rot / 2;
  float* cs = sm;             // [half]
  float* sn = sm + half;      // [half]
  float* rows = sm + 2 * half;  // [8][D]
  const int t = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float p = (float)pos[t];
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    // 1f32 / (theta^(2i/rot) as f32), the power in f64 (qwen3.rs:109-112).
    const float inv = 1.0f / (float)pow(theta, (double)(2 * i) / (double)rot);
    const float ang = p * inv;
    cs[i] = cosf(ang);
    sn[i] = sinf(ang);
  }
  __syncthreads();
  float* buf = rows + warp * D;
  const int heads = hq + 2 * hkv;
  for (int h = warp; h < heads; h += 8) {
    const T* src;
    T* dst;
    const T* w = nullptr;
    if (h < hq) {
      src = qkv + (size_t)t * row_stride + (size_t)h * q_head_stride;
      dst = q_out + ((size_t)t * hq + h) * D;
      w = qw;
    } else if (h < hq + hkv) {
      src = qkv + (size_t)t * row_stride + k_col + (size_t)(h - hq) * D;
      dst = k_arena + (size_t)kv_rows[t] * kv_rs + (size_t)(h - hq) * D;
      w = kw;
    } else {
      src = qkv + (size_t)t * row_stride + v_col + (size_t)(h - hq - hkv) * D;
      dst = v_arena + (size_t)kv_rows[t] * kv_rs + (size_t)(h - hq - hkv) * D;
    }
    if (!w) {  // V: a plain copy into the arena
      for (int d = lane; d < D; d += 32) dst[d] = src[d];
      continue;
    }
    float ss = 0.f;
    for (int d = lane; d < D; d += 32) {
      const float x = to_f(src[d]);
      buf[d] = x;
      ss += x * x;
    }
    ss = warp_sum(ss);
    const float r = rsqrtf(ss / D + eps);
    for (int d = lane; d < D; d += 32) {
      const float wv = to_f(w[d]) + (plus_one ? 1.f : 0.f);
      // Like the reference, the normed value is in the model dtype before RoPE.
      buf[d] = to_f(from_f<T>(buf[d] * r * wv));
    }
    __syncwarp();
    for (int d = lane; d < D; d += 32) {
      float y = buf[d];
      if (d < rot) {
        const int i = d < half ? d : d - half;
        y = d < half ? buf[d] * cs[i] - buf[d + half] * sn[i] : buf[d] * cs[i] + buf[d - half] * sn[i];
      }
      dst[d] = from_f<T>(y);
    }
    __syncwarp();
  }
}

}  // namespace cevk

using namespace cevk;

extern "C" int cevk_qk_norm_rope(const void* qkv, int32_t row_stride, int32_t q_head_stride, int32_t k_col,
                                 int32_t v_col, const void* q_norm_w, const void* k_norm_w, float eps,
                                 int32_t norm_plus_one, const int32_t* pos, double theta, int32_t rotary_dim,
                                 void* q_out, void* k_arena, void* v_arena, int32_t kv_row_stride,
                                 const int32_t* kv_rows, int32_t n_tokens, int32_t hq, int32_t hkv, int32_t head_dim,
                                 int32_t dtype, void* stream) {
  if (!qkv || !q_norm_w || !k_norm_w || !pos || !q_out || !k_arena || !v_arena || !kv_rows)
    return set_error(CEVK_E_SHAPE, "qk_norm_rope: null pointer");
  if (head_dim <= 0 || head_dim > 512 || rotary_dim < 0 || rotary_dim > head_dim || (rotary_dim & 1))
    return set_error(CEVK_E_SHAPE, "qk_norm_rope: head_dim %d / rotary_dim %d", head_dim, rotary_dim);
  if (kv_row_stride < hkv * head_dim) return set_error(CEVK_E_SHAPE, "qk_norm_rope: kv row stride too small");
  if (n_tokens <= 0) return CEVK_OK;
  const unsigned blocks = (unsigned)n_tokens;
  const size_t smem = (rotary_dim + 8 * head_dim) * sizeof(float);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == CEVK_BF16) {
    qk_norm_rope_kernel<__nv_bfloat16><<<blocks, 256, smem, st>>>(
        (const __nv_bfloat16*)qkv, row_stride, q_head_stride, k_col, v_col, (const __nv_bfloat16*)q_norm_w,
        (const __nv_bfloat16*)k_norm_w, eps, norm_plus_one, pos, theta, rotary_dim, (__nv_bfloat16*)q_out,
        (__nv_bfloat16*)k_arena, (__nv_bfloat16*)v_arena, kv_row_stride, kv_rows, hq, hkv, head_dim);
  } else if (dtype == CEVK_F32) {
    qk_norm_rope_kernel<float><<<blocks, 256, smem, st>>>(
        (const float*)qkv, row_stride, q_head_stride, k_col, v_col, (const float*)q_norm_w, (const float*)k_norm_w, eps,
        norm_plus_one, pos, theta, rotary_dim, (float*)q_out, (float*)k_arena, (float*)v_arena, kv_row_stride, kv_rows,
        hq, hkv, head_dim);
  } else {
    return set_error(CEVK_E_UNSUPPORTED, "qk_norm_rope: dtype %d", dtype);
  }
  return check_launch("qk_norm_rope_kernel");
}
