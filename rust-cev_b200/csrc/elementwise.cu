// Bandwidth-bound glue of the decoder forward, each a single pass over HBM:
// residual add + RMSNorm, SwiGLU, embedding gather, sigmoid output gate and
// the Codes readout (final norm at the answer rows + f32 code logits).
#include "common.cuh"

namespace cevk {

// 8 consecutive elements <-> 8 floats (16 B for bf16, 32 B for f32).
__device__ __forceinline__ void load8(const __nv_bfloat16* p, float* f) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 v = __bfloat1622float2(h[i]);
    f[2 * i] = v.x;
    f[2 * i + 1] = v.y;
  }
}
__device__ __forceinline__ void store8(__nv_bfloat16* p, const float* f) {
  uint4 u;
  u.x = pack_bf16x2(f[0], f[1]);
  u.y = pack_bf16x2(f[2], f[3]);
  u.z = pack_bf16x2(f[4], f[5]);
  u.w = pack_bf16x2(f[6], f[7]);
  *reinterpret_cast<uint4*>(p) = u;
}
__device__ __forceinline__ void load8(const float* p, float* f) {
  const float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
  f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}
__device__ __forceinline__ void store8(float* p, const float* f) {
  reinterpret_cast<float4*>(p)[0] = make_float4(f[0], f[1], f[2], f[3]);
  reinterpret_cast<float4*>(p)[1] = make_float4(f[4], f[5], f[6], f[7]);
}
template <typename T>
__device__ __forceinline__ void round8(float* f) {
#pragma unroll
  for (int i = 0; i < 8; ++i) f[i] = to_f(from_f<T>(f[i]));
}

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float s = 0.f;
  const int nw = blockDim.x >> 5;
  for (int i = 0; i < nw; ++i) s += red[i];
  return s;
}

// residual (optional) += add; out = rms_norm(residual or x) * (w or 1+w).
// One block per row; the row stays in registers (V vectors of 8 per
// thread), and every load is issued before the first use (columns past the
// row are clamped and masked, so no load sits behind a branch).
template <typename T, int V, bool RESID, bool OUT>
__global__ void __launch_bounds__(256) rms_norm_kernel(const T* __restrict__ x, T* __restrict__ residual,
                                                       const T* __restrict__ add, const T* __restrict__ w,
                                                       T* __restrict__ out, int hidden, float eps, int plus_one) {
  __shared__ float red[32];
  const size_t row = (size_t)blockIdx.x * hidden;
  const T* src = RESID ? residual + row : x + row;
  float f[V][8], a[V][8];
#pragma unroll
  for (int v = 0; v < V; ++v) {
    const int c = min((v * 256 + (int)threadIdx.x) * 8, hidden - 8);
    load8(src + c, f[v]);
    if (RESID) load8(add + row + c, a[v]);
  }
  float ss = 0.f;
#pragma unroll
  for (int v = 0; v < V; ++v) {
    const int c = (v * 256 + threadIdx.x) * 8;
    if (RESID) {
#pragma unroll
      for (int i = 0; i < 8; ++i) f[v][i] += a[v][i];
      round8<T>(f[v]);  // the sum is a model-dtype tensor in the reference
      if (c < hidden) store8(residual + row + c, f[v]);
    }
    if (c < hidden)
#pragma unroll
      for (int i = 0; i < 8; ++i) ss += f[v][i] * f[v][i];
  }
  if constexpr (OUT) {  // else: residual add only
    float g[V][8];
#pragma unroll
    for (int v = 0; v < V; ++v) load8(w + min((v * 256 + (int)threadIdx.x) * 8, hidden - 8), g[v]);
    const float r = rsqrtf(block_sum(ss, red) / hidden + eps);
    const float one = plus_one ? 1.f : 0.f;
#pragma unroll
    for (int v = 0; v < V; ++v) {
      const int c = (v * 256 + threadIdx.x) * 8;
#pragma unroll
      for (int i = 0; i < 8; ++i) f[v][i] = f[v][i] * r * (g[v][i] + one);
      if (c < hidden) store8(out + row + c, f[v]);
    }
  }
}

// One vector of 8 per thread: blockIdx.x over the row, blockIdx.y over rows.
template <typename T>
__global__ void __launch_bounds__(256) swiglu_kernel(const T* __restrict__ gu, T* __restrict__ out, int n, int inter) {
  const int c = (blockIdx.x * 256 + threadIdx.x) * 8;
  if (c >= inter) return;
  for (int r = blockIdx.y; r < n; r += gridDim.y) {
    float g[8], u[8];
    load8(gu + (size_t)r * 2 * inter + c, g);
    load8(gu + (size_t)r * 2 * inter + inter + c, u);
#pragma unroll
    for (int j = 0; j < 8; ++j) g[j] = g[j] / (1.f + __expf(-g[j])) * u[j];
    store8(out + (size_t)r * inter + c, g);
  }
}

template <typename T>
__global__ void embed_kernel(const T* __restrict__ table, const int32_t* __restrict__ ids, T* __restrict__ out,
                             int hidden) {
  const size_t src = (size_t)ids[blockIdx.x] * hidden, dst = (size_t)blockIdx.x * hidden;
  for (int c = threadIdx.x * 8; c < hidden; c += blockDim.x * 8) {
    float f[8];
    load8(table + src + c, f);
    store8(out + dst + c, f);
  }
}

// One vector of 8 per thread: blockIdx.x over the token's heads x D,
// blockIdx.y over tokens.
template <typename T>
__global__ void __launch_bounds__(256) sigmoid_gate_kernel(const T* __restrict__ a, const T* __restrict__ gate, int grs,
                                                           int ghs, T* __restrict__ out, int n, int heads, int D) {
  const int i = blockIdx.x * 256 + threadIdx.x;  // vector index within a token
  if (i >= heads * (D / 8)) return;
  const int h = i / (D / 8), c = (i % (D / 8)) * 8;
  for (int t = blockIdx.y; t < n; t += gridDim.y) {
    float x[8], g[8];
    load8(a + ((size_t)t * heads + h) * D + c, x);
    load8(gate + (size_t)t * grs + (size_t)h * ghs + c, g);
#pragma unroll
    for (int j = 0; j < 8; ++j) x[j] = x[j] * (1.f / (1.f + __expf(-g[j])));
    store8(out + ((size_t)t * heads + h) * D + c, x);
  }
}

template <typename T>
__global__ void __launch_bounds__(256) readout_kernel(const T* __restrict__ x, const int32_t* __restrict__ rows,
                                                      const T* __restrict__ w, float eps, int plus_one,
                                                      const float* __restrict__ head, int n_codes,
                                                      float* __restrict__ hidden_out, float* __restrict__ logits,
                                                      int hidden) {
  extern __shared__ float hs[];
  __shared__ float red[32];
  const T* src = x + (size_t)rows[blockIdx.x] * hidden;
  float ss = 0.f;
  for (int c = threadIdx.x; c < hidden; c += blockDim.x) {
    const float v = to_f(src[c]);
    hs[c] = v;
    ss += v * v;
  }
  const float r = rsqrtf(block_sum(ss, red) / hidden + eps);
  for (int c = threadIdx.x; c < hidden; c += blockDim.x) {
    // final norm output is a model-dtype tensor, then cast to f32
    const float v = to_f(from_f<T>(hs[c] * r * (to_f(w[c]) + (plus_one ? 1.f : 0.f))));
    hs[c] = v;
    hidden_out[(size_t)blockIdx.x * hidden + c] = v;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int k = warp; k < n_codes; k += blockDim.x >> 5) {
    const float* hr = head + (size_t)k * hidden;
    float acc = 0.f;
    for (int c = lane; c < hidden; c += 32) acc += hs[c] * hr[c];
    acc = warp_sum(acc);
    if (lane == 0) logits[(size_t)blockIdx.x * n_codes + k] = acc;
  }
}


}  // namespace cevk

using namespace cevk;

#define CEVK_DISPATCH(dtype, BF16_CALL, F32_CALL)                                   \
  do {                                                                             \
    if ((dtype) == CEVK_BF16) {                                                    \
      using T = __nv_bfloat16;                                                     \
      BF16_CALL;                                                                   \
    } else if ((dtype) == CEVK_F32) {                                              \
      using T = float;                                                             \
      F32_CALL;                                                                    \
    } else {                                                                       \
      return set_error(CEVK_E_UNSUPPORTED, "dtype %d", (int)(dtype));              \
    }                                                                              \
  } while (0)

extern "C" {

int cevk_rms_norm(const void* x, void* residual, const void* add, const void* w, void* out, int32_t n, int32_t hidden,
                  float eps, int32_t plus_one, int32_t dtype, void* stream) {
  if ((!x && !residual) || (residual && !add) || (out && !w) || (!out && !residual))
    return set_error(CEVK_E_SHAPE, "rms_norm: null pointer");
  if (hidden % 8 || hidden > 256 * 8 * 8)
    return set_error(CEVK_E_SHAPE, "rms_norm: hidden %d (a multiple of 8, at most 16384)", hidden);
  if (n <= 0) return CEVK_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int V = hidden <= 2048 ? 1 : hidden <= 4096 ? 2 : hidden <= 8192 ? 4 : 8;
#define RN(VV, RS, OU)                                                                                       \
  rms_norm_kernel<T, VV, RS, OU><<<n, 256, 0, st>>>((const T*)x, (T*)residual, (const T*)add, (const T*)w, \
                                                    (T*)out, hidden, eps, plus_one)
#define RNV(RS, OU)                    \
  switch (V) {                         \
    case 1: RN(1, RS, OU); break;      \
    case 2: RN(2, RS, OU); break;      \
    case 4: RN(4, RS, OU); break;      \
    default: RN(8, RS, OU); break;     \
  }
#define CALL                                    \
  if (residual && out) { RNV(true, true); }     \
  else if (residual) { RNV(true, false); }      \
  else { RNV(false, true); }
  CEVK_DISPATCH(dtype, CALL, CALL);
#undef CALL
#undef RNV
#undef RN
  return check_launch("rms_norm_kernel");
}

int cevk_swiglu(const void* gu, void* out, int32_t n, int32_t inter, int32_t dtype, void* stream) {
  if (!gu || !out) return set_error(CEVK_E_SHAPE, "swiglu: null pointer");
  if (inter % 8) return set_error(CEVK_E_SHAPE, "swiglu: inter %d not a multiple of 8", inter);
  if (n <= 0) return CEVK_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const dim3 g((unsigned)((inter / 8 + 255) / 256), (unsigned)(n < 65535 ? n : 65535));
#define CALL swiglu_kernel<T><<<g, 256, 0, st>>>((const T*)gu, (T*)out, n, inter)
  CEVK_DISPATCH(dtype, CALL, CALL);
#undef CALL
  return check_launch("swiglu_kernel");
}

int cevk_embed(const void* table, const int32_t* ids, void* out, int32_t n, int32_t hidden, int32_t vocab,
               int32_t dtype, void* stream) {
  (void)vocab;
  if (!table || !ids || !out) return set_error(CEVK_E_SHAPE, "embed: null pointer");
  if (hidden % 8) return set_error(CEVK_E_SHAPE, "embed: hidden %d not a multiple of 8", hidden);
  if (n <= 0) return CEVK_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
#define CALL embed_kernel<T><<<n, 256, 0, st>>>((const T*)table, ids, (T*)out, hidden)
  CEVK_DISPATCH(dtype, CALL, CALL);
#undef CALL
  return check_launch("embed_kernel");
}

int cevk_sigmoid_gate(const void* a, const void* gate, int32_t gate_row_stride, int32_t gate_head_stride, void* out,
                      int32_t n, int32_t heads, int32_t head_dim, int32_t dtype, void* stream) {
  if (!a || !gate || !out) return set_error(CEVK_E_SHAPE, "sigmoid_gate: null pointer");
  if (head_dim % 8 || gate_row_stride % 8 || gate_head_stride % 8)
    return set_error(CEVK_E_SHAPE, "sigmoid_gate: sizes must be multiples of 8");
  if (n <= 0) return CEVK_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const dim3 g((unsigned)((heads * (head_dim / 8) + 255) / 256), (unsigned)(n < 65535 ? n : 65535));
#define CALL sigmoid_gate_kernel<T><<<g, 256, 0, st>>>((const T*)a, (const T*)gate, gate_row_stride, gate_head_stride, (T*)out, n, heads, head_dim)
  CEVK_DISPATCH(dtype, CALL, CALL);
#undef CALL
  return check_launch("sigmoid_gate_kernel");
}

int cevk_readout(const void* x, const int32_t* rows, int32_t n_rows, const void* norm_w, float eps,
                 int32_t norm_plus_one, const float* code_head, int32_t n_codes, float* hidden_out, float* logits_out,
                 int32_t hidden, int32_t dtype, void* stream) {
  if (!x || !rows || !norm_w || !code_head || !hidden_out || !logits_out)
    return set_error(CEVK_E_SHAPE, "readout: null pointer");
  if (hidden > 12288) return set_error(CEVK_E_SHAPE, "readout: hidden %d too large", hidden);
  if (n_rows <= 0) return CEVK_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const size_t smem = hidden * sizeof(float);
#define CALL readout_kernel<T><<<n_rows, 256, smem, st>>>((const T*)x, rows, (const T*)norm_w, eps, norm_plus_one, code_head, n_codes, hidden_out, logits_out, hidden)
  CEVK_DISPATCH(dtype, CALL, CALL);
#undef CALL
  return check_launch("readout_kernel");
}

}  // extern "C"
