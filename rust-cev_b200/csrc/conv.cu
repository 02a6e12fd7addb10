// Causal depthwise convolutions that continue from a cached tail of K-1
// inputs: the LFM2 gated short conv (y = C * conv_K(B * X), lfm2.rs:199-219)
// and the Gated DeltaNet q/k/v conv with SiLU (qwen35.rs:419-431), both
// replacing depthwise_conv1d's K shifted full-tensor passes plus the
// narrow / mul / cat copies (decoder.rs:137-151) with one HBM pass.
//
// One thread per (row, token, 8 channels): 16-byte loads across channels
// are coalesced; the K-1 earlier tokens a thread also reads were read by the
// neighbouring tokens' threads and come from L2.  The tail is read in place
// (batch stride 0 broadcasts one prefix state to every row) and the new tail
// is written by the threads of the last token.
#include "common.cuh"

namespace cevk {

template <typename T>
__device__ __forceinline__ void ld8(const T* p, float* f) {
#pragma unroll
  for (int i = 0; i < 8; ++i) f[i] = to_f(p[i]);
}
__device__ __forceinline__ void ld8(const __nv_bfloat16* p, float* f) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 v = __bfloat1622float2(h[i]);
    f[2 * i] = v.x;
    f[2 * i + 1] = v.y;
  }
}

// GATED: y = c * (bias + sum_k w_k * (b*x)[t-K+1+k]); else y = silu(sum_k w_k * x[t-K+1+k]).
template <typename T, bool GATED, int K>
__global__ void __launch_bounds__(256) causal_conv_kernel(const T* __restrict__ in, int in_row, const T* __restrict__ w,
                                                          const T* __restrict__ bias, const T* __restrict__ tail_in,
                                                          long long tail_bs, T* __restrict__ tail_out,
                                                          T* __restrict__ y, int B, int Tn, int C) {
  const int groups = C / 8;
  const long long total = (long long)B * Tn * groups;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const int g = (int)(i % groups);
    const long long bt = i / groups;
    const int t = (int)(bt % Tn);
    const int b = (int)(bt / Tn);
    const int ch0 = g * 8;
    // window[k] = input of token t-K+1+k (gated: b*x, rounded like the
    // reference's model-dtype product)
    float win[K][8];
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const int tt = t - (K - 1) + k;
      if (tt >= 0) {
        const T* row = in + ((long long)b * Tn + tt) * in_row;
        if (GATED) {
          float bb[8], xx[8];
          ld8(row + ch0, bb);
          ld8(row + 2 * C + ch0, xx);
#pragma unroll
          for (int j = 0; j < 8; ++j) win[k][j] = to_f(from_f<T>(bb[j] * xx[j]));
        } else {
          ld8(row + ch0, win[k]);
        }
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j)
          win[k][j] = tail_in ? to_f(tail_in[b * tail_bs + (long long)(ch0 + j) * (K - 1) + (K - 1 + tt)]) : 0.f;
      }
    }
    float out[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float acc = 0.f;
#pragma unroll
      for (int k = 0; k < K; ++k) acc += to_f(w[(ch0 + j) * K + k]) * win[k][j];
      if (GATED) {
        if (bias) acc += to_f(bias[ch0 + j]);
        out[j] = acc;
      } else {
        out[j] = acc / (1.f + __expf(-acc));
      }
    }
    T* yr = y + ((long long)b * Tn + t) * C + ch0;
    if (GATED) {
      float cc[8];
      ld8(in + ((long long)b * Tn + t) * in_row + C + ch0, cc);
#pragma unroll
      for (int j = 0; j < 8; ++j) yr[j] = from_f<T>(cc[j] * to_f(from_f<T>(out[j])));
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) yr[j] = from_f<T>(out[j]);
    }
    if (tail_out && t == Tn - 1) {
      // new tail = the last K-1 inputs of [tail | sequence]: window[1..K-1]
#pragma unroll
      for (int k = 1; k < K; ++k)
#pragma unroll
        for (int j = 0; j < 8; ++j) tail_out[((long long)b * C + ch0 + j) * (K - 1) + (k - 1)] = from_f<T>(win[k][j]);
    }
  }
}

template <typename T, bool GATED>
static int launch_conv(const void* in, int in_row, const void* w, const void* bias, const void* tail_in, long long tbs,
                       void* tail_out, void* y, int B, int Tn, int C, int K, cudaStream_t st) {
  const long long total = (long long)B * Tn * (C / 8);
  long long blocks = (total + 255) / 256;
  if (blocks > 148 * 32) blocks = 148 * 32;
  if (blocks < 1) blocks = 1;
#define L(KK)                                                                                                      \
  causal_conv_kernel<T, GATED, KK><<<(unsigned)blocks, 256, 0, st>>>((const T*)in, in_row, (const T*)w, (const T*)bias, \
                                                                     (const T*)tail_in, tbs, (T*)tail_out, (T*)y, B, Tn, C)
  switch (K) {
    case 2: L(2); break;
    case 3: L(3); break;
    case 4: L(4); break;
    default: return set_error(CEVK_E_SHAPE, "conv kernel size %d unsupported (2..4)", K);
  }
#undef L
  return check_launch("causal_conv_kernel");
}

}  // namespace cevk

using namespace cevk;

extern "C" {

int cevk_short_conv(const void* bcx, const void* conv_w, const void* bias, const void* tail_in, int64_t tail_batch_stride,
                    void* tail_out, void* y, int32_t B, int32_t T, int32_t d, int32_t K, int32_t dtype, void* stream) {
  if (!bcx || !conv_w || !y) return set_error(CEVK_E_SHAPE, "short_conv: null pointer");
  if (d % 8) return set_error(CEVK_E_SHAPE, "short_conv: d %d not a multiple of 8", d);
  if (B <= 0 || T <= 0) return CEVK_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == CEVK_BF16)
    return launch_conv<__nv_bfloat16, true>(bcx, 3 * d, conv_w, bias, tail_in, tail_batch_stride, tail_out, y, B, T, d, K, st);
  if (dtype == CEVK_F32)
    return launch_conv<float, true>(bcx, 3 * d, conv_w, bias, tail_in, tail_batch_stride, tail_out, y, B, T, d, K, st);
  return set_error(CEVK_E_UNSUPPORTED, "short_conv: dtype %d", dtype);
}

int cevk_gdn_conv(const void* mixed, int32_t mixed_row_stride, const void* conv_w, const void* tail_in,
                  int64_t tail_batch_stride, void* tail_out, void* out, int32_t B, int32_t T, int32_t C, int32_t K,
                  int32_t dtype, void* stream) {
  if (!mixed || !conv_w || !out) return set_error(CEVK_E_SHAPE, "gdn_conv: null pointer");
  if (C % 8 || mixed_row_stride % 8 || mixed_row_stride < C)
    return set_error(CEVK_E_SHAPE, "gdn_conv: C %d / row stride %d", C, mixed_row_stride);
  if (B <= 0 || T <= 0) return CEVK_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == CEVK_BF16)
    return launch_conv<__nv_bfloat16, false>(mixed, mixed_row_stride, conv_w, nullptr, tail_in, tail_batch_stride, tail_out, out, B, T, C, K, st);
  if (dtype == CEVK_F32)
    return launch_conv<float, false>(mixed, mixed_row_stride, conv_w, nullptr, tail_in, tail_batch_stride, tail_out, out, B, T, C, K, st);
  return set_error(CEVK_E_UNSUPPORTED, "gdn_conv: dtype %d", dtype);
}

}  // extern "C"
