// Causal depthwise convolutions that continue from a cached tail of K-1
// inputs: the LFM2 gated short conv (y = C * conv_K(B * X), lfm2.rs:199-219)
// and the Gated DeltaNet q/k/v conv with SiLU (qwen35.rs:419-431), both
// replacing depthwise_conv1d's K shifted full-tensor passes plus the
// narrow / mul / cat copies (decoder.rs:137-151) with one HBM pass.
//
// One thread per (row, run of R tokens, 8 channels): every input row of the
// run and its K-1 earlier tokens is loaded once, all loads in flight before
// the first use (16 or 32 bytes per row and thread, coalesced across the
// channel groups of a warp); weights are loaded once per thread; each output
// row is one 16- or 32-byte store.  The tail is read in place (batch stride
// 0 broadcasts one prefix state to every row) and the new tail is written by
// the thread whose run holds the last token.
#include "common.cuh"

namespace cevk {

// f32 -> 8 consecutive elements (16-byte aligned for bf16, 32 for f32).
__device__ __forceinline__ void st8(__nv_bfloat16* p, const float* f) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  *reinterpret_cast<uint4*>(p) = u;
}
__device__ __forceinline__ void st8(float* p, const float* f) {
  reinterpret_cast<float4*>(p)[0] = make_float4(f[0], f[1], f[2], f[3]);
  reinterpret_cast<float4*>(p)[1] = make_float4(f[4], f[5], f[6], f[7]);
}

constexpr int CONV_RUN = 4;  // tokens per thread

// 8 elements in their storage form (one 16-byte vector for bf16, two for f32).
template <typename T>
struct Raw8 {
  uint4 a, b;
};
template <typename T>
__device__ __forceinline__ Raw8<T> ldraw(const T* p) {
  Raw8<T> r;
  r.a = *reinterpret_cast<const uint4*>(p);
  if (sizeof(T) == 4) r.b = *reinterpret_cast<const uint4*>(p + 16 / sizeof(T));
  return r;
}
__device__ __forceinline__ void unraw(const Raw8<__nv_bfloat16>& r, float* f) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&r.a);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 v = __bfloat1622float2(h[i]);
    f[2 * i] = v.x;
    f[2 * i + 1] = v.y;
  }
}
__device__ __forceinline__ void unraw(const Raw8<float>& r, float* f) {
  f[0] = __uint_as_float(r.a.x); f[1] = __uint_as_float(r.a.y); f[2] = __uint_as_float(r.a.z); f[3] = __uint_as_float(r.a.w);
  f[4] = __uint_as_float(r.b.x); f[5] = __uint_as_float(r.b.y); f[6] = __uint_as_float(r.b.z); f[7] = __uint_as_float(r.b.w);
}

// GATED: y = c * (bias + sum_k w_k * (b*x)[t-K+1+k]); else y = silu(sum_k w_k * x[t-K+1+k]).
// Every global load of the run is issued before any is used: token indices
// are clamped into the row so that no load sits behind a branch, and rows
// outside the sequence are replaced afterwards (tail state or zero).
template <typename T, bool GATED, int K>
__global__ void __launch_bounds__(256, 2) causal_conv_kernel(const T* __restrict__ in, int in_row, const T* __restrict__ w,
                                                             const T* __restrict__ bias, const T* __restrict__ tail_in,
                                                             long long tail_bs, T* __restrict__ tail_out,
                                                             T* __restrict__ y, int B, int Tn, int C) {
  constexpr int R = CONV_RUN, NW = R + K - 1;
  const int groups = C / 8, runs = (Tn + R - 1) / R;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;  // < 2^31 (checked on the host)
  if (i >= B * runs * groups) return;
  const int g = i % groups, br = i / groups;
  const int run = br % runs, b = br / runs;
  const int ch0 = g * 8, t0 = run * R;
  const T* rows = in + (long long)b * Tn * in_row;
  Raw8<T> rx[NW], rb[GATED ? NW : 1], rc[GATED ? R : 1];
#pragma unroll
  for (int r = 0; r < NW; ++r) {
    const int tt = min(max(t0 - (K - 1) + r, 0), Tn - 1);
    const T* row = rows + (long long)tt * in_row;
    if (GATED) {
      rb[r] = ldraw(row + ch0);
      rx[r] = ldraw(row + 2 * C + ch0);
    } else {
      rx[r] = ldraw(row + ch0);
    }
  }
  if (GATED)
#pragma unroll
    for (int r = 0; r < R; ++r) rc[r] = ldraw(rows + (long long)min(t0 + r, Tn - 1) * in_row + C + ch0);
  // the group's 8 x K weights are contiguous: K vector loads of 8
  float wk[8 * K], bs[8];
#pragma unroll
  for (int k = 0; k < K; ++k) unraw(ldraw(w + ch0 * K + 8 * k), wk + 8 * k);
  if (GATED && bias) unraw(ldraw(bias + ch0), bs);
  else
#pragma unroll
    for (int j = 0; j < 8; ++j) bs[j] = 0.f;
  // window row r = input of token t0 - (K-1) + r (gated: b*x, rounded like
  // the reference's model-dtype product)
  float win[NW][8];
#pragma unroll
  for (int r = 0; r < NW; ++r) {
    const int tt = t0 - (K - 1) + r;
    unraw(rx[r], win[r]);
    if (GATED) {
      float bb[8];
      unraw(rb[r], bb);
#pragma unroll
      for (int j = 0; j < 8; ++j) win[r][j] = to_f(from_f<T>(bb[j] * win[r][j]));
    }
    if (tt < 0) {
#pragma unroll
      for (int j = 0; j < 8; ++j)
        win[r][j] = tail_in ? to_f(tail_in[b * tail_bs + (long long)(ch0 + j) * (K - 1) + (K - 1 + tt)]) : 0.f;
    }
  }
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int t = t0 + r;
    if (t >= Tn) break;
    float out[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float acc = 0.f;
#pragma unroll
      for (int k = 0; k < K; ++k) acc += wk[j * K + k] * win[r + k][j];
      out[j] = GATED ? acc + bs[j] : acc / (1.f + __expf(-acc));
    }
    if (GATED) {
      float cc[8];
      unraw(rc[r], cc);
#pragma unroll
      for (int j = 0; j < 8; ++j) out[j] = cc[j] * to_f(from_f<T>(out[j]));
    }
    st8(y + ((long long)b * Tn + t) * C + ch0, out);
  }
  if (tail_out && t0 <= Tn - 1 && Tn - 1 < t0 + R) {
    // new tail = the last K-1 inputs of [tail | sequence]: tokens Tn-K+1 .. Tn-1
#pragma unroll
    for (int k = 0; k < K - 1; ++k) {
      const int r = Tn - t0 + k;  // window row of token Tn-K+1+k
#pragma unroll
      for (int rr = 0; rr < NW; ++rr)
        if (rr == r)
#pragma unroll
          for (int j = 0; j < 8; ++j) tail_out[((long long)b * C + ch0 + j) * (K - 1) + k] = from_f<T>(win[rr][j]);
    }
  }
}

template <typename T, bool GATED>
static int launch_conv(const void* in, int in_row, const void* w, const void* bias, const void* tail_in, long long tbs,
                       void* tail_out, void* y, int B, int Tn, int C, int K, cudaStream_t st) {
  if (((uintptr_t)in | (uintptr_t)y | (uintptr_t)w | (uintptr_t)bias) & (8 * sizeof(T) - 1))
    return set_error(CEVK_E_SHAPE, "conv: input, output, weights and bias must be %d-byte aligned",
                     (int)(8 * sizeof(T)));
  const long long total = (long long)B * ((Tn + CONV_RUN - 1) / CONV_RUN) * (C / 8);
  if (total >= (1ll << 31) - 256) return set_error(CEVK_E_SHAPE, "conv: %lld thread jobs", total);
  const unsigned blocks = (unsigned)((total + 255) / 256);
#define L(KK)                                                                                                 \
  causal_conv_kernel<T, GATED, KK><<<blocks, 256, 0, st>>>((const T*)in, in_row, (const T*)w, (const T*)bias, \
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
