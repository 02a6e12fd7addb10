// Per-head RMSNorm + (partial) half-split RoPE at explicit positions, with
// Q written densely and K/V written straight into their arena rows: one
// pass over the projection output replaces the reference's q_norm / k_norm,
// Rotary::apply, the head transposes and the K/V concatenation
// (qwen3.rs:190-200, qwen35.rs:529-541, lfm2.rs:147-156).
//
// bf16 with aligned rows (qk_norm_rope_rows_kernel): one warp per token, a
// head row over D/8 lanes with 16-byte accesses.  Otherwise one block per
// token (cos/sin computed once per token), one warp per head row.  For
// head_dim 64 / 128 / 256 (qk_norm_rope_vec_kernel) a lane holds
// D/32 consecutive elements and takes the rotation partner (d +- rot/2) from
// another lane by shuffle; other shapes go through a shared-memory row so
// the partner can live in any lane.  HBM-bound: each element is read once
// and written once.
#include <cmath>
#include <type_traits>

#include "common.cuh"

namespace cevk {

// 1f32 / (theta^(2i/rot) as f32) for i < rot/2, the power in f64 on the
// host (qwen3.rs:109-112): the same for every token, passed by value.
struct InvFreq {
  float v[256];
};

template <typename T>
__global__ void __launch_bounds__(256) qk_norm_rope_kernel(
    const T* __restrict__ qkv, int row_stride, int q_head_stride, int k_col, int v_col, const T* __restrict__ qw,
    const T* __restrict__ kw, float eps, int plus_one, const int32_t* __restrict__ pos, const InvFreq inv, int rot,
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
    const float ang = p * inv.v[i];
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

// E consecutive elements per lane (E = head_dim / 32), one vector access.
template <typename T, int E>
__device__ __forceinline__ void load_row(const T* __restrict__ p, float* x) {
  constexpr int BYTES = E * (int)sizeof(T);
  static_assert(BYTES == 2 || BYTES % 4 == 0, "vector width");
  if constexpr (BYTES == 2) {
    x[0] = to_f(*p);
  } else if constexpr (BYTES <= 16) {
    using V = typename std::conditional<BYTES == 4, uint32_t, typename std::conditional<BYTES == 8, uint2, uint4>::type>::type;
    V v = *reinterpret_cast<const V*>(p);
    const T* e = reinterpret_cast<const T*>(&v);
#pragma unroll
    for (int i = 0; i < E; ++i) x[i] = to_f(e[i]);
  } else {
#pragma unroll
    for (int c = 0; c < BYTES / 16; ++c) {
      uint4 v = reinterpret_cast<const uint4*>(p)[c];
      const T* e = reinterpret_cast<const T*>(&v);
#pragma unroll
      for (int i = 0; i < 16 / (int)sizeof(T); ++i) x[c * (16 / (int)sizeof(T)) + i] = to_f(e[i]);
    }
  }
}
template <typename T, int E>
__device__ __forceinline__ void store_row(T* __restrict__ p, const float* y) {
  constexpr int BYTES = E * (int)sizeof(T);
  if constexpr (BYTES == 2) {
    *p = from_f<T>(y[0]);
  } else if constexpr (BYTES <= 16) {
    using V = typename std::conditional<BYTES == 4, uint32_t, typename std::conditional<BYTES == 8, uint2, uint4>::type>::type;
    V v;
    T* e = reinterpret_cast<T*>(&v);
#pragma unroll
    for (int i = 0; i < E; ++i) e[i] = from_f<T>(y[i]);
    *reinterpret_cast<V*>(p) = v;
  } else {
#pragma unroll
    for (int c = 0; c < BYTES / 16; ++c) {
      uint4 v;
      T* e = reinterpret_cast<T*>(&v);
#pragma unroll
      for (int i = 0; i < 16 / (int)sizeof(T); ++i) e[i] = from_f<T>(y[c * (16 / (int)sizeof(T)) + i]);
      reinterpret_cast<uint4*>(p)[c] = v;
    }
  }
}

// The same computation with each head row held in registers, E = D / 32
// consecutive elements per lane (one vector load / store), and the rotation
// partner (d +- rot/2, in lane +- rot/2/E with the same element slot) taken
// by a warp shuffle: no shared-memory round trip per head, so a warp's head
// rows are independent and their loads overlap.
template <typename T, int E>
__global__ void __launch_bounds__(256) qk_norm_rope_vec_kernel(
    const T* __restrict__ qkv, int row_stride, int q_head_stride, int k_col, int v_col, const T* __restrict__ qw,
    const T* __restrict__ kw, float eps, int plus_one, const int32_t* __restrict__ pos, const InvFreq inv, int rot,
    T* __restrict__ q_out, T* __restrict__ k_arena, T* __restrict__ v_arena, int kv_rs, const int32_t* __restrict__ kv_rows,
    int hq, int hkv) {
  constexpr int D = 32 * E;
  __shared__ float cs[256], sn[256];
  const int half = rot / 2;
  const int t = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float p = (float)pos[t];
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    const float ang = p * inv.v[i];
    cs[i] = cosf(ang);
    sn[i] = sinf(ang);
  }
  __syncthreads();
  const int d0 = lane * E;
  const int hop = half / E;  // lanes between rotation partners
  const int partner = d0 < half ? lane + hop : (d0 < rot ? lane - hop : lane);
  float c[E], s[E];
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const int d = d0 + e;
    const int i = d < half ? d : d - half;
    c[e] = d < rot ? cs[i] : 1.f;
    s[e] = d < rot ? (d < half ? -sn[i] : sn[i]) : 0.f;
  }
  float qwv[E], kwv[E];
  load_row<T, E>(qw + d0, qwv);
  load_row<T, E>(kw + d0, kwv);
  const float add = plus_one ? 1.f : 0.f;
  const size_t kv_row = (size_t)kv_rows[t];
  const int heads = hq + 2 * hkv;
#pragma unroll 2
  for (int h = warp; h < heads; h += 8) {
    const T* src;
    T* dst;
    if (h < hq) {
      src = qkv + (size_t)t * row_stride + (size_t)h * q_head_stride;
      dst = q_out + ((size_t)t * hq + h) * D;
    } else if (h < hq + hkv) {
      src = qkv + (size_t)t * row_stride + k_col + (size_t)(h - hq) * D;
      dst = k_arena + kv_row * kv_rs + (size_t)(h - hq) * D;
    } else {
      src = qkv + (size_t)t * row_stride + v_col + (size_t)(h - hq - hkv) * D;
      dst = v_arena + kv_row * kv_rs + (size_t)(h - hq - hkv) * D;
    }
    float x[E];
    load_row<T, E>(src + d0, x);
    if (h < hq + hkv) {  // warp-uniform
      const float* w = h < hq ? qwv : kwv;
      float ss = 0.f;
#pragma unroll
      for (int e = 0; e < E; ++e) ss += x[e] * x[e];
      const float r = rsqrtf(warp_sum(ss) / D + eps);
      // Like the reference, the normed value is in the model dtype before RoPE.
#pragma unroll
      for (int e = 0; e < E; ++e) x[e] = to_f(from_f<T>(x[e] * r * (w[e] + add)));
      float y[E];
#pragma unroll
      for (int e = 0; e < E; ++e) y[e] = x[e] * c[e] + __shfl_sync(0xffffffffu, x[e], partner) * s[e];
      store_row<T, E>(dst + d0, y);
    } else {
      store_row<T, E>(dst + d0, x);  // V: a plain copy into the arena
    }
  }
}

// bf16, head_dim 64 / 128 / 256 with every row start 16-byte aligned: one
// warp per token, a head row spread over D/8 lanes of eight consecutive
// elements (one 16-byte load / store), 32/(D/8) head rows per warp step.
// Each lane computes the cos / sin of its eight element slots once and
// reuses them for all of the token's heads; the RMS is reduced over the
// row's lanes and the rotation partner (d +- rot/2, in lane +- rot/16 with
// the same slot) comes by shuffle.
template <int D>
__global__ void __launch_bounds__(256, 3) qk_norm_rope_rows_kernel(
    const __nv_bfloat16* __restrict__ qkv, int row_stride, int q_head_stride, int k_col, int v_col,
    const __nv_bfloat16* __restrict__ qw, const __nv_bfloat16* __restrict__ kw, float eps, int plus_one,
    const int32_t* __restrict__ pos, const InvFreq inv, int rot, __nv_bfloat16* __restrict__ q_out,
    __nv_bfloat16* __restrict__ k_arena, __nv_bfloat16* __restrict__ v_arena, int kv_rs,
    const int32_t* __restrict__ kv_rows, int hq, int hkv, int n_tokens) {
  constexpr int L = D / 8;   // lanes per head row
  constexpr int R = 32 / L;  // head rows per warp step
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * 8 + warp;
  if (t >= n_tokens) return;  // warp-uniform
  const int sub = lane / L, d0 = (lane % L) * 8, half = rot / 2;
  const float p = (float)pos[t];
  float c[8], s[8];
  if constexpr (D <= 128) {
    // the warp's lanes each take 1 (D 64) or 2 (D 128) of the token's rot/2
    // frequencies and hand the cos / sin out by shuffles: a lane needs 8
    // of them, and each is needed by every lane pair (d, d + rot/2) of
    // every head row in the warp
    constexpr int NF = D / 64;
    float cf[NF], sf[NF];
#pragma unroll
    for (int k = 0; k < NF; ++k) {
      const int fi = lane + 32 * k;
      cf[k] = 1.f;
      sf[k] = 0.f;
      if (fi < half) sincosf(p * inv.v[fi], &sf[k], &cf[k]);
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int d = d0 + e, f = d < half ? d : d - half;
      float cs = 1.f, sn = 0.f;
#pragma unroll
      for (int k = 0; k < NF; ++k) {
        const float a = __shfl_sync(0xffffffffu, cf[k], f & 31), b = __shfl_sync(0xffffffffu, sf[k], f & 31);
        if ((f >> 5) == k) {
          cs = a;
          sn = b;
        }
      }
      c[e] = d < rot ? cs : 1.f;
      s[e] = d < rot ? (d < half ? -sn : sn) : 0.f;
    }
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int d = d0 + e;
      c[e] = 1.f;
      s[e] = 0.f;
      if (d < rot) {
        float sn, cs;
        sincosf(p * inv.v[d < half ? d : d - half], &sn, &cs);
        c[e] = cs;
        s[e] = d < half ? -sn : sn;
      }
    }
  }
  const int partner = d0 < half ? lane + half / 8 : (d0 < rot ? lane - half / 8 : lane);
  const float add = plus_one ? 1.f : 0.f;
  const size_t kv_row = (size_t)kv_rows[t];
  const __nv_bfloat16* row = qkv + (size_t)t * row_stride;
  const int heads = hq + 2 * hkv;
  // U steps' loads go out back to back before any of them is used, so a
  // warp keeps U 16-byte loads in flight
  constexpr int U = 6;
  auto src_of = [&](int h) -> const __nv_bfloat16* {
    return h < hq ? row + (size_t)h * q_head_stride
                  : (h < hq + hkv ? row + k_col + (size_t)(h - hq) * D : row + v_col + (size_t)(h - hq - hkv) * D);
  };
  auto dst_of = [&](int h) -> __nv_bfloat16* {
    return h < hq ? q_out + ((size_t)t * hq + h) * D
                  : (h < hq + hkv ? k_arena + kv_row * kv_rs + (size_t)(h - hq) * D
                                  : v_arena + kv_row * kv_rs + (size_t)(h - hq - hkv) * D);
  };
  for (int h0 = 0; h0 < heads; h0 += R * U) {
    uint4 raw[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int h = h0 + u * R + sub;
      raw[u] = h < heads ? *reinterpret_cast<const uint4*>(src_of(h) + d0) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int h = h0 + u * R + sub;
      const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&raw[u]);
      float x[8], ss = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        x[i] = __bfloat162float(e[i]);
        ss += x[i] * x[i];
      }
#pragma unroll
      for (int o = L / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      const float r = rsqrtf(ss / D + eps);
      float wv[8];  // the norm weight (L1-resident, shared by every token)
      load_row<__nv_bfloat16, 8>((h < hq ? qw : kw) + d0, wv);
      float y[8];
      // Like the reference, the normed value is in the model dtype before RoPE.
#pragma unroll
      for (int i = 0; i < 8; ++i) y[i] = to_f(from_f<__nv_bfloat16>(x[i] * r * (wv[i] + add)));
#pragma unroll
      for (int i = 0; i < 8; ++i) y[i] = y[i] * c[i] + __shfl_sync(0xffffffffu, y[i], partner) * s[i];
      if (h < heads) {
        if (h < hq + hkv) {
          store_row<__nv_bfloat16, 8>(dst_of(h) + d0, y);
        } else {
          *reinterpret_cast<uint4*>(dst_of(h) + d0) = raw[u];  // V: a plain copy
        }
      }
    }
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
  if (rotary_dim / 2 > 256) return set_error(CEVK_E_SHAPE, "qk_norm_rope: rotary_dim %d above 512", rotary_dim);
  if (n_tokens <= 0) return CEVK_OK;
  InvFreq inv{};
  for (int i = 0; i < rotary_dim / 2; ++i)
    inv.v[i] = 1.0f / (float)std::pow(theta, (double)(2 * i) / (double)rotary_dim);
  const unsigned blocks = (unsigned)n_tokens;
  const size_t smem = (rotary_dim + 8 * head_dim) * sizeof(float);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // Vector path: head_dim 64 / 128 / 256, rotation partners in lanes with
  // the same element slot, every row start aligned to the vector width.
  const int E = head_dim / 32, es = dtype == CEVK_BF16 ? 2 : 4;
  const bool vec = (head_dim == 64 || head_dim == 128 || head_dim == 256) && (rotary_dim / 2) % E == 0 &&
                   row_stride % E == 0 && q_head_stride % E == 0 && k_col % E == 0 && v_col % E == 0 &&
                   kv_row_stride % E == 0 &&
                   (((uintptr_t)qkv | (uintptr_t)q_out | (uintptr_t)k_arena | (uintptr_t)v_arena |
                     (uintptr_t)q_norm_w | (uintptr_t)k_norm_w) % (E * es)) == 0;
  // bf16 rows on 16-byte boundaries, rotation halves in whole 8-element slots
  const bool rows8 = dtype == CEVK_BF16 && (head_dim == 64 || head_dim == 128 || head_dim == 256) &&
                     (rotary_dim / 2) % 8 == 0 && row_stride % 8 == 0 && q_head_stride % 8 == 0 && k_col % 8 == 0 &&
                     v_col % 8 == 0 && kv_row_stride % 8 == 0 &&
                     (((uintptr_t)qkv | (uintptr_t)q_out | (uintptr_t)k_arena | (uintptr_t)v_arena |
                       (uintptr_t)q_norm_w | (uintptr_t)k_norm_w) % 16) == 0;
  if (rows8) {
    const unsigned grid = (unsigned)((n_tokens + 7) / 8);
#define CEVK_ROPE_ROWS(DD)                                                                                              \
  qk_norm_rope_rows_kernel<DD><<<grid, 256, 0, st>>>(                                                                  \
      (const __nv_bfloat16*)qkv, row_stride, q_head_stride, k_col, v_col, (const __nv_bfloat16*)q_norm_w,              \
      (const __nv_bfloat16*)k_norm_w, eps, norm_plus_one, pos, inv, rotary_dim, (__nv_bfloat16*)q_out,                \
      (__nv_bfloat16*)k_arena, (__nv_bfloat16*)v_arena, kv_row_stride, kv_rows, hq, hkv, n_tokens)
    if (head_dim == 64) CEVK_ROPE_ROWS(64);
    else if (head_dim == 128) CEVK_ROPE_ROWS(128);
    else CEVK_ROPE_ROWS(256);
#undef CEVK_ROPE_ROWS
    return check_launch("qk_norm_rope_rows_kernel");
  }
  if (vec && (dtype == CEVK_BF16 || dtype == CEVK_F32)) {
#define CEVK_ROPE_VEC(TT, EE)                                                                                          \
  qk_norm_rope_vec_kernel<TT, EE><<<blocks, 256, 0, st>>>(                                                             \
      (const TT*)qkv, row_stride, q_head_stride, k_col, v_col, (const TT*)q_norm_w, (const TT*)k_norm_w, eps,          \
      norm_plus_one, pos, inv, rotary_dim, (TT*)q_out, (TT*)k_arena, (TT*)v_arena, kv_row_stride, kv_rows, hq, hkv)
    if (dtype == CEVK_BF16) {
      if (E == 2) CEVK_ROPE_VEC(__nv_bfloat16, 2);
      else if (E == 4) CEVK_ROPE_VEC(__nv_bfloat16, 4);
      else CEVK_ROPE_VEC(__nv_bfloat16, 8);
    } else {
      if (E == 2) CEVK_ROPE_VEC(float, 2);
      else if (E == 4) CEVK_ROPE_VEC(float, 4);
      else CEVK_ROPE_VEC(float, 8);
    }
#undef CEVK_ROPE_VEC
    return check_launch("qk_norm_rope_vec_kernel");
  }
  if (dtype == CEVK_BF16) {
    qk_norm_rope_kernel<__nv_bfloat16><<<blocks, 256, smem, st>>>(
        (const __nv_bfloat16*)qkv, row_stride, q_head_stride, k_col, v_col, (const __nv_bfloat16*)q_norm_w,
        (const __nv_bfloat16*)k_norm_w, eps, norm_plus_one, pos, inv, rotary_dim, (__nv_bfloat16*)q_out,
        (__nv_bfloat16*)k_arena, (__nv_bfloat16*)v_arena, kv_row_stride, kv_rows, hq, hkv, head_dim);
  } else if (dtype == CEVK_F32) {
    qk_norm_rope_kernel<float><<<blocks, 256, smem, st>>>(
        (const float*)qkv, row_stride, q_head_stride, k_col, v_col, (const float*)q_norm_w, (const float*)k_norm_w, eps,
        norm_plus_one, pos, inv, rotary_dim, (float*)q_out, (float*)k_arena, (float*)v_arena, kv_row_stride, kv_rows,
        hq, hkv, head_dim);
  } else {
    return set_error(CEVK_E_UNSUPPORTED, "qk_norm_rope: dtype %d", dtype);
  }
  return check_launch("qk_norm_rope_kernel");
}
