// Gated DeltaNet chunked prefill on tensor cores (bf16 models): the same
// chunked delta rule as gdn.cu (qwen35.rs:301-368), split into a
// chunk-parallel phase and the sequential state scan, with every matrix
// product on the tensor cores as a bf16 three-term split (mma.sync m16n8k16,
// f32 accumulate; x = hi + lo with hi = bf16(x), lo = bf16(x - hi), three
// products hi*hi + hi*lo + lo*hi): about 16 significant bits per operand
// instead of plain bf16's 8, because the reference runs the delta rule in
// f32, the state carries every chunk's error forward, and a bf16 model
// amplifies small output differences layer by layer.  These kernels are
// bound by the mma.sync issue rate, so the split's MMA count is the cost: a
// TF32 split at K = 8 (about 22 bits) needed twice the instructions and
// measured 1.35x slower for both kernels together.
//
// gdn_prep_kernel -- one CTA per (chunk of 64 tokens, value head, row):
//   q, k <- l2norm (q * dk^-1/2); beta = sigmoid(b); g = -exp(A_log) *
//   softplus(a + dt_bias); cum = cumsum(g) over the chunk;
//   A = strict_lower(beta_i k_i.k_j e^(cum_i - cum_j)), T = (I + A)^-1 by
//   recursive block inversion; intra = lower(q_i.k_j e^(cum_i - cum_j));
//   W = T (k beta e^cum), U = T (v beta), q' = q e^cum, k' = k e^(last - cum).
//   All of it to the workspace: W, q', k' and intra as split bf16 planes
//   (hi, lo) in their f32-sized slots, U and e^last in f32.
// gdn_scan_kernel -- one CTA per (value head, 32 value columns, row), over
//   the chunks in order, state slice S (dk x 32) in registers of its
//   update warps, with a split bf16 copy in shared memory for the products:
//   v_new = U - W S;  out = q' S + intra v_new;  S = e^last S + k'^T v_new.
// The raw output goes to the workspace's core array; gdn.cu's gated-norm
// kernel finishes y.
#include "common.cuh"

namespace cevk {

namespace gtc {

constexpr int C = 64;   // chunk length (qwen35.rs:302)
constexpr int VS = 32;  // value columns per scan CTA

// An m16n8 accumulator whose three split products run as independent chains
// (hi*hi, hi*lo, lo*hi), summed when read.
struct Acc {
  float d[4], c[4], e[4];
  __device__ __forceinline__ void zero() {
#pragma unroll
    for (int i = 0; i < 4; ++i) d[i] = c[i] = e[i] = 0.f;
  }
  __device__ __forceinline__ float get(int i) const { return d[i] + (c[i] + e[i]); }
};
// Fragments of m16n8k16 (lane = 4 * gid + tig), two bf16 per register,
// lower k first; D as for every m16n8 shape:
//   A: a0 (gid, 2tig..+1), a1 (gid+8, 2tig..+1), a2 (gid, 2tig+8..+9), a3 (gid+8, 2tig+8..+9)
//   B: b0 (k = 2tig..+1, n = gid), b1 (k = 2tig+8..+9, n = gid)
//   D: d0 (gid, 2tig), d1 (gid, 2tig+1), d2 (gid+8, 2tig), d3 (gid+8, 2tig+1)
struct FragH {
  uint32_t hi[4], lo[4];
};
__device__ __forceinline__ void split_bf16(float x0, float x1, uint32_t& hi, uint32_t& lo) {
  hi = pack_bf16x2(x0, x1);
  lo = pack_bf16x2(x0 - __uint_as_float(hi << 16), x1 - __uint_as_float(hi & 0xffff0000u));
}
__device__ __forceinline__ void mma_bf16(float* d, const uint32_t* a, const uint32_t* b) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}
// The three products into one register set (the prep kernel's accumulators).
__device__ __forceinline__ void mma16(float* d, const FragH& a, const FragH& b) {
  mma_bf16(d, a.hi, b.hi);
  mma_bf16(d, a.hi, b.lo);
  mma_bf16(d, a.lo, b.hi);
}
// A (16 x 16) from row-major M at (r0, k0).
__device__ __forceinline__ FragH frag_a16(const float* M, int ld, int r0, int k0, int gid, int tig) {
  FragH f;
  const float* p0 = M + (r0 + gid) * ld + k0 + 2 * tig;
  const float* p1 = p0 + 8 * ld;
  const float2 v0 = *reinterpret_cast<const float2*>(p0), v1 = *reinterpret_cast<const float2*>(p1);
  const float2 v2 = *reinterpret_cast<const float2*>(p0 + 8), v3 = *reinterpret_cast<const float2*>(p1 + 8);
  split_bf16(v0.x, v0.y, f.hi[0], f.lo[0]);
  split_bf16(v1.x, v1.y, f.hi[1], f.lo[1]);
  split_bf16(v2.x, v2.y, f.hi[2], f.lo[2]);
  split_bf16(v3.x, v3.y, f.hi[3], f.lo[3]);
  return f;
}
// B (16 x 8) with B(k, n) = M[k][n] (row-major [K][N]).
__device__ __forceinline__ FragH frag_b16(const float* M, int ld, int k0, int n0, int gid, int tig) {
  FragH f;
  const float* p = M + (k0 + 2 * tig) * ld + n0 + gid;
  split_bf16(p[0], p[ld], f.hi[0], f.lo[0]);
  split_bf16(p[8 * ld], p[9 * ld], f.hi[1], f.lo[1]);
  return f;
}

// ---------------------------------------------------------------------------
// ldmatrix: four 8 x 8 b16 matrices, row addresses from lanes 8i .. 8i + 7.
__device__ __forceinline__ void ldm_x4(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldm_x4_t(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
// A split-bf16 operand tile in shared memory: planes hi, lo of [rows][ld].
struct Planes {
  uint32_t base;  // shared address of the hi plane
  int ld;         // elements per row (a multiple of 8)
  int plane;      // bytes between the hi and the lo plane
};
// A (16 x 16) at (r0, k0) of a row-major plane: a0..a3 of m16n8k16.
__device__ __forceinline__ FragH lda16(const Planes& P, int r0, int k0, int lane) {
  const int row = r0 + (lane & 7) + ((lane >> 3) & 1) * 8, col = k0 + (lane >> 4) * 8;
  const uint32_t addr = P.base + (uint32_t)(row * P.ld + col) * 2;
  FragH f;
  ldm_x4(addr, f.hi);
  ldm_x4(addr + P.plane, f.lo);
  return f;
}
// A (16 x 16) = the transpose of a row-major plane stored [K][M]: A(m, k) =
// P[k][m], rows m0 .., k0 ...
__device__ __forceinline__ FragH lda16_t(const Planes& P, int m0, int k0, int lane) {
  const int row = k0 + (lane & 7) + (lane >> 4) * 8, col = m0 + ((lane >> 3) & 1) * 8;
  const uint32_t addr = P.base + (uint32_t)(row * P.ld + col) * 2;
  FragH f;
  ldm_x4_t(addr, f.hi);
  ldm_x4_t(addr + P.plane, f.lo);
  return f;
}
// B for two n-blocks (k 16 x n 16) of a plane stored [K][N]: b0, b1 of
// n0 .. n0 + 7 in hi[0..1] / lo[0..1], of n0 + 8 .. in hi[2..3] / lo[2..3].
__device__ __forceinline__ FragH ldb16x2(const Planes& P, int k0, int n0, int lane) {
  const int row = k0 + (lane & 7) + ((lane >> 3) & 1) * 8, col = n0 + (lane >> 4) * 8;
  const uint32_t addr = P.base + (uint32_t)(row * P.ld + col) * 2;
  FragH f;
  ldm_x4_t(addr, f.hi);
  ldm_x4_t(addr + P.plane, f.lo);
  return f;
}
// hi*hi + hi*lo + lo*hi of A with the n-block (0 or 1) of a two-block B.
__device__ __forceinline__ void mma16b(Acc& acc, const FragH& a, const FragH& b, int nb) {
  mma_bf16(acc.d, a.hi, b.hi + 2 * nb);
  mma_bf16(acc.c, a.hi, b.lo + 2 * nb);
  mma_bf16(acc.e, a.lo, b.hi + 2 * nb);
}

// B for two n-blocks (k 16 x n 16) of a plane stored [N][K] (B = P^T):
// B(k, n) = P[n][k], n-blocks n0 .. n0 + 7 and n0 + 8 .. n0 + 15.
__device__ __forceinline__ FragH ldb16x2_nt(const Planes& P, int n0, int k0, int lane) {
  const int row = n0 + (lane & 7) + (lane >> 4) * 8, col = k0 + ((lane >> 3) & 1) * 8;
  const uint32_t addr = P.base + (uint32_t)(row * P.ld + col) * 2;
  FragH f;
  ldm_x4(addr, f.hi);
  ldm_x4(addr + P.plane, f.lo);
  return f;
}
// The three products of A with n-block nb of a two-block B into one
// register set.
__device__ __forceinline__ void mma16n(float* d, const FragH& a, const FragH& b, int nb) {
  mma_bf16(d, a.hi, b.hi + 2 * nb);
  mma_bf16(d, a.hi, b.lo + 2 * nb);
  mma_bf16(d, a.lo, b.hi + 2 * nb);
}
// A (16 x 16) from f32 row-major M at (r0, k0) with column scale: A(r, k) =
// M[r][k] * s[k].
__device__ __forceinline__ FragH frag_a16s(const float* M, int ld, int r0, int k0, int gid, int tig, const float* s) {
  FragH f;
  const int k = k0 + 2 * tig;
  const float* p0 = M + (r0 + gid) * ld + k;
  const float* p1 = p0 + 8 * ld;
  const float s0 = s[k], s1 = s[k + 1], s8 = s[k + 8], s9 = s[k + 9];
  split_bf16(p0[0] * s0, p0[1] * s1, f.hi[0], f.lo[0]);
  split_bf16(p1[0] * s0, p1[1] * s1, f.hi[1], f.lo[1]);
  split_bf16(p0[8] * s8, p0[9] * s9, f.hi[2], f.lo[2]);
  split_bf16(p1[8] * s8, p1[9] * s9, f.hi[3], f.lo[3]);
  return f;
}

__device__ __forceinline__ void cp_async16(float* dst, const float* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
}

struct Params {
  const __nv_bfloat16* conv;  // [B, T, Cc]: q (nk dk) | k (nk dk) | v (nv dv)
  int Cc;
  const __nv_bfloat16* ab;  // per token: b (nv) | a (nv)
  int ab_rs;
  const float* a_log;
  const float* dt_bias;
  const float* s_in;
  long long s_bs;
  float* s_out;
  float* core;  // [B, T, nv, dv]
  // per (row, chunk, head): W, q', k' [C][dk]; U [C][dv]; intra [C][C]; e^last
  float *w, *qp, *kp, *u, *intra, *elast;
  int B, T, nk, nv, dk, dv, n_chunks;
};

__host__ __device__ inline size_t chunk_index(const Params& p, int b, int ch, int h) {
  return ((size_t)b * p.n_chunks + ch) * p.nv + h;
}

// ---------------------------------------------------------------------------
// 107.8 KB of shared memory (dk = dv = 128): two CTAs per SM.  v reuses the
// q buffer once q' is written.
template <int DK, int DV>
__global__ void __launch_bounds__(128, 2) gdn_prep_kernel(Params p) {
  static_assert(DK == DV, "v is staged in the q buffer");
  constexpr int LK = DK + 8, AP = C + 4;
  constexpr int NL = C * (DK / 8) / 128;  // 16-byte loads per thread per matrix
  extern __shared__ __align__(16) float sm[];
  // q (then v) and k as split bf16 planes [2][C][LK] (hi, lo), each in the
  // bytes of an f32 [C][LK] tile; every product fragment is an ldmatrix.
  uint16_t* sQh = reinterpret_cast<uint16_t*>(sm);
  uint16_t* sKh = sQh + 2 * C * LK;
  float* sA = sm + 2 * C * LK;  // [C][AP]  A (strict lower)
  float* sT = sA + C * AP;    // [C][AP]  T = (I + A)^-1
  float* sG = sT + C * AP;    // cum
  float* sB = sG + C;         // beta
  float* sSw = sB + C;        // beta e^cum
  float* sEq = sSw + C;       // e^cum
  float* sEk = sEq + C;       // e^(last - cum)
  float* sX = sEk + C;        // [32][36] products of the block inverse
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, gid = lane >> 2, tig = lane & 3;
  const int ch = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int kh = h / (p.nv / p.nk);  // key head shared by nv/nk value heads (qwen35.rs:436-441)
  const int t0 = ch * C;
  const int key_dim = p.nk * DK;
  const size_t ci = chunk_index(p, b, ch, h);
  const Planes pQ{smem_u32(sQh), LK, C * LK * 2};
  const Planes pK{smem_u32(sKh), LK, C * LK * 2};
  auto store_split8 = [&](uint16_t* P, int r, int c8, const float* f, float sc) {
    uint4 hv, lv;
    split_bf16(f[0] * sc, f[1] * sc, hv.x, lv.x);
    split_bf16(f[2] * sc, f[3] * sc, hv.y, lv.y);
    split_bf16(f[4] * sc, f[5] * sc, hv.z, lv.z);
    split_bf16(f[6] * sc, f[7] * sc, hv.w, lv.w);
    *reinterpret_cast<uint4*>(P + r * LK + c8) = hv;
    *reinterpret_cast<uint4*>(P + C * LK + r * LK + c8) = lv;
  };

  // ---- all q, k, v loads in flight at once (bf16), zero past T ----
  uint4 qv[NL], kv[NL], vv[NL];
#pragma unroll
  for (int u = 0; u < NL; ++u) {
    const int i = tid + u * 128, r = i / (DK / 8), c8 = (i % (DK / 8)) * 8;
    qv[u] = kv[u] = vv[u] = make_uint4(0, 0, 0, 0);
    if (t0 + r < p.T) {
      const __nv_bfloat16* row = p.conv + ((size_t)b * p.T + t0 + r) * p.Cc;
      qv[u] = *reinterpret_cast<const uint4*>(row + kh * DK + c8);
      kv[u] = *reinterpret_cast<const uint4*>(row + key_dim + kh * DK + c8);
      vv[u] = *reinterpret_cast<const uint4*>(row + 2 * key_dim + h * DV + c8);
    }
  }
  if (tid < C) {
    const int t = t0 + tid;
    float beta = 0.f, g = 0.f;
    if (t < p.T) {
      const __nv_bfloat16* row = p.ab + ((size_t)b * p.T + t) * p.ab_rs;
      beta = 1.f / (1.f + expf(-__bfloat162float(row[h])));
      const float x = __bfloat162float(row[p.nv + h]) + p.dt_bias[h];
      // softplus(x) = max(x, 0) + ln(1 + e^{-|x|}) (qwen35.rs:243-248)
      g = (fmaxf(x, 0.f) + logf(1.f + expf(-fabsf(x)))) * -expf(p.a_log[h]);
    }
    sB[tid] = beta;
    sG[tid] = g;
  }
  auto unpack8 = [](const uint4& u, float* f) {
    const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
    for (int x = 0; x < 8; ++x) f[x] = __bfloat162float(e[x]);
  };
  // l2norm of the q and k rows from registers (q also * dk^-1/2): the DK/8
  // threads of a row are consecutive lanes, reduced with shuffles.
  const float qscale = rsqrtf((float)DK);
#pragma unroll
  for (int u = 0; u < NL; ++u) {
    const int i = tid + u * 128, r = i / (DK / 8), c8 = (i % (DK / 8)) * 8;
    float fq[8], fk[8];
    unpack8(qv[u], fq);
    unpack8(kv[u], fk);
    float sq = 0.f, sk = 0.f;
#pragma unroll
    for (int x = 0; x < 8; ++x) {
      sq += fq[x] * fq[x];
      sk += fk[x] * fk[x];
    }
#pragma unroll
    for (int o = DK / 16; o > 0; o >>= 1) {
      sq += __shfl_xor_sync(0xffffffffu, sq, o);
      sk += __shfl_xor_sync(0xffffffffu, sk, o);
    }
    store_split8(sQh, r, c8, fq, (1.f / sqrtf(sq + 1e-6f)) * qscale);
    store_split8(sKh, r, c8, fk, 1.f / sqrtf(sk + 1e-6f));
  }
  __syncthreads();
  // ---- cumsum of g over the chunk: warp 0, two tokens a lane, lane scan ----
  if (warp == 0) {
    const float g0 = sG[2 * lane], g1 = sG[2 * lane + 1];
    float sc = g0 + g1;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float t = __shfl_up_sync(0xffffffffu, sc, o);
      if (lane >= o) sc += t;
    }
    const float before = sc - (g0 + g1);
    sG[2 * lane] = before + g0;
    sG[2 * lane + 1] = before + g0 + g1;
  }
  __syncthreads();
  if (tid < C) {
    const float last = sG[C - 1];
    sSw[tid] = sB[tid] * expf(sG[tid]);
    sEq[tid] = expf(sG[tid]);
    sEk[tid] = expf(last - sG[tid]);
    if (tid == 0) p.elast[ci] = expf(last);
  }

  // ---- A = strict_lower(beta_i k_i.k_j dec), intra = lower(q_i.k_j dec) ----
  {
    const int r0 = warp * 16;
    float ak[8][4], aq[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) ak[n][e] = aq[n][e] = 0.f;
#pragma unroll 1
    for (int k0 = 0; k0 < DK; k0 += 16) {
      const FragH fk = lda16(pK, r0, k0, lane);
      const FragH fq = lda16(pQ, r0, k0, lane);
#pragma unroll
      for (int n = 0; n < 8; n += 2) {
        if (n * 8 > r0 + 15) continue;  // strictly above the diagonal block
        const FragH fb = ldb16x2_nt(pK, n * 8, k0, lane);  // k^T for column blocks n, n + 1
        mma16n(ak[n], fk, fb, 0);
        mma16n(aq[n], fq, fb, 0);
        if ((n + 1) * 8 <= r0 + 15) {
          mma16n(ak[n + 1], fk, fb, 1);
          mma16n(aq[n + 1], fq, fb, 1);
        }
      }
    }
    // intra as two bf16 planes (hi, lo) in its f32-sized slot
    uint16_t* intra_h = reinterpret_cast<uint16_t*>(p.intra + ci * C * C);
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int hlf = 0; hlf < 2; ++hlf) {
        const int i = r0 + gid + hlf * 8, j = n * 8 + 2 * tig;
        float a[2], q[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          a[e] = q[e] = 0.f;
          if (j + e <= i) {
            const float dec = expf(sG[i] - sG[j + e]);
            q[e] = aq[n][2 * hlf + e] * dec;
            if (j + e < i) a[e] = sB[i] * ak[n][2 * hlf + e] * dec;
          }
          sA[i * AP + j + e] = a[e];
        }
        uint32_t qh, ql;
        split_bf16(q[0], q[1], qh, ql);
        *reinterpret_cast<uint32_t*>(intra_h + i * C + j) = qh;
        *reinterpret_cast<uint32_t*>(intra_h + C * C + i * C + j) = ql;
      }
  }
  __syncthreads();
  // q' = q e^cum, k' = k e^(last - cum)
  {
    // as two bf16 planes (hi, lo) each, in their f32-sized slots
    uint2* qp = reinterpret_cast<uint2*>(p.qp + ci * C * DK);
    uint2* kp = reinterpret_cast<uint2*>(p.kp + ci * C * DK);
    for (int i = tid; i < C * DK / 4; i += 128) {
      const int r = (i * 4) / DK, d = (i * 4) % DK;
      // q, k = hi + lo from the planes
      auto rd4 = [&](const uint16_t* P) {
        const uint2 hv = *reinterpret_cast<const uint2*>(P + r * LK + d);
        const uint2 lv = *reinterpret_cast<const uint2*>(P + C * LK + r * LK + d);
        return make_float4(__uint_as_float(hv.x << 16) + __uint_as_float(lv.x << 16),
                           __uint_as_float(hv.x & 0xffff0000u) + __uint_as_float(lv.x & 0xffff0000u),
                           __uint_as_float(hv.y << 16) + __uint_as_float(lv.y << 16),
                           __uint_as_float(hv.y & 0xffff0000u) + __uint_as_float(lv.y & 0xffff0000u));
      };
      const float4 q4 = rd4(sQh), k4 = rd4(sKh);
      const float eq = sEq[r], ek = sEk[r];
      uint2 h, l;
      split_bf16(q4.x * eq, q4.y * eq, h.x, l.x);
      split_bf16(q4.z * eq, q4.w * eq, h.y, l.y);
      qp[i] = h;
      qp[C * DK / 4 + i] = l;
      split_bf16(k4.x * ek, k4.y * ek, h.x, l.x);
      split_bf16(k4.z * ek, k4.w * ek, h.y, l.y);
      kp[i] = h;
      kp[C * DK / 4 + i] = l;
    }
  }
  // ---- T = (I + A)^-1 by recursive block inversion, the reference's
  //      scheme (qwen35.rs:266-296): inv(I + [[a, 0], [c, d]]) =
  //      [[ai, 0], [-di c ai, di]].  16 x 16 leaves by forward substitution
  //      (warp w: diagonal block w, two lanes per column), then the two
  //      levels' products on the tensor cores. ----
  {
    const int b0 = warp * 16, c = lane >> 1, half = lane & 1;
    for (int i = 0; i < 16; ++i) {
      float acc = 0.f;
      if (i > c)
        for (int j = c + half; j < i; j += 2) acc += sA[(b0 + i) * AP + b0 + j] * sT[(b0 + j) * AP + b0 + c];
      acc += __shfl_xor_sync(0xffffffffu, acc, 1);
      if (half == 0) sT[(b0 + i) * AP + b0 + c] = i == c ? 1.f : (i > c ? -acc : 0.f);
      __syncwarp();
    }
  }
  __syncthreads();
  // 16 x 16 tile = A (16 x K) * B (K x 16), split bf16, into acc[2][4] (D layout)
  auto mm16 = [&](const float* A, int lda, const float* B, int ldb, int K, float (*acc)[4]) {
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[n][e] = 0.f;
    for (int k0 = 0; k0 < K; k0 += 16) {
      const FragH fa = frag_a16(A, lda, 0, k0, gid, tig);
#pragma unroll
      for (int n = 0; n < 2; ++n) mma16(acc[n], fa, frag_b16(B, ldb, k0, n * 8, gid, tig));
    }
  };
  auto put16 = [&](float* D, int ldd, const float (*acc)[4], float sgn) {
#pragma unroll
    for (int n = 0; n < 2; ++n) {
      *reinterpret_cast<float2*>(D + gid * ldd + n * 8 + 2 * tig) = make_float2(sgn * acc[n][0], sgn * acc[n][1]);
      *reinterpret_cast<float2*>(D + (gid + 8) * ldd + n * 8 + 2 * tig) = make_float2(sgn * acc[n][2], sgn * acc[n][3]);
    }
  };
  constexpr int XP = 36;
  if (warp < 2) {  // level 1: T[b+1, b] = -D_{b+1} (A[b+1, b] D_b), b = 0, 2
    const int r0 = 16 * (2 * warp + 1), c0 = 16 * (2 * warp);
    float acc[2][4];
    mm16(sA + r0 * AP + c0, AP, sT + c0 * AP + c0, AP, 16, acc);
    put16(sX + warp * 16 * XP, XP, acc, 1.f);
    __syncwarp();
    mm16(sT + r0 * AP + r0, AP, sX + warp * 16 * XP, XP, 16, acc);
    put16(sT + r0 * AP + c0, AP, acc, -1.f);
  }
  __syncthreads();
  {  // level 2: X = A[32:, :32] T[:32, :32], then T[32:, :32] = -T[32:, 32:] X (a quadrant per warp)
    const int qr = (warp >> 1) * 16, qc = (warp & 1) * 16;
    float acc[2][4];
    mm16(sA + (32 + qr) * AP, AP, sT + qc, AP, 32, acc);
    put16(sX + qr * XP + qc, XP, acc, 1.f);
    __syncthreads();
    mm16(sT + (32 + qr) * AP + 32, AP, sX + qc, XP, 32, acc);
    put16(sT + (32 + qr) * AP + qc, AP, acc, -1.f);
  }
  __syncthreads();  // T complete; q no longer needed
#pragma unroll
  for (int u = 0; u < NL; ++u) {
    const int i = tid + u * 128, r = i / (DK / 8), c8 = (i % (DK / 8)) * 8;
    // v is exact in bf16: hi = v, lo = 0
    *reinterpret_cast<uint4*>(sQh + r * LK + c8) = vv[u];
    *reinterpret_cast<uint4*>(sQh + C * LK + r * LK + c8) = make_uint4(0, 0, 0, 0);
  }
  __syncthreads();
  // ---- W = T (k beta e^cum), U = T (v beta) (T lower triangular) ----
  {
    const int r0 = warp * 16;
    const int kend = r0 + 16;  // T[i][j] = 0 for j > i
#pragma unroll 1
    for (int part = 0; part < 2 * (DK / 64); ++part) {  // 64 output columns of W, then of U
      const bool is_u = part >= DK / 64;
      const int cb = (part % (DK / 64)) * 64;
      // W = T diag(beta e^cum) k, U = T diag(beta) v: the row scales of k / v
      // go onto T's columns so that k and v feed the MMAs by ldmatrix
      const Planes& pB = is_u ? pQ : pK;
      const float* scale = is_u ? sB : sSw;
      float* dst = (is_u ? p.u : p.w) + ci * C * DK;
      float acc[8][4];
#pragma unroll
      for (int n = 0; n < 8; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[n][e] = 0.f;
#pragma unroll 1
      for (int k0 = 0; k0 < kend; k0 += 16) {
        const FragH fa = frag_a16s(sT, AP, r0, k0, gid, tig, scale);
#pragma unroll
        for (int n = 0; n < 8; n += 2) {
          const FragH fb = ldb16x2(pB, k0, cb + n * 8, lane);
          mma16n(acc[n], fa, fb, 0);
          mma16n(acc[n + 1], fa, fb, 1);
        }
      }
      if (is_u) {  // U stays f32: the scan subtracts W S from it at full precision
#pragma unroll
        for (int n = 0; n < 8; ++n) {
          const int col = cb + n * 8 + 2 * tig;
          *reinterpret_cast<float2*>(dst + (r0 + gid) * DK + col) = make_float2(acc[n][0], acc[n][1]);
          *reinterpret_cast<float2*>(dst + (r0 + gid + 8) * DK + col) = make_float2(acc[n][2], acc[n][3]);
        }
      } else {  // W as two bf16 planes (hi, lo)
        uint16_t* wh = reinterpret_cast<uint16_t*>(dst);
#pragma unroll
        for (int n = 0; n < 8; ++n) {
          const int col = cb + n * 8 + 2 * tig;
          uint32_t h, l;
          split_bf16(acc[n][0], acc[n][1], h, l);
          *reinterpret_cast<uint32_t*>(wh + (r0 + gid) * DK + col) = h;
          *reinterpret_cast<uint32_t*>(wh + C * DK + (r0 + gid) * DK + col) = l;
          split_bf16(acc[n][2], acc[n][3], h, l);
          *reinterpret_cast<uint32_t*>(wh + (r0 + gid + 8) * DK + col) = h;
          *reinterpret_cast<uint32_t*>(wh + C * DK + (r0 + gid + 8) * DK + col) = l;
        }
      }
    }
  }
}

// 16 warps in two groups of 8; within a group warp w covers rows 16 (w & 3)
// .. +16 and value columns 16 (w >> 2) .. +16 of the 64 x 32 chunk block.
//   group 0: W S, then v_new = U - W S, then the state update S = e^last S +
//            k'^T v_new for state rows 16 w .. +16 (w < dk/16), whose f32
//            values it keeps in registers across chunks;
//   group 1: q' S, then out = q' S + intra v_new and its store.
// Operands sit in shared memory as split bf16 planes (W, q', k', intra as
// the prep kernel wrote them; S and v_new split when written) and every
// fragment is one ldmatrix per plane.  U stays f32.
constexpr int SCAN_THREADS = 512;
template <int DK, int DV>
struct ScanSmem {
  static constexpr int LK = DK + 8, LS = VS + 8, LC = C + 8;  // bf16 row pitches
  static constexpr int UP = VS + 8;                           // f32 U row pitch
  static constexpr int S_B = 2 * DK * LS * 2;                 // S hi/lo
  static constexpr int M_B = 2 * C * LK * 2;                  // W, q', one k' buffer
  static constexpr int U_B = C * UP * 4;                      // one U buffer
  static constexpr int V_B = 2 * C * LS * 2;                  // v_new hi/lo
  static constexpr int I_B = 2 * C * LC * 2;                  // one intra buffer
  static constexpr int OFF_S = 0, OFF_W = OFF_S + S_B, OFF_Q = OFF_W + M_B, OFF_K = OFF_Q + M_B;
  static constexpr int OFF_U = OFF_K + 2 * M_B, OFF_V = OFF_U + 2 * U_B, OFF_I = OFF_V + V_B;
  static constexpr int BYTES = OFF_I + 2 * I_B;
  static_assert(BYTES <= 232448, "scan shared memory");
};

template <int DK, int DV>
__global__ void __launch_bounds__(SCAN_THREADS) gdn_scan_kernel(Params p) {
  using L = ScanSmem<DK, DV>;
  static_assert(DK % 16 == 0 && DK / 16 <= 8, "16 state rows per warp of group 0");
  extern __shared__ __align__(16) uint8_t smb[];
  const uint32_t sb = smem_u32(smb);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, gid = lane >> 2, tig = lane & 3;
  const int sl = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int c0 = sl * VS;
  const int grp = warp >> 3, w8 = warp & 7;
  const int r0 = (w8 & 3) * 16, n0 = (w8 >> 2) * 16;  // rows / columns of v_new and out
  const Planes pS{sb + L::OFF_S, L::LS, DK * L::LS * 2};
  const Planes pW{sb + L::OFF_W, L::LK, C * L::LK * 2};
  const Planes pQ{sb + L::OFF_Q, L::LK, C * L::LK * 2};
  const Planes pV{sb + L::OFF_V, L::LS, C * L::LS * 2};
  uint16_t* sSh = reinterpret_cast<uint16_t*>(smb + L::OFF_S);
  uint16_t* sVh = reinterpret_cast<uint16_t*>(smb + L::OFF_V);
  const bool upd = grp == 0 && warp < DK / 16;
  const int d0 = warp * 16;  // state rows of an updating warp
  // An updating warp's 16 state rows x 32 columns, f32, in m16n8 layout.
  float st[4][4];
  auto put_s = [&]() {  // the split copy of this warp's state rows
#pragma unroll
    for (int n = 0; n < 4; ++n)
#pragma unroll
      for (int hl = 0; hl < 2; ++hl) {
        uint32_t hi, lo;
        split_bf16(st[n][2 * hl], st[n][2 * hl + 1], hi, lo);
        const int o = (d0 + gid + hl * 8) * L::LS + n * 8 + 2 * tig;
        *reinterpret_cast<uint32_t*>(sSh + o) = hi;
        *reinterpret_cast<uint32_t*>(sSh + DK * L::LS + o) = lo;
      }
  };
  if (upd) {
#pragma unroll
    for (int n = 0; n < 4; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int d = d0 + gid + (e >> 1) * 8, c = n * 8 + 2 * tig + (e & 1);
        st[n][e] = p.s_in ? p.s_in[b * p.s_bs + ((size_t)h * DK + d) * DV + c0 + c] : 0.f;
      }
    put_s();
  }
  // 16-byte copies of a [2][rows][cols] bf16 slot into planes of pitch ld.
  auto load_planes = [&](uint8_t* dst, const float* src, int rows, int cols, int ld) {
    const uint8_t* s8 = reinterpret_cast<const uint8_t*>(src);
    const int per_row = cols / 8, n = 2 * rows * per_row;
    for (int i = tid; i < n; i += SCAN_THREADS) {
      const int pl = i / (rows * per_row), rem = i % (rows * per_row), r = rem / per_row, c8 = rem % per_row;
      cp_async16(reinterpret_cast<float*>(dst + ((pl * rows + r) * ld + c8 * 8) * 2),
                 reinterpret_cast<const float*>(s8 + ((size_t)(pl * rows + r) * cols + c8 * 8) * 2));
    }
  };
  auto load_wq = [&](size_t cj) {
    load_planes(smb + L::OFF_W, p.w + cj * C * DK, C, DK, L::LK);
    load_planes(smb + L::OFF_Q, p.qp + cj * C * DK, C, DK, L::LK);
  };
  auto load_rest = [&](size_t cj, int buf) {
    load_planes(smb + L::OFF_K + buf * L::M_B, p.kp + cj * C * DK, C, DK, L::LK);
    load_planes(smb + L::OFF_I + buf * L::I_B, p.intra + cj * C * C, C, C, L::LC);
    const float* u = p.u + cj * C * DV + c0;
    float* du = reinterpret_cast<float*>(smb + L::OFF_U + buf * L::U_B);
    for (int i = tid; i < C * VS / 4; i += SCAN_THREADS) {
      const int r = (i * 4) / VS, c = (i * 4) % VS;
      cp_async16(du + r * L::UP + c, u + r * DV + c);
    }
  };
  if (p.n_chunks > 0) {
    load_wq(chunk_index(p, b, 0, h));
    load_rest(chunk_index(p, b, 0, h), 0);
  }
  for (int ch = 0; ch < p.n_chunks; ++ch) {
    const size_t ci = chunk_index(p, b, ch, h);
    const int buf = ch & 1;
    const Planes pK{sb + L::OFF_K + buf * L::M_B, L::LK, C * L::LK * 2};
    const Planes pI{sb + L::OFF_I + buf * L::I_B, L::LC, C * L::LC * 2};
    const float* sU = reinterpret_cast<const float*>(smb + L::OFF_U + buf * L::U_B);
    // This chunk's copies (issued during the previous chunk) have landed,
    // the previous chunk is done with the other buffers and the split state
    // is written.
    cp_async_wait_all();
    __syncthreads();
    if (ch + 1 < p.n_chunks) load_rest(chunk_index(p, b, ch + 1, h), buf ^ 1);
    const float el = p.elast[ci];
    // group 0: W S; group 1: q' S (over dk)
    Acc acc2[2];
    acc2[0].zero();
    acc2[1].zero();
    const Planes& pA = grp == 0 ? pW : pQ;
#pragma unroll 2
    for (int k0 = 0; k0 < DK; k0 += 16) {
      const FragH fa = lda16(pA, r0, k0, lane);
      const FragH fs = ldb16x2(pS, k0, n0, lane);
      mma16b(acc2[0], fa, fs, 0);
      mma16b(acc2[1], fa, fs, 1);
    }
    if (grp == 0) {
      // v_new = U - W S, split into its planes (each warp owns its 16 x 16 block)
#pragma unroll
      for (int n = 0; n < 2; ++n)
#pragma unroll
        for (int hl = 0; hl < 2; ++hl) {
          const int i = r0 + gid + hl * 8, j = n0 + n * 8 + 2 * tig;
          const float v0 = sU[i * L::UP + j] - acc2[n].get(2 * hl);
          const float v1 = sU[i * L::UP + j + 1] - acc2[n].get(2 * hl + 1);
          uint32_t hi, lo;
          split_bf16(v0, v1, hi, lo);
          *reinterpret_cast<uint32_t*>(sVh + i * L::LS + j) = hi;
          *reinterpret_cast<uint32_t*>(sVh + C * L::LS + i * L::LS + j) = lo;
        }
    }
    __syncthreads();
    // W and q' are done for this chunk: the next chunk's stream in behind
    // the output and state-update phases.
    if (ch + 1 < p.n_chunks) load_wq(chunk_index(p, b, ch + 1, h));
    if (grp == 1) {
      // out = q' S + intra v_new (intra lower triangular)
#pragma unroll 1
      for (int k0 = 0; k0 < r0 + 16; k0 += 16) {
        const FragH fi = lda16(pI, r0, k0, lane);
        const FragH fv = ldb16x2(pV, k0, n0, lane);
        mma16b(acc2[0], fi, fv, 0);
        mma16b(acc2[1], fi, fv, 1);
      }
#pragma unroll
      for (int n = 0; n < 2; ++n)
#pragma unroll
        for (int hl = 0; hl < 2; ++hl) {
          const int t = ch * C + r0 + gid + hl * 8;
          if (t < p.T)
            *reinterpret_cast<float2*>(p.core + (((size_t)b * p.T + t) * p.nv + h) * DV + c0 + n0 + n * 8 + 2 * tig) =
                make_float2(acc2[n].get(2 * hl), acc2[n].get(2 * hl + 1));
        }
    } else if (upd) {
      // S = e^last S + k'^T v_new on this warp's rows
      Acc acc[4];
#pragma unroll
      for (int n = 0; n < 4; ++n) {
        acc[n].zero();
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[n].d[e] = st[n][e] * el;
      }
#pragma unroll 2
      for (int k0 = 0; k0 < C; k0 += 16) {
        const FragH fk = lda16_t(pK, d0, k0, lane);
        const FragH fv0 = ldb16x2(pV, k0, 0, lane), fv1 = ldb16x2(pV, k0, 16, lane);
        mma16b(acc[0], fk, fv0, 0);
        mma16b(acc[1], fk, fv0, 1);
        mma16b(acc[2], fk, fv1, 0);
        mma16b(acc[3], fk, fv1, 1);
      }
#pragma unroll
      for (int n = 0; n < 4; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) st[n][e] = acc[n].get(e);
      // the split copy for the next chunk's W S / q' S: nobody reads S
      // before the next chunk's barrier
      put_s();
    }
  }
  if (upd && p.s_out)
#pragma unroll
    for (int n = 0; n < 4; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int d = d0 + gid + (e >> 1) * 8, c = n * 8 + 2 * tig + (e & 1);
        p.s_out[(size_t)b * p.nv * DK * DV + ((size_t)h * DK + d) * DV + c0 + c] = st[n][e];
      }
}

template <int DK, int DV>
size_t prep_smem() {
  return sizeof(float) * (2 * C * (DK + 8) + 2 * C * (C + 4) + 5 * C + 32 * 36);
}
template <int DK, int DV>
size_t scan_smem() {
  return ScanSmem<DK, DV>::BYTES;
}

template <int DK, int DV>
int launch(const Params& p, cudaStream_t st) {
  int rc;
  if ((rc = opt_in_smem((const void*)gdn_prep_kernel<DK, DV>, (int)prep_smem<DK, DV>(), "gdn_prep_kernel")) ||
      (rc = opt_in_smem((const void*)gdn_scan_kernel<DK, DV>, (int)scan_smem<DK, DV>(), "gdn_scan_kernel")))
    return rc;
  gdn_prep_kernel<DK, DV><<<dim3(p.n_chunks, p.nv, p.B), 128, prep_smem<DK, DV>(), st>>>(p);
  rc = check_launch("gdn_prep_kernel");
  if (rc) return rc;
  gdn_scan_kernel<DK, DV><<<dim3(DV / VS, p.nv, p.B), SCAN_THREADS, scan_smem<DK, DV>(), st>>>(p);
  return check_launch("gdn_scan_kernel");
}

}  // namespace gtc

// Workspace floats of the tensor-core path beyond the core output.
size_t gdn_tc_extra_floats(int B, int T, int nv, int dk, int dv) {
  const size_t nc = (size_t)(T + gtc::C - 1) / gtc::C;
  return (size_t)B * nc * nv * ((size_t)gtc::C * (3 * dk + dv + gtc::C) + 1);
}

bool gdn_tc_supported(int dk, int dv) { return (dk == 128 && dv == 128) || (dk == 64 && dv == 64); }

int gdn_tc_run(const void* conv_out, int C_, const void* ab, int ab_rs, const float* a_log, const float* dt_bias,
               const float* s_in, long long s_bs, float* s_out, float* workspace, int B, int T, int nk, int nv, int dk,
               int dv, cudaStream_t st) {
  gtc::Params p;
  p.conv = reinterpret_cast<const __nv_bfloat16*>(conv_out);
  p.Cc = C_;
  p.ab = reinterpret_cast<const __nv_bfloat16*>(ab);
  p.ab_rs = ab_rs;
  p.a_log = a_log;
  p.dt_bias = dt_bias;
  p.s_in = s_in;
  p.s_bs = s_bs;
  p.s_out = s_out;
  p.B = B;
  p.T = T;
  p.nk = nk;
  p.nv = nv;
  p.dk = dk;
  p.dv = dv;
  p.n_chunks = (T + gtc::C - 1) / gtc::C;
  const size_t per = (size_t)B * p.n_chunks * nv * gtc::C;
  p.core = workspace;
  float* x = workspace + (size_t)B * T * nv * dv;
  p.w = x;
  x += per * dk;
  p.qp = x;
  x += per * dk;
  p.kp = x;
  x += per * dk;
  p.u = x;
  x += per * dv;
  p.intra = x;
  x += per * gtc::C;
  p.elast = x;
  if (dk == 128) return gtc::launch<128, 128>(p, st);
  return gtc::launch<64, 64>(p, st);
}

}  // namespace cevk
