// Gated DeltaNet chunked prefill on the sm_100 tensor cores (tcgen05 UMMA,
// TMEM accumulators) for bf16 models with dk = dv = 128 -- the chunked
// delta rule of qwen35.rs:301-368 with its prologue, in two kernels:
//
// gdn_umma_prep_kernel, one CTA per (64-token chunk, value head, row),
// chunk-parallel:
//   q, k <- l2norm (q * dk^-1/2); beta = sigmoid(b); g = -exp(A_log) *
//   softplus(a + dt_bias); cum = cumsum(g) over the chunk;
//   [k; q] k^T on the tensor cores (one M = 128 product): A =
//   strict_lower(beta_i k_i.k_j e^(cum_i - cum_j)) and intra =
//   lower(q_i.k_j e^(cum_i - cum_j));
//   T = (I + A)^-1 by the reference's recursive block inversion
//   (qwen35.rs:266-296) on 16 x 16 leaves;
//   W^T = k^T (T diag(beta e^cum))^T and U^T = v^T (T diag(beta))^T on the
//   tensor cores (M = dk = 128);
//   q' = q e^cum, k' = k e^(last - cum), e^last.
// gdn_umma_scan_kernel, one CTA per (64 value columns, value head, row),
// sequential over the chunks, the state slice S (dk x 64) in registers:
//   D1 = [q'; W] S                       (M = 128: q' S rows, W S rows)
//   v_new = U - W S                      (from D1's W S rows)
//   D2 = k'^T v_new,  D1 += [intra; 0] v_new
//   out = q' S + intra v_new (D1's first 64 rows);  S = e^last S + D2.
//
// Precision: every product is a bf16 three-term split (x = hi + lo, hi =
// bf16(x), lo = bf16(x - hi); hi*hi + hi*lo + lo*hi accumulated in f32 in
// TMEM), about 16 significant bits per operand, because the reference runs
// the delta rule in f32 and the state carries every chunk's error forward;
// v is exact in bf16, so U takes two terms.
//
// The prep kernel writes each chunk's scan operands to the workspace as
// finished shared-memory images (the 128-byte-swizzled layouts the UMMA
// descriptors read), so that the scan brings them in with plain bulk copies:
//   AWQ  [q'^T hi][W^T hi][q'^T lo][W^T lo]  4 x (128 d-rows x 64 tokens)
//   AK   [k' hi d0-63][k' hi d64-127][k' lo ..][..]  4 x (64 tokens x 64 d)
//   AI   [intra hi][intra lo]               2 x (64 x 64)
//   UT   U^T f32 [dv][64]
// 144 KB per (chunk, head, row): the size of the f32 workspace the host
// sizes with cevk_gdn_workspace_size().
#include <algorithm>
#include <deque>
#include <mutex>

#include "common.cuh"

namespace cevk {

namespace gum {

constexpr int C = 64;    // chunk length (qwen35.rs:302)
constexpr int DK = 128;  // key head dim
constexpr int DV = 128;  // value head dim
constexpr int NS = 64;   // value columns per scan CTA
constexpr int T128 = 128 * 128;  // bytes of a 128-row x 64-column bf16 tile
constexpr int T64 = 64 * 128;    // bytes of a 64-row tile
constexpr uint32_t AWQ_B = 4 * T128, AK_B = 4 * T64, AI_B = 2 * T64, UT_B = DV * C * 4;
constexpr size_t REC_B = (size_t)AWQ_B + AK_B + AI_B + UT_B;  // 147456
constexpr long long WAIT = 1ll << 30;
constexpr int PIECE = 21;  // chunks per piece of a long single-row call

// Byte offset of (row r, column c < 64) in a 128-byte-swizzled tile of
// 64-element bf16 rows: 16-byte chunk c/8 of row r sits at chunk (c/8) ^ (r%8).
__device__ __forceinline__ uint32_t sw(int r, int c) {
  return (uint32_t)(r * 128 + ((((c >> 3) ^ (r & 7)) & 7) << 4) + ((c & 7) << 1));
}

__device__ __forceinline__ void split2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
  hi = pack_bf16x2(x0, x1);
  lo = pack_bf16x2(x0 - __uint_as_float(hi << 16), x1 - __uint_as_float(hi & 0xffff0000u));
}
// 8 floats -> one 16-byte chunk of hi and one of lo.
__device__ __forceinline__ void split8(const float* f, uint4& h, uint4& l) {
  split2(f[0], f[1], h.x, l.x);
  split2(f[2], f[3], h.y, l.y);
  split2(f[4], f[5], h.z, l.z);
  split2(f[6], f[7], h.w, l.w);
}
__device__ __forceinline__ float bf_lo(uint32_t u) { return __uint_as_float(u << 16); }
// Programmatic dependent launch: the scan is launched while the prep still
// runs (its CTAs take SMs as prep CTAs leave); griddepcontrol.wait holds a
// thread until the prep grid has completed and its writes are visible, and
// is a no-op when the kernel was launched without the attribute.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ float bf_hi(uint32_t u) { return __uint_as_float(u & 0xffff0000u); }

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
  float* core;       // [B, T, nv, dv]
  uint8_t* rec;      // per (row, chunk, head): REC_B bytes
  float* elast;      // per (row, chunk, head)
  int B, T, nk, nv, n_chunks;
  int c0, c1;        // the chunks [c0, c1) this launch runs (prep: c0 + blockIdx.x)
};

__host__ __device__ inline size_t chunk_index(const Params& p, int b, int ch, int h) {
  return ((size_t)b * p.n_chunks + ch) * p.nv + h;
}

// Legacy-fragment helpers for the small block products of the inverse
// (16 x 16 tiles, mma.sync m16n8k16, bf16 three-term split).
__device__ __forceinline__ void mma_bf16(float* d, const uint32_t* a, const uint32_t* b) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}
// D (16 x 16 at acc[n][4], n = 8-column block) += A (16 x K) B (K x 16), f32
// row-major operands in shared memory, split on the fly.
__device__ __forceinline__ void mm16(const float* A, int lda, const float* B, int ldb, int K, float (*acc)[4],
                                     int gid, int tig) {
#pragma unroll
  for (int n = 0; n < 2; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[n][e] = 0.f;
  for (int k0 = 0; k0 < K; k0 += 16) {
    uint32_t ah[4], al[4];
    const float* p0 = A + gid * lda + k0 + 2 * tig;
    const float* p1 = p0 + 8 * lda;
    split2(p0[0], p0[1], ah[0], al[0]);
    split2(p1[0], p1[1], ah[1], al[1]);
    split2(p0[8], p0[9], ah[2], al[2]);
    split2(p1[8], p1[9], ah[3], al[3]);
#pragma unroll
    for (int n = 0; n < 2; ++n) {
      uint32_t bh[2], bl[2];
      const float* q = B + (k0 + 2 * tig) * ldb + n * 8 + gid;
      split2(q[0], q[ldb], bh[0], bl[0]);
      split2(q[8 * ldb], q[9 * ldb], bh[1], bl[1]);
      mma_bf16(acc[n], ah, bh);
      mma_bf16(acc[n], ah, bl);
      mma_bf16(acc[n], al, bh);
    }
  }
}
__device__ __forceinline__ void put16(float* D, int ldd, const float (*acc)[4], float sgn, int gid, int tig) {
#pragma unroll
  for (int n = 0; n < 2; ++n) {
    *reinterpret_cast<float2*>(D + gid * ldd + n * 8 + 2 * tig) = make_float2(sgn * acc[n][0], sgn * acc[n][1]);
    *reinterpret_cast<float2*>(D + (gid + 8) * ldd + n * 8 + 2 * tig) = make_float2(sgn * acc[n][2], sgn * acc[n][3]);
  }
}

// ---------------------------------------------------------------------------
// Prep kernel.  256 threads, two CTAs per SM; shared memory (1024-byte
// aligned base), regions reused as the kernel goes:
//   P_KQ  4 x 128-row tiles [blk0 hi][blk1 hi][blk0 lo][blk1 lo]: rows 0-63
//         k, rows 64-127 q; once q' is written, v (exact bf16) takes the q
//         rows of the two hi tiles; after the last products, the staging
//         area of W^T and U^T
//   P_A   f32 A [C][AP], then the T diag(beta e^cum) image (hi, lo)
//   P_T   the intra image staging, then f32 T [C][AP], then the
//         T diag(beta) image (hi, lo)
constexpr int P_KQ = 0;
constexpr int AP = C + 4;                 // f32 pitch of A / T
constexpr int XP = 36;
constexpr int P_A = P_KQ + 4 * T128;      // f32 [C][AP] (17 KB, 1024-byte multiple)
constexpr int P_T = P_A + C * AP * 4;     // f32 [C][AP]
constexpr int P_X = P_T + C * AP * 4;     // f32 [32][XP]
constexpr int P_VEC = P_X + 32 * XP * 4;  // cum, beta, beta e^cum, e^cum, e^(last - cum): 5 x C f32
constexpr int P_BAR = P_VEC + 5 * C * 4;  // 2 mbarriers
constexpr int P_MISC = P_BAR + 16;        // TMEM base, abort flag
constexpr int P_SMEM = P_MISC + 16;
constexpr int PREP_THREADS = 256;
static_assert((C * AP * 4) % 1024 == 0 && C * AP * 4 >= 2 * T64, "T images in the A / T areas");
constexpr int P_TMEM_COLS = 256;  // D1 [0, 64), W^T [64, 128), U^T [128, 192)

__global__ void __launch_bounds__(PREP_THREADS, 2) gdn_umma_prep_kernel(Params p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t sb = smem_u32(smem);
  if (sb & 1023u) {  // the swizzled tiles need a 1024-byte aligned base
    if (threadIdx.x == 0) atomicExch(&g_device_error, kErrWaitTimeout);
    return;
  }
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int ch = p.c0 + blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  griddep_launch_dependents();  // the scan may be scheduled (it waits for this grid before reading its output)
  const int kh = h / (p.nv / p.nk);  // key head read by this value head (qwen35.rs:436-441)
  const int t0 = ch * C;
  const int key_dim = p.nk * DK;
  const size_t ci = chunk_index(p, b, ch, h);
  uint8_t* rec = p.rec + ci * REC_B;
  float* sA = reinterpret_cast<float*>(smem + P_A);
  float* sT = reinterpret_cast<float*>(smem + P_T);
  float* sX = reinterpret_cast<float*>(smem + P_X);
  float* sG = reinterpret_cast<float*>(smem + P_VEC);  // cum
  float* sB = sG + C;                                  // beta
  float* sSw = sB + C;                                 // beta e^cum
  float* sEq = sSw + C;                                // e^cum
  float* sEk = sEq + C;                                // e^(last - cum)
  const uint32_t bar_p1 = sb + P_BAR, bar_p2 = sb + P_BAR + 8;
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(smem + P_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + P_MISC + 4);

  if (tid == 0) {
    mbar_init(bar_p1, 1);
    mbar_init(bar_p2, 1);
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32((const void*)tmem_slot), P_TMEM_COLS);
    tmem_relinquish();
  }

  // ---- loads: q, k, v of the chunk (16 threads per row of 128), zero past T ----
  constexpr int NL = C * (DK / 8) / PREP_THREADS;  // 4
  uint4 qv[NL], kv[NL];
#pragma unroll
  for (int u = 0; u < NL; ++u) {
    const int i = tid + u * PREP_THREADS, r = i >> 4, c8 = (i & 15) * 8;
    qv[u] = kv[u] = make_uint4(0, 0, 0, 0);
    if (t0 + r < p.T) {
      const __nv_bfloat16* row = p.conv + ((size_t)b * p.T + t0 + r) * p.Cc;
      qv[u] = *reinterpret_cast<const uint4*>(row + kh * DK + c8);
      kv[u] = *reinterpret_cast<const uint4*>(row + key_dim + kh * DK + c8);
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
  // l2norm of the q and k rows (q also * dk^-1/2), reduced over the row's 16
  // lanes; split planes into the [k; q] tiles.
  {
    const float qscale = rsqrtf((float)DK);
#pragma unroll
    for (int u = 0; u < NL; ++u) {
      const int i = tid + u * PREP_THREADS, r = i >> 4, c8 = (i & 15) * 8;
      const __nv_bfloat16* qe = reinterpret_cast<const __nv_bfloat16*>(&qv[u]);
      const __nv_bfloat16* ke = reinterpret_cast<const __nv_bfloat16*>(&kv[u]);
      float fq[8], fk[8], sq = 0.f, sk = 0.f;
#pragma unroll
      for (int x = 0; x < 8; ++x) {
        fq[x] = __bfloat162float(qe[x]);
        fk[x] = __bfloat162float(ke[x]);
        sq += fq[x] * fq[x];
        sk += fk[x] * fk[x];
      }
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) {
        sq += __shfl_xor_sync(0xffffffffu, sq, o);
        sk += __shfl_xor_sync(0xffffffffu, sk, o);
      }
      const float rq = (1.f / sqrtf(sq + 1e-6f)) * qscale, rk = 1.f / sqrtf(sk + 1e-6f);
#pragma unroll
      for (int x = 0; x < 8; ++x) {
        fq[x] *= rq;
        fk[x] *= rk;
      }
      uint4 qh, ql, khh, kl;
      split8(fq, qh, ql);
      split8(fk, khh, kl);
      const int blk = c8 >> 6, cc = c8 & 63;
      *reinterpret_cast<uint4*>(smem + P_KQ + blk * T128 + sw(r, cc)) = khh;
      *reinterpret_cast<uint4*>(smem + P_KQ + (2 + blk) * T128 + sw(r, cc)) = kl;
      *reinterpret_cast<uint4*>(smem + P_KQ + blk * T128 + sw(64 + r, cc)) = qh;
      *reinterpret_cast<uint4*>(smem + P_KQ + (2 + blk) * T128 + sw(64 + r, cc)) = ql;
    }
  }
  __syncthreads();
  // ---- cumsum of g over the chunk (warp 0, two tokens a lane) ----
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
  fence_proxy_async_smem();  // the tiles written above are read by the tensor cores
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (tid < C) {
    const float last = sG[C - 1];
    sSw[tid] = sB[tid] * expf(sG[tid]);
    sEq[tid] = expf(sG[tid]);
    sEk[tid] = expf(last - sG[tid]);
    if (tid == 0) p.elast[ci] = expf(last);
  }

  // ---- [k; q] k^T: M = 128, N = 64, K = dk (three split products) ----
  if (warp == 1 && lane == 0) {
    constexpr uint32_t idesc = umma_idesc_bf16(128, 64, 0, 0);
#pragma unroll
    for (int kk = 0; kk < DK / 16; ++kk) {
      const uint32_t off = (kk >> 2) * T128 + (kk & 3) * 32;
      const uint64_t hi = umma_desc_sw128(sb + P_KQ + off, 16, 1024);
      const uint64_t lo = umma_desc_sw128(sb + P_KQ + 2 * T128 + off, 16, 1024);
      umma_bf16_ss(tmem, hi, hi, idesc, kk > 0 ? 1u : 0u);
      umma_bf16_ss(tmem, hi, lo, idesc, 1u);
      umma_bf16_ss(tmem, lo, hi, idesc, 1u);
    }
    umma_commit(bar_p1);
  }
  __syncthreads();  // e^cum etc. written

  if (warp < 4) {
    // ---- A (rows 0-63) and intra (rows 64-127) from the products ----
    const int r = tid;  // TMEM lane = row of [k; q]
    float v[64];
    const bool ok = __all_sync(0xffffffffu, mbar_wait(bar_p1, 0, abort_flag, WAIT));
    tc_fence_after();
    if (ok) {  // tcgen05.ld is warp-collective
      tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16), v);
      tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + 32, v + 32);
      tmem_wait_ld();
    }
    // decay e^(cum_i - cum_j) <= 1 for j <= i (the exponent is a sum of
    // log-decays, never positive); __expf's error is relative to the value.
    // Every element is computed and then masked (the exponent clamped at 0
    // so that the masked-out ones stay finite): a lane-dependent condition
    // around the exponential would split the warp at every column.
    if (r < C) {
      const int i = r;
      const float ci_ = sG[i], bi = sB[i];
#pragma unroll
      for (int j4 = 0; j4 < C; j4 += 4) {
        float a[4];
#pragma unroll
        for (int x = 0; x < 4; ++x) {
          const float e = __expf(fminf(ci_ - sG[j4 + x], 0.f));
          a[x] = (bi * v[j4 + x]) * (j4 + x < i ? e : 0.f);
        }
        *reinterpret_cast<float4*>(sA + i * AP + j4) = make_float4(a[0], a[1], a[2], a[3]);
      }
    } else {
      // intra rows into the (not yet used) T area, then out coalesced
      const int i = r - C;
      const float ci_ = sG[i];
#pragma unroll
      for (int c8 = 0; c8 < C; c8 += 8) {
        float f[8];
#pragma unroll
        for (int x = 0; x < 8; ++x) {
          const float e = __expf(fminf(ci_ - sG[c8 + x], 0.f));
          f[x] = v[c8 + x] * ((c8 + x) <= i ? e : 0.f);
        }
        uint4 hv, lv;
        split8(f, hv, lv);
        *reinterpret_cast<uint4*>(smem + P_T + sw(i, c8)) = hv;
        *reinterpret_cast<uint4*>(smem + P_T + T64 + sw(i, c8)) = lv;
      }
      named_bar_sync(2, 64);
      const uint4* src = reinterpret_cast<const uint4*>(smem + P_T);
      uint4* dst = reinterpret_cast<uint4*>(rec + AWQ_B + AK_B);
#pragma unroll 4
      for (int e = tid - 64; e < AI_B / 16; e += 64) dst[e] = src[e];
    }
    named_bar_sync(1, 128);
    // ---- T = (I + A)^-1, the reference's recursive block inversion
    //      (qwen35.rs:266-296): inv(I + [[a, 0], [c, d]]) =
    //      [[ai, 0], [-di c ai, di]], with 16 x 16 leaves by forward
    //      substitution (warp w: diagonal block w, two lanes per column) ----
    {
      // lane c < 16 holds column c of the block's inverse in registers:
      // t_i = [i == c] - sum_{j < i} A_ij t_j (t_j = 0 above the diagonal),
      // accumulated column by column (once t_j is final it updates every
      // t_i below it), so the dependent chain is one FMA per row
      const int b0 = warp * 16, c = lane & 15;
      float t[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) t[i] = i == c ? 1.f : 0.f;
#pragma unroll
      for (int j = 0; j < 15; ++j)
#pragma unroll
        for (int i = j + 1; i < 16; ++i) t[i] = fmaf(-sA[(b0 + i) * AP + b0 + j], t[j], t[i]);
      if (lane < 16)
#pragma unroll
        for (int i = 0; i < 16; ++i) sT[(b0 + i) * AP + b0 + c] = t[i];
      // zero the strictly upper 16 x 16 blocks of T
      for (int e = lane; e < 256; e += 32) {
        const int rr = e >> 4, cc = e & 15;
        for (int cb = warp + 1; cb < 4; ++cb) sT[(b0 + rr) * AP + cb * 16 + cc] = 0.f;
      }
    }
    named_bar_sync(1, 128);
    const int gid = lane >> 2, tig = lane & 3;
    if (warp < 2) {  // level 1: T[b+1, b] = -D_{b+1} (A[b+1, b] D_b), b = 0, 2
      const int r0 = 16 * (2 * warp + 1), c0 = 16 * (2 * warp);
      float acc[2][4];
      mm16(sA + r0 * AP + c0, AP, sT + c0 * AP + c0, AP, 16, acc, gid, tig);
      put16(sX + warp * 16 * XP, XP, acc, 1.f, gid, tig);
      __syncwarp();
      mm16(sT + r0 * AP + r0, AP, sX + warp * 16 * XP, XP, 16, acc, gid, tig);
      put16(sT + r0 * AP + c0, AP, acc, -1.f, gid, tig);
    }
    named_bar_sync(1, 128);
    {  // level 2: X = A[32:, :32] T[:32, :32], then T[32:, :32] = -T[32:, 32:] X (a quadrant per warp)
      const int qr = (warp >> 1) * 16, qc = (warp & 1) * 16;
      float acc[2][4];
      mm16(sA + (32 + qr) * AP, AP, sT + qc, AP, 32, acc, gid, tig);
      put16(sX + qr * XP + qc, XP, acc, 1.f, gid, tig);
      named_bar_sync(1, 128);
      mm16(sT + (32 + qr) * AP + 32, AP, sX + qc, XP, 32, acc, gid, tig);
      put16(sT + (32 + qr) * AP + qc, AP, acc, -1.f, gid, tig);
    }
    named_bar_sync(1, 128);
    // ---- B images T diag(beta e^cum) (into the A area) and T diag(beta)
    //      (over T itself): [i][j], split; all of T is read before any of
    //      it is overwritten ----
    {
      uint4 img[4][4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int e = tid + k * 128, i = e >> 3, c8 = (e & 7) * 8;
        float fs[8], fb[8];
#pragma unroll
        for (int x = 0; x < 8; ++x) {
          const float t = sT[i * AP + c8 + x];
          fs[x] = t * sSw[c8 + x];
          fb[x] = t * sB[c8 + x];
        }
        split8(fs, img[k][0], img[k][1]);
        split8(fb, img[k][2], img[k][3]);
      }
      named_bar_sync(1, 128);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int e = tid + k * 128, i = e >> 3, c8 = (e & 7) * 8;
        *reinterpret_cast<uint4*>(smem + P_A + sw(i, c8)) = img[k][0];
        *reinterpret_cast<uint4*>(smem + P_A + T64 + sw(i, c8)) = img[k][1];
        *reinterpret_cast<uint4*>(smem + P_T + sw(i, c8)) = img[k][2];
        *reinterpret_cast<uint4*>(smem + P_T + T64 + sw(i, c8)) = img[k][3];
      }
    }
    fence_proxy_async_smem();
  } else {
    // ---- warps 4-7: q'^T rows (q' = q e^cum) and k' (k e^(last - cum)) ----
    const int u = tid - 128;
    // q'^T image rows d (128) x 8 chunks of 8 tokens: a warp stores 4 rows
    // x 128 bytes, contiguous.  The eight lanes of one row d read tokens t8
    // + x in an order rotated by the lane's t8 group, so that each read hits
    // eight different swizzle chunks (rows t8 + x share their chunk, and
    // hence their banks, for a fixed x); the values are rotated back after.
    const int rot = u & 7;
#pragma unroll 1
    for (int e = u; e < DK * 8; e += 128) {
      const int d = e >> 3, t8 = (e & 7) * 8;
      const uint8_t* th = smem + P_KQ + (d >> 6) * T128;
      const uint8_t* tl = th + 2 * T128;
      float g[8];  // g[x]: token t8 + ((x + rot) & 7)
#pragma unroll
      for (int x = 0; x < 8; ++x) {
        const int xr = (x + rot) & 7;
        const uint32_t o = sw(64 + t8 + xr, d & 63);
        const float q = __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(th + o)) +
                        __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(tl + o));
        g[x] = q * sEq[t8 + xr];
      }
      // f[y] = g[(y - rot) & 7], a barrel rotation with constant indices
      float f[8];
#pragma unroll
      for (int y = 0; y < 8; ++y) f[y] = (rot & 4) ? g[(y + 4) & 7] : g[y];
#pragma unroll
      for (int y = 0; y < 8; ++y) g[y] = (rot & 2) ? f[(y + 6) & 7] : f[y];
#pragma unroll
      for (int y = 0; y < 8; ++y) f[y] = (rot & 1) ? g[(y + 7) & 7] : g[y];
      uint4 hv, lv;
      split8(f, hv, lv);
      *reinterpret_cast<uint4*>(rec + sw(d, t8)) = hv;             // q'^T hi
      *reinterpret_cast<uint4*>(rec + 2 * T128 + sw(d, t8)) = lv;  // q'^T lo
    }
    uint8_t* ak = rec + AWQ_B;
#pragma unroll 1
    for (int e = u; e < C * 2 * 8; e += 128) {  // (64-column block, token, 8-column chunk)
      const int blk = e >> 9, t = (e >> 3) & 63, c8 = (e & 7) * 8;
      const uint4 hv = *reinterpret_cast<const uint4*>(smem + P_KQ + blk * T128 + sw(t, c8));
      const uint4 lv = *reinterpret_cast<const uint4*>(smem + P_KQ + (2 + blk) * T128 + sw(t, c8));
      const float ek = sEk[t];
      float f[8] = {(bf_lo(hv.x) + bf_lo(lv.x)) * ek, (bf_hi(hv.x) + bf_hi(lv.x)) * ek,
                    (bf_lo(hv.y) + bf_lo(lv.y)) * ek, (bf_hi(hv.y) + bf_hi(lv.y)) * ek,
                    (bf_lo(hv.z) + bf_lo(lv.z)) * ek, (bf_hi(hv.z) + bf_hi(lv.z)) * ek,
                    (bf_lo(hv.w) + bf_lo(lv.w)) * ek, (bf_hi(hv.w) + bf_hi(lv.w)) * ek};
      uint4 h2, l2;
      split8(f, h2, l2);
      *reinterpret_cast<uint4*>(ak + blk * T64 + sw(t, c8)) = h2;
      *reinterpret_cast<uint4*>(ak + (2 + blk) * T64 + sw(t, c8)) = l2;
    }
    // q is no longer read (by these warps, and by the [k; q] k^T product,
    // which has completed): v (exact bf16) into the q rows of the two hi
    // tiles, [t][d] per 64-column block (zero past T)
    named_bar_sync(3, 128);
    mbar_wait(bar_p1, 0, abort_flag, WAIT);
#pragma unroll 4
    for (int e = u; e < C * (DV / 8); e += 128) {
      const int t = e >> 4, c8 = (e & 15) * 8;
      uint4 vv = make_uint4(0, 0, 0, 0);
      if (t0 + t < p.T)
        vv = *reinterpret_cast<const uint4*>(p.conv + ((size_t)b * p.T + t0 + t) * p.Cc + 2 * key_dim + h * DV + c8);
      *reinterpret_cast<uint4*>(smem + P_KQ + (c8 >> 6) * T128 + sw(64 + t, c8 & 63)) = vv;
    }
    fence_proxy_async_smem();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  // ---- W^T = k^T Ts^T (three terms) and U^T = v^T Tb^T (two terms):
  //      M = dk = 128 (A = k^T / v^T, MN-major from the [t][d] tiles), N = 64 ----
  if (warp == 1 && lane == 0 && !*abort_flag) {
    constexpr uint32_t idesc = umma_idesc_bf16(128, 64, 1, 0);
#pragma unroll
    for (int s = 0; s < C / 16; ++s) {
      const uint64_t kh = umma_desc_sw128(sb + P_KQ + s * 2048, T128, 1024);
      const uint64_t kl = umma_desc_sw128(sb + P_KQ + 2 * T128 + s * 2048, T128, 1024);
      const uint64_t vd = umma_desc_sw128(sb + P_KQ + 64 * 128 + s * 2048, T128, 1024);  // v in the q rows
      const uint64_t tsh = umma_desc_sw128(sb + P_A + s * 32, 16, 1024);
      const uint64_t tsl = umma_desc_sw128(sb + P_A + T64 + s * 32, 16, 1024);
      const uint64_t tbh = umma_desc_sw128(sb + P_T + s * 32, 16, 1024);
      const uint64_t tbl = umma_desc_sw128(sb + P_T + T64 + s * 32, 16, 1024);
      umma_bf16_ss(tmem + 64, kh, tsh, idesc, s > 0 ? 1u : 0u);
      umma_bf16_ss(tmem + 64, kh, tsl, idesc, 1u);
      umma_bf16_ss(tmem + 64, kl, tsh, idesc, 1u);
      umma_bf16_ss(tmem + 128, vd, tbh, idesc, s > 0 ? 1u : 0u);
      umma_bf16_ss(tmem + 128, vd, tbl, idesc, 1u);
    }
    umma_commit(bar_p2);
  }
  // ---- W^T rows (split) and U^T rows (f32), lane = d: staged in the [k; q]
  //      area (free once these products are done), then out coalesced ----
  uint8_t* stage = smem + P_KQ;  // [W^T hi][W^T lo][U^T f32 [dk][64]]
  if (warp < 4) {
    const int d = tid;
    const bool ok = __all_sync(0xffffffffu, mbar_wait(bar_p2, 0, abort_flag, WAIT));
    tc_fence_after();
    if (ok) {
      float w[64];
      tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + 64, w);
      tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + 96, w + 32);
      tmem_wait_ld();
#pragma unroll
      for (int t8 = 0; t8 < C; t8 += 8) {
        uint4 hv, lv;
        split8(w + t8, hv, lv);
        *reinterpret_cast<uint4*>(stage + sw(d, t8)) = hv;
        *reinterpret_cast<uint4*>(stage + T128 + sw(d, t8)) = lv;
      }
      tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + 128, w);
      tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + 160, w + 32);
      tmem_wait_ld();
      // 16-byte chunk t4 of row d at chunk t4 ^ (d % 16): a warp's stores
      // spread over the banks (the copy-out undoes it)
      float4* ut = reinterpret_cast<float4*>(stage + 2 * T128 + (size_t)d * C * 4);
#pragma unroll
      for (int t4 = 0; t4 < C / 4; ++t4)
        ut[t4 ^ (d & 15)] = make_float4(w[4 * t4], w[4 * t4 + 1], w[4 * t4 + 2], w[4 * t4 + 3]);
    }
  }
  if (warp == 1 && lane == 0) {
    // every UMMA this CTA issued has completed before TMEM is freed
    volatile int never = 0;
    mbar_wait(bar_p2, 0, &never, WAIT);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  {
    const uint4* src = reinterpret_cast<const uint4*>(stage);
    uint4* wdst_h = reinterpret_cast<uint4*>(rec + T128);
    uint4* wdst_l = reinterpret_cast<uint4*>(rec + 3 * T128);
    uint4* udst = reinterpret_cast<uint4*>(rec + AWQ_B + AK_B + AI_B);
#pragma unroll 4
    for (int e = tid; e < T128 / 16; e += PREP_THREADS) {
      wdst_h[e] = src[e];
      wdst_l[e] = src[T128 / 16 + e];
    }
#pragma unroll 4
    for (int e = tid; e < UT_B / 16; e += PREP_THREADS)
      udst[e] = src[2 * T128 / 16 + (e & ~15) + ((e & 15) ^ ((e >> 4) & 15))];
  }
  if (warp == 1) tmem_dealloc(*tmem_slot, P_TMEM_COLS);
}

// ---------------------------------------------------------------------------
// Scan kernel.  320 threads: warp 0 brings each chunk's operand images in by
// bulk copies, warp 1 allocates TMEM and issues the UMMAs, warps 2-9 (two
// per TMEM lane quarter, each on 32 of the 64 columns) compute v_new, the
// state and the output.  D1 alternates between two TMEM buffers by chunk,
// so a chunk's output is read after the next chunk's products have started.
// The chain from one chunk's state to the next is D1's W S rows -> v_new ->
// D2 -> S: D2 commits on its own (s23) ahead of the intra v_new products
// (out), which run while the epilogue updates the state, and the v_new
// warps hold U in registers before D1 completes.
constexpr int S_AWQ = 0;                  // [q'^T hi][W^T hi][q'^T lo][W^T lo], 128 d-rows x 64 tokens each
constexpr int S_AK = S_AWQ + AWQ_B;       // [k' hi d0-63][k' hi d64-127][k' lo ..][..], 64 tokens x 64 d each
constexpr int S_AI = S_AK + AK_B;         // [intra hi][0][intra lo][0]: two 128-row A tiles [intra; 0]
constexpr int S_S = S_AI + 4 * T64;       // S hi, lo: 128 d-rows x 64 columns (MN-major B)
constexpr int S_V = S_S + 2 * T128;       // v_new hi, lo: 64 tokens x 64 columns (MN-major B)
constexpr int S_U = S_V + 2 * T64;        // U^T slice f32 [64 columns][64 tokens]
constexpr int S_BAR = S_U + NS * C * 4;   // 11 mbarriers
constexpr int S_MISC = S_BAR + 96;
constexpr int S_SMEM = S_MISC + 16;
constexpr int EPI = 256;                  // epilogue threads
constexpr int SCAN_THREADS = 64 + EPI;
constexpr uint32_t REST_B = AK_B + NS * C * 4;  // k' images and the U^T slice
constexpr int TM_D2 = 64;                 // D2 columns; D1 at 0 and 128 by chunk parity

__global__ void __launch_bounds__(SCAN_THREADS, 1) gdn_umma_scan_kernel(Params p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t sb = smem_u32(smem);
  if (sb & 1023u) {
    if (threadIdx.x == 0) atomicExch(&g_device_error, kErrWaitTimeout);
    return;
  }
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n0 = blockIdx.x * NS, h = blockIdx.y, b = blockIdx.z;
  // awq_hi / awq_lo: the hi / lo planes of [q'^T; W^T] landed; s1a: the
  // UMMAs reading the hi planes completed, s1: all of D1 = [q'; W] S;
  // rest: the k' images and U landed, ai: the intra images landed; s23: D2
  // completed, out: D1 += [intra; 0] v_new completed
  const uint32_t bar_awq = sb + S_BAR, bar_rest = bar_awq + 8, bar_s1 = bar_awq + 16, bar_s23 = bar_awq + 24,
                 bar_vnew = bar_awq + 32, bar_sready = bar_awq + 40, bar_drain = bar_awq + 48,
                 bar_awq_lo = bar_awq + 56, bar_s1a = bar_awq + 64, bar_ai = bar_awq + 72, bar_out = bar_awq + 80;
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(smem + S_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + S_MISC + 4);
  const int nc = p.c1 - p.c0;  // chunk c of the loops below is chunk p.c0 + c

  if (tid == 0) {
    mbar_init(bar_awq, 1);
    mbar_init(bar_awq_lo, 1);
    mbar_init(bar_s1a, 1);
    mbar_init(bar_rest, 1);
    mbar_init(bar_s1, 1);
    mbar_init(bar_s23, 1);
    mbar_init(bar_vnew, EPI / 32);  // one arrival per epilogue warp
    mbar_init(bar_sready, EPI / 32);
    mbar_init(bar_drain, 1);
    mbar_init(bar_ai, 1);
    mbar_init(bar_out, 1);
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32((const void*)tmem_slot), 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- operand loads ----------------
      griddep_wait();  // the records are the prep grid's output
      int n_awq = 0, n_lo = 0, n_rest = 0, n_ai = 0;  // copies issued on each barrier
      for (int c = 0; c < nc; ++c) {
        const uint8_t* rec = p.rec + chunk_index(p, b, p.c0 + c, h) * REC_B;
        // hi planes once the previous chunk's UMMAs reading them are done,
        // lo planes once all of its D1 products are
        if (c > 0 && !mbar_wait(bar_s1a, (c - 1) & 1, abort_flag, WAIT)) break;
        mbar_arrive_expect_tx(bar_awq, AWQ_B / 2);
#pragma unroll
        for (int k = 0; k < 4; ++k) bulk_g2s(sb + S_AWQ + k * T64, rec + k * T64, T64, bar_awq);
        ++n_awq;
        if (c > 0 && !mbar_wait(bar_s1, (c - 1) & 1, abort_flag, WAIT)) break;
        mbar_arrive_expect_tx(bar_awq_lo, AWQ_B / 2);
#pragma unroll
        for (int k = 4; k < 8; ++k) bulk_g2s(sb + S_AWQ + k * T64, rec + k * T64, T64, bar_awq_lo);
        ++n_lo;
        // k' and U once the previous chunk's D2 is done (U was read before
        // D2 was issued), intra once its intra products are
        if (c > 0 && !mbar_wait(bar_s23, (c - 1) & 1, abort_flag, WAIT)) break;
        mbar_arrive_expect_tx(bar_rest, REST_B);
        bulk_g2s(sb + S_AK, rec + AWQ_B, AK_B / 2, bar_rest);
        bulk_g2s(sb + S_AK + AK_B / 2, rec + AWQ_B + AK_B / 2, AK_B / 2, bar_rest);
        bulk_g2s(sb + S_U, rec + AWQ_B + AK_B + AI_B + (size_t)n0 * C * 4, NS * C * 4, bar_rest);
        ++n_rest;
        if (c > 0 && !mbar_wait(bar_out, (c - 1) & 1, abort_flag, WAIT)) break;
        mbar_arrive_expect_tx(bar_ai, AI_B);
        bulk_g2s(sb + S_AI, rec + AWQ_B + AK_B, T64, bar_ai);
        bulk_g2s(sb + S_AI + 2 * T64, rec + AWQ_B + AK_B + T64, T64, bar_ai);
        ++n_ai;
      }
      // drain: every copy has landed before the CTA exits
      volatile int never = 0;
      if (n_awq > 0) mbar_wait(bar_awq, (n_awq - 1) & 1, &never, WAIT);
      if (n_lo > 0) mbar_wait(bar_awq_lo, (n_lo - 1) & 1, &never, WAIT);
      if (n_rest > 0) mbar_wait(bar_rest, (n_rest - 1) & 1, &never, WAIT);
      if (n_ai > 0) mbar_wait(bar_ai, (n_ai - 1) & 1, &never, WAIT);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- UMMA issuer ----------------
      constexpr uint32_t id_mnmn = umma_idesc_bf16(128, NS, 1, 1);
      constexpr uint32_t id_kmn = umma_idesc_bf16(128, NS, 0, 1);
      bool any = false;
      for (int c = 0; c < nc; ++c) {
        const uint32_t d1 = tmem + (c & 1) * 128;
        if (!mbar_wait(bar_awq, c & 1, abort_flag, WAIT) || !mbar_wait(bar_sready, c & 1, abort_flag, WAIT)) break;
        tc_fence_after();
        // D1 = [q'; W] S  (A MN-major: q'^T then W^T blocks; B = S MN-major):
        // the two products with the hi planes of A first, then A lo x S hi
#pragma unroll
        for (int s = 0; s < DK / 16; ++s) {
          const uint64_t ah = umma_desc_sw128(sb + S_AWQ + s * 2048, T128, 1024);
          const uint64_t bh = umma_desc_sw128(sb + S_S + s * 2048, T128, 1024);
          const uint64_t bl = umma_desc_sw128(sb + S_S + T128 + s * 2048, T128, 1024);
          umma_bf16_ss(d1, ah, bh, id_mnmn, s > 0 ? 1u : 0u);
          umma_bf16_ss(d1, ah, bl, id_mnmn, 1u);
        }
        umma_commit(bar_s1a);
        any = true;
        if (!mbar_wait(bar_awq_lo, c & 1, abort_flag, WAIT)) break;
        tc_fence_after();
#pragma unroll
        for (int s = 0; s < DK / 16; ++s) {
          const uint64_t al = umma_desc_sw128(sb + S_AWQ + 2 * T128 + s * 2048, T128, 1024);
          const uint64_t bh = umma_desc_sw128(sb + S_S + s * 2048, T128, 1024);
          umma_bf16_ss(d1, al, bh, id_mnmn, 1u);
        }
        umma_commit(bar_s1);
        any = true;
        if (!mbar_wait(bar_rest, c & 1, abort_flag, WAIT) || !mbar_wait(bar_vnew, c & 1, abort_flag, WAIT)) break;
        tc_fence_after();
#pragma unroll
        for (int s = 0; s < C / 16; ++s) {
          // D2 = k'^T v_new (A MN-major from the k' [t][d] tiles)
          const uint64_t kh = umma_desc_sw128(sb + S_AK + s * 2048, T64, 1024);
          const uint64_t kl = umma_desc_sw128(sb + S_AK + 2 * T64 + s * 2048, T64, 1024);
          const uint64_t vh = umma_desc_sw128(sb + S_V + s * 2048, T64, 1024);
          const uint64_t vl = umma_desc_sw128(sb + S_V + T64 + s * 2048, T64, 1024);
          umma_bf16_ss(tmem + TM_D2, kh, vh, id_mnmn, s > 0 ? 1u : 0u);
          umma_bf16_ss(tmem + TM_D2, kh, vl, id_mnmn, 1u);
          umma_bf16_ss(tmem + TM_D2, kl, vh, id_mnmn, 1u);
        }
        umma_commit(bar_s23);
        if (!mbar_wait(bar_ai, c & 1, abort_flag, WAIT)) break;
        tc_fence_after();
#pragma unroll
        for (int s = 0; s < C / 16; ++s) {
          // D1 += [intra; 0] v_new (A K-major)
          const uint64_t vh = umma_desc_sw128(sb + S_V + s * 2048, T64, 1024);
          const uint64_t vl = umma_desc_sw128(sb + S_V + T64 + s * 2048, T64, 1024);
          const uint64_t ih = umma_desc_sw128(sb + S_AI + s * 32, 16, 1024);
          const uint64_t il = umma_desc_sw128(sb + S_AI + 2 * T64 + s * 32, 16, 1024);
          umma_bf16_ss(d1, ih, vh, id_kmn, 1u);
          umma_bf16_ss(d1, ih, vl, id_kmn, 1u);
          umma_bf16_ss(d1, il, vh, id_kmn, 1u);
        }
        umma_commit(bar_out);
      }
      if (any) {  // every UMMA issued has completed before TMEM is freed
        umma_commit(bar_drain);
        volatile int never = 0;
        mbar_wait(bar_drain, 0, &never, WAIT);
      }
    }
  } else {
    // ---------------- v_new, state, output ----------------
    // TMEM lane r: state row d = r, and (r >= 64) the W S row of token
    // r - 64, (r < 64) the output row of token r; this thread's columns:
    // [c0, c0 + 32) of the CTA's 64.
    const int q4 = warp & 3, r = q4 * 32 + lane, c0 = ((warp - 2) >> 2) * 32;
    const uint32_t tl = tmem + ((uint32_t)(q4 * 32) << 16);
    float st[32];
#pragma unroll
    for (int n = 0; n < 32; ++n)
      st[n] = p.s_in ? p.s_in[b * p.s_bs + ((size_t)h * DK + r) * DV + n0 + c0 + n] : 0.f;
    auto put_s = [&]() {  // row r of the split state, MN-major [d][n]
#pragma unroll
      for (int n8 = 0; n8 < 32; n8 += 8) {
        uint4 hv, lv;
        split8(st + n8, hv, lv);
        *reinterpret_cast<uint4*>(smem + S_S + sw(r, c0 + n8)) = hv;
        *reinterpret_cast<uint4*>(smem + S_S + T128 + sw(r, c0 + n8)) = lv;
      }
    };
    put_s();
    // the zero halves of the two [intra; 0] tiles
    const uint4 z = make_uint4(0, 0, 0, 0);
    for (int e = tid - 64; e < 2 * T64 / 16; e += EPI) {
      const int slot = e < T64 / 16 ? 1 : 3, o = (e % (T64 / 16)) * 16;
      *reinterpret_cast<uint4*>(smem + S_AI + slot * T64 + o) = z;
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(bar_sready);
    const float* sU = reinterpret_cast<const float*>(smem + S_U);
    griddep_wait();  // e^last is the prep grid's output
    int c = 0;
    for (; c < nc; ++c) {
      const uint32_t d1 = (c & 1) * 128;
      const float el = p.elast[chunk_index(p, b, p.c0 + c, h)];
      float u[32];  // U for token r - 64 (v_new rows), loaded while D1 runs
      if (r >= C) {
        if (!__all_sync(0xffffffffu, mbar_wait(bar_rest, c & 1, abort_flag, WAIT))) break;
#pragma unroll
        for (int n = 0; n < 32; ++n) u[n] = sU[(c0 + n) * C + r - C];
      }
      if (!__all_sync(0xffffffffu, mbar_wait(bar_s1, c & 1, abort_flag, WAIT))) break;
      tc_fence_after();
      if (r >= C) {  // v_new = U - W S for token r - 64
        const int i = r - C;
        float ws[32];
        tmem_ld32(tl + d1 + c0, ws);
        tmem_wait_ld();
#pragma unroll
        for (int n8 = 0; n8 < 32; n8 += 8) {
          float f[8];
#pragma unroll
          for (int x = 0; x < 8; ++x) f[x] = u[n8 + x] - ws[n8 + x];
          uint4 hv, lv;
          split8(f, hv, lv);
          *reinterpret_cast<uint4*>(smem + S_V + sw(i, c0 + n8)) = hv;
          *reinterpret_cast<uint4*>(smem + S_V + T64 + sw(i, c0 + n8)) = lv;
        }
        fence_proxy_async_smem();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_vnew);
      if (!__all_sync(0xffffffffu, mbar_wait(bar_s23, c & 1, abort_flag, WAIT))) break;
      tc_fence_after();
      // S = e^last S + k'^T v_new on state row r, then release the next chunk
      float d2[32];
      tmem_ld32(tl + TM_D2 + c0, d2);
      tmem_wait_ld();
#pragma unroll
      for (int n = 0; n < 32; ++n) st[n] = fmaf(el, st[n], d2[n]);
      put_s();
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_sready);
      if (r < C) {  // out = q' S + intra v_new for token r (this chunk's D1 buffer)
        if (!__all_sync(0xffffffffu, mbar_wait(bar_out, c & 1, abort_flag, WAIT))) break;
        tc_fence_after();
        tmem_ld32(tl + d1 + c0, d2);
        tmem_wait_ld();
        const int t = (p.c0 + c) * C + r;
        if (t < p.T) {
          float4* o = reinterpret_cast<float4*>(p.core + (((size_t)b * p.T + t) * p.nv + h) * DV + n0 + c0);
#pragma unroll
          for (int n4 = 0; n4 < 8; ++n4) o[n4] = make_float4(d2[4 * n4], d2[4 * n4 + 1], d2[4 * n4 + 2], d2[4 * n4 + 3]);
        }
      }
    }
    if (c == nc && p.s_out) {
      float4* so =
          reinterpret_cast<float4*>(p.s_out + (size_t)b * p.nv * DK * DV + ((size_t)h * DK + r) * DV + n0 + c0);
#pragma unroll
      for (int n4 = 0; n4 < 8; ++n4) so[n4] = make_float4(st[4 * n4], st[4 * n4 + 1], st[4 * n4 + 2], st[4 * n4 + 3]);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(*tmem_slot, 256);
}

}  // namespace gum

namespace {

// A long single-row call (a state run once through the layer) leaves most
// SMs idle during its scan: 2 CTAs per value head, one per SM.  It runs in
// pieces of PIECE chunks instead, the prep of piece i + 1 on the SMs the scan
// of piece i leaves free: scans on a high-priority stream, preps on a
// low-priority one, the state carried from piece to piece through s_out.  A
// prep runs at most two pieces ahead of the scans (piece i's prep waits for
// the scan of piece i - 2), so that a freed SM goes to the next scan first.
// The gated norm of each piece runs on a third stream once its scan is done
// (it needs no shared memory, so it shares SMs with the preps and scans).
// The streams fork from and join back into the caller's stream.
struct PieceStreams {
  int dev;
  cudaStream_t scan, prep, norm;
  std::deque<cudaEvent_t> ev;
};
std::mutex g_piece_mu;
std::deque<PieceStreams> g_piece;

// The calling thread holds g_piece_mu.
int piece_streams(PieceStreams** out) {
  int dev = 0, lo = 0, hi = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess)
    for (PieceStreams& s : g_piece)
      if (s.dev == dev) {
        *out = &s;
        return CEVK_OK;
      }
  PieceStreams s;
  s.dev = dev;
  if (e == cudaSuccess) e = cudaDeviceGetStreamPriorityRange(&lo, &hi);
  if (e == cudaSuccess) e = cudaStreamCreateWithPriority(&s.scan, cudaStreamNonBlocking, hi);
  if (e == cudaSuccess) e = cudaStreamCreateWithPriority(&s.prep, cudaStreamNonBlocking, lo);
  if (e == cudaSuccess) e = cudaStreamCreateWithPriority(&s.norm, cudaStreamNonBlocking, lo);
  if (e != cudaSuccess) return set_error(CEVK_E_CUDA, "gdn pieces: streams: %s", cudaGetErrorString(e));
  g_piece.push_back(s);
  *out = &g_piece.back();
  return CEVK_OK;
}

int piece_event(PieceStreams& s, size_t i, cudaEvent_t* out) {
  while (s.ev.size() <= i) {
    cudaEvent_t x;
    cudaError_t e = cudaEventCreateWithFlags(&x, cudaEventDisableTiming);
    if (e != cudaSuccess) return set_error(CEVK_E_CUDA, "gdn pieces: event: %s", cudaGetErrorString(e));
    s.ev.push_back(x);
  }
  *out = s.ev[i];
  return CEVK_OK;
}

}  // namespace

struct GdnNorm {
  const void* z;
  int z_rs;
  const void* w;
  float eps;
  void* y;
};
void gdn_gated_norm_rows_bf16(const float* core, const void* z, int z_rs, const void* w, float eps, void* y,
                              long long t0, long long rows, int nv, int dv, cudaStream_t st);

// Event slots: 0 the fork, 1 + 2 i the prep of piece i, 2 + 2 i its scan,
// the last slot the last norm.
int gdn_umma_pieces(const gum::Params& p0, const GdnNorm& nm, cudaStream_t st) {
  std::lock_guard<std::mutex> lock(g_piece_mu);
  PieceStreams* ps = nullptr;
  int rc = piece_streams(&ps);
  if (rc) return rc;
  const int n = (p0.n_chunks + gum::PIECE - 1) / gum::PIECE;
  cudaEvent_t fork, last_prep = nullptr, last_scan = nullptr, last_norm = nullptr, norm_done;
  if ((rc = piece_event(*ps, 0, &fork)) || (rc = piece_event(*ps, 1 + 2 * n, &norm_done))) return rc;
  cudaError_t e = cudaEventRecord(fork, st);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(ps->prep, fork, 0);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(ps->scan, fork, 0);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(ps->norm, fork, 0);
  if (e != cudaSuccess) return set_error(CEVK_E_CUDA, "gdn pieces: fork: %s", cudaGetErrorString(e));
  for (int i = 0; i < n && !rc; ++i) {
    gum::Params p = p0;
    p.c0 = i * gum::PIECE;
    p.c1 = std::min(p0.n_chunks, p.c0 + gum::PIECE);
    if (i > 0) {  // continue the state the previous piece wrote
      p.s_in = p0.s_out;
      p.s_bs = 0;
    }
    cudaEvent_t ep, es, es2;
    if ((rc = piece_event(*ps, 1 + 2 * i, &ep)) || (rc = piece_event(*ps, 2 + 2 * i, &es))) break;
    if (i >= 2) {
      if ((rc = piece_event(*ps, 2 * i - 2, &es2))) break;
      if ((e = cudaStreamWaitEvent(ps->prep, es2, 0)) != cudaSuccess) break;
    }
    gum::gdn_umma_prep_kernel<<<dim3(p.c1 - p.c0, p.nv, 1), gum::PREP_THREADS, gum::P_SMEM, ps->prep>>>(p);
    if ((rc = check_launch("gdn_umma_prep_kernel"))) break;
    if ((e = cudaEventRecord(ep, ps->prep)) != cudaSuccess) break;
    last_prep = ep;
    if ((e = cudaStreamWaitEvent(ps->scan, ep, 0)) != cudaSuccess) break;
    gum::gdn_umma_scan_kernel<<<dim3(gum::DV / gum::NS, p.nv, 1), gum::SCAN_THREADS, gum::S_SMEM, ps->scan>>>(p);
    if ((rc = check_launch("gdn_umma_scan_kernel"))) break;
    if ((e = cudaEventRecord(es, ps->scan)) != cudaSuccess) break;
    last_scan = es;
    if ((e = cudaStreamWaitEvent(ps->norm, es, 0)) != cudaSuccess) break;
    const long long t0 = (long long)p.c0 * gum::C, t1 = std::min((long long)p.c1 * gum::C, (long long)p.T);
    gdn_gated_norm_rows_bf16(p.core, nm.z, nm.z_rs, nm.w, nm.eps, nm.y, t0, t1 - t0, p.nv, gum::DV, ps->norm);
    if ((rc = check_launch("gdn_gated_norm_kernel"))) break;
    if ((e = cudaEventRecord(norm_done, ps->norm)) != cudaSuccess) break;
    last_norm = norm_done;
  }
  // join: the caller's stream waits for everything enqueued above
  if (last_prep && cudaStreamWaitEvent(st, last_prep, 0) != cudaSuccess && e == cudaSuccess) e = cudaErrorUnknown;
  if (last_scan && cudaStreamWaitEvent(st, last_scan, 0) != cudaSuccess && e == cudaSuccess) e = cudaErrorUnknown;
  if (last_norm && cudaStreamWaitEvent(st, last_norm, 0) != cudaSuccess && e == cudaSuccess) e = cudaErrorUnknown;
  if (rc) return rc;
  if (e != cudaSuccess) return set_error(CEVK_E_CUDA, "gdn pieces: %s", cudaGetErrorString(e));
  return CEVK_OK;
}

// Workspace floats of the tcgen05 path beyond the core output: one operand
// record per (row, chunk, value head) plus e^last.
size_t gdn_umma_extra_floats(int B, int T, int nv) {
  const size_t nc = (size_t)(T + gum::C - 1) / gum::C;
  return (size_t)B * nc * nv * (gum::REC_B / sizeof(float) + 1);
}

void gdn_gated_norm_rows_bf16(const float* core, const void* z, int z_rs, const void* w, float eps, void* y,
                              long long t0, long long rows, int nv, int dv, cudaStream_t st);

// Runs the delta rule into the f32 core output and the gated norm from it
// into y.
int gdn_umma_run(const void* conv_out, int C_, const void* ab, int ab_rs, const float* a_log, const float* dt_bias,
                 const float* s_in, long long s_bs, float* s_out, float* workspace, int B, int T, int nk, int nv,
                 const void* z, int z_rs, const void* norm_w, float eps, void* y, cudaStream_t st) {
  gum::Params p;
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
  p.n_chunks = (T + gum::C - 1) / gum::C;
  p.core = workspace;
  uint8_t* x = reinterpret_cast<uint8_t*>(workspace + (size_t)B * T * nv * gum::DV);
  // the records are read by bulk copies: 16-byte alignment
  x = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(x) + 15) & ~uintptr_t(15));
  p.rec = x;
  p.elast = reinterpret_cast<float*>(x + (size_t)B * p.n_chunks * nv * gum::REC_B);
  p.c0 = 0;
  p.c1 = p.n_chunks;
  int rc;
  if ((rc = opt_in_smem((const void*)gum::gdn_umma_prep_kernel, gum::P_SMEM, "gdn_umma_prep_kernel")) ||
      (rc = opt_in_smem((const void*)gum::gdn_umma_scan_kernel, gum::S_SMEM, "gdn_umma_scan_kernel")))
    return rc;
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (B == 1 && s_out && p.n_chunks >= 2 * gum::PIECE && cudaStreamIsCapturing(st, &cap) == cudaSuccess &&
      cap == cudaStreamCaptureStatusNone)
    return gdn_umma_pieces(p, GdnNorm{z, z_rs, norm_w, eps, y}, st);
  gum::gdn_umma_prep_kernel<<<dim3(p.n_chunks, nv, B), gum::PREP_THREADS, gum::P_SMEM, st>>>(p);
  if ((rc = check_launch("gdn_umma_prep_kernel"))) return rc;
  {  // the scan as a programmatic dependent of the prep
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(gum::DV / gum::NS, nv, B);
    cfg.blockDim = dim3(gum::SCAN_THREADS);
    cfg.dynamicSmemBytes = gum::S_SMEM;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, gum::gdn_umma_scan_kernel, p);
    if (e != cudaSuccess)
      return set_error(CEVK_E_CUDA, "gdn_umma_scan_kernel: launch: %s", cudaGetErrorString(e));
  }
  if ((rc = check_launch("gdn_umma_scan_kernel"))) return rc;
  gdn_gated_norm_rows_bf16(p.core, z, z_rs, norm_w, eps, y, 0, (long long)B * T, nv, gum::DV, st);
  return CEVK_OK;
}

}  // namespace cevk
