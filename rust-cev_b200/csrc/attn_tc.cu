// Packed block-masked prefill attention on sm_100a tensor cores.
//
// One CTA computes one work tile: 128 query rows of one segment and one KV
// head -- the G = hq/hkv query heads of that KV head times 128/G tokens,
// row r <-> (token t0 + r/G, head r%G) -- so every K/V tile it loads serves
// all G heads (GQA without copies).  The tile walks the segment's visible
// keys only: the prefix range (full) and its own rows (causal, only up to
// the tile's last token).  Key tiles of other segments are never loaded,
// and no mask is materialised: validity is decided per element from the
// segment descriptor.
//
// Warp roles (256 threads):
//   warp 0  TMA producer for Q and K (one elected lane)
//   warp 1  TMEM allocator + UMMA issuer (one elected lane)
//   warp 2  TMA producer for V
//   warps 4-7  softmax / O correction / epilogue, one query row per thread
//             (TMEM lane = row).
// TMEM: two S buffers (BN columns each, f32) so QK^T of block j+1 runs
// while block j is in softmax, and the O accumulator (D columns, f32).
// P (bf16) overwrites its own S in TMEM and feeds the PV UMMA as the TMEM A
// operand, so the softmax never waits for the previous PV (only an O
// rescale does).  Online softmax in the log2 domain; O is only rescaled when
// a row max grows by more than 2^8 (values of P stay <= 256, exact in f32
// accumulation), which keeps TMEM traffic off the common path.
#include <cudaTypedefs.h>

#include <cmath>
#include <cstdio>

#include "common.cuh"

namespace cevk {

template <int D, int BN, int KST>
struct AttnTc {
  static constexpr int BM = 128;
  static constexpr int ATOM = BM * 128;         // one 64-column (128 B) slab of a 128-row tile
  static constexpr int Q_BYTES = BM * D * 2;
  static constexpr int KV_BYTES = BN * D * 2;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + Q_BYTES;
  static constexpr int OFF_V = OFF_K + KST * KV_BYTES;
  static constexpr int OFF_BAR = OFF_V + KST * KV_BYTES;
  // barriers: q_full, k_full[KST], k_empty[KST], v_full[KST], v_empty[KST],
  // s_full[2], p_full, o_done, drain
  static constexpr int N_BAR = 1 + 4 * KST + 2 + 3;
  static constexpr int OFF_MISC = OFF_BAR + N_BAR * 8;
  static constexpr int SMEM = OFF_MISC + 16;
  static constexpr int TM_S0 = 0;
  static constexpr int TM_S1 = BN;
  static constexpr int TM_O = 2 * BN;
  static constexpr int TM_COLS = (2 * BN + D) <= 256 ? 256 : 512;
  // Two CTAs per SM when both fit (228 KB per SM, 1 KB reserved per CTA):
  // one CTA's softmax then overlaps the other's UMMAs.
  static constexpr int MIN_BLOCKS = (2 * (SMEM + 1024) <= 233472 && TM_COLS <= 256) ? 2 : 1;
  static_assert(D % 64 == 0 && BN % 64 == 0 && BN <= 128, "tile shape");
  static_assert(OFF_K % 1024 == 0 && OFF_V % 1024 == 0, "1024-aligned tiles");
};

struct AttnParams {
  __nv_bfloat16* o;
  const cevk_segment* segs;
  int n_segs;
  int hq, hkv, group, rows_t;
  int o_row_stride;
  float scale_log2;
};

__device__ __forceinline__ int find_segment(const cevk_segment* segs, int n, int tile) {
  int lo = 0, hi = n - 1;
  while (lo < hi) {
    int mid = (lo + hi + 1) >> 1;
    if (__ldg(&segs[mid].tile_start) <= tile) lo = mid; else hi = mid - 1;
  }
  return lo;
}

template <int D, int BN, int KST>
__global__ void __launch_bounds__(256, AttnTc<D, BN, KST>::MIN_BLOCKS)
attn_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
               const __grid_constant__ CUtensorMap tm_v, AttnParams p) {
  using C = AttnTc<D, BN, KST>;
  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t sbase = smem_u32(smem);
  // The swizzled tiles need a 1024-byte aligned base (no static shared
  // memory precedes the dynamic window, so this holds).
  if (sbase & 1023u) {
    if (threadIdx.x == 0) atomicExch(&g_device_error, kErrWaitTimeout);
    return;
  }
  const uint32_t sQ = sbase + C::OFF_Q, sK = sbase + C::OFF_K, sV = sbase + C::OFF_V;
  const uint32_t bar0 = sbase + C::OFF_BAR;
  const uint32_t b_qfull = bar0;
  auto b_kfull = [&](int s) { return bar0 + 8u * (1 + s); };
  auto b_kempty = [&](int s) { return bar0 + 8u * (1 + KST + s); };
  auto b_vfull = [&](int s) { return bar0 + 8u * (1 + 2 * KST + s); };
  auto b_vempty = [&](int s) { return bar0 + 8u * (1 + 3 * KST + s); };
  auto b_sfull = [&](int s) { return bar0 + 8u * (1 + 4 * KST + s); };
  const uint32_t b_pfull = bar0 + 8u * (3 + 4 * KST);
  const uint32_t b_odone = bar0 + 8u * (4 + 4 * KST);
  const uint32_t b_drain = bar0 + 8u * (5 + 4 * KST);
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(smem + C::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // ---- work decode (every thread; cheap) ----
  const int tile = blockIdx.x / p.hkv;
  const int kvh = blockIdx.x % p.hkv;
  const int si = find_segment(p.segs, p.n_segs, tile);
  const cevk_segment seg = p.segs[si];
  const int t0 = (tile - seg.tile_start) * p.rows_t;
  const int nt = min(p.rows_t, seg.q_len - t0);
  const int n_pre = (seg.prefix_len + BN - 1) / BN;
  const int n_self = (t0 + nt + BN - 1) / BN;
  const int n_blk = n_pre + n_self;
  auto kv_row = [&](int j) { return j < n_pre ? seg.prefix_off + j * BN : seg.self_off + (j - n_pre) * BN; };

  if (threadIdx.x == 0) {
    mbar_init(b_qfull, 1);
    for (int s = 0; s < KST; ++s) {
      mbar_init(b_kfull(s), 1);
      mbar_init(b_kempty(s), 1);
      mbar_init(b_vfull(s), 1);
      mbar_init(b_vempty(s), 1);
    }
    mbar_init(b_sfull(0), 1);
    mbar_init(b_sfull(1), 1);
    mbar_init(b_pfull, 128);
    mbar_init(b_odone, 1);
    mbar_init(b_drain, 1);
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32((const void*)tmem_slot), C::TM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ---------------- Q + K producer ----------------
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    mbar_arrive_expect_tx(b_qfull, C::Q_BYTES);
#pragma unroll
    for (int a = 0; a < D / 64; ++a) tma_load_3d(sQ + a * C::ATOM, &tm_q, b_qfull, a * 64, kvh * p.group, seg.q_start + t0);
    int issued = 0;
    for (int j = 0; j < n_blk; ++j) {
      const int st = j % KST;
      if (j >= KST && !mbar_wait(b_kempty(st), ((j / KST) - 1) & 1, abort_flag)) break;
      mbar_arrive_expect_tx(b_kfull(st), C::KV_BYTES);
#pragma unroll
      for (int a = 0; a < D / 64; ++a) tma_load_3d(sK + st * C::KV_BYTES + a * BN * 128, &tm_k, b_kfull(st), a * 64, kvh, kv_row(j));
      issued = j + 1;
    }
    // Drain: the last load of every stage has landed before the CTA exits.
    volatile int never = 0;
    mbar_wait(b_qfull, 0, &never, 1ll << 30);
    for (int j = max(0, issued - KST); j < issued; ++j) mbar_wait(b_kfull(j % KST), (j / KST) & 1, &never, 1ll << 30);
  } else if (warp == 2 && lane == 0) {
    // ---------------- V producer ----------------
    tma_prefetch_desc(&tm_v);
    int issued = 0;
    for (int j = 0; j < n_blk; ++j) {
      const int st = j % KST;
      if (j >= KST && !mbar_wait(b_vempty(st), ((j / KST) - 1) & 1, abort_flag)) break;
      mbar_arrive_expect_tx(b_vfull(st), C::KV_BYTES);
#pragma unroll
      for (int a = 0; a < D / 64; ++a) tma_load_3d(sV + st * C::KV_BYTES + a * BN * 128, &tm_v, b_vfull(st), a * 64, kvh, kv_row(j));
      issued = j + 1;
    }
    for (int j = max(0, issued - KST); j < issued; ++j) {
      volatile int never = 0;
      mbar_wait(b_vfull(j % KST), (j / KST) & 1, &never, 1ll << 30);
    }
  } else if (warp == 1 && lane == 0) {
    // ---------------- UMMA issuer ----------------
    constexpr uint32_t idesc_s = umma_idesc_bf16(128, BN, 0, 0);
    constexpr uint32_t idesc_o = umma_idesc_bf16(128, D, 0, 1);
    bool ok = mbar_wait(b_qfull, 0, abort_flag);
    auto issue_s = [&](int j) -> bool {
      const int st = j % KST;
      if (!mbar_wait(b_kfull(st), (j / KST) & 1, abort_flag)) return false;
      tc_fence_after();
      const uint32_t d = tmem + ((j & 1) ? C::TM_S1 : C::TM_S0);
      const uint32_t kb = sK + st * C::KV_BYTES;
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const uint64_t ad = umma_desc_sw128(sQ + (kk >> 2) * C::ATOM + (kk & 3) * 32, 16, 1024);
        const uint64_t bd = umma_desc_sw128(kb + (kk >> 2) * (BN * 128) + (kk & 3) * 32, 16, 1024);
        umma_bf16_ss(d, ad, bd, idesc_s, kk > 0 ? 1u : 0u);
      }
      umma_commit(b_sfull(j & 1));
      umma_commit(b_kempty(st));
      return true;
    };
    if (ok) ok = issue_s(0);
    if (ok && n_blk > 1) ok = issue_s(1);
    for (int j = 0; ok && j < n_blk; ++j) {
      if (!mbar_wait(b_pfull, j & 1, abort_flag)) break;
      const int st = j % KST;
      if (!mbar_wait(b_vfull(st), (j / KST) & 1, abort_flag)) break;
      tc_fence_after();
      const uint32_t vb = sV + st * C::KV_BYTES;
      // P_j (bf16) sits in the first BN/2 columns of S_j's buffer.
      const uint32_t pa = tmem + ((j & 1) ? C::TM_S1 : C::TM_S0);
#pragma unroll
      for (int kk = 0; kk < BN / 16; ++kk) {
        const uint64_t bd = umma_desc_sw128(vb + kk * 16 * 128, BN * 128, 1024);
        umma_bf16_ts(tmem + C::TM_O, pa + kk * 8, bd, idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
      }
      umma_commit(b_odone);
      umma_commit(b_vempty(st));
      if (j + 2 < n_blk) ok = issue_s(j + 2);
    }
    // Every UMMA this thread issued has completed before TMEM is freed.
    umma_commit(b_drain);
    volatile int never = 0;
    mbar_wait(b_drain, 0, &never, 1ll << 30);
  } else if (warp >= 4) {
    // ---------------- softmax / correction / epilogue ----------------
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;
    const int t = t0 + r / p.group;
    const int h = r % p.group;
    const uint32_t tl = tmem + ((uint32_t)(q4 * 32) << 16);
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    float s[BN];
    uint32_t pk[BN / 2];
    for (int j = 0; j < n_blk; ++j) {
      if (!mbar_wait(b_sfull(j & 1), (j >> 1) & 1, abort_flag)) { ok = false; break; }
      tc_fence_after();
      const uint32_t sc = tl + ((j & 1) ? C::TM_S1 : C::TM_S0);
#pragma unroll
      for (int c = 0; c < BN; c += 32) tmem_ld32(sc + c, s + c);
      tmem_wait_ld();
      // Key column c is visible if c <= lim: inside the prefix for a prefix
      // block, causal for an own block.  Full blocks skip the mask.
      const int lim = (j < n_pre) ? seg.prefix_len - j * BN - 1 : t - (j - n_pre) * BN;
      if (lim < BN - 1) {
#pragma unroll
        for (int c = 0; c < BN; ++c) s[c] = (c <= lim) ? s[c] : -INFINITY;
      }
      // Row max of the raw scores (scale > 0 commutes with max): 8
      // independent chains, then a tree.
      float mx[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) mx[i] = s[i];
#pragma unroll
      for (int c = 8; c < BN; c += 8)
#pragma unroll
        for (int i = 0; i < 8; ++i) mx[i] = fmaxf(mx[i], s[c + i]);
      const float mb = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                             fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7]))) * p.scale_log2;
      // Rescale only when the running max grows by more than 2^8.
      const bool need = (j == 0) || (mb > m_run + 8.f);
      const float m_new = need ? mb : m_run;
      const float factor = (j > 0 && need) ? fast_exp2(m_run - m_new) : 1.f;
      // P = 2^(s*scale - m): one FFMA + one ex2 per element, computed while
      // the previous block's PV is still on the tensor cores.
      const float neg = -m_new;
      float sm8[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) sm8[i] = 0.f;
#pragma unroll
      for (int c = 0; c < BN; c += 2) {
        const float e0 = fast_exp2(fmaf(s[c], p.scale_log2, neg));
        const float e1 = fast_exp2(fmaf(s[c + 1], p.scale_log2, neg));
        sm8[c & 7] += e0;
        sm8[(c + 1) & 7] += e1;
        pk[c >> 1] = pack_bf16x2(e0, e1);
      }
      const float sum = ((sm8[0] + sm8[1]) + (sm8[2] + sm8[3])) + ((sm8[4] + sm8[5]) + (sm8[6] + sm8[7]));
      if (__any_sync(0xffffffffu, factor != 1.f)) {
        // O is rescaled in TMEM: PV of the previous block must be done (and
        // PV of this block cannot start before P_j is signalled).
        if (!mbar_wait(b_odone, (j - 1) & 1, abort_flag)) { ok = false; break; }
        tc_fence_after();
        {
#pragma unroll 1
          for (int c = 0; c < D; c += 32) {
            float o[32];
            tmem_ld32(tl + C::TM_O + c, o);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= factor;
            tmem_st32(tl + C::TM_O + c, o);
          }
          tmem_wait_st();
        }
      }
      l_run = l_run * factor + sum;
      m_run = m_new;
      // Key rows past the tile's last visible key carry P = 0, but their V
      // rows are whatever the buffer holds there (possibly NaN/Inf, and
      // 0 * NaN = NaN in the MMA): zero them before PV reads the stage.
      {
        const int vcount = (j < n_pre) ? seg.prefix_len - j * BN : (t0 + nt) - (j - n_pre) * BN;
        if (vcount < BN) {
          const int vst = j % KST;
          if (!mbar_wait(b_vfull(vst), (j / KST) & 1, abort_flag)) { ok = false; break; }
          const int rows0 = vcount < 0 ? 0 : vcount;
          const int chunks = (BN - rows0) * 8 * (D / 64);
          uint8_t* vb = smem + C::OFF_V + vst * C::KV_BYTES;
          for (int i = threadIdx.x - 128; i < chunks; i += 128) {
            const int a = i / ((BN - rows0) * 8), rem = i % ((BN - rows0) * 8);
            *reinterpret_cast<uint4*>(vb + a * BN * 128 + (rows0 + rem / 8) * 128 + (rem % 8) * 16) = make_uint4(0, 0, 0, 0);
          }
          fence_proxy_async_smem();
        }
      }
      // P_j overwrites the (already read) S_j in TMEM, packed bf16x2.
#pragma unroll
      for (int c = 0; c < BN / 2; c += 32) tmem_st32(sc + c, reinterpret_cast<const float*>(pk + c));
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(b_pfull);
    }
    if (ok && mbar_wait(b_odone, (n_blk - 1) & 1, abort_flag)) {
      tc_fence_after();
      const float inv = 1.f / l_run;
      const bool store = (t < seg.q_len) && (r / p.group < nt);
      __nv_bfloat16* orow = p.o + (size_t)(seg.q_start + t) * p.o_row_stride + (size_t)(kvh * p.group + h) * D;
#pragma unroll 1
      for (int c = 0; c < D; c += 32) {
        float o[32];
        tmem_ld32(tl + C::TM_O + c, o);
        tmem_wait_ld();
        if (store) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            uint4 pk;
            pk.x = pack_bf16x2(o[i] * inv, o[i + 1] * inv);
            pk.y = pack_bf16x2(o[i + 2] * inv, o[i + 3] * inv);
            pk.z = pack_bf16x2(o[i + 4] * inv, o[i + 5] * inv);
            pk.w = pack_bf16x2(o[i + 6] * inv, o[i + 7] * inv);
            *reinterpret_cast<uint4*>(orow + c + i) = pk;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TM_COLS);
  }
}

// ---------------------------------------------------------------------------
// Host side.
// ---------------------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// 3-D bf16 map over [rows][heads][D] (row stride in elements), 128B swizzle.
static int make_map(CUtensorMap* m, const void* base, int D, int heads, int rows, int row_stride, int box_h,
                    int box_rows) {
  auto enc = get_encode();
  if (!enc) return set_error(CEVK_E_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)heads, (cuuint64_t)rows};
  cuuint64_t strides[2] = {(cuuint64_t)D * 2, (cuuint64_t)row_stride * 2};
  cuuint32_t box[3] = {64, (cuuint32_t)box_h, (cuuint32_t)box_rows};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(CEVK_E_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return CEVK_OK;
}

template <int D, int BN, int KST>
static int launch_tc(const void* q, const void* k, const void* v, void* o, int n_tokens, int n_kv_rows, int hq, int hkv,
                     int q_rs, int kv_rs, int o_rs, const cevk_segment* segs, int n_segs, int n_tiles, float scale,
                     cudaStream_t stream) {
  using C = AttnTc<D, BN, KST>;
  const int group = hq / hkv, rows_t = 128 / group;
  CUtensorMap tq, tk, tv;
  int rc;
  if ((rc = make_map(&tq, q, D, hq, n_tokens, q_rs, group, rows_t))) return rc;
  if ((rc = make_map(&tk, k, D, hkv, n_kv_rows, kv_rs, 1, BN))) return rc;
  if ((rc = make_map(&tv, v, D, hkv, n_kv_rows, kv_rs, 1, BN))) return rc;
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(attn_tc_kernel<D, BN, KST>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM) !=
        cudaSuccess)
      return set_error(CEVK_E_CUDA, "cannot opt in to %d B of shared memory", C::SMEM);
    attr = true;
  }
  AttnParams prm;
  prm.o = reinterpret_cast<__nv_bfloat16*>(o);
  prm.segs = segs;
  prm.n_segs = n_segs;
  prm.hq = hq;
  prm.hkv = hkv;
  prm.group = group;
  prm.rows_t = rows_t;
  prm.o_row_stride = o_rs;
  prm.scale_log2 = scale * 1.4426950408889634f;
  attn_tc_kernel<D, BN, KST><<<(unsigned)n_tiles * hkv, 256, C::SMEM, stream>>>(tq, tk, tv, prm);
  return check_launch("attn_tc_kernel");
}

int attn_tc_launch(const void* q, const void* k, const void* v, void* o, int n_tokens, int n_kv_rows, int hq, int hkv,
                   int D, int q_rs, int kv_rs, int o_rs, const cevk_segment* segs, int n_segs, int n_tiles, float scale,
                   cudaStream_t stream) {
  switch (D) {
    case 64:
      return launch_tc<64, 64, 3>(q, k, v, o, n_tokens, n_kv_rows, hq, hkv, q_rs, kv_rs, o_rs, segs, n_segs, n_tiles,
                                  scale, stream);
    case 128:
      return launch_tc<128, 64, 2>(q, k, v, o, n_tokens, n_kv_rows, hq, hkv, q_rs, kv_rs, o_rs, segs, n_segs, n_tiles,
                                   scale, stream);
    case 256:
      return launch_tc<256, 64, 2>(q, k, v, o, n_tokens, n_kv_rows, hq, hkv, q_rs, kv_rs, o_rs, segs, n_segs, n_tiles,
                                   scale, stream);
    default:
      return set_error(CEVK_E_SHAPE, "bf16 attention supports head_dim 64, 128, 256 (got %d)", D);
  }
}

}  // namespace cevk
