// Packed block-masked prefill attention on sm_100a tensor cores.
//
// A work tile is 128 query rows of one segment and one KV head -- the
// G = hq/hkv query heads of that KV head times 128/G tokens, row r <->
// (token t0 + r/G, head r%G) -- so every K/V tile loaded serves all G heads
// (GQA without copies).  A tile walks the segment's visible keys only: the
// prefix range (full) and its own rows (causal, only up to the tile's last
// token).  Key tiles of other segments are never loaded, and no mask is
// materialised: validity is decided per element from the segment descriptor.
//
// A CTA runs one work tile, two CTAs per SM for head_dim 64 / 128 (one
// CTA's softmax overlaps the other's UMMAs), one per SM for head_dim 256.
// Warp roles (256 threads):
//   warp 0        TMA producer for Q and K (one lane)
//   warp 2        TMA producer for V
//   warp 1        TMEM allocator + issuer of the S = Q K^T UMMAs (one lane)
//   warp 3        issuer of the O += P V UMMAs (one lane)
//   warps 4-7     softmax / O correction / epilogue, one query row per
//                 thread (TMEM lane = row).
// The two UMMA streams only meet through the softmax (S_j -> P_j), so with
// one issuing thread each a burst of one never queues behind the other's
// issue (a tcgen05.mma takes tens of cycles to issue from one thread).
// TMEM per tile: S (BN f32 columns), a double buffer for P (bf16 packed in
// pairs, BN/2 columns each) and the O accumulator (D f32 columns).  S_{j+1}
// is issued as soon as the softmax has S_j in registers, so it runs while
// block j is in softmax; P_j feeds the PV UMMA as the TMEM A operand.  The
// S issuer commits S_j only after PV_{j-2} completed, so a softmax that has
// S_j may overwrite PV_{j-2}'s P buffer without a wait of its own (it waits
// for PV_{j-1} only before an O rescale).  Online softmax in the log2 domain; O is
// only rescaled when a row max grows by more than 2^8 (values of P stay
// <= 256, exact in f32 accumulation), which keeps TMEM traffic off the
// common path.
//
// Split-KV (n_split > 1): when the call has too few tiles to fill the GPU
// (a prefill chunk after a long cached prefix), each tile's key blocks are
// cut into up to n_split contiguous ranges, one CTA each.  Every range
// starts inside the prefix, whose keys every row of the tile sees, so no
// row of a range is fully masked.  A ranged CTA writes its normalised f32
// output rows and their log2-sum-exp to a workspace and attn_combine_kernel
// merges the ranges; a tile left with one range stores o directly.
#include <cudaTypedefs.h>

#include <cmath>
#include <cstdio>

#include "common.cuh"

namespace cevk {

template <int D, int BN, int KSK, int KSV, int NT>
struct AttnTc {
  static constexpr int BM = 128;
  static constexpr int ATOM = BM * 128;         // one 64-column (128 B) slab of a 128-row tile
  static constexpr int Q_BYTES = BM * D * 2;
  static constexpr int KV_BYTES = BN * D * 2;
  // per work tile: Q, K ring, V ring
  static constexpr int T_OFF_Q = 0;
  static constexpr int T_OFF_K = Q_BYTES;
  static constexpr int T_OFF_V = T_OFF_K + KSK * KV_BYTES;
  static constexpr int T_BYTES = T_OFF_V + KSV * KV_BYTES;
  // barriers per tile: q_full, k_full[KSK], k_empty[KSK], v_full[KSV],
  // v_empty[KSV], s_full, s_free, p_full[2], o_done[2] (by block parity).
  // A parity wait cannot tell phase k from k+2, so every waiter must be at
  // most one phase away from its barrier; the comments at each wait say why.
  static constexpr int T_BARS = 1 + 2 * KSK + 2 * KSV + 6;
  static constexpr int OFF_BAR = NT * T_BYTES;
  static constexpr int OFF_MISC = OFF_BAR + (NT * T_BARS + 2) * 8;  // + drain of the S and PV issuers
  static constexpr int SMEM = OFF_MISC + 16;
  // TMEM per tile: S (BN f32 columns), P double buffer (BN/2 columns of
  // packed bf16 each), O (D f32 columns).
  static constexpr int TM_S = 0;
  static constexpr int TM_P = BN;
  static constexpr int TM_O = 2 * BN;
  static constexpr int TM_TILE = 256;           // TMEM columns per tile
  static constexpr int TM_COLS = NT == 1 && (2 * BN + D) <= 256 ? 256 : 512;
  static constexpr int THREADS = NT == 2 ? 416 : 256;
  static constexpr int MIN_BLOCKS = (NT == 1 && TM_COLS <= 256 && 2 * (OFF_MISC + 16 + 1024) <= 233472) ? 2 : 1;
  static_assert(2 * BN + D <= 512 / NT, "TMEM budget");
  static_assert(D % 64 == 0 && BN % 64 == 0 && BN <= 128, "tile shape");
  static_assert(T_OFF_K % 1024 == 0 && T_OFF_V % 1024 == 0 && T_BYTES % 1024 == 0, "1024-aligned tiles");
  static_assert(SMEM <= 232448, "shared memory");
};

// Output buffers: every bf16 output row is stored to each of o[0 .. n_o)
// (one buffer normally; every rank's gathered buffer, through peer
// pointers, for the fused head all-gather).
constexpr int kMaxOut = 8;
struct AttnParams {
  __nv_bfloat16* o[kMaxOut];
  int n_o;
  const cevk_segment* segs;
  int n_segs;
  int n_work;   // work tiles = segment tiles x KV heads
  int n_split;  // key ranges per work tile (1: no split); CTA items = n_work * n_split
  int hq, hkv, group, rows_t;
  int o_row_stride;
  float scale_log2;
  float* part_o;    // [n_work * n_split][128][D] f32 partial outputs (n_split > 1)
  float* part_lse;  // [n_work * n_split][128] log2-sum-exp of each partial row
};

__device__ __forceinline__ int find_segment(const cevk_segment* segs, int n, int tile) {
  int lo = 0, hi = n - 1;
  while (lo < hi) {
    int mid = (lo + hi + 1) >> 1;
    if (__ldg(&segs[mid].tile_start) <= tile) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// One CTA item: 128 query rows (G heads x 128/G tokens) of one segment and
// one KV head, and the key blocks jb .. jb + n_blk - 1 it walks (block
// numbers count the prefix blocks first, then the segment's own blocks).
struct Work {
  cevk_segment seg;
  int kvh, t0, nt, n_pre, n_blk, jb;
  int item, n_eff;  // CTA item index; key ranges of this tile (1: o stored directly)
  __device__ __forceinline__ int kv_row(int j, int BN) const {
    return j < n_pre ? seg.prefix_off + j * BN : seg.self_off + (j - n_pre) * BN;
  }
};

// First block of key range s of n_eff over a tile of `total` blocks whose
// first n_pre are prefix blocks (n_eff <= n_pre when n_eff > 1): even cuts,
// pulled back so every range after the first starts inside the prefix.
__device__ __forceinline__ int range_start(int s, int n_eff, int total, int n_pre) {
  if (s <= 0) return 0;
  if (s >= n_eff) return total;
  return min((int)((long long)s * total / n_eff), n_pre - n_eff + s);
}

__device__ __forceinline__ Work decode_work(const AttnParams& p, int item, int BN) {
  Work k;
  k.n_blk = 0;
  k.nt = 0;
  k.jb = 0;
  k.n_eff = 1;
  k.item = item;
  if (item >= p.n_work * p.n_split) return k;
  const int w = item / p.n_split, sp = item - w * p.n_split;
  const int tile = w / p.hkv;
  k.kvh = w % p.hkv;
  k.seg = p.segs[find_segment(p.segs, p.n_segs, tile)];
  k.t0 = (tile - k.seg.tile_start) * p.rows_t;
  k.n_pre = (k.seg.prefix_len + BN - 1) / BN;
  // own blocks: up to the tile's last row (causal) or all of them (bidirectional)
  const int nt = min(p.rows_t, k.seg.q_len - k.t0);
  const int own_end = (k.seg.flags & CEVK_SEG_BIDIRECTIONAL) ? k.seg.q_len : k.t0 + nt;
  const int total = k.n_pre + (own_end + BN - 1) / BN;
  k.n_eff = k.n_pre > 0 ? min(p.n_split, k.n_pre) : 1;
  if (sp >= k.n_eff) return k;
  k.nt = nt;
  k.jb = range_start(sp, k.n_eff, total, k.n_pre);
  k.n_blk = range_start(sp + 1, k.n_eff, total, k.n_pre) - k.jb;
  return k;
}

template <int D, int BN, int KSK, int KSV, int NT>
__global__ void __launch_bounds__(AttnTc<D, BN, KSK, KSV, NT>::THREADS, AttnTc<D, BN, KSK, KSV, NT>::MIN_BLOCKS)
attn_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
               const __grid_constant__ CUtensorMap tm_v, AttnParams p) {
  using C = AttnTc<D, BN, KSK, KSV, NT>;
  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t sbase = smem_u32(smem);
  // The swizzled tiles need a 1024-byte aligned base (no static shared
  // memory precedes the dynamic window, so this holds).
  if (sbase & 1023u) {
    if (threadIdx.x == 0) atomicExch(&g_device_error, kErrWaitTimeout);
    return;
  }
  auto sQ = [&](int t) { return sbase + t * C::T_BYTES + C::T_OFF_Q; };
  auto sK = [&](int t, int st) { return sbase + t * C::T_BYTES + C::T_OFF_K + st * C::KV_BYTES; };
  auto sV = [&](int t, int st) { return sbase + t * C::T_BYTES + C::T_OFF_V + st * C::KV_BYTES; };
  auto bar = [&](int t, int i) { return sbase + C::OFF_BAR + 8u * (t * C::T_BARS + i); };
  auto b_qfull = [&](int t) { return bar(t, 0); };
  constexpr int KV4 = 2 * KSK + 2 * KSV;
  auto b_kfull = [&](int t, int s) { return bar(t, 1 + s); };
  auto b_kempty = [&](int t, int s) { return bar(t, 1 + KSK + s); };
  auto b_vfull = [&](int t, int s) { return bar(t, 1 + 2 * KSK + s); };
  auto b_vempty = [&](int t, int s) { return bar(t, 1 + 2 * KSK + KSV + s); };
  auto b_sfull = [&](int t) { return bar(t, 1 + KV4); };
  auto b_sfree = [&](int t) { return bar(t, 2 + KV4); };
  auto b_pfull = [&](int t, int s) { return bar(t, 3 + KV4 + s); };
  auto b_odone = [&](int t, int s) { return bar(t, 5 + KV4 + s); };
  const uint32_t b_drain_s = sbase + C::OFF_BAR + 8u * (NT * C::T_BARS);
  const uint32_t b_drain_o = b_drain_s + 8u;
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(smem + C::OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_MISC + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int t = 0; t < NT; ++t) {
      mbar_init(b_qfull(t), 1);
      for (int s = 0; s < KSK; ++s) {
        mbar_init(b_kfull(t, s), 1);
        mbar_init(b_kempty(t, s), 1);
      }
      for (int s = 0; s < KSV; ++s) {
        mbar_init(b_vfull(t, s), 1);
        mbar_init(b_vempty(t, s), 1);
      }
      mbar_init(b_sfull(t), 1);
      mbar_init(b_sfree(t), 128);
      mbar_init(b_pfull(t, 0), 128);
      mbar_init(b_pfull(t, 1), 128);
      mbar_init(b_odone(t, 0), 1);
      mbar_init(b_odone(t, 1), 1);
    }
    mbar_init(b_drain_s, 1);
    mbar_init(b_drain_o, 1);
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

  // Roles: warp 0 loads Q and K, warp 2 loads V, warps 1 / 3 issue the S /
  // PV UMMAs, warps 4-7 run the softmax.
  static_assert(NT == 1, "one work tile per CTA");
  const int qk_tile = warp == 0 ? 0 : -1;
  const int v_tile = warp == 2 ? 0 : -1;

  if (qk_tile >= 0 && lane == 0) {
    // ---------------- Q + K producer of one tile ----------------
    const int t = qk_tile;
    const Work wk = decode_work(p, blockIdx.x * NT + t, BN);
    volatile int never = 0;
    if (wk.n_blk > 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      mbar_arrive_expect_tx(b_qfull(t), C::Q_BYTES);
#pragma unroll
      for (int a = 0; a < D / 64; ++a)
        tma_load_3d(sQ(t) + a * C::ATOM, &tm_q, b_qfull(t), a * 64, wk.kvh * p.group, wk.seg.q_start + wk.t0);
      int issued = 0;
      for (int j = 0; j < wk.n_blk; ++j) {
        const int st = j % KSK;
        if (j >= KSK && !mbar_wait(b_kempty(t, st), ((j / KSK) - 1) & 1, abort_flag)) break;
        mbar_arrive_expect_tx(b_kfull(t, st), C::KV_BYTES);
#pragma unroll
        for (int a = 0; a < D / 64; ++a)
          tma_load_3d(sK(t, st) + a * BN * 128, &tm_k, b_kfull(t, st), a * 64, wk.kvh, wk.kv_row(wk.jb + j, BN));
        issued = j + 1;
      }
      // Drain: the Q load and the last load of every stage have landed.
      mbar_wait(b_qfull(t), 0, &never, 1ll << 30);
      for (int j = max(0, issued - KSK); j < issued; ++j)
        mbar_wait(b_kfull(t, j % KSK), (j / KSK) & 1, &never, 1ll << 30);
    }
  } else if (v_tile >= 0 && lane == 0) {
    // ---------------- V producer of one tile ----------------
    const int t = v_tile;
    const Work wk = decode_work(p, blockIdx.x * NT + t, BN);
    volatile int never = 0;
    if (wk.n_blk > 0) {
      tma_prefetch_desc(&tm_v);
      int issued = 0;
      for (int j = 0; j < wk.n_blk; ++j) {
        const int st = j % KSV;
        if (j >= KSV && !mbar_wait(b_vempty(t, st), ((j / KSV) - 1) & 1, abort_flag)) break;
        mbar_arrive_expect_tx(b_vfull(t, st), C::KV_BYTES);
#pragma unroll
        for (int a = 0; a < D / 64; ++a)
          tma_load_3d(sV(t, st) + a * BN * 128, &tm_v, b_vfull(t, st), a * 64, wk.kvh, wk.kv_row(wk.jb + j, BN));
        issued = j + 1;
      }
      for (int j = max(0, issued - KSV); j < issued; ++j)
        mbar_wait(b_vfull(t, j % KSV), (j / KSV) & 1, &never, 1ll << 30);
    }
  } else if ((warp == 1 || warp == 3) && lane == 0) {
    // ---------------- UMMA issuers ----------------
    // Warp 1 issues S = Q K^T, warp 3 issues O += P V.  The two streams only
    // meet through the softmax (S_j -> P_j), so a burst of one never waits
    // behind the other's issue; each thread commits and drains its own UMMAs.
    constexpr int t = 0;
    const int nb = decode_work(p, blockIdx.x, BN).n_blk;
    bool ok = nb > 0, issued_any = false;
    if (warp == 1) {
      constexpr uint32_t idesc_s = umma_idesc_bf16(128, BN, 0, 0);
      if (ok) ok = mbar_wait(b_qfull(t), 0, abort_flag);
      for (int j = 0; ok && j < nb; ++j) {
        // S_j as soon as the softmax has S_{j-1} in registers: it runs on
        // the tensor cores while the softmax computes block j-1.  (s_free
        // cannot lead this wait by two phases: the softmax only loads S_j
        // after this thread issued it.)
        if (j > 0 && !mbar_wait(b_sfree(t), (j - 1) & 1, abort_flag)) break;
        const int st = j % KSK;
        if (!mbar_wait(b_kfull(t, st), (j / KSK) & 1, abort_flag)) break;
        tc_fence_after();
        const uint32_t d = tmem + C::TM_S;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t ad = umma_desc_sw128(sQ(t) + (kk >> 2) * C::ATOM + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = umma_desc_sw128(sK(t, st) + (kk >> 2) * (BN * 128) + (kk & 3) * 32, 16, 1024);
          umma_bf16_ss(d, ad, bd, idesc_s, kk > 0 ? 1u : 0u);
        }
        // s_full_j also stands for "PV_{j-2} completed", so the softmax can
        // write P_j into PV_{j-2}'s buffer without a wait of its own: this
        // thread observes o_done before the commit whose arrival the softmax
        // waits for.  (PV_{j-2} completes during the softmax of block j-1,
        // well before S_j is needed.  o_done[j&1] is not two phases ahead:
        // PV_j needs P_j, which needs this commit; nor behind: PV_{j-4} was
        // waited here for S_{j-2}.)
        if (j >= 2) {
          if (!mbar_wait(b_odone(t, j & 1), ((j - 2) >> 1) & 1, abort_flag)) break;
          tc_fence_after();
        }
        umma_commit(b_sfull(t));
        umma_commit(b_kempty(t, st));
        issued_any = true;
      }
    } else {
      constexpr uint32_t idesc_o = umma_idesc_bf16(128, D, 0, 1);
      for (int j = 0; ok && j < nb; ++j) {
        // p_full[j&1] cannot lead by two phases: P_{j+2} is only written
        // after PV_j (issued right below) completed.
        if (!mbar_wait(b_pfull(t, j & 1), (j >> 1) & 1, abort_flag)) break;
        const int st = j % KSV;
        if (!mbar_wait(b_vfull(t, st), (j / KSV) & 1, abort_flag)) break;
        tc_fence_after();
        const uint32_t pa = tmem + C::TM_P + (j & 1) * (BN / 2);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          const uint64_t bd = umma_desc_sw128(sV(t, st) + kk * 16 * 128, BN * 128, 1024);
          umma_bf16_ts(tmem + C::TM_O, pa + kk * 8, bd, idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(b_odone(t, j & 1));
        umma_commit(b_vempty(t, st));
        issued_any = true;
      }
    }
    // Every UMMA this thread issued has completed before TMEM is freed
    // (an item with no key blocks -- a key range past its tile's last --
    // issued none).
    if (issued_any) {
      const uint32_t b_drain = warp == 1 ? b_drain_s : b_drain_o;
      umma_commit(b_drain);
      volatile int never = 0;
      mbar_wait(b_drain, 0, &never, 1ll << 30);
    }
  } else if (warp >= 4 && warp < 4 + 4 * NT) {
    // ---------------- softmax / correction / epilogue of one tile ----------------
    const int t = (warp - 4) >> 2;
    const Work wk = decode_work(p, blockIdx.x * NT + t, BN);
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;
    const int tq = wk.t0 + r / p.group;
    const int h = r % p.group;
    const uint32_t tl = tmem + t * C::TM_TILE + ((uint32_t)(q4 * 32) << 16);
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    float s[BN];
    uint32_t pk[BN / 2];
    for (int j = 0; j < wk.n_blk; ++j) {
      // s_full cannot lead by two phases: S_{j+1} is only issued after this
      // thread released S_j through s_free.
      if (!__all_sync(0xffffffffu, mbar_wait(b_sfull(t), j & 1, abort_flag))) { ok = false; break; }
      tc_fence_after();
      const uint32_t sc = tl + C::TM_S;
#pragma unroll
      for (int c = 0; c < BN; c += 32) tmem_ld32(sc + c, s + c);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(b_sfree(t));
      // Key column c is visible if c <= lim: inside the prefix for a prefix
      // block, causal for an own block.  Full blocks skip the mask.  (j
      // counts this item's blocks; jg is the tile's block number.)
      const int jg = wk.jb + j;
      const int own_last = (wk.seg.flags & CEVK_SEG_BIDIRECTIONAL) ? wk.seg.q_len - 1 : tq;
      const int lim = (jg < wk.n_pre) ? wk.seg.prefix_len - jg * BN - 1 : own_last - (jg - wk.n_pre) * BN;
      if (lim < BN - 1) {
#pragma unroll
        for (int c = 0; c < BN; ++c) s[c] = (c <= lim) ? s[c] : -INFINITY;
      }
      // Row max of the raw scores (scale > 0 commutes with max): 8
      // independent chains of three-input max, then a tree.
      static_assert(BN % 16 == 0, "max chains take 16 columns a step");
      float mx[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) mx[i] = fmaxf(s[i], s[8 + i]);
#pragma unroll
      for (int c = 16; c < BN; c += 16)
#pragma unroll
        for (int i = 0; i < 8; ++i) mx[i] = fmax3(mx[i], s[c + i], s[c + 8 + i]);
      const float mb = fmax3(fmax3(mx[0], mx[1], mx[2]), fmax3(mx[3], mx[4], mx[5]), fmaxf(mx[6], mx[7])) *
                       p.scale_log2;
      // Rescale only when the running max grows by more than 2^8.
      const bool need = (j == 0) || (mb > m_run + 8.f);
      const float m_new = need ? mb : m_run;
      const float factor = (j > 0 && need) ? fast_exp2(m_run - m_new) : 1.f;
      // P = 2^(s*scale - m): one packed FFMA per two elements, one ex2
      // each; the row sum in four packed accumulator pairs.
      const float neg = -m_new, sl = p.scale_log2;
      float sm8[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) sm8[i] = 0.f;
#pragma unroll
      for (int c = 0; c < BN; c += 2) {
        float x0, x1;
        ffma2(x0, x1, s[c], s[c + 1], sl, sl, neg, neg);
        const float e0 = fast_exp2(x0), e1 = fast_exp2(x1);
        const int a = (c >> 1) & 3;
        fadd2(sm8[2 * a], sm8[2 * a + 1], sm8[2 * a], sm8[2 * a + 1], e0, e1);
        pk[c >> 1] = pack_bf16x2(e0, e1);
      }
      const float sum = ((sm8[0] + sm8[1]) + (sm8[2] + sm8[3])) + ((sm8[4] + sm8[5]) + (sm8[6] + sm8[7]));
      // P buffer j&1 is free: PV_{j-2} completed before S_j was committed
      // (the S issuer waits for it), and this thread observed s_full_j.
      if (__any_sync(0xffffffffu, factor != 1.f)) {
        // O is rescaled in TMEM: PV of the previous block must be done (and
        // PV of this block cannot start before P_j is signalled).
        if (!__all_sync(0xffffffffu, mbar_wait(b_odone(t, (j - 1) & 1), ((j - 1) >> 1) & 1, abort_flag))) { ok = false; break; }
        tc_fence_after();
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
      l_run = l_run * factor + sum;
      m_run = m_new;
      // Key rows past the tile's last visible key carry P = 0, but their V
      // rows are whatever the buffer holds there (possibly NaN/Inf, and
      // 0 * NaN = NaN in the MMA): zero them before PV reads the stage.
      {
        const int own_rows = (wk.seg.flags & CEVK_SEG_BIDIRECTIONAL) ? wk.seg.q_len : wk.t0 + wk.nt;
        const int vcount = (jg < wk.n_pre) ? wk.seg.prefix_len - jg * BN : own_rows - (jg - wk.n_pre) * BN;
        if (vcount < BN) {
          const int vst = j % KSV;
          if (!__all_sync(0xffffffffu, mbar_wait(b_vfull(t, vst), (j / KSV) & 1, abort_flag))) { ok = false; break; }
          const int rows0 = vcount < 0 ? 0 : vcount;
          const int chunks = (BN - rows0) * 8 * (D / 64);
          uint8_t* vb = smem + t * C::T_BYTES + C::T_OFF_V + vst * C::KV_BYTES;
          for (int i = q4 * 32 + lane; i < chunks; i += 128) {
            const int a = i / ((BN - rows0) * 8), rem = i % ((BN - rows0) * 8);
            *reinterpret_cast<uint4*>(vb + a * BN * 128 + (rows0 + rem / 8) * 128 + (rem % 8) * 16) = make_uint4(0, 0, 0, 0);
          }
          fence_proxy_async_smem();
        }
      }
      // P_j into its TMEM buffer, packed bf16x2.
#pragma unroll
      for (int c = 0; c < BN / 2; c += 32)
        tmem_st32(tl + C::TM_P + (j & 1) * (BN / 2) + c, reinterpret_cast<const float*>(pk + c));
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(b_pfull(t, j & 1));
    }
    // PV of the last block completed (its commit covers every earlier UMMA).
    if (ok && wk.n_blk > 0 &&
        mbar_wait(b_odone(t, (wk.n_blk - 1) & 1), ((wk.n_blk - 1) >> 1) & 1, abort_flag)) {
      tc_fence_after();
      const float inv = 1.f / l_run;
      const bool store = (tq < wk.seg.q_len) && (r / p.group < wk.nt);
      const size_t orow = (size_t)(wk.seg.q_start + tq) * p.o_row_stride + (size_t)(wk.kvh * p.group + h) * D;
      float* prow = p.part_o + ((size_t)wk.item * 128 + r) * D;
      if (wk.n_eff > 1 && store) p.part_lse[(size_t)wk.item * 128 + r] = m_run + log2f(l_run);
#pragma unroll 1
      for (int c = 0; c < D; c += 32) {
        float o[32];
        tmem_ld32(tl + C::TM_O + c, o);
        tmem_wait_ld();
        if (store && wk.n_eff > 1) {
#pragma unroll
          for (int i = 0; i < 32; i += 4)
            *reinterpret_cast<float4*>(prow + c + i) =
                make_float4(o[i] * inv, o[i + 1] * inv, o[i + 2] * inv, o[i + 3] * inv);
        } else if (store) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            uint4 pv;
            pv.x = pack_bf16x2(o[i] * inv, o[i + 1] * inv);
            pv.y = pack_bf16x2(o[i + 2] * inv, o[i + 3] * inv);
            pv.z = pack_bf16x2(o[i + 4] * inv, o[i + 5] * inv);
            pv.w = pack_bf16x2(o[i + 6] * inv, o[i + 7] * inv);
            for (int d = 0; d < p.n_o; ++d) *reinterpret_cast<uint4*>(p.o[d] + orow + c + i) = pv;
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

// Merges the key ranges of split tiles: o = sum_s 2^(lse_s - m) o_s /
// sum_s 2^(lse_s - m), m = max_s lse_s, per row; one block of 128 threads
// per (work tile, group of 1024 / D rows), 8 columns per thread.
template <int D, int BN>
__global__ void __launch_bounds__(128) attn_combine_kernel(AttnParams p) {
  const Work wk = decode_work(p, blockIdx.x * p.n_split, BN);
  if (wk.n_eff <= 1) return;
  constexpr int CH = D / 8;
  const int r = blockIdx.y * (128 / CH) + threadIdx.x / CH;
  const int c = (threadIdx.x % CH) * 8;
  const int tq = wk.t0 + r / p.group, h = r % p.group;
  if (!(tq < wk.seg.q_len && r / p.group < wk.nt)) return;
  const size_t it0 = (size_t)blockIdx.x * p.n_split;
  float m = -INFINITY;
  for (int s = 0; s < wk.n_eff; ++s) m = fmaxf(m, p.part_lse[(it0 + s) * 128 + r]);
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f}, wsum = 0.f;
  for (int s = 0; s < wk.n_eff; ++s) {
    const float wt = exp2f(p.part_lse[(it0 + s) * 128 + r] - m);
    const float4* src = reinterpret_cast<const float4*>(p.part_o + ((it0 + s) * 128 + r) * D + c);
    const float4 a = src[0], b = src[1];
    wsum += wt;
    acc[0] += wt * a.x; acc[1] += wt * a.y; acc[2] += wt * a.z; acc[3] += wt * a.w;
    acc[4] += wt * b.x; acc[5] += wt * b.y; acc[6] += wt * b.z; acc[7] += wt * b.w;
  }
  const float inv = 1.f / wsum;
  uint4 pv;
  pv.x = pack_bf16x2(acc[0] * inv, acc[1] * inv);
  pv.y = pack_bf16x2(acc[2] * inv, acc[3] * inv);
  pv.z = pack_bf16x2(acc[4] * inv, acc[5] * inv);
  pv.w = pack_bf16x2(acc[6] * inv, acc[7] * inv);
  const size_t orow = (size_t)(wk.seg.q_start + tq) * p.o_row_stride + (size_t)(wk.kvh * p.group + h) * D + c;
  for (int d = 0; d < p.n_o; ++d) *reinterpret_cast<uint4*>(p.o[d] + orow) = pv;
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

template <int D, int BN, int KSK, int KSV, int NT>
static int launch_tc(const void* q, const void* k, const void* v, void* const* o, int n_o, int n_tokens, int n_kv_rows,
                     int hq, int hkv,
                     int q_rs, int kv_rs, int o_rs, const cevk_segment* segs, int n_segs, int n_tiles, float scale,
                     int n_split, void* workspace, cudaStream_t stream) {
  using C = AttnTc<D, BN, KSK, KSV, NT>;
  const int group = hq / hkv, rows_t = 128 / group;
  CUtensorMap tq, tk, tv;
  int rc;
  if ((rc = make_map(&tq, q, D, hq, n_tokens, q_rs, group, rows_t))) return rc;
  if ((rc = make_map(&tk, k, D, hkv, n_kv_rows, kv_rs, 1, BN))) return rc;
  if ((rc = make_map(&tv, v, D, hkv, n_kv_rows, kv_rs, 1, BN))) return rc;
  if ((rc = opt_in_smem((const void*)attn_tc_kernel<D, BN, KSK, KSV, NT>, C::SMEM, "attn_tc_kernel"))) return rc;
  AttnParams prm;
  if (n_o < 1 || n_o > kMaxOut) return set_error(CEVK_E_SHAPE, "attention: %d output buffers (1..%d)", n_o, kMaxOut);
  for (int d = 0; d < kMaxOut; ++d) prm.o[d] = d < n_o ? reinterpret_cast<__nv_bfloat16*>(o[d]) : nullptr;
  prm.n_o = n_o;
  prm.segs = segs;
  prm.n_segs = n_segs;
  prm.n_work = n_tiles * hkv;
  prm.n_split = n_split;
  prm.part_o = reinterpret_cast<float*>(workspace);
  prm.part_lse = prm.part_o + (size_t)prm.n_work * n_split * 128 * D;
  prm.hq = hq;
  prm.hkv = hkv;
  prm.group = group;
  prm.rows_t = rows_t;
  prm.o_row_stride = o_rs;
  prm.scale_log2 = scale * 1.4426950408889634f;
  const unsigned grid = (unsigned)((prm.n_work * n_split + NT - 1) / NT);
  attn_tc_kernel<D, BN, KSK, KSV, NT><<<grid, C::THREADS, C::SMEM, stream>>>(tq, tk, tv, prm);
  const int rc2 = check_launch("attn_tc_kernel");
  if (rc2 || n_split == 1) return rc2;
  attn_combine_kernel<D, BN><<<dim3((unsigned)prm.n_work, D / 8), 128, 0, stream>>>(prm);
  return check_launch("attn_combine_kernel");
}

int attn_tc_launch(const void* q, const void* k, const void* v, void* const* o, int n_o, int n_tokens, int n_kv_rows,
                   int hq, int hkv, int D, int q_rs, int kv_rs, int o_rs, const cevk_segment* segs, int n_segs,
                   int n_tiles, float scale, int n_split, void* workspace, cudaStream_t stream) {
  // head_dim 64 / 128: two CTAs per SM; 256: one (its O takes 256 TMEM columns)
#define CEVK_ATTN(DD, KSK, KSV)                                                                                    \
  return launch_tc<DD, 64, KSK, KSV, 1>(q, k, v, o, n_o, n_tokens, n_kv_rows, hq, hkv, q_rs, kv_rs, o_rs, segs, \
                                        n_segs, n_tiles, scale, n_split, workspace, stream)
  switch (D) {
    case 64: CEVK_ATTN(64, 6, 4);
    case 128: CEVK_ATTN(128, 3, 2);
    case 256: CEVK_ATTN(256, 3, 2);
    default: return set_error(CEVK_E_SHAPE, "bf16 attention supports head_dim 64, 128, 256 (got %d)", D);
  }
#undef CEVK_ATTN
}

}  // namespace cevk
