// Gated DeltaNet chunked prefill (qwen35.rs:301-368 and the prologue /
// epilogue of GatedDeltaNet::forward, qwen35.rs:419-451), all arithmetic in
// f32 like the reference.
//
// Kernel 1, gdn_chunk_kernel: one CTA per (row b, value head h, slice of 32
// value columns).  The columns of the recurrent state S (dk x dv), of v_new
// and of the output are independent, so a head's sequential scan over its
// 64-token chunks is split over dv/32 CTAs (128 CTAs for one 32-head row).
// Per chunk, in shared memory:
//   q, k <- l2norm (q * dk^-1/2), beta = sigmoid(b), g = -exp(A_log) *
//   softplus(a + dt_bias), cum = cumsum(g);
//   A = strict_lower((k*beta) k^T o exp(cum_i - cum_j)), T = (I + A)^-1
//   (column-wise forward substitution -- the same inverse the reference
//   builds by recursive block inversion, qwen35.rs:266-296);
//   U = T (v*beta), W = T (k*beta*exp(cum)), intra = lower(q k^T o decay);
//   v_new = U - W S;  out = (q*exp(cum)) S + intra v_new;
//   S = S*exp(cum_last) + (k*exp(cum_last - cum))^T v_new.
// The raw f32 output goes to the caller's workspace.
// Kernel 2, gdn_gated_norm_kernel: y = rmsnorm(out) * w * silu(z) per head,
// cast to the model dtype (qwen35.rs:446-451).
#include "common.cuh"

namespace cevk {

constexpr int GC = 64;    // chunk length (qwen35.rs:302)
constexpr int GDVS = 32;  // value columns per CTA

struct GdnParams {
  const void* conv;  // [B, T, Cc]
  int Cc;
  const void* ab;  // per token: b (nv) | a (nv)
  int ab_rs;
  const float* a_log;
  const float* dt_bias;
  const float* s_in;
  long long s_bs;
  float* s_out;
  float* core;  // [B, T, nv, dv] f32 workspace
  int B, T, nk, nv, dk, dv;
};

template <typename T>
__global__ void __launch_bounds__(256, 1) gdn_chunk_kernel(GdnParams p) {
  extern __shared__ float sm[];
  const int dk = p.dk, dv = p.dv;
  const int KP = dk + 1;  // padded row pitch (conflict-free column walks)
  float* sQ = sm;                 // [GC][KP]
  float* sK = sQ + GC * KP;       // [GC][KP]
  float* sW = sK + GC * KP;       // [GC][KP]
  float* sA = sW + GC * KP;       // [GC][GC+1]  A, then T = (I+A)^-1
  float* sI = sA + GC * (GC + 1); // [GC][GC+1]  intra
  float* sV = sI + GC * (GC + 1); // [GC][GDVS]  v*beta -> U -> v_new
  float* sS = sV + GC * GDVS;     // [dk][GDVS]
  float* sG = sS + dk * GDVS;     // cum [GC]
  float* sB = sG + GC;            // beta [GC]
  float* sE = sB + GC;            // beta * exp(cum) [GC]
  const int AP = GC + 1;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int slices = dv / GDVS;
  const int sl = blockIdx.x % slices;
  const int h = blockIdx.x / slices;
  const int b = blockIdx.y;
  const int kh = h / (p.nv / p.nk);  // k-head repeat nk -> nv (qwen35.rs:436-441)
  const int c0 = sl * GDVS;
  const T* conv = reinterpret_cast<const T*>(p.conv);
  const T* ab = reinterpret_cast<const T*>(p.ab);
  const int key_dim = p.nk * dk;
  const float qscale = rsqrtf((float)dk);
  const float neg_a = -expf(p.a_log[h]);
  const float dtb = p.dt_bias[h];

  // initial state slice
  for (int i = tid; i < dk * GDVS; i += 256) {
    const int d = i / GDVS, c = i % GDVS;
    sS[i] = p.s_in ? p.s_in[b * p.s_bs + ((long long)h * dk + d) * dv + c0 + c] : 0.f;
  }

  const int n_chunks = (p.T + GC - 1) / GC;
  for (int ch = 0; ch < n_chunks; ++ch) {
    const int t0 = ch * GC;
    __syncthreads();
    // ---- load q, k (full dk), v slice; gates ----
    for (int i = tid; i < GC * dk; i += 256) {
      const int r = i / dk, d = i % dk;
      const int t = t0 + r;
      float qv = 0.f, kv = 0.f;
      if (t < p.T) {
        const T* row = conv + ((long long)b * p.T + t) * p.Cc;
        qv = to_f(row[kh * dk + d]);
        kv = to_f(row[key_dim + kh * dk + d]);
      }
      sQ[r * KP + d] = qv;
      sK[r * KP + d] = kv;
    }
    if (tid < GC) {
      const int t = t0 + tid;
      float beta = 0.f, g = 0.f;
      if (t < p.T) {
        const T* row = ab + ((long long)b * p.T + t) * p.ab_rs;
        beta = 1.f / (1.f + expf(-to_f(row[h])));
        const float x = to_f(row[p.nv + h]) + dtb;
        // softplus(x) = max(x, 0) + ln(1 + e^{-|x|}) (qwen35.rs:243-248)
        g = (fmaxf(x, 0.f) + logf(1.f + expf(-fabsf(x)))) * neg_a;
      }
      sB[tid] = beta;
      sG[tid] = g;
    }
    __syncthreads();
    if (tid == 0) {
      float acc = 0.f;
      for (int r = 0; r < GC; ++r) { acc += sG[r]; sG[r] = acc; }
    }
    for (int i = tid; i < GC * GDVS; i += 256) {
      const int r = i / GDVS, c = i % GDVS;
      const int t = t0 + r;
      float vv = 0.f;
      if (t < p.T) vv = to_f(conv[((long long)b * p.T + t) * p.Cc + 2 * key_dim + h * dv + c0 + c]);
      sV[i] = vv * sB[r];
    }
    // l2norm rows of q (then * dk^-1/2) and k: one warp per row
    for (int r = warp; r < 2 * GC; r += 8) {
      float* row = r < GC ? sQ + r * KP : sK + (r - GC) * KP;
      float ss = 0.f;
      for (int d = lane; d < dk; d += 32) ss += row[d] * row[d];
      ss = warp_sum(ss);
      const float inv = 1.f / sqrtf(ss + 1e-6f);
      const float sc = r < GC ? inv * qscale : inv;
      for (int d = lane; d < dk; d += 32) row[d] *= sc;
    }
    __syncthreads();
    // ---- A (strict lower, with beta_i) and intra (lower incl. diagonal) ----
    for (int idx = tid; idx < GC * GC; idx += 256) {
      const int i = idx / GC, j = idx % GC;
      float a = 0.f, q = 0.f;
      if (j <= i) {
        const float* ki = sK + i * KP;
        const float* kj = sK + j * KP;
        const float* qi = sQ + i * KP;
        float dkk = 0.f, dqk = 0.f;
        for (int d = 0; d < dk; ++d) {
          dkk += ki[d] * kj[d];
          dqk += qi[d] * kj[d];
        }
        const float dec = expf(sG[i] - sG[j]);
        q = dqk * dec;
        if (j < i) a = sB[i] * dkk * dec;
      }
      sA[i * AP + j] = a;
      sI[i * AP + j] = q;
    }
    if (tid < GC) sE[tid] = sB[tid] * expf(sG[tid]);
    __syncthreads();
    // ---- T = (I + A)^-1: column c by forward substitution ----
    if (tid < GC) {
      const int c = tid;
      for (int i = 0; i < GC; ++i) {
        float x = 0.f;
        if (i == c) x = 1.f;
        else if (i > c) {
          float acc = 0.f;
          for (int j = c; j < i; ++j) acc += sA[i * AP + j] * sW[j * KP + c];  // sW column c holds T[:, c]
          x = -acc;
        }
        sW[i * KP + c] = x;
      }
    }
    __syncthreads();
    for (int idx = tid; idx < GC * GC; idx += 256) {
      const int i = idx / GC, j = idx % GC;
      sA[i * AP + j] = sW[i * KP + j];
    }
    __syncthreads();
    // ---- U = T (v beta) (into sV via registers), W = T (k beta e^cum) ----
    {
      float u[GC * GDVS / 256];
#pragma unroll
      for (int r = 0; r < GC * GDVS / 256; ++r) {
        const int i = warp + 8 * r, c = lane;
        float acc = 0.f;
        for (int j = 0; j <= i; ++j) acc += sA[i * AP + j] * sV[j * GDVS + c];
        u[r] = acc;
      }
      for (int idx = tid; idx < GC * dk; idx += 256) {
        const int i = idx / dk, d = idx % dk;
        float acc = 0.f;
        for (int j = 0; j <= i; ++j) acc += sA[i * AP + j] * (sK[j * KP + d] * sE[j]);
        sW[i * KP + d] = acc;
      }
      __syncthreads();
#pragma unroll
      for (int r = 0; r < GC * GDVS / 256; ++r) sV[(warp + 8 * r) * GDVS + lane] = u[r];
    }
    // q <- q e^cum, k <- k e^(cum_last - cum)
    const float last = sG[GC - 1];
    for (int i = tid; i < GC * dk; i += 256) {
      const int r = i / dk, d = i % dk;
      sQ[r * KP + d] *= expf(sG[r]);
      sK[r * KP + d] *= expf(last - sG[r]);
    }
    __syncthreads();
    // ---- v_new = U - W S ----
    {
      float vn[GC * GDVS / 256];
#pragma unroll
      for (int r = 0; r < GC * GDVS / 256; ++r) {
        const int i = warp + 8 * r, c = lane;
        float acc = 0.f;
        for (int d = 0; d < dk; ++d) acc += sW[i * KP + d] * sS[d * GDVS + c];
        vn[r] = sV[i * GDVS + c] - acc;
      }
      __syncthreads();
#pragma unroll
      for (int r = 0; r < GC * GDVS / 256; ++r) sV[(warp + 8 * r) * GDVS + lane] = vn[r];
    }
    __syncthreads();
    // ---- out = (q e^cum) S + intra v_new ----
#pragma unroll
    for (int r = 0; r < GC * GDVS / 256; ++r) {
      const int i = warp + 8 * r, c = lane;
      float acc = 0.f;
      for (int d = 0; d < dk; ++d) acc += sQ[i * KP + d] * sS[d * GDVS + c];
      float acc2 = 0.f;
      for (int j = 0; j <= i; ++j) acc2 += sI[i * AP + j] * sV[j * GDVS + c];
      const int t = t0 + i;
      if (t < p.T) p.core[(((long long)b * p.T + t) * p.nv + h) * dv + c0 + c] = acc + acc2;
    }
    __syncthreads();
    // ---- S = S e^last + (k e^(last-cum))^T v_new ----
    const float el = expf(last);
    for (int idx = tid; idx < dk * GDVS; idx += 256) {
      const int d = idx / GDVS, c = idx % GDVS;
      float acc = 0.f;
      for (int j = 0; j < GC; ++j) acc += sK[j * KP + d] * sV[j * GDVS + c];
      sS[idx] = sS[idx] * el + acc;
    }
  }
  __syncthreads();
  if (p.s_out)
    for (int i = tid; i < dk * GDVS; i += 256) {
      const int d = i / GDVS, c = i % GDVS;
      p.s_out[(long long)b * p.nv * dk * dv + ((long long)h * dk + d) * dv + c0 + c] = sS[i];
    }
}

// N consecutive 32-bit words in one or two vector accesses (N = 1, 2, 4, 8).
template <int N>
__device__ __forceinline__ void ldw(const void* p, uint32_t* w) {
  if constexpr (N == 1) {
    w[0] = *reinterpret_cast<const uint32_t*>(p);
  } else if constexpr (N == 2) {
    const uint2 v = *reinterpret_cast<const uint2*>(p);
    w[0] = v.x; w[1] = v.y;
  } else {
#pragma unroll
    for (int i = 0; i < N / 4; ++i) {
      const uint4 v = reinterpret_cast<const uint4*>(p)[i];
      w[4 * i] = v.x; w[4 * i + 1] = v.y; w[4 * i + 2] = v.z; w[4 * i + 3] = v.w;
    }
  }
}
template <int N>
__device__ __forceinline__ void stw(void* p, const uint32_t* w) {
  if constexpr (N == 1) {
    *reinterpret_cast<uint32_t*>(p) = w[0];
  } else if constexpr (N == 2) {
    *reinterpret_cast<uint2*>(p) = make_uint2(w[0], w[1]);
  } else {
#pragma unroll
    for (int i = 0; i < N / 4; ++i)
      reinterpret_cast<uint4*>(p)[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
  }
}

// y = rmsnorm(o) * w * silu(z) per (token, head): one warp per row of dv =
// 32 * E values, E consecutive values per lane, every load issued first.
template <typename T, int E>
__global__ void __launch_bounds__(256) gdn_gated_norm_kernel(const float* __restrict__ core, const T* __restrict__ z,
                                                             int z_rs, const T* __restrict__ w, float eps,
                                                             T* __restrict__ y, long long rows, int nv, int dv) {
  constexpr int WT = E * (int)sizeof(T) / 4;  // 32-bit words of E model-dtype values
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long job = (long long)blockIdx.x * (blockDim.x >> 5) + warp;  // (b*T + t) * nv + h
  if (job >= rows * nv) return;
  const long long bt = job / nv;
  const int h = (int)(job % nv);
  uint32_t ow[E], zw[WT], ww[WT];
  ldw<E>(core + job * dv + lane * E, ow);
  ldw<WT>(z + bt * z_rs + (long long)h * dv + lane * E, zw);
  ldw<WT>(w + lane * E, ww);
  const float* o = reinterpret_cast<const float*>(ow);
  const T* zz = reinterpret_cast<const T*>(zw);
  const T* wv = reinterpret_cast<const T*>(ww);
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < E; ++i) ss += o[i] * o[i];
  ss = warp_sum(ss);
  const float r = 1.f / sqrtf(ss / dv + eps);
  T out[E];
#pragma unroll
  for (int i = 0; i < E; ++i) {
    const float zf = to_f(zz[i]);
    out[i] = from_f<T>(o[i] * r * to_f(wv[i]) * (zf / (1.f + expf(-zf))));
  }
  stw<WT>(y + bt * (long long)nv * dv + (long long)h * dv + lane * E, reinterpret_cast<const uint32_t*>(out));
}

template <typename T>
static void launch_gated_norm(const float* core, const T* z, int z_rs, const T* w, float eps, T* y, long long rows,
                              int nv, int dv, cudaStream_t st) {
  const unsigned ng = (unsigned)((rows * nv + 7) / 8);
  switch (dv) {
    case 64: gdn_gated_norm_kernel<T, 2><<<ng, 256, 0, st>>>(core, z, z_rs, w, eps, y, rows, nv, dv); break;
    case 128: gdn_gated_norm_kernel<T, 4><<<ng, 256, 0, st>>>(core, z, z_rs, w, eps, y, rows, nv, dv); break;
    default: gdn_gated_norm_kernel<T, 8><<<ng, 256, 0, st>>>(core, z, z_rs, w, eps, y, rows, nv, dv); break;
  }
}

// The bf16 gated norm of rows [t0, t0 + rows) of a single-row call (the
// pieces of gdn_umma.cu launch it piece by piece on their own stream).
void gdn_gated_norm_rows_bf16(const float* core, const void* z, int z_rs, const void* w, float eps, void* y,
                              long long t0, long long rows, int nv, int dv, cudaStream_t st) {
  launch_gated_norm<__nv_bfloat16>(core + t0 * nv * dv, reinterpret_cast<const __nv_bfloat16*>(z) + t0 * z_rs, z_rs,
                                   reinterpret_cast<const __nv_bfloat16*>(w), eps,
                                   reinterpret_cast<__nv_bfloat16*>(y) + t0 * nv * dv, rows, nv, dv, st);
}

static size_t gdn_smem(int dk) {
  const int KP = dk + 1;
  return sizeof(float) * (3 * GC * KP + 2 * GC * (GC + 1) + GC * GDVS + dk * GDVS + 3 * GC);
}

size_t gdn_tc_extra_floats(int B, int T, int nv, int dk, int dv);
bool gdn_tc_supported(int dk, int dv);
size_t gdn_umma_extra_floats(int B, int T, int nv);
int gdn_umma_run(const void* conv_out, int C_, const void* ab, int ab_rs, const float* a_log, const float* dt_bias,
                 const float* s_in, long long s_bs, float* s_out, float* workspace, int B, int T, int nk, int nv,
                 const void* z, int z_rs, const void* norm_w, float eps, void* y, cudaStream_t st);
int gdn_tc_run(const void* conv_out, int C_, const void* ab, int ab_rs, const float* a_log, const float* dt_bias,
               const float* s_in, long long s_bs, float* s_out, float* workspace, int B, int T, int nk, int nv, int dk,
               int dv, cudaStream_t st);

}  // namespace cevk

using namespace cevk;

extern "C" {

size_t cevk_gdn_workspace_size(int32_t B, int32_t T, int32_t nv, int32_t dk, int32_t dv) {
  // core output [B, T, nv, dv] f32, then (bf16 tensor-core paths) the
  // per-chunk operands of the scan: the tcgen05 kernels' records
  // (gdn_umma.cu, dk = dv = 128, plus 16 bytes of alignment slack) or the
  // W, q', k', U, intra and e^last of gdn_tc.cu (dk = dv = 64).
  const size_t extra = dk == 128 && dv == 128 ? gdn_umma_extra_floats(B, T, nv) + 4
                                              : gdn_tc_extra_floats(B, T, nv, dk, dv);
  return ((size_t)B * T * nv * dv + extra) * sizeof(float);
}

int cevk_gdn_chunk_prefill(const void* conv_out, int32_t C, const void* ab, int32_t ab_row_stride, const void* z,
                           int32_t z_row_stride, const float* a_log, const float* dt_bias, const void* norm_w,
                           float eps, const float* s_in, int64_t s_batch_stride, float* s_out, void* y, int32_t B,
                           int32_t T, int32_t nk, int32_t nv, int32_t dk, int32_t dv, void* workspace,
                           size_t workspace_bytes, int32_t dtype, void* stream) {
  if (!conv_out || !ab || !z || !a_log || !dt_bias || !norm_w || !y)
    return set_error(CEVK_E_SHAPE, "gdn: null pointer");
  if (nk <= 0 || nv % nk || dk % 32 || dk < 64 || dk > 128 || (dv != 64 && dv != 128 && dv != 256))
    return set_error(CEVK_E_SHAPE, "gdn: heads %d/%d, dk %d, dv %d unsupported", nk, nv, dk, dv);
  {
    // the gated norm reads dv/32 consecutive z / norm_w values per lane
    const size_t vb = (size_t)(dv / 32) * (dtype == CEVK_BF16 ? 2 : 4);
    if (((uintptr_t)z | (uintptr_t)norm_w | (uintptr_t)y) % vb || (z_row_stride * (dtype == CEVK_BF16 ? 2 : 4)) % vb)
      return set_error(CEVK_E_SHAPE, "gdn: z, norm_w, y and the z row stride must be %zu-byte aligned", vb);
  }
  if (C != 2 * nk * dk + nv * dv) return set_error(CEVK_E_SHAPE, "gdn: C %d != 2*nk*dk + nv*dv", C);
  if (B <= 0 || T <= 0) return CEVK_OK;
  // A workspace of cevk_gdn_workspace_size() bytes runs bf16 on the tensor
  // cores; one that holds only the f32 core output runs the SIMT kernel.
  const size_t need_core = (size_t)B * T * nv * dv * sizeof(float);
  if (!workspace || workspace_bytes < need_core)
    return set_error(CEVK_E_SHAPE, "gdn: workspace of %zu bytes needed (got %zu)",
                     cevk_gdn_workspace_size(B, T, nv, dk, dv), workspace_bytes);
  const bool full_ws = workspace_bytes >= cevk_gdn_workspace_size(B, T, nv, dk, dv);
  GdnParams prm;
  prm.conv = conv_out;
  prm.Cc = C;
  prm.ab = ab;
  prm.ab_rs = ab_row_stride;
  prm.a_log = a_log;
  prm.dt_bias = dt_bias;
  prm.s_in = s_in;
  prm.s_bs = s_batch_stride;
  prm.s_out = s_out;
  prm.core = reinterpret_cast<float*>(workspace);
  prm.B = B;
  prm.T = T;
  prm.nk = nk;
  prm.nv = nv;
  prm.dk = dk;
  prm.dv = dv;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const size_t smem = gdn_smem(dk);
  dim3 grid(nv * (dv / GDVS), B);
  const long long rows = (long long)B * T;
  const unsigned ng = (unsigned)((rows * nv + 7) / 8);
  if (dtype == CEVK_BF16) {
    int rc;
    const bool aligned = ((uintptr_t)conv_out & 15) == 0 && C % 8 == 0 && ((uintptr_t)workspace & 15) == 0;
    if (full_ws && aligned && dk == 128 && dv == 128) {
      // tcgen05 UMMA with TMEM accumulators (gdn_umma.cu): chunk-parallel
      // prep + state scan
      // prep + state scan, and the gated norm
      rc = gdn_umma_run(conv_out, C, ab, ab_row_stride, a_log, dt_bias, s_in, s_batch_stride, s_out, prm.core, B, T,
                        nk, nv, z, z_row_stride, norm_w, eps, y, st);
      return rc ? rc : check_launch("gdn_gated_norm_kernel");
    } else if (full_ws && aligned && gdn_tc_supported(dk, dv)) {
      // mma.sync (gdn_tc.cu), dk = dv = 64
      rc = gdn_tc_run(conv_out, C, ab, ab_row_stride, a_log, dt_bias, s_in, s_batch_stride, s_out, prm.core, B, T,
                      nk, nv, dk, dv, st);
    } else {
      if ((rc = opt_in_smem((const void*)gdn_chunk_kernel<__nv_bfloat16>, (int)smem, "gdn_chunk_kernel"))) return rc;
      gdn_chunk_kernel<__nv_bfloat16><<<grid, 256, smem, st>>>(prm);
      rc = check_launch("gdn_chunk_kernel");
    }
    if (rc) return rc;
    launch_gated_norm<__nv_bfloat16>(prm.core, (const __nv_bfloat16*)z, z_row_stride, (const __nv_bfloat16*)norm_w,
                                     eps, (__nv_bfloat16*)y, rows, nv, dv, st);
  } else if (dtype == CEVK_F32) {
    int rc = opt_in_smem((const void*)gdn_chunk_kernel<float>, (int)smem, "gdn_chunk_kernel");
    if (rc) return rc;
    gdn_chunk_kernel<float><<<grid, 256, smem, st>>>(prm);
    rc = check_launch("gdn_chunk_kernel");
    if (rc) return rc;
    launch_gated_norm<float>(prm.core, (const float*)z, z_row_stride, (const float*)norm_w, eps, (float*)y, rows, nv,
                             dv, st);
  } else {
    return set_error(CEVK_E_UNSUPPORTED, "gdn: dtype %d", dtype);
  }
  return check_launch("gdn_gated_norm_kernel");
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free variant of cevk_gdn_chunk_prefill.
//
// Some hosts cannot hand this library a workspace: their device memory is
// owned by a fixed pool of their own (an embedding runtime that only gives
// out its tensors), or they run the decision forward on a path where a
// cudaMalloc is not allowed or would stall it.  For them the f32 scratch of
// the chunked delta rule lives in a fixed device array in this file.  Every
// GPU that loads the library holds the array until the process exits.
// ---------------------------------------------------------------------------
#include <mutex>

namespace cevk {

constexpr size_t kGdnStaticScratchBytes = CEVK_GDN_NOALLOC_MAX_BYTES;
static __device__ __align__(256) float g_gdn_scratch[kGdnStaticScratchBytes / sizeof(float)];

// Device address of g_gdn_scratch for the current device, looked up once per
// device (the host-side name is only a stand-in, not a device address).
static int gdn_static_scratch(float** out) {
  static std::mutex mu;
  static float* addr[128] = {nullptr};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(CEVK_E_CUDA, "gdn noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 128) return set_error(CEVK_E_CUDA, "gdn noalloc: device ordinal %d", dev);
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_gdn_scratch);
    if (e != cudaSuccess || !p)
      return set_error(CEVK_E_CUDA, "gdn noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    addr[dev] = static_cast<float*>(p);
  }
  *out = addr[dev];
  return CEVK_OK;
}

}  // namespace cevk

extern "C" int cevk_gdn_chunk_prefill_noalloc(const void* conv_out, int32_t C, const void* ab, int32_t ab_row_stride,
                                              const void* z, int32_t z_row_stride, const float* a_log,
                                              const float* dt_bias, const void* norm_w, float eps, const float* s_in,
                                              int64_t s_batch_stride, float* s_out, void* y, int32_t B, int32_t T,
                                              int32_t nk, int32_t nv, int32_t dk, int32_t dv, int32_t dtype,
                                              void* stream) {
  if (B <= 0 || T <= 0) return CEVK_OK;
  // The array runs the tensor-core path when its scratch fits, else the SIMT
  // kernel, whose scratch is the f32 core output alone.
  const size_t need = (size_t)B * T * nv * dv * sizeof(float);
  if (need > cevk::kGdnStaticScratchBytes)
    return cevk::set_error(CEVK_E_SHAPE,
                           "gdn noalloc: %d rows x %d tokens x %d heads x %d columns need %zu bytes of scratch, "
                           "over the %zu-byte static array; split the call or use cevk_gdn_chunk_prefill",
                           B, T, nv, dv, need, cevk::kGdnStaticScratchBytes);
  float* ws = nullptr;
  const int rc = cevk::gdn_static_scratch(&ws);
  if (rc) return rc;
  return cevk_gdn_chunk_prefill(conv_out, C, ab, ab_row_stride, z, z_row_stride, a_log, dt_bias, norm_w, eps, s_in,
                                s_batch_stride, s_out, y, B, T, nk, nv, dk, dv, ws, cevk::kGdnStaticScratchBytes, dtype,
                                stream);
}
