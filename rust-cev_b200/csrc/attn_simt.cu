// Packed block-masked attention on CUDA cores for f32 runs (the exact
// parity path of the reference's f32 pipeline).  One warp per (token, query head);
// lanes split the head dimension; online softmax over the segment's visible
// keys (prefix range in full, own rows causally or -- bidirectional segments
// -- in full).  Same segment descriptors
// and the same semantics as attn_tc.cu.
#include "common.cuh"

namespace cevk {

template <typename T, int PER>
__global__ void __launch_bounds__(128) attn_simt_kernel(const T* __restrict__ q, const T* __restrict__ k,
                                                        const T* __restrict__ v, T* __restrict__ o,
                                                        const cevk_segment* __restrict__ segs, int hq, int hkv,
                                                        int D, int q_rs, int kv_rs, int o_rs, float scale) {
  const cevk_segment seg = segs[blockIdx.x];
  const int h = blockIdx.y;
  const int kvh = h / (hq / hkv);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int t = blockIdx.z * 4 + warp; t < seg.q_len; t += gridDim.z * 4) {
    const T* qr = q + (size_t)(seg.q_start + t) * q_rs + (size_t)h * D;
    float qv[PER], acc[PER];
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int d = lane + 32 * i;
      qv[i] = d < D ? to_f(qr[d]) : 0.f;
      acc[i] = 0.f;
    }
    float m = -INFINITY, l = 0.f;
    auto visit = [&](int row) {
      const T* kr = k + (size_t)row * kv_rs + (size_t)kvh * D;
      const T* vr = v + (size_t)row * kv_rs + (size_t)kvh * D;
      float dot = 0.f;
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        const int d = lane + 32 * i;
        if (d < D) dot += qv[i] * to_f(kr[d]);
      }
      const float s = warp_sum(dot) * scale;
      const float mn = fmaxf(m, s);
      const float corr = expf(m - mn);
      const float pexp = expf(s - mn);
      l = l * corr + pexp;
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        const int d = lane + 32 * i;
        acc[i] = acc[i] * corr + (d < D ? pexp * to_f(vr[d]) : 0.f);
      }
      m = mn;
    };
    for (int j = 0; j < seg.prefix_len; ++j) visit(seg.prefix_off + j);
    const int own = (seg.flags & CEVK_SEG_BIDIRECTIONAL) ? seg.q_len : t + 1;
    for (int j = 0; j < own; ++j) visit(seg.self_off + j);
    T* orow = o + (size_t)(seg.q_start + t) * o_rs + (size_t)h * D;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int d = lane + 32 * i;
      if (d < D) orow[d] = from_f<T>(acc[i] / l);
    }
  }
}

int attn_simt_launch(const void* q, const void* k, const void* v, void* o, int hq, int hkv, int D, int q_rs, int kv_rs,
                     int o_rs, const cevk_segment* segs, int n_segs, float scale, cudaStream_t stream) {
  if (D > 256 || D % 32 != 0) return set_error(CEVK_E_SHAPE, "f32 attention: head_dim %d unsupported", D);
  dim3 grid(n_segs, hq, 8);
  attn_simt_kernel<float, 8><<<grid, 128, 0, stream>>>((const float*)q, (const float*)k, (const float*)v, (float*)o,
                                                        segs, hq, hkv, D, q_rs, kv_rs, o_rs, scale);
  return check_launch("attn_simt_kernel");
}

}  // namespace cevk
