// Served debiased probabilities on the device (run_debiased's answer math,
// service.rs:288-348, with math::{softmax, log_softmax}, math.rs:7-18).
//
// Per question: the mean over its rotation variants of log_softmax(z_v) at
// each display position, minus log_softmax of the variant's content-free
// calibration logits when given, accumulated at the canonical option that
// position shows; the score is rounded to f32 (the reference's f32 score
// vector) and the served probabilities are its softmax.  f64 throughout like
// the reference's host code.  One thread per question: a question has at
// most a few variants of at most a few options.
#include <cmath>

#include "common.cuh"

namespace cevk {

constexpr int kMaxOptions = 32;

__global__ void debias_kernel(const float* __restrict__ logits, const float* __restrict__ cf, int ld,
                              const int32_t* __restrict__ span, const int32_t* __restrict__ n_opts,
                              const int32_t* __restrict__ order, int n_q, float* __restrict__ scores,
                              double* __restrict__ probs, int out_ld) {
  const int qi = blockIdx.x * blockDim.x + threadIdx.x;
  if (qi >= n_q) return;
  const int k = min(max(n_opts[qi], 1), ld), v0 = span[qi], v1 = span[qi + 1];
  const double n = (double)(v1 - v0);
  double score[kMaxOptions];
  for (int o = 0; o < k; ++o) score[o] = 0.0;
  for (int v = v0; v < v1; ++v) {
    const float* z = logits + (size_t)v * ld;
    double m = (double)z[0];
    for (int j = 1; j < k; ++j) m = fmax(m, (double)z[j]);
    double s = 0.0;
    for (int j = 0; j < k; ++j) s += exp((double)z[j] - m);
    const double lse = m + log(s);
    double base_lse = 0.0;
    const float* c = cf ? cf + (size_t)v * ld : nullptr;
    if (c) {
      double mc = (double)c[0];
      for (int j = 1; j < k; ++j) mc = fmax(mc, (double)c[j]);
      double sc = 0.0;
      for (int j = 0; j < k; ++j) sc += exp((double)c[j] - mc);
      base_lse = mc + log(sc);
    }
    for (int pos = 0; pos < k; ++pos) {
      const double lp = (double)z[pos] - lse;
      const double base = c ? (double)c[pos] - base_lse : 0.0;
      const int o = order[(size_t)v * ld + pos];
      if (o >= 0 && o < k) score[o] += (lp - base) / n;
    }
  }
  double mx = -INFINITY;
  for (int o = 0; o < k; ++o) {
    score[o] = (double)(float)score[o];  // the served score vector is f32
    mx = fmax(mx, score[o]);
  }
  double sum = 0.0;
  for (int o = 0; o < k; ++o) sum += exp(score[o] - mx);
  for (int o = 0; o < k; ++o) {
    scores[(size_t)qi * out_ld + o] = (float)score[o];
    probs[(size_t)qi * out_ld + o] = exp(score[o] - mx) / sum;
  }
}

}  // namespace cevk

using namespace cevk;

extern "C" int cevk_debias(const float* logits, const float* cf_logits, int32_t ld, const int32_t* span,
                           const int32_t* n_options, const int32_t* order, int32_t n_questions, float* scores,
                           double* probs, int32_t out_ld, void* stream) {
  if (!logits || !span || !n_options || !order || !scores || !probs)
    return set_error(CEVK_E_SHAPE, "debias: null pointer");
  if (ld < 1 || ld > kMaxOptions || out_ld < ld)
    return set_error(CEVK_E_SHAPE, "debias: %d options per row (at most %d), output stride %d", ld, kMaxOptions,
                     out_ld);
  if (n_questions <= 0) return CEVK_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  debias_kernel<<<(n_questions + 127) / 128, 128, 0, st>>>(logits, cf_logits, ld, span, n_options, order, n_questions,
                                                           scores, probs, out_ld);
  return check_launch("debias_kernel");
}
