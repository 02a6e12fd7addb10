// The C ABI: status codes, thread-local error messages, host-side
// validation of shapes and descriptors, and dispatch to the kernels.
#include <cstdarg>
#include <cstdio>
#include <algorithm>
#include <cstring>
#include <mutex>
#include <vector>

#include "common.cuh"

namespace cevk {

__device__ int g_device_error = 0;
__device__ int g_device_error_info[4] = {0, 0, 0, 0};
__device__ int g_device_error_n = 0;
__device__ int g_device_error_more[64];

static thread_local char g_msg[512] = "";

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(CEVK_E_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return CEVK_OK;
}

int opt_in_smem(const void* fn, int bytes, const char* what) {
  struct Done {
    const void* fn;
    int dev, bytes;
  };
  static std::mutex mu;
  static std::vector<Done> done;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(CEVK_E_CUDA, "%s: cudaGetDevice: %s", what, cudaGetErrorString(e));
  std::lock_guard<std::mutex> lock(mu);
  for (const Done& d : done)
    if (d.fn == fn && d.dev == dev && d.bytes >= bytes) return CEVK_OK;
  e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess)
    return set_error(CEVK_E_CUDA, "%s: cannot opt in to %d B of shared memory: %s", what, bytes, cudaGetErrorString(e));
  done.push_back(Done{fn, dev, bytes});
  return CEVK_OK;
}

int attn_tc_launch(const void* q, const void* k, const void* v, void* const* o, int n_o, int n_tokens, int n_kv_rows,
                   int hq, int hkv, int D, int q_rs, int kv_rs, int o_rs, const cevk_segment* segs, int n_segs,
                   int n_tiles, float scale, int n_split, void* workspace, cudaStream_t stream);
int attn_simt_launch(const void* q, const void* k, const void* v, void* o, int hq, int hkv, int D, int q_rs, int kv_rs,
                     int o_rs, const cevk_segment* segs, int n_segs, float scale, cudaStream_t stream);

// One thread waits, through the library's bounded wait, on an mbarrier that
// nothing arrives on: the wait gives up after `limit` clock cycles, raises the
// device error record and the kernel returns normally.
__global__ void wait_timeout_probe_kernel(long long limit) {
  __shared__ __align__(8) unsigned long long bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    const uint32_t b = smem_u32(&bar);
    mbar_init(b, 1);
    abort_flag = 0;
    mbar_fence_init();
    mbar_wait(b, 0, &abort_flag, limit);
  }
}

}  // namespace cevk

using namespace cevk;

extern "C" {

const char* cevk_last_error(void) { return g_msg; }

int cevk_version(void) { return 100; }

int cevk_device_status(void) {
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return set_error(CEVK_E_CUDA, "device: %s", cudaGetErrorString(e));
  DeviceErrorRecord r;
  if (!take_device_error(&r)) return set_error(CEVK_E_CUDA, "cannot read the device error flag");
  if (r.flag) {
    char extra[384] = "";
    int len = 0;
    for (int i = 0; i < r.n && i < 16 && len < 320; ++i)
      if (r.more[4 * i] == r.info[0])
        len += snprintf(extra + len, sizeof(extra) - len, " [t%d 0x%x p%d]", r.more[4 * i + 1], r.more[4 * i + 2],
                        r.more[4 * i + 3]);
    if (r.flag == 2)
      return set_error(CEVK_E_TIMEOUT,
                       "a bounded device wait gave up (code 2, head all-gather): rank %d's flag reads %d, epoch %d",
                       r.info[1], r.info[2], r.info[3]);
    return set_error(CEVK_E_TIMEOUT,
                     "a bounded device wait gave up (code %d): block %d thread %d barrier smem offset 0x%x parity %d;"
                     " also stopped in that block:%s",
                     r.flag, r.info[0], r.info[1], r.info[2], r.info[3], extra);
  }
  return CEVK_OK;
}

int cevk_selftest_wait_timeout(int64_t limit_cycles, void* stream) {
  if (limit_cycles <= 0 || limit_cycles > (1ll << 32)) return set_error(CEVK_E_SHAPE, "selftest: limit out of range");
  wait_timeout_probe_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(limit_cycles);
  return check_launch("wait_timeout_probe_kernel");
}

int cevk_attn_schedule(cevk_segment* segs, int32_t n_segs, int32_t n_tokens, int32_t n_kv_rows, int32_t hq,
                       int32_t hkv, int32_t head_dim, int32_t dtype, int32_t* n_tiles) {
  if (!segs || n_segs < 0 || !n_tiles) return set_error(CEVK_E_SHAPE, "schedule: null argument");
  if (hkv <= 0 || hq % hkv != 0) return set_error(CEVK_E_SHAPE, "hq (%d) must be a multiple of hkv (%d)", hq, hkv);
  const int group = hq / hkv;
  int rows_t = 1;
  if (dtype == CEVK_BF16) {
    if (128 % group != 0) return set_error(CEVK_E_SHAPE, "bf16 attention needs hq/hkv dividing 128 (got %d)", group);
    rows_t = 128 / group;
  }
  int64_t tiles = 0;
  for (int i = 0; i < n_segs; ++i) {
    const cevk_segment& g = segs[i];
    if (g.flags & ~CEVK_SEG_BIDIRECTIONAL) return set_error(CEVK_E_SHAPE, "segment %d: unknown flags 0x%x", i, g.flags);
    if (g.q_len < 0 || g.prefix_len < 0 || g.q_start < 0 || g.prefix_off < 0 || g.self_off < 0)
      return set_error(CEVK_E_RANGE, "segment %d: negative offset or length", i);
    if ((int64_t)g.q_start + g.q_len > n_tokens)
      return set_error(CEVK_E_RANGE, "segment %d: query rows %d..%d past %d tokens", i, g.q_start, g.q_start + g.q_len, n_tokens);
    if ((int64_t)g.prefix_off + g.prefix_len > n_kv_rows || (int64_t)g.self_off + g.q_len > n_kv_rows)
      return set_error(CEVK_E_RANGE, "segment %d: K/V rows past %d", i, n_kv_rows);
    segs[i].tile_start = (int32_t)tiles;
    tiles += (segs[i].q_len + rows_t - 1) / rows_t;
  }
  if (tiles > (1ll << 30)) return set_error(CEVK_E_RANGE, "too many tiles");
  *n_tiles = (int32_t)tiles;
  (void)head_dim;
  return CEVK_OK;
}

int64_t cevk_attn_split_workspace_size(int32_t n_tiles, int32_t hkv, int32_t head_dim, int32_t n_split) {
  if (n_split <= 1 || n_tiles <= 0 || hkv <= 0 || head_dim <= 0) return 0;
  return (int64_t)n_tiles * hkv * n_split * 128 * (head_dim + 1) * 4;
}

int cevk_attn_split_plan(const cevk_segment* segs, int32_t n_segs, int32_t n_tiles, int32_t hkv, int32_t head_dim,
                         int32_t dtype, int32_t n_sms, int32_t* n_split, int64_t* workspace_bytes) {
  if ((!segs && n_segs > 0) || !n_split || !workspace_bytes) return set_error(CEVK_E_SHAPE, "split plan: null argument");
  *n_split = 1;
  *workspace_bytes = 0;
  if (dtype != CEVK_BF16 || n_segs <= 0 || n_tiles <= 0 || hkv <= 0 || n_sms <= 0) return CEVK_OK;
  // Resident CTAs: two per SM for head_dim <= 128, one for 256.
  const int64_t slots = (int64_t)n_sms * (head_dim <= 128 ? 2 : 1);
  const int64_t n_work = (int64_t)n_tiles * hkv;
  int max_pre = 0, max_total = 0;
  for (int i = 0; i < n_segs; ++i) {
    max_pre = std::max(max_pre, (segs[i].prefix_len + 63) / 64);
    max_total = std::max(max_total, (segs[i].prefix_len + segs[i].q_len + 63) / 64);
  }
  // Cost model in 64-key blocks: a CTA item of b blocks costs b + kFix
  // (its Q load, first S and epilogue, about three block periods measured),
  // and equal items run in waves of `slots`.  Take the split count with the
  // lowest waves x (blocks per range + kFix), at least 8 blocks (512 keys)
  // per range, and only when it saves 3% over fewer ranges (the merge
  // reads every range's rows once more).  Wave quantisation is what the
  // count trades against: 128 items on 296 slots fill 86% of one wave,
  // 1152 items fill 97% of four.
  constexpr int64_t kFix = 3;
  auto cost = [&](int64_t s) {
    const int64_t waves = (n_work * s + slots - 1) / slots;
    return waves * ((max_total + s - 1) / s + kFix);
  };
  int64_t s = 1, best = cost(1);
  const int64_t s_max = std::min<int64_t>((int64_t)max_pre / 8, 32);
  for (int64_t c = 2; c <= s_max && n_work * c < (1ll << 30); ++c) {
    const int64_t k = cost(c);
    if (k * 100 < best * 97) {
      best = k;
      s = c;
    }
  }
  if (s < 2) return CEVK_OK;
  *n_split = (int32_t)s;
  *workspace_bytes = cevk_attn_split_workspace_size(n_tiles, hkv, head_dim, (int32_t)s);
  return CEVK_OK;
}

static int packed_prefill(const void* q, const void* k, const void* v, void* const* o, int32_t n_o, int32_t n_tokens,
                          int32_t n_kv_rows, int32_t hq, int32_t hkv, int32_t head_dim, int32_t q_row_stride,
                          int32_t kv_row_stride, int32_t o_row_stride, const cevk_segment* segs_dev, int32_t n_segs,
                          int32_t n_tiles, float scale, int32_t n_split, void* workspace, int64_t workspace_bytes,
                          int32_t dtype, void* stream) {
  if (!q || !k || !v || !o || n_o < 1 || (!segs_dev && n_segs > 0))
    return set_error(CEVK_E_SHAPE, "attention: null pointer");
  for (int i = 0; i < n_o; ++i)
    if (!o[i]) return set_error(CEVK_E_SHAPE, "attention: null output buffer %d", i);
  if (hkv <= 0 || hq % hkv != 0) return set_error(CEVK_E_SHAPE, "hq (%d) must be a multiple of hkv (%d)", hq, hkv);
  if (q_row_stride < hq * head_dim || o_row_stride < hq * head_dim || kv_row_stride < hkv * head_dim)
    return set_error(CEVK_E_SHAPE, "attention: row stride smaller than heads * head_dim");
  if (n_segs == 0 || n_tiles == 0) return CEVK_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == CEVK_BF16) {
    uintptr_t addr = (uintptr_t)q | (uintptr_t)k | (uintptr_t)v;
    for (int i = 0; i < n_o; ++i) addr |= (uintptr_t)o[i];
    if (addr & 15) return set_error(CEVK_E_SHAPE, "attention: q/k/v/o must be 16-byte aligned");
    if ((q_row_stride % 8) || (kv_row_stride % 8) || (o_row_stride % 8))
      return set_error(CEVK_E_SHAPE, "attention: bf16 row strides must be multiples of 8 elements");
    if (128 % (hq / hkv) != 0) return set_error(CEVK_E_SHAPE, "attention: hq/hkv must divide 128");
    if (n_split < 1 || (int64_t)n_tiles * hkv * n_split >= (1ll << 30))
      return set_error(CEVK_E_SHAPE, "attention: split count %d out of range", n_split);
    if (n_split > 1) {
      const int64_t need = cevk_attn_split_workspace_size(n_tiles, hkv, head_dim, n_split);
      if (!workspace || workspace_bytes < need)
        return set_error(CEVK_E_SHAPE, "attention: split workspace of %lld bytes, %lld needed", (long long)workspace_bytes,
                         (long long)need);
      if ((uintptr_t)workspace & 15) return set_error(CEVK_E_SHAPE, "attention: split workspace must be 16-byte aligned");
    }
    return attn_tc_launch(q, k, v, o, n_o, n_tokens, n_kv_rows, hq, hkv, head_dim, q_row_stride, kv_row_stride,
                          o_row_stride, segs_dev, n_segs, n_tiles, scale, n_split, workspace, st);
  }
  if (dtype == CEVK_F32 && n_o == 1)
    return attn_simt_launch(q, k, v, o[0], hq, hkv, head_dim, q_row_stride, kv_row_stride, o_row_stride, segs_dev,
                            n_segs, scale, st);
  return set_error(CEVK_E_UNSUPPORTED, "attention: dtype %d", dtype);
}

int cevk_attn_packed_prefill(const void* q, const void* k, const void* v, void* o, int32_t n_tokens,
                             int32_t n_kv_rows, int32_t hq, int32_t hkv, int32_t head_dim, int32_t q_row_stride,
                             int32_t kv_row_stride, int32_t o_row_stride, const cevk_segment* segs_dev,
                             int32_t n_segs, int32_t n_tiles, float scale, int32_t dtype, void* stream) {
  return packed_prefill(q, k, v, &o, 1, n_tokens, n_kv_rows, hq, hkv, head_dim, q_row_stride, kv_row_stride,
                        o_row_stride, segs_dev, n_segs, n_tiles, scale, 1, nullptr, 0, dtype, stream);
}

int cevk_attn_packed_prefill_split(const void* q, const void* k, const void* v, void* o, int32_t n_tokens,
                                   int32_t n_kv_rows, int32_t hq, int32_t hkv, int32_t head_dim, int32_t q_row_stride,
                                   int32_t kv_row_stride, int32_t o_row_stride, const cevk_segment* segs_dev,
                                   int32_t n_segs, int32_t n_tiles, float scale, int32_t n_split, void* workspace,
                                   int64_t workspace_bytes, int32_t dtype, void* stream) {
  return packed_prefill(q, k, v, &o, 1, n_tokens, n_kv_rows, hq, hkv, head_dim, q_row_stride, kv_row_stride,
                        o_row_stride, segs_dev, n_segs, n_tiles, scale, n_split, workspace, workspace_bytes, dtype,
                        stream);
}

int cevk_attn_packed_prefill_gather(const void* q, const void* k, const void* v, void* const* o_bufs, int32_t n_bufs,
                                    int32_t n_tokens, int32_t n_kv_rows, int32_t hq, int32_t hkv, int32_t head_dim,
                                    int32_t q_row_stride, int32_t kv_row_stride, int32_t o_row_stride,
                                    const cevk_segment* segs_dev, int32_t n_segs, int32_t n_tiles, float scale,
                                    int32_t n_split, void* workspace, int64_t workspace_bytes, void* stream) {
  if (!o_bufs || n_bufs < 1 || n_bufs > 8) return set_error(CEVK_E_SHAPE, "attention gather: %d buffers (1..8)", n_bufs);
  return packed_prefill(q, k, v, o_bufs, n_bufs, n_tokens, n_kv_rows, hq, hkv, head_dim, q_row_stride, kv_row_stride,
                        o_row_stride, segs_dev, n_segs, n_tiles, scale, n_split, workspace, workspace_bytes, CEVK_BF16,
                        stream);
}

}  // extern "C"
