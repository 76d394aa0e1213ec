// Fused decode-step KV append behind ta_decode_append.
//
// One launch per layer and step writes the step's new K and V rows of every
// (request, KV head) into the token-major pools [HK, T, D] at the request's
// target position -- the reference's two index_copy_ calls (qwen.py:89-90) --
// and, when asked (the step's first layer), sets every decode tail's length in
// the plan to a count read on the device, the reference's
// CachedDecodePlan.update (kernels.py:184-186).  Reading the count on the
// device lets a captured decode step advance without the host.
#include <algorithm>

#include "ta_common.cuh"
#include "ta_kernels.cuh"

namespace ta {

namespace {

constexpr int kAppendThreads = 256;   // eight rows (warps) per block

// One warp per (request, KV head) row; a row is head_dim / 2 four-byte words.
__global__ void __launch_bounds__(kAppendThreads)
    decode_append_kernel(uint32_t* kpool, uint32_t* vpool, const uint32_t* k_new, const uint32_t* v_new,
                         int64_t stride_r, int64_t stride_h, const int64_t* targets, int num_requests,
                         int num_kv_heads, int64_t pool_tokens, int words, int32_t* klen, const int32_t* tail_jobs,
                         int num_tails, const int64_t* count, int offset, int num_jobs, int32_t* status) {
  if (klen && blockIdx.x == 0) {
    const int64_t value = *count + offset;
    for (int i = threadIdx.x; i < num_tails; i += blockDim.x) {
      const int j = tail_jobs[i];
      if (j < 0 || j >= num_jobs || value < 0 || value > INT32_MAX)
        set_status(status, TA_ERR_BOUNDS);
      else
        klen[j] = int32_t(value);
    }
  }
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (row >= num_requests * num_kv_heads) return;
  const int r = row / num_kv_heads, h = row % num_kv_heads;
  const int64_t pos = targets[r];
  if (pos < 0 || pos >= pool_tokens) {
    if (lane == 0) set_status(status, TA_ERR_BOUNDS);
    return;
  }
  const int64_t src = int64_t(r) * stride_r + int64_t(h) * stride_h;
  const int64_t dst = (int64_t(h) * pool_tokens + pos) * words;
  for (int i = lane; i < words; i += 32) {
    kpool[dst + i] = k_new[src + i];
    vpool[dst + i] = v_new[src + i];
  }
}

bool aligned4(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 3u) == 0; }

}  // namespace

}  // namespace ta

extern "C" int ta_decode_append(void* kpool, void* vpool, const void* k_new, const void* v_new,
                                int64_t new_stride_request, int64_t new_stride_head, const int64_t* targets,
                                int32_t num_requests, int32_t num_kv_heads, int64_t pool_tokens, int32_t head_dim,
                                int32_t dtype, int32_t* klen, const int32_t* tail_jobs, int32_t num_tails,
                                const int64_t* count, int32_t offset, int32_t num_jobs, int32_t* status,
                                void* stream) {
  using namespace ta;
  if (dtype != TA_DTYPE_BF16 && dtype != TA_DTYPE_F16) return TA_ERR_UNSUPPORTED;
  if (num_requests < 0 || num_kv_heads <= 0 || pool_tokens < 0 || head_dim <= 0 || (head_dim & 1)) return TA_ERR_ARG;
  if (new_stride_request < 0 || new_stride_head < 0 || (new_stride_request & 1) || (new_stride_head & 1))
    return TA_ERR_ARG;
  if (klen && (!tail_jobs || !count || num_tails < 0 || num_jobs < 0)) return TA_ERR_ARG;
  const bool rows = num_requests > 0;
  if (rows && (!kpool || !vpool || !k_new || !v_new || !targets)) return TA_ERR_ARG;
  if (rows && !(aligned4(kpool) && aligned4(vpool) && aligned4(k_new) && aligned4(v_new))) return TA_ERR_ARG;
  if (!rows && (!klen || num_tails == 0)) return TA_OK;
  const int64_t threads = std::max<int64_t>(1, int64_t(num_requests) * num_kv_heads) * 32;
  const int blocks = int((threads + kAppendThreads - 1) / kAppendThreads);
  decode_append_kernel<<<blocks, kAppendThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<uint32_t*>(kpool), static_cast<uint32_t*>(vpool), static_cast<const uint32_t*>(k_new),
      static_cast<const uint32_t*>(v_new), new_stride_request / 2, new_stride_head / 2, targets, num_requests,
      num_kv_heads, pool_tokens, head_dim / 2, klen, tail_jobs, klen ? num_tails : 0, count, offset, num_jobs,
      status);
  return cudaGetLastError() == cudaSuccess ? TA_OK : TA_ERR_LAUNCH;
}
