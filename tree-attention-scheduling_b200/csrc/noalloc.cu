// ta_attention_noalloc: the decode-step attention for callers that cannot
// allocate device memory.
//
// Some hosts of this library are not in a position to call cudaMalloc when
// they run attention: a process whose device memory was handed out up front
// to another allocator that owns it all, a foreign-language binding with no
// handle on a CUDA allocator, or a latency-bound serving loop that must not
// allocate (or free) on its decode path.  They still own their inputs (queries, pools, plan metadata) and
// the output, but not the partial-output / LSE scratch that ta_attention takes
// as arguments.  This entry point supplies that scratch from one file-scope
// device array of fixed size instead.
//
// Properties a caller must know:
//   * capacity: TA_NOALLOC_SCRATCH_BYTES (32 MiB) per device, enough for a
//     plan whose partials need num_kv_heads * num_partials * G * (head_dim + 1)
//     floats (plus 256 bytes of alignment); larger problems are rejected with
//     TA_ERR_TOO_LARGE before anything is launched;
//   * footprint: every GPU on which the library is loaded holds the array until
//     the process exits, whether or not this entry point is called;
//   * set-up: the first call on a device looks up the array's device address
//     (cudaGetSymbolAddress, with that device current) and caches it; make that
//     first call before starting any stream capture;
//   * sharing: all calls share the one array and it keeps the previous call's
//     contents.  Nothing in it has to start at zero (every partial row the merge
//     reads is written by the segment kernels of the same call), but calls
//     whose kernels overlap on the GPU -- different streams, or different
//     threads without ordering -- race on it and must be serialised by the
//     caller.
#include <mutex>

#include "ta_common.cuh"

namespace {

constexpr size_t kScratchBytes = TA_NOALLOC_SCRATCH_BYTES;
constexpr size_t kAlign = 256;

// The scratch itself.  In host code this name is only a stand-in for the
// symbol, never a device address: the address comes from cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mutex;
unsigned char* g_device_scratch[kMaxDevices] = {};

// Device address of the scratch on the current device (set up once per device).
int current_device_scratch(unsigned char** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return TA_ERR_LAUNCH;
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (!g_device_scratch[dev]) {
    void* ptr = nullptr;
    const cudaError_t err = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (err != cudaSuccess || ptr == nullptr) return TA_ERR_LAUNCH;
    g_device_scratch[dev] = static_cast<unsigned char*>(ptr);
  }
  *out = g_device_scratch[dev];
  return TA_OK;
}

}  // namespace

extern "C" int ta_attention_noalloc(const ta_plan_layout* plan, const int32_t* meta, const void* q, const void* kpool,
                                    const void* vpool, int64_t pool_tokens, int32_t num_q_heads, int32_t num_kv_heads,
                                    int32_t head_dim, int32_t dtype, void* out, float* out_lse, int32_t* status,
                                    void* stream) {
  if (!plan || plan->num_partials < 0 || num_kv_heads <= 0 || num_q_heads <= 0 || head_dim <= 0 ||
      num_q_heads % num_kv_heads)
    return TA_ERR_ARG;
  if (head_dim != 32 && head_dim != 64 && head_dim != 128) return TA_ERR_UNSUPPORTED;
  // Partial rows = num_partials x G x num_kv_heads = num_partials x num_q_heads.
  // Bound the factors before multiplying so no product can wrap around.
  const size_t max_rows = kScratchBytes / ((size_t(head_dim) + 1) * sizeof(float));
  if (size_t(plan->num_partials) > max_rows / size_t(num_q_heads)) return TA_ERR_TOO_LARGE;
  const size_t rows = size_t(plan->num_partials) * size_t(num_q_heads);
  const size_t part_bytes = (rows * size_t(head_dim) * sizeof(float) + kAlign - 1) / kAlign * kAlign;
  const size_t lse_bytes = rows * sizeof(float);
  if (part_bytes + lse_bytes > kScratchBytes) return TA_ERR_TOO_LARGE;
  unsigned char* scratch = nullptr;
  const int rc = current_device_scratch(&scratch);
  if (rc != TA_OK) return rc;
  float* part = reinterpret_cast<float*>(scratch);
  float* lse = reinterpret_cast<float*>(scratch + part_bytes);
  return ta_attention(plan, meta, q, kpool, vpool, pool_tokens, num_q_heads, num_kv_heads, head_dim, dtype, part,
                      lse, out, out_lse, status, stream);
}
