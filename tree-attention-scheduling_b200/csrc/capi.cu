// extern "C" entry points declared in include/tree_attn.h.
//
// The host side only validates arguments, resolves the plan layout into kernel
// parameter blocks and launches on the caller's stream: no allocation, no
// synchronisation, so every call can be captured into a CUDA graph.
#include <cmath>
#include <cstdlib>
#include <cstring>

#include "ta_common.cuh"
#include "ta_kernels.cuh"

using namespace ta;

namespace {

bool layout_ok(const ta_plan_layout* L) {
  if (!L) return false;
  if (L->num_jobs < 0 || L->max_requests < 0 || L->max_slots < 0 || L->num_requests < 0 || L->num_pieces < 0 ||
      L->num_partials < 0 || L->max_pslots < 0)
    return false;
  if (L->num_small_tasks < 0 || L->num_tc_tasks < 0 || L->num_kn_tasks < 0 || L->kn_ctas < 0 || L->kstart_stride < 1)
    return false;
  int64_t class_ctas = 0;
  for (int c = 0; c < 5; ++c) {
    if (L->kn_class_ctas[c] < 0) return false;
    class_ctas += L->kn_class_ctas[c];
  }
  if (class_ctas != L->kn_ctas) return false;
  if (L->num_kn_tasks > 0 && (L->kn_ctas < 1 || L->num_kn_segs < 1)) return false;
  if ((L->off_kn_tasks & 3) || (L->off_kn_segs & 3) || (L->off_tc_tasks & 3)) return false;   // int4 loads
  const int32_t* e = L->small_class_end;
  if (e[0] < 0 || e[1] < e[0] || e[2] < e[1] || e[2] != L->num_small_tasks) return false;
  return true;
}

bool heads_ok(int32_t hq, int32_t hk, int32_t d, int32_t dtype) {
  if (hq <= 0 || hk <= 0 || hq % hk) return false;
  if (d != 32 && d != 64 && d != 128) return false;
  return dtype == TA_DTYPE_BF16 || dtype == TA_DTYPE_F16;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int launch_status(cudaError_t err) { return err == cudaSuccess ? TA_OK : TA_ERR_LAUNCH; }

MergeParams merge_params(const ta_plan_layout* plan, const int32_t* meta, const float* part, const float* lse,
                         void* out, float* out_lse, int32_t num_q_heads, int32_t num_kv_heads, int32_t* status) {
  MergeParams p{};
  p.part = part;
  p.lse = lse;
  p.cslots = meta + plan->off_cslots;
  p.counts = meta + plan->off_pcounts;
  p.out = out;
  p.out_lse = out_lse;
  p.status = status;
  p.num_requests = plan->num_requests;
  p.max_slots = plan->max_pslots;
  p.num_partials = plan->num_partials;
  p.num_q_heads = num_q_heads;
  p.group = num_q_heads / num_kv_heads;
  return p;
}

// The segment launches of a step.
int run_segment(const ta_plan_layout* plan, const int32_t* meta, const void* q, const void* kpool,
                const void* vpool, int64_t pool_tokens, int32_t num_q_heads, int32_t num_kv_heads,
                int32_t head_dim, int32_t dtype, float* part, float* lse, int32_t* status, void* stream) {
  if (!layout_ok(plan) || !meta || pool_tokens < 0) return TA_ERR_ARG;
  if (!heads_ok(num_q_heads, num_kv_heads, head_dim, dtype)) return TA_ERR_UNSUPPORTED;
  const int tasks = plan->num_small_tasks + plan->num_tc_tasks + plan->num_kn_tasks;
  if (tasks == 0) return TA_OK;
  if (!q || !kpool || !vpool || !part || !lse) return TA_ERR_ARG;
  // bulk copies and TMA need 16-byte aligned bases; rows are 2*head_dim bytes
  if (!aligned16(meta) || !aligned16(q) || !aligned16(kpool) || !aligned16(vpool) || !aligned16(part)) return TA_ERR_ARG;
  if ((plan->num_tc_tasks > 0 || plan->num_kn_tasks > 0) && head_dim != 128) return TA_ERR_UNSUPPORTED;
  // keys-in-lanes kernels are built for tasks of up to 8 query rows
  if (plan->kn_class_ctas[2] > 0 || plan->kn_class_ctas[3] > 0 || plan->kn_class_ctas[4] > 0) return TA_ERR_UNSUPPORTED;
  // TMA coordinates are 32-bit
  if ((plan->num_tc_tasks > 0 || plan->num_kn_tasks > 0) && pool_tokens > int64_t(INT32_MAX) - 512) return TA_ERR_ARG;

  SegParams p{};
  p.q = static_cast<const uint16_t*>(q);
  p.k = static_cast<const uint16_t*>(kpool);
  p.v = static_cast<const uint16_t*>(vpool);
  p.part = part;
  p.lse = lse;
  p.qids = meta + plan->off_qids;
  p.kstart = meta + plan->off_kstart;
  p.qlen = meta + plan->off_qlen;
  p.klen = meta + plan->off_klen;
  p.pieces = meta + plan->off_pieces;
  p.small_tasks = meta + plan->off_small_tasks;
  p.tc_tasks = meta + plan->off_tc_tasks;
  p.kn_offsets = meta + plan->off_kn_offsets;
  p.kn_tasks = meta + plan->off_kn_tasks;
  p.kn_segs = meta + plan->off_kn_segs;
  p.status = status;
  p.pool_tokens = pool_tokens;
  p.num_jobs = plan->num_jobs;
  p.num_pieces = plan->num_pieces;
  p.max_requests = plan->max_requests;
  p.kstart_stride = plan->kstart_stride;
  p.num_requests = plan->num_requests;
  p.num_partials = plan->num_partials;
  p.num_q_heads = num_q_heads;
  p.num_kv_heads = num_kv_heads;
  p.group = num_q_heads / num_kv_heads;
  p.num_kn_tasks = plan->num_kn_tasks;
  p.num_kn_segs = plan->num_kn_segs;
  p.kn_ctas = plan->kn_ctas;
  p.scale_log2 = kLog2e / std::sqrt(float(head_dim));
  p.gmul = (65536u + uint32_t(p.group) - 1u) / uint32_t(p.group);

  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t err = cudaSuccess;
  if (plan->num_tc_tasks > 0) err = launch_seg_tc(p, plan->num_tc_tasks, dtype, s);
  p.kn_after_tc = plan->num_tc_tasks > 0 && err == cudaSuccess;
  if (err == cudaSuccess && plan->num_kn_tasks > 0) err = launch_seg_kn(p, plan->kn_class_ctas, dtype, s);
  if (err == cudaSuccess && plan->num_small_tasks > 0) {
    // Test hook (TREE_ATTN_TEST_STALL=1): the SIMT kernel waits on a barrier
    // nothing completes, so its bounded waits give up and report TA_ERR_TIMEOUT.
    const char* stall = std::getenv("TREE_ATTN_TEST_STALL");
    p.test_stall = stall && std::strcmp(stall, "1") == 0;
    err = launch_seg_simt(p, plan->small_class_end, plan->small_max_keys, head_dim, dtype, s);
  }
  return launch_status(err);
}

}  // namespace

extern "C" {

int ta_abi_version(void) { return TA_ABI_VERSION; }

const char* ta_error_string(int code) {
  switch (code) {
    case TA_OK: return "ok";
    case TA_ERR_ARG: return "invalid argument";
    case TA_ERR_LAUNCH: return "kernel launch failed";
    case TA_ERR_BOUNDS: return "plan index out of range on the device";
    case TA_ERR_TIMEOUT: return "bounded device wait gave up";
    case TA_ERR_UNSUPPORTED: return "shape or dtype not supported";
    case TA_ERR_TOO_LARGE: return "problem exceeds a fixed scratch or buffer size";
    default: return "multiple errors";
  }
}

int ta_segment(const ta_plan_layout* plan, const int32_t* meta, const void* q, const void* kpool,
               const void* vpool, int64_t pool_tokens, int32_t num_q_heads, int32_t num_kv_heads,
               int32_t head_dim, int32_t dtype, float* part, float* lse, int32_t* status, void* stream) {
  return run_segment(plan, meta, q, kpool, vpool, pool_tokens, num_q_heads, num_kv_heads, head_dim, dtype, part,
                     lse, status, stream);
}

int ta_merge(const ta_plan_layout* plan, const int32_t* meta, const float* part, const float* lse, void* out,
             float* out_lse, int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim, int32_t dtype,
             int32_t* status, void* stream) {
  if (!layout_ok(plan) || !meta) return TA_ERR_ARG;
  if (!heads_ok(num_q_heads, num_kv_heads, head_dim, dtype)) return TA_ERR_UNSUPPORTED;
  if (plan->num_requests == 0) return TA_OK;
  if (!part || !lse || !out || !aligned16(part) || !aligned16(out)) return TA_ERR_ARG;
  const MergeParams p = merge_params(plan, meta, part, lse, out, out_lse, num_q_heads, num_kv_heads, status);
  return launch_status(launch_merge(p, head_dim, dtype, static_cast<cudaStream_t>(stream)));
}

int ta_attention(const ta_plan_layout* plan, const int32_t* meta, const void* q, const void* kpool,
                 const void* vpool, int64_t pool_tokens, int32_t num_q_heads, int32_t num_kv_heads,
                 int32_t head_dim, int32_t dtype, float* part, float* lse, void* out, float* out_lse,
                 int32_t* status, void* stream) {
  // Validated up front so a rejected merge argument launches nothing.
  if (!layout_ok(plan) || !meta) return TA_ERR_ARG;
  if (!heads_ok(num_q_heads, num_kv_heads, head_dim, dtype)) return TA_ERR_UNSUPPORTED;
  if (plan->num_requests > 0 && (!out || !aligned16(out))) return TA_ERR_ARG;
  int rc = run_segment(plan, meta, q, kpool, vpool, pool_tokens, num_q_heads, num_kv_heads, head_dim, dtype, part,
                       lse, status, stream);
  if (rc != TA_OK) return rc;
  return ta_merge(plan, meta, part, lse, out, out_lse, num_q_heads, num_kv_heads, head_dim, dtype, status,
                  stream);
}

int ta_update_tail_klen(int32_t* klen, const int32_t* tail_jobs, int32_t num_tails, int32_t value,
                        int32_t num_jobs, int32_t* status, void* stream) {
  if (num_tails < 0 || value < 0 || num_jobs < 0) return TA_ERR_ARG;
  if (num_tails == 0) return TA_OK;
  if (!klen || !tail_jobs) return TA_ERR_ARG;
  return launch_status(
      launch_fill_klen(klen, tail_jobs, num_tails, value, num_jobs, status, static_cast<cudaStream_t>(stream)));
}

}  // extern "C"
