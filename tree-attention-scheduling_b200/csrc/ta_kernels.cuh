// Kernel parameter blocks and launchers shared by the C ABI (capi.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace ta {

// Everything a segment kernel reads, resolved from ta_plan_layout + meta.
struct SegParams {
  const uint16_t* q;         // [nreq, hq, D]
  const uint16_t* k;         // [hk, T, D]
  const uint16_t* v;         // [hk, T, D]
  float* part;               // [hk, S*G, D]
  float* lse;                // [hk, S*G]
  const int32_t* qids;       // [J, max_requests]
  const int32_t* kstart;     // [J, kstart_stride]
  const int32_t* qlen;       // [J]
  const int32_t* klen;       // [J]
  const int32_t* slot_base;  // [J]
  const int32_t* small_tasks;  // [n, 2] (job, 16-row tile)
  const int32_t* tc_tasks;     // [n, 2] (job, 128-row tile)
  int32_t* status;
  int64_t pool_tokens;
  int32_t num_jobs, max_requests, kstart_stride, num_requests, num_partials;
  int32_t num_q_heads, num_kv_heads, group;
  float scale_log2;          // log2(e) / sqrt(D)
};

struct MergeParams {
  const float* part;
  const float* lse;
  const int32_t* cslots;     // [nreq, max_slots]
  const int32_t* counts;     // [nreq]
  void* out;                 // [nreq, hq, D]
  float* out_lse;            // [nreq, hq] or null
  int32_t* status;
  int32_t num_requests, max_slots, num_partials, num_q_heads, group;
};

cudaError_t launch_seg_simt(const SegParams& p, const int32_t class_end[3], int max_keys, int head_dim, int dtype,
                            cudaStream_t stream);
cudaError_t launch_seg_tc(const SegParams& p, int num_tasks, int dtype, cudaStream_t stream);
cudaError_t launch_merge(const MergeParams& p, int head_dim, int dtype, cudaStream_t stream);
cudaError_t launch_fill_klen(int32_t* klen, const int32_t* idx, int n, int value, int num_jobs, int32_t* status,
                             cudaStream_t stream);

}  // namespace ta
