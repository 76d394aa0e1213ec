// The per-(request, query head) global log-sum-exp merge (reference _merge,
// kernels.py:58-83) as a device function of the merge kernel.
#pragma once

#include "ta_common.cuh"
#include "ta_kernels.cuh"

namespace ta {

// Merge of one (request, query head) by one warp: lane k loads the LSE of
// partial k so the maximum and the weights come from warp reductions, then
// the partial rows are read with independent loads (lanes split head_dim),
// nine rows in flight.  `count` and `pre_slot` (this lane's first slot, or
// -1) were loaded by the caller.
template <typename T, int D>
__device__ __forceinline__ void merge_one(const MergeParams& p, int request, int head, int count, int pre_slot,
                                          int lane) {
  constexpr int DL = D / 32;
  constexpr int kBatch = 9;   // partial rows in flight: one round for up to 9 partials (8 root pieces + 1 leaf)
  const int G = p.group, kv_head = head / G, g = head % G;
  const int32_t* slots = p.cslots + int64_t(request) * p.max_slots;
  if (count < 0 || count > p.max_slots) {
    if (lane == 0) set_status(p.status, TA_ERR_BOUNDS);
    count = 0;
  }
  const int64_t head_rows = int64_t(kv_head) * p.num_partials;

  float acc[DL];
#pragma unroll
  for (int e = 0; e < DL; ++e) acc[e] = 0.f;
  float m = -INFINITY, z = 0.f;
  // Lane k holds partial k0 + k of each group of 32: its LSE, weight and row.
  // Groups after the first (more than 32 partials) rescale the running sums.
  for (int k0 = 0; k0 < count; k0 += 32) {
    const int k = k0 + lane;
    float l = -INFINITY;
    int64_t row = 0;
    if (k < count) {
      const int s = k0 == 0 ? pre_slot : slots[k];
      if (s >= 0 && s < p.num_partials) {
        row = (head_rows + s) * G + g;
        l = p.lse[row];
      } else {
        set_status(p.status, TA_ERR_BOUNDS);
      }
    }
    const float m_new = fmaxf(m, warp_max(l));
    if (m_new == -INFINITY) continue;               // nothing but empty partials so far
    const float scale = fast_exp2((m - m_new) * kLog2e);   // m = -inf gives 0
    z *= scale;
#pragma unroll
    for (int e = 0; e < DL; ++e) acc[e] *= scale;
    m = m_new;
    const float w = fast_exp2((l - m) * kLog2e);        // -inf lse gives 0
    z += warp_sum(w);
    // the group's rows in flight kBatch at a time
    const int n = min(32, count - k0);
    for (int j = 0; j < n; j += kBatch) {
      float wj[kBatch];
      float x[kBatch][DL];
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        const int src = min(j + u, n - 1);
        wj[u] = __shfl_sync(0xffffffffu, w, src);
        const int64_t rj = __shfl_sync(0xffffffffu, row, src);
        if (j + u >= n) wj[u] = 0.f;
        // an empty partial (weight 0) may hold anything: do not read it
        const float* ptr = p.part + rj * D + lane * DL;
#pragma unroll
        for (int e = 0; e < DL; ++e) x[u][e] = 0.f;
        if (wj[u] != 0.f) {
          if constexpr (DL == 4) {
            const float4 v = *reinterpret_cast<const float4*>(ptr);
            x[u][0] = v.x; x[u][1] = v.y; x[u][2] = v.z; x[u][3] = v.w;
          } else if constexpr (DL == 2) {
            const float2 v = *reinterpret_cast<const float2*>(ptr);
            x[u][0] = v.x; x[u][1] = v.y;
          } else {
            x[u][0] = ptr[0];
          }
        }
      }
#pragma unroll
      for (int u = 0; u < kBatch; ++u)
#pragma unroll
        for (int e = 0; e < DL; ++e) acc[e] = fmaf(wj[u], x[u][e], acc[e]);
    }
  }
  const float inv = z > 0.f ? 1.f / z : 0.f;
  uint16_t* out = reinterpret_cast<uint16_t*>(p.out) + (int64_t(request) * p.num_q_heads + head) * D + lane * DL;
  if constexpr (DL == 4) {
    uint2 bits;
    bits.x = Elem<T>::pack2(acc[0] * inv, acc[1] * inv);
    bits.y = Elem<T>::pack2(acc[2] * inv, acc[3] * inv);
    *reinterpret_cast<uint2*>(out) = bits;
  } else if constexpr (DL == 2) {
    *reinterpret_cast<uint32_t*>(out) = Elem<T>::pack2(acc[0] * inv, acc[1] * inv);
  } else {
    *out = Elem<T>::from_float(acc[0] * inv);
  }
  if (p.out_lse && lane == 0) {
    p.out_lse[int64_t(request) * p.num_q_heads + head] = z > 0.f ? m + fast_log2(z) * kLn2 : -INFINITY;
  }
}

}  // namespace ta
