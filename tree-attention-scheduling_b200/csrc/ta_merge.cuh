// The per-(request, query head) global log-sum-exp merge (reference _merge,
// kernels.py:58-83) as a device function, shared by the merge kernel and the
// merge phase of the small-group kernel.
#pragma once

#include "ta_common.cuh"
#include "ta_kernels.cuh"

namespace ta {

// Merge of one (request, query head) by one warp: lane k loads the LSE of
// partial k so the maximum and the weights come from warp reductions, then
// the partial rows are read with independent loads (lanes split head_dim),
// eight rows in flight.  `count` and `pre_slot` (this lane's first slot, or
// -1) were loaded by the caller.
template <typename T, int D>
__device__ __forceinline__ void merge_one(const MergeParams& p, int request, int head, int count, int pre_slot,
                                          int lane) {
  constexpr int DL = D / 32;
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
    // every row of the group in flight at once (eight at a time)
    const int n = min(32, count - k0);
    for (int j = 0; j < n; j += 8) {
      float wj[8];
      float x[8][DL];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
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
      for (int u = 0; u < 8; ++u)
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

// Merge of one (request, KV head) by one warp: its G query heads at once
// (G = 1, 2, 4 or 8, head_dim 128).  A slot's G partial rows are contiguous
// (G x 128 floats), so lane l reads head l / (32 / G), 128 * G / 32 dims of it,
// and the G LSEs of a slot are one vector load.  `count` and `pre_slot` (this
// lane's first slot, or -1) were loaded by the caller.
template <typename T, int G, int ROWS_IN_FLIGHT = 64>
__device__ __forceinline__ void merge_group(const MergeParams& p, int request, int kv_head, int count,
                                            int pre_slot, int lane) {
  constexpr int D = 128;
  constexpr int LPH = 32 / G;                 // lanes per query head
  constexpr int DL = D / LPH;                 // dims per lane
  constexpr int NF4 = DL / 4;                 // float4 loads per partial row piece
  // partial rows whose loads are in flight at once (ROWS_IN_FLIGHT floats per lane)
  constexpr int INFLIGHT = ROWS_IN_FLIGHT / DL > 0 ? ROWS_IN_FLIGHT / DL : 1;
  static_assert(G == 1 || G == 2 || G == 4 || G == 8, "group size");
  const int gm = lane / LPH, d0 = (lane % LPH) * DL;
  const int32_t* slots = p.cslots + int64_t(request) * p.max_slots;
  if (count < 0 || count > p.max_slots) {
    if (lane == 0) set_status(p.status, TA_ERR_BOUNDS);
    count = 0;
  }
  const int64_t head_rows = int64_t(kv_head) * p.num_partials;   // in slots

  float acc[DL];
#pragma unroll
  for (int e = 0; e < DL; ++e) acc[e] = 0.f;
  float m[G], z[G];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    z[g] = 0.f;
  }
  for (int k0 = 0; k0 < count; k0 += 32) {
    const int k = k0 + lane;
    int s = -1;
    if (k < count) {
      s = k0 == 0 ? pre_slot : slots[k];
      if (s < 0 || s >= p.num_partials) {
        set_status(p.status, TA_ERR_BOUNDS);
        s = -1;
      }
    }
    float l[G];
    if (s >= 0) {
      const float* src = p.lse + (head_rows + s) * G;
      if constexpr (G == 4) {
        const float4 v = *reinterpret_cast<const float4*>(src);
        l[0] = v.x; l[1] = v.y; l[2] = v.z; l[3] = v.w;
      } else {
#pragma unroll
        for (int g = 0; g < G; ++g) l[g] = src[g];
      }
    } else {
#pragma unroll
      for (int g = 0; g < G; ++g) l[g] = -INFINITY;
    }
    float w[G], scale_mine = 1.f;
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float mn = fmaxf(m[g], warp_max(l[g]));
      const float sc = mn == -INFINITY ? 1.f : fast_exp2((m[g] - mn) * kLog2e);   // m = -inf gives 0
      w[g] = mn == -INFINITY ? 0.f : fast_exp2((l[g] - mn) * kLog2e);           // -inf lse gives 0
      z[g] = z[g] * sc + warp_sum(w[g]);
      m[g] = mn;
      if (g == gm) scale_mine = sc;
    }
#pragma unroll
    for (int e = 0; e < DL; ++e) acc[e] *= scale_mine;
    const int n = min(32, count - k0);
    for (int j = 0; j < n; j += INFLIGHT) {
      float wj[INFLIGHT];
      float4 x[INFLIGHT][NF4];
#pragma unroll
      for (int u = 0; u < INFLIGHT; ++u) {
        const int src = min(j + u, n - 1);
        float wsel = 0.f;
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float wg = __shfl_sync(0xffffffffu, w[g], src);
          if (g == gm) wsel = wg;
        }
        wj[u] = j + u < n ? wsel : 0.f;
        const int sj = __shfl_sync(0xffffffffu, s, src);
        const float4* ptr = reinterpret_cast<const float4*>(p.part + ((head_rows + sj) * G + gm) * D + d0);
#pragma unroll
        for (int f = 0; f < NF4; ++f) x[u][f] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (wj[u] != 0.f) {                   // an empty partial (weight 0) may hold anything
#pragma unroll
          for (int f = 0; f < NF4; ++f) x[u][f] = ptr[f];
        }
      }
#pragma unroll
      for (int u = 0; u < INFLIGHT; ++u)
#pragma unroll
        for (int f = 0; f < NF4; ++f) {
          acc[4 * f + 0] = fmaf(wj[u], x[u][f].x, acc[4 * f + 0]);
          acc[4 * f + 1] = fmaf(wj[u], x[u][f].y, acc[4 * f + 1]);
          acc[4 * f + 2] = fmaf(wj[u], x[u][f].z, acc[4 * f + 2]);
          acc[4 * f + 3] = fmaf(wj[u], x[u][f].w, acc[4 * f + 3]);
        }
    }
  }
  float zm = z[0], mm = m[0];
#pragma unroll
  for (int g = 1; g < G; ++g)
    if (g == gm) {
      zm = z[g];
      mm = m[g];
    }
  const float inv = zm > 0.f ? 1.f / zm : 0.f;
  const int head = kv_head * G + gm;
  uint32_t* out = reinterpret_cast<uint32_t*>(reinterpret_cast<uint16_t*>(p.out) +
                                              (int64_t(request) * p.num_q_heads + head) * D + d0);
#pragma unroll
  for (int e = 0; e < DL; e += 2) out[e / 2] = Elem<T>::pack2(acc[e] * inv, acc[e + 1] * inv);
  if (p.out_lse && lane % LPH == 0)
    p.out_lse[int64_t(request) * p.num_q_heads + head] = zm > 0.f ? mm + fast_log2(zm) * kLn2 : -INFINITY;
}

}  // namespace ta
