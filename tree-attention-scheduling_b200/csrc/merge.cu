// Global log-sum-exp merge of each request's partials (reference _merge,
// kernels.py:58-83), plus the tiny device update of a reused decode plan.
//
// One warp per (request, query head).  Instead of the reference's serial
// running-max loop, lane k loads the LSE of partial k so the maximum and the
// weights come from two warp reductions; the partial rows are then read with
// independent 16-byte loads (lanes split head_dim), eight rows in flight.
#include "ta_common.cuh"
#include "ta_kernels.cuh"
#include "ta_merge.cuh"

namespace ta {

namespace {

constexpr int kMergeWarps = 4;

template <typename T, int D>
// (at most 72 registers: seven CTAs per SM hold every (request, head) warp of a 128 x 32 step at once)
__global__ void __launch_bounds__(kMergeWarps * 32, 7) merge_kernel(MergeParams p) {
  const int lane = threadIdx.x & 31;
  const int item = blockIdx.x * kMergeWarps + (threadIdx.x >> 5);
  const bool active = item < p.num_requests * p.num_q_heads;
  const int request = active ? item / p.num_q_heads : 0, head = active ? item % p.num_q_heads : 0;

  // The count and the slot list are plan metadata, which no kernel writes: they
  // are loaded before waiting for the segment kernels (slot loads past the
  // count are discarded), so after the wait the chain is LSEs -> rows.
  const int32_t* slots = p.cslots + int64_t(request) * p.max_slots;
  int count = active ? p.counts[request] : 0;
  const int pre_slot = active && lane < p.max_slots ? slots[lane] : -1;
  pdl_wait();                // the segment kernels before this one have completed
  pdl_trigger();             // the next step's query-tile kernel may set up meanwhile (it waits before any data)
  if (!active) return;
  merge_one<T, D>(p, request, head, count, pre_slot, lane);
}

// Requests with many partials (a plan whose long segments were cut into many
// pieces, e.g. one KV head per GPU): one CTA of kSplitWarps warps per
// (request, query head).  Warp w merges partials w, w + kSplitWarps, ... with
// its own running maximum; the warps' results are then combined through
// shared memory, so the latency chain per warp is a quarter as long.
constexpr int kSplitWarps = 4;
constexpr int kSplitAbove = 24;      // most partials of any request above which the split kernel runs (measured: 19 slower, 33 faster)

template <typename T, int D>
__global__ void __launch_bounds__(kSplitWarps * 32) merge_split_kernel(MergeParams p) {
  constexpr int DL = D / 32;
  __shared__ float s_acc[kSplitWarps][D];
  __shared__ float s_m[kSplitWarps], s_z[kSplitWarps];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int item = blockIdx.x;                       // the grid is exactly requests x query heads
  const int request = item / p.num_q_heads, head = item % p.num_q_heads;
  const int G = p.group, kv_head = head / G, g = head % G;
  const int32_t* slots = p.cslots + int64_t(request) * p.max_slots;
  int count = p.counts[request];                     // plan metadata: loaded before the wait
  pdl_wait();
  pdl_trigger();
  if (count < 0 || count > p.max_slots) {
    if (threadIdx.x == 0) set_status(p.status, TA_ERR_BOUNDS);
    count = 0;
  }
  const int64_t head_rows = int64_t(kv_head) * p.num_partials;
  const int mine = count > w ? (count - w + kSplitWarps - 1) / kSplitWarps : 0;   // this warp's partials

  float acc[DL];
#pragma unroll
  for (int e = 0; e < DL; ++e) acc[e] = 0.f;
  float m = -INFINITY, z = 0.f;
  for (int i0 = 0; i0 < mine; i0 += 32) {
    const int i = i0 + lane;                         // lane holds this warp's partial i: k = w + kSplitWarps * i
    float l = -INFINITY;
    int64_t row = 0;
    if (i < mine) {
      const int s = slots[w + kSplitWarps * i];
      if (s >= 0 && s < p.num_partials) {
        row = (head_rows + s) * G + g;
        l = p.lse[row];
      } else {
        set_status(p.status, TA_ERR_BOUNDS);
      }
    }
    const float m_new = fmaxf(m, warp_max(l));
    if (m_new == -INFINITY) continue;
    const float scale = fast_exp2((m - m_new) * kLog2e);
    z *= scale;
#pragma unroll
    for (int e = 0; e < DL; ++e) acc[e] *= scale;
    m = m_new;
    const float wgt = fast_exp2((l - m) * kLog2e);
    z += warp_sum(wgt);
    const int n = min(32, mine - i0);
    for (int j = 0; j < n; j += 8) {
      float wj[8];
      float x[8][DL];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int src = min(j + u, n - 1);
        wj[u] = __shfl_sync(0xffffffffu, wgt, src);
        const int64_t rj = __shfl_sync(0xffffffffu, row, src);
        if (j + u >= n) wj[u] = 0.f;
        const float* ptr = p.part + rj * D + lane * DL;
#pragma unroll
        for (int e = 0; e < DL; ++e) x[u][e] = 0.f;
        if (wj[u] != 0.f) {                  // an empty partial (weight 0) may hold anything
          if constexpr (DL == 4) {
            const float4 v = *reinterpret_cast<const float4*>(ptr);
            x[u][0] = v.x; x[u][1] = v.y; x[u][2] = v.z; x[u][3] = v.w;
          } else {
#pragma unroll
            for (int e = 0; e < DL; ++e) x[u][e] = ptr[e];
          }
        }
      }
#pragma unroll
      for (int u = 0; u < 8; ++u)
#pragma unroll
        for (int e = 0; e < DL; ++e) acc[e] = fmaf(wj[u], x[u][e], acc[e]);
    }
  }
  if (lane == 0) {
    s_m[w] = m;
    s_z[w] = z;
  }
#pragma unroll
  for (int e = 0; e < DL; ++e) s_acc[w][lane * DL + e] = acc[e];
  __syncthreads();
  if (w != 0) return;
  float mm = s_m[0];
#pragma unroll
  for (int v = 1; v < kSplitWarps; ++v) mm = fmaxf(mm, s_m[v]);
  float zz = 0.f, a[DL];
#pragma unroll
  for (int e = 0; e < DL; ++e) a[e] = 0.f;
  if (mm != -INFINITY) {
#pragma unroll
    for (int v = 0; v < kSplitWarps; ++v) {
      const float f = fast_exp2((s_m[v] - mm) * kLog2e);   // a warp with no live partial: -inf gives 0
      zz += f * s_z[v];
#pragma unroll
      for (int e = 0; e < DL; ++e) a[e] += f * s_acc[v][lane * DL + e];
    }
  }
  const float inv = zz > 0.f ? 1.f / zz : 0.f;
  uint16_t* out = reinterpret_cast<uint16_t*>(p.out) + (int64_t(request) * p.num_q_heads + head) * D + lane * DL;
#pragma unroll
  for (int e = 0; e < DL; ++e) out[e] = Elem<T>::from_float(a[e] * inv);
  if (p.out_lse && lane == 0)
    p.out_lse[int64_t(request) * p.num_q_heads + head] = zz > 0.f ? mm + fast_log2(zz) * kLn2 : -INFINITY;
}

__global__ void fill_klen_kernel(int32_t* klen, const int32_t* idx, int n, int value, int num_jobs,
                                 int32_t* status) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int j = idx[i];
  if (j < 0 || j >= num_jobs) {
    set_status(status, TA_ERR_BOUNDS);
    return;
  }
  klen[j] = value;
}

template <typename T, int D>
cudaError_t launch_merge_typed(const MergeParams& p, cudaStream_t stream) {
  const int items = p.num_requests * p.num_q_heads;
  if (items == 0) return cudaSuccess;
  cudaError_t err;
  if (p.max_slots > kSplitAbove) {
    err = launch_dependent(merge_split_kernel<T, D>, dim3(items), dim3(kSplitWarps * 32), 0, stream, p);
  } else {
    const int blocks = (items + kMergeWarps - 1) / kMergeWarps;
    err = launch_dependent(merge_kernel<T, D>, dim3(blocks), dim3(kMergeWarps * 32), 0, stream, p);
  }
  if (err != cudaSuccess) return err;
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_merge(const MergeParams& p, int head_dim, int dtype, cudaStream_t stream) {
  if (dtype == TA_DTYPE_BF16) {
    if (head_dim == 128) return launch_merge_typed<__nv_bfloat16, 128>(p, stream);
    if (head_dim == 64) return launch_merge_typed<__nv_bfloat16, 64>(p, stream);
    if (head_dim == 32) return launch_merge_typed<__nv_bfloat16, 32>(p, stream);
  } else if (dtype == TA_DTYPE_F16) {
    if (head_dim == 128) return launch_merge_typed<__half, 128>(p, stream);
    if (head_dim == 64) return launch_merge_typed<__half, 64>(p, stream);
    if (head_dim == 32) return launch_merge_typed<__half, 32>(p, stream);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_fill_klen(int32_t* klen, const int32_t* idx, int n, int value, int num_jobs, int32_t* status,
                             cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  fill_klen_kernel<<<(n + 127) / 128, 128, 0, stream>>>(klen, idx, n, value, num_jobs, status);
  return cudaGetLastError();
}

}  // namespace ta
