// Segment attention for small groups (<= 16 query rows per job x KV head).
//
// Work of one CTA: one (job, 16-row tile, KV head).  The job's key rows are a
// contiguous run of the token-major pool, so each 64-key chunk of K and of V is
// ONE 1-D bulk copy (cp.async.bulk, no multicast) into shared memory, double
// buffered on two mbarriers.  The arithmetic is HBM-bound (4 rows x 128 dims
// per 512 bytes of KV for a private request), so it stays on the FP32 pipe:
//   scores   lanes split head_dim; a warp transpose-reduction turns 32 lane
//            partials into 32 (row, key) dot products with 31 shuffles;
//   softmax  per row over the chunk, exp2 on pre-scaled scores, running max /
//            denominator in shared memory (online softmax across chunks);
//   P.V      lanes split head_dim; each warp accumulates its keys, the four
//            warps are summed once at the end.
// Output: softmax-normalised partial O (f32) and natural-log LSE per row, as
// the reference's _segment kernel (kernels.py:8-55) writes them.
#include "ta_common.cuh"
#include "ta_kernels.cuh"

namespace ta {

namespace {

constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kChunk = 64;           // keys per chunk
constexpr int kKeysPerWarp = kChunk / kWarps;
constexpr int kStages = 2;

template <int D, int R>
struct SimtSmem {
  static constexpr int kSPitch = kChunk + 4;
  static constexpr size_t kv_bytes = size_t(kStages) * kChunk * D * 2;  // one of K / V
  static constexpr size_t off_k = 0;
  static constexpr size_t off_v = off_k + kv_bytes;
  static constexpr size_t off_s = off_v + kv_bytes;                    // [R][kSPitch] f32
  static constexpr size_t off_p = off_s + size_t(R) * kSPitch * 4;     // [kChunk][R] f32
  static constexpr size_t off_m = off_p + size_t(kChunk) * R * 4;      // [R] running max (log2)
  static constexpr size_t off_z = off_m + R * 4;                       // [R] denominators
  static constexpr size_t off_a = off_z + R * 4;                       // [R] chunk rescale
  static constexpr size_t off_bar = (off_a + R * 4 + 15) / 16 * 16;    // [kStages] mbarriers
  static constexpr size_t bytes = off_bar + kStages * 8;
  static_assert(size_t(kWarps) * R * D * 4 <= 2 * kv_bytes, "final reduction reuses the KV buffers");
};

template <typename T, int D>
__device__ __forceinline__ void load_slice(const uint16_t* base, float (&x)[D / 32]) {
  constexpr int DL = D / 32;
  if constexpr (DL == 4) {
    uint2 raw = *reinterpret_cast<const uint2*>(base);
    float2 a = Elem<T>::to_float2(raw.x), b = Elem<T>::to_float2(raw.y);
    x[0] = a.x; x[1] = a.y; x[2] = b.x; x[3] = b.y;
  } else if constexpr (DL == 2) {
    float2 a = Elem<T>::to_float2(*reinterpret_cast<const uint32_t*>(base));
    x[0] = a.x; x[1] = a.y;
  } else {
    x[0] = Elem<T>::to_float(*base);
  }
}

template <typename T, int D, int R>
__global__ void __launch_bounds__(kThreads) seg_simt_kernel(SegParams p, int task_begin) {
  using L = SimtSmem<D, R>;
  constexpr int DL = D / 32;
  constexpr int KB = 32 / R;                  // keys per transpose-reduction batch
  static_assert(32 % R == 0 && kKeysPerWarp % KB == 0, "row padding must divide the warp");

  extern __shared__ __align__(128) unsigned char smem[];
  uint16_t* k_s = reinterpret_cast<uint16_t*>(smem + L::off_k);
  uint16_t* v_s = reinterpret_cast<uint16_t*>(smem + L::off_v);
  float* s_s = reinterpret_cast<float*>(smem + L::off_s);
  float* p_s = reinterpret_cast<float*>(smem + L::off_p);
  float* m_s = reinterpret_cast<float*>(smem + L::off_m);
  float* z_s = reinterpret_cast<float*>(smem + L::off_z);
  float* a_s = reinterpret_cast<float*>(smem + L::off_a);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::off_bar);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int task = task_begin + blockIdx.x;
  const int head = blockIdx.y;
  const int G = p.group;

  const int job = p.small_tasks[2 * task];
  const int tile = p.small_tasks[2 * task + 1];
  if (job < 0 || job >= p.num_jobs) {
    if (tid == 0) set_status(p.status, TA_ERR_BOUNDS);
    return;
  }
  const int nr = p.qlen[job];
  int nk = p.klen[job];
  const int64_t k0 = p.kstart[int64_t(job) * p.kstart_stride];
  const int r0 = tile * 16;
  const int rows = min(R, nr * G - r0);
  const int64_t part_row0 = int64_t(p.slot_base[job]) * G + r0;
  bool bad = nr < 0 || nr > p.max_requests || rows <= 0 || nk < 0 || k0 < 0 || k0 + nk > p.pool_tokens ||
             part_row0 < 0 || part_row0 + rows > int64_t(p.num_partials) * G;
  if (bad) {
    if (tid == 0) set_status(p.status, TA_ERR_BOUNDS);
    if (rows <= 0 || part_row0 < 0 || part_row0 + rows > int64_t(p.num_partials) * G) return;
    nk = 0;  // rows are addressable: publish an empty partial (O = 0, LSE = -inf)
  }

  // Query slice of every row, pre-scaled into the log2 domain.
  float qr[R][DL];
#pragma unroll
  for (int r = 0; r < R; ++r) {
#pragma unroll
    for (int e = 0; e < DL; ++e) qr[r][e] = 0.f;
    if (r < rows) {
      const int row = r0 + r;
      const int rid = p.qids[int64_t(job) * p.max_requests + row / G];
      if (rid >= 0 && rid < p.num_requests) {
        const uint16_t* src = p.q + (int64_t(rid) * p.num_q_heads + head * G + row % G) * D + lane * DL;
        load_slice<T, D>(src, qr[r]);
#pragma unroll
        for (int e = 0; e < DL; ++e) qr[r][e] *= p.scale_log2;
      } else if (lane == 0) {
        set_status(p.status, TA_ERR_BOUNDS);
      }
    }
  }

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) mbar_init(&bars[s], 1);
    fence_barrier_init();
  }
  if (tid < R) {
    m_s[tid] = -INFINITY;
    z_s[tid] = 0.f;
  }
  __syncthreads();

  const int nchunks = (nk + kChunk - 1) / kChunk;
  const uint16_t* kbase = p.k + (int64_t(head) * p.pool_tokens + k0) * D;
  const uint16_t* vbase = p.v + (int64_t(head) * p.pool_tokens + k0) * D;
  auto issue = [&](int c) {
    const int keys = min(kChunk, nk - c * kChunk);
    const uint32_t bytes = uint32_t(keys) * D * 2;
    const int st = c % kStages;
    mbar_arrive_expect_tx(&bars[st], 2 * bytes);
    bulk_g2s(k_s + size_t(st) * kChunk * D, kbase + int64_t(c) * kChunk * D, bytes, &bars[st]);
    bulk_g2s(v_s + size_t(st) * kChunk * D, vbase + int64_t(c) * kChunk * D, bytes, &bars[st]);
  };
  if (tid == 0) {
    for (int c = 0; c < min(nchunks, kStages); ++c) issue(c);
  }

  float acc[R][DL];
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int e = 0; e < DL; ++e) acc[r][e] = 0.f;

  bool alive = true;
  for (int c = 0; c < nchunks; ++c) {
    const int st = c % kStages;
    const int keys = min(kChunk, nk - c * kChunk);
    if (!mbar_wait(&bars[st], (c / kStages) & 1, p.status)) alive = false;
    if (__syncthreads_or(!alive)) {
      alive = false;
      break;
    }
    const uint16_t* kc = k_s + size_t(st) * kChunk * D;
    const uint16_t* vc = v_s + size_t(st) * kChunk * D;

    // -- scores: warp `warp` owns keys [16*warp, 16*warp + 16) of the chunk
#pragma unroll
    for (int b = 0; b < kKeysPerWarp / KB; ++b) {
      const int kb = warp * kKeysPerWarp + b * KB;
      float part[32];
#pragma unroll
      for (int kk = 0; kk < KB; ++kk) {
        float kx[DL];
        load_slice<T, D>(kc + (kb + kk) * D + lane * DL, kx);
#pragma unroll
        for (int r = 0; r < R; ++r) {
          float s = 0.f;
#pragma unroll
          for (int e = 0; e < DL; ++e) s = fmaf(qr[r][e], kx[e], s);
          part[kk * R + r] = s;
        }
      }
      const float dot = warp_transpose_sum32(part, lane);
      const int key = kb + lane / R, r = lane % R;
      s_s[r * L::kSPitch + key] = key < keys ? dot : -INFINITY;
    }
    __syncthreads();

    // -- online softmax, one warp per row (rows warp, warp+4, ...)
    for (int r = warp; r < R; r += kWarps) {
      const float s0 = s_s[r * L::kSPitch + lane];
      const float s1 = s_s[r * L::kSPitch + lane + 32];
      const float m_old = m_s[r];
      const float m_new = fmaxf(m_old, warp_max(fmaxf(s0, s1)));
      const float base = m_new == -INFINITY ? 0.f : m_new;
      const float p0 = fast_exp2(s0 - base), p1 = fast_exp2(s1 - base);
      p_s[lane * R + r] = p0;
      p_s[(lane + 32) * R + r] = p1;
      const float sum = warp_sum(p0 + p1);
      if (lane == 0) {
        const float alpha = fast_exp2(m_old - base);  // m_old = -inf gives 0
        a_s[r] = alpha;
        z_s[r] = z_s[r] * alpha + sum;
        m_s[r] = m_new;
      }
    }
    __syncthreads();

    // -- P.V: warp owns the same 16 keys, lanes split head_dim
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const float alpha = a_s[r];
#pragma unroll
      for (int e = 0; e < DL; ++e) acc[r][e] *= alpha;
    }
    const int kend = min(keys, (warp + 1) * kKeysPerWarp);
    for (int key = warp * kKeysPerWarp; key < kend; ++key) {
      float vx[DL];
      load_slice<T, D>(vc + key * D + lane * DL, vx);
      const float4* prow = reinterpret_cast<const float4*>(p_s + key * R);
#pragma unroll
      for (int r4 = 0; r4 < R / 4; ++r4) {
        const float4 pv = prow[r4];
        const float pr[4] = {pv.x, pv.y, pv.z, pv.w};
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
          for (int e = 0; e < DL; ++e) acc[r4 * 4 + j][e] = fmaf(pr[j], vx[e], acc[r4 * 4 + j][e]);
      }
    }
    __syncthreads();  // stage `st` and s_s / p_s are free again
    if (tid == 0 && c + kStages < nchunks) issue(c + kStages);
  }

  // -- sum the four warps' accumulators (reusing the KV buffers) and publish
  float* red = reinterpret_cast<float*>(smem + L::off_k);
  if (alive) {
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int e = 0; e < DL; ++e) red[(warp * R + r) * D + lane * DL + e] = acc[r][e];
  }
  __syncthreads();
  for (int i = tid; i < rows * D; i += kThreads) {
    const int r = i / D, d = i % D;
    float o = 0.f;
    const float z = z_s[r];
    if (alive && z > 0.f) {
      o = red[(0 * R + r) * D + d] + red[(1 * R + r) * D + d] + red[(2 * R + r) * D + d] +
          red[(3 * R + r) * D + d];
      o /= z;
    }
    p.part[(int64_t(head) * p.num_partials * G + part_row0 + r) * D + d] = o;
  }
  if (tid < rows) {
    const float z = z_s[tid];
    const float l = (alive && z > 0.f) ? (m_s[tid] + fast_log2(z)) * kLn2 : -INFINITY;
    p.lse[int64_t(head) * p.num_partials * G + part_row0 + tid] = l;
  }
}

}  // namespace

template <typename T, int D, int R>
static cudaError_t launch_simt_class(const SegParams& p, int begin, int count, cudaStream_t stream) {
  if (count <= 0) return cudaSuccess;
  using L = SimtSmem<D, R>;
  auto kernel = seg_simt_kernel<T, D, R>;
  static bool configured = false;  // the attribute is per function and persists
  if (!configured) {
    cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(L::bytes));
    if (err != cudaSuccess) return err;
    configured = true;
  }
  dim3 grid(count, p.num_kv_heads);
  kernel<<<grid, kThreads, L::bytes, stream>>>(p, begin);
  return cudaGetLastError();
}

template <typename T, int D>
static cudaError_t launch_simt_dim(const SegParams& p, const int32_t class_end[3], cudaStream_t stream) {
  cudaError_t err = launch_simt_class<T, D, 4>(p, 0, class_end[0], stream);
  if (err == cudaSuccess) err = launch_simt_class<T, D, 8>(p, class_end[0], class_end[1] - class_end[0], stream);
  if (err == cudaSuccess) err = launch_simt_class<T, D, 16>(p, class_end[1], class_end[2] - class_end[1], stream);
  return err;
}

cudaError_t launch_seg_simt(const SegParams& p, const int32_t class_end[3], int head_dim, int dtype,
                            cudaStream_t stream) {
  if (dtype == TA_DTYPE_BF16) {
    if (head_dim == 128) return launch_simt_dim<__nv_bfloat16, 128>(p, class_end, stream);
    if (head_dim == 64) return launch_simt_dim<__nv_bfloat16, 64>(p, class_end, stream);
    if (head_dim == 32) return launch_simt_dim<__nv_bfloat16, 32>(p, class_end, stream);
  } else if (dtype == TA_DTYPE_F16) {
    if (head_dim == 128) return launch_simt_dim<__half, 128>(p, class_end, stream);
    if (head_dim == 64) return launch_simt_dim<__half, 64>(p, class_end, stream);
    if (head_dim == 32) return launch_simt_dim<__half, 32>(p, class_end, stream);
  }
  return cudaErrorInvalidValue;
}

}  // namespace ta
