// Segment attention for small groups (<= 16 query rows per job x KV head).
//
// Work of one CTA: one (job, 16-row tile, KV head).  The job's key rows are a
// contiguous run of the token-major pool, so each 64-key chunk of K and of V is
// ONE 1-D bulk copy (cp.async.bulk, no multicast) into shared memory.  The
// arithmetic is HBM-bound (4 rows x 128 dims per 512 bytes of KV for a private
// request), so it stays on the FP32 pipe, and every warp runs its own online
// softmax over its quarter of each chunk -- no CTA-wide barrier per chunk:
//   scores   lanes split head_dim; a warp transpose-reduction turns 32 lane
//            partials into 32 (key, row) dot products with 31 shuffles
//   softmax  row max / sum over the warp's keys by shuffles within the lanes
//            that hold the same row; exp2 on pre-scaled scores
//   P.V      lanes split head_dim; p broadcast by shuffles
// The four warps' (max, sum, accumulator) are merged once at the end with the
// same log-sum-exp rule as the global merge.  Chunks live in STAGES shared
// buffers (one when every task fits one chunk, two otherwise), refilled by
// thread 0 once all warps have released the buffer on its EMPTY mbarrier.
// Output: softmax-normalised partial O (f32) and natural-log LSE per row, as
// the reference's _segment kernel (kernels.py:8-55) writes them.
#include "ta_common.cuh"
#include "ta_kernels.cuh"

namespace ta {

namespace {

constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kChunk = 64;                 // keys per chunk
constexpr int kKeysPerWarp = kChunk / kWarps;

template <int D, int R, int STAGES>
struct SimtSmem {
  static constexpr size_t stage_bytes = size_t(kChunk) * D * 2 * 2;   // K and V of one chunk
  static constexpr size_t off_stage = 0;
  static constexpr size_t off_mz = off_stage + STAGES * stage_bytes;   // [4 warps][R] max, then sum
  static constexpr size_t off_bar = (off_mz + 2 * kWarps * R * 4 + 15) / 16 * 16;
  static constexpr size_t bytes = off_bar + (2 * STAGES + 1) * 8;        // full, empty, never
  static_assert(size_t(kWarps) * R * D * 4 <= STAGES * stage_bytes, "warp combine reuses the chunk buffers");
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

template <typename T, int D, int R, int STAGES>
__global__ void __launch_bounds__(kThreads) seg_simt_kernel(SegParams p, int task_begin) {
  using L = SimtSmem<D, R, STAGES>;
  constexpr int DL = D / 32;
  constexpr int KB = 32 / R;                           // keys per transpose-reduction batch
  constexpr int NB = kKeysPerWarp / KB;                // batches per warp and chunk
  static_assert(32 % R == 0 && kKeysPerWarp % KB == 0, "row padding must divide the warp");

  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::off_bar);
  uint64_t* empty = full + STAGES;
  uint64_t* never = empty + STAGES;                    // a barrier nothing arrives on (p.test_stall)
  float* mz = reinterpret_cast<float*>(smem + L::off_mz);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int task = task_begin + blockIdx.x;
  const int head = blockIdx.y;
  const int G = p.group;

  const int piece = p.small_tasks[2 * task];
  const int tile = p.small_tasks[2 * task + 1];
  Piece pc;
  const int state = resolve_piece(p, piece, pc);
  const int r0 = tile * 16;
  const int rows = state == PIECE_SKIP ? 0 : min(R, pc.nr * G - r0);
  if (rows <= 0) {
    if (tid == 0) set_status(p.status, TA_ERR_BOUNDS);
    return;
  }
  if (state == PIECE_BAD_KEYS && tid == 0) set_status(p.status, TA_ERR_BOUNDS);
  const int job = pc.job;
  const int nk = pc.nk;
  const int64_t k0 = pc.k0;
  const int64_t part_row0 = pc.slot * G + r0;
  const int nchunks = (nk + kChunk - 1) / kChunk;
  const uint16_t* kbase = p.k + (int64_t(head) * p.pool_tokens + k0) * D;
  const uint16_t* vbase = p.v + (int64_t(head) * p.pool_tokens + k0) * D;
  auto stage_k = [&](int s) { return reinterpret_cast<uint16_t*>(smem + L::off_stage + s * L::stage_bytes); };
  auto stage_v = [&](int s) { return stage_k(s) + kChunk * D; };
  int issued = 0;                                      // thread 0: chunks issued
  auto issue = [&](int c) {
    ++issued;
    const int keys = min(kChunk, nk - c * kChunk);
    const uint32_t bytes = uint32_t(keys) * D * 2;
    const int st = c % STAGES;
    mbar_arrive_expect_tx(&full[st], 2 * bytes);
    bulk_g2s(stage_k(st), kbase + int64_t(c) * kChunk * D, bytes, &full[st]);
    bulk_g2s(stage_v(st), vbase + int64_t(c) * kChunk * D, bytes, &full[st]);
  };

  // Thread 0 starts the KV stream before anything else.
  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kWarps);
    }
    mbar_init(never, 1);
    fence_barrier_init();
    for (int c = 0; c < min(nchunks, STAGES); ++c) issue(c);
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
  __syncthreads();  // barrier initialisation is visible to every warp

  // Per-warp online softmax state.  Lane l holds the state of row l % R.
  float m_run = -INFINITY, z_run = 0.f;
  float acc[R][DL];
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int e = 0; e < DL; ++e) acc[r][e] = 0.f;

  bool alive = true;
  int consumed = 0;                                    // chunks whose copies this warp saw land
  for (int c = 0; c < nchunks; ++c) {
    const int st = c % STAGES;
    const int keys = min(kChunk, nk - c * kChunk);
    // Test hook: wait on a barrier that nothing completes, so the bounded wait
    // gives up with TA_ERR_TIMEOUT and the error path below runs.
    if (p.test_stall && c == 0) alive = __all_sync(0xffffffffu, mbar_wait(never, 0, p.status));
    if (!alive) break;
    alive = __all_sync(0xffffffffu, mbar_wait(&full[st], (c / STAGES) & 1, p.status));
    if (!alive) break;
    consumed = c + 1;
    const uint16_t* kc = stage_k(st);
    const uint16_t* vc = stage_v(st);
    const int kw = warp * kKeysPerWarp;                  // this warp's first key in the chunk

    // -- scores of this warp's 16 keys: s[b] for key kw + b*KB + lane/R, row lane%R
    float s[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      const int kb = kw + b * KB;
      float part[32];
#pragma unroll
      for (int kk = 0; kk < KB; ++kk) {
        float kx[DL];
        load_slice<T, D>(kc + (kb + kk) * D + lane * DL, kx);
#pragma unroll
        for (int r = 0; r < R; ++r) {
          float acc_s = 0.f;
#pragma unroll
          for (int e = 0; e < DL; ++e) acc_s = fmaf(qr[r][e], kx[e], acc_s);
          part[kk * R + r] = acc_s;
        }
      }
      const float dot = warp_transpose_sum32(part, lane);
      s[b] = (kb + lane / R < keys) ? dot : -INFINITY;
    }

    // -- row max / sum within the lanes holding the same row (lane % R)
    float mx = s[0];
#pragma unroll
    for (int b = 1; b < NB; ++b) mx = fmaxf(mx, s[b]);
#pragma unroll
    for (int off = R; off < 32; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    const float m_new = fmaxf(m_run, mx);
    const float base = m_new == -INFINITY ? 0.f : m_new;
    const float alpha = fast_exp2(m_run - base);          // m_run = -inf gives 0
    float sum = 0.f;
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      s[b] = fast_exp2(s[b] - base);                       // now p
      sum += s[b];
    }
#pragma unroll
    for (int off = R; off < 32; off <<= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
    z_run = z_run * alpha + sum;
    m_run = m_new;

    // -- P.V over this warp's keys; lanes split head_dim
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const float a_r = __shfl_sync(0xffffffffu, alpha, r);
#pragma unroll
      for (int e = 0; e < DL; ++e) acc[r][e] *= a_r;
    }
#pragma unroll
    for (int b = 0; b < NB; ++b) {
#pragma unroll
      for (int kk = 0; kk < KB; ++kk) {
        const int key = kw + b * KB + kk;
        if (key < keys) {                                  // warp-uniform
          float vx[DL];
          load_slice<T, D>(vc + key * D + lane * DL, vx);
#pragma unroll
          for (int r = 0; r < R; ++r) {
            const float pr = __shfl_sync(0xffffffffu, s[b], kk * R + r);
#pragma unroll
            for (int e = 0; e < DL; ++e) acc[r][e] = fmaf(pr, vx[e], acc[r][e]);
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
    if (tid == 0 && c + STAGES < nchunks) {
      // refill this buffer once every warp has released it
      if (mbar_wait(&empty[st], (c / STAGES) & 1, p.status)) issue(c + STAGES);
    }
  }

  // -- combine the four warps (reusing the chunk buffers) and publish.  After
  // a wait gave up, copies may still be in flight: they must land before the
  // buffers are reused or the CTA exits.  Thread 0 waits (bounded) for every
  // chunk it issued past the ones its warp saw land.  (Each warp reconverges
  // before a CTA-wide barrier.)
  __syncwarp();
  __syncthreads();
  if (tid == 0)
    for (int c = consumed; c < issued; ++c) mbar_wait(&full[c % STAGES], (c / STAGES) & 1, p.status);
  __syncwarp();
  __syncthreads();
  float* red = reinterpret_cast<float*>(smem + L::off_stage);
  if (lane < R) {
    mz[warp * R + lane] = alive ? m_run : -INFINITY;
    mz[kWarps * R + warp * R + lane] = alive ? z_run : 0.f;
  }
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int e = 0; e < DL; ++e) red[(warp * R + r) * D + lane * DL + e] = acc[r][e];
  __syncthreads();
  for (int i = tid; i < rows * D; i += kThreads) {
    const int r = i / D, d = i % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, mz[w * R + r]);
    float o = 0.f, zt = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        const float wgt = fast_exp2(mz[w * R + r] - M);   // -inf max (no keys) gives 0
        o = fmaf(wgt, red[(w * R + r) * D + d], o);
        zt = fmaf(wgt, mz[kWarps * R + w * R + r], zt);
      }
    }
    p.part[(int64_t(head) * p.num_partials * G + part_row0 + r) * D + d] = zt > 0.f ? o / zt : 0.f;
  }
  if (tid < rows) {
    const int r = tid;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, mz[w * R + r]);
    float zt = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kWarps; ++w) zt = fmaf(fast_exp2(mz[w * R + r] - M), mz[kWarps * R + w * R + r], zt);
    }
    p.lse[int64_t(head) * p.num_partials * G + part_row0 + r] = zt > 0.f ? (M + fast_log2(zt)) * kLn2 : -INFINITY;
  }
}

}  // namespace

template <typename T, int D, int R, int STAGES>
static cudaError_t launch_simt_class(const SegParams& p, int begin, int count, cudaStream_t stream) {
  if (count <= 0) return cudaSuccess;
  using L = SimtSmem<D, R, STAGES>;
  auto kernel = seg_simt_kernel<T, D, R, STAGES>;
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

template <typename T, int D, int STAGES>
static cudaError_t launch_simt_stages(const SegParams& p, const int32_t class_end[3], cudaStream_t stream) {
  cudaError_t err = launch_simt_class<T, D, 4, STAGES>(p, 0, class_end[0], stream);
  if (err == cudaSuccess)
    err = launch_simt_class<T, D, 8, STAGES>(p, class_end[0], class_end[1] - class_end[0], stream);
  if (err == cudaSuccess)
    err = launch_simt_class<T, D, 16, STAGES>(p, class_end[1], class_end[2] - class_end[1], stream);
  return err;
}

template <typename T, int D>
static cudaError_t launch_simt_dim(const SegParams& p, const int32_t class_end[3], int max_keys, cudaStream_t stream) {
  // One buffer suffices when every task fits one chunk (leaves, short tails);
  // longer tasks double-buffer so the next chunk streams during compute.
  if (max_keys <= kChunk) return launch_simt_stages<T, D, 1>(p, class_end, stream);
  return launch_simt_stages<T, D, 2>(p, class_end, stream);
}

cudaError_t launch_seg_simt(const SegParams& p, const int32_t class_end[3], int max_keys, int head_dim, int dtype,
                            cudaStream_t stream) {
  if (dtype == TA_DTYPE_BF16) {
    if (head_dim == 128) return launch_simt_dim<__nv_bfloat16, 128>(p, class_end, max_keys, stream);
    if (head_dim == 64) return launch_simt_dim<__nv_bfloat16, 64>(p, class_end, max_keys, stream);
    if (head_dim == 32) return launch_simt_dim<__nv_bfloat16, 32>(p, class_end, max_keys, stream);
  } else if (dtype == TA_DTYPE_F16) {
    if (head_dim == 128) return launch_simt_dim<__half, 128>(p, class_end, max_keys, stream);
    if (head_dim == 64) return launch_simt_dim<__half, 64>(p, class_end, max_keys, stream);
    if (head_dim == 32) return launch_simt_dim<__half, 32>(p, class_end, max_keys, stream);
  }
  return cudaErrorInvalidValue;
}

}  // namespace ta
