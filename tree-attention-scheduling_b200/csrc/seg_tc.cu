// Segment attention for large groups on the 5th-generation tensor cores.
//
// Work of one CTA: one (job, 128-row query tile, KV head).  The query tile
// stacks the GQA rows of up to 32 requests that share the job's KV segment, so
// S = Q K^T and O = P V are dense 128 x 128 x 128 contractions per 128-key tile:
//
//   warp 0      TMA producer: K and V tiles (token-major pools, 2 x 64-column
//               boxes with 128-byte swizzle, no multicast), 2-stage ring
//   warp 1      TMEM owner + MMA issuer: tcgen05.mma kind::f16, A and B from
//               shared memory, S double-buffered in TMEM, O accumulated in TMEM
//   warps 2-5   softmax: one query row per thread (TMEM lane), S read with
//               tcgen05.ld, exp2 on pre-scaled scores, P written to shared
//               memory as bf16/f16 in the canonical K-major 128B-swizzle layout;
//               O is rescaled in TMEM only when a row's running max grows by
//               more than 2^8 (otherwise the stale max is kept, which is exact
//               after the final division); epilogue O / z and the LSE.
//
// TMEM columns: [0,128) S0, [128,256) S1, [256,384) O.  Shared memory: Q 32 KB,
// K 2 x 32 KB, V 2 x 32 KB, P 32 KB.  All waits are bounded (ta_common.cuh).
//
// The reference's _segment (kernels.py:8-55) computes the same partial O / LSE
// with Triton tiles of 64 query rows x 64 keys.
#include <cstring>
#include <mutex>

#include "ta_common.cuh"
#include "ta_kernels.cuh"

namespace ta {

namespace {

constexpr int kRows = 128;      // query rows per CTA (MMA M)
constexpr int kKeys = 128;      // keys per tile (MMA N of S, K of P.V)
constexpr int kDim = 128;       // head_dim (MMA K of S, N of P.V)
constexpr int kStages = 2;
constexpr int kThreads = 192;
constexpr uint32_t kTileBytes = kKeys * kDim * 2;       // 32 KB per K or V tile
constexpr uint32_t kHalfBytes = kTileBytes / 2;         // one 64-column swizzled block
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS0 = 0, kColO = 256;
constexpr float kRescaleThreshold = 8.0f;               // log2 units

struct TcSmem {
  static constexpr uint32_t off_q = 0;
  static constexpr uint32_t off_k = off_q + kTileBytes;
  static constexpr uint32_t off_v = off_k + kStages * kTileBytes;
  static constexpr uint32_t off_p = off_v + kStages * kTileBytes;
  static constexpr uint32_t off_bar = off_p + kTileBytes;
  // barriers: k_full[2], v_full[2], kv_empty[2], s_full[2], s_free[2], q_full, p_full, pv_done
  static constexpr int kBars = 13;
  static constexpr uint32_t off_tmem = off_bar + kBars * 8;
  static constexpr uint32_t bytes = off_tmem + 16;
  static constexpr uint32_t alloc = bytes + 1024;         // slack to align the base to 1 KB
};

enum Bar { K_FULL = 0, V_FULL = 2, KV_EMPTY = 4, S_FULL = 6, S_FREE = 8, Q_FULL = 10, P_FULL = 11, PV_DONE = 12 };

// ---- UMMA descriptors -------------------------------------------------------
// Shared-memory matrix descriptor (sm_100): start>>4 [0,14), LBO>>4 [16,30),
// SBO>>4 [32,46), version 1 [46,48), base offset 0, layout [61,64) = 2 (128B swizzle).
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= uint64_t((addr >> 4) & 0x3fff);
  d |= uint64_t((lbo >> 4) & 0x3fff) << 16;
  d |= uint64_t((sbo >> 4) & 0x3fff) << 32;
  d |= uint64_t(1) << 46;
  d |= uint64_t(2) << 61;
  return d;
}

// Instruction descriptor, kind::f16: D f32, A/B f16 (0) or bf16 (1), both
// operands from shared memory, M = 128, N = 128; b_mn_major selects an
// N-contiguous B (the V tile).
__host__ __device__ constexpr uint32_t instr_desc(uint32_t ab_format, uint32_t b_mn_major) {
  return (1u << 4) | (ab_format << 7) | (ab_format << 10) | (b_mn_major << 16) | ((uint32_t(kKeys) >> 3) << 17) |
         ((uint32_t(kRows) >> 4) << 24);
}

__device__ __forceinline__ void umma(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
      ::"r"(d_tmem), "l"(a), "l"(b), "r"(idesc), "r"(acc), "r"(0), "r"(0), "r"(0), "r"(0));
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// 32 consecutive f32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};"
      ::"r"(taddr), "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
        "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
        "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
        "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
        "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
        "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
        "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
        "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
        "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
        "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
        "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31])));
}

// Bounded wait whose outcome is the same for every lane of the warp, so the
// warp-collective tcgen05 instructions that follow never run diverged.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int32_t* status) {
  const bool ok = mbar_wait(bar, parity, status);
  return __all_sync(0xffffffffu, ok);
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// Byte offset of 16-byte chunk `c` (0..15 over a 128-element row) of row `r`
// in a K-major tile stored as two 64-column blocks with the 128-byte swizzle.
__device__ __forceinline__ uint32_t swz_offset(int r, int c) {
  return uint32_t(c >> 3) * kHalfBytes + uint32_t(r) * 128u + uint32_t(((c & 7) ^ (r & 7)) << 4);
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    seg_tc_kernel(SegParams p, const __grid_constant__ CUtensorMap tmap_k, const __grid_constant__ CUtensorMap tmap_v) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + TcSmem::off_bar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + TcSmem::off_tmem);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int task = blockIdx.x, head = blockIdx.y;
  const int G = p.group;

  const int job = p.tc_tasks[2 * task];
  const int tile = p.tc_tasks[2 * task + 1];
  if (job < 0 || job >= p.num_jobs) {
    if (tid == 0) set_status(p.status, TA_ERR_BOUNDS);
    return;
  }
  const int nr = p.qlen[job];
  int nk = p.klen[job];
  const int64_t k0 = p.kstart[int64_t(job) * p.kstart_stride];
  const int r0 = tile * kRows;
  const int rows = min(kRows, nr * G - r0);
  const int64_t part_row0 = int64_t(p.slot_base[job]) * G + r0;
  const bool rows_ok = rows > 0 && part_row0 >= 0 && part_row0 + rows <= int64_t(p.num_partials) * G;
  if (!rows_ok || nr > p.max_requests || nk < 0 || k0 < 0 || k0 + nk > p.pool_tokens || k0 > INT32_MAX - kKeys) {
    if (tid == 0) set_status(p.status, TA_ERR_BOUNDS);
    if (!rows_ok) return;
    nk = 0;
  }
  const int ntiles = (nk + kKeys - 1) / kKeys;
  const int64_t head_rows = int64_t(head) * p.num_partials * G;

  if (ntiles == 0) {  // empty segment: O = 0, LSE = -inf
    for (int i = tid; i < rows * kDim; i += kThreads) p.part[(head_rows + part_row0 + i / kDim) * kDim + i % kDim] = 0.f;
    for (int i = tid; i < rows; i += kThreads) p.lse[head_rows + part_row0 + i] = -INFINITY;
    return;
  }

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars[K_FULL + s], 1);
      mbar_init(&bars[V_FULL + s], 1);
      mbar_init(&bars[KV_EMPTY + s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars[S_FULL + s], 1);
      mbar_init(&bars[S_FREE + s], 4);
    }
    mbar_init(&bars[Q_FULL], 4);
    mbar_init(&bars[P_FULL], 4);
    mbar_init(&bars[PV_DONE], 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool alive = true;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      for (int j = 0; j < ntiles && alive; ++j) {
        const int st = j % kStages;
        if (j >= kStages && !mbar_wait(&bars[KV_EMPTY + st], ((j / kStages) + 1) & 1, p.status)) {
          alive = false;
          break;
        }
        const int y = int(k0) + j * kKeys;
        unsigned char* kdst = smem + TcSmem::off_k + st * kTileBytes;
        unsigned char* vdst = smem + TcSmem::off_v + st * kTileBytes;
        mbar_arrive_expect_tx(&bars[K_FULL + st], kTileBytes);
        tma_load_3d(kdst, &tmap_k, 0, y, head, &bars[K_FULL + st]);
        tma_load_3d(kdst + kHalfBytes, &tmap_k, 64, y, head, &bars[K_FULL + st]);
        mbar_arrive_expect_tx(&bars[V_FULL + st], kTileBytes);
        tma_load_3d(vdst, &tmap_v, 0, y, head, &bars[V_FULL + st]);
        tma_load_3d(vdst + kHalfBytes, &tmap_v, 64, y, head, &bars[V_FULL + st]);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    constexpr uint32_t ab = Elem<T>::kCode == TA_DTYPE_BF16 ? 1u : 0u;
    constexpr uint32_t idesc_s = instr_desc(ab, 0);
    constexpr uint32_t idesc_o = instr_desc(ab, 1);
    const uint32_t q_addr = smem_u32(smem + TcSmem::off_q);
    const uint32_t p_addr = smem_u32(smem + TcSmem::off_p);
    const int last_keys = nk - (ntiles - 1) * kKeys;

    auto issue_pv = [&](int j) -> bool {
      const int st = j % kStages;
      if (!warp_wait(&bars[P_FULL], j & 1, p.status)) return false;
      if (!warp_wait(&bars[V_FULL + st], (j / kStages) & 1, p.status)) return false;
      unsigned char* vtile = smem + TcSmem::off_v + st * kTileBytes;
      if (j == ntiles - 1 && last_keys < kKeys) {
        // keys past the segment: their P is 0 but their V rows may hold
        // anything (NaN in unwritten pool capacity), so zero them.
        for (int i = lane; i < (kKeys - last_keys) * 16; i += 32) {
          const int r = last_keys + i / 16, c = i % 16;
          *reinterpret_cast<uint4*>(vtile + (c >> 3) * kHalfBytes + r * 128 + (c & 7) * 16) = make_uint4(0, 0, 0, 0);
        }
        fence_async_smem();
        __syncwarp();
      }
      tc_fence_after();
      if (lane == 0) {
        const uint32_t v_addr = smem_u32(vtile);
#pragma unroll
        for (int k = 0; k < kKeys / 16; ++k) {
          // A = P: 16 keys = 32 bytes along the swizzled row; B = V (N-major):
          // 16 keys = two 8-row atoms = 2048 bytes; LBO = 64-column block stride.
          const uint64_t a = smem_desc(p_addr + (k >> 2) * kHalfBytes + (k & 3) * 32, 16, 1024);
          const uint64_t b = smem_desc(v_addr + k * 2048, kHalfBytes, 1024);
          umma(tmem + kColO, a, b, idesc_o, (j > 0 || k > 0) ? 1u : 0u);
        }
        umma_commit(&bars[PV_DONE]);
        umma_commit(&bars[KV_EMPTY + st]);
      }
      __syncwarp();
      return true;
    };

    if (!warp_wait(&bars[Q_FULL], 0, p.status)) alive = false;
    for (int j = 0; j < ntiles && alive; ++j) {
      const int st = j % kStages, sb = j & 1;
      if (!warp_wait(&bars[K_FULL + st], (j / kStages) & 1, p.status)) { alive = false; break; }
      if (j >= 2 && !warp_wait(&bars[S_FREE + sb], ((j >> 1) + 1) & 1, p.status)) { alive = false; break; }
      tc_fence_after();
      if (lane == 0) {
        const uint32_t k_addr = smem_u32(smem + TcSmem::off_k + st * kTileBytes);
#pragma unroll
        for (int k = 0; k < kDim / 16; ++k) {
          const uint32_t off = (k >> 2) * kHalfBytes + (k & 3) * 32;
          umma(tmem + kColS0 + sb * kKeys, smem_desc(q_addr + off, 16, 1024), smem_desc(k_addr + off, 16, 1024),
               idesc_s, k > 0 ? 1u : 0u);
        }
        umma_commit(&bars[S_FULL + sb]);
      }
      __syncwarp();
      if (j >= 1 && !issue_pv(j - 1)) { alive = false; break; }
    }
    if (alive && !issue_pv(ntiles - 1)) alive = false;
    // The last commits' arrivals must land before the CTA's shared memory is
    // released: wait for the final release of each stage.
    if (alive) {
      for (int j = max(0, ntiles - kStages); j < ntiles; ++j)
        if (!warp_wait(&bars[KV_EMPTY + j % kStages], (j / kStages) & 1, p.status)) break;
    }
  } else {
    // ---------------- softmax / correction / epilogue ----------------
    const int quad = warp & 3;                 // TMEM lane quadrant of this warp
    const int row = quad * 32 + lane;          // query row of this thread
    const uint32_t lane_addr = tmem + (uint32_t(quad * 32) << 16);

    // Q row -> shared memory (K-major, 128B swizzle), zero for padding rows.
    {
      unsigned char* qs = smem + TcSmem::off_q;
      const uint4* src = nullptr;
      if (row < rows) {
        const int grow = r0 + row;
        const int rid = p.qids[int64_t(job) * p.max_requests + grow / G];
        if (rid >= 0 && rid < p.num_requests)
          src = reinterpret_cast<const uint4*>(p.q + (int64_t(rid) * p.num_q_heads + head * G + grow % G) * kDim);
        else
          set_status(p.status, TA_ERR_BOUNDS);
      }
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        const uint4 v = src ? src[c] : make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(qs + swz_offset(row, c)) = v;
      }
      fence_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[Q_FULL]);
    }

    const float scale = p.scale_log2;
    float m_run = -INFINITY, z = 0.f;
    unsigned char* ps = smem + TcSmem::off_p;
    for (int j = 0; j < ntiles && alive; ++j) {
      const int sb = j & 1;
      if (!warp_wait(&bars[S_FULL + sb], (j >> 1) & 1, p.status)) { alive = false; break; }
      tc_fence_after();
      float s[kKeys];
#pragma unroll
      for (int c = 0; c < kKeys / 32; ++c) {
        float chunk[32];
        tmem_ld32(lane_addr + kColS0 + sb * kKeys + c * 32, chunk);
#pragma unroll
        for (int i = 0; i < 32; ++i) s[c * 32 + i] = chunk[i];
      }
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[S_FREE + sb]);

      const int valid = min(kKeys, nk - j * kKeys);
      float mx = -INFINITY;
#pragma unroll
      for (int i = 0; i < kKeys; ++i) {
        if (i >= valid) s[i] = -INFINITY;
        mx = fmaxf(mx, s[i]);
      }
      const float m_tile = mx * scale;          // valid >= 1, so finite
      float m_new = m_run;
      bool rescale = false;
      if (j == 0) {
        m_new = m_tile;
      } else if (m_tile > m_run + kRescaleThreshold) {
        m_new = m_tile;
        rescale = true;
      }
      // P buffer and O are free once the previous P.V has completed.
      if (j >= 1 && !warp_wait(&bars[PV_DONE], (j - 1) & 1, p.status)) { alive = false; break; }
      tc_fence_after();
      if (__any_sync(0xffffffffu, rescale)) {
        const float alpha = rescale ? fast_exp2(m_run - m_new) : 1.f;
        z *= alpha;
#pragma unroll
        for (int c = 0; c < kDim / 32; ++c) {
          float o[32];
          tmem_ld32(lane_addr + kColO + c * 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] *= alpha;
          tmem_st32(lane_addr + kColO + c * 32, o);
        }
        tmem_wait_st();
      }
      m_run = m_new;
      float sum = 0.f;
#pragma unroll
      for (int c = 0; c < kKeys / 8; ++c) {
        uint32_t packed[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float a = fast_exp2(fmaf(s[c * 8 + 2 * i], scale, -m_run));
          const float b = fast_exp2(fmaf(s[c * 8 + 2 * i + 1], scale, -m_run));
          sum += a + b;
          packed[i] = Elem<T>::pack2(a, b);
        }
        *reinterpret_cast<uint4*>(ps + swz_offset(row, c)) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
      }
      z += sum;
      fence_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[P_FULL]);
    }

    // epilogue: wait for the last P.V, then O / z and the natural-log LSE
    if (alive && !warp_wait(&bars[PV_DONE], (ntiles - 1) & 1, p.status)) alive = false;
    tc_fence_after();
    const float inv = (alive && z > 0.f) ? 1.f / z : 0.f;
    float* dst = p.part + (head_rows + part_row0 + row) * kDim;
#pragma unroll
    for (int c = 0; c < kDim / 32; ++c) {
      float o[32];
      tmem_ld32(lane_addr + kColO + c * 32, o);
      tmem_wait_ld();
      if (row < rows) {
#pragma unroll
        for (int i = 0; i < 32; i += 4)
          *reinterpret_cast<float4*>(dst + c * 32 + i) =
              make_float4(o[i] * inv, o[i + 1] * inv, o[i + 2] * inv, o[i + 3] * inv);
      }
    }
    if (row < rows)
      p.lse[head_rows + part_row0 + row] = (alive && z > 0.f) ? (m_run + fast_log2(z)) * kLn2 : -INFINITY;
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

// ---- host side: tensor maps through the driver entry point -------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// Pool [heads, tokens, 128] of 16-bit elements; box = 64 columns x 128 rows x 1 head.
bool make_pool_map(CUtensorMap* map, const void* base, int64_t tokens, int heads) {
  EncodeTiledFn fn = encode_fn();
  if (!fn || tokens <= 0) return false;
  cuuint64_t dims[3] = {cuuint64_t(kDim), cuuint64_t(tokens), cuuint64_t(heads)};
  cuuint64_t strides[2] = {cuuint64_t(kDim) * 2, cuuint64_t(tokens) * kDim * 2};
  cuuint32_t box[3] = {64, cuuint32_t(kKeys), 1};
  cuuint32_t elem[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, const_cast<void*>(base), dims, strides, box, elem,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <typename T>
cudaError_t launch_typed(const SegParams& p, int num_tasks, cudaStream_t stream) {
  CUtensorMap tk, tv;
  if (!make_pool_map(&tk, p.k, p.pool_tokens, p.num_kv_heads) || !make_pool_map(&tv, p.v, p.pool_tokens, p.num_kv_heads))
    return cudaErrorInvalidValue;
  auto kernel = seg_tc_kernel<T>;
  static bool configured = false;
  if (!configured) {
    cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(TcSmem::alloc));
    if (err != cudaSuccess) return err;
    configured = true;
  }
  dim3 grid(num_tasks, p.num_kv_heads);
  kernel<<<grid, kThreads, TcSmem::alloc, stream>>>(p, tk, tv);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_seg_tc(const SegParams& p, int num_tasks, int dtype, cudaStream_t stream) {
  if (num_tasks <= 0) return cudaSuccess;
  if (dtype == TA_DTYPE_BF16) return launch_typed<__nv_bfloat16>(p, num_tasks, stream);
  if (dtype == TA_DTYPE_F16) return launch_typed<__half>(p, num_tasks, stream);
  return cudaErrorInvalidValue;
}

}  // namespace ta
