// Segment attention for large groups on the 5th-generation tensor cores.
//
// Work of one CTA: one (job, 256-row query pair, KV head).  The query rows
// stack the GQA rows of the requests that share the job's KV segment; they are
// split into two 128-row tiles A and B that consume every K/V tile together,
// so each 64 KB K/V tile fetched through L2 feeds four 128 x 128 x 128 MMAs
// (the L2-to-SM path, about 8 TB/s, is what bounds a kernel that streams the
// tiles once per 128 rows).
//
//   warp 0      TMA producer of K tiles (token-major pool, 2 x 64-column boxes
//               with 128-byte swizzle, no multicast), 2-stage ring (an optional
//               L2 prefetch kPrefetch tiles ahead is off by default)
//   warp 2      TMA producer of V tiles, likewise; it also zeroes the rows of
//               the segment's last V tile that lie past the segment
//   warp 1      the MMA issuer, a converged warp whose elected lane issues every
//               tcgen05.mma: S_t = Q_t K^T (A = Q_t and B = K from shared
//               memory) and O_t += P_t V (A = P_t from TMEM, written by softmax
//               over its own S_t; B = V from shared memory), in the order
//               S_A(0) S_B(0) | PV_A(j) S_A(j+1) PV_B(j) S_B(j+1) ... so the
//               tensor pipe works on one tile while softmax works on the other
//   warps 3-6   softmax of tile A, warps 7-10 of tile B (a warp reaches the
//               TMEM lane quadrant warp % 4): one thread per query
//               row (TMEM lane) holding the row's 128 scores, so row maxima and
//               sums stay in the thread; the two warpgroups run concurrently
//               (one warp of each on every SM sub-partition).  exp2 on
//               pre-scaled scores, an eighth of them by a polynomial on the FMA
//               pipe (measured best among none, 1/8, 1/4, 1/3); P packed to bf16/f16 pairs and stored to TMEM over S.
//               O_t is rescaled in TMEM only when a row's running max grows by
//               more than 2^8 (otherwise the stale max is kept, which is exact
//               after the final division).  Epilogue: O_t / z and the
//               natural-log LSE per row; a full tile is staged (swizzled) in
//               a K or V ring the tile no longer needs and leaves by four TMA
//               stores, a partial tile by 32-byte stores per thread.
//
// Ordering facts the barrier scheme relies on: tcgen05.mma operations issued
// by one thread execute in issue order, so S_t(j+1) cannot overwrite P_t(j)
// before P_t(j) V(j) has read it, and observing S_t(j) complete implies
// P_t(j-1) V(j-1) has completed (it was issued just before S_t(j)).  No waiter
// can fall two phases behind a barrier, so parity waits never alias.
//
// TMEM columns: [0,128) S_A / P_A, [128,256) S_B / P_B, [256,384) O_A,
// [384,512) O_B.  Shared memory: Q_A, Q_B 2 x 32 KB, K 2 x 32 KB, V 2 x 32 KB.
// All waits are bounded (ta_common.cuh).
//
// The reference's _segment (kernels.py:8-55) computes the same partial O / LSE
// with Triton tiles of 64 query rows x 64 keys.
#include "ta_kernels.cuh"
#include "tc_common.cuh"

namespace ta {

namespace {

constexpr int kRows = 128;      // query rows per tile (MMA M); a CTA holds two tiles
constexpr int kKeys = 128;      // keys per K/V tile (MMA N of S, K of P.V)
constexpr int kDim = 128;       // head_dim (MMA K of S, N of P.V)
constexpr int kKStages = 2;
constexpr int kVStages = 2;
constexpr int kPrefetch = 0;   // L2 prefetch distance in tiles (0: off; a 6-tile burst delayed the first loads)
constexpr int kSoftmaxWarp0 = 3;          // warps 3-6: tile A, 7-10: tile B
constexpr int kSoftmaxWarps = 8;
constexpr int kVProducerWarp = 2;
constexpr int kThreads = (kSoftmaxWarp0 + kSoftmaxWarps) * 32;
constexpr uint32_t kTileBytes = kKeys * kDim * 2;       // 32 KB per K, V or Q tile
constexpr uint32_t kHalfBytes = kTileBytes / 2;         // one 64-column swizzled block
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0, kColO = 256;              // + tile * 128
constexpr float kRescaleThreshold = 8.0f;               // log2 units
constexpr int kPolyPairs = 1;                           // of every 8 exp2 pairs, this many by polynomial (rest SFU)

struct TcSmem {
  static constexpr uint32_t off_q = 0;                                 // Q_A, Q_B
  static constexpr uint32_t off_k = off_q + 2 * kTileBytes;
  static constexpr uint32_t off_v = off_k + kKStages * kTileBytes;
  static constexpr uint32_t off_bar = off_v + kVStages * kTileBytes;
  static constexpr int kBars = 18;
  static constexpr uint32_t off_tmem = off_bar + kBars * 8;
  static constexpr uint32_t bytes = off_tmem + 16;
  static constexpr uint32_t alloc = bytes + 1024;         // slack to align the base to 1 KB
};

// k_full[2], k_empty[2], v_full[2], v_empty[2], s_full[A,B], p_full[A,B], pv_done[A,B], q_full[A,B], v_tail
enum Bar {
  K_FULL = 0, K_EMPTY = 2, V_FULL = 4, V_EMPTY = 6, S_FULL = 8, P_FULL = 10, PV_DONE = 12, Q_FULL = 14, V_TAIL = 16
};

// Instruction descriptor of this kernel's MMAs: M = 128 query rows, N = 128
// (keys for S, head dims for P.V), K-major A; b_mn_major selects an
// N-contiguous B (the V tile).
__host__ __device__ constexpr uint32_t instr_desc(uint32_t ab_format, uint32_t b_mn_major) {
  return umma_idesc(ab_format, 0, b_mn_major, kRows, kKeys);
}

__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));   // sm_100 three-input max
  return d;
}

// Maximum of 128 values as a three-way tree: 65 max instructions, depth 5.
__device__ __forceinline__ float max128(const float (&s)[kKeys]) {
  float m[43];
#pragma unroll
  for (int i = 0; i < 42; ++i) m[i] = fmax3(s[3 * i], s[3 * i + 1], s[3 * i + 2]);
  m[42] = fmaxf(s[126], s[127]);
  float n[15];
#pragma unroll
  for (int i = 0; i < 14; ++i) n[i] = fmax3(m[3 * i], m[3 * i + 1], m[3 * i + 2]);
  n[14] = m[42];
  float o[5];
#pragma unroll
  for (int i = 0; i < 5; ++i) o[i] = fmax3(n[3 * i], n[3 * i + 1], n[3 * i + 2]);
  return fmaxf(fmax3(o[0], o[1], o[2]), fmaxf(o[3], o[4]));
}

// 2^x for a pair on the FMA pipe: x = n + f with n = round(x) via the
// 1.5 * 2^23 shift and f in [-0.5, 0.5]; 2^f by a degree-3 polynomial whose
// coefficients are a Remez (minimax relative error) fit computed for this
// kernel, max relative error 7.5e-5 -- far below the 2^-9 rounding of the
// bf16 P it feeds; 2^n is added to the exponent field.  Arguments are clamped
// at -125, so a masked key (-inf) yields 2^-125 instead of 0: such keys only
// occur past the end of a segment, where the V rows are zeroed, and 2^-125 is
// far below the resolution of the row sum.
__device__ __forceinline__ F2 poly_exp2x2(F2 x) {
  F2 xc;
  xc.f = make_float2(fmaxf(x.f.x, -125.f), fmaxf(x.f.y, -125.f));
  const F2 t = fadd2(xc, splat(12582912.f));                 // 1.5 * 2^23
  const F2 f = fsub2(xc, fsub2(t, splat(12582912.f)));
  F2 p = ffma2(splat(0.0551716685295105f), f, splat(0.2426111251115799f));
  p = ffma2(p, f, splat(0.6932609677314758f));
  p = ffma2(p, f, splat(0.9999280571937561f));
  const int nx = __float_as_int(t.f.x) - 0x4B400000, ny = __float_as_int(t.f.y) - 0x4B400000;
  F2 r;
  r.f = make_float2(__int_as_float(__float_as_int(p.f.x) + (nx << 23)),
                    __int_as_float(__float_as_int(p.f.y) + (ny << 23)));
  return r;
}

// Byte offset of 16-byte chunk `c` (0..15 over a 128-element row) of row `r`
// in a K-major tile stored as two 64-column blocks with the 128-byte swizzle.
__device__ __forceinline__ uint32_t swz_offset(int r, int c) {
  return uint32_t(c >> 3) * kHalfBytes + uint32_t(r) * 128u + uint32_t(((c & 7) ^ (r & 7)) << 4);
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    seg_tc_kernel(SegParams p, const __grid_constant__ CUtensorMap tmap_k, const __grid_constant__ CUtensorMap tmap_v,
                  const __grid_constant__ CUtensorMap tmap_q, int q_map_ok,
                  const __grid_constant__ CUtensorMap tmap_part, int part_map_ok) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + TcSmem::off_bar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + TcSmem::off_tmem);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int task = blockIdx.x, head = blockIdx.y;
  const int G = p.group;

  const int4 rec = reinterpret_cast<const int4*>(p.tc_tasks)[task];
  const int piece = rec.x, pair = rec.y;
  // Before the dependency wait only records that no kernel writes are read
  // (task, piece, request count, slot): a job's key count may be rewritten by
  // the kernel before this one (a decode step's append or tail update), so it
  // is read after pdl_wait below.
  PieceRows pr;
  const bool addressable = resolve_piece_rows(p, piece, pr);
  const int r0 = pair * 2 * kRows;
  const int rows = addressable ? min(2 * kRows, pr.nr * G - r0) : 0;   // rows of this pair
  if (rows <= 0) {
    pdl_wait();
    if (tid == 0) set_status(p.status, TA_ERR_BOUNDS);
    return;
  }
  const int job = pr.job;
  const int ntile = rows > kRows ? 2 : 1;                  // tile B present?
  const int64_t part_row0 = pr.slot * G + r0;
  const int64_t head_rows = int64_t(head) * p.num_partials * G;
  // The job's requests are consecutive: the query tiles come in by TMA
  // (boxes of 128/G requests x G query heads), issued before the first K tile.
  const int q0 = (rec.z >= 0 && int64_t(rec.z) + pr.nr <= p.num_requests) ? rec.z : -1;
  const bool tma_q = q_map_ok && q0 >= 0;

  if (tid == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars[K_FULL + s], 1);
      mbar_init(&bars[K_EMPTY + s], 1);
      mbar_init(&bars[V_FULL + s], 1);
      mbar_init(&bars[V_EMPTY + s], 1);
      mbar_init(&bars[S_FULL + s], 1);
      mbar_init(&bars[P_FULL + s], kSoftmaxWarps / 2);
      mbar_init(&bars[PV_DONE + s], 1);
      mbar_init(&bars[Q_FULL + s], tma_q ? 1 : kSoftmaxWarps / 2);
    }
    mbar_init(&bars[V_TAIL], 1);
    fence_barrier_init();
    prefetch_tensormap(&tmap_k);
    prefetch_tensormap(&tmap_v);
    if (tma_q) prefetch_tensormap(&tmap_q);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool alive = true;
  // This kernel may have been placed while the kernel before it (the previous
  // step's merge, or a decode step's KV append that rewrites the tails' key
  // counts) still runs; everything above read only plan records no kernel
  // writes.  Key counts, queries, pools and partial outputs wait for its
  // completion, and only then may the next segment kernel be placed (it
  // writes partials too).  Every CTA, early exits included, waits before it
  // triggers or exits.
  pdl_wait();
  pdl_trigger();
  Piece pc;
  const int state = resolve_piece(p, piece, pc);
  if (state == PIECE_BAD_KEYS && tid == 0) set_status(p.status, TA_ERR_BOUNDS);
  const int nk = state == PIECE_OK ? pc.nk : 0;
  const int64_t k0 = pc.k0;
  const int ntiles = (nk + kKeys - 1) / kKeys;

  if (ntiles == 0) {  // empty segment: O = 0, LSE = -inf
    for (int i = tid; i < rows * kDim; i += kThreads) p.part[(head_rows + part_row0 + i / kDim) * kDim + i % kDim] = 0.f;
    for (int i = tid; i < rows; i += kThreads) p.lse[head_rows + part_row0 + i] = -INFINITY;
  } else if (warp == 0 || warp == kVProducerWarp) {
    // ---------------- TMA producers (K ring / V ring) ----------------
    const bool is_k = warp == 0;
    if (lane == 0) {
      const int stages = is_k ? kKStages : kVStages;
      const CUtensorMap* map = is_k ? &tmap_k : &tmap_v;
      unsigned char* ring = smem + (is_k ? TcSmem::off_k : TcSmem::off_v);
      uint64_t* full = &bars[is_k ? K_FULL : V_FULL];
      uint64_t* empty = &bars[is_k ? K_EMPTY : V_EMPTY];
      const uint64_t policy = l2_evict_first_policy();   // a K/V tile is read by this CTA only
      if (is_k && tma_q) {
        for (int t = 0; t < ntile; ++t) {
          unsigned char* qs = smem + TcSmem::off_q + t * kTileBytes;
          const int z = q0 + (r0 + t * kRows) / G;
          mbar_arrive_expect_tx(&bars[Q_FULL + t], kTileBytes);
          tma_load_3d(qs, &tmap_q, 0, head * G, z, &bars[Q_FULL + t]);
          tma_load_3d(qs + kHalfBytes, &tmap_q, 64, head * G, z, &bars[Q_FULL + t]);
        }
      }
      // K(s) of the first round has landed -- K_FULL's first phase -- or has
      // been consumed already -- K_EMPTY's first phase, should K_FULL have
      // moved on (it cannot before K(s) is consumed, and K_EMPTY cannot move
      // past its first phase before V(s) is loaded).
      auto k_landed = [&](int s) {
        const uint64_t start = global_ns();
        while (!mbar_try_wait_for(&bars[K_FULL + s], 0, 100) && !mbar_test_wait(&bars[K_EMPTY + s], 0)) {
          if (global_ns() - start > TA_WAIT_NS) {
            set_status(p.status, TA_ERR_TIMEOUT);
            return false;
          }
        }
        return true;
      };
      for (int j = 0; j < min(ntiles, kPrefetch); ++j) {
        tma_prefetch_l2(map, 0, int(k0) + j * kKeys, head);
        tma_prefetch_l2(map, 64, int(k0) + j * kKeys, head);
      }
      for (int j = 0; j < ntiles; ++j) {
        const int st = j % stages;
        if (j + kPrefetch < ntiles) {
          tma_prefetch_l2(map, 0, int(k0) + (j + kPrefetch) * kKeys, head);
          tma_prefetch_l2(map, 64, int(k0) + (j + kPrefetch) * kKeys, head);
        }
        if (j >= stages && !mbar_wait(&empty[st], ((j / stages) + 1) & 1, p.status)) break;
        // Start-up order, the most needed first: the queries and K(0) (the
        // first S), V(0) once K(0) has landed, K(1) once tile A's queries are
        // in, V(1) once K(1) has landed.  All CTAs start together and share
        // the HBM bandwidth, so a V tile requested early delays the first S.
        if (is_k ? (j == 1 && !mbar_wait(&bars[Q_FULL], 0, p.status)) : (j < kKStages && !k_landed(j))) break;
        const int y = int(k0) + j * kKeys;
        unsigned char* dst = ring + st * kTileBytes;
        mbar_arrive_expect_tx(&full[st], kTileBytes);
        tma_load_3d_hint(dst, map, 0, y, head, &full[st], policy);
        tma_load_3d_hint(dst + kHalfBytes, map, 64, y, head, &full[st], policy);
      }
    }
    if (!is_k) {
      // Keys past the segment in its last tile: their P is 0 but their V rows
      // may hold anything (NaN in unwritten pool capacity), so zero them once
      // the tile has landed and publish it on V_TAIL instead of V_FULL.
      const int last = ntiles - 1, last_keys = nk - last * kKeys;
      if (last_keys < kKeys) {
        const int st = last % kVStages;
        const bool ok = __all_sync(0xffffffffu, mbar_wait(&bars[V_FULL + st], (last / kVStages) & 1, p.status));
        if (ok) {
          unsigned char* vtile = smem + TcSmem::off_v + st * kTileBytes;
          for (int i = lane; i < (kKeys - last_keys) * 16; i += 32) {
            const int r = last_keys + i / 16, c = i % 16;
            *reinterpret_cast<uint4*>(vtile + (c >> 3) * kHalfBytes + r * 128 + (c & 7) * 16) = make_uint4(0, 0, 0, 0);
          }
          fence_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bars[V_TAIL]);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    // The whole warp runs the loop and its waits; one elected lane issues (the
    // same lane every time, so its commits track its MMAs).  An MMA issue holds
    // the thread for about the MMA's duration (64 cycles at M = N = 128), so
    // the issuer is busy for most of each tile and every instruction between
    // bursts delays the other tile.  Descriptors are precomputed; per MMA only
    // the 14-bit start-address field of the low word changes (shared
    // addresses < 256 KB never carry out of it).
    {
      constexpr uint32_t ab = Elem<T>::kCode == TA_DTYPE_BF16 ? 1u : 0u;
      constexpr uint32_t idesc_s = instr_desc(ab, 0);
      constexpr uint32_t idesc_o = instr_desc(ab, 1);
      const uint64_t qdesc0 = smem_desc(smem_u32(smem + TcSmem::off_q), 16, 1024);
      const uint64_t kdesc0 = smem_desc(smem_u32(smem + TcSmem::off_k), 16, 1024);
      const uint64_t vdesc0 = smem_desc(smem_u32(smem + TcSmem::off_v), kHalfBytes, 1024);
      const bool tail = nk - (ntiles - 1) * kKeys < kKeys;

      auto issue_s = [&](int t, int j) {   // S_t(j) = Q_t K(j)^T
        const uint64_t qd = qdesc0 + uint64_t(t) * (kTileBytes >> 4);
        const uint64_t kd = kdesc0 + uint64_t(j % kKStages) * (kTileBytes >> 4);
#pragma unroll
        for (int k = 0; k < kDim / 16; ++k) {
          // 16 dims = 32 bytes along the swizzled K-major rows of Q and K
          const uint64_t off = ((k >> 2) * kHalfBytes + (k & 3) * 32) >> 4;
          umma_ss_warp(tmem + kColS + t * kKeys, qd + off, kd + off, idesc_s, k > 0 ? 1u : 0u);
        }
        umma_commit_warp(&bars[S_FULL + t]);
      };
      auto issue_pv = [&](int t, int j) {  // O_t += P_t(j) V(j)
        const uint64_t vd = vdesc0 + uint64_t(j % kVStages) * (kTileBytes >> 4);
        const uint32_t p_tmem = tmem + kColS + t * kKeys;
#pragma unroll
        for (int k = 0; k < kKeys / 16; ++k)
          // A = P in TMEM (16 keys = 8 packed columns); B = V, N-major: 16 keys
          // = two 8-row atoms = 2048 bytes; LBO = 64-column block stride.
          umma_ts_warp(tmem + kColO + t * kDim, p_tmem + k * 8, vd + ((k * 2048) >> 4), idesc_o,
                  (j > 0 || k > 0) ? 1u : 0u);
        // only the last P.V is waited for (the epilogue); an earlier one is
        // known complete once the S issued after it is
        if (j == ntiles - 1) umma_commit_warp(&bars[PV_DONE + t]);
      };

      if (!warp_wait(&bars[Q_FULL], 0, p.status)) alive = false;
      if (alive && !warp_wait(&bars[K_FULL], 0, p.status)) alive = false;
      if (alive) {
        tc_fence_after();
        issue_s(0, 0);
        if (ntile == 2) {
          if (warp_wait(&bars[Q_FULL + 1], 0, p.status)) {
            tc_fence_after();
            issue_s(1, 0);
          } else {
            alive = false;
          }
        }
        umma_commit_warp(&bars[K_EMPTY]);
      }
      for (int j = 0; j < ntiles && alive; ++j) {
        const bool more = j + 1 < ntiles;
        const bool zeroed = tail && j == ntiles - 1;
        // V(j) and K(j+1) have normally landed well before tile A's P(j):
        // wait for them first, so that P's arrival is followed by MMAs only.
        if (!warp_wait(&bars[zeroed ? V_TAIL : V_FULL + j % kVStages], zeroed ? 0 : (j / kVStages) & 1, p.status) ||
            (more && !warp_wait(&bars[K_FULL + (j + 1) % kKStages], ((j + 1) / kKStages) & 1, p.status))) {
          alive = false;
          break;
        }
        for (int t = 0; t < ntile; ++t) {
          if (!warp_wait(&bars[P_FULL + t], j & 1, p.status)) { alive = false; break; }
          tc_fence_after();
          issue_pv(t, j);
          if (t == ntile - 1) umma_commit_warp(&bars[V_EMPTY + j % kVStages]);
          if (more) {
            issue_s(t, j + 1);
            if (t == ntile - 1) umma_commit_warp(&bars[K_EMPTY + (j + 1) % kKStages]);
          }
        }
      }
      // The last commits' arrivals must land before the CTA's shared memory
      // is released: wait for the final release of each ring slot.
      if (alive) {
        for (int j = max(0, ntiles - kKStages); j < ntiles; ++j)
          if (!warp_wait(&bars[K_EMPTY + j % kKStages], (j / kKStages) & 1, p.status)) break;
        for (int j = max(0, ntiles - kVStages); j < ntiles; ++j)
          if (!warp_wait(&bars[V_EMPTY + j % kVStages], (j / kVStages) & 1, p.status)) break;
      }
    }
  } else if (warp >= kSoftmaxWarp0) {
    // ---------------- softmax / correction / epilogue ----------------
    // Warpgroup t (warps 3-6: tile A, 7-10: tile B); one thread per query row
    // (TMEM lane), holding the row's 128 scores of a K tile in registers, so
    // the row maximum and sum need no exchange between threads.
    const int t = (warp - kSoftmaxWarp0) >> 2;
    const int quad = warp & 3;                       // TMEM lane quadrant of this warp
    const int row = quad * 32 + lane;                // query row of this thread within its tile
    const int trow = t * kRows + row;                // row within the pair
    const uint32_t lane_addr = tmem + (uint32_t(quad * 32) << 16);
    const uint32_t s_col = kColS + t * kKeys, o_col = kColO + t * kDim;
    if (t < ntile) {
      // this row of Q -> shared memory (K-major, 128B swizzle), zero for padding
      // rows, unless the producer brings the tile in by TMA
      if (!tma_q) {
        unsigned char* qs = smem + TcSmem::off_q + t * kTileBytes;
        const uint4* src = nullptr;
        if (trow < rows) {
          const int grow = r0 + trow;
          const int rid = q0 >= 0 ? q0 + grow / G : p.qids[int64_t(job) * p.max_requests + grow / G];
          if (rid >= 0 && rid < p.num_requests)
            src = reinterpret_cast<const uint4*>(p.q + (int64_t(rid) * p.num_q_heads + head * G + grow % G) * kDim);
          else
            set_status(p.status, TA_ERR_BOUNDS);
        }
        uint4 v[16];
#pragma unroll
        for (int c = 0; c < 16; ++c) v[c] = src ? src[c] : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int c = 0; c < 16; ++c) *reinterpret_cast<uint4*>(qs + swz_offset(row, c)) = v[c];
        fence_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[Q_FULL + t]);
      }

      const float scale = p.scale_log2;
      float m_run = -INFINITY, z = 0.f;
      for (int j = 0; j < ntiles && alive; ++j) {
        const int valid = min(kKeys, nk - j * kKeys);
        if (!warp_wait(&bars[S_FULL + t], j & 1, p.status)) { alive = false; break; }
        tc_fence_after();
        float s[kKeys];
        {
          uint32_t a[4][32];                  // four loads in flight, one wait
#pragma unroll
          for (int c = 0; c < 4; ++c) tmem_ld32(lane_addr + s_col + c * 32, a[c]);
          tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int i = 0; i < 32; ++i) s[c * 32 + i] = __uint_as_float(a[c][i]);
        }
        if (valid < kKeys) {
#pragma unroll
          for (int i = 0; i < kKeys; ++i)
            if (i >= valid) s[i] = -INFINITY;
        }
        const float m_tile = max128(s) * scale;      // at least one key is valid: finite
        float m_new = m_run;
        bool rescale = false;
        if (j == 0) {
          m_new = m_tile;
        } else if (m_tile > m_run + kRescaleThreshold) {
          m_new = m_tile;
          rescale = true;
        }
        const float alpha = rescale ? fast_exp2(m_run - m_new) : 1.f;
        z *= alpha;
        m_run = m_new;
        F2 sum = splat(0.f);
        const F2 sc = splat(scale), neg_m = splat(-m_new);
        // P over the row: key columns [32h, 32h+32) -> packed columns [16h, 16h+16)
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          uint32_t packed[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            F2 x;
            x.f = make_float2(s[32 * h + 2 * i], s[32 * h + 2 * i + 1]);
            x = ffma2(x, sc, neg_m);
            F2 e;
            if ((16 * h + i) % 8 >= 8 - kPolyPairs) {   // kPolyPairs of every eight pairs on the FMA pipe
              e = poly_exp2x2(x);
            } else {
              e.f = make_float2(fast_exp2(x.f.x), fast_exp2(x.f.y));
            }
            sum = fadd2(sum, e);
            packed[i] = Elem<T>::pack2(e.f.x, e.f.y);
          }
          tmem_st16(lane_addr + s_col + h * 16, packed);
        }
        z += sum.f.x + sum.f.y;
        if (__any_sync(0xffffffffu, rescale)) {
          // O_t holds P_t(j-1) V(j-1) already (S_t(j) was issued after it);
          // P_t(j) V(j) is not issued before this thread's P_FULL arrival.
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t o[32];
            tmem_ld32(lane_addr + o_col + c * 32, o);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st32(lane_addr + o_col + c * 32, o);
          }
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[P_FULL + t]);
      }

      // epilogue: wait for the last P.V of this tile, then O / z and the LSE.
      // PV_DONE_t completes once, with the last P.V of the tile.
      if (alive && !warp_wait(&bars[PV_DONE + t], 0, p.status)) alive = false;
      tc_fence_after();
      const float inv = (alive && z > 0.f) ? 1.f / z : 0.f;
      float* dst = p.part + (head_rows + part_row0 + trow) * kDim;
      const bool part32 = (reinterpret_cast<uintptr_t>(p.part) & 31u) == 0;   // rows are 512 bytes
      uint32_t oa[4][32];                     // the whole O row: four loads in flight, one wait
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(lane_addr + o_col + c * 32, oa[c]);
      tmem_wait_ld();
      if (part_map_ok && (t + 1) * kRows <= rows) {
        // A full tile leaves by four TMA stores (32 columns x 128 rows each,
        // 128-byte swizzled) staged in a ring this tile no longer needs: all S
        // and P.V MMAs have completed once P.V_t(last) has, so tile A reuses
        // the K ring and tile B the V ring.
        unsigned char* stage = smem + (t == 0 ? TcSmem::off_k : TcSmem::off_v);
        // Each box leaves as soon as it is staged: the stores of all CTAs
        // finish together and run at the L2 write rate, so starting them a
        // box at a time overlaps them with the staging of the next boxes.
        const int y = int(head_rows + part_row0 + t * kRows);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          unsigned char* box_row = stage + c * (kRows * 128) + row * 128;
#pragma unroll
          for (int i = 0; i < 8; ++i)
            *reinterpret_cast<float4*>(box_row + ((i ^ (row & 7)) << 4)) =
                make_float4(__uint_as_float(oa[c][4 * i]) * inv, __uint_as_float(oa[c][4 * i + 1]) * inv,
                            __uint_as_float(oa[c][4 * i + 2]) * inv, __uint_as_float(oa[c][4 * i + 3]) * inv);
          fence_async_smem();
          named_sync(1 + t, kSoftmaxWarps / 2 * 32);
          if (quad == 0 && lane == 0) {
            tma_store_2d(&tmap_part, stage + c * (kRows * 128), 32 * c, y);
            bulk_commit_group();
          }
        }
        if (quad == 0 && lane == 0) bulk_wait_read_all();   // shared memory must outlive the reads
      } else {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const uint32_t (&o)[32] = oa[c];
        if (trow < rows) {
          if (part32) {
#pragma unroll
            for (int i = 0; i < 32; i += 8) {     // full 32-byte sectors
              float v[8];
#pragma unroll
              for (int u = 0; u < 8; ++u) v[u] = __uint_as_float(o[i + u]) * inv;
              st_global_v8(dst + c * 32 + i, v);
            }
          } else {
#pragma unroll
            for (int i = 0; i < 32; i += 4)
              *reinterpret_cast<float4*>(dst + c * 32 + i) =
                  make_float4(__uint_as_float(o[i]) * inv, __uint_as_float(o[i + 1]) * inv,
                              __uint_as_float(o[i + 2]) * inv, __uint_as_float(o[i + 3]) * inv);
          }
        }
      }
      }
      if (trow < rows)
        p.lse[head_rows + part_row0 + trow] = (alive && z > 0.f) ? (m_run + fast_log2(z)) * kLn2 : -INFINITY;
    }
  }

  // Every warp reconverges (roles ran on one lane) before the CTA-wide barrier.
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

template <typename T>
cudaError_t launch_typed(const SegParams& p, int num_tasks, cudaStream_t stream) {
  CUtensorMap tk, tv, tq;
  if (!make_pool_map(&tk, p.k, p.pool_tokens, p.num_kv_heads, kKeys) ||
      !make_pool_map(&tv, p.v, p.pool_tokens, p.num_kv_heads, kKeys))
    return cudaErrorInvalidValue;
  // query tiles by TMA when G divides the 128-row tile (else per-thread loads)
  const int q_map_ok = make_query_map(&tq, p.q, p.num_requests, p.num_q_heads, p.group) ? 1 : 0;
  if (!q_map_ok) tq = tk;
  // full 128-row tiles of partial outputs by TMA store
  CUtensorMap tpart;
  const int part_map_ok =
      make_partial_map(&tpart, p.part, int64_t(p.num_kv_heads) * p.num_partials * p.group) ? 1 : 0;
  if (!part_map_ok) tpart = tk;
  auto kernel = seg_tc_kernel<T>;
  static bool configured = false;
  if (!configured) {
    cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(TcSmem::alloc));
    if (err != cudaSuccess) return err;
    configured = true;
  }
  dim3 grid(num_tasks, p.num_kv_heads);
  cudaError_t err = launch_dependent(kernel, grid, dim3(kThreads), TcSmem::alloc, stream, p, tk, tv, tq, q_map_ok,
                                     tpart, part_map_ok);
  if (err != cudaSuccess) return err;
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
