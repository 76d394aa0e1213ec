// Segment attention for small query groups (<= 16 rows per job x KV head, cut
// into tasks of <= 8 rows) on the 5th-generation tensor cores, with the keys in
// the TMEM lanes.
//
// A decode-time job shared by a few requests has few query rows (requests x
// GQA group, e.g. 4 for a private leaf) and many keys.  Putting the keys on the
// MMA's M side and the queries on N makes such a job a thin tcgen05 problem:
//   S^T [128 keys x N] = K_tile [128 x 128 dims] . Q^T          (kind::f16, both K-major)
//   O^T [128 dims x N] += V_tile^T [128 dims x 128 keys] . P^T  (A = V MN-major, B = P K-major)
// with N = max(16, R) for a row class R (the library instantiates R = 4 and 8;
// the template is written for up to 64); only R rows are
// touched on the CUDA cores.  Each thread of the softmax warps owns one key of
// the tile (one TMEM lane), so scores need no cross-lane reduction; row sums
// are kept per thread and reduced once per task.  Row maxima are handled with
// a stale maximum: the softmax uses the last agreed maximum m_r and only when
// some live key of the tile exceeds m_r + 8 (log2 units) do the warps agree
// (bar.red.or) on a new maximum and rescale their sums and the O^T columns in
// TMEM.  Every result is exact after the final division; P <= 2^8 keeps the
// bf16 P and f32 sums safe.
//
// Tasks.  A task is either one long segment (a piece of a job for one KV head)
// spanning several 128-key tiles, or up to four short segments packed into ONE
// tile: each segment owns a slot of the tile's keys (32-key aligned, slots
// back to back) and a range of the N query rows, and a row only sees the keys
// of its own segment.  Packing turns the many one-tile private leaves of a
// decode tree into full tiles, so their fixed per-tile costs are shared.
//
// The kernel is persistent: each CTA (two per SM for R <= 8) walks a host-built list of tasks
// (longest-processing-time balanced).  A scheduler warp decodes and checks
// each task ONCE into a ring of shared-memory task slots and gathers its Q^T
// rows, running ahead of every other role; the K and V TMA producers run ahead
// across task boundaries too, so the HBM stream does not stop between short
// tasks and no role waits on global-memory metadata.  Loads are 32-key boxes
// (64 columns, 128-byte swizzle, no multicast).  P.V reads V rows up to the
// next 16-key step past the last live key; any of those rows that is not a
// live key of its slot (rows a box brought in past its segment, the rest of an
// empty or short slot) is zeroed first -- pool rows there may hold anything.
//
//   warps 0-3  softmax (thread = key = TMEM lane) and the per-task epilogue
//              (thread = head dim = TMEM lane of O^T), deferred until after
//              the next task's first tile so its P.V has time to finish
//   warp 4     K producer (ring of STAGES 32 KB tiles; loads carry an
//              evict-first L2 hint: segment K/V is read once, and the step's
//              partial outputs should stay in L2 for the merge)
//   warp 5     V producer, likewise
//   warp 6     MMA issue (lane 0): polls its inputs and issues S(g) up to
//              kLook tiles ahead of P.V, and P.V(g) as soon as P(g) is
//              written, zeroing V rows where needed
//   warp 7     scheduler: task slots (warp-parallel decode + checks) and Q^T
//              gathers (cp.async, published one task later) into kQBufs
//              buffers, each released by the MMA's commit after the last S of
//              its previous task
//
// Ordering facts the barrier scheme relies on: MMAs issued by one thread run in
// issue order, and S(g) is issued only once P.V(g-3) has been issued (S runs
// at most three tiles ahead), so observing S(g) complete implies PV(g-3) has
// completed, and P^T(g) is rewritten (as P^T(g+3)) only after S(g+3), issued
// after PV(g).  A parity wait is only correct while its barrier is at most one
// phase behind, so every per-tile barrier exists three times, by tile index
// mod 3 (S_FULL, P_FULL, PV_DONE): waiting for PV(g) or PV(g-1) after
// observing S(g) then never aliases.  All waits are bounded and every decision
// that guards a named barrier is made CTA-uniform first.
//
// TMEM columns: [0, 3N) three S^T buffers (tile index mod 3), [3N, 5N) two
// O^T buffers (by task parity: a task's epilogue runs after the next task's
// first tile, while that task already accumulates into the other buffer).
// The reference's _segment (kernels.py:8-55) computes the same partial O / LSE
// per (job, KV head) with Triton tiles of 16 query rows x 64 keys.
#include "ta_kernels.cuh"
#include "tc_common.cuh"

namespace ta {

namespace {

constexpr int kKeys = 128;                  // keys per tile = MMA M = TMEM lanes
constexpr int kDim = 128;                   // head_dim
constexpr int kBoxRows = 32;                // TMA box height
constexpr int kSegMax = 4;                  // segments packed into one tile
constexpr int kTQ = 8;                      // task slots
constexpr int kSoftmaxThreads = 128;
constexpr int kKWarp = 4, kVWarp = 5, kMmaWarp = 6, kSchedWarp = 7;
constexpr int kThreads = 8 * 32;
constexpr uint32_t kTileBytes = kKeys * kDim * 2;          // 32 KB
constexpr uint32_t kHalfBytes = kTileBytes / 2;            // one 64-column swizzled block
constexpr uint32_t kBoxBytes = kBoxRows * 128;              // one 32-row x 64-column box
constexpr float kRescaleThreshold = 8.0f;                   // log2 units
constexpr int kLook = 3;                    // S runs this many tiles ahead of P.V (S / P buffers)
// task slot: int4 {nseg, ntiles, rows, flags}, then per segment three int4
// {head, row0, rows, keys now} {first key of its slot, slot keys, job, k0}
// {first partial row, first request (-1 unless the job's requests are
// contiguous), first request index within the job, 0}.  Every role copies a slot into registers with vector
// loads once per task (no shared-memory store in between), so no access to it
// waits on another.
constexpr int kSegWords = 12;
constexpr int kTaskWords = 4 + kSegMax * kSegWords;         // 52
enum TaskFlag { TASK_BAD = 1, TASK_WRITE = 2 };

struct SegR {
  int head, row0, rows, nk, kt, span, job, k0, prow0, q0, qofs;
};
struct TaskR {
  int nseg, ntiles, rows, flags;
  SegR seg[kSegMax];
};

__device__ __forceinline__ TaskR load_task(const int* w) {
  const int4* v = reinterpret_cast<const int4*>(w);
  const int4 h = v[0];
  TaskR t;
  t.nseg = h.x;
  t.ntiles = h.y;
  t.rows = h.z;
  t.flags = h.w;
#pragma unroll
  for (int s = 0; s < kSegMax; ++s) {
    const int4 a = v[1 + 3 * s], b = v[2 + 3 * s], c = v[3 + 3 * s];
    t.seg[s] = SegR{a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w, c.x, c.y, c.z};
  }
  return t;
}

template <int R>
struct KnCfg {
  static constexpr int N = R < 16 ? 16 : R;                 // MMA N
  static constexpr int CW = R < 16 ? R : 16;                // TMEM columns per load
  static constexpr int NC = R / CW;                          // loads per row set
  // Up to 8 rows: two CTAs per SM (one K and one V stage each, at most 128
  // registers per thread) so two softmax chains interleave on every SM.
  static constexpr int kCtasPerSm = R <= 8 ? 2 : 1;
  static constexpr int kStages = kCtasPerSm == 2 ? 1 : (N <= 16 ? 3 : 2);
  static constexpr uint32_t kQHalf = N * 128;               // 64-column block of N rows
  static constexpr uint32_t kQBytes = 2 * kQHalf;           // Q^T or P^T buffer
  static constexpr uint32_t off_k = 0;
  static constexpr uint32_t off_v = off_k + kStages * kTileBytes;
  static constexpr int kQBufs = N <= 32 ? 4 : 2;            // Q^T buffers (how far the scheduler runs ahead)
  static constexpr uint32_t off_q = off_v + kStages * kTileBytes;    // Q^T[kQBufs]
  static constexpr uint32_t off_p = off_q + kQBufs * kQBytes;         // P^T[kLook]
  static constexpr uint32_t off_red = off_p + kLook * kQBytes;        // [2][4][R] tile maxima by tile parity
  static constexpr uint32_t off_suml = off_red + 2 * 4 * R * 4;       // [2][4][R] row sums per warp, by task parity
  static constexpr uint32_t off_mfin = off_suml + 2 * 4 * R * 4;      // [2][R] final row maxima, by task parity
  static constexpr uint32_t off_tasks = off_mfin + 2 * R * 4;         // [kTQ][kTaskWords] task slots
  static constexpr uint32_t off_stage = off_tasks + kTQ * kTaskWords * 4;   // [2][3 * kSegMax] int4 staged segment records
  static constexpr uint32_t off_rowsrc = off_stage + 2 * 3 * kSegMax * 16;  // [R] int64 Q row offsets of a task
  static constexpr uint32_t off_bar = off_rowsrc + R * 8;
  // k_full[S], k_empty[S], v_full[S], v_empty[S], s_full[L], p_full[L], pv_done[L], q_full[QB],
  // q_empty[QB], task_full[kTQ], task_empty[kTQ]
  static constexpr int kBars = 4 * kStages + 3 * kLook + 2 * kQBufs + 2 * kTQ;
  static constexpr uint32_t off_tmem = off_bar + kBars * 8;
  static constexpr uint32_t bytes = off_tmem + 16;
  static constexpr uint32_t alloc = bytes + 1024;             // slack to align the base to 1 KB
  static constexpr uint32_t kTmemCols = N == 16 ? 128 : (N == 32 ? 256 : 512);   // S^T[kLook] + O^T[2]
  static_assert(alloc <= 227 * 1024, "shared memory budget");
  static_assert(kCtasPerSm == 1 || alloc <= 113 * 1024, "two CTAs per SM");
  static_assert((kLook + 2) * N <= kTmemCols, "TMEM budget");
};

// Header of list entry i: first segment, segment count, 0, 0.
__device__ __forceinline__ int4 load_header(const SegParams& p, int i) {
  return reinterpret_cast<const int4*>(p.kn_tasks)[i];
}

// Decode and check one task into a task slot (the scheduler warp; lane s
// checks segment s).  `nseg` and the task's segment records, staged in shared
// memory, are as the host wrote them (12 int32 each): KV head, first query row
// of the tile's N rows, rows, first partial row (slot * G), first pool
// position, first key of its slot in the tile, keys (at most), job | growing
// << 30, first request of the job if its requests are contiguous (else -1),
// 0, 0, 0.  Segment s must start where segment s-1 ends, in rows and in tile
// keys; a task with any malformed segment gets nseg 0 and writes nothing.
template <int R>
__device__ __forceinline__ void decode_task(const SegParams& p, int nseg, const int4* segs, int* w, int lane) {
  const int G = p.group;
  const bool mine = lane < kSegMax && lane < nseg;
  int4 a = make_int4(0, 0, 0, 0), b = a, c = a;
  if (mine) {
    a = segs[3 * lane];
    b = segs[3 * lane + 1];
    c = segs[3 * lane + 2];
  }
  const int head = a.x, row0 = a.y, srows = a.z, prow0 = a.w, k0 = b.x, kt = b.y, kmax = b.z;
  const int job = b.w & 0x3fffffff, growing = (b.w >> 30) & 1;
  const bool rows_ok = srows >= 1 && srows <= R;
  const int nreq = rows_ok ? int((uint32_t(srows) * p.gmul) >> 16) : 0;   // srows / G (srows <= 64, G <= 64)
  const bool kmax_ok = kmax >= 0 && kmax <= INT32_MAX - 512;
  const int span = kmax_ok ? ((kmax + kBoxRows - 1) / kBoxRows) * kBoxRows : 0;
  bool ok = rows_ok && kmax_ok && nreq * G == srows && nreq <= p.max_requests && head >= 0 &&
            head < p.num_kv_heads && job >= 0 && job < p.num_jobs && prow0 >= 0 &&
            int64_t(prow0) + srows <= int64_t(p.num_partials) * G && (nseg == 1 || kt + span <= kKeys);
  // chain: this segment starts where the previous one ends
  const int rend = __shfl_up_sync(0xffffffffu, row0 + srows, 1);
  const int kend = __shfl_up_sync(0xffffffffu, kt + span, 1);
  ok = ok && (lane == 0 ? (row0 == 0 && kt == 0) : (row0 == rend && kt == kend));
  int nk = kmax;
  if (mine && growing) nk = min(kmax, p.klen[job]);   // a growing decode tail (always a whole job)
  if (nk < 0) nk = 0;
  bool bad = false;
  if (k0 < 0 || int64_t(k0) + nk > p.pool_tokens || k0 > INT32_MAX - 512) {
    nk = 0;
    bad = true;
  }
  const int q0 = (c.x >= 0 && int64_t(c.x) + nreq <= p.num_requests) ? c.x : -1;
  const int qofs = c.y;                            // the segment's first request within its job
  ok = ok && qofs >= 0 && qofs + nreq <= p.max_requests;
  const bool all_ok = nseg >= 1 && nseg <= kSegMax && __all_sync(0xffffffffu, !mine || ok);
  const int rows = __shfl_sync(0xffffffffu, row0 + srows, (nseg - 1) & 31);
  const bool any = __any_sync(0xffffffffu, mine && nk > 0);
  const bool any_bad = __any_sync(0xffffffffu, mine && bad);
  const int nk0 = __shfl_sync(0xffffffffu, nk, 0);
  const bool good = all_ok && rows <= R;
  int4* v = reinterpret_cast<int4*>(w);
  if (lane < kSegMax) {
    const bool keep = good && mine;
    v[1 + 3 * lane] = keep ? make_int4(head, row0, srows, nk) : make_int4(0, 0, 0, 0);
    v[2 + 3 * lane] = keep ? make_int4(kt, nseg == 1 ? kKeys : span, job, k0) : make_int4(0, 0, 0, 0);
    v[3 + 3 * lane] = keep ? make_int4(prow0, q0, qofs, 0) : make_int4(0, -1, 0, 0);
  }
  if (lane == 0) {
    v[0] = good ? make_int4(nseg, nseg == 1 ? (nk0 + kKeys - 1) / kKeys : (any ? 1 : 0), rows,
                            TASK_WRITE | (any_bad ? TASK_BAD : 0))
                : make_int4(0, 0, 0, TASK_BAD);
  }
}

// Keys of segment s inside tile j (a packed task has one tile).
__device__ __forceinline__ int seg_keys(const TaskR& t, int s, int j) {
  return t.nseg == 1 ? min(kKeys, t.seg[0].nk - j * kKeys) : t.seg[s].nk;
}

__device__ __forceinline__ uint64_t row_mask(int row0, int rows) {
  return (rows >= 64 ? ~0ull : ((1ull << rows) - 1ull)) << row0;
}

// Byte offset of element (row r, column c) of a K-major operand held as two
// 64-column blocks of `half` bytes with the 128-byte swizzle.
__device__ __forceinline__ uint32_t swz(uint32_t half, int r, int c) {
  return uint32_t(c >> 6) * half + uint32_t(r) * 128u + ((uint32_t((c & 63) >> 3) ^ uint32_t(r & 7)) << 4) +
         uint32_t(c & 7) * 2u;
}

// Float max over the warp (sm_100a redux.sync on f32; -inf for a row with no live key).
__device__ __forceinline__ float warp_max_redux(float x) {
  float r;
  asm volatile("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(r) : "f"(x));
  return r;
}

// W consecutive 32-bit TMEM columns of this thread's lane (W = 4, 8 or 16).
template <int W>
__device__ __forceinline__ void tmem_ldw(uint32_t taddr, uint32_t (&r)[W]) {
  if constexpr (W == 16) {
    tmem_ld16(taddr, r);
  } else if constexpr (W == 8) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
  } else {
    static_assert(W == 4, "column group");
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(taddr));
  }
}
template <int W>
__device__ __forceinline__ void tmem_stw(uint32_t taddr, const uint32_t (&r)[W]) {
  if constexpr (W == 16) {
    tmem_st16(taddr, r);
  } else if constexpr (W == 8) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
                 "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]));
  } else {
    static_assert(W == 4, "column group");
    asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};" ::"r"(taddr), "r"(r[0]), "r"(r[1]),
                 "r"(r[2]), "r"(r[3]));
  }
}

template <typename T, int R>
__global__ void __launch_bounds__(kThreads, KnCfg<R>::kCtasPerSm)
    seg_kn_kernel(SegParams p, const __grid_constant__ CUtensorMap tmap_k, const __grid_constant__ CUtensorMap tmap_v) {
  using C = KnCfg<R>;
  constexpr int N = C::N, CW = C::CW, NC = C::NC;
  constexpr int S = C::kStages;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::off_bar);
  uint64_t* k_full = bars;
  uint64_t* k_empty = bars + S;
  uint64_t* v_full = bars + 2 * S;
  uint64_t* v_empty = bars + 3 * S;
  uint64_t* s_full = bars + 4 * S;            // [kLook], by tile index mod kLook
  uint64_t* p_full = s_full + kLook;
  uint64_t* pv_done = p_full + kLook;
  constexpr int QB = C::kQBufs;
  uint64_t* q_full = pv_done + kLook;        // [QB], by Q^T buffer
  uint64_t* q_empty = q_full + QB;
  uint64_t* task_full = q_empty + QB;
  uint64_t* task_empty = task_full + kTQ;
  int* tasks = reinterpret_cast<int*>(smem + C::off_tasks);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::off_tmem);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // Placed early after the query-tile kernel of the same call (which places
  // it only once the previous step's kernels are complete); after anything
  // else, wait for it first.  Then the next launch (another row class or the
  // merge, which waits for completion before reading) may be placed.
  if (!p.kn_after_tc) pdl_wait();
  pdl_trigger();
  const int G = p.group;
  const int cta = p.kn_cta_base + int(blockIdx.x);
  int begin = p.kn_offsets[cta], end = p.kn_offsets[cta + 1];
  if (begin < 0 || end < begin || end > p.num_kn_tasks) {
    if (tid == 0) set_status(p.status, TA_ERR_BOUNDS);
    begin = end = 0;
  }
  const int count = end - begin;
  auto slot_of = [&](int k) { return tasks + (k % kTQ) * kTaskWords; };   // k: index within this CTA's list
  // The scheduler's first loads (two task headers, the first task's segment
  // records) overlap the set-up below.
  int4 first_hdr = make_int4(0, 0, 0, 0), second_hdr = first_hdr, first_rec = first_hdr;
  if (warp == kSchedWarp && count > 0) {
    first_hdr = load_header(p, begin);
    if (count > 1) second_hdr = load_header(p, begin + 1);
    if (first_hdr.y >= 1 && first_hdr.y <= kSegMax && first_hdr.x >= 0 &&
        int64_t(first_hdr.x) + first_hdr.y <= p.num_kn_segs && lane < 3 * first_hdr.y)
      first_rec = reinterpret_cast<const int4*>(p.kn_segs)[3 * int64_t(first_hdr.x) + lane];
  }

  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int b = 0; b < kLook; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&p_full[b], 4);
      mbar_init(&pv_done[b], 1);
    }
    for (int b = 0; b < QB; ++b) {
      mbar_init(&q_full[b], 1);
      mbar_init(&q_empty[b], 1);
    }
    for (int b = 0; b < kTQ; ++b) {
      mbar_init(&task_full[b], 1);
      mbar_init(&task_empty[b], 7);   // K, V, MMA and the 4 softmax warps
    }
    fence_barrier_init();
  }
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(C::kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == kSchedWarp) {
    // ---------------- scheduler: task slots and Q^T gathers ----------------
    unsigned char* qbuf = smem + C::off_q;
    int qi = 0;
    bool alive = true;
    // Software pipeline over the list: while task k is decoded and its Q^T
    // gathered, the segment records of task k+1 (whose header arrived during
    // task k-1) and the header of task k+2 are in flight.
    int4* stage = reinterpret_cast<int4*>(smem + C::off_stage);     // [2][3 * kSegMax]
    int64_t* rowsrc = reinterpret_cast<int64_t*>(smem + C::off_rowsrc);
    int pending_qb = -1;           // Q^T buffer whose copies are issued but not yet published
    auto flush = [&]() {
      if (pending_qb >= 0) {
        cp_async_wait_group<0>();
        fence_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&q_full[pending_qb]);
        pending_qb = -1;
      }
    };
    // Bounded wait that first publishes the pending Q^T if the phase is not complete yet.
    auto wait_or_flush = [&](uint64_t* bar, uint32_t parity) -> bool {
      int ok = 1;
      if (lane == 0) ok = mbar_test_wait(bar, parity);
      if (__shfl_sync(0xffffffffu, ok, 0)) return true;
      flush();
      if (lane == 0) ok = mbar_wait(bar, parity, p.status);
      return __shfl_sync(0xffffffffu, ok, 0) != 0;
    };
    auto header_ok = [&](int4 h) { return h.y >= 1 && h.y <= kSegMax && h.x >= 0 && int64_t(h.x) + h.y <= p.num_kn_segs; };
    int4 hdr = first_hdr;
    if (count > 0 && header_ok(hdr) && lane < 3 * hdr.y) stage[lane] = first_rec;
    int4 hdr_next = second_hdr;
    __syncwarp();
    for (int k = 0; k < count && alive; ++k) {
      int* w = slot_of(k);
      // prefetch: records of task k+1, header of task k+2
      int4 pre = make_int4(0, 0, 0, 0);
      const bool pre_ok = k + 1 < count && header_ok(hdr_next) && lane < 3 * hdr_next.y;
      if (pre_ok) pre = reinterpret_cast<const int4*>(p.kn_segs)[3 * int64_t(hdr_next.x) + lane];
      const int4 hdr_after = k + 2 < count ? load_header(p, begin + k + 2) : make_int4(0, 0, 0, 0);
      if (k >= kTQ && !wait_or_flush(&task_empty[k % kTQ], ((k / kTQ) - 1) & 1)) { alive = false; break; }
      decode_task<R>(p, header_ok(hdr) ? hdr.y : 0, stage + (k & 1) * 3 * kSegMax, w, lane);
      __syncwarp();
      if (lane == 0) mbar_arrive(&task_full[k % kTQ]);
      if (pre_ok) stage[((k + 1) & 1) * 3 * kSegMax + lane] = pre;
      hdr = hdr_next;
      hdr_next = hdr_after;
      __syncwarp();
      const TaskR t = load_task(w);
      if (t.nseg == 0 || t.ntiles == 0) continue;    // no tiles: no Q^T
      const int qb = qi % QB;
      if (qi >= QB && !wait_or_flush(&q_empty[qb], ((qi / QB) - 1) & 1)) { alive = false; break; }
      // Each lane finds the Q row behind tile rows lane and lane + 32, then the
      // warp copies rows x 16 chunks of 16 bytes, swizzled K-major, with
      // asynchronous copies (zero-filled where a row is out of range).  The
      // first task's Q^T is published as soon as it lands (nothing else is
      // ready yet); a later task's once the next task's copies are issued (or
      // before the warp blocks), so the copy latency of consecutive tasks
      // overlaps.
      const int rows = t.rows;
      for (int r = lane; r < rows; r += 32) {
        SegR sg = t.seg[0];
#pragma unroll
        for (int x = 1; x < kSegMax; ++x)
          if (x < t.nseg && r >= t.seg[x].row0) sg = t.seg[x];
        const int lr = r - sg.row0;
        const int req = int((uint32_t(lr) * p.gmul) >> 16);         // lr / G (lr < 64, G <= 64)
        const int rid = sg.q0 >= 0 ? sg.q0 + req : p.qids[int64_t(sg.job) * p.max_requests + sg.qofs + req];
        int64_t src_row = -1;
        if (rid >= 0 && rid < p.num_requests)
          src_row = (int64_t(rid) * p.num_q_heads + sg.head * G + (lr - req * G)) * kDim;
        else
          set_status(p.status, TA_ERR_BOUNDS);
        rowsrc[r] = src_row;
      }
      __syncwarp();
      unsigned char* dst = qbuf + qb * C::kQBytes;
      for (int e = lane; e < rows * 16; e += 32) {
        const int r = e >> 4, c = e & 15;
        const int64_t s = rowsrc[r];
        cp_async16_zfill(dst + (c >> 3) * C::kQHalf + r * 128 + (((c & 7) ^ (r & 7)) << 4),
                         s >= 0 ? p.q + s + c * 8 : p.q, s >= 0 ? 16u : 0u);
      }
      cp_async_commit();
      if (qi == 0) {                     // the first Q^T: nothing else is ready, publish it at once
        cp_async_wait_group<0>();
        fence_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&q_full[qb]);
        ++qi;
        continue;
      }
      if (pending_qb >= 0) {             // the previous task's copies: the older group
        cp_async_wait_group<1>();
        fence_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&q_full[pending_qb]);
      }
      pending_qb = qb;
      ++qi;
    }
    flush();
  } else if (warp == kKWarp || warp == kVWarp) {
    // ---------------- TMA producers ----------------
    if (lane == 0) {
      const bool is_k = warp == kKWarp;
      const CUtensorMap* map = is_k ? &tmap_k : &tmap_v;
      unsigned char* ring = smem + (is_k ? C::off_k : C::off_v);
      uint64_t* full = is_k ? k_full : v_full;
      uint64_t* empty = is_k ? k_empty : v_empty;
      const uint64_t policy = l2_evict_first_policy();   // segment K/V is read once
      int g = 0;
      bool alive = true;
      for (int k = 0; k < count && alive; ++k) {
        if (!mbar_wait(&task_full[k % kTQ], (k / kTQ) & 1, p.status)) break;
        const TaskR t = load_task(slot_of(k));
        mbar_arrive(&task_empty[k % kTQ]);           // the task now lives in registers
        for (int j = 0; j < t.ntiles; ++j, ++g) {
          const int st = g % S;
          if (g >= S && !mbar_wait(&empty[st], ((g / S) + 1) & 1, p.status)) { alive = false; break; }
          int boxes_total = 0;
#pragma unroll
          for (int s = 0; s < kSegMax; ++s)
            if (s < t.nseg) boxes_total += (max(0, seg_keys(t, s, j)) + kBoxRows - 1) / kBoxRows;
          mbar_arrive_expect_tx(&full[st], uint32_t(boxes_total) * 2 * kBoxBytes);
          unsigned char* dst = ring + st * kTileBytes;
#pragma unroll
          for (int s = 0; s < kSegMax; ++s) {
            if (s >= t.nseg) break;
            const SegR& sg = t.seg[s];
            const int keys = max(0, seg_keys(t, s, j));
            const int y = sg.k0 + j * kKeys;
            // (kept rolled: unrolled copies of the TMA issue made the kernel
            // outgrow the instruction cache)
#pragma unroll 1
            for (int b = 0; b * kBoxRows < keys; ++b) {
              const uint32_t row = uint32_t(sg.kt + b * kBoxRows) * 128u;
              tma_load_3d_hint(dst + row, map, 0, y + b * kBoxRows, sg.head, &full[st], policy);
              tma_load_3d_hint(dst + kHalfBytes + row, map, 64, y + b * kBoxRows, sg.head, &full[st], policy);
            }
          }
        }
      }
      // Nothing may still be landing when the CTA exits: wait (bounded) for
      // the last loads of each ring slot.
      for (int q = max(0, g - S); q < g; ++q)
        if (!mbar_wait(&full[q % S], (q / S) & 1, p.status)) break;
    }
  } else if (warp == kMmaWarp) {
    // ---------------- MMA issue (lane 0) ----------------
    if (lane == 0) {
      constexpr uint32_t ab = Elem<T>::kCode == TA_DTYPE_BF16 ? 1u : 0u;
      constexpr uint32_t idesc_s = umma_idesc(ab, 0, 0, kKeys, N);    // A = K tile, B = Q^T
      constexpr uint32_t idesc_pv = umma_idesc(ab, 1, 0, kDim, N);    // A = V^T (MN-major), B = P^T
      const uint64_t kdesc0 = smem_desc(smem_u32(smem + C::off_k), 16, 1024);
      const uint64_t vdesc0 = smem_desc(smem_u32(smem + C::off_v), kHalfBytes, 1024);
      const uint64_t qdesc0 = smem_desc(smem_u32(smem + C::off_q), 16, 1024);
      const uint64_t pdesc0 = smem_desc(smem_u32(smem + C::off_p), 16, 1024);
      bool alive = true;

      // Two cursors over the CTA's tiles: `sc` issues S up to kLook tiles ahead
      // of `pc`, which issues P.V.  The loop polls: whichever of the two has
      // its inputs in goes first, so a P.V never waits behind the inputs of a
      // later S (a later task's Q^T or K tile) and vice versa.  Tasks without
      // tiles are skipped; `qi` counts the tasks with tiles, which alone use
      // the Q^T and O^T buffers.  The S cursor waits for each task slot; the
      // P.V cursor, which trails it, copies each slot and releases it.
      struct Cursor {
        int k, j, g, qi;      // index within the list, tile in task, global tile, index among tasks with tiles
        TaskR t;
      };
      auto issue_s = [&](const Cursor& c) {
        const int st = c.g % S;
        const uint64_t kd = kdesc0 + ((uint64_t(st) * kTileBytes) >> 4);
        const uint64_t qd = qdesc0 + ((uint64_t(c.qi % QB) * C::kQBytes) >> 4);
        const uint32_t d = tmem + uint32_t(c.g % kLook) * N;
#pragma unroll
        for (int s = 0; s < kDim / 16; ++s) {
          const uint64_t ka = ((s >> 2) * kHalfBytes + (s & 3) * 32) >> 4;
          const uint64_t qa = ((s >> 2) * C::kQHalf + (s & 3) * 32) >> 4;
          umma_ss(d, kd + ka, qd + qa, idesc_s, s > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[c.g % kLook]);
        umma_commit(&k_empty[st]);
        if (c.j == c.t.ntiles - 1) umma_commit(&q_empty[c.qi % QB]);   // the task's last S: its Q^T buffer is free
      };
      // P.V reads key rows [0, 16 * steps); every such row that is not a live
      // key of its slot is zeroed first.
      auto issue_pv = [&](const Cursor& c) {
        const int st = c.g % S;
        const TaskR& t = c.t;
        int steps = 8;
        if (t.nseg > 1 || seg_keys(t, 0, c.j) < kKeys) {
          unsigned char* vt = smem + C::off_v + st * kTileBytes;
          int extent = 0;
#pragma unroll
          for (int s = 0; s < kSegMax; ++s)
            if (s < t.nseg && seg_keys(t, s, c.j) > 0) extent = t.seg[s].kt + seg_keys(t, s, c.j);
          steps = (extent + 15) >> 4;
          bool zeroed = false;
#pragma unroll
          for (int s = 0; s < kSegMax; ++s) {
            if (s >= t.nseg) break;
            const int kt = t.seg[s].kt;
            const int lo = kt + max(0, seg_keys(t, s, c.j));
            const int hi = min(kt + t.seg[s].span, 16 * steps);
#pragma unroll 1
            for (int r = lo; r < hi; ++r) {
#pragma unroll
              for (int c16 = 0; c16 < 16; ++c16)
                *reinterpret_cast<uint4*>(vt + (c16 >> 3) * kHalfBytes + r * 128 + (c16 & 7) * 16) = make_uint4(0, 0, 0, 0);
            }
            zeroed |= hi > lo;
          }
          if (zeroed) fence_async_smem();
        }
        tc_fence_after();
        const uint64_t vd = vdesc0 + ((uint64_t(st) * kTileBytes) >> 4);
        const uint64_t pd = pdesc0 + ((uint64_t(c.g % kLook) * C::kQBytes) >> 4);
        const uint32_t o = tmem + kLook * N + uint32_t(c.qi & 1) * N;     // O^T of this task's parity
#pragma unroll 1
        for (int s = 0; s < steps; ++s) {
          const uint64_t va = (uint64_t(s) * 2048) >> 4;           // 16 keys = two 8-row atoms
          const uint64_t pa = ((s >> 2) * C::kQHalf + (s & 3) * 32) >> 4;
          umma_ss(o, vd + va, pd + pa, idesc_pv, (c.j > 0 || s > 0) ? 1u : 0u);
        }
        umma_commit(&v_empty[st]);
        umma_commit(&pv_done[c.g % kLook]);
      };

      Cursor sc, pc;
      sc.k = sc.j = sc.g = sc.qi = 0;
      pc.k = pc.j = pc.g = pc.qi = 0;
      bool s_loaded = false, p_loaded = false;
      // Lead: point sc at a waited-for task with tiles, without blocking.
      // False while its slot is not published or when no task is left.
      auto lead_ready = [&]() -> bool {
        while (sc.k < count) {
          if (!s_loaded) {
            if (!mbar_test_wait(&task_full[sc.k % kTQ], (sc.k / kTQ) & 1)) return false;
            sc.t = load_task(slot_of(sc.k));
            s_loaded = true;
          }
          if (sc.t.nseg > 0 && sc.t.ntiles > 0) return true;
          ++sc.k;
          s_loaded = false;
        }
        return false;
      };
      // Trail: copy and release every slot up to the next task with tiles,
      // never past the lead (only slots the lead has waited for).  It runs on
      // every pass, not only while a P.V is outstanding: slots of tasks without
      // tiles must be released even when no S is in flight, since the scheduler
      // needs them to publish the tasks 8 places later, which the lead may be
      // waiting for.
      auto trail_settle = [&]() {
        while (pc.k < count && !p_loaded && (pc.k < sc.k || (pc.k == sc.k && s_loaded))) {
          pc.t = load_task(slot_of(pc.k));
          mbar_arrive(&task_empty[pc.k % kTQ]);
          if (pc.t.nseg > 0 && pc.t.ntiles > 0) {
            p_loaded = true;
            break;
          }
          ++pc.k;
        }
      };
      uint64_t idle_since = 0;
      while (alive) {
        bool did = false;
        if (!p_loaded) trail_settle();
        if (pc.g < sc.g) {                              // P.V of the oldest tile whose S is issued
          if (!p_loaded) trail_settle();
          const int st = pc.g % S;
          if (mbar_test_wait(&p_full[pc.g % kLook], (pc.g / kLook) & 1) &&
              mbar_test_wait(&v_full[st], (pc.g / S) & 1)) {
            issue_pv(pc);
            ++pc.g;
            if (++pc.j >= pc.t.ntiles) {
              pc.j = 0;
              ++pc.k;
              ++pc.qi;
              p_loaded = false;
            }
            did = true;
          }
        }
        if (sc.g - pc.g < kLook && lead_ready()) {       // S of the next tile, up to kLook ahead
          const int st = sc.g % S;
          if ((sc.j != 0 || mbar_test_wait(&q_full[sc.qi % QB], (sc.qi / QB) & 1)) &&
              mbar_test_wait(&k_full[st], (sc.g / S) & 1)) {
            tc_fence_after();
            issue_s(sc);
            ++sc.g;
            if (++sc.j >= sc.t.ntiles) {
              sc.j = 0;
              ++sc.k;
              ++sc.qi;
              s_loaded = false;
            }
            did = true;
          }
        }
        if (sc.k >= count && pc.g == sc.g) break;        // every tile issued and its P.V too
        if (did) {
          idle_since = 0;
        } else {
          // nothing ready: rest on the oldest pending P.V (or briefly) rather
          // than taking issue slots from the softmax warp on this sub-partition
          if (pc.g < sc.g)
            mbar_try_wait_for(&p_full[pc.g % kLook], (pc.g / kLook) & 1, 200);
          else
            __nanosleep(64);
          const uint64_t now = global_ns();
          if (idle_since == 0) {
            idle_since = now;
          } else if (now - idle_since > TA_WAIT_NS) {
            set_status(p.status, TA_ERR_TIMEOUT);
            alive = false;
          }
        }
      }
      if (alive) trail_settle();                          // release the trailing slots without tiles
      // The last commits must land before the CTA's shared memory is released.
      const int total = pc.g;
      if (alive) {
        for (int q = max(0, total - S); q < total; ++q) {
          if (!mbar_wait(&k_empty[q % S], (q / S) & 1, p.status)) break;
          if (!mbar_wait(&v_empty[q % S], (q / S) & 1, p.status)) break;
        }
      }
    }
    __syncwarp();
  } else {
    // ---------------- softmax / epilogue (warps 0-3) ----------------
    const int kk = tid;                                   // key of the tile = TMEM lane; head dim in the epilogue
    const uint32_t lane_base = tmem + (uint32_t(warp * 32) << 16);
    float* red = reinterpret_cast<float*>(smem + C::off_red);      // [2][4][R]
    float* suml = reinterpret_cast<float*>(smem + C::off_suml);    // [2][4][R] by task parity
    float* mfin = reinterpret_cast<float*>(smem + C::off_mfin);    // [2][R] by task parity
    unsigned char* pbuf = smem + C::off_p;
    const float scale = p.scale_log2;
    const int64_t head_stride = int64_t(p.num_partials) * G;
    bool alive = true;

    // Partial row of task row r (rows are laid out segment after segment).
    auto out_row = [&](const TaskR& t, int r) -> int64_t {
      SegR sg = t.seg[0];
#pragma unroll
      for (int x = 1; x < kSegMax; ++x)
        if (x < t.nseg && r >= t.seg[x].row0) sg = t.seg[x];
      return int64_t(sg.head) * head_stride + sg.prow0 + (r - sg.row0);
    };
    auto release = [&](int k) {
      __syncwarp();
      if (lane == 0) mbar_arrive(&task_empty[k % kTQ]);
    };
    // Epilogue of a task with tiles whose last tile was `g_last` and whose O^T
    // and row statistics sit in buffer `b`: O / l and the LSE of every row.
    auto epilogue = [&](int k, int g_last, int b) {
      const TaskR t = load_task(slot_of(k));
      const bool w_ok = alive && warp_wait(&pv_done[g_last % kLook], (g_last / kLook) & 1, p.status);
      if (named_sync_or(2, kSoftmaxThreads, !w_ok)) alive = false;     // also orders suml / mfin
      const bool o_ok = alive;
      if (o_ok) tc_fence_after();
      const float* sl = suml + b * 4 * R;
      const float* mf = mfin + b * R;
      const int rows = t.rows;
#pragma unroll
      for (int c = 0; c < NC; ++c) {
        if (c * CW < rows) {
          float z[CW], mr[CW];
#pragma unroll
          for (int q = 0; q < CW; ++q) {         // all loads before the global stores below
            const int r = c * CW + q;
            z[q] = (sl[r] + sl[R + r]) + (sl[2 * R + r] + sl[3 * R + r]);
            mr[q] = mf[r];
          }
          uint32_t o[CW];
          if (o_ok) {
            tmem_ldw<CW>(lane_base + kLook * N + uint32_t(b) * N + c * CW, o);
            tmem_wait_ld();
          } else {
#pragma unroll
            for (int q = 0; q < CW; ++q) o[q] = 0u;
          }
          float inv[CW];
#pragma unroll
          for (int q = 0; q < CW; ++q) inv[q] = (o_ok && z[q] > 0.f) ? __fdividef(1.f, z[q]) : 0.f;
#pragma unroll
          for (int q = 0; q < CW; ++q) {
            const int r = c * CW + q;
            if (r < rows) {
              const int64_t row = out_row(t, r);
              p.part[row * kDim + kk] = __uint_as_float(o[q]) * inv[q];
              if (kk == r) p.lse[row] = inv[q] > 0.f ? (mr[q] + fast_log2(z[q])) * kLn2 : -INFINITY;
            }
          }
        }
      }
      release(k);
    };

    int g = 0;            // global tile index
    int qi = 0;           // index among tasks with tiles
    int pend_k = -1, pend_g = 0;   // task whose epilogue is deferred past the next task's first tile
    float m[R];           // agreed row maxima of the current task (identical in every thread)
    // One pass past the end of the list (k == count) runs the last pending
    // epilogue at the same call site as a task without tiles does.
    for (int k = 0; k <= count; ++k) {
      const bool end = k == count;
      if (!end) {
        const bool t_ok = alive && warp_wait(&task_full[k % kTQ], (k / kTQ) & 1, p.status);
        if (named_sync_or(1, kSoftmaxThreads, !t_ok)) alive = false;
      }
      TaskR t = {};
      if (!end && alive) t = load_task(slot_of(k));
      const int ntiles = t.ntiles, rows = t.rows, flags = t.flags;
      if ((flags & TASK_BAD) && kk == 0) set_status(p.status, TA_ERR_BOUNDS);
      if ((end || !alive || !(flags & TASK_WRITE) || ntiles == 0) && pend_k >= 0) {
        // A task without tiles has nothing to overlap with the pending
        // epilogue, so run it now: the pending task's slot must be released
        // before the scheduler can publish the task 8 places after it, and a
        // list may hold 7 or more tasks without tiles in a row (empty decode
        // tails) -- waiting for the next task with tiles would stall.
        epilogue(pend_k, pend_g, (qi - 1) & 1);
        pend_k = -1;
      }
      if (end || !alive) break;
      if (!(flags & TASK_WRITE)) {
        release(k);
        continue;
      }
      if (ntiles == 0) {
        // an empty task: O = 0, LSE = -inf, no tensor work
        for (int r = 0; r < rows; ++r) {
          const int64_t row = out_row(t, r);
          p.part[row * kDim + kk] = 0.f;
          if (kk == r) p.lse[row] = -INFINITY;
        }
        release(k);
        continue;
      }
      float l[R];
#pragma unroll
      for (int r = 0; r < R; ++r) {
        l[r] = 0.f;
        m[r] = -INFINITY;
      }
      // Rows that see this thread's key: a packed task has one tile with a
      // fixed set; a long segment's key is live while it is below the keys left.
      const bool single = t.nseg == 1;
      const int keys_total = t.seg[0].nk;
      const uint64_t single_mask = row_mask(0, rows);
      uint64_t packed_rows = 0;
#pragma unroll
      for (int s = 0; s < kSegMax; ++s)
        if (s < t.nseg && kk >= t.seg[s].kt && kk < t.seg[s].kt + t.seg[s].nk)
          packed_rows |= row_mask(t.seg[s].row0, t.seg[s].rows);

      for (int j = 0; j < ntiles; ++j, ++g) {
        const int b = g & 1;               // tile-maxima exchange buffer
        const int sb = g % kLook;          // S^T / P^T buffer and its barriers
        const uint64_t live_rows = single ? (kk < keys_total - j * kKeys ? single_mask : 0ull) : packed_rows;
        const bool ok = alive && warp_wait(&s_full[sb], (g / kLook) & 1, p.status);
        const uint32_t s_addr = lane_base + uint32_t(sb) * N;
        uint32_t keep[CW];          // scores of the first (for R <= 16: the only) column group
        bool need = false;
        if (ok) {
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < NC; ++c) {
            if (c * CW < rows) {
              uint32_t raw[CW];
              tmem_ldw<CW>(s_addr + c * CW, raw);
              tmem_wait_ld();
#pragma unroll
              for (int q = 0; q < CW; ++q) {
                const int r = c * CW + q;
                if (j > 0)              // (a task's first tile always sets the maxima)
                  need |= ((live_rows >> r) & 1ull) && __uint_as_float(raw[q]) * scale > m[r] + kRescaleThreshold;
                if (c == 0) keep[q] = raw[q];
              }
            }
          }
        }
        // One barrier in the common case: the OR of "a wait was lost" and "a
        // row needs a new maximum"; a second one tells the two apart.
        bool rescale = false;
        if (j == 0) {
          // a task's first tile always sets the maxima (every row starts at
          // -inf and the task has live keys): one barrier, for lost waits only
          if (named_sync_or(1, kSoftmaxThreads, !ok))
            alive = false;
          else
            rescale = true;
        } else if (named_sync_or(1, kSoftmaxThreads, need || !ok)) {
          if (named_sync_or(1, kSoftmaxThreads, !ok))
            alive = false;
          else
            rescale = true;
        }
        if (rescale) {
          // tile maxima over each row's live keys: warp maxima, then the 4 warps
          float* rt = red + b * 4 * R;
#pragma unroll
          for (int c = 0; c < NC; ++c) {
            if (c * CW < rows) {
              uint32_t raw[CW];
              if (c == 0) {
#pragma unroll
                for (int q = 0; q < CW; ++q) raw[q] = keep[q];
              } else {
                tmem_ldw<CW>(s_addr + c * CW, raw);
                tmem_wait_ld();
              }
              float wm[CW];
#pragma unroll
              for (int q = 0; q < CW; ++q) {
                const int r = c * CW + q;
                wm[q] = warp_max_redux(((live_rows >> r) & 1ull) ? __uint_as_float(raw[q]) * scale : -INFINITY);
              }
              if (lane == 0) {
#pragma unroll
                for (int q = 0; q < CW; q += 4)
                  *reinterpret_cast<float4*>(rt + warp * R + c * CW + q) = make_float4(wm[q], wm[q + 1], wm[q + 2], wm[q + 3]);
              }
            }
          }
          named_sync(2, kSoftmaxThreads);
          bool o_ok = j > 0;
          if (j > 0) {
            const bool w_ok = warp_wait(&pv_done[(g - 1) % kLook], ((g - 1) / kLook) & 1, p.status);
            if (named_sync_or(2, kSoftmaxThreads, !w_ok)) alive = false;
            o_ok = alive;
            if (o_ok) tc_fence_after();
          }
          const uint32_t o_addr = lane_base + kLook * N + uint32_t(qi & 1) * N;
#pragma unroll
          for (int c = 0; c < NC; ++c) {
            if (c * CW < rows) {
              // the four warps' maxima of four rows per vector load
              float mt[CW];
#pragma unroll
              for (int q = 0; q < CW; q += 4) {
                const float4 w0 = *reinterpret_cast<const float4*>(rt + c * CW + q);
                const float4 w1 = *reinterpret_cast<const float4*>(rt + R + c * CW + q);
                const float4 w2 = *reinterpret_cast<const float4*>(rt + 2 * R + c * CW + q);
                const float4 w3 = *reinterpret_cast<const float4*>(rt + 3 * R + c * CW + q);
                mt[q] = fmaxf(fmaxf(w0.x, w1.x), fmaxf(w2.x, w3.x));
                mt[q + 1] = fmaxf(fmaxf(w0.y, w1.y), fmaxf(w2.y, w3.y));
                mt[q + 2] = fmaxf(fmaxf(w0.z, w1.z), fmaxf(w2.z, w3.z));
                mt[q + 3] = fmaxf(fmaxf(w0.w, w1.w), fmaxf(w2.w, w3.w));
              }
              float alpha[CW];
#pragma unroll
              for (int q = 0; q < CW; ++q) {
                const int r = c * CW + q;
                const float mn = fmaxf(m[r], mt[q]);
                // a task's first tile has no sum or output to rescale yet
                alpha[q] = (j > 0 && mn != -INFINITY) ? fast_exp2(m[r] - mn) : 1.f;   // m = -inf gives 0
                l[r] *= alpha[q];
                m[r] = mn;                  // rows past `rows` have no live key and stay at -inf
              }
              if (o_ok) {
                uint32_t o[CW];
                tmem_ldw<CW>(o_addr + c * CW, o);
                tmem_wait_ld();
#pragma unroll
                for (int q = 0; q < CW; ++q) o[q] = __float_as_uint(__uint_as_float(o[q]) * alpha[q]);
                tmem_stw<CW>(o_addr + c * CW, o);
              }
            }
          }
          if (o_ok) tmem_wait_st();
        }
        // P^T = exp2(s - m) over each row's live keys, bf16/f16, K-major swizzled
        if (alive) {
          unsigned char* pt = pbuf + sb * C::kQBytes;
#pragma unroll
          for (int c = 0; c < NC; ++c) {
            if (c * CW < rows) {
              uint32_t raw[CW];
              if (c == 0) {
#pragma unroll
                for (int q = 0; q < CW; ++q) raw[q] = keep[q];
              } else {
                tmem_ldw<CW>(s_addr + c * CW, raw);
                tmem_wait_ld();
              }
              uint16_t e16[CW];
#pragma unroll
              for (int q = 0; q < CW; ++q) {
                const int r = c * CW + q;
                const float e = ((live_rows >> r) & 1ull) ? fast_exp2(__uint_as_float(raw[q]) * scale - m[r]) : 0.f;
                l[r] += e;
                e16[q] = Elem<T>::from_float(e);
              }
#pragma unroll
              for (int q = 0; q < CW; ++q)            // rows past `rows` get P = 0
                *reinterpret_cast<uint16_t*>(pt + swz(C::kQHalf, c * CW + q, kk)) = e16[q];
            }
          }
        }
        fence_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[sb]);
        if (j == 0 && pend_k >= 0) {
          // the previous task's epilogue: its P.V has had this tile to finish
          epilogue(pend_k, pend_g, (qi - 1) & 1);
          pend_k = -1;
        }
      }
      // this task's row sums and maxima, for its deferred epilogue
      {
        const int b = qi & 1;
        float* sl = suml + b * 4 * R;
        if constexpr (R <= 16) {
          // lane l ends with the warp's sum of row l >> (5 - log2 R)
          constexpr int kShift = R == 4 ? 3 : (R == 8 ? 2 : 1);
          const float s = warp_transpose_sum<R>(l, lane);
          if ((lane & ((1 << kShift) - 1)) == 0) sl[warp * R + (lane >> kShift)] = s;
        } else {
#pragma unroll
          for (int c = 0; c < R / 32; ++c) {
            float v[32];
#pragma unroll
            for (int q = 0; q < 32; ++q) v[q] = l[c * 32 + q];
            sl[warp * R + c * 32 + lane] = warp_transpose_sum32(v, lane);
          }
        }
#pragma unroll
        for (int r = 0; r < R; ++r)
          if (kk == r && r < rows) mfin[b * R + r] = m[r];
      }
      pend_k = k;
      pend_g = g - 1;
      ++qi;
    }
  }

  // Every warp reconverges (roles ran on one lane) before the CTA-wide barrier.
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::kTmemCols));
  }
  // This kernel may have started while the query-tile kernel before it was
  // still running (it reads nothing that kernel writes); it completes only
  // after that kernel, so whatever waits for this one also waits for both.
  pdl_wait();
}

template <typename T, int R>
cudaError_t launch_r(const SegParams& p, int ctas, cudaStream_t stream) {
  CUtensorMap tk, tv;
  if (!make_pool_map(&tk, p.k, p.pool_tokens, p.num_kv_heads, kBoxRows) ||
      !make_pool_map(&tv, p.v, p.pool_tokens, p.num_kv_heads, kBoxRows))
    return cudaErrorInvalidValue;
  auto kernel = seg_kn_kernel<T, R>;
  static bool configured = false;
  if (!configured) {
    cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(KnCfg<R>::alloc));
    if (err != cudaSuccess) return err;
    configured = true;
  }
  cudaError_t err = launch_dependent(kernel, dim3(ctas), dim3(kThreads), KnCfg<R>::alloc, stream, p, tk, tv);
  if (err != cudaSuccess) return err;
  return cudaGetLastError();
}

// One launch per non-empty row class, each over its own range of CTAs.
template <typename T>
cudaError_t launch_t(const SegParams& p, const int32_t class_ctas[5], cudaStream_t stream) {
  SegParams q = p;
  q.kn_cta_base = 0;
  cudaError_t err = cudaSuccess;
  for (int c = 0; c < 5 && err == cudaSuccess; ++c) {
    const int n = class_ctas[c];
    if (n <= 0) continue;
    switch (c) {                  // the host builds tasks of at most 8 rows (classes 16-64 are rejected)
      case 0: err = launch_r<T, 4>(q, n, stream); break;
      case 1: err = launch_r<T, 8>(q, n, stream); break;
      default: err = cudaErrorInvalidValue; break;
    }
    q.kn_cta_base += n;
  }
  return err;
}

}  // namespace

cudaError_t launch_seg_kn(const SegParams& p, const int32_t class_ctas[5], int dtype, cudaStream_t stream) {
  if (p.num_kn_tasks <= 0 || p.kn_ctas <= 0) return cudaSuccess;
  if (dtype == TA_DTYPE_BF16) return launch_t<__nv_bfloat16>(p, class_ctas, stream);
  if (dtype == TA_DTYPE_F16) return launch_t<__half>(p, class_ctas, stream);
  return cudaErrorInvalidValue;
}

}  // namespace ta
