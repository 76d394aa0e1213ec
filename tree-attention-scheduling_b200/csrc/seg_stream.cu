// Segment attention for small query groups (head_dim 128), streamed by
// independent warps that take their work from a queue, with the global LSE
// merge of the step as an optional last phase.
//
// Work.  The plan's small-group segments (kn_segs: one KV head, the query rows
// of a few whole requests of one job -- at most 16 rows -- and a contiguous
// key range).  A decode step's private leaves are such segments: one
// request's GQA group (4 rows) over a few dozen keys.  Their work is reading
// the keys and values once; the arithmetic per byte is tiny, so the kernel is
// HBM-bound and is built for bytes in flight per SM, not for math.
//
// Placement.  Persistent CTAs (one per SM) of kWarps warps; every warp is an
// independent streaming worker that takes segments from a queue -- an atomic
// counter in the plan's metadata (`queue`, zero between calls) -- instead of
// a fixed list.  Launched right after the query-tile kernel of the same call,
// the CTAs start on the SMs that kernel leaves free and stream leaves while it
// runs; CTAs placed later, on the SMs it frees, take what is left.
//
// A warp.  Lane 0 is its own producer: it loads the segment's K and V in
// chunks of 16 keys by tiled TMA (token-major pool, boxes of 64 dims x 16 keys
// with the 128-byte swizzle, no multicast, an evict-first L2 hint) into a ring
// of kStages stages of the warp's own shared memory, running up to kStages
// chunks ahead across segment boundaries (the next segment is taken from the
// queue and decoded one segment ahead, with its query fragments loaded into
// registers early, and two more are in flight behind it).  Per chunk:
//   S = Q K^T      mma.sync m16n8k16 (bf16/f16 in, f32 accumulate): the
//                  segment's query rows (up to 16, zero-padded) as A from
//                  registers, K^T fragments by ldmatrix from the swizzled tile;
//   softmax        online, base 2 on pre-scaled scores, per query row held by
//                  a lane quad; a stale running maximum (O and the sums are
//                  rescaled only when a row's maximum grows by more than 2^8,
//                  exact after the final division); keys past the segment are
//                  masked and their V rows zeroed in shared memory;
//   O += P V       P rounded to the input dtype (as the reference does,
//                  kernels.py:49), straight from the S accumulators into A
//                  fragments; V fragments by transposing ldmatrix.
// The warp-synchronous MMA keeps the issue cost at a few instructions per key
// (dot products on the CUDA cores took about a hundred, which no SM can issue
// fast enough to stream HBM) with no tensor-memory allocation or commit round
// trips, so each warp's chain is short and the SM's bytes in flight --
// kWarps x kStages x 8 KB -- set the throughput.  At the end of a segment the
// warp writes its rows' partial outputs and natural-log LSEs.
//
// Merge (ta_attention).  Once the queue is empty every CTA waits for the
// query-tile kernel before it (griddepcontrol.wait) and for every segment of
// this launch (a done counter), then merges the step's partials, one warp per
// (request, KV head) -- the reference's _merge -- so the step needs no
// separate merge launch.  Waiting for other CTAs of this launch cannot
// deadlock: a segment is only ever held by a warp that is running, and nothing
// on that path waits on anything but its own loads.
//
// The last CTA to finish resets the queue counters, so a plan can be replayed
// (CUDA graphs) and the next call finds them at zero.  Every wait is bounded
// and records TA_ERR_TIMEOUT; malformed records are skipped with
// TA_ERR_BOUNDS.
//
// The reference's _segment (kernels.py:8-55) computes the same partial O / LSE
// per (job, KV head) with Triton tiles of 16 query rows x 64 keys; its _merge
// (kernels.py:58-83) the merge.
#include <algorithm>

#include "ta_kernels.cuh"
#include "ta_merge.cuh"
#include "tc_common.cuh"

namespace ta {

namespace {

constexpr int kDim = 128;
constexpr int kMaxRows = 16;                        // query rows of a segment (MMA M)
constexpr int kWarps = 6;                           // streaming warps per CTA
constexpr int kThreads = kWarps * 32;
constexpr int kChunk = 16;                          // keys per stage, a multiple of 16 (the MMA K of P.V)
constexpr int kStages = 4;                          // stages per warp
constexpr uint32_t kBoxBytes = kChunk * 128;        // kChunk keys x 64 dims, swizzled
constexpr uint32_t kStageBytes = 4 * kBoxBytes;     // K dims 0-63, 64-127, then V likewise
constexpr uint32_t kWarpBytes = kStages * kStageBytes;
constexpr float kRescaleThreshold = 8.0f;           // log2 units
enum Queue { Q_NEXT = 0, Q_DONE = 1, Q_EXITED = 2 };

struct StreamSmem {
  static constexpr uint32_t off_stage = 0;                               // [warps][stages][8 KB]
  static constexpr uint32_t off_bar = off_stage + kWarps * kWarpBytes;   // [warps][stages]
  static constexpr uint32_t off_flag = off_bar + kWarps * kStages * 8;
  static constexpr uint32_t bytes = off_flag + 16;
  static constexpr uint32_t alloc = bytes + 1024;                         // slack to align the base to 1 KB
};

__device__ __forceinline__ int ld_acquire(const int32_t* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

template <typename T> struct Mma;
template <> struct Mma<__nv_bfloat16> {
  __device__ __forceinline__ static void run(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
};
template <> struct Mma<__half> {
  __device__ __forceinline__ static void run(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

// Byte offset of 16-byte chunk c (0..15 over a 128-dim row) of key row r
// (0..kChunk-1) in the K or V half of a stage: two 64-dim boxes with the
// 128-byte swizzle.
__device__ __forceinline__ uint32_t swz(int r, int c) {
  return uint32_t(c >> 3) * kBoxBytes + uint32_t(r) * 128u + uint32_t(((c & 7) ^ (r & 7)) << 4);
}

// A segment as one warp sees it (every field warp-uniform except the query rows).
struct Seg {
  int valid;          // 0: the queue is empty
  int rows, nk, head, k0;
  int64_t prow;       // first partial row: head * num_partials * G + row
  int64_t qa, qb;     // element offsets in q of this lane's query rows lane/4 and lane/4 + 8, or -1
};

// A segment record as loaded from kn_segs, decoded one segment later (so the
// load's latency hides behind the current segment).
struct Raw {
  int index;
  int4 a, b, c;
};

__device__ __forceinline__ void load_raw(const SegParams& p, int index, Raw& r) {
  r.index = index;
  if (index < p.num_kn_segs) {
    const int4* rec = reinterpret_cast<const int4*>(p.kn_segs) + 3 * int64_t(index);
    r.a = rec[0];
    r.b = rec[1];
    r.c = rec[2];
  }
}

// Check a segment record and resolve its key count and this lane's query rows.
// False: malformed (nothing of it may be written).
__device__ __forceinline__ bool decode_seg(const SegParams& p, const Raw& r, Seg& s, int lane) {
  const int G = p.group;
  const int4 a = r.a, b = r.b, c = r.c;
  const int head = a.x, srows = a.z, prow0 = a.w, kmax = b.z, job = b.w & 0x3fffffff;
  const bool growing = ((b.w >> 30) & 1) != 0;
  const int qofs = c.y;
  const int nreq = srows >= 1 && srows <= kMaxRows ? srows / G : 0;
  const int64_t head_stride = int64_t(p.num_partials) * G;
  const bool ok = srows >= 1 && srows <= kMaxRows && nreq * G == srows && nreq <= p.max_requests && head >= 0 &&
                  head < p.num_kv_heads && job >= 0 && job < p.num_jobs && prow0 >= 0 &&
                  int64_t(prow0) + srows <= head_stride && kmax >= 0 && qofs >= 0 && qofs + nreq <= p.max_requests;
  if (!ok) return false;
  int nk = growing ? min(kmax, p.klen[job]) : kmax;   // a growing decode tail (always a whole job)
  if (nk < 0) nk = 0;
  int64_t k0 = b.x;
  if (k0 < 0 || k0 + nk > p.pool_tokens) {
    if (lane == 0) set_status(p.status, TA_ERR_BOUNDS);
    nk = 0;
    k0 = 0;
  }
  const int q0 = (c.x >= 0 && int64_t(c.x) + nreq <= p.num_requests) ? c.x : -1;
  auto qrow = [&](int i) -> int64_t {           // query row i of the segment
    if (i >= srows) return -1;
    const int req = i / G;
    const int rid = q0 >= 0 ? q0 + req : p.qids[int64_t(job) * p.max_requests + qofs + req];
    if (rid < 0 || rid >= p.num_requests) {
      set_status(p.status, TA_ERR_BOUNDS);
      return -1;
    }
    return (int64_t(rid) * p.num_q_heads + head * G + (i - req * G)) * kDim;
  };
  s.valid = 1;
  s.rows = srows;
  s.nk = nk;
  s.head = head;
  s.k0 = int(k0);
  s.prow = int64_t(head) * head_stride + prow0;
  s.qa = qrow(lane >> 2);
  s.qb = qrow((lane >> 2) + 8);
  return true;
}

// The A fragments (m16 x k16, row-major) of a segment's query rows for the 8
// k-steps of head_dim 128: this lane's two rows, words (lane % 4) and
// (lane % 4) + 4 of each 16-dim step.
__device__ __forceinline__ void load_q(const SegParams& p, const Seg& s, int lane, uint32_t (&qf)[8][4]) {
  const uint32_t* ra = s.valid && s.qa >= 0 ? reinterpret_cast<const uint32_t*>(p.q + s.qa) : nullptr;
  const uint32_t* rb = s.valid && s.qb >= 0 ? reinterpret_cast<const uint32_t*>(p.q + s.qb) : nullptr;
  const int w = lane & 3;
#pragma unroll
  for (int ks = 0; ks < 8; ++ks) {
    qf[ks][0] = ra ? ra[ks * 8 + w] : 0u;
    qf[ks][1] = rb ? rb[ks * 8 + w] : 0u;
    qf[ks][2] = ra ? ra[ks * 8 + w + 4] : 0u;
    qf[ks][3] = rb ? rb[ks * 8 + w + 4] : 0u;
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    seg_stream_kernel(SegParams p, MergeParams mp, const __grid_constant__ CUtensorMap tmap_k,
                      const __grid_constant__ CUtensorMap tmap_v, int do_merge) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  int32_t* queue = p.queue;
  unsigned char* ring = smem + StreamSmem::off_stage + warp * kWarpBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + StreamSmem::off_bar) + warp * kStages;
  int* flag = reinterpret_cast<int*>(smem + StreamSmem::off_flag);

  if (lane == 0) {
    for (int s = 0; s < kStages; ++s) mbar_init(&full[s], 1);
    fence_barrier_init();
    prefetch_tensormap(&tmap_k);
    prefetch_tensormap(&tmap_v);
  }
  __syncwarp();
  // Launched right after the query-tile kernel of the same call, whose CTAs
  // place this one only after the previous step's kernels have completed:
  // start at once (nothing here reads what that kernel writes).  After
  // anything else, wait for it first (it may have written key counts, pools
  // or queries).
  if (!p.kn_after_tc) pdl_wait();
  pdl_trigger();

  const float scale = p.scale_log2;
  const uint64_t policy = l2_evict_first_policy();
  int done = 0;                                     // segments this warp completed
  bool alive = true;

  // Segments flow through three stages ahead of the one being computed: a
  // queue index taken by lane 0 (`pending`), its record in flight (`raw`), and
  // the decoded next segment with its query fragments in flight.  Each stage's
  // latency hides behind one segment of computation.
  int pending = 0;
  Raw raw;
  auto take = [&]() {
    const int index = __shfl_sync(0xffffffffu, pending, 0);
    if (lane == 0) pending = atomicAdd(queue + Q_NEXT, 1);
    load_raw(p, index, raw);
  };
  // Decode `raw` into s and refill it; malformed records are counted and skipped.
  auto next_seg = [&](Seg& s) {
    for (;;) {
      if (raw.index >= p.num_kn_segs) {
        s.valid = 0;                                // the queue is empty: take nothing more
        return;
      }
      const bool ok = decode_seg(p, raw, s, lane);
      take();
      if (ok) return;
      if (lane == 0) {
        set_status(p.status, TA_ERR_BOUNDS);
        atomicAdd(queue + Q_DONE, 1);               // nothing of it is written, but it is accounted for
      }
    }
  };

  // Loader: chunks are issued in the order they are computed, across segments.
  uint32_t g_load = 0, g_comp = 0;                  // chunk sequence numbers of this warp
  auto issue = [&](const Seg& s, int chunk) {
    const int st = int(g_load % kStages);
    if (lane == 0) {                                // one TMA each for the chunk's K and V (both halves)
      unsigned char* dst = ring + st * kStageBytes;
      const int y = s.k0 + chunk * kChunk;
      mbar_arrive_expect_tx(&full[st], kStageBytes);
      tma_load_4d_hint(dst, &tmap_k, 0, y, 0, s.head, &full[st], policy);
      tma_load_4d_hint(dst + 2 * kBoxBytes, &tmap_v, 0, y, 0, s.head, &full[st], policy);
    }
    ++g_load;
  };

  // Start-up: the first three segments with one queue access and their
  // records loaded together; a malformed one is replaced from the queue.
  Seg cur, nxt;
  {
    int base = 0;
    if (lane == 0) base = atomicAdd(queue + Q_NEXT, 3);
    base = __shfl_sync(0xffffffffu, base, 0);
    if (lane == 0) pending = atomicAdd(queue + Q_NEXT, 1);
    Raw ra, rb;
    load_raw(p, base, ra);
    load_raw(p, base + 1, rb);
    load_raw(p, base + 2, raw);
    auto adopt = [&](const Raw& r, Seg& sg) -> bool {
      if (r.index >= p.num_kn_segs) {
        sg.valid = 0;
        return true;
      }
      if (decode_seg(p, r, sg, lane)) return true;
      if (lane == 0) {
        set_status(p.status, TA_ERR_BOUNDS);
        atomicAdd(queue + Q_DONE, 1);
      }
      return false;
    };
    if (!adopt(ra, cur)) next_seg(cur);
    if (!adopt(rb, nxt)) next_seg(nxt);
  }
  uint32_t qf[8][4], qn[8][4];
  // load position: segment (0 = cur, 1 = nxt) and chunk within it
  int ld_which = 0, ld_chunk = 0;
  auto chunks_of = [](const Seg& s) { return s.valid ? (s.nk + kChunk - 1) / kChunk : 0; };
  auto fill = [&]() {                               // issue chunks while a stage is free
    while (g_load - g_comp < uint32_t(kStages)) {
      const Seg& s = ld_which == 0 ? cur : nxt;
      if (!s.valid) break;
      if (ld_chunk >= chunks_of(s)) {
        if (ld_which == 1) break;                   // the segment after nxt is not in place yet
        ld_which = 1;
        ld_chunk = 0;
        continue;
      }
      issue(s, ld_chunk++);
    }
  };
  fill();
  load_q(p, cur, lane, qf);
  load_q(p, nxt, lane, qn);

  const int r0 = lane >> 2, qd = lane & 3;         // MMA fragment row and column pair of this lane
  const int mi = lane >> 3, mr = lane & 7;         // ldmatrix: the matrix and row this lane addresses
  while (cur.valid && alive) {
    const int nchunks = chunks_of(cur);
    float o[16][4];                                 // O: 16 dim tiles x (rows r0, r0 + 8) x 2 dims
#pragma unroll
    for (int t = 0; t < 16; ++t)
#pragma unroll
      for (int e = 0; e < 4; ++e) o[t][e] = 0.f;
    float m0 = -INFINITY, m1 = -INFINITY, z0 = 0.f, z1 = 0.f;   // rows r0, r0 + 8
    for (int c = 0; c < nchunks; ++c) {
      const int st = int(g_comp % kStages);
      if (!warp_wait(&full[st], (g_comp / kStages) & 1, p.status)) {
        alive = false;
        break;
      }
      const uint32_t kbase = smem_u32(ring + st * kStageBytes);
      const uint32_t vbase = kbase + 2 * kBoxBytes;
      const int nv = min(kChunk, cur.nk - c * kChunk);   // live keys of this chunk
      const int vend = min(kChunk, (nv + 15) & ~15);      // V rows the last 16-key step reads
      if (nv < vend) {
        // V rows past the segment may hold anything (another segment, unwritten
        // capacity): zero them so P = 0 never meets a NaN
        unsigned char* vrow = ring + st * kStageBytes + 2 * kBoxBytes;
        for (int i = lane; i < (vend - nv) * 16; i += 32) {
          const int r = nv + i / 16, cc = i % 16;
          *reinterpret_cast<uint4*>(vrow + swz(r, cc)) = make_uint4(0, 0, 0, 0);
        }
        fence_async_smem();                         // before the stage is refilled by TMA
        __syncwarp();
      }
      // 16 keys at a time: the K of one P.V MMA
      for (int u = 0; u * 16 < nv; ++u) {
        const int nu = nv - u * 16;                 // live keys of this 16-key step (may exceed 16)
        // ---- S = Q K^T: two 8-key tiles ----
        // even and odd k-steps accumulate separately: two MMA chains of four per tile
        float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
        float s2[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          uint32_t kb[4];                           // b0, b1 of keys 0-7, then of keys 8-15
          ldsm_x4(kbase + swz(u * 16 + (mi >> 1) * 8 + mr, 2 * ks + (mi & 1)), kb);
          Mma<T>::run(ks & 1 ? s2[0] : s[0], qf[ks], kb[0], kb[1]);
          Mma<T>::run(ks & 1 ? s2[1] : s[1], qf[ks], kb[2], kb[3]);
        }
#pragma unroll
        for (int t = 0; t < 2; ++t)
#pragma unroll
          for (int e = 0; e < 4; ++e) s[t][e] += s2[t][e];
        // ---- online softmax: this lane's keys 8t + 2qd + {0, 1}, rows r0 (e 0, 1) and r0 + 8 (e 2, 3) ----
        float x[2][4];
#pragma unroll
        for (int t = 0; t < 2; ++t)
#pragma unroll
          for (int e = 0; e < 4; ++e) x[t][e] = 8 * t + 2 * qd + (e & 1) < nu ? s[t][e] * scale : -INFINITY;
        float t0 = fmaxf(fmaxf(x[0][0], x[0][1]), fmaxf(x[1][0], x[1][1]));
        float t1 = fmaxf(fmaxf(x[0][2], x[0][3]), fmaxf(x[1][2], x[1][3]));
        t0 = fmaxf(t0, __shfl_xor_sync(0xffffffffu, t0, 1));
        t1 = fmaxf(t1, __shfl_xor_sync(0xffffffffu, t1, 1));
        t0 = fmaxf(t0, __shfl_xor_sync(0xffffffffu, t0, 2));
        t1 = fmaxf(t1, __shfl_xor_sync(0xffffffffu, t1, 2));
        const bool g0 = t0 > m0 + kRescaleThreshold, g1 = t1 > m1 + kRescaleThreshold;
        if (__any_sync(0xffffffffu, g0 || g1)) {
          const float n0 = g0 ? t0 : m0, n1 = g1 ? t1 : m1;
          const float a0 = fast_exp2(m0 - n0), a1 = fast_exp2(m1 - n1);   // -inf (first keys) gives 0
          m0 = n0;
          m1 = n1;
          z0 *= a0;
          z1 *= a1;
#pragma unroll
          for (int t = 0; t < 16; ++t) {
            o[t][0] *= a0;
            o[t][1] *= a0;
            o[t][2] *= a1;
            o[t][3] *= a1;
          }
        }
        uint32_t pa[4];                             // P as the A fragment of the 16-key step
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          const float p0 = fast_exp2(x[t][0] - m0), p1 = fast_exp2(x[t][1] - m0);
          const float p2 = fast_exp2(x[t][2] - m1), p3 = fast_exp2(x[t][3] - m1);
          z0 += p0 + p1;
          z1 += p2 + p3;
          pa[2 * t] = Elem<T>::pack2(p0, p1);
          pa[2 * t + 1] = Elem<T>::pack2(p2, p3);
        }
        // ---- O += P V: 16 dim tiles of 8 ----
#pragma unroll
        for (int dt = 0; dt < 16; dt += 2) {
          uint32_t vb[4];                           // b0, b1 of dim tile dt, then of dt + 1
          ldsm_x4_trans(vbase + swz(u * 16 + (mi & 1) * 8 + mr, dt + (mi >> 1)), vb);
          Mma<T>::run(o[dt], pa, vb[0], vb[1]);
          Mma<T>::run(o[dt + 1], pa, vb[2], vb[3]);
        }
      }
      __syncwarp();                                 // every lane's reads of the stage are done
      ++g_comp;
      fill();
    }
    if (!alive) break;
    // ---- the segment's partial rows ----
    z0 += __shfl_xor_sync(0xffffffffu, z0, 1);
    z1 += __shfl_xor_sync(0xffffffffu, z1, 1);
    z0 += __shfl_xor_sync(0xffffffffu, z0, 2);
    z1 += __shfl_xor_sync(0xffffffffu, z1, 2);
    if (r0 < cur.rows) {
      const float inv = z0 > 0.f ? 1.f / z0 : 0.f;
      float* dst = p.part + (cur.prow + r0) * kDim + 2 * qd;
#pragma unroll
      for (int t = 0; t < 16; ++t) *reinterpret_cast<float2*>(dst + 8 * t) = make_float2(o[t][0] * inv, o[t][1] * inv);
      if (qd == 0) p.lse[cur.prow + r0] = z0 > 0.f ? (m0 + fast_log2(z0)) * kLn2 : -INFINITY;
    }
    if (r0 + 8 < cur.rows) {
      const float inv = z1 > 0.f ? 1.f / z1 : 0.f;
      float* dst = p.part + (cur.prow + r0 + 8) * kDim + 2 * qd;
#pragma unroll
      for (int t = 0; t < 16; ++t) *reinterpret_cast<float2*>(dst + 8 * t) = make_float2(o[t][2] * inv, o[t][3] * inv);
      if (qd == 0) p.lse[cur.prow + r0 + 8] = z1 > 0.f ? (m1 + fast_log2(z1)) * kLn2 : -INFINITY;
    }
    ++done;
    // ---- advance: nxt becomes the current segment ----
    cur = nxt;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks)
#pragma unroll
      for (int e = 0; e < 4; ++e) qf[ks][e] = qn[ks][e];
    next_seg(nxt);
    load_q(p, nxt, lane, qn);
    // the loader was on the old nxt (now cur) or had not reached it yet
    if (ld_which == 0) ld_chunk = 0;
    ld_which = 0;
    fill();
  }

  if (do_merge) {
    // this warp's partial rows before its segments enter the done count
    __threadfence();
    __syncwarp();
    if (lane == 0 && done) atomicAdd(queue + Q_DONE, done);
  }
  __syncthreads();

  if (do_merge) {
    // ---------------- merge phase ----------------
    // One warp per (request, KV head) when the group size has a kernel (its G
    // query heads at once), else per (request, query head).  The first item's
    // count and slots are plan records, loaded before the waits.
    const int G = mp.group;
    const bool grouped = G == 1 || G == 2 || G == 4 || G == 8;
    const int per_request = grouped ? mp.num_q_heads / G : mp.num_q_heads;
    const int items = mp.num_requests * per_request;
    const int warps = int(gridDim.x) * kWarps;
    int item = int(blockIdx.x) * kWarps + warp;
    auto records = [&](int i, int& count, int& pre) {
      const int request = i / per_request;
      count = mp.counts[request];
      pre = lane < mp.max_slots ? mp.cslots[int64_t(request) * mp.max_slots + lane] : -1;
    };
    int count = 0, pre = -1;
    if (item < items) records(item, count, pre);
    // The query-tile kernel's partials: complete once the wait returns.  This
    // launch's: complete once every segment is counted.
    pdl_wait();
    if (tid == 0) {
      int ok = 1;
      if (ld_acquire(queue + Q_DONE) < p.num_kn_segs) {
        const uint64_t start = global_ns();
        while (ld_acquire(queue + Q_DONE) < p.num_kn_segs) {
          if (global_ns() - start > TA_WAIT_NS) {
            set_status(p.status, TA_ERR_TIMEOUT);
            ok = 0;
            break;
          }
          __nanosleep(64);
        }
      }
      *flag = ok;
    }
    __syncthreads();
    if (*flag) {
      for (bool first = true; item < items; item += warps, first = false) {
        if (!first) records(item, count, pre);
        const int request = item / per_request, sub = item % per_request;
        switch (grouped ? G : 0) {
          case 1: merge_group<T, 1>(mp, request, sub, count, pre, lane); break;
          case 2: merge_group<T, 2>(mp, request, sub, count, pre, lane); break;
          case 4: merge_group<T, 4>(mp, request, sub, count, pre, lane); break;
          case 8: merge_group<T, 8>(mp, request, sub, count, pre, lane); break;
          default: merge_one<T, kDim>(mp, request, sub, count, pre, lane); break;
        }
      }
    }
    __syncthreads();
  }
  // Complete only after the kernel before this one (a query-tile kernel this
  // launch may have started beside): whatever waits for this kernel then
  // waits for both.
  if (!do_merge) pdl_wait();
  if (tid == 0) {
    __threadfence();
    if (atomicAdd(queue + Q_EXITED, 1) == int(gridDim.x) - 1) {   // every CTA is past its last queue access
      queue[Q_NEXT] = 0;
      queue[Q_DONE] = 0;
      queue[Q_EXITED] = 0;
      __threadfence();
    }
  }
}

template <typename T>
cudaError_t launch_typed(const SegParams& p, const MergeParams* mp, cudaStream_t stream) {
  CUtensorMap tk, tv;
  if (!make_pool_map_halves(&tk, p.k, p.pool_tokens, p.num_kv_heads, kChunk) ||
      !make_pool_map_halves(&tv, p.v, p.pool_tokens, p.num_kv_heads, kChunk))
    return cudaErrorInvalidValue;
  auto kernel = seg_stream_kernel<T>;
  static int configured_device = -1;
  static int sms = 0;
  int device = 0;
  cudaError_t err = cudaGetDevice(&device);
  if (err != cudaSuccess) return err;
  if (configured_device != device) {
    err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(StreamSmem::alloc));
    if (err == cudaSuccess) err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    if (err != cudaSuccess) return err;
    configured_device = device;
  }
  // One CTA per SM.  Without the merge phase no CTA is needed beyond one warp
  // per segment; with it, every SM takes a share of the merge.
  const int ctas = mp ? sms : std::max(1, std::min(sms, (p.num_kn_segs + kWarps - 1) / kWarps));
  MergeParams m = mp ? *mp : MergeParams{};
  err = launch_dependent(kernel, dim3(ctas), dim3(kThreads), StreamSmem::alloc, stream, p, m, tk, tv, mp ? 1 : 0);
  if (err != cudaSuccess) return err;
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_seg_stream(const SegParams& p, const MergeParams* merge, int dtype, cudaStream_t stream) {
  if (p.num_kn_segs <= 0 || !p.queue) return cudaErrorInvalidValue;
  if (dtype == TA_DTYPE_BF16) return launch_typed<__nv_bfloat16>(p, merge, stream);
  if (dtype == TA_DTYPE_F16) return launch_typed<__half>(p, merge, stream);
  return cudaErrorInvalidValue;
}

}  // namespace ta
