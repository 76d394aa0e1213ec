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
  const int32_t* pieces;     // [P, 4] job, key offset, keys, first partial slot
  const int32_t* small_tasks;  // [n, 2] (piece, 16-row tile)
  const int32_t* tc_tasks;     // [n, 4] (piece, 256-row pair, first request if contiguous else -1, 0)
  const int32_t* kn_offsets;   // [kn_ctas + 1]
  const int32_t* kn_tasks;     // [n, 4] task headers
  const int32_t* kn_segs;      // [m, 8] segments
  int32_t* status;
  int64_t pool_tokens;
  int32_t num_jobs, num_pieces, max_requests, kstart_stride, num_requests, num_partials;
  int32_t num_q_heads, num_kv_heads, group;
  int32_t num_kn_tasks, num_kn_segs, kn_ctas;
  int32_t kn_cta_base;         // first kn_offsets entry of the current keys-in-lanes launch
  int32_t kn_after_tc;         // the keys-in-lanes launches follow a query-tile launch of the same call
  int32_t test_stall;        // test hook: the SIMT kernel's waits give up (TA_ERR_TIMEOUT)
  float scale_log2;          // log2(e) / sqrt(D)
  uint32_t gmul;             // ceil(65536 / group): x / group == (x * gmul) >> 16 for x < 65536 / group
};

// One piece resolved against the (possibly updated) job lengths.
struct Piece {
  int job;        // job index
  int nr;         // requests of the job
  int nk;         // keys of this piece now (0 for an empty or rejected piece)
  int64_t k0;     // first pool position of the piece
  int64_t slot;   // first partial slot
};

// The parts of a piece that no kernel writes: its job, request count and
// first partial slot.
struct PieceRows {
  int job;
  int nr;
  int64_t slot;
};

// Resolve the fixed records of `piece` (no key count: that may be rewritten by
// the kernel before).  False: its partial slots are not addressable, nothing
// may be written.
__device__ __forceinline__ bool resolve_piece_rows(const SegParams& p, int piece, PieceRows& out) {
  if (piece < 0 || piece >= p.num_pieces) return false;
  const int job = p.pieces[4 * piece], slot = p.pieces[4 * piece + 3];
  if (job < 0 || job >= p.num_jobs) return false;
  const int nr = p.qlen[job];
  if (nr <= 0 || nr > p.max_requests || slot < 0 || int64_t(slot) + nr > p.num_partials) return false;
  out.job = job;
  out.nr = nr;
  out.slot = slot;
  return true;
}

// Outcome of resolve_piece.
enum PieceState { PIECE_SKIP = 0, PIECE_OK = 1, PIECE_BAD_KEYS = 2 };

// Resolve `piece`.  PIECE_SKIP: its partial slots are not addressable, nothing
// may be written.  PIECE_BAD_KEYS: its key range leaves the pool; the caller
// records TA_ERR_BOUNDS and publishes the rows as empty (O = 0, LSE = -inf).
__device__ __forceinline__ int resolve_piece(const SegParams& p, int piece, Piece& out) {
  if (piece < 0 || piece >= p.num_pieces) return PIECE_SKIP;
  const int job = p.pieces[4 * piece], kofs = p.pieces[4 * piece + 1], kmax = p.pieces[4 * piece + 2];
  const int slot = p.pieces[4 * piece + 3];
  if (job < 0 || job >= p.num_jobs) return PIECE_SKIP;
  const int nr = p.qlen[job];
  if (nr <= 0 || nr > p.max_requests || slot < 0 || int64_t(slot) + nr > p.num_partials) return PIECE_SKIP;
  out.job = job;
  out.nr = nr;
  out.slot = slot;
  const int total = p.klen[job];
  int nk = min(kmax, total - kofs);
  if (nk < 0) nk = 0;
  const int64_t k0 = int64_t(p.kstart[int64_t(job) * p.kstart_stride]) + kofs;
  if (kofs < 0 || kmax < 0 || total < 0 || k0 < 0 || k0 + nk > p.pool_tokens || k0 > INT32_MAX - 256) {
    nk = 0;
    out.k0 = 0;
    out.nk = 0;
    return PIECE_BAD_KEYS;
  }
  out.k0 = k0;
  out.nk = nk;
  return PIECE_OK;
}

struct MergeParams {
  const float* part;
  const float* lse;
  const int32_t* cslots;     // [nreq, max_slots]
  const int32_t* counts;     // [nreq] partials per request
  void* out;                 // [nreq, hq, D]
  float* out_lse;            // [nreq, hq] or null
  int32_t* status;
  int32_t num_requests, max_slots, num_partials, num_q_heads, group;
};

cudaError_t launch_seg_simt(const SegParams& p, const int32_t class_end[3], int max_keys, int head_dim, int dtype,
                            cudaStream_t stream);
cudaError_t launch_seg_tc(const SegParams& p, int num_tasks, int dtype, cudaStream_t stream);
cudaError_t launch_seg_kn(const SegParams& p, const int32_t class_ctas[5], int dtype, cudaStream_t stream);
cudaError_t launch_merge(const MergeParams& p, int head_dim, int dtype, cudaStream_t stream);
cudaError_t launch_fill_klen(int32_t* klen, const int32_t* idx, int n, int value, int num_jobs, int32_t* status,
                             cudaStream_t stream);

}  // namespace ta
