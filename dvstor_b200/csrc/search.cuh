// Launch-side view of the search kernels (shared by search.cu and api.cu).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "dvs_b200.h"

namespace dvs {

// Device layout of one index copy (dense slot order).
//   adj      n*R u32 slot ids, kEmptySlot fill (non-empty first)
//   rec      n records of rec_words u32: [codes zero-padded to code_words words |
//            f32 add | f32 rescale | zero pad to a 16-byte multiple]
//   vecs     n rows of vec_stride floats (dim, zero-padded to a multiple of 4)
//   ids      n u32 node ids as stored in the shards
constexpr uint32_t kMaxShards = 16;

struct DevLayout {
  // Node g lives in shard (g & shard_mask) at local row (g >> shard_log); a
  // replicated layout is one shard.  Shard arrays of other devices are peer
  // pointers (NVLink).
  const uint32_t* adj_s[kMaxShards] = {};
  const uint32_t* rec_s[kMaxShards] = {};
  const float* vecs_s[kMaxShards] = {};
  uint32_t shard_log = 0, shard_mask = 0;
  const uint32_t* adj = nullptr;    // shard 0 (the whole index when replicated)
  const uint32_t* rec = nullptr;
  const float* vecs = nullptr;
  const uint32_t* ids = nullptr;    // replicated: every node's stored id
  const float* P = nullptr;         // dim*dim column-major rotation
  const float* c_rot = nullptr;     // rotated centroid
  uint64_t n = 0;
  uint32_t dim = 0, R = 0, bits = 0, medoid = 0, metric = 0;
  uint32_t rec_words = 0, code_words = 0, vec_stride = 0;
};

__device__ __forceinline__ const uint32_t* adj_row(const DevLayout& ix, uint32_t g) {
  if (ix.shard_log == 0) return ix.adj + size_t(g) * ix.R;
  return ix.adj_s[g & ix.shard_mask] + size_t(g >> ix.shard_log) * ix.R;
}
__device__ __forceinline__ const uint32_t* rec_row(const DevLayout& ix, uint32_t g) {
  if (ix.shard_log == 0) return ix.rec + size_t(g) * ix.rec_words;
  return ix.rec_s[g & ix.shard_mask] + size_t(g >> ix.shard_log) * ix.rec_words;
}
__device__ __forceinline__ const float* vec_row(const DevLayout& ix, uint32_t g) {
  if (ix.shard_log == 0) return ix.vecs + size_t(g) * ix.vec_stride;
  return ix.vecs_s[g & ix.shard_mask] + size_t(g >> ix.shard_log) * ix.vec_stride;
}

struct SearchArgs {
  DevLayout ix;
  const float* queries = nullptr;   // nq*dim, row stride dim
  const float* qrot = nullptr;      // nq*vec_stride rotated queries
  const float* qfac = nullptr;      // nq*4 {add, k1xSumq, kBxSumq, 0}
  uint32_t nq = 0, k = 0, L = 0, cap = 0, mode = 0, hop_limit = 0;
  uint32_t* out_ids = nullptr;
  float* out_dist = nullptr;
  uint32_t* counters = nullptr;     // nq*4: H, E, C_r, count | error bits << 16
  uint32_t* work = nullptr;         // [0] next query, [1] error bits, [2] overflowed queries
  uint32_t* ovf = nullptr;          // per warp slot visited spill tables (ovf_cap words each), zeroed at allocation
  uint32_t* ovf_epoch = nullptr;    // per warp slot epoch of its table (zeroed at allocation)
  uint32_t ovf_cap = 0, ovf_limit = 0;
  uint32_t ovf_tagged = 0;          // 1: entries are (epoch << 24) | id (indexes of fewer than 2^24 nodes)
  uint32_t hcap = 0, hlimit = 0;    // shared-memory visited table: words, entry limit
  uint32_t vt16 = 0;                // compact 16-bit two-choice table: its hash width (20 or 24), 0 = 32-bit table
  uint32_t hbuckets = 0;            // its bucket count (8 entries each)
  uint32_t hb_magic = 0;            // ceil(2^32 / hbuckets): division by the bucket count as a multiply-high
  uint32_t cap_pad = 0, dim_pad = 0;
  uint32_t out_slots = 0;           // 1: results are dense slots (online insert), else stored node ids
};

constexpr int kMaxBlockSmem = 227 * 1024;  // dynamic shared memory a block may have on sm_100

constexpr uint32_t kErrCapacity = 1u;
constexpr uint32_t kErrHopLimit = 2u;
constexpr uint32_t kErrTimeout = 4u;
constexpr uint32_t kErrNonFinite = 8u;  // the query held a NaN or an infinity: no search, empty results

// How a search warp holds its query in shared memory.
//   kQueryRaw:   exact_gpu; the query itself, read by every distance.
//   kQueryRot:   rabitq_gpu; the rotated query q' in dimension order.
//   kQueryPair:  rabitq_gpu with wide 1/2/4-bit records; q' in two halves,
//                chains (0, 1) then chains (2, 3) (chain c = dims j = c mod 4),
//                each half interleaving its two chains by position (dims 4p + 2h
//                and 4p + 2h + 1 adjacent), so the lane that sums chains 2h and
//                2h + 1 of a record reads both chains' next two positions with
//                one 16-byte load.
// In both rabitq layouts the query itself is not resident during the search:
// the seed distance reads it from global memory and the rerank copies it into
// the visited table's words, which are dead by then.
constexpr uint32_t kQueryRaw = 0, kQueryRot = 1, kQueryPair = 2;

// Words between the starts of the two halves of a pair-major q': at least
// dim_pad / 2, and 8 mod 16 so that the two halves' 16-byte reads at one
// position fall in distinct bank groups.
__host__ __device__ inline uint32_t pair_stride(uint32_t dim_pad) { return 2 * (((dim_pad / 4 + 3) & ~7u) + 4); }

// Words of shared memory one warp of the search kernel uses: the beam (cap_pad
// distances + ids), the query in the given layout, four candidate staging
// arrays of 32 x slots-per-lane entries (slots per lane = 2 when R > 32, else
// 1), the visited table (at least dim_pad words in the rabitq layouts, which
// put the query there for the rerank).  Every part is a multiple of 4 words, so
// each starts 16-byte aligned.
__host__ __device__ inline uint32_t search_warp_words(uint32_t cap_pad, uint32_t dim_pad, uint32_t hcap, uint32_t R,
                                                      uint32_t qlayout) {
  const uint32_t qwords = qlayout == kQueryPair ? 2 * pair_stride(dim_pad) : dim_pad;
  const uint32_t twords = qlayout == kQueryRaw ? hcap : (hcap > dim_pad ? hcap : dim_pad);
  return 2 * cap_pad + qwords + (R > 32 ? 256 : 128) + twords;
}

// q' = P^T q (the sequential fmaf chain over i per output) and the query
// factors, for nq queries; rows padded with zeros to qrot_stride.
cudaError_t launch_prepare(const float* queries, uint32_t q_stride, const float* P, const float* c_rot, float* qrot,
                           uint32_t qrot_stride, float* qfac, uint32_t fac_stride, uint32_t dim, uint32_t bits,
                           uint32_t nq, cudaStream_t stream);

// The factors alone, from rows already rotated in qrot (and their zero padding).
cudaError_t launch_query_factors(float* qrot, uint32_t qrot_stride, const float* c_rot, float* qfac,
                                 uint32_t fac_stride, uint32_t dim, uint32_t bits, uint32_t nq, cudaStream_t stream);

// The rotation P split for the tensor cores: tf32 hi and lo planes of dim rows
// x kp floats (K zero-padded to a multiple of 32) in one allocation, and the
// TMA descriptors that read them in 32-float x N-tile boxes.
struct TcRotation {
  CUtensorMap map_hi, map_lo;
  float* split = nullptr;
  uint32_t dim = 0, kp = 0;
};

// Splits P (on `stream`) into t, replacing what t held; allocates.
cudaError_t tc_rotation_prepare(const float* P, uint32_t dim, TcRotation* t, cudaStream_t stream);
void tc_rotation_release(TcRotation* t);

// Q' = Q P^T on tcgen05 tensor cores (3xTF32, P split by tc_rotation_prepare)
// plus the query factors; a bounded mbarrier wait that expires ORs
// kErrTimeout into *err.
cudaError_t launch_prepare_tc(const float* queries, uint32_t q_stride, const TcRotation& t, const float* c_rot,
                              float* qrot, uint32_t qrot_stride, float* qfac, uint32_t fac_stride, uint32_t dim,
                              uint32_t bits, uint32_t nq, uint32_t* err, cudaStream_t stream);

// Launches the persistent search kernel; warps_per_block and blocks come from
// the caller's occupancy computation.
cudaError_t launch_search(const SearchArgs& a, uint32_t warps_per_block, uint32_t blocks, cudaStream_t stream);

// Occupancy helper: blocks per SM for `warps_per_block` warps with the given
// shared memory per block; also sets the kernel's dynamic shared memory
// allowance (to kMaxBlockSmem, whatever the shape).
cudaError_t search_occupancy(uint32_t bits, uint32_t R, uint32_t code_words, bool exact, uint32_t warps_per_block,
                             size_t smem_bytes, int* blocks_per_sm);

// The query layout (kQueryRaw / kQueryRot / kQueryPair) of the search kernel
// instantiation that serves this mode and record shape.
uint32_t search_query_layout(bool exact, uint32_t bits, uint32_t code_words);

// Whether that instantiation loads records after the visited check (records
// wider than 128 bytes) rather than holding them in registers.
bool search_wide_records(bool exact, uint32_t code_words);

// Dynamic shared memory of a search block of `wpb` warps.
size_t search_block_smem(uint32_t cap_pad, uint32_t dim_pad, uint32_t hcap, uint32_t R, bool exact, uint32_t bits,
                         uint32_t code_words, uint32_t wpb);

}  // namespace dvs

struct dvs_index;
namespace dvs {

cudaError_t launch_estimate_ref_layout(const float* qrot, const float* f3, const uint8_t* records, float* out,
                                       uint32_t n, uint32_t dim, uint32_t bits, cudaStream_t stream);
cudaError_t launch_l2_rows(const float* q, const float* cand, float* out, uint32_t n, uint32_t dim,
                           cudaStream_t stream);
cudaError_t launch_fill_f32(float* p, size_t n, float v, cudaStream_t stream);

}  // namespace dvs
