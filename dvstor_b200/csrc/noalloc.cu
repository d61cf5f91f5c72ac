// dvs_search_device_noalloc: the device-resident search of dvs_search_device
// for callers that may not allocate device memory.
//
// Who needs it: processes whose device memory is owned by someone else once
// they are running — a serving engine that reserves the GPU's free HBM for its
// own pool at start-up and fails any later cudaMalloc, or a host framework
// that forbids allocations on its request path because a cudaMalloc there
// synchronises the device and can fail under memory pressure.  dvs_search_device
// sizes its scratch (rotated queries, query factors, work counters, per-warp
// visited-set spill tables) on demand with cudaMalloc; this entry point takes
// all of it from one file-scope __device__ array instead.
//
// The array is kNoAllocScratchBytes (64 MiB).  Every GPU that loads the library
// holds it until the process exits.  Its layout is fixed, whatever the call:
//   work words (256 B) | spill-table epochs (4 B per warp slot, 4096 slots) |
//   rotated queries + factors (8 MiB) | spill tables (64 KB per warp slot)
// The spill tables are as large as dvs_search_device's, so a query that fits
// there fits here and the results are the same; what the fixed size limits is
// the number of warps in flight (kNoAllocTables, about 38 % of a B200's warp
// slots at the 96-dim shape), so a call runs slower than dvs_search_device.
// Its address is looked up once per device with cudaGetSymbolAddress the first
// time the entry point runs on that device (with the device current); make
// that first call before any stream capture.  All calls on a device share the
// array and it keeps the last call's contents: the work counters are cleared
// on the call's stream before every search, and a spill table belongs to one
// warp slot, whose epoch word marks the entries of earlier calls as empty.
// Calls on one index and device are ordered on the GPU after each other (and
// after that index's other searches); calls on different indexes whose work
// overlaps on the GPU race on the array and must be serialised by the caller.

#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>
#include <string>

#include "index_state.h"

using dvs::fail;

namespace dvs {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(64) << 20;
constexpr size_t kWorkBytes = 256;
constexpr uint32_t kNoAllocMaxSlots = 4096;                    // epoch words
constexpr size_t kEpochBytes = size_t(kNoAllocMaxSlots) * 4;
constexpr size_t kNoAllocQueryBytes = size_t(8) << 20;          // rotated queries + factors
constexpr size_t kTableBytes = size_t(kOverflowSlots) * 4;
constexpr size_t kTablesOffset = kWorkBytes + kEpochBytes + kNoAllocQueryBytes;
constexpr uint32_t kNoAllocTables = uint32_t((kNoAllocScratchBytes - kTablesOffset) / kTableBytes);
static_assert(kNoAllocTables > 0 && kNoAllocTables <= kNoAllocMaxSlots, "scratch layout");

// zero-initialised at module load: every spill table empty, every epoch 0
__device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
unsigned char* g_scratch_addr[kMaxDevices] = {};

dvs_status scratch_address(int device, unsigned char** out) {
  if (device < 0 || device >= kMaxDevices) return fail(DVS_ERR_ARG, "device ordinal out of range");
  std::lock_guard<std::mutex> g(g_mu);
  if (!g_scratch_addr[device]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess)
      return fail(DVS_ERR_CUDA, std::string("cudaGetSymbolAddress(scratch): ") + cudaGetErrorString(e));
    g_scratch_addr[device] = static_cast<unsigned char*>(p);
  }
  *out = g_scratch_addr[device];
  return DVS_OK;
}

dvs_status noalloc_enqueue(dvs_index* ix, Device& d, const float* d_queries, uint32_t nq, uint32_t k,
                           uint32_t beam_width, bool rabitq, uint32_t* d_out_ids, float* d_out_dist,
                           uint32_t* d_counters, cudaStream_t st) {
  const DevLayout& lay = d.lay;
  if (lay.n == 0) {
    // an index created empty and not yet inserted into: every result slot is empty
    DVS_CUDA(cudaMemsetAsync(d_out_ids, 0xFF, size_t(nq) * k * 4, st));
    DVS_CUDA(launch_fill_f32(d_out_dist, size_t(nq) * k, __builtin_huge_valf(), st));
    if (d_counters) DVS_CUDA(cudaMemsetAsync(d_counters, 0, size_t(nq) * 16, st));
    return DVS_OK;
  }
  unsigned char* base = nullptr;
  dvs_status s = scratch_address(d.ordinal, &base);
  if (s != DVS_OK) return s;
  const uint32_t cap = rabitq ? beam_width + kBeamSlack : beam_width;
  LaunchShape sh;
  s = launch_shape(d, cap, ix->slots_per_entry, !rabitq, sh);
  if (s != DVS_OK) return s;

  uint32_t* work = reinterpret_cast<uint32_t*>(base);
  uint32_t* epochs = reinterpret_cast<uint32_t*>(base + kWorkBytes);
  float* qfac = reinterpret_cast<float*>(base + kWorkBytes + kEpochBytes);
  const size_t qfac_bytes = (size_t(nq) * 16 + 255) / 256 * 256;
  float* qrot = reinterpret_cast<float*>(base + kWorkBytes + kEpochBytes + qfac_bytes);
  uint32_t* tables = reinterpret_cast<uint32_t*>(base + kTablesOffset);
  // one spill table per warp slot: as many blocks as have a table for every warp
  const uint32_t blocks_needed = (nq + sh.wpb - 1) / sh.wpb;
  const uint32_t blocks_fit = std::max(1u, kNoAllocTables / sh.wpb);
  const uint32_t blocks = std::max(1u, std::min({sh.blocks_per_sm * d.sm_count, blocks_needed, blocks_fit}));

  DVS_CUDA(cudaMemsetAsync(work, 0, 16, st));
  if (rabitq) {
    if (ix->rotation == DVS_ROTATION_TENSOR)
      DVS_CUDA(launch_prepare_tc(d_queries, lay.dim, d.tc, lay.c_rot, qrot, lay.vec_stride, qfac, 4, lay.dim,
                                 lay.bits, nq, work + 1, st));
    else
      DVS_CUDA(launch_prepare(d_queries, lay.dim, lay.P, lay.c_rot, qrot, lay.vec_stride, qfac, 4, lay.dim, lay.bits,
                              nq, st));
  }
  SearchArgs a;
  a.ix = lay;
  a.queries = d_queries;
  a.qrot = qrot;
  a.qfac = qfac;
  a.nq = nq;
  a.k = k;
  a.L = beam_width;
  a.cap = cap;
  a.mode = rabitq ? 0u : 1u;
  a.hop_limit = ix->hop_limit;
  a.out_ids = d_out_ids;
  a.out_dist = d_out_dist;
  a.counters = d_counters;
  a.work = work;
  a.ovf = tables;
  a.ovf_epoch = epochs;
  a.ovf_cap = kOverflowSlots;
  a.ovf_limit = kOverflowSlots / 10 * 8;
  a.ovf_tagged = lay.n < (uint64_t(1) << 24) ? 1u : 0u;
  a.hcap = sh.hcap;
  a.hlimit = sh.hlimit;
  a.vt16 = sh.vt16;
  a.hbuckets = sh.hbuckets;
  a.hb_magic = sh.hbuckets ? uint32_t(0xFFFFFFFFull / sh.hbuckets + 1) : 0u;
  a.cap_pad = sh.cap_pad;
  a.dim_pad = lay.vec_stride;
  DVS_CUDA(launch_search(a, sh.wpb, blocks, st));
  return DVS_OK;
}

}  // namespace
}  // namespace dvs

extern "C" dvs_status dvs_search_device_noalloc(dvs_index* index, uint32_t device_slot, const float* d_queries,
                                                uint32_t nq, uint32_t dim, uint32_t k, uint32_t beam_width,
                                                dvs_mode mode, uint32_t* d_out_ids, float* d_out_dist,
                                                uint32_t* d_counters, void* stream) {
  using namespace dvs;
  if (!index) return fail(DVS_ERR_ARG, "null index");
  if (device_slot >= index->devs.size()) return fail(DVS_ERR_ARG, "device slot out of range");
  if (mode != DVS_MODE_RABITQ_GPU && mode != DVS_MODE_EXACT_GPU)
    return fail(DVS_ERR_ARG, "search-mode must be exact_gpu or rabitq_gpu");
  if (dim != index->host.info.dim) return fail(DVS_ERR_DIM, "search dimension mismatch");
  if (k == 0 || beam_width < k) return fail(DVS_ERR_ARG, "k must be > 0 and beam_width >= k");
  if (beam_width > 4096) return fail(DVS_ERR_ARG, "beam_width above 4096 is not supported");
  if (nq == 0) return DVS_OK;
  if (!d_queries || !d_out_ids || !d_out_dist) return fail(DVS_ERR_ARG, "null buffer");
  // the index's arrays are replaced by dvs_insert / dvs_reserve under this lock
  std::lock_guard<std::mutex> g(index->mu);
  Device& d = index->devs[device_slot];
  const DevLayout& lay = d.lay;
  if (lay.R > 64) return fail(DVS_ERR_UNSUPPORTED, "max out-degree above 64 is not supported by the search kernel");
  const size_t per_query = size_t(lay.vec_stride) * 4 + 16;
  const size_t max_nq = (kNoAllocQueryBytes - 256) / per_query;
  if (nq > max_nq)
    return fail(DVS_ERR_CAPACITY, "dvs_search_device_noalloc takes at most " + std::to_string(max_nq) +
                                      " queries of dim " + std::to_string(dim) + " per call (" +
                                      std::to_string(kNoAllocQueryBytes >> 20) +
                                      " MiB of its fixed scratch); got " + std::to_string(nq));
  DVS_CUDA(cudaSetDevice(d.ordinal));
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : d.sc.stream;
  // after the previous search on this device, whichever stream it used
  DVS_CUDA(cudaStreamWaitEvent(st, d.sc.done, 0));
  const dvs_status rc = noalloc_enqueue(index, d, d_queries, nq, k, beam_width, mode == DVS_MODE_RABITQ_GPU,
                                        d_out_ids, d_out_dist, d_counters, st);
  const cudaError_t e = cudaEventRecord(d.sc.done, st);
  if (rc == DVS_OK && e != cudaSuccess)
    return fail(DVS_ERR_CUDA, std::string("cudaEventRecord: ") + cudaGetErrorString(e));
  return rc;
}
