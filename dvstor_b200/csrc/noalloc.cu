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
// The array is kNoAllocScratchBytes (16 MiB).  Every GPU that loads the library
// holds it until the process exits.  Its address is looked up once per device
// with cudaGetSymbolAddress the first time the entry point runs on that device
// (with the device current); make that first call before any stream capture.
// All calls on a device share the array and it keeps the last call's
// contents: the work counters are cleared on the call's stream before every
// search and the spill tables by the kernel when a query first spills, so
// back-to-back calls are independent, but calls whose work overlaps on the
// GPU (different streams, or different threads) race on the array and must be
// serialised by the caller.

#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>
#include <string>

#include "internal.h"
#include "search.cuh"

using dvs::fail;

namespace dvs {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;
constexpr size_t kNoAllocQueryBytes = size_t(8) << 20;  // rotated queries + factors
constexpr size_t kWorkBytes = 256;

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

}  // namespace
}  // namespace dvs

extern "C" dvs_status dvs_search_device_noalloc(dvs_index* index, uint32_t device_slot, const float* d_queries,
                                                uint32_t nq, uint32_t dim, uint32_t k, uint32_t beam_width,
                                                dvs_mode mode, uint32_t* d_out_ids, float* d_out_dist,
                                                uint32_t* d_counters, void* stream) {
  using namespace dvs;
  DeviceView v;
  dvs_status s = device_view(index, device_slot, &v);
  if (s != DVS_OK) return s;
  if (mode != DVS_MODE_RABITQ_GPU && mode != DVS_MODE_EXACT_GPU)
    return fail(DVS_ERR_ARG, "search-mode must be exact_gpu or rabitq_gpu");
  if (dim != v.index_dim) return fail(DVS_ERR_DIM, "search dimension mismatch");
  if (k == 0 || beam_width < k) return fail(DVS_ERR_ARG, "k must be > 0 and beam_width >= k");
  if (beam_width > 4096) return fail(DVS_ERR_ARG, "beam_width above 4096 is not supported");
  if (nq == 0) return DVS_OK;
  if (!d_queries || !d_out_ids || !d_out_dist) return fail(DVS_ERR_ARG, "null buffer");
  const bool rabitq = mode == DVS_MODE_RABITQ_GPU;
  const DevLayout& lay = v.lay;
  if (lay.R > 64) return fail(DVS_ERR_UNSUPPORTED, "max out-degree above 64 is not supported by the search kernel");
  const size_t per_query = size_t(lay.vec_stride) * 4 + 16;
  const size_t max_nq = kNoAllocQueryBytes / per_query;
  if (nq > max_nq)
    return fail(DVS_ERR_CAPACITY, "dvs_search_device_noalloc takes at most " + std::to_string(max_nq) +
                                      " queries of dim " + std::to_string(dim) + " per call (" +
                                      std::to_string(kNoAllocQueryBytes >> 20) +
                                      " MiB of its fixed scratch); got " + std::to_string(nq));

  cudaError_t e = cudaSetDevice(v.ordinal);
  if (e != cudaSuccess) return fail(DVS_ERR_CUDA, std::string("cudaSetDevice: ") + cudaGetErrorString(e));
  if (lay.n == 0) {
    // an index created empty and not yet inserted into: every result slot is empty
    cudaStream_t st0 = static_cast<cudaStream_t>(stream);
    e = cudaMemsetAsync(d_out_ids, 0xFF, size_t(nq) * k * 4, st0);
    if (e == cudaSuccess) e = launch_fill_f32(d_out_dist, size_t(nq) * k, __builtin_huge_valf(), st0);
    if (e == cudaSuccess && d_counters) e = cudaMemsetAsync(d_counters, 0, size_t(nq) * 16, st0);
    if (e != cudaSuccess) return fail(DVS_ERR_CUDA, std::string("empty-index result fill: ") + cudaGetErrorString(e));
    return DVS_OK;
  }
  unsigned char* base = nullptr;
  s = scratch_address(v.ordinal, &base);
  if (s != DVS_OK) return s;
  const uint32_t cap = rabitq ? beam_width + kBeamSlack : beam_width;
  SearchShape sh;
  s = search_shape(index, device_slot, cap, !rabitq, &sh);
  if (s != DVS_OK) return s;

  // layout of the fixed scratch: work words | factors | rotated queries | spill tables
  uint32_t* work = reinterpret_cast<uint32_t*>(base);
  float* qfac = reinterpret_cast<float*>(base + kWorkBytes);
  const size_t qfac_bytes = (size_t(nq) * 16 + 255) / 256 * 256;
  float* qrot = reinterpret_cast<float*>(base + kWorkBytes + qfac_bytes);
  const size_t qrot_bytes = (size_t(nq) * lay.vec_stride * 4 + 255) / 256 * 256;
  unsigned char* spill = base + kWorkBytes + qfac_bytes + qrot_bytes;
  const size_t spill_bytes = kNoAllocScratchBytes - (kWorkBytes + qfac_bytes + qrot_bytes);
  // per-warp spill tables: the largest power of two (<= 16384 entries) that
  // gives every resident warp one; with fewer than 1024 entries per warp, run
  // fewer warps instead
  const uint32_t blocks_needed = (nq + sh.wpb - 1) / sh.wpb;
  uint32_t blocks = std::max(1u, std::min(sh.blocks_per_sm * v.sm_count, blocks_needed));
  uint32_t ovf_cap = 16384;
  while (ovf_cap > 1024 && size_t(blocks) * sh.wpb * ovf_cap * 4 > spill_bytes) ovf_cap >>= 1;
  while (blocks > 1 && size_t(blocks) * sh.wpb * ovf_cap * 4 > spill_bytes) --blocks;

  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : v.stream;
  e = cudaMemsetAsync(work, 0, 16, st);
  if (e != cudaSuccess) return fail(DVS_ERR_CUDA, std::string("cudaMemsetAsync: ") + cudaGetErrorString(e));
  if (rabitq) {
    e = launch_prepare(d_queries, lay.dim, lay.P, lay.c_rot, qrot, lay.vec_stride, qfac, 4, lay.dim, lay.bits, nq, st);
    if (e != cudaSuccess) return fail(DVS_ERR_CUDA, std::string("prepare launch: ") + cudaGetErrorString(e));
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
  a.hop_limit = v.hop_limit;
  a.out_ids = d_out_ids;
  a.out_dist = d_out_dist;
  a.counters = d_counters;
  a.work = work;
  a.ovf = reinterpret_cast<uint32_t*>(spill);
  a.ovf_cap = ovf_cap;
  a.ovf_limit = ovf_cap / 10 * 8;
  a.hcap = sh.hcap;
  a.hlimit = sh.hlimit;
  a.vt16 = sh.vt16;
  a.hbuckets = sh.hbuckets;
  a.inv_hbuckets = sh.hbuckets ? 1.0f / float(sh.hbuckets) : 0.f;
  a.cap_pad = sh.cap_pad;
  a.dim_pad = lay.vec_stride;
  e = launch_search(a, sh.wpb, blocks, st);
  if (e != cudaSuccess) return fail(DVS_ERR_CUDA, std::string("search launch: ") + cudaGetErrorString(e));
  return DVS_OK;
}
