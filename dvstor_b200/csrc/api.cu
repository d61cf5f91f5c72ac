// C ABI of the query path: index lifetime, device layout upload, search
// orchestration and the kernel-level entry points.  Replaces the reference's
// GPU launcher (src/gpu/gpu_kernel_launcher.cu) and per-coroutine buffer
// manager (src/gpu/gpu_buffer_manager.cu) for queries: the library owns the
// device copy of the index and every scratch buffer, and reports failures as
// status codes instead of abort().

#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <mutex>
#include <thread>
#include <vector>

#include "index_state.h"

using dvs::fail;

namespace dvs {
namespace {

// Uploads the rows of shard `shard` of `nshard` (slot g with g mod nshard ==
// shard, local row g / nshard; nshard == 1 uploads everything).
dvs_status upload(Device& d, const HostIndex& h, uint32_t shard, uint32_t nshard) {
  const dvs_index_info& in = h.info;
  const uint64_t n = in.num_vectors;
  const uint64_t nl = (n + nshard - 1 - shard) / nshard;
  const uint32_t dim = in.dim, R = in.R, bits = in.rabitq_bits;
  const uint32_t packed = (bits * dim + 7) / 8;
  const uint32_t code_words = (packed + 3) / 4;
  const uint32_t rec_words = (code_words + 2 + 3) / 4 * 4;
  const uint32_t vec_stride = (dim + 3) / 4 * 4;
  DVS_CUDA(cudaSetDevice(d.ordinal));
  int sms = 0;
  DVS_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, d.ordinal));
  d.sm_count = uint32_t(sms);
  DVS_CUDA(d.sc.create());
  DVS_CUDA(d.ins.create());
  // records: reference layout -> [codes | pad to word | add | rescale | pad to 16 B]
  std::vector<uint32_t> rec(size_t(nl) * rec_words, 0u);
  std::vector<uint32_t> adj(size_t(nl) * R);
  std::vector<float> vecs(size_t(nl) * vec_stride, 0.f);
  for (uint64_t l = 0; l < nl; ++l) {
    const uint64_t g = l * nshard + shard;
    const uint8_t* src = h.records.data() + g * in.rabitq_size;
    uint8_t* dst = reinterpret_cast<uint8_t*>(rec.data() + l * rec_words);
    std::memcpy(dst, src, packed);
    std::memcpy(dst + size_t(code_words) * 4, src + packed, 8);
    std::memcpy(&adj[l * R], &h.adj[g * R], size_t(R) * 4);
    std::memcpy(&vecs[l * vec_stride], &h.vecs[g * dim], size_t(dim) * 4);
  }
  DVS_CUDA(cudaMalloc(&d.adj, adj.size() * 4));
  DVS_CUDA(cudaMalloc(&d.rec, rec.size() * 4));
  DVS_CUDA(cudaMalloc(&d.vecs, vecs.size() * 4));
  DVS_CUDA(cudaMalloc(&d.ids, size_t(n) * 4));
  DVS_CUDA(cudaMalloc(&d.P, size_t(dim) * dim * 4));
  DVS_CUDA(cudaMalloc(&d.c_rot, size_t(dim) * 4));
  DVS_CUDA(cudaMemcpy(d.adj, adj.data(), adj.size() * 4, cudaMemcpyHostToDevice));
  DVS_CUDA(cudaMemcpy(d.rec, rec.data(), rec.size() * 4, cudaMemcpyHostToDevice));
  DVS_CUDA(cudaMemcpy(d.vecs, vecs.data(), vecs.size() * 4, cudaMemcpyHostToDevice));
  DVS_CUDA(cudaMemcpy(d.ids, h.ids.data(), size_t(n) * 4, cudaMemcpyHostToDevice));
  DVS_CUDA(cudaMemcpy(d.P, h.rotation.data(), size_t(dim) * dim * 4, cudaMemcpyHostToDevice));
  DVS_CUDA(cudaMemcpy(d.c_rot, h.rotated_centroid.data(), size_t(dim) * 4, cudaMemcpyHostToDevice));
  d.shard = shard;
  d.rows = nl;
  d.cap_rows = nl;
  DevLayout& L = d.lay;
  L.adj = d.adj;
  L.rec = d.rec;
  L.vecs = d.vecs;
  L.ids = d.ids;
  L.P = d.P;
  L.c_rot = d.c_rot;
  L.n = n;
  L.dim = dim;
  L.R = R;
  L.bits = bits;
  L.medoid = in.medoid;
  L.metric = in.metric == DVS_METRIC_IP ? 1u : 0u;
  L.rec_words = rec_words;
  L.code_words = code_words;
  L.vec_stride = vec_stride;
  L.adj_s[0] = d.adj;
  L.rec_s[0] = d.rec;
  L.vecs_s[0] = d.vecs;
  return DVS_OK;
}

// Sharded placement: every device may read every other device's shard.
dvs_status link_shards(std::vector<Device>& devs) {
  const uint32_t ns = uint32_t(devs.size());
  for (uint32_t i = 0; i < ns; ++i) {
    for (uint32_t j = 0; j < ns; ++j) {
      if (devs[i].ordinal == devs[j].ordinal) continue;
      int can = 0;
      DVS_CUDA(cudaDeviceCanAccessPeer(&can, devs[i].ordinal, devs[j].ordinal));
      if (!can)
        return fail(DVS_ERR_PEER, "device " + std::to_string(devs[i].ordinal) + " cannot access device " +
                                      std::to_string(devs[j].ordinal) + "'s memory; open the index replicated");
      DVS_CUDA(cudaSetDevice(devs[i].ordinal));
      const cudaError_t e = cudaDeviceEnablePeerAccess(devs[j].ordinal, 0);
      if (e == cudaErrorPeerAccessAlreadyEnabled)
        cudaGetLastError();
      else if (e != cudaSuccess)
        return fail(DVS_ERR_PEER, std::string("cudaDeviceEnablePeerAccess: ") + cudaGetErrorString(e));
    }
  }
  uint32_t log = 0;
  while ((1u << log) < ns) ++log;
  for (auto& d : devs) {
    d.lay.shard_log = log;
    d.lay.shard_mask = ns - 1;
    for (uint32_t s = 0; s < ns; ++s) {
      d.lay.adj_s[s] = devs[s].adj;
      d.lay.rec_s[s] = devs[s].rec;
      d.lay.vecs_s[s] = devs[s].vecs;
    }
  }
  return DVS_OK;
}

}  // namespace

dvs_status ensure_scratch(Device& d, Scratch& sc, size_t nq, size_t k, bool host_path) {
  const size_t vs = d.lay.vec_stride;
  if (nq > sc.q_cap) {
    const size_t cap = std::max(nq, sc.q_cap * 2);
    dev_free(sc.queries);
    dev_free(sc.qrot);
    dev_free(sc.qfac);
    dev_free(sc.counters);
    DVS_CUDA(cudaMalloc(&sc.queries, cap * d.lay.dim * 4));
    DVS_CUDA(cudaMalloc(&sc.qrot, cap * vs * 4));
    DVS_CUDA(cudaMalloc(&sc.qfac, cap * 16));
    DVS_CUDA(cudaMalloc(&sc.counters, cap * 16));
    sc.q_cap = cap;
  }
  if (host_path && nq * k > sc.out_cap) {
    const size_t cap = std::max(nq * k, sc.out_cap * 2);
    dev_free(sc.out_ids);
    dev_free(sc.out_dist);
    DVS_CUDA(cudaMalloc(&sc.out_ids, cap * 4));
    DVS_CUDA(cudaMalloc(&sc.out_dist, cap * 4));
    sc.out_cap = cap;
  }
  return DVS_OK;
}

namespace {
std::mutex g_shape_mu;  // guards Device::shapes
}  // namespace

dvs_status launch_shape(Device& d, uint32_t cap, uint32_t slots_per_entry, bool exact, LaunchShape& s) {
  const bool t16 = d.lay.n < (1u << 24);
  const uint32_t vt16 = d.lay.n < (1u << 20) ? 20u : 24u;
  const uint64_t key = uint64_t(cap) | uint64_t(slots_per_entry) << 24 | uint64_t(exact) << 40 |
                       uint64_t(t16) << 41 | uint64_t(vt16 == 20) << 42;
  {
    std::lock_guard<std::mutex> g(g_shape_mu);
    const auto it = d.shapes.find(key);
    if (it != d.shapes.end()) {
      s = it->second;
      return DVS_OK;
    }
  }
  // the given table size, or the largest in [kSlotsMin, kSlotsMax] that keeps
  // the most warps resident
  const uint32_t hi = slots_per_entry ? slots_per_entry : kSlotsMax;
  const uint32_t lo = slots_per_entry ? slots_per_entry : kSlotsMin;
  int best_warps = 0;
  LaunchShape best;
  for (uint32_t spe = hi; spe >= lo; --spe) {
    LaunchShape c;
    c.cap = cap;
    c.cap_pad = (cap + 31) / 32 * 32;
    if (t16) {
      // 16-bit entries, 8 per 16-byte bucket; at least 2^(W-14) buckets for
      // hash width W.  Two-choice buckets fill to the last entry: an id spills
      // only when both its buckets are full.
      c.vt16 = vt16;
      c.hbuckets = std::max(1u << (vt16 - 14), (cap * spe + 7) / 8);
      c.hcap = c.hbuckets * 4;
      c.hlimit = c.hbuckets * 8;
    } else {
      c.hcap = std::max(64u, (cap * spe + 31) / 32 * 32);
      c.hlimit = c.hcap / 10 * 9;
    }
    for (uint32_t wpb : {1u, 2u, 4u, 8u}) {
      const size_t smem =
          search_block_smem(c.cap_pad, d.lay.vec_stride, c.hcap, d.lay.R, exact, d.lay.bits, d.lay.code_words, wpb);
      if (smem > size_t(kMaxBlockSmem)) break;
      int bps = 0;
      const cudaError_t e = search_occupancy(d.lay.bits, d.lay.R, d.lay.code_words, exact, wpb, smem, &bps);
      if (e != cudaSuccess) return fail(DVS_ERR_CUDA, std::string("occupancy query: ") + cudaGetErrorString(e));
      if (bps == 0) break;  // more than a block's shared memory
      if (int(wpb) * bps > best_warps) {
        best_warps = int(wpb) * bps;
        c.wpb = wpb;
        c.blocks_per_sm = uint32_t(bps);
        best = c;
      }
    }
    if (spe == 0) break;
  }
  if (best_warps == 0)
    return fail(DVS_ERR_CAPACITY, "beam capacity " + std::to_string(cap) + " needs more shared memory than a block has");
  s = best;
  std::lock_guard<std::mutex> g(g_shape_mu);
  d.shapes[key] = best;
  return DVS_OK;
}

}  // namespace dvs


namespace dvs {

// Prepare + search for nq device-resident queries on one device.
dvs_status search_on(dvs_index* ix, Device& d, Scratch& sc, const float* d_q, uint32_t nq, uint32_t k, uint32_t L,
                     dvs_mode mode, uint32_t* d_ids, float* d_dist, uint32_t* d_counters, cudaStream_t st,
                     bool timed, bool out_slots) {
  if (d.lay.R > 64) return fail(DVS_ERR_UNSUPPORTED, "max out-degree above 64 is not supported by the search kernel");
  // after the previous search on this scratch, whichever stream it used
  DVS_CUDA(cudaStreamWaitEvent(st, sc.done, 0));
  dvs_status rc = search_enqueue(ix, d, sc, d_q, nq, k, L, mode, d_ids, d_dist, d_counters, st, timed, out_slots);
  const cudaError_t e = cudaEventRecord(sc.done, st);
  if (rc == DVS_OK && e != cudaSuccess)
    return fail(DVS_ERR_CUDA, std::string("cudaEventRecord: ") + cudaGetErrorString(e));
  return rc;
}

dvs_status search_enqueue(dvs_index* ix, Device& d, Scratch& sc, const float* d_q, uint32_t nq, uint32_t k,
                          uint32_t L, dvs_mode mode, uint32_t* d_ids, float* d_dist, uint32_t* d_counters,
                          cudaStream_t st, bool timed, bool out_slots) {
  const DevLayout& lay = d.lay;
  const bool rabitq = mode == DVS_MODE_RABITQ_GPU;
  if (lay.n == 0) {
    // an index created empty and not yet inserted into: every result slot is empty
    if (timed) DVS_CUDA(cudaEventRecord(sc.ev0, st));
    DVS_CUDA(cudaMemsetAsync(d_ids, 0xFF, size_t(nq) * k * 4, st));
    DVS_CUDA(launch_fill_f32(d_dist, size_t(nq) * k, __builtin_huge_valf(), st));
    if (d_counters) DVS_CUDA(cudaMemsetAsync(d_counters, 0, size_t(nq) * 16, st));
    DVS_CUDA(cudaMemsetAsync(sc.work, 0, 16, st));
    if (timed) DVS_CUDA(cudaEventRecord(sc.ev1, st));
    return DVS_OK;
  }
  const uint32_t cap = rabitq ? L + kBeamSlack : L;
  LaunchShape s;
  dvs_status rc = launch_shape(d, cap, ix->slots_per_entry, !rabitq, s);
  if (rc != DVS_OK) return rc;
  rc = ensure_scratch(d, sc, nq, k, false);
  if (rc != DVS_OK) return rc;
  const uint32_t blocks_full = s.blocks_per_sm * d.sm_count;
  const uint32_t blocks_needed = (nq + s.wpb - 1) / s.wpb;
  const uint32_t blocks = std::max(1u, std::min(blocks_full, blocks_needed));
  const size_t slots = size_t(blocks) * s.wpb;
  if (slots > sc.ovf_slots) {
    // spill tables and their epoch words start zeroed: every entry empty
    dev_free(sc.ovf);
    DVS_CUDA(cudaMalloc(&sc.ovf, slots * (size_t(kOverflowSlots) + 1) * 4));
    DVS_CUDA(cudaMemsetAsync(sc.ovf, 0, slots * (size_t(kOverflowSlots) + 1) * 4, st));
    sc.ovf_slots = slots;
  }
  DVS_CUDA(cudaMemsetAsync(sc.work, 0, 16, st));
  cudaEvent_t* tr = nullptr;
  if (ix->kernel_timing && &sc == &d.sc && !d.tev.empty()) {
    if (d.tcount < Device::kRing) tr = &d.tev[3 * d.tcount++];
  }
  if (timed) DVS_CUDA(cudaEventRecord(sc.ev0, st));
  if (tr) DVS_CUDA(cudaEventRecord(tr[0], st));
  if (rabitq) {
    if (ix->rotation == DVS_ROTATION_TENSOR)
      DVS_CUDA(launch_prepare_tc(d_q, lay.dim, d.tc, lay.c_rot, sc.qrot, lay.vec_stride, sc.qfac, 4, lay.dim, lay.bits,
                                 nq, sc.work + 1, st));
    else
      DVS_CUDA(launch_prepare(d_q, lay.dim, lay.P, lay.c_rot, sc.qrot, lay.vec_stride, sc.qfac, 4, lay.dim, lay.bits, nq,
                              st));
  }
  if (tr) DVS_CUDA(cudaEventRecord(tr[1], st));
  SearchArgs a;
  a.ix = lay;
  a.queries = d_q;
  a.qrot = sc.qrot;
  a.qfac = sc.qfac;
  a.nq = nq;
  a.k = k;
  a.L = L;
  a.cap = cap;
  a.mode = rabitq ? 0u : 1u;
  a.hop_limit = ix->hop_limit;
  a.out_ids = d_ids;
  a.out_dist = d_dist;
  a.counters = d_counters ? d_counters : sc.counters;
  a.work = sc.work;
  a.ovf = sc.ovf;
  a.ovf_epoch = sc.ovf + sc.ovf_slots * kOverflowSlots;
  a.ovf_cap = kOverflowSlots;
  a.ovf_limit = kOverflowSlots / 10 * 8;
  a.ovf_tagged = lay.n < (uint64_t(1) << 24) ? 1u : 0u;
  a.hcap = s.hcap;
  a.hlimit = s.hlimit;
  a.vt16 = s.vt16;
  a.hbuckets = s.hbuckets;
  a.hb_magic = s.hbuckets ? uint32_t(0xFFFFFFFFull / s.hbuckets + 1) : 0u;
  a.cap_pad = s.cap_pad;
  a.dim_pad = lay.vec_stride;
  a.out_slots = out_slots ? 1u : 0u;
  DVS_CUDA(launch_search(a, s.wpb, blocks, st));
  if (tr) DVS_CUDA(cudaEventRecord(tr[2], st));
  if (timed) DVS_CUDA(cudaEventRecord(sc.ev1, st));
  return DVS_OK;
}

namespace {

dvs_status check_query_args(const dvs_index* ix, uint32_t nq, uint32_t dim, uint32_t k, uint32_t L, dvs_mode mode) {
  if (!ix) return fail(DVS_ERR_ARG, "null index");
  if (mode != DVS_MODE_RABITQ_GPU && mode != DVS_MODE_EXACT_GPU)
    return fail(DVS_ERR_ARG, "search-mode must be exact_gpu or rabitq_gpu");
  if (dim != ix->host.info.dim)
    return fail(DVS_ERR_DIM, "search dimension mismatch: index " + std::to_string(ix->host.info.dim) + ", query " +
                                 std::to_string(dim));
  if (k == 0) return fail(DVS_ERR_ARG, "k must be > 0");
  if (L < k) return fail(DVS_ERR_ARG, "beam_width must be >= k");
  if (L > 4096) return fail(DVS_ERR_ARG, "beam_width above 4096 is not supported");
  (void)nq;
  return DVS_OK;
}

}  // namespace
}  // namespace dvs

extern "C" {

int dvs_device_count(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

dvs_status dvs_open(const dvs_open_params* p, dvs_index** out) {
  if (!p || !out || !p->index_prefix) return fail(DVS_ERR_ARG, "null argument");
  *out = nullptr;
  if (p->placement != DVS_PLACE_REPLICATE && p->placement != DVS_PLACE_SHARD)
    return fail(DVS_ERR_ARG, "placement must be DVS_PLACE_REPLICATE or DVS_PLACE_SHARD");
  const int ndev_vis = dvs_device_count();
  if (ndev_vis == 0) return fail(DVS_ERR_NO_DEVICE, "no CUDA device is visible");
  std::vector<int> devs;
  const uint32_t nd = p->num_devices ? p->num_devices : 1;
  for (uint32_t i = 0; i < nd; ++i) {
    const int o = p->devices ? p->devices[i] : int(i);
    if (o < 0 || o >= ndev_vis) return fail(DVS_ERR_ARG, "device ordinal " + std::to_string(o) + " is not visible");
    devs.push_back(o);
  }
  auto* ix = new (std::nothrow) dvs_index;
  if (!ix) return fail(DVS_ERR_OOM, "host allocation failed");
  dvs_status s = dvs::load_host_index(p->index_prefix, ix->host);
  const dvs_index_info& in = ix->host.info;
  if (s == DVS_OK && p->expect_dim && p->expect_dim != in.dim)
    s = fail(DVS_ERR_DIM, "RaBitQ artifact dim mismatch: expected " + std::to_string(p->expect_dim) + ", got " +
                              std::to_string(in.dim));
  if (s == DVS_OK && p->expect_bits && p->expect_bits != in.rabitq_bits)
    s = fail(DVS_ERR_BITS, "RaBitQ artifact bits mismatch: expected " + std::to_string(p->expect_bits) + ", got " +
                               std::to_string(in.rabitq_bits));
  if (s == DVS_OK && p->expect_memory_nodes && p->expect_memory_nodes != in.num_memory_nodes)
    s = fail(DVS_ERR_FORMAT, "RaBitQ artifact memory-node count mismatch: expected " +
                                 std::to_string(p->expect_memory_nodes) + ", got " +
                                 std::to_string(in.num_memory_nodes));
  const bool sharded = p->placement == DVS_PLACE_SHARD && devs.size() > 1;
  if (s == DVS_OK && sharded) {
    const size_t ns = devs.size();
    if (ns > dvs::kMaxShards || (ns & (ns - 1)) != 0)
      s = fail(DVS_ERR_ARG, "sharded placement needs a power-of-two device count up to 16");
    else if (in.num_vectors < ns)
      s = fail(DVS_ERR_ARG, "fewer nodes than shards");
  }
  if (s == DVS_OK) {
    ix->devs.resize(devs.size());
    for (size_t i = 0; i < devs.size() && s == DVS_OK; ++i) {
      ix->devs[i].ordinal = devs[i];
      s = sharded ? dvs::upload(ix->devs[i], ix->host, uint32_t(i), uint32_t(devs.size()))
                  : dvs::upload(ix->devs[i], ix->host, 0, 1);
    }
    if (s == DVS_OK && sharded) s = dvs::link_shards(ix->devs);
  }
  if (s != DVS_OK) {
    for (auto& d : ix->devs) d.release();
    delete ix;
    return s;
  }
  *out = ix;
  return DVS_OK;
}

dvs_status dvs_create(const dvs_create_params* p, dvs_index** out) {
  if (!p || !out || !p->rotation || !p->rotated_centroid) return fail(DVS_ERR_ARG, "null argument");
  *out = nullptr;
  if (p->dim == 0) return fail(DVS_ERR_DIM, "dim must be > 0");
  if (p->R == 0 || p->R > 64) return fail(DVS_ERR_ARG, "R must be in 1..64");
  if (p->rabitq_bits != 1 && p->rabitq_bits != 2 && p->rabitq_bits != 4 && p->rabitq_bits != 8)
    return fail(DVS_ERR_BITS, "rabitq_bits must be 1, 2, 4, or 8");
  if (p->metric != DVS_METRIC_L2 && p->metric != DVS_METRIC_IP) return fail(DVS_ERR_ARG, "metric must be l2 or ip");
  const int ndev_vis = dvs_device_count();
  if (ndev_vis == 0) return fail(DVS_ERR_NO_DEVICE, "no CUDA device is visible");
  const uint32_t nd = p->num_devices ? p->num_devices : 1;
  std::vector<int> devs;
  for (uint32_t i = 0; i < nd; ++i) {
    const int o = p->devices ? p->devices[i] : int(i);
    if (o < 0 || o >= ndev_vis) return fail(DVS_ERR_ARG, "device ordinal " + std::to_string(o) + " is not visible");
    devs.push_back(o);
  }
  auto* ix = new (std::nothrow) dvs_index;
  if (!ix) return fail(DVS_ERR_OOM, "host allocation failed");
  dvs_index_info& in = ix->host.info;
  in.num_vectors = 0;
  in.dim = p->dim;
  in.R = p->R;
  in.rabitq_bits = p->rabitq_bits;
  in.rabitq_size = (p->rabitq_bits * p->dim + 7) / 8 + 8;
  in.num_memory_nodes = 1;
  in.medoid = 0;
  in.metric = p->metric;
  in.t_const = p->t_const;
  ix->host.rotation.assign(p->rotation, p->rotation + size_t(p->dim) * p->dim);
  ix->host.rotated_centroid.assign(p->rotated_centroid, p->rotated_centroid + p->dim);
  dvs_status s = DVS_OK;
  ix->devs.resize(devs.size());
  for (size_t i = 0; i < devs.size() && s == DVS_OK; ++i) {
    ix->devs[i].ordinal = devs[i];
    s = dvs::upload(ix->devs[i], ix->host, 0, 1);
    if (s == DVS_OK) s = dvs::grow_rows(ix->devs[i], p->capacity ? p->capacity : 1024);
  }
  if (s != DVS_OK) {
    for (auto& d : ix->devs) d.release();
    delete ix;
    return s;
  }
  *out = ix;
  return DVS_OK;
}

dvs_status dvs_close(dvs_index* ix) {
  if (!ix) return fail(DVS_ERR_ARG, "null index");
  for (auto& d : ix->devs) {
    d.release();
  }
  delete ix;
  return DVS_OK;
}

dvs_status dvs_index_artifacts(const dvs_index* ix, float* h_rotation, float* h_rotated_centroid) {
  if (!ix) return fail(DVS_ERR_ARG, "null index");
  const size_t d = ix->host.info.dim;
  if (h_rotation) std::memcpy(h_rotation, ix->host.rotation.data(), d * d * 4);
  if (h_rotated_centroid) std::memcpy(h_rotated_centroid, ix->host.rotated_centroid.data(), d * 4);
  return DVS_OK;
}

dvs_status dvs_index_get_info(const dvs_index* ix, dvs_index_info* out) {
  if (!ix || !out) return fail(DVS_ERR_ARG, "null argument");
  *out = ix->host.info;
  return DVS_OK;
}

dvs_status dvs_set_hop_limit(dvs_index* ix, uint32_t max_expansions) {
  if (!ix) return fail(DVS_ERR_ARG, "null index");
  ix->hop_limit = max_expansions;
  return DVS_OK;
}

dvs_status dvs_set_visited_slots(dvs_index* ix, uint32_t slots_per_beam_entry) {
  if (!ix) return fail(DVS_ERR_ARG, "null index");
  if (slots_per_beam_entry != 0 && (slots_per_beam_entry < 2 || slots_per_beam_entry > 256))
    return fail(DVS_ERR_ARG, "visited slots per beam entry must be in 2..256");
  std::lock_guard<std::mutex> g(ix->mu);
  ix->slots_per_entry = slots_per_beam_entry;
  return DVS_OK;
}

dvs_status dvs_set_rotation(dvs_index* ix, dvs_rotation rotation) {
  if (!ix) return fail(DVS_ERR_ARG, "null index");
  if (rotation != DVS_ROTATION_EXACT && rotation != DVS_ROTATION_TENSOR) return fail(DVS_ERR_ARG, "unknown rotation");
  std::lock_guard<std::mutex> g(ix->mu);
  if (rotation == DVS_ROTATION_TENSOR) {
    // P split into tf32 planes once per device, read by every tensor-core rotation
    for (auto& d : ix->devs) {
      if (d.tc.split) continue;
      DVS_CUDA(cudaSetDevice(d.ordinal));
      DVS_CUDA(cudaStreamSynchronize(d.sc.stream));
      DVS_CUDA(dvs::tc_rotation_prepare(d.P, d.lay.dim, &d.tc, d.sc.stream));
      DVS_CUDA(cudaStreamSynchronize(d.sc.stream));
    }
  }
  ix->rotation = rotation;
  return DVS_OK;
}

dvs_status dvs_set_kernel_timing(dvs_index* ix, int enable) {
  if (!ix) return fail(DVS_ERR_ARG, "null index");
  std::lock_guard<std::mutex> g(ix->mu);
  if (enable) {
    // the event ring is made here, not by the first timed search, so that
    // creating its events never stalls a timed loop
    for (auto& d : ix->devs) {
      if (!d.tev.empty()) continue;
      DVS_CUDA(cudaSetDevice(d.ordinal));
      d.tev.resize(3 * dvs::Device::kRing);
      for (auto& e : d.tev) DVS_CUDA(cudaEventCreate(&e));
    }
  }
  ix->kernel_timing = enable != 0;
  return DVS_OK;
}

dvs_status dvs_kernel_times(dvs_index* ix, uint32_t slot, uint32_t* searches, double* prepare_ms, double* search_ms) {
  if (!ix || !searches || !prepare_ms || !search_ms) return fail(DVS_ERR_ARG, "null argument");
  if (slot >= ix->devs.size()) return fail(DVS_ERR_ARG, "device slot out of range");
  std::lock_guard<std::mutex> g(ix->mu);
  dvs::Device& d = ix->devs[slot];
  DVS_CUDA(cudaSetDevice(d.ordinal));
  double pm = 0.0, sm = 0.0;
  for (size_t i = 0; i < d.tcount; ++i) {
    DVS_CUDA(cudaEventSynchronize(d.tev[3 * i + 2]));
    float a = 0.f, b = 0.f;
    DVS_CUDA(cudaEventElapsedTime(&a, d.tev[3 * i], d.tev[3 * i + 1]));
    DVS_CUDA(cudaEventElapsedTime(&b, d.tev[3 * i + 1], d.tev[3 * i + 2]));
    pm += a;
    sm += b;
  }
  *searches = uint32_t(d.tcount);
  *prepare_ms = pm;
  *search_ms = sm;
  d.tcount = 0;
  return DVS_OK;
}

dvs_status dvs_index_download(const dvs_index* ix, uint32_t* h_adj, uint8_t* h_records, float* h_vecs,
                              uint32_t* h_ids) {
  if (!ix || ix->devs.empty()) return fail(DVS_ERR_ARG, "null index");
  const dvs::DevLayout& L0 = ix->devs[0].lay;
  const uint32_t ns = L0.shard_log == 0 ? 1u : uint32_t(ix->devs.size());
  if (h_ids) {
    DVS_CUDA(cudaSetDevice(ix->devs[0].ordinal));
    DVS_CUDA(cudaMemcpy(h_ids, ix->devs[0].ids, size_t(L0.n) * 4, cudaMemcpyDeviceToHost));
  }
  for (uint32_t sh = 0; sh < ns; ++sh) {
    const dvs::Device& d = ix->devs[sh];
    const dvs::DevLayout& L = d.lay;
    const uint64_t nl = d.rows;
    DVS_CUDA(cudaSetDevice(d.ordinal));
    std::vector<uint32_t> a(size_t(nl) * L.R), r(size_t(nl) * L.rec_words);
    std::vector<float> v(size_t(nl) * L.vec_stride);
    DVS_CUDA(cudaMemcpy(a.data(), d.adj, a.size() * 4, cudaMemcpyDeviceToHost));
    DVS_CUDA(cudaMemcpy(r.data(), d.rec, r.size() * 4, cudaMemcpyDeviceToHost));
    DVS_CUDA(cudaMemcpy(v.data(), d.vecs, v.size() * 4, cudaMemcpyDeviceToHost));
    const uint32_t packed = (L.bits * L.dim + 7) / 8, rs = packed + 8;
    for (uint64_t l = 0; l < nl; ++l) {
      const uint64_t g = l * ns + sh;
      if (h_adj) std::memcpy(h_adj + g * L.R, &a[l * L.R], size_t(L.R) * 4);
      if (h_vecs) std::memcpy(h_vecs + g * L.dim, &v[l * L.vec_stride], size_t(L.dim) * 4);
      if (h_records) {
        const uint8_t* src = reinterpret_cast<const uint8_t*>(r.data() + l * L.rec_words);
        std::memcpy(h_records + g * rs, src, packed);
        std::memcpy(h_records + g * rs + packed, src + size_t(L.code_words) * 4, 8);
      }
    }
  }
  return DVS_OK;
}

dvs_status dvs_search_device(dvs_index* ix, uint32_t slot, const float* d_queries, uint32_t nq, uint32_t dim,
                             uint32_t k, uint32_t L, dvs_mode mode, uint32_t* d_out_ids, float* d_out_dist,
                             uint32_t* d_counters, void* stream) {
  dvs_status s = dvs::check_query_args(ix, nq, dim, k, L, mode);
  if (s != DVS_OK) return s;
  if (slot >= ix->devs.size()) return fail(DVS_ERR_ARG, "device slot out of range");
  if (nq == 0) return DVS_OK;
  if (!d_queries || !d_out_ids || !d_out_dist) return fail(DVS_ERR_ARG, "null buffer");
  std::lock_guard<std::mutex> g(ix->mu);
  dvs::Device& d = ix->devs[slot];
  DVS_CUDA(cudaSetDevice(d.ordinal));
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : d.sc.stream;
  return dvs::search_on(ix, d, d.sc, d_queries, nq, k, L, mode, d_out_ids, d_out_dist, d_counters, st, false);
}

dvs_status dvs_search(dvs_index* ix, const float* h_queries, uint32_t nq, uint32_t dim, uint32_t k, uint32_t L,
                      dvs_mode mode, uint32_t* h_out_ids, float* h_out_dist, dvs_stats* stats) {
  dvs_status s = dvs::check_query_args(ix, nq, dim, k, L, mode);
  if (s != DVS_OK) return s;
  if (stats) *stats = dvs_stats{};
  if (nq == 0) return DVS_OK;
  if (!h_queries || !h_out_ids || !h_out_dist) return fail(DVS_ERR_ARG, "null buffer");
  std::lock_guard<std::mutex> g(ix->mu);
  const size_t nd = ix->devs.size();
  std::vector<dvs_status> st(nd, DVS_OK);
  std::vector<std::string> msg(nd);
  std::vector<dvs_stats> part(nd);
  auto run = [&](size_t i) {
    dvs::Device& d = ix->devs[i];
    const size_t q0 = nq * i / nd, q1 = nq * (i + 1) / nd, m = q1 - q0;
    if (m == 0) return;
    auto body = [&]() -> dvs_status {
      dvs::Scratch& sc = d.sc;
      DVS_CUDA(cudaSetDevice(d.ordinal));
      dvs_status r = dvs::ensure_scratch(d, sc, m, k, true);
      if (r != DVS_OK) return r;
      DVS_CUDA(cudaMemcpyAsync(sc.queries, h_queries + q0 * dim, m * dim * 4, cudaMemcpyHostToDevice, sc.stream));
      r = dvs::search_on(ix, d, sc, sc.queries, uint32_t(m), k, L, mode, sc.out_ids, sc.out_dist, sc.counters, sc.stream, true);
      if (r != DVS_OK) return r;
      DVS_CUDA(cudaMemcpyAsync(h_out_ids + q0 * k, sc.out_ids, m * k * 4, cudaMemcpyDeviceToHost, sc.stream));
      DVS_CUDA(cudaMemcpyAsync(h_out_dist + q0 * k, sc.out_dist, m * k * 4, cudaMemcpyDeviceToHost, sc.stream));
      // per-query counters come back only when the caller asked for statistics
      std::vector<uint32_t> cnt(stats ? m * 4 : 0);
      uint32_t work[4] = {0, 0, 0, 0};
      if (stats) DVS_CUDA(cudaMemcpyAsync(cnt.data(), sc.counters, m * 16, cudaMemcpyDeviceToHost, sc.stream));
      DVS_CUDA(cudaMemcpyAsync(work, sc.work, 16, cudaMemcpyDeviceToHost, sc.stream));
      DVS_CUDA(cudaStreamSynchronize(sc.stream));
      if (stats) {
        float ms = 0.f;
        DVS_CUDA(cudaEventElapsedTime(&ms, sc.ev0, sc.ev1));
        dvs_stats& ps = part[i];
        for (size_t q = 0; q < m; ++q) {
          ps.expansions += cnt[q * 4 + 0];
          ps.estimates += cnt[q * 4 + 1];
          ps.reranked += cnt[q * 4 + 2];
        }
        ps.overflow_queries = work[2];
        ps.device_ms = ms;
      }
      if (work[1] & dvs::kErrNonFinite)
        return fail(DVS_ERR_ARG, "a query contains a non-finite value; its results are empty");
      if (work[1] & dvs::kErrCapacity)
        return fail(DVS_ERR_CAPACITY, "a query's visited set exceeded its capacity; its results are partial");
      if (work[1] & dvs::kErrHopLimit)
        return fail(DVS_ERR_HOP_LIMIT, "a query reached the expansion limit; its results are partial");
      if (work[1] & dvs::kErrTimeout)
        return fail(DVS_ERR_TIMEOUT, "the tensor-core rotation gave up waiting for its MMAs");
      return DVS_OK;
    };
    st[i] = body();
    if (st[i] != DVS_OK) msg[i] = dvs_last_error();
  };
  if (nd == 1) {
    run(0);
  } else {
    std::vector<std::thread> th;
    for (size_t i = 0; i < nd; ++i) th.emplace_back(run, i);
    for (auto& t : th) t.join();
  }
  for (size_t i = 0; i < nd; ++i) {
    if (stats) {
      stats->expansions += part[i].expansions;
      stats->estimates += part[i].estimates;
      stats->reranked += part[i].reranked;
      stats->overflow_queries += part[i].overflow_queries;
      stats->device_ms = std::max(stats->device_ms, part[i].device_ms);
    }
  }
  for (size_t i = 0; i < nd; ++i)
    if (st[i] != DVS_OK) return fail(st[i], msg[i]);
  return DVS_OK;
}

dvs_status dvs_query_prepare(const float* d_query, const float* d_P, const float* d_centroid, float* d_rot_query,
                             float* d_factor, uint32_t nq, uint32_t dim, uint32_t bits, void* stream) {
  if (!d_query || !d_P || !d_centroid || !d_rot_query || !d_factor) return fail(DVS_ERR_ARG, "null buffer");
  if (bits != 1 && bits != 2 && bits != 4 && bits != 8) return fail(DVS_ERR_BITS, "bits must be 1, 2, 4, or 8");
  if (dim == 0) return fail(DVS_ERR_DIM, "dim must be > 0");
  DVS_CUDA(dvs::launch_prepare(d_query, dim, d_P, d_centroid, d_rot_query, dim, d_factor, 3, dim, bits, nq,
                               static_cast<cudaStream_t>(stream)));
  return DVS_OK;
}

dvs_status dvs_query_prepare_tc(const float* d_query, const float* d_P, const float* d_centroid, float* d_rot_query,
                                float* d_factor, uint32_t nq, uint32_t dim, uint32_t bits, void* stream) {
  if (!d_query || !d_P || !d_centroid || !d_rot_query || !d_factor) return fail(DVS_ERR_ARG, "null buffer");
  if (bits != 1 && bits != 2 && bits != 4 && bits != 8) return fail(DVS_ERR_BITS, "bits must be 1, 2, 4, or 8");
  if (dim == 0) return fail(DVS_ERR_DIM, "dim must be > 0");
  if (nq == 0) return DVS_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint32_t* d_err = nullptr;
  DVS_CUDA(cudaMallocAsync(&d_err, 4, st));
  DVS_CUDA(cudaMemsetAsync(d_err, 0, 4, st));
  // P is split for this call alone (an open index keeps its split)
  struct Split {
    dvs::TcRotation t;
    ~Split() { dvs::tc_rotation_release(&t); }
  } sp;
  DVS_CUDA(dvs::tc_rotation_prepare(d_P, dim, &sp.t, st));
  DVS_CUDA(dvs::launch_prepare_tc(d_query, dim, sp.t, d_centroid, d_rot_query, dim, d_factor, 3, dim, bits, nq, d_err,
                                  st));
  uint32_t h_err = 0;
  DVS_CUDA(cudaMemcpyAsync(&h_err, d_err, 4, cudaMemcpyDeviceToHost, st));
  DVS_CUDA(cudaFreeAsync(d_err, st));
  DVS_CUDA(cudaStreamSynchronize(st));
  if (h_err & dvs::kErrTimeout) return fail(DVS_ERR_TIMEOUT, "the tensor-core rotation gave up waiting for its MMAs");
  return DVS_OK;
}

dvs_status dvs_rabitq_estimate(const float* d_rot_query, const float* d_factor, const uint8_t* d_records,
                               float* d_dist, uint32_t n, uint32_t dim, uint32_t bits, void* stream) {
  if (!d_rot_query || !d_factor || !d_records || !d_dist) return fail(DVS_ERR_ARG, "null buffer");
  if (bits != 1 && bits != 2 && bits != 4 && bits != 8)
    return fail(DVS_ERR_BITS, "bits must be 1, 2, 4, or 8; got " + std::to_string(bits));
  DVS_CUDA(dvs::launch_estimate_ref_layout(d_rot_query, d_factor, d_records, d_dist, n, dim, bits,
                                           static_cast<cudaStream_t>(stream)));
  return DVS_OK;
}

dvs_status dvs_l2_distances(const float* d_query, const float* d_candidates, float* d_dist, uint32_t n, uint32_t dim,
                            void* stream) {
  if (!d_query || !d_candidates || !d_dist) return fail(DVS_ERR_ARG, "null buffer");
  if (dim == 0) return fail(DVS_ERR_DIM, "dim must be > 0");
  DVS_CUDA(dvs::launch_l2_rows(d_query, d_candidates, d_dist, n, dim, static_cast<cudaStream_t>(stream)));
  return DVS_OK;
}

}  // extern "C"
