// Host-side state of an open index, shared by the translation units that
// implement the C ABI (api.cu: open, search, kernel entry points; insert.cu:
// create and online insert).
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "internal.h"
#include "search.cuh"

struct dvs_index;

namespace dvs {

#define DVS_CUDA(call)                                                                             \
  do {                                                                                             \
    const cudaError_t e_ = (call);                                                                 \
    if (e_ != cudaSuccess) {                                                                       \
      return fail(e_ == cudaErrorMemoryAllocation ? DVS_ERR_OOM : DVS_ERR_CUDA,                    \
                  std::string(#call) + ": " + cudaGetErrorString(e_));                             \
    }                                                                                              \
  } while (0)

template <class T>
void dev_free(T*& p) {
  if (p) cudaFree(p);
  p = nullptr;
}

// Visited-set sizing.  Without an explicit size the shared-memory table gets
// between kSlotsMin and kSlotsMax slots per beam entry: the largest size that
// keeps the most warps resident (40 for the 96-dim L = 64 search, 20 warps per
// SM; 32 for L = 128).  Queries that outgrow it continue in a per-warp table in
// global memory, which costs little since those tables are reused under
// epochs instead of cleared (96-dim L = 128: 32 slots, every query spilling,
// 6.93 ms per 10,000 queries; 48 slots, 22 % spilling, 7.84 ms).
constexpr uint32_t kSlotsMin = 32;
constexpr uint32_t kSlotsMax = 48;
constexpr uint32_t kOverflowSlots = 1u << 14;

struct LaunchShape {
  uint32_t cap = 0, cap_pad = 0, hcap = 0, wpb = 0, blocks_per_sm = 0;
  uint32_t vt16 = 0, hbuckets = 0, hlimit = 0;
};

// Working memory and stream of the searches on one device.  Every device has
// two: one for searches, one for the online insert (its vectors, its exact
// search and its counters), so a search runs on the GPU while an insert step
// does.  Searches on one scratch are ordered on the GPU through `done`,
// whatever stream the caller gives them: they share its buffers.
struct Scratch {
  cudaStream_t stream = nullptr;
  cudaEvent_t ev0 = nullptr, ev1 = nullptr;
  cudaEvent_t done = nullptr;  // recorded after every search's work
  size_t q_cap = 0;            // queries the buffers hold
  size_t out_cap = 0;          // result slots the host-path buffers hold
  float* queries = nullptr;
  float* qrot = nullptr;
  float* qfac = nullptr;
  uint32_t* out_ids = nullptr;
  float* out_dist = nullptr;
  uint32_t* counters = nullptr;
  uint32_t* work = nullptr;
  uint32_t* ovf = nullptr;     // spill tables, then their epoch words
  size_t ovf_slots = 0;

  // stream, events and work words (the current device must be the scratch's)
  cudaError_t create() {
    cudaError_t e = cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreate(&ev0);
    if (e == cudaSuccess) e = cudaEventCreate(&ev1);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&done, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventRecord(done, stream);
    if (e == cudaSuccess) e = cudaMalloc(&work, 16);
    return e;
  }
  void release() {
    dev_free(queries);
    dev_free(qrot);
    dev_free(qfac);
    dev_free(out_ids);
    dev_free(out_dist);
    dev_free(counters);
    dev_free(work);
    dev_free(ovf);
    q_cap = out_cap = ovf_slots = 0;
    for (cudaEvent_t* e : {&ev0, &ev1, &done}) {
      if (*e) cudaEventDestroy(*e);
      *e = nullptr;
    }
    if (stream) cudaStreamDestroy(stream);
    stream = nullptr;
  }
};

struct Device {
  int ordinal = 0;
  uint32_t sm_count = 0;
  uint32_t shard = 0;     // shard held (sharded placement), rows = its row count
  uint64_t rows = 0;
  uint64_t cap_rows = 0;  // rows the index arrays have room for (online insert grows them)
  // index
  uint32_t* adj = nullptr;
  uint32_t* rec = nullptr;
  float* vecs = nullptr;
  uint32_t* ids = nullptr;
  float* P = nullptr;
  float* c_rot = nullptr;
  TcRotation tc;          // P split for the tensor-core rotation (made by dvs_set_rotation)
  DevLayout lay;
  Scratch sc;             // searches
  Scratch ins;            // online insert
  // online insert scratch, kept between calls so a step allocates nothing:
  // sort keys/values (in, out), run targets/counts/offsets, CUB temp storage,
  // step counters, phase events
  uint32_t* ins_buf = nullptr;
  size_t ins_buf_words = 0;
  void* ins_temp = nullptr;
  size_t ins_temp_bytes = 0;
  unsigned long long* ins_stats = nullptr;
  cudaEvent_t ins_ev[4] = {nullptr, nullptr, nullptr, nullptr};
  // launch shapes already worked out, by (capacity, slots per entry, mode, table kind)
  std::map<uint64_t, LaunchShape> shapes;
  // kernel timing ring of the searches: (before prepare, after prepare, after search)
  static constexpr size_t kRing = 4096;
  std::vector<cudaEvent_t> tev;
  size_t tcount = 0;

  void release() {
    if (ordinal < 0) return;
    cudaSetDevice(ordinal);
    if (sc.stream) cudaStreamSynchronize(sc.stream);
    if (ins.stream) cudaStreamSynchronize(ins.stream);
    dev_free(adj);
    dev_free(rec);
    dev_free(vecs);
    dev_free(ids);
    dev_free(P);
    dev_free(c_rot);
    tc_rotation_release(&tc);
    sc.release();
    ins.release();
    dev_free(ins_buf);
    dev_free(ins_temp);
    dev_free(ins_stats);
    ins_buf_words = ins_temp_bytes = 0;
    for (auto& e : ins_ev)
      if (e) cudaEventDestroy(e);
    for (auto& e : ins_ev) e = nullptr;
    for (cudaEvent_t e : tev) cudaEventDestroy(e);
    tev.clear();
  }
};

// Search-kernel launch shape for beam capacity `cap` on device `d` (exact: exact_gpu mode).
dvs_status launch_shape(Device& d, uint32_t cap, uint32_t slots_per_entry, bool exact, LaunchShape& s);
// Grows a scratch of device d to nq queries (and nq*k results for host calls).
dvs_status ensure_scratch(Device& d, Scratch& sc, size_t nq, size_t k, bool host_path);
// Prepare + search for nq device-resident queries on one device with scratch
// sc (asynchronous on st, after the scratch's previous search).
dvs_status search_on(dvs_index* ix, Device& d, Scratch& sc, const float* d_q, uint32_t nq, uint32_t k, uint32_t L,
                     dvs_mode mode, uint32_t* d_ids, float* d_dist, uint32_t* d_counters, cudaStream_t st,
                     bool timed, bool out_slots = false);

// search_on's work without the ordering against the scratch's other searches.
dvs_status search_enqueue(dvs_index* ix, Device& d, Scratch& sc, const float* d_q, uint32_t nq, uint32_t k,
                          uint32_t L, dvs_mode mode, uint32_t* d_ids, float* d_dist, uint32_t* d_counters,
                          cudaStream_t st, bool timed, bool out_slots);

// Grows the device arrays of a replicated index to hold `rows` nodes (online insert).
dvs_status grow_rows(Device& d, uint64_t rows);

}  // namespace dvs

struct dvs_index {
  dvs::HostIndex host;              // kept for downloads and metadata
  std::vector<dvs::Device> devs;
  // settings: written under mu, read by searches and by the insert thread
  std::atomic<uint32_t> hop_limit{0};
  std::atomic<uint32_t> slots_per_entry{0};  // 0 = sized for the most resident warps (kSlotsMin..kSlotsMax)
  std::atomic<bool> kernel_timing{false};
  std::atomic<dvs_rotation> rotation{DVS_ROTATION_EXACT};
  // mu guards the host state (device layouts, scratch, settings); an insert
  // holds it only to grow the arrays and to publish a step, and ins_mu for the
  // whole call, so searches proceed while an insert step runs on the GPU
  std::mutex mu;
  std::mutex ins_mu;
};
