/*
 * dvs_b200.h — C ABI of the B200-native DVSTOR `rabitq_gpu` query path.
 *
 * One shared library (dvstor_b200/lib/libdvs_b200.so) replaces the reference's
 * GPU launcher (src/gpu/gpu_kernel_launcher.hh) and the query loop of
 * Vamana<Distance>::knn (src/vamana/vamana.hh:57-452) that drives it.  The index
 * is read from the reference's offline formats (`<prefix>_nodeS_ofM.dat`,
 * `<prefix>.meta.json`, `<prefix>.rotation.bin`) into HBM once; a batch of
 * queries is then answered by one persistent CUDA kernel (one warp per query)
 * with no host round trip per expansion.
 *
 * Conventions: plain pointers and sizes only; every entry point returns a
 * dvs_status and never aborts (the reference's CUDA_CHECK/lib_assert abort the
 * process, src/gpu/gpu_kernel_launcher.cu:16-34); dvs_last_error() returns a
 * thread-local message for the last failure on the calling thread.  Pointers
 * named h_* are host memory, d_* device memory of the index's device.  `stream`
 * is a cudaStream_t passed as void* (NULL = the library's internal stream for
 * that device); calls that take a stream are asynchronous on it.
 */
#ifndef DVS_B200_H
#define DVS_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum dvs_status {
  DVS_OK = 0,
  DVS_ERR_ARG = 1,        /* invalid argument (null pointer, k > beam width, ...) */
  DVS_ERR_IO = 2,         /* missing / unreadable / unwritable file */
  DVS_ERR_FORMAT = 3,     /* malformed shard, meta or rotation file */
  DVS_ERR_DIM = 4,        /* dimension mismatch (query vs index, rotation vs meta) */
  DVS_ERR_BITS = 5,       /* unsupported RaBitQ bit width */
  DVS_ERR_CUDA = 6,       /* CUDA runtime error */
  DVS_ERR_PEER = 7,       /* peer access between devices unavailable */
  DVS_ERR_HOP_LIMIT = 8,  /* a query exceeded the configured expansion cap */
  DVS_ERR_TIMEOUT = 9,    /* a bounded device-side wait gave up */
  DVS_ERR_OOM = 10,       /* device or host allocation failed */
  DVS_ERR_CAPACITY = 11,  /* a per-query visited set or buffer limit was exceeded */
  DVS_ERR_UNSUPPORTED = 12,
  DVS_ERR_NO_DEVICE = 13  /* no CUDA device is visible */
} dvs_status;

/* search-mode (src/common/configuration.hh:128-130, validated at :170-174). */
typedef enum dvs_mode { DVS_MODE_RABITQ_GPU = 0, DVS_MODE_EXACT_GPU = 1 } dvs_mode;

/* distance named in <prefix>.meta.json ("l2" or "ip"); it selects the medoid seed
 * distance (src/vamana/vamana.hh:118).  Estimates and rerank are L2 in both
 * cases, as in the reference (src/gpu/gpu_kernel_launcher.cu:51-117). */
typedef enum dvs_metric { DVS_METRIC_L2 = 0, DVS_METRIC_IP = 1 } dvs_metric;

/* How an index spans devices.  REPLICATE: every device holds the whole index
 * and a query batch is split across devices.  SHARD: node i lives on device
 * (i mod ndev), the memory-node layout of assign_nodes_to_shards
 * (tools/vamana_offline_builder.cc:1116-1134); searches read peer HBM. */
typedef enum dvs_placement { DVS_PLACE_REPLICATE = 0, DVS_PLACE_SHARD = 1 } dvs_placement;

typedef struct dvs_index dvs_index;

typedef struct dvs_open_params {
  const char* index_prefix;   /* path prefix without _nodeX_ofN.dat (configuration.hh:83-86) */
  const int* devices;         /* CUDA device ordinals; NULL = {0} (`gpu-device`) */
  uint32_t num_devices;       /* 0 treated as 1 */
  dvs_placement placement;
  uint32_t expect_dim;        /* 0 = take from meta; else must match (compute_service.cc:548-554) */
  uint32_t expect_bits;       /* 0 = take from meta; else must match (compute_service.cc:555-561) */
  uint32_t expect_memory_nodes; /* 0 = take from meta; else must match (compute_service.cc:569-575) */
} dvs_open_params;

typedef struct dvs_index_info {
  uint64_t num_vectors;
  uint32_t dim;
  uint32_t R;                 /* max out-degree */
  uint32_t rabitq_bits;
  uint32_t rabitq_size;       /* (bits*dim+7)/8 + 8, VamanaNode::RABITQ_SIZE */
  uint32_t num_memory_nodes;  /* shard files */
  uint32_t medoid;            /* dense slot of the medoid */
  dvs_metric metric;
  double t_const;
} dvs_index_info;

/* Per-batch statistics, the device-side counterparts of statistics::ThreadStatistics'
 * visited_neighborlists / query_distcomps / query_exact_reranks
 * (src/common/statistics.hh:188-251). */
typedef struct dvs_stats {
  uint64_t expansions;        /* H summed over queries */
  uint64_t estimates;         /* E: RaBitQ estimates (rabitq_gpu) or exact distances (exact_gpu) */
  uint64_t reranked;          /* C_r: exact rerank rows */
  uint64_t overflow_queries;  /* queries whose visited set spilled from shared to global memory */
  float device_ms;            /* kernel time of the batch (prepare + search), CUDA events */
} dvs_stats;

/* ---- index lifetime ------------------------------------------------------ */

/* Opens an index: reads and validates the shard/meta/rotation files and uploads
 * a device layout to every listed device.  Replaces ComputeService's
 * load_index + maybe_load_rabitq_artifacts (src/service/compute_service.cc:520-593,
 * src/service/rabitq_artifacts.cc:22-73). */
dvs_status dvs_open(const dvs_open_params* params, dvs_index** out);
dvs_status dvs_close(dvs_index* index);
dvs_status dvs_index_get_info(const dvs_index* index, dvs_index_info* out);

/* Copies the device layout back to the host (dense slot order) — for checks.
 * Any output pointer may be NULL.  adj: n*R (0xFFFFFFFF = empty); records:
 * n*rabitq_size in the reference record layout; vecs: n*dim; ids: n node ids. */
dvs_status dvs_index_download(const dvs_index* index, uint32_t* h_adj, uint8_t* h_records, float* h_vecs,
                              uint32_t* h_ids);

/* The RaBitQ artifacts every vector of the index is quantized with: the
 * rotation P (dim*dim, column-major) and the rotated centroid (dim floats),
 * as loaded from <prefix>.rotation.bin or given to dvs_create.  Either output
 * may be NULL. */
dvs_status dvs_index_artifacts(const dvs_index* index, float* h_rotation, float* h_rotated_centroid);

/* ---- search -------------------------------------------------------------- */

/* Batched search through host buffers: ComputeService<Distance>::search
 * (src/service/compute_service.hh:91, src/service/compute_service.cc:227) for nq
 * queries at once.  h_queries: nq*dim floats.  Results per query: the first
 * min(k, |beam|) ids (node ids as stored in the shards) and their final
 * distances, sorted ascending; unused slots are 0xFFFFFFFF / +inf.
 * beam_width must be >= k (src/vamana/vamana.hh:49).  stats may be NULL.
 * With several devices the batch is split into contiguous chunks, one per
 * device, searched concurrently.  Blocks until the results are in host memory. */
dvs_status dvs_search(dvs_index* index, const float* h_queries, uint32_t nq, uint32_t dim, uint32_t k,
                      uint32_t beam_width, dvs_mode mode, uint32_t* h_out_ids, float* h_out_dist,
                      dvs_stats* stats);

/* Same search on device-resident buffers of device `device_slot` (index into
 * the open params' device list), asynchronous on `stream`.  d_counters (may be
 * NULL) receives nq*4 uint32 per query: expansions H, estimates E, reranked
 * rows C_r, and result count | error bits << 16 (1: visited set over capacity,
 * 2: expansion limit, 8: the query held a NaN or an infinity and was not
 * searched — its result slots are empty).  dvs_search reports the same
 * conditions as DVS_ERR_CAPACITY, DVS_ERR_HOP_LIMIT and DVS_ERR_ARG.  A NULL
 * stream means the index's internal stream.  Searches on one device run on
 * the GPU one after another, whichever streams they are given (they share the
 * index's scratch). */
dvs_status dvs_search_device(dvs_index* index, uint32_t device_slot, const float* d_queries, uint32_t nq,
                             uint32_t dim, uint32_t k, uint32_t beam_width, dvs_mode mode, uint32_t* d_out_ids,
                             float* d_out_dist, uint32_t* d_counters, void* stream);

/* dvs_search_device without any device allocation, for callers that may not
 * call cudaMalloc once running (a serving engine that has reserved the GPU's
 * free memory for its own pool, a request path where allocation is
 * forbidden).  No counterpart in the reference.  Same arguments and results
 * as dvs_search_device; the scratch (rotated queries, factors, work counters,
 * visited-set spill tables of the same size as dvs_search_device's) comes from
 * one fixed 64 MiB __device__ array per GPU instead of cudaMalloc.  That caps
 * a call at (8 MiB - 256) / (4*round_up(dim,4) + 16) queries (20,970 at dim 96;
 * more returns DVS_ERR_CAPACITY) and at 895 warps in flight, so a call runs
 * slower than dvs_search_device on a full GPU.  The first call on a device
 * looks the array up with cudaGetSymbolAddress; make it before any stream
 * capture.  A NULL stream means the index's internal stream.  Calls on one
 * index and device are ordered on the GPU after that index's other searches;
 * calls on different indexes whose work overlaps on the GPU race on the shared
 * array and must be serialised by the caller. */
dvs_status dvs_search_device_noalloc(dvs_index* index, uint32_t device_slot, const float* d_queries, uint32_t nq,
                                     uint32_t dim, uint32_t k, uint32_t beam_width, dvs_mode mode,
                                     uint32_t* d_out_ids, float* d_out_dist, uint32_t* d_counters, void* stream);

/* How the query rotation q' = P^T q is computed (src/gpu/gpu_kernel_launcher.cu
 * :289-297 uses cublasSgemv).  EXACT: fp32 FMA chains in a fixed order (the
 * default; results equal the CPU oracle's bit for bit).  TENSOR: tcgen05 MMAs
 * with the 3xTF32 split, fp32 accuracy (~1e-6 relative) at tensor-core speed;
 * the rotated query then differs from the fixed order in the last bits. */
typedef enum dvs_rotation { DVS_ROTATION_EXACT = 0, DVS_ROTATION_TENSOR = 1 } dvs_rotation;
dvs_status dvs_set_rotation(dvs_index* index, dvs_rotation rotation);

/* Expansion cap per query (0 = none, the reference's behaviour).  A query that
 * reaches it stops expanding, still reranks, and makes the search return
 * DVS_ERR_HOP_LIMIT. */
dvs_status dvs_set_hop_limit(dvs_index* index, uint32_t max_expansions);

/* Shared-memory visited-set size in slots per beam entry (indexes of fewer
 * than 2^24 nodes use 16-bit entries, larger ones 32-bit).  By default each
 * search shape takes the largest size in 40..48 that keeps the most warps
 * resident per SM.  A query whose visited set outgrows it continues in a
 * per-warp global-memory table with identical results; smaller values trade
 * shared memory (and therefore more resident queries per SM) for spills.
 * Valid range 2..256; 0 restores the default. */
dvs_status dvs_set_visited_slots(dvs_index* index, uint32_t slots_per_beam_entry);

/* Kernel timing: when enabled, every search on a device records CUDA events
 * around its prepare and search kernels on the stream they run on.
 * dvs_kernel_times waits for the recorded events of device slot `slot` and
 * returns the number of searches recorded since the last call with the summed
 * kernel durations in milliseconds (at most 4096 searches are kept). */
dvs_status dvs_set_kernel_timing(dvs_index* index, int enable);
dvs_status dvs_kernel_times(dvs_index* index, uint32_t slot, uint32_t* searches, double* prepare_ms,
                            double* search_ms);

/* ---- kernel-level entry points (device pointers, reference launcher layout) -- */

/* gpu::launch_rabitq_query_prepare (src/gpu/gpu_kernel_launcher.hh:139-146) for
 * nq queries: d_rot_query[q] = P^T d_query[q] (P column-major, dim*dim) and
 * d_factor[q] = {add, k1xSumq, kBxSumq} (RabitqQueryFactor, 12 bytes). */
dvs_status dvs_query_prepare(const float* d_query, const float* d_P, const float* d_centroid, float* d_rot_query,
                             float* d_factor, uint32_t nq, uint32_t dim, uint32_t bits, void* stream);

/* dvs_query_prepare with the rotation on tcgen05 tensor cores (3xTF32).
 * Returns DVS_ERR_TIMEOUT if a bounded wait inside the kernel expired. */
dvs_status dvs_query_prepare_tc(const float* d_query, const float* d_P, const float* d_centroid, float* d_rot_query,
                                float* d_factor, uint32_t nq, uint32_t dim, uint32_t bits, void* stream);

/* gpu::launch_batch_rabitq_distances (src/gpu/gpu_kernel_launcher.hh:53-59):
 * n records of rabitq_size bytes each, packed back to back as the reference
 * stages them ([codes | f32 add | f32 rescale]); one query.  bits 1, 2, 4
 * follow batch_rabitq_distance_kernel<4,B>; bits 8 follows
 * batch_rabitq_8bit_distance_kernel<4> (char4 steps; only the first
 * 4*floor(dim/4) dims count, as there). */
dvs_status dvs_rabitq_estimate(const float* d_rot_query, const float* d_factor, const uint8_t* d_records,
                               float* d_dist, uint32_t n, uint32_t dim, uint32_t bits, void* stream);

/* gpu::launch_batch_l2_distances (src/gpu/gpu_kernel_launcher.hh:34-37). */
dvs_status dvs_l2_distances(const float* d_query, const float* d_candidates, float* d_dist, uint32_t n,
                            uint32_t dim, void* stream);

/* ---- host-side format access (no GPU needed) ------------------------------ */

typedef struct dvs_host_index dvs_host_index;

/* Reads and validates the offline files into host memory (dense slot order:
 * slot g = k*M + s for the k-th node of shard s).  Same validation as dvs_open. */
dvs_status dvs_host_index_load(const char* index_prefix, dvs_host_index** out);
dvs_status dvs_host_index_info(const dvs_host_index* h, dvs_index_info* out);
/* Borrowed pointers, valid until dvs_host_index_free.  Any output may be NULL. */
dvs_status dvs_host_index_arrays(const dvs_host_index* h, const uint32_t** adj, const uint8_t** records,
                                 const float** vecs, const uint32_t** ids, const float** rotation,
                                 const float** rotated_centroid);
void dvs_host_index_free(dvs_host_index* h);

/* Writes an index in the reference's offline formats (write_vamana_shards,
 * tools/vamana_offline_builder.cc:1136-1267): node i goes to shard i mod M at
 * offset 16 + (i div M)*align8(node_size), stored id = h_ids[i] (i when h_ids
 * is NULL).  adj: n*R slot indices (0xFFFFFFFF = empty, non-empty entries
 * first); records: n*rabitq_size. */
typedef struct dvs_write_params {
  const char* index_prefix;
  uint64_t num_vectors;
  uint32_t dim;
  uint32_t R;
  uint32_t rabitq_bits;
  uint32_t num_memory_nodes;
  uint32_t medoid;
  uint32_t beam_width;        /* recorded in meta.json only */
  double alpha;               /* recorded in meta.json only */
  dvs_metric metric;
  double t_const;
} dvs_write_params;

dvs_status dvs_write_index(const dvs_write_params* p, const float* h_vecs, const uint32_t* h_adj,
                           const uint8_t* h_records, const float* h_rotation, const float* h_rotated_centroid,
                           const uint32_t* h_ids);

/* ---- online insert (Vamana::insert, src/vamana/vamana.hh:458-999) ----------- */

/* An empty, replicated index on the given devices, for a service that starts
 * without an offline build: inserts then grow it, the first one becoming the
 * medoid (vamana.hh:479-546).  The rotation P (dim*dim, column-major), the
 * rotated centroid and t_const are the artifacts every vector is quantized
 * with (rabitq_artifacts.cc:22-73). */
typedef struct dvs_create_params {
  uint32_t dim;
  uint32_t R;                      /* max out-degree, <= 64 */
  uint32_t rabitq_bits;            /* 1, 2, 4 or 8 */
  dvs_metric metric;               /* the medoid seed distance (distance.hh:80-159) */
  const float* rotation;
  const float* rotated_centroid;
  double t_const;
  const int* devices;              /* NULL = {0, 1, ..., num_devices-1} */
  uint32_t num_devices;            /* 0 = 1 */
  uint64_t capacity;               /* rows reserved up front, 0 = 1024 */
} dvs_create_params;

dvs_status dvs_create(const dvs_create_params* params, dvs_index** out);

/* Reserves device rows for `capacity` nodes (inserts grow the arrays by
 * doubling when they run out). */
dvs_status dvs_reserve(dvs_index* index, uint64_t capacity);

typedef struct dvs_insert_params {
  uint32_t beam_width_construction;  /* L_c, 0 = 200 (--beam-width-construction, configuration.hh:120) */
  float alpha;                       /* RobustPrune alpha, 0 = 1.2 (--alpha, configuration.hh:126) */
  uint32_t max_batch;                /* vectors per step, 0 = 1024 */
} dvs_insert_params;

typedef struct dvs_insert_stats {
  uint64_t inserted;
  uint64_t steps;        /* frozen-graph steps the batch was split into */
  uint64_t expansions;   /* beam expansions of the insert searches */
  uint64_t distances;    /* exact distances of the insert searches */
  uint64_t full_prunes;  /* reverse edges that met a full list and re-pruned it */
  float device_ms;       /* insert-search kernel time */
  float prune_ms;        /* new-node RobustPrune kernel time */
  float reverse_ms;      /* reverse-edge grouping and kernel time */
  uint32_t max_incoming; /* most new nodes linking to one old node in a step */
} dvs_insert_stats;

/* ComputeService::insert (src/service/compute_service.cc:152-196) into a
 * replicated index (DVS_ERR_UNSUPPORTED when sharded): node ids h_ids[i]
 * (NULL: the current node count + i).  The vectors are inserted in steps of
 * min(max_batch, current node count) vectors; every vector of a step searches
 * the graph as it stood when the step began (exact distances, beam capacity
 * L_c), its final beam is pruned with RobustPrune (robust_prune_kernel), the
 * vector is quantized by the GPU quantizer (rabitq_quantize_single_kernel),
 * and reverse edges are added in insert order (append, or RobustPrune of a
 * full list).  Steps of one vector reproduce the reference's sequential
 * insert.  Inserts run one at a time, on their own stream and scratch; other
 * threads' searches run meanwhile (they see the graph as the insert kernels
 * leave it, every step's node count once the step is done, as concurrent
 * readers of the reference's graph do).  When the arrays must grow, work in
 * flight on the devices finishes first (dvs_reserve grows them ahead of
 * time). */
dvs_status dvs_insert(dvs_index* index, const float* h_vectors, const uint32_t* h_ids, uint32_t n, uint32_t dim,
                      const dvs_insert_params* params, dvs_insert_stats* stats);

/* ---- offline builder (GPU) ---------------------------------------------- */

/* Builds an index from n vectors on one device and, when output_prefix is set,
 * writes it in the offline formats: the work of tools/vamana_offline_builder.cc
 * (compute_medoid :473-507, random R-regular init :700-718, build_vamana_graph
 * :673-861 with construction alpha 1.0, init_rabitq :978-1024,
 * rabitq_quantize_vector :1030-1102, write_vamana_shards :1136-1267) with the
 * graph pass in deterministic batches of the shuffled insertion order (1, 2,
 * 4, ... up to batch_cap nodes; each batch searches the graph as it stood when
 * the batch began).  out_adj (n*R) / out_records (n*rabitq_size) may be NULL. */
typedef struct dvs_build_params {
  const char* output_prefix;  /* NULL: do not write files */
  uint32_t R;                 /* max out-degree, <= 64 */
  uint32_t beam_width;        /* construction beam width L */
  double alpha;               /* recorded in meta.json (construction uses 1.0) */
  uint32_t rabitq_bits;
  int32_t seed;               /* --seed, default 1234 in the reference */
  uint32_t num_memory_nodes;  /* shard files to write */
  dvs_metric metric;          /* written to meta.json; the graph uses L2 distances,
                                 which rank unit-norm vectors as inner product does */
  int device;
  uint32_t batch_cap;         /* 0 = 2% of n (at most 65536) */
  uint32_t visited_cap;       /* per-node visited-set capacity, 0 = 16384 */
  uint32_t* out_adj;
  uint8_t* out_records;
} dvs_build_params;

typedef struct dvs_build_stats {
  uint32_t medoid;
  uint64_t batches;
  float graph_ms;             /* graph pass wall time on the device */
  double mean_visited;        /* mean |V| + |N(u)| per inserted node */
  double mean_degree;
} dvs_build_stats;

dvs_status dvs_build_index(const dvs_build_params* params, const float* h_vectors, uint64_t n, uint32_t dim,
                           dvs_build_stats* stats);

/* ---- misc ----------------------------------------------------------------- */

const char* dvs_last_error(void);
const char* dvs_status_string(dvs_status s);
/* Number of CUDA devices visible (0 on a host without a GPU). */
int dvs_device_count(void);

#ifdef __cplusplus
}
#endif

#endif /* DVS_B200_H */
