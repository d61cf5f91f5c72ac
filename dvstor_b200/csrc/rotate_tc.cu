// Query rotation Q' = Q P^T on the 5th-generation tensor cores (tcgen05), the one
// dense contraction of the query path (gpu_kernel_launcher.cu:289-297 does it
// per query with cublasSgemv).
//
// fp32 accuracy from tf32 MMAs by the 3xTF32 split: x = hi + lo with hi, lo tf32
// (round to nearest), and Q'P^T ~= Qhi Phi + Qhi Plo + Qlo Phi accumulated in fp32
// in tensor memory (the dropped Qlo Plo term is ~2^-22 relative).
//
// P is split once per index and device (tc_rotation_prepare): hi and lo planes,
// K padded with zeros to a multiple of 32, read by TMA.  One CTA computes a
// 128-query x NT-column tile (NT <= 256, a multiple of 16) in 32-float K chunks
// through a two-stage ring of shared-memory tiles in the 128-byte-swizzled
// K-major layout the MMA reads:
//   * thread 0 starts the TMA copy of the chunk's P hi/lo tiles (this GPU's
//     memory, no multicast) on the stage's mbarrier;
//   * every thread splits the query values it loaded during the previous
//     chunk's MMAs and stores them into the stage, then loads the next chunk's;
//   * thread 0 waits for the TMA bytes, issues 4 K-steps x 3 MMAs (M=128,
//     N=NT, K=8) into the TMEM accumulator and commits them to the stage's
//     MMA mbarrier, which frees the stage two chunks later.
// Eight warps share the splitting (16 query rows each).  After the last chunk
// the two warps of each 32-lane TMEM row group read alternate 16-column blocks
// with tcgen05.ld and store them.  Every mbarrier wait is bounded: on expiry the CTA records
// an error, waits (bounded) for its copies and MMAs in flight, frees its TMEM
// and exits.

#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdint>
#include <mutex>

#include "device_math.cuh"
#include "search.cuh"

namespace dvs {
namespace {

constexpr uint32_t kTileM = 128;     // queries per CTA (MMA M)
constexpr uint32_t kChunk = 32;      // K floats per smem chunk (one 128-byte swizzle row)
constexpr uint32_t kStages = 2;
constexpr uint32_t kWarps = 8;       // two warpgroups: each row group of 32 TMEM lanes has two warps
constexpr uint32_t kRowsPerWarp = kTileM / kWarps;
constexpr uint32_t kWaitLimit = 1u << 20;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ float to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// Byte offset of the 16-byte group (row, k4) of a K-major, 128-byte-swizzled
// tile whose rows are 32 floats: 8-row atoms of 1024 bytes, the 16-byte group
// index of a row XORed with the row's index inside its atom (the layout TMA's
// 128-byte swizzle writes).
__device__ __forceinline__ uint32_t swz_offset16(uint32_t row, uint32_t k4) {
  return (row >> 3) * 1024u + (row & 7u) * 128u + (((k4 ^ (row & 7u)) & 7u) << 4);
}

// Shared-memory matrix descriptor (tcgen05): start address, leading byte offset
// (unused by swizzled K-major tiles, 16), stride byte offset (1024: next 8-row
// atom), descriptor version 1, 128-byte swizzle.
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= uint64_t((saddr & 0x3FFFFu) >> 4);
  d |= uint64_t(16u >> 4) << 16;
  d |= uint64_t(1024u >> 4) << 32;
  d |= uint64_t(1u) << 46;
  d |= uint64_t(2u) << 61;
  return d;
}

// Instruction descriptor: D f32, A and B tf32, both K-major, N, M = 128.
__host__ __device__ constexpr uint32_t instr_desc_tf32(uint32_t n) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((n >> 3) << 17) | ((kTileM >> 4) << 24);
}

__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(acc));
}

__device__ __forceinline__ void mma_commit(uint32_t mbar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(mbar) : "memory");
}

__device__ __forceinline__ bool mbar_wait(uint32_t mbar, uint32_t parity) {
  for (uint32_t it = 0; it < kWaitLimit; ++it) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.b32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(mbar), "r"(parity)
        : "memory");
    if (ok) return true;
  }
  return false;
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t mbar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(mbar), "r"(bytes) : "memory");
}

// 2-D tiled TMA load of box {32 floats, rows} at (x, y) into shared memory,
// completing on `mbar`.  x is a multiple of 32 floats (128 bytes).
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t x, uint32_t y,
                                            uint32_t mbar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(mbar)
      : "memory");
}

__global__ void __launch_bounds__(kWarps * 32, 1)
    rotate_tc_kernel(const __grid_constant__ CUtensorMap map_hi, const __grid_constant__ CUtensorMap map_lo,
                     const float* __restrict__ Q, uint32_t q_stride, uint32_t q_vec4, float* __restrict__ out,
                     uint32_t out_stride, uint32_t out_vec4, uint32_t dim, uint32_t kp, uint32_t nq, uint32_t nt,
                     uint32_t* __restrict__ err) {
  extern __shared__ __align__(1024) unsigned char dsm[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(dsm) + 1023) & ~uintptr_t(1023));
  const uint32_t stage_bytes = 2 * kTileM * 128 + 2 * nt * 128;
  __shared__ __align__(8) uint64_t tma_bar[kStages], mma_bar[kStages];
  __shared__ uint32_t tmem_base;
  __shared__ uint32_t failed;

  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t q0 = blockIdx.x * kTileM, n0 = blockIdx.y * nt;
  uint32_t ncols = 32;
  while (ncols < nt) ncols <<= 1;

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base)),
                 "r"(ncols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
  }
  if (threadIdx.x == 0) {
    failed = 0;
    for (uint32_t s = 0; s < kStages; ++s) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&tma_bar[s])));
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&mma_bar[s])));
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tmem_base;
  const uint32_t idesc = instr_desc_tf32(nt);
  const uint32_t nchunks = kp / kChunk;

  // this thread's query values of one chunk: rows warp*16 + 4i + lane/8, floats 4*(lane%8) .. +3
  const uint32_t k4 = lane & 7;
  constexpr int kRowIters = kRowsPerWarp / 4;
  float4 ra[kRowIters];
  auto load_a = [&](uint32_t c) {
    const uint32_t k = c * kChunk + 4 * k4;
#pragma unroll
    for (int i = 0; i < kRowIters; ++i) {
      const uint32_t q = q0 + warp * kRowsPerWarp + 4 * i + (lane >> 3);
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (q < nq) {
        const float* row = Q + size_t(q) * q_stride;
        if (q_vec4 && k + 3 < dim) {
          v = __ldg(reinterpret_cast<const float4*>(row + k));
        } else {
          if (k < dim) v.x = __ldg(row + k);
          if (k + 1 < dim) v.y = __ldg(row + k + 1);
          if (k + 2 < dim) v.z = __ldg(row + k + 2);
          if (k + 3 < dim) v.w = __ldg(row + k + 3);
        }
      }
      ra[i] = v;
    }
  };

  // thread 0's book-keeping of what it started, for a clean exit after a timeout
  uint32_t tma_started[kStages] = {0, 0}, tma_done[kStages] = {0, 0}, commits[kStages] = {0, 0};
  load_a(0);
  for (uint32_t c = 0; c < nchunks; ++c) {
    const uint32_t s = c & 1, use = c >> 1;
    unsigned char* a_hi = base + s * stage_bytes;
    unsigned char* a_lo = a_hi + kTileM * 128;
    unsigned char* b_hi = a_lo + kTileM * 128;
    unsigned char* b_lo = b_hi + nt * 128;
    // the stage was last read by chunk c - 2's MMAs
    if (c >= kStages && !mbar_wait(smem_u32(&mma_bar[s]), (use - 1) & 1)) atomicOr(&failed, 1u);
    __syncthreads();
    if (failed) break;
    if (threadIdx.x == 0) {
      mbar_expect_tx(smem_u32(&tma_bar[s]), 2 * nt * 128);
      tma_load_2d(smem_u32(b_hi), &map_hi, c * kChunk, n0, smem_u32(&tma_bar[s]));
      tma_load_2d(smem_u32(b_lo), &map_lo, c * kChunk, n0, smem_u32(&tma_bar[s]));
      ++tma_started[s];
    }
#pragma unroll
    for (int i = 0; i < kRowIters; ++i) {
      const uint32_t row = warp * kRowsPerWarp + 4 * i + (lane >> 3);
      const float4 x = ra[i];
      float4 hi, lo;
      hi.x = to_tf32(x.x);
      hi.y = to_tf32(x.y);
      hi.z = to_tf32(x.z);
      hi.w = to_tf32(x.w);
      lo.x = to_tf32(x.x - hi.x);
      lo.y = to_tf32(x.y - hi.y);
      lo.z = to_tf32(x.z - hi.z);
      lo.w = to_tf32(x.w - hi.w);
      const uint32_t off = swz_offset16(row, k4);
      *reinterpret_cast<float4*>(a_hi + off) = hi;
      *reinterpret_cast<float4*>(a_lo + off) = lo;
    }
    if (c + 1 < nchunks) load_a(c + 1);  // in flight during this chunk's MMAs
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
    if (threadIdx.x == 0) {
      if (mbar_wait(smem_u32(&tma_bar[s]), use & 1)) {
        ++tma_done[s];
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
        for (uint32_t ks = 0; ks < kChunk / 8; ++ks) {
          const uint32_t off = ks * 32;  // 8 tf32 = 32 bytes along the swizzled row
          const uint64_t ah = smem_desc(smem_u32(a_hi) + off), al = smem_desc(smem_u32(a_lo) + off);
          const uint64_t bh = smem_desc(smem_u32(b_hi) + off), bl = smem_desc(smem_u32(b_lo) + off);
          mma_tf32(tmem, al, bh, idesc, (c | ks) != 0);
          mma_tf32(tmem, ah, bl, idesc, 1);
          mma_tf32(tmem, ah, bh, idesc, 1);
        }
        mma_commit(smem_u32(&mma_bar[s]));
        ++commits[s];
      } else {
        atomicOr(&failed, 1u);
      }
    }
  }
  __syncthreads();
  // the last chunk's commit covers every MMA issued before it
  if (!failed && !mbar_wait(smem_u32(&mma_bar[(nchunks - 1) & 1]), ((nchunks - 1) >> 1) & 1)) atomicOr(&failed, 1u);
  __syncthreads();

  if (!failed) {
    // warp w reads TMEM lanes 32 (w mod 4) .. +31 (its rows); the two warps of
    // a row group take alternate 16-column blocks
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t group = warp & 3, half = warp >> 2;
    const uint32_t row = group * 32 + lane;
    const uint32_t q = q0 + row;
    for (uint32_t c0 = 16 * half; c0 < nt; c0 += 32) {
      uint32_t v[16];
      const uint32_t taddr = tmem + ((group * 32) << 16) + c0;
      asm volatile(
          "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
          : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
            "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
          : "r"(taddr));
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
      if (q < nq) {
        const uint32_t j0 = n0 + c0;
        float* o = out + size_t(q) * out_stride + j0;
        if (out_vec4 && j0 + 16 <= dim) {
#pragma unroll
          for (int e = 0; e < 16; e += 4)
            *reinterpret_cast<float4*>(o + e) = make_float4(__uint_as_float(v[e]), __uint_as_float(v[e + 1]),
                                                            __uint_as_float(v[e + 2]), __uint_as_float(v[e + 3]));
        } else {
#pragma unroll
          for (int e = 0; e < 16; ++e)
            if (c0 + e < nt && j0 + e < dim) o[e] = __uint_as_float(v[e]);
        }
      }
    }
  } else if (threadIdx.x == 0) {
    atomicOr(err, kErrTimeout);
    // copies and MMAs still in flight finish (bounded) before their memory goes
    for (uint32_t s = 0; s < kStages; ++s) {
      for (uint32_t u = tma_done[s]; u < tma_started[s]; ++u) mbar_wait(smem_u32(&tma_bar[s]), u & 1);
      if (commits[s]) mbar_wait(smem_u32(&mma_bar[s]), (commits[s] - 1) & 1);
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(ncols));
  }
}

// P (column-major dim x dim: row j of B = P[j*dim .. j*dim + dim)) into tf32
// hi and lo planes of dim rows x kp floats, K zero-padded.
__global__ void split_p_kernel(const float* __restrict__ P, uint32_t dim, uint32_t kp, float* __restrict__ hi,
                               float* __restrict__ lo) {
  const size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= size_t(dim) * kp) return;
  const uint32_t j = uint32_t(i / kp), k = uint32_t(i % kp);
  const float x = k < dim ? P[size_t(j) * dim + k] : 0.f;
  const float h = to_tf32(x);
  hi[i] = h;
  lo[i] = to_tf32(x - h);
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    else
      cudaGetLastError();
  });
  return fn;
}

}  // namespace

uint32_t rotate_tc_tile_n(uint32_t dim) {
  // N tile: a multiple of 16 up to 256, as few tiles as possible
  const uint32_t tiles = (dim + 255) / 256;
  const uint32_t per = (dim + tiles - 1) / tiles;
  return (per + 15) / 16 * 16;
}

size_t rotate_tc_smem(uint32_t dim) {
  const uint32_t nt = rotate_tc_tile_n(dim);
  return 1024 + kStages * (2 * size_t(kTileM) * 128 + 2 * size_t(nt) * 128);
}

cudaError_t tc_rotation_prepare(const float* P, uint32_t dim, TcRotation* t, cudaStream_t stream) {
  tc_rotation_release(t);
  const uint32_t kp = (dim + kChunk - 1) / kChunk * kChunk;
  const uint32_t nt = rotate_tc_tile_n(dim);
  cudaError_t e = cudaMalloc(&t->split, 2 * size_t(dim) * kp * 4);
  if (e != cudaSuccess) return e;
  t->kp = kp;
  float* hi = t->split;
  float* lo = t->split + size_t(dim) * kp;
  const size_t n = size_t(dim) * kp;
  split_p_kernel<<<uint32_t((n + 255) / 256), 256, 0, stream>>>(P, dim, kp, hi, lo);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  auto enc = encode_fn();
  if (!enc) return cudaErrorNotSupported;
  const cuuint64_t gdim[2] = {kp, dim};
  const cuuint64_t gstride[1] = {cuuint64_t(kp) * 4};
  const cuuint32_t box[2] = {kChunk, nt};
  const cuuint32_t estride[2] = {1, 1};
  for (int h = 0; h < 2; ++h) {
    const CUresult r = enc(h == 0 ? &t->map_hi : &t->map_lo, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, h == 0 ? hi : lo,
                           gdim, gstride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  }
  t->dim = dim;
  return cudaSuccess;
}

void tc_rotation_release(TcRotation* t) {
  if (t->split) cudaFree(t->split);
  t->split = nullptr;
  t->dim = t->kp = 0;
}

cudaError_t launch_prepare_tc(const float* queries, uint32_t q_stride, const TcRotation& t, const float* c_rot,
                              float* qrot, uint32_t qrot_stride, float* qfac, uint32_t fac_stride, uint32_t dim,
                              uint32_t bits, uint32_t nq, uint32_t* err, cudaStream_t stream) {
  if (nq == 0) return cudaSuccess;
  if (!t.split || t.dim != dim) return cudaErrorInvalidValue;
  const uint32_t nt = rotate_tc_tile_n(dim);
  const size_t smem = rotate_tc_smem(dim);
  cudaError_t e = cudaFuncSetAttribute(rotate_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return e;
  const uint32_t q_vec4 = (q_stride % 4 == 0 && reinterpret_cast<uintptr_t>(queries) % 16 == 0) ? 1u : 0u;
  const uint32_t o_vec4 = (qrot_stride % 4 == 0 && reinterpret_cast<uintptr_t>(qrot) % 16 == 0) ? 1u : 0u;
  const dim3 grid((nq + kTileM - 1) / kTileM, (dim + nt - 1) / nt);
  rotate_tc_kernel<<<grid, kWarps * 32, smem, stream>>>(t.map_hi, t.map_lo, queries, q_stride, q_vec4, qrot, qrot_stride,
                                                o_vec4, dim, t.kp, nq, nt, err);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  return launch_query_factors(qrot, qrot_stride, c_rot, qfac, fac_stride, dim, bits, nq, stream);
}

}  // namespace dvs
