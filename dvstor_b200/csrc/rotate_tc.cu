// Query rotation Q' = Q P^T on the 5th-generation tensor cores (tcgen05), the one
// dense contraction of the query path (gpu_kernel_launcher.cu:289-297 does it
// per query with cublasSgemv).
//
// fp32 accuracy from tf32 MMAs by the 3xTF32 split: x = hi + lo with hi, lo tf32
// (round to nearest), and Q'P^T ~= Qhi Phi + Qhi Plo + Qlo Phi accumulated in fp32
// in tensor memory (the dropped Qlo Plo term is ~2^-22 relative).  One CTA of 4
// warps computes a 128-query x NT-column tile (NT <= 256, a multiple of 16):
// per 32-float K chunk the warps load Q and P rows with coalesced loads, split
// them and store them in the 128-byte-swizzled K-major layout the MMA reads;
// one elected thread issues 4 K-steps x 3 MMAs (M=128, N=NT, K=8) into a TMEM
// accumulator and commits them to an mbarrier; after the last chunk every warp
// reads its 32 TMEM lanes with tcgen05.ld and stores the rows.  Every mbarrier
// wait is bounded: on expiry the CTA records an error, frees its TMEM and exits.

#include <cuda_runtime.h>

#include <cstdint>

#include "device_math.cuh"
#include "search.cuh"

namespace dvs {
namespace {

constexpr uint32_t kTileM = 128;     // queries per CTA (MMA M)
constexpr uint32_t kChunk = 32;      // K floats per smem chunk (one 128-byte swizzle row)
constexpr uint32_t kWaitLimit = 1u << 20;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ float to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// Byte offset of element (row, k) of a K-major, 128-byte-swizzled tile whose
// rows are 32 floats: 8-row atoms of 1024 bytes, the 16-byte chunk index of a
// row XORed with the row's index inside its atom.
__device__ __forceinline__ uint32_t swz_offset(uint32_t row, uint32_t k) {
  return (row >> 3) * 1024u + (row & 7u) * 128u + ((((k >> 2) ^ (row & 7u)) & 7u) << 4) + ((k & 3u) << 2);
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

__global__ void __launch_bounds__(128, 1) rotate_tc_kernel(const float* __restrict__ Q, uint32_t q_stride,
                                                            const float* __restrict__ P, float* __restrict__ out,
                                                            uint32_t out_stride, uint32_t dim, uint32_t nq,
                                                            uint32_t nt, uint32_t* __restrict__ err) {
  extern __shared__ __align__(1024) unsigned char dsm[];
  // 1024-byte aligned tiles: A hi, A lo (128 rows), B hi, B lo (nt rows, padded to 8)
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(dsm) + 1023) & ~uintptr_t(1023));
  const uint32_t b_rows = (nt + 7) & ~7u;
  unsigned char* a_hi = base;
  unsigned char* a_lo = a_hi + kTileM * 128;
  unsigned char* b_hi = a_lo + kTileM * 128;
  unsigned char* b_lo = b_hi + b_rows * 128;
  __shared__ __align__(8) uint64_t mbar;
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
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&mbar)));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tmem_base;
  const uint32_t idesc = instr_desc_tf32(nt);
  const uint32_t nchunks = (dim + kChunk - 1) / kChunk;

  for (uint32_t c = 0; c < nchunks; ++c) {
    const uint32_t k = c * kChunk + lane;
    // A: query rows q0 .. q0+127, one warp row at a time (coalesced 128-byte loads)
    for (uint32_t r = warp; r < kTileM; r += 4) {
      const uint32_t q = q0 + r;
      const float x = (q < nq && k < dim) ? Q[size_t(q) * q_stride + k] : 0.f;
      const float hi = to_tf32(x);
      const float lo = to_tf32(x - hi);
      *reinterpret_cast<float*>(a_hi + swz_offset(r, lane)) = hi;
      *reinterpret_cast<float*>(a_lo + swz_offset(r, lane)) = lo;
    }
    // B: row j of B is column n0+j of P (contiguous in P's column-major storage)
    for (uint32_t r = warp; r < b_rows; r += 4) {
      const uint32_t j = n0 + r;
      const float x = (r < nt && j < dim && k < dim) ? P[size_t(j) * dim + k] : 0.f;
      const float hi = to_tf32(x);
      const float lo = to_tf32(x - hi);
      *reinterpret_cast<float*>(b_hi + swz_offset(r, lane)) = hi;
      *reinterpret_cast<float*>(b_lo + swz_offset(r, lane)) = lo;
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
    if (threadIdx.x == 0) {
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
      mma_commit(smem_u32(&mbar));
    }
    // the tiles are rewritten next chunk: wait until the MMAs have read them
    if (!mbar_wait(smem_u32(&mbar), c & 1)) {
      if (lane == 0) atomicOr(&failed, 1u);
    }
    __syncthreads();
    if (failed) break;
  }

  if (!failed) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t row = warp * 32 + lane;
    const uint32_t q = q0 + row;
    for (uint32_t c0 = 0; c0 < nt; c0 += 16) {
      uint32_t v[16];
      const uint32_t taddr = tmem + ((warp * 32) << 16) + c0;
      asm volatile(
          "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
          : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
            "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
          : "r"(taddr));
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
      if (q < nq) {
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const uint32_t j = n0 + c0 + e;
          if (c0 + e < nt && j < dim) out[size_t(q) * out_stride + j] = __uint_as_float(v[e]);
        }
      }
    }
  } else if (threadIdx.x == 0) {
    atomicOr(err, kErrTimeout);
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(ncols));
  }
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
  return 1024 + 2 * size_t(kTileM) * 128 + 2 * size_t((nt + 7) & ~7u) * 128;
}

cudaError_t launch_prepare_tc(const float* queries, uint32_t q_stride, const float* P, const float* c_rot, float* qrot,
                              uint32_t qrot_stride, float* qfac, uint32_t fac_stride, uint32_t dim, uint32_t bits,
                              uint32_t nq, uint32_t* err, cudaStream_t stream) {
  if (nq == 0) return cudaSuccess;
  const uint32_t nt = rotate_tc_tile_n(dim);
  const size_t smem = rotate_tc_smem(dim);
  cudaError_t e = cudaFuncSetAttribute(rotate_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return e;
  const dim3 grid((nq + kTileM - 1) / kTileM, (dim + nt - 1) / nt);
  rotate_tc_kernel<<<grid, 128, smem, stream>>>(queries, q_stride, P, qrot, qrot_stride, dim, nq, nt, err);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  return launch_query_factors(qrot, qrot_stride, c_rot, qfac, fac_stride, dim, bits, nq, stream);
}

}  // namespace dvs
