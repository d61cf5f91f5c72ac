// Query prepare: q' = P^T q and the RaBitQ query factors, for a whole batch.
//
// The reference does one query per call: cublasSgemv(CUBLAS_OP_T) on the
// column-major P, then rabitq_query_prepare_kernel<4,B> (<<<1,4>>>)
// (src/gpu/gpu_kernel_launcher.cu:280-320, src/gpu/kernels/distance_kernels.cuh:470-501).
// cuBLAS's summation order is not public, so the rotation here fixes one order:
// output j is the sequential chain acc = fmaf(P[j*D + i], q[i], acc) over
// i = 0..D-1 from acc = +0.  Every kernel below keeps that chain, so all of them
// give the same bits; the factors keep the reference kernel's 4-lane split
// (lane t sums j = t mod 4, then the butterfly).
//
//   dim <= 128  prepare_tile_kernel: P^T resident in shared memory, 64 queries
//               per tile, rotation and factors in one launch.
//   dim  > 128  rotate_tile_kernel + factors_kernel: a register-tiled product
//               (64 queries x 64 outputs per block, 4 x 4 per thread, the i axis
//               staged 32 at a time); 2*D^2 FLOP per query is compute work, so
//               this is an FP32-pipe kernel (D = 960: 1.84 MFLOP per query).

#include <cuda_runtime.h>

#include "device_math.cuh"
#include "search.cuh"

namespace dvs {
namespace {

constexpr uint32_t kPrepTileQ = 64;

// dim <= 128: each thread owns one output column for 8 queries, so every P^T
// element loaded feeds 8 FMAs; each output is the sequential chain over i.
__global__ void __launch_bounds__(256) prepare_tile_kernel(const float* __restrict__ Q, uint32_t q_stride,
                                                           const float* __restrict__ P, const float* __restrict__ c,
                                                           float* __restrict__ qrot, uint32_t qrot_stride,
                                                           float* __restrict__ qfac, uint32_t fac_stride,
                                                           uint32_t dim, uint32_t nq, float c_b) {
  extern __shared__ __align__(16) float sm[];
  float* PT = sm;                        // dim x dim, PT[i*dim + j] = P[j*dim + i]
  float* qT = PT + dim * dim;            // dim x 64, qT[i*64 + b]
  float* rs = qT + dim * kPrepTileQ;     // 64 x dim rotated queries
  for (uint32_t t = threadIdx.x; t < dim * dim; t += blockDim.x) {
    const uint32_t j = t / dim, i = t - j * dim;
    PT[i * dim + j] = P[t];
  }
  for (uint32_t q0 = blockIdx.x * kPrepTileQ; q0 < nq; q0 += gridDim.x * kPrepTileQ) {
    const uint32_t nb = min(kPrepTileQ, nq - q0);
    for (uint32_t t = threadIdx.x; t < dim * kPrepTileQ; t += blockDim.x) {
      const uint32_t b = t / dim, i = t - b * dim;
      qT[i * kPrepTileQ + b] = b < nb ? Q[size_t(q0 + b) * q_stride + i] : 0.f;
    }
    __syncthreads();
    const uint32_t tiles = dim * (kPrepTileQ / 8);
    for (uint32_t t = threadIdx.x; t < tiles; t += blockDim.x) {
      const uint32_t j = t % dim, bg = t / dim;
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (uint32_t i = 0; i < dim; ++i) {
        const float p = PT[i * dim + j];
        const float4 qa = *reinterpret_cast<const float4*>(qT + i * kPrepTileQ + 8 * bg);
        const float4 qb = *reinterpret_cast<const float4*>(qT + i * kPrepTileQ + 8 * bg + 4);
        acc[0] = __fmaf_rn(p, qa.x, acc[0]);
        acc[1] = __fmaf_rn(p, qa.y, acc[1]);
        acc[2] = __fmaf_rn(p, qa.z, acc[2]);
        acc[3] = __fmaf_rn(p, qa.w, acc[3]);
        acc[4] = __fmaf_rn(p, qb.x, acc[4]);
        acc[5] = __fmaf_rn(p, qb.y, acc[5]);
        acc[6] = __fmaf_rn(p, qb.z, acc[6]);
        acc[7] = __fmaf_rn(p, qb.w, acc[7]);
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) rs[(8 * bg + k) * dim + j] = acc[k];
    }
    __syncthreads();
    for (uint32_t t = threadIdx.x; t < nb * qrot_stride; t += blockDim.x) {
      const uint32_t b = t / qrot_stride, j = t - b * qrot_stride;
      qrot[size_t(q0 + b) * qrot_stride + j] = j < dim ? rs[b * dim + j] : 0.f;
    }
    // factors: one lane quad per query, the 4-lane butterfly of rabitq_query_prepare_kernel
    const uint32_t lane = threadIdx.x & 31, quad = threadIdx.x >> 2;
    for (uint32_t b0 = 0; b0 < kPrepTileQ; b0 += blockDim.x / 4) {
      const uint32_t b = b0 + quad;
      float sq = 0.f, sm2 = 0.f;
      if (b < nb) {
        for (uint32_t j = lane & 3; j < dim; j += 4) {
          const float v = rs[b * dim + j];
          const float diff = __fsub_rn(v, __ldg(c + j));
          sq = __fmaf_rn(diff, diff, sq);
          sm2 = __fadd_rn(sm2, v);
        }
      }
      sq = quad_butterfly(sq);
      sm2 = quad_butterfly(sm2);
      if (b < nb && (lane & 3) == 0) {
        float* f = qfac + size_t(q0 + b) * fac_stride;
        f[0] = sq;
        f[1] = __fmul_rn(-0.5f, sm2);
        f[2] = __fmul_rn(c_b, sm2);
        if (fac_stride > 3) f[3] = 0.f;
      }
    }
    __syncthreads();
  }
}

constexpr uint32_t kRotTile = 64;            // queries and outputs per block
constexpr uint32_t kRotK = 32;               // i values per staged chunk
constexpr uint32_t kRotLd = kRotTile + 4;    // staged row length (floats): float4-aligned, 4-way store conflicts

// 16 accumulators, one step of the i chain each.
__device__ __forceinline__ void rot_step(float (&acc)[4][4], const float* qs, const float* ps, uint32_t k,
                                         uint32_t tq, uint32_t tj) {
  const float4 a = *reinterpret_cast<const float4*>(qs + k * kRotLd + 4 * tq);
  const float4 b = *reinterpret_cast<const float4*>(ps + k * kRotLd + 4 * tj);
  const float av[4] = {a.x, a.y, a.z, a.w};
  const float bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int c = 0; c < 4; ++c) acc[r][c] = __fmaf_rn(bv[c], av[r], acc[r][c]);
}

// Block (x, y) computes rotated queries q0..q0+63, outputs j0..j0+63.  A warp
// stages one row of 32 consecutive i per load (128-byte coalesced) into
// i-major tiles; thread (tq, tj) = (tid / 16, tid % 16) owns queries 4tq..4tq+3
// x outputs 4tj..4tj+3.  The chain runs exactly over i < dim: the last, partial
// chunk stops at dim rather than adding zero terms (an all-underflow chain can
// end at -0, which +0 terms would turn into +0).
__global__ void __launch_bounds__(256) rotate_tile_kernel(const float* __restrict__ Q, uint32_t q_stride,
                                                          const float* __restrict__ P, float* __restrict__ qrot,
                                                          uint32_t qrot_stride, uint32_t dim, uint32_t nq) {
  __shared__ __align__(16) float qs[kRotK * kRotLd];  // qs[k*kRotLd + b] = Q[q0+b][i0+k]
  __shared__ __align__(16) float ps[kRotK * kRotLd];  // ps[k*kRotLd + c] = P[(j0+c)*dim + i0+k]
  const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t q0 = blockIdx.x * kRotTile, j0 = blockIdx.y * kRotTile;
  const uint32_t tq = tid >> 4, tj = tid & 15;
  float acc[4][4];
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int c = 0; c < 4; ++c) acc[r][c] = 0.f;

  for (uint32_t i0 = 0; i0 < dim; i0 += kRotK) {
    const uint32_t i = i0 + lane;
#pragma unroll
    for (uint32_t r = warp; r < kRotTile; r += 8) {
      const uint32_t q = q0 + r, j = j0 + r;
      qs[lane * kRotLd + r] = (q < nq && i < dim) ? __ldg(Q + size_t(q) * q_stride + i) : 0.f;
      ps[lane * kRotLd + r] = (j < dim && i < dim) ? __ldg(P + size_t(j) * dim + i) : 0.f;
    }
    __syncthreads();
    const uint32_t kn = min(kRotK, dim - i0);
    if (kn == kRotK) {
#pragma unroll 8
      for (uint32_t k = 0; k < kRotK; ++k) rot_step(acc, qs, ps, k, tq, tj);
    } else {
      for (uint32_t k = 0; k < kn; ++k) rot_step(acc, qs, ps, k, tq, tj);
    }
    __syncthreads();
  }
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const uint32_t q = q0 + 4 * tq + r;
    if (q >= nq) continue;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const uint32_t j = j0 + 4 * tj + c;
      if (j < dim) qrot[size_t(q) * qrot_stride + j] = acc[r][c];
    }
  }
}

// Factors of rabitq_query_prepare_kernel<4,B> from rotated rows (one lane quad
// per query), and zeros in the row padding [dim, qrot_stride).
__global__ void factors_kernel(float* __restrict__ qrot, uint32_t qrot_stride, const float* __restrict__ c,
                               float* __restrict__ qfac, uint32_t fac_stride, uint32_t dim, uint32_t nq, float c_b) {
  const uint32_t gq = (blockIdx.x * blockDim.x + threadIdx.x) >> 2;
  const uint32_t t = threadIdx.x & 3;
  float sq = 0.f, sm = 0.f;
  if (gq < nq) {
    float* r = qrot + size_t(gq) * qrot_stride;
    for (uint32_t j = t; j < dim; j += 4) {
      const float v = r[j];
      const float diff = __fsub_rn(v, __ldg(c + j));
      sq = __fmaf_rn(diff, diff, sq);
      sm = __fadd_rn(sm, v);
    }
    for (uint32_t j = dim + t; j < qrot_stride; j += 4) r[j] = 0.f;
  }
  sq = quad_butterfly(sq);
  sm = quad_butterfly(sm);
  if (gq < nq && t == 0) {
    float* f = qfac + size_t(gq) * fac_stride;
    f[0] = sq;
    f[1] = __fmul_rn(-0.5f, sm);
    f[2] = __fmul_rn(c_b, sm);
    if (fac_stride > 3) f[3] = 0.f;
  }
}

}  // namespace

cudaError_t launch_query_factors(float* qrot, uint32_t qrot_stride, const float* c_rot, float* qfac,
                                 uint32_t fac_stride, uint32_t dim, uint32_t bits, uint32_t nq, cudaStream_t stream) {
  if (nq == 0) return cudaSuccess;
  const float c_b = -static_cast<float>((1u << bits) - 1u) / 2.0f;
  const uint64_t threads = uint64_t(nq) * 4;
  factors_kernel<<<uint32_t((threads + 127) / 128), 128, 0, stream>>>(qrot, qrot_stride, c_rot, qfac, fac_stride, dim,
                                                                       nq, c_b);
  return cudaGetLastError();
}

cudaError_t launch_prepare(const float* queries, uint32_t q_stride, const float* P, const float* c_rot, float* qrot,
                           uint32_t qrot_stride, float* qfac, uint32_t fac_stride, uint32_t dim, uint32_t bits,
                           uint32_t nq, cudaStream_t stream) {
  if (nq == 0) return cudaSuccess;
  if (dim <= 128) {
    const float c_b = -static_cast<float>((1u << bits) - 1u) / 2.0f;
    const size_t smem = (size_t(dim) * dim + size_t(dim) * kPrepTileQ * 2) * sizeof(float);
    cudaError_t e = cudaFuncSetAttribute(prepare_tile_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return e;
    int dev = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const uint32_t tiles = (nq + kPrepTileQ - 1) / kPrepTileQ;
    const uint32_t grid = tiles < uint32_t(2 * sms) ? tiles : uint32_t(2 * sms);
    prepare_tile_kernel<<<grid, 256, smem, stream>>>(queries, q_stride, P, c_rot, qrot, qrot_stride, qfac, fac_stride,
                                                     dim, nq, c_b);
    return cudaGetLastError();
  }
  const dim3 grid((nq + kRotTile - 1) / kRotTile, (dim + kRotTile - 1) / kRotTile);
  rotate_tile_kernel<<<grid, 256, 0, stream>>>(queries, q_stride, P, qrot, qrot_stride, dim, nq);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  return launch_query_factors(qrot, qrot_stride, c_rot, qfac, fac_stride, dim, bits, nq, stream);
}

}  // namespace dvs
