// Device arithmetic shared by the kernels.  Every routine fixes the order of its
// floating-point operations (explicit __f*_rn intrinsics, so nvcc cannot
// re-contract them) to the order the reference's kernels use, which the CPU
// oracle restates; results are therefore identical bit for bit.
#pragma once

#include <cfloat>
#include <cstdint>

namespace dvs {

constexpr uint32_t kEmptySlot = 0xFFFFFFFFu;
constexpr uint32_t kExpandedBit = 0x80000000u;

__device__ __forceinline__ float tile4_sum(float s0, float s1, float s2, float s3) {
  // cg::reduce over a 4-lane tile: xor 2, then xor 1.
  return __fadd_rn(__fadd_rn(s0, s2), __fadd_rn(s1, s3));
}

// Reduce the 4 lanes of an aligned lane quad with the same butterfly; every lane
// of the quad receives the tile sum.
__device__ __forceinline__ float quad_butterfly(float v) {
  v = __fadd_rn(v, __shfl_xor_sync(0xFFFFFFFFu, v, 2));
  v = __fadd_rn(v, __shfl_xor_sync(0xFFFFFFFFu, v, 1));
  return v;
}

// Small non-negative integer (< 2^23) to float, exact, without the conversion unit.
__device__ __forceinline__ float small_u2f(uint32_t x) {
  return __fsub_rn(__uint_as_float(0x4B000000u | x), 8388608.0f);
}

// One lane's share of batch_l2_squared_distance_kernel<4>
// (src/gpu/kernels/distance_kernels.cuh:38-81): lane t of the quad walks float4
// chunks t, t+4, ... then tail dim n4*4+t.  `q` and `x` are 16-byte aligned;
// `x` is global memory (read through the read-only data path).
__device__ __forceinline__ float l2_quad_partial(const float* __restrict__ q, const float* __restrict__ x,
                                                 uint32_t dim, uint32_t t) {
  const uint32_t n4 = dim >> 2;
  const float4* q4 = reinterpret_cast<const float4*>(q);
  const float4* x4 = reinterpret_cast<const float4*>(x);
  float acc = 0.f;
  uint32_t i = t;
#define DVS_ACC4(B, A)                                   \
  {                                                      \
    float d;                                             \
    d = __fsub_rn(B.x, A.x); acc = __fmaf_rn(d, d, acc); \
    d = __fsub_rn(B.y, A.y); acc = __fmaf_rn(d, d, acc); \
    d = __fsub_rn(B.z, A.z); acc = __fmaf_rn(d, d, acc); \
    d = __fsub_rn(B.w, A.w); acc = __fmaf_rn(d, d, acc); \
  }
  // long rows: eight chunks per trip in flight
  for (; i + 28 < n4; i += 32) {
    float4 a[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) a[k] = __ldg(x4 + i + 4 * k);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float4 b = q4[i + 4 * k];
      DVS_ACC4(b, a[k])
    }
  }
  // four chunks per trip keep four independent loads in flight
  for (; i + 12 < n4; i += 16) {
    const float4 a0 = __ldg(x4 + i), a1 = __ldg(x4 + i + 4), a2 = __ldg(x4 + i + 8), a3 = __ldg(x4 + i + 12);
    const float4 b0 = q4[i], b1 = q4[i + 4], b2 = q4[i + 8], b3 = q4[i + 12];
    DVS_ACC4(b0, a0) DVS_ACC4(b1, a1) DVS_ACC4(b2, a2) DVS_ACC4(b3, a3)
  }
  for (; i < n4; i += 4) {
    const float4 a = __ldg(x4 + i);
    const float4 b = q4[i];
    DVS_ACC4(b, a)
  }
#undef DVS_ACC4
  const uint32_t tail = (n4 << 2) + t;
  if (tail < dim) {
    const float d = __fsub_rn(q[tail], __ldg(x + tail));
    acc = __fmaf_rn(d, d, acc);
  }
  return acc;
}

// L2 cache policies (createpolicy): lines read under `keep` are evicted after
// other lines, lines read under `stream` first.
__device__ __forceinline__ uint64_t l2_policy_keep() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t l2_policy_stream() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// A read-only 16-byte load under an L2 cache policy.
__device__ __forceinline__ uint4 ldg_hint(const uint4* p, uint64_t pol) {
  uint4 v;
  asm volatile("ld.global.nc.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p), "l"(pol));
  return v;
}
__device__ __forceinline__ float4 ldg_hint(const float4* p, uint64_t pol) {
  const uint4 v = ldg_hint(reinterpret_cast<const uint4*>(p), pol);
  return make_float4(__uint_as_float(v.x), __uint_as_float(v.y), __uint_as_float(v.z), __uint_as_float(v.w));
}

// l2_quad_partial of two rows at once (xB may equal xA): the same chain per
// row, the two chains interleaved so their loads and FMAs overlap, each q
// chunk read once for both.  HINT: the rows are read under L2 policy `pol`.
template <bool HINT = false>
__device__ __forceinline__ void l2_quad_partial2(const float* __restrict__ q, const float* __restrict__ xA,
                                                 const float* __restrict__ xB, uint32_t dim, uint32_t t, float& accA,
                                                 float& accB, uint64_t pol = 0) {
  const uint32_t n4 = dim >> 2;
  const float4* q4 = reinterpret_cast<const float4*>(q);
  const float4* a4 = reinterpret_cast<const float4*>(xA);
  const float4* b4 = reinterpret_cast<const float4*>(xB);
  auto ld = [pol](const float4* p) { return HINT ? ldg_hint(p, pol) : __ldg(p); };
  float sa = 0.f, sb = 0.f;
#define DVS_ACC4_2(Q, A, B)                                              \
  {                                                                      \
    float d;                                                             \
    d = __fsub_rn(Q.x, A.x); sa = __fmaf_rn(d, d, sa);                   \
    d = __fsub_rn(Q.x, B.x); sb = __fmaf_rn(d, d, sb);                   \
    d = __fsub_rn(Q.y, A.y); sa = __fmaf_rn(d, d, sa);                   \
    d = __fsub_rn(Q.y, B.y); sb = __fmaf_rn(d, d, sb);                   \
    d = __fsub_rn(Q.z, A.z); sa = __fmaf_rn(d, d, sa);                   \
    d = __fsub_rn(Q.z, B.z); sb = __fmaf_rn(d, d, sb);                   \
    d = __fsub_rn(Q.w, A.w); sa = __fmaf_rn(d, d, sa);                   \
    d = __fsub_rn(Q.w, B.w); sb = __fmaf_rn(d, d, sb);                   \
  }
  uint32_t i = t;
  // four chunks of each row per trip in flight
  for (; i + 12 < n4; i += 16) {
    float4 a[4], b[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      a[k] = ld(a4 + i + 4 * k);
      b[k] = ld(b4 + i + 4 * k);
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float4 c = q4[i + 4 * k];
      DVS_ACC4_2(c, a[k], b[k])
    }
  }
  for (; i < n4; i += 4) {
    const float4 a = ld(a4 + i), b = ld(b4 + i);
    const float4 c = q4[i];
    DVS_ACC4_2(c, a, b)
  }
#undef DVS_ACC4_2
  const uint32_t tail = (n4 << 2) + t;
  if (tail < dim) {
    const float qt = q[tail];
    float d = __fsub_rn(qt, __ldg(xA + tail));
    sa = __fmaf_rn(d, d, sa);
    d = __fsub_rn(qt, __ldg(xB + tail));
    sb = __fmaf_rn(d, d, sb);
  }
  accA = sa;
  accB = sb;
}

// Same chain order on a single thread (all four lanes' chains), for callers that
// give one thread a whole row.
__device__ __forceinline__ float l2_single(const float* __restrict__ q, const float* __restrict__ x, uint32_t dim) {
  float s[4] = {0.f, 0.f, 0.f, 0.f};
  const uint32_t n4 = dim >> 2;
  for (uint32_t i = 0; i < n4; ++i) {
    float& a = s[i & 3];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float d = __fsub_rn(q[4 * i + k], x[4 * i + k]);
      a = __fmaf_rn(d, d, a);
    }
  }
  for (uint32_t i = n4 << 2; i < dim; ++i) {
    const float d = __fsub_rn(q[i], x[i]);
    float& a = s[(i - (n4 << 2)) & 3];
    a = __fmaf_rn(d, d, a);
  }
  return tile4_sum(s[0], s[1], s[2], s[3]);
}

// RaBitQ estimate from the four chain sums (distance_kernels.cuh:132-136 as nvcc
// contracts it): add_o + q.add + rescale_o * (dot + k1xSumq * (2^B - 1)).
__device__ __forceinline__ float rabitq_finish(float dot, float add_o, float rescale_o, float q_add, float q_k1,
                                               float k1) {
  return __fmaf_rn(rescale_o, __fmaf_rn(q_k1, k1, dot), __fadd_rn(add_o, q_add));
}

// Accumulates one 32-bit word of packed B-bit codes (B in {1,2,4}) that covers
// dims [j0, j0 + 32/B) into the four chains (dim j -> chain j & 3).  `qr` is the
// rotated query in shared memory.
template <int BITS>
__device__ __forceinline__ void rabitq_word(uint32_t word, const float* __restrict__ qr, uint32_t j0, uint32_t dim,
                                            float& s0, float& s1, float& s2, float& s3) {
  constexpr int kPer = 32 / BITS;
  constexpr uint32_t kMask = (1u << BITS) - 1u;
  if (BITS == 4 && j0 + kPer <= dim) {
    // nibble n of the word sits in byte n/2 of (n even ? lo : hi); PRMT places
    // it under the exponent of 2^23 so a subtraction yields the exact value
    const uint32_t lo = word & 0x0F0F0F0Fu, hi = (word >> 4) & 0x0F0F0F0Fu;
#pragma unroll
    for (int b = 0; b < 4; b += 2) {
      const float4 qv = *reinterpret_cast<const float4*>(qr + j0 + 2 * b);
      s0 = __fmaf_rn(__fsub_rn(__uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7440u + b)), 8388608.0f), qv.x, s0);
      s1 = __fmaf_rn(__fsub_rn(__uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7440u + b)), 8388608.0f), qv.y, s1);
      s2 = __fmaf_rn(__fsub_rn(__uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7441u + b)), 8388608.0f), qv.z, s2);
      s3 = __fmaf_rn(__fsub_rn(__uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7441u + b)), 8388608.0f), qv.w, s3);
    }
  } else if (j0 + kPer <= dim) {
#pragma unroll
    for (int n = 0; n < kPer; n += 4) {
      const float4 qv = *reinterpret_cast<const float4*>(qr + j0 + n);
      s0 = __fmaf_rn(small_u2f((word >> (BITS * (n + 0))) & kMask), qv.x, s0);
      s1 = __fmaf_rn(small_u2f((word >> (BITS * (n + 1))) & kMask), qv.y, s1);
      s2 = __fmaf_rn(small_u2f((word >> (BITS * (n + 2))) & kMask), qv.z, s2);
      s3 = __fmaf_rn(small_u2f((word >> (BITS * (n + 3))) & kMask), qv.w, s3);
    }
  } else {
    for (int n = 0; n < kPer && j0 + n < dim; ++n) {
      const float val = small_u2f((word >> (BITS * n)) & kMask);
      const float qv = qr[j0 + n];
      switch (n & 3) {
        case 0: s0 = __fmaf_rn(val, qv, s0); break;
        case 1: s1 = __fmaf_rn(val, qv, s1); break;
        case 2: s2 = __fmaf_rn(val, qv, s2); break;
        default: s3 = __fmaf_rn(val, qv, s3); break;
      }
    }
  }
}

// One char4 step of batch_rabitq_8bit_distance_kernel
// (src/gpu/kernels/distance_kernels.cuh:181-221): bytes b0..b3 of `word` are
// dims 4i..4i+3; x0*q0 + x1*q1 + x2*q2 + x3*q3 as nvcc contracts it
// (fma(x3,q3, fma(x2,q2, fma(x0,q0, x1*q1)))), to be added to chain i mod 4.
__device__ __forceinline__ float rabitq_char4(uint32_t word, float4 q) {
  const float x0 = __fsub_rn(__uint_as_float(__byte_perm(word, 0x4B000000u, 0x7440u)), 8388608.0f);
  const float x1 = __fsub_rn(__uint_as_float(__byte_perm(word, 0x4B000000u, 0x7441u)), 8388608.0f);
  const float x2 = __fsub_rn(__uint_as_float(__byte_perm(word, 0x4B000000u, 0x7442u)), 8388608.0f);
  const float x3 = __fsub_rn(__uint_as_float(__byte_perm(word, 0x4B000000u, 0x7443u)), 8388608.0f);
  float t = __fmul_rn(x1, q.y);
  t = __fmaf_rn(x0, q.x, t);
  t = __fmaf_rn(x2, q.z, t);
  return __fmaf_rn(x3, q.w, t);
}

// Medoid seed distance (L2Distance / IPDistance on the host in the reference,
// src/common/distance.hh:80-159): eight AVX lanes over 16-float chunks, a
// left-to-right horizontal sum, then the tail.  Lanes 0..7 of the warp each own
// one AVX lane; the result is returned on every lane.
__device__ __forceinline__ float seed_distance_warp(const float* __restrict__ q, const float* __restrict__ x,
                                                    uint32_t dim, bool ip, uint32_t lane) {
  const uint32_t q16 = dim >> 4 << 4;
  float acc = 0.f;
  if (lane < 8) {
    for (uint32_t c = 0; c < q16; c += 16) {
      const float a0 = q[c + lane], b0 = __ldg(x + c + lane);
      const float a1 = q[c + 8 + lane], b1 = __ldg(x + c + 8 + lane);
      if (ip) {
        acc = __fmaf_rn(a0, b0, acc);
        acc = __fmaf_rn(a1, b1, acc);
      } else {
        const float d0 = __fsub_rn(a0, b0);
        acc = __fmaf_rn(d0, d0, acc);
        const float d1 = __fsub_rn(a1, b1);
        acc = __fmaf_rn(d1, d1, acc);
      }
    }
  }
  float r = __shfl_sync(0xFFFFFFFFu, acc, 0);
#pragma unroll
  for (int l = 1; l < 8; ++l) r = __fadd_rn(r, __shfl_sync(0xFFFFFFFFu, acc, l));
  if (ip) {
    float tail = 0.f;
    for (uint32_t i = q16; i < dim; ++i) tail = __fmaf_rn(q[i], __ldg(x + i), tail);
    return __fsub_rn(1.0f, __fadd_rn(r, tail));
  }
  for (uint32_t i = q16; i < dim; ++i) {
    const float d = __fsub_rn(q[i], __ldg(x + i));
    r = __fmaf_rn(d, d, r);
  }
  return r;
}

__device__ __forceinline__ uint32_t lanemask_lt() {
  uint32_t m;
  asm volatile("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

__device__ __forceinline__ uint32_t hash_slot(uint32_t id, uint32_t cap) {
  const uint32_t h = id * 0x9E3779B1u;
  return uint32_t((uint64_t(h) * cap) >> 32);
}

}  // namespace dvs
