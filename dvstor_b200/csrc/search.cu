// Query-path kernels for sm_100a.
//
// search_kernel: a persistent kernel in which every warp takes queries from an
// atomic counter and runs the whole of Vamana::knn (src/vamana/vamana.hh:57-452)
// for one query at a time, on device-resident adjacency, RaBitQ records and
// vectors: medoid seed, beam expansion with a shared-memory visited set, RaBitQ
// estimates (rabitq_gpu) or exact distances (exact_gpu), lower_bound insertion
// into a beam of capacity L+64 (L), exact rerank of the whole beam and the final
// ordering.  The reference does each expansion as an RDMA read, an H2D copy, a
// tiny kernel launch and a blocking D2H copy (src/vamana/vamana.hh:131-356);
// here an expansion is ~1 µs of on-chip work and two dependent HBM reads.
//
// Beam semantics reproduced exactly (ids match the oracle bit for bit):
//   * a new candidate goes before every entry of equal distance
//     (std::lower_bound in insert_into_beam, vamana.hh:1014-1030); of several
//     equal new candidates of one expansion, the later-inserted comes first;
//   * the beam is trimmed to its capacity after the insertions;
//   * the next node to expand is the first unexpanded entry with distance
//     < FLT_MAX (vamana.hh:134-141);
//   * the visited set holds every neighbour ever seen (vamana.hh:174-182);
//   * after the loop, rabitq_gpu replaces every beam distance by the exact L2
//     (vamana.hh:358-422) and the beam is ordered by distance (vamana.hh:425);
//     entries of equal distance keep beam order (std::sort leaves their order
//     unspecified; this is the one documented tie).

#include <cuda_runtime.h>

#include "device_math.cuh"
#include "search.cuh"

namespace dvs {

namespace {

constexpr uint32_t kFull = 0xFFFFFFFFu;

// Per-warp spill table in global memory (linear probing).  For indexes of
// fewer than 2^24 nodes an entry is (epoch << 24) | id, and an entry whose
// epoch is not the query's own counts as empty: a query takes a fresh epoch
// instead of clearing the table, which is cleared only when the 8-bit epoch
// wraps.  Larger indexes store the bare id with kEmptySlot as empty, and the
// table is cleared by the query that first spills.  `tag` is the query's
// epoch << 24 (0 for the bare form).  Slots never become empty during a query,
// so a probe chain ends at the first empty slot.
__device__ __forceinline__ bool spill_empty(uint32_t v, uint32_t tag) {
  return tag ? (v & 0xFF000000u) != tag : v == kEmptySlot;
}

// Inserts `id`; true when it was not present.  The table never fills: callers
// keep its load under the limit.
__device__ __forceinline__ bool table_insert(uint32_t* tab, uint32_t cap, uint32_t id, uint32_t tag) {
  volatile uint32_t* vt = tab;
  const uint32_t key = tag | id;
  uint32_t s = hash_slot(id, cap);
  for (uint32_t probe = 0; probe < cap; ++probe) {
    uint32_t cur = vt[s];
    for (int tries = 0; tries < 32; ++tries) {  // another lane of the warp may take the slot first
      if (cur == key) return false;
      if (!spill_empty(cur, tag)) break;
      const uint32_t old = atomicCAS(tab + s, cur, key);
      if (old == cur) return true;
      cur = old;
    }
    s = (s + 1 == cap) ? 0 : s + 1;
  }
  return false;
}

__device__ __forceinline__ bool table_contains(const uint32_t* tab, uint32_t cap, uint32_t id, uint32_t tag) {
  const volatile uint32_t* vt = tab;
  const uint32_t key = tag | id;
  uint32_t s = hash_slot(id, cap);
  for (uint32_t probe = 0; probe < cap; ++probe) {
    const uint32_t cur = vt[s];
    if (cur == key) return true;
    if (spill_empty(cur, tag)) return false;
    s = (s + 1 == cap) ? 0 : s + 1;
  }
  return false;
}

// Shared-memory visited table probed in buckets of four slots (one 16-byte
// load per step): an id lives in the first bucket of its probe sequence that
// had a free slot when it was inserted, and slots never empty during a query,
// so a bucket with a free slot that lacks the id ends the search.
__device__ __forceinline__ uint4 load_bucket(const uint32_t* tab, uint32_t b) {
  uint4 v;
  asm volatile("ld.volatile.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(static_cast<uint32_t>(__cvta_generic_to_shared(tab + 4 * b))));
  return v;
}

__device__ __forceinline__ bool bucket_insert(uint32_t* tab, uint32_t nbuckets, uint32_t id) {
  uint32_t b = hash_slot(id, nbuckets);
  for (uint32_t probe = 0; probe < nbuckets; ++probe) {
    const uint4 v = load_bucket(tab, b);
    if (v.x == id || v.y == id || v.z == id || v.w == id) return false;
    const uint32_t sl[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      if (sl[e] == kEmptySlot) {
        const uint32_t old = atomicCAS(tab + 4 * b + e, kEmptySlot, id);
        if (old == kEmptySlot) return true;
        if (old == id) return false;
      }
    }
    b = (b + 1 == nbuckets) ? 0 : b + 1;
  }
  return false;
}

__device__ __forceinline__ bool bucket_contains(const uint32_t* tab, uint32_t nbuckets, uint32_t id) {
  uint32_t b = hash_slot(id, nbuckets);
  for (uint32_t probe = 0; probe < nbuckets; ++probe) {
    const uint4 v = load_bucket(tab, b);
    if (v.x == id || v.y == id || v.z == id || v.w == id) return true;
    if (v.x == kEmptySlot || v.y == kEmptySlot || v.z == kEmptySlot || v.w == kEmptySlot) return false;
    b = (b + 1 == nbuckets) ? 0 : b + 1;
  }
  return false;
}

// Compact visited table for indexes of fewer than 2^24 nodes: NB buckets of
// eight 16-bit entries, two-choice placement.  An id is mixed by two W-bit
// bijections h1, h2 (W = 20 for indexes of fewer than 2^20 nodes, else 24);
// for hash k it may live in bucket hk mod NB as the entry (k << 14) |
// (hk div NB).  (bucket, entry) determines hk and hence the id, so membership
// is exact with half the bytes of a 32-bit table, and a lookup is two
// independent 16-byte loads instead of a probe chain.  0xFFFF is empty
// (entries use 15 bits; NB >= 2^(W-14) keeps hk div NB below 2^14, so W = 20
// lets the table shrink to what the beam needs).
__device__ __forceinline__ uint32_t mixw(uint32_t x, uint32_t w) {
  const uint32_t mask = (1u << w) - 1u, s = w >> 1;
  x = (x * 0x9E3779u) & mask;  // odd multiplier: a bijection modulo 2^w
  x ^= x >> s;
  x = (x * 0x85EBCBu) & mask;
  x ^= x >> (s - 1);
  return x;
}

struct Slot16 {
  uint32_t b, tag;
};

// (hk mod nb, which << 14 | hk div nb).  The quotient is the high word of
// hk * magic with magic = ceil(2^32 / nb): for hk < 2^24 it is the exact
// quotient or one more, which the remainder's sign corrects.
__device__ __forceinline__ Slot16 split16(uint32_t h, uint32_t nb, uint32_t magic, uint32_t which) {
  uint32_t q = __umulhi(h, magic);
  int32_t r = int32_t(h) - int32_t(q * nb);
  if (r < 0) {
    --q;
    r += int32_t(nb);
  }
  return {uint32_t(r), (which << 14) | q};
}

// Entries hold at most 15 bits, and 0xFFFF is empty, so both tests are exact
// zero-halfword detections: (x - 0x00010001) & ~x & 0x80008000 sets bit 15 of a
// halfword iff it is zero, given that a nonzero halfword of x (or of ~v) never
// has bit 15 clear where the borrow from a zero halfword below could set it.
__device__ __forceinline__ uint32_t zero_halves(uint32_t x) { return (x - 0x00010001u) & ~x & 0x80008000u; }

__device__ __forceinline__ bool holds16(const uint4& v, uint32_t tag) {
  const uint32_t t = tag * 0x10001u;
  return (zero_halves(v.x ^ t) | zero_halves(v.y ^ t) | zero_halves(v.z ^ t) | zero_halves(v.w ^ t)) != 0;
}

// Empty entries of a bucket: bit 15 - w (entry 2w) and bit 31 - w (entry 2w + 1).
__device__ __forceinline__ uint32_t empty16(const uint4& v) {
  return zero_halves(~v.x) | (zero_halves(~v.y) >> 1) | (zero_halves(~v.z) >> 2) | (zero_halves(~v.w) >> 3);
}

__device__ __forceinline__ uint32_t empty_entry(uint32_t bit) { return bit >= 16 ? 2 * (31 - bit) + 1 : 2 * (15 - bit); }

enum : uint32_t { kVisited = 0, kFresh = 1, kNoRoom = 2 };

// Looks `id` up and, when absent and one of its two buckets has a free entry,
// inserts it.  Returns kVisited, kFresh, or kNoRoom (absent, both buckets
// full).  Entries are never removed during a query, so an id that was once
// refused for want of room still finds both its buckets full.
__device__ __forceinline__ uint32_t visit16(uint32_t* tab, uint32_t nb, uint32_t magic, uint32_t id, uint32_t w) {
  const uint32_t mask = (1u << w) - 1u;
  // the second hash is an odd multiple of the first modulo 2^w: a bijection of it, hence of the id
  const uint32_t h1 = mixw(id ^ (0x5A5A5Au & mask), w);
  const Slot16 s1 = split16(h1, nb, magic, 0);
  const Slot16 s2 = split16((h1 * 0x2C1B3Du) & mask, nb, magic, 1);
  unsigned short* t16 = reinterpret_cast<unsigned short*>(tab);
  // a failed claim means another lane filled an entry of these buckets: at most 16 can
  for (int attempt = 0; attempt < 17; ++attempt) {
    const uint4 v1 = load_bucket(tab, s1.b), v2 = load_bucket(tab, s2.b);
    if (holds16(v1, s1.tag) || holds16(v2, s2.tag)) return kVisited;
    const uint32_t e1 = empty16(v1), e2 = empty16(v2);
    if ((e1 | e2) == 0) return kNoRoom;
    const bool first = __popc(e1) >= __popc(e2);
    uint32_t em = first ? e1 : e2;
    const Slot16 c = first ? s1 : s2;
    while (em) {
      const uint32_t e = empty_entry(__ffs(em) - 1);
      em &= em - 1;
      const unsigned short old = atomicCAS(t16 + 8 * c.b + e, (unsigned short)0xFFFF, (unsigned short)c.tag);
      if (old == 0xFFFF) return kFresh;
    }
  }
  return kNoRoom;
}

// One 32-bit word of codes into the chains.  B in {1,2,4}: dim j -> chain
// j & 3 (rabitq_word).  B = 8: the word is one char4 step of the 8-bit kernel
// and goes whole to chain (word index) & 3 = e, the word's position in its
// 16-byte chunk; words past floor(dim/4) are not part of the sum.
template <int BITS>
__device__ __forceinline__ void code_word(uint32_t word, uint32_t wi, int e, const DevLayout& ix,
                                          const float* __restrict__ qr, float& s0, float& s1, float& s2, float& s3) {
  if constexpr (BITS == 8) {
    if (wi < (ix.dim >> 2)) {
      const float t = rabitq_char4(word, *reinterpret_cast<const float4*>(qr + 4 * wi));
      switch (e) {
        case 0: s0 = __fadd_rn(s0, t); break;
        case 1: s1 = __fadd_rn(s1, t); break;
        case 2: s2 = __fadd_rn(s2, t); break;
        default: s3 = __fadd_rn(s3, t); break;
      }
    }
  } else {
    rabitq_word<BITS>(word, qr, wi * (32 / BITS), ix.dim, s0, s1, s2, s3);
  }
}

// Chain t of NR records' 8-bit estimates (ids c[r]; a record may repeat c[0]
// when the round has fewer), computed by lane t of a lane quad: the reference
// kernel's own tile-of-4 split (lane t sums the char4 steps c = t mod 4), each
// chain in ascending order.  Used for 8-bit records wider than 128 bytes.  The
// NR chains are independent, so their loads and FMAs interleave; each q' read
// serves all of them; KB words of every record are in flight per batch.  `q`
// is q' in dimension order.  Lane 0 also returns the records' add and rescale
// factors.
template <int NR, int KB>
__device__ __forceinline__ void estimate_quad_chains8(const DevLayout& ix, const uint32_t (&c)[NR],
                                                      const float* __restrict__ q, uint32_t t, float (&s)[NR],
                                                      float (&f)[NR][2]) {
  const uint32_t* r[NR];
#pragma unroll
  for (int k = 0; k < NR; ++k) {
    r[k] = reinterpret_cast<const uint32_t*>(rec_row(ix, c[k]));
    s[k] = 0.f;
    if (t == 0) {
      f[k][0] = __uint_as_float(__ldg(r[k] + ix.code_words));
      f[k][1] = __uint_as_float(__ldg(r[k] + ix.code_words + 1));
    }
  }
  // lane t takes words t, t+4, ...: KB of each record in flight per batch
  const uint32_t nw = ix.dim >> 2;
  for (uint32_t w0 = t; w0 < nw; w0 += 4 * KB) {
    uint32_t a[NR][KB];
#pragma unroll
    for (int j = 0; j < KB; ++j)
      if (w0 + 4 * j < nw) {
#pragma unroll
        for (int k = 0; k < NR; ++k) a[k][j] = __ldg(r[k] + w0 + 4 * j);
      }
#pragma unroll
    for (int j = 0; j < KB; ++j)
      if (w0 + 4 * j < nw) {
        const float4 q4 = *reinterpret_cast<const float4*>(q + 4 * (w0 + 4 * j));
#pragma unroll
        for (int k = 0; k < NR; ++k) s[k] = __fadd_rn(s[k], rabitq_char4(a[k][j], q4));
      }
  }
}

// Chains 2h and 2h + 1 of the 1/2/4-bit estimate of record g, computed by lane
// h of a lane pair: the reference kernel's tile-of-4 chains (chain c sums dims
// j = c mod 4 in ascending order), both on one packed two-lane FP32 FMA per
// position (each lane of a packed FMA is the same fmaf).  `q` is this lane's
// half of the pair-major q'; the pair's other lane returns chains 2(1-h) and
// 2(1-h) + 1.  KB 16-byte chunks of the record are in flight per batch.
template <int BITS, int KB>
__device__ __forceinline__ float2 estimate_pair_chains(const DevLayout& ix, uint32_t g, const float* __restrict__ q,
                                                       uint32_t h) {
  const uint32_t* r = reinterpret_cast<const uint32_t*>(rec_row(ix, g));
  constexpr uint32_t kPer = 32 / BITS, kMask = (1u << BITS) - 1u;
  const float2 neg_magic = make_float2(-8388608.0f, -8388608.0f);
  float2 s = make_float2(0.f, 0.f);
  // a word holds kPer dims, kPer / 4 positions of each chain: this lane takes
  // dims n = 4i + 2h and 4i + 2h + 1 of it (position i of its two chains)
  const uint32_t nch = (ix.dim / kPer) >> 2;  // 16-byte chunks whose every dim is < dim
  for (uint32_t ch = 0; ch < nch; ch += KB) {
    uint4 v[KB];
#pragma unroll
    for (int j = 0; j < KB; ++j)
      if (ch + j < nch) v[j] = __ldg(reinterpret_cast<const uint4*>(r) + ch + j);
#pragma unroll
    for (int j = 0; j < KB; ++j) {
      if (ch + j < nch) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const uint32_t w = e == 0 ? v[j].x : e == 1 ? v[j].y : e == 2 ? v[j].z : v[j].w;
          const float* qw = q + 2 * ((ch + j) * 4 + e) * (kPer / 4);
          if constexpr (BITS == 4) {
            // dims 4i + 2h, 4i + 2h + 1 are the low and high nibble of byte 2i + h;
            // PRMT places each under the exponent of 2^23, the subtraction
            // leaves it exact
            const uint32_t lo = w & 0x0F0F0F0Fu, hi = (w >> 4) & 0x0F0F0F0Fu;
            const float4 qv = *reinterpret_cast<const float4*>(qw);
            const float2 c0 = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7440u + h)),
                                                     __uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7440u + h))),
                                         neg_magic);
            s = __ffma2_rn(c0, make_float2(qv.x, qv.y), s);
            const float2 c1 = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7442u + h)),
                                                     __uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7442u + h))),
                                         neg_magic);
            s = __ffma2_rn(c1, make_float2(qv.z, qv.w), s);
          } else {
#pragma unroll
            for (uint32_t i = 0; i < kPer / 4; i += 2) {
              const float4 qv = *reinterpret_cast<const float4*>(qw + 2 * i);
              const uint32_t n0 = 4 * i + 2 * h, n1 = n0 + 4;
              const float2 c0 = __fadd2_rn(make_float2(__uint_as_float(0x4B000000u | ((w >> (BITS * n0)) & kMask)),
                                                       __uint_as_float(0x4B000000u | ((w >> (BITS * (n0 + 1))) & kMask))),
                                           neg_magic);
              s = __ffma2_rn(c0, make_float2(qv.x, qv.y), s);
              const float2 c1 = __fadd2_rn(make_float2(__uint_as_float(0x4B000000u | ((w >> (BITS * n1)) & kMask)),
                                                       __uint_as_float(0x4B000000u | ((w >> (BITS * (n1 + 1))) & kMask))),
                                           neg_magic);
              s = __ffma2_rn(c1, make_float2(qv.z, qv.w), s);
            }
          }
        }
      }
    }
  }
  // words past the last whole chunk, the partial last word included
  for (uint32_t wi = nch * 4; wi * kPer < ix.dim; ++wi) {
    const uint32_t w = __ldg(r + wi), j0 = wi * kPer;
    for (uint32_t i = 0; i < kPer / 4; ++i) {
      const uint32_t n = 4 * i + 2 * h;
      const float* qp = q + 2 * ((j0 + n) >> 2);
      if (j0 + n < ix.dim) s.x = __fmaf_rn(small_u2f((w >> (BITS * n)) & kMask), qp[0], s.x);
      if (j0 + n + 1 < ix.dim) s.y = __fmaf_rn(small_u2f((w >> (BITS * (n + 1))) & kMask), qp[1], s.y);
    }
  }
  return s;
}

// Asks L2 for every 128-byte line of node g's RaBitQ record (wide records:
// their chunks are loaded in several dependent batches, which then hit L2).
__device__ __forceinline__ void prefetch_record_l2(const DevLayout& ix, uint32_t g) {
  const uintptr_t r = reinterpret_cast<uintptr_t>(rec_row(ix, g));
  const uintptr_t last = (r + ix.rec_words * 4 - 1) & ~uintptr_t(127);
  for (uintptr_t line = r & ~uintptr_t(127); line <= last; line += 128)
    asm volatile("prefetch.global.L2 [%0];" ::"l"(line));
}

// Exact L2 of `count` rows (slot ids in `rows`) against q, written to `out`;
// 4 lanes per row, two rows per lane quad (rows i and i + 8), 16 rows per
// round.  Warp-uniform control flow.
template <bool HINT = false>
__device__ __forceinline__ void l2_rows_warp(const DevLayout& ix, const float* __restrict__ q,
                                             const uint32_t* rows, uint32_t count, float* out, uint32_t lane,
                                             uint32_t row_mask, uint64_t pol = 0) {
  const uint32_t t = lane & 3;
  for (uint32_t r0 = 0; r0 < count; r0 += 16) {
    const uint32_t iA = r0 + (lane >> 2), iB = iA + 8;
    float pA = 0.f, pB = 0.f;
    if (iA < count) {
      const float* xA = vec_row(ix, rows[iA] & row_mask);
      const float* xB = iB < count ? vec_row(ix, rows[iB] & row_mask) : xA;
      l2_quad_partial2<HINT>(q, xA, xB, ix.dim, t, pA, pB, pol);
    }
    const float tA = quad_butterfly(pA), tB = quad_butterfly(pB);
    if (t == 0) {
      if (iA < count) out[iA] = tA;
      if (iB < count) out[iB] = tB;
    }
  }
}

// RaBitQ estimate of a record already held in registers (RCH 16-byte chunks).
// 4-bit codes: the chains run in pairs (0,1) and (2,3) on packed two-lane FP32
// instructions; each lane of a packed FMA is the same fmaf, so every chain
// sees the reference's sequence of operations.
template <int BITS, int RCH>
__device__ __forceinline__ float estimate_regs(const uint4 (&v)[RCH], const DevLayout& ix, const float* __restrict__ qr,
                                               float q_add, float q_k1) {
  float add_o = 0.f, rs_o = 0.f;
  if constexpr (BITS == 4) {
    float2 s01 = make_float2(0.f, 0.f), s23 = make_float2(0.f, 0.f);
    const float2 neg_magic = make_float2(-8388608.0f, -8388608.0f);
#pragma unroll
    for (int t = 0; t < RCH; ++t) {
      const uint32_t w[4] = {v[t].x, v[t].y, v[t].z, v[t].w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const uint32_t wi = t * 4 + e;
        if (wi < ix.code_words) {
          const uint32_t j0 = wi * 8;
          if (j0 + 8 <= ix.dim) {
            // nibble n of the word sits in byte n/2 of (n even ? lo : hi); PRMT
            // places it under the exponent of 2^23, the subtraction leaves it exact
            const uint32_t lo = w[e] & 0x0F0F0F0Fu, hi = (w[e] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
            for (int b = 0; b < 4; b += 2) {
              const float4 qv = *reinterpret_cast<const float4*>(qr + j0 + 2 * b);
              const float2 c01 = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7440u + b)),
                                                        __uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7440u + b))),
                                            neg_magic);
              const float2 c23 = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7441u + b)),
                                                        __uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7441u + b))),
                                            neg_magic);
              s01 = __ffma2_rn(c01, make_float2(qv.x, qv.y), s01);
              s23 = __ffma2_rn(c23, make_float2(qv.z, qv.w), s23);
            }
          } else {
            rabitq_word<4>(w[e], qr, j0, ix.dim, s01.x, s01.y, s23.x, s23.y);
          }
        } else if (wi == ix.code_words) {
          add_o = __uint_as_float(w[e]);
        } else if (wi == ix.code_words + 1) {
          rs_o = __uint_as_float(w[e]);
        }
      }
    }
    return rabitq_finish(tile4_sum(s01.x, s01.y, s23.x, s23.y), add_o, rs_o, q_add, q_k1, 15.0f);
  } else {
    float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll
    for (int t = 0; t < RCH; ++t) {
      const uint32_t w[4] = {v[t].x, v[t].y, v[t].z, v[t].w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const uint32_t wi = t * 4 + e;
        if (wi < ix.code_words)
          code_word<BITS>(w[e], wi, e, ix, qr, s0, s1, s2, s3);
        else if (wi == ix.code_words)
          add_o = __uint_as_float(w[e]);
        else if (wi == ix.code_words + 1)
          rs_o = __uint_as_float(w[e]);
      }
    }
    return rabitq_finish(tile4_sum(s0, s1, s2, s3), add_o, rs_o, q_add, q_k1, float((1u << BITS) - 1u));
  }
}

// Warp-uniform first index p >= lo of a sorted shared array with a[p] >= x.
__device__ __forceinline__ uint32_t lower_bound_smem(const float* a, uint32_t n, float x) {
  uint32_t lo = 0, hi = n;
  while (lo < hi) {
    const uint32_t mid = (lo + hi) >> 1;
    if (a[mid] < x)
      lo = mid + 1;
    else
      hi = mid;
  }
  return lo;
}

// Wide records: 8-bit records per lane quad per round and words of each in
// flight per batch; 16-byte chunks of a 1/2/4-bit record in flight per batch.
constexpr int kWideRecs = 3, kWideBatch = 6, kPairBatch = 15;

// Register cap of a search_kernel instantiation.  R <= 32 with records of up
// to 64 bytes in registers (and exact_gpu): 96, five warps per SM
// sub-partition (16,384 registers each), so that 20 warps fit an SM when
// shared memory allows (measured on the 96-dim L = 64 search: 96 registers and
// a 40-slot table, 2.64 M queries/s; 128 registers and 48 slots, 2.55 M).
// Records of up to 128 bytes in registers: 128 (at 96 they spill).  Records
// loaded after the visited check (wider than 128 bytes): 168, three warps per
// sub-partition.  The rest are bounded by shared memory or need their
// registers, and keep up to 255.
__host__ __device__ constexpr int search_max_regs(int npl, int rch, bool exact) {
  return npl == 1 && (rch == 4 || exact) ? 96 : npl == 1 && rch == 8 ? 128 : (rch == 0 && !exact) ? 168 : 255;
}

// EXACT: exact_gpu (exact distances, no records; BITS and RCH unused) or
// rabitq_gpu.  BITS: code width.  NPL: adjacency slots per lane (R <= 32 * NPL).  RCH: 16-byte
// chunks of a RaBitQ record a lane holds in registers (0 = records too large:
// they are loaded after the visited check instead).
template <int BITS, int NPL, int RCH, bool EXACT>
__global__ void __maxnreg__(search_max_regs(NPL, RCH, EXACT)) search_kernel(const SearchArgs a) {
  extern __shared__ __align__(16) uint32_t smem[];
  const uint32_t lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
  const DevLayout& ix = a.ix;
  constexpr uint32_t qlayout = EXACT ? kQueryRaw : (RCH == 0 && BITS != 8 ? kQueryPair : kQueryRot);
  uint32_t* base = smem + size_t(wib) * search_warp_words(a.cap_pad, a.dim_pad, a.hcap, ix.R, qlayout);
  float* bd = reinterpret_cast<float*>(base);  // the beam: distances
  uint32_t* bi = base + a.cap_pad;            // and slot | expanded bit
  // exact_gpu: the query (qv); rabitq_gpu: q' (qr) in dimension order or pair-major
  float* qv = reinterpret_cast<float*>(base + 2 * a.cap_pad);
  float* qr = qv;
  uint32_t* cid = base + 2 * a.cap_pad + (qlayout == kQueryPair ? 2 * pair_stride(a.dim_pad) : a.dim_pad);
  float* cd = reinterpret_cast<float*>(cid + 32 * NPL);
  float* sd = reinterpret_cast<float*>(cid + 64 * NPL);
  uint32_t* sid = cid + 96 * NPL;
  uint32_t* htab = cid + 128 * NPL;
  const uint32_t warp_slot = blockIdx.x * (blockDim.x >> 5) + wib;
  uint32_t* gtab = a.ovf ? a.ovf + size_t(warp_slot) * a.ovf_cap : nullptr;
  constexpr bool rabitq = !EXACT;  // the mode is a template parameter: each kernel holds one loop body
  const uint32_t dim = ix.dim, R = ix.R;
  const uint32_t nch = (ix.code_words + 2 + 3) >> 2;
  const float kInf = __int_as_float(0x7F800000);
  // RaBitQ records in registers are read under an L2 keep policy (1M 64-byte
  // records fit L2), the rerank's full vectors under a stream policy
  const uint64_t pol_keep = l2_policy_keep(), pol_stream = l2_policy_stream();

  for (;;) {
    uint32_t qi = 0;
    if (lane == 0) qi = atomicAdd(a.work, 1u);
    qi = __shfl_sync(kFull, qi, 0);
    if (qi >= a.nq) break;

    // ---- per-query set-up ----
    bool finite = true;
    const float* qg = a.queries + size_t(qi) * dim;
    for (uint32_t j = lane; j < a.dim_pad; j += 32) {
      const float x = j < dim ? qg[j] : 0.f;
      finite &= isfinite(x);
      if constexpr (qlayout == kQueryRaw) {
        qv[j] = x;
      } else {
        const float y = a.qrot[size_t(qi) * ix.vec_stride + j];
        // pair-major: half (j mod 4) / 2, position j / 4, chain (j mod 4) odd second
        qr[qlayout == kQueryPair ? ((j & 3) >> 1) * pair_stride(a.dim_pad) + 2 * (j >> 2) + (j & 1) : j] = y;
      }
    }
    const bool nonfinite = !__all_sync(kFull, finite);
    float q_add = 0.f, q_k1 = 0.f;
    if (rabitq) {
      q_add = a.qfac[size_t(qi) * 4 + 0];
      q_k1 = a.qfac[size_t(qi) * 4 + 1];
    }
    {
      uint4* h4 = reinterpret_cast<uint4*>(htab);
      const uint4 e = make_uint4(kEmptySlot, kEmptySlot, kEmptySlot, kEmptySlot);
      for (uint32_t j = lane; j < (a.hcap >> 2); j += 32) h4[j] = e;
    }
    __syncwarp();
    const float md = seed_distance_warp(rabitq ? qg : qv, vec_row(ix, ix.medoid), dim, ix.metric == 1, lane);
    if (lane == 0) {
      bd[0] = md;
      bi[0] = ix.medoid;
      if (!a.vt16) htab[4 * hash_slot(ix.medoid, a.hcap >> 2)] = ix.medoid;
    }
    __syncwarp();
    if (a.vt16 && lane == 0) visit16(htab, a.hbuckets, a.hb_magic, ix.medoid, a.vt16);
    __syncwarp();
    uint32_t nb = 1, hcount = 1, gcount = 0, H = 0, E = 0, err = 0, scan_from = 0;
    if (nonfinite) {
      nb = 0;  // nothing is selectable: the loop ends at once and every result slot is empty
      err = kErrNonFinite;
    }
    bool overflow = false;
    uint32_t gtag = 0;
    uint32_t pf_node = kEmptySlot, pf[NPL];

    for (;;) {
      // ---- select the first unexpanded entry (vamana.hh:134-141) ----
      // entries before scan_from are expanded or not selectable; the next
      // selectable entry of the same chunk is the guess for the following hop
      int best = -1, next = -1;
      for (uint32_t b = scan_from & ~31u; b < nb; b += 32) {
        const uint32_t p = b + lane;
        const bool ok = p < nb && !(bi[p] & kExpandedBit) && bd[p] < FLT_MAX;
        const uint32_t msk = __ballot_sync(kFull, ok);
        if (msk) {
          best = int(b + __ffs(msk) - 1);
          const uint32_t rest = msk & (msk - 1);
          if (rest) next = int(b + __ffs(rest) - 1);
          break;
        }
      }
      if (best < 0) break;
      if (a.hop_limit && H >= a.hop_limit) {
        err |= kErrHopLimit;
        break;
      }
      const uint32_t u = bi[best];
      const uint32_t guess = next >= 0 ? bi[next] : kEmptySlot;
      __syncwarp();
      if (lane == 0) bi[best] = u | kExpandedBit;
      ++H;

      // ---- neighbours (vamana.hh:162-168): prefetched one hop ahead when guessed ----
      uint32_t nbr[NPL];
      const bool hit = u == pf_node;
#pragma unroll
      for (int s = 0; s < NPL; ++s) {
        const uint32_t j = lane + 32u * s;
        nbr[s] = hit ? pf[s] : (j < R ? __ldg(adj_row(ix, u) + j) : kEmptySlot);
      }
      pf_node = guess;
#pragma unroll
      for (int s = 0; s < NPL; ++s) {
        const uint32_t j = lane + 32u * s;
        pf[s] = (guess != kEmptySlot && j < R) ? __ldg(adj_row(ix, guess) + j) : kEmptySlot;
      }
      if (RCH == 0 && rabitq && !hit) {
        // wide records: every listed neighbour's record is brought towards L2
        // now (unless the previous hop already did, for a guessed row)
#pragma unroll
        for (int s = 0; s < NPL; ++s)
          if (nbr[s] != kEmptySlot) prefetch_record_l2(ix, nbr[s]);
      }
      // records of every listed neighbour are requested before the visited
      // check so their latency overlaps it; visited ones are discarded
      uint4 rv[NPL][RCH > 0 ? RCH : 1];
      if (RCH > 0 && rabitq) {
#pragma unroll
        for (int s = 0; s < NPL; ++s) {
          if (nbr[s] != kEmptySlot) {
#pragma unroll
            for (int c = 0; c < RCH; ++c)
              if (c < int(nch)) rv[s][c] = ldg_hint(reinterpret_cast<const uint4*>(rec_row(ix, nbr[s])) + c, pol_keep);
          }
        }
      }

      // ---- visited filter (vamana.hh:172-182) ----
      // Shared table first; ids it cannot hold go to this warp's spill table in
      // global memory, which every later miss then consults.
      uint32_t m = 0;
      bool fresh[NPL];
#pragma unroll
      for (int s = 0; s < NPL; ++s) {
        fresh[s] = false;
        const uint32_t id = nbr[s];
        const uint32_t peers = __match_any_sync(kFull, id);
        const bool first = id != kEmptySlot && (peers & lanemask_lt()) == 0;
        bool full = false;
        if (first) {
          if (a.vt16) {
            // an id in the spill table found both its buckets full when it
            // spilled, and they still are: only such a lookup probes the spill
            uint32_t r = visit16(htab, a.hbuckets, a.hb_magic, id, a.vt16);
            if (r == kNoRoom && overflow && table_contains(gtab, a.ovf_cap, id, gtag)) r = kVisited;
            fresh[s] = r == kFresh;
            full = r == kNoRoom;
          } else if (!(overflow && table_contains(gtab, a.ovf_cap, id, gtag))) {
            // the 32-bit table is linear-probed: it stops taking ids at its load limit
            const bool may_insert = hcount + 32 <= a.hlimit;
            const uint32_t r = may_insert ? (bucket_insert(htab, a.hcap >> 2, id) ? kFresh : kVisited)
                                          : (bucket_contains(htab, a.hcap >> 2, id) ? kVisited : kNoRoom);
            fresh[s] = r == kFresh;
            full = r == kNoRoom;
          }
        }
        const uint32_t need = __ballot_sync(kFull, full);
        if (need) {
          if (!overflow) {
            if (gtab == nullptr) {
              err |= kErrCapacity;
              break;
            }
            // a fresh epoch for this query's entries; the table is cleared only
            // when the epoch wraps (or, for bare ids, every time)
            uint32_t ep = 0;
            if (lane == 0) ep = a.ovf_epoch[warp_slot];
            ep = __shfl_sync(kFull, ep, 0) + 1;
            const bool clear = !a.ovf_tagged || ep > 255u;
            if (clear) {
              uint4* g4 = reinterpret_cast<uint4*>(gtab);
              const uint32_t f = a.ovf_tagged ? 0u : kEmptySlot;
              const uint4 e = make_uint4(f, f, f, f);
              for (uint32_t j = lane; j < (a.ovf_cap >> 2); j += 32) g4[j] = e;
              if (ep > 255u) ep = 1;
            }
            // bare ids leave the next tagged query a wrapped epoch, so it clears
            if (lane == 0) a.ovf_epoch[warp_slot] = a.ovf_tagged ? ep : 255u;
            gtag = a.ovf_tagged ? ep << 24 : 0u;
            __syncwarp();
            overflow = true;
          }
          if (gcount + 32 > a.ovf_limit) {
            err |= kErrCapacity;
            break;
          }
          if (full) fresh[s] = table_insert(gtab, a.ovf_cap, id, gtag);
          gcount += __popc(__ballot_sync(kFull, full && fresh[s]));
        }
        const uint32_t cnt = __popc(__ballot_sync(kFull, fresh[s]));
        m += cnt;
        hcount += cnt;
      }
      if (err & kErrCapacity) break;
      if (m == 0) {
        scan_from = best + 1;
        continue;
      }
      E += m;

      // ---- distances of the unvisited neighbours, staged in insertion order ----
      {
        uint32_t base_pos = 0;
#pragma unroll
        for (int s = 0; s < NPL; ++s) {
          const uint32_t bal = __ballot_sync(kFull, fresh[s]);
          if (fresh[s]) {
            const uint32_t pos = base_pos + __popc(bal & lanemask_lt());
            cid[pos] = nbr[s];
            if (RCH > 0 && rabitq) cd[pos] = estimate_regs<BITS, (RCH > 0 ? RCH : 1)>(rv[s], ix, qr, q_add, q_k1);
          }
          base_pos += __popc(bal);
        }
      }
      __syncwarp();
      if (!rabitq) {
        l2_rows_warp(ix, qv, cid, m, cd, lane, 0xFFFFFFFFu);
      } else if (RCH == 0) {
        if constexpr (BITS == 8) {
          // wide 8-bit records: 8 * kWideRecs per round, kWideRecs per lane quad
          // (candidates i, i + 8, ...), chains reduced with the tile butterfly
          const uint32_t t = lane & 3;
          for (uint32_t i0 = 0; i0 < m; i0 += 8 * kWideRecs) {
            const uint32_t i = i0 + (lane >> 2);
            float p[kWideRecs], f[kWideRecs][2];
#pragma unroll
            for (int k = 0; k < kWideRecs; ++k) {
              p[k] = 0.f;
              f[k][0] = f[k][1] = 0.f;
            }
            if (i < m) {
              uint32_t c[kWideRecs];
#pragma unroll
              for (int k = 0; k < kWideRecs; ++k) c[k] = i + 8u * k < m ? cid[i + 8u * k] : cid[i];
              estimate_quad_chains8<kWideRecs, kWideBatch>(ix, c, qr, t, p, f);
            }
#pragma unroll
            for (int k = 0; k < kWideRecs; ++k) {
              const float d = quad_butterfly(p[k]);
              if (t == 0 && i + 8u * k < m) cd[i + 8u * k] = rabitq_finish(d, f[k][0], f[k][1], q_add, q_k1, 255.0f);
            }
          }
        } else {
          // wide 1/2/4-bit records: a lane pair per record, 16 per round; lane h
          // sums chains 2h and 2h + 1, and the tile sum (s0 + s2) + (s1 + s3)
          // takes the partner's two chains by shuffle
          const uint32_t h = lane & 1;
          const float* qh = qr + h * pair_stride(a.dim_pad);
          for (uint32_t i0 = 0; i0 < m; i0 += 16) {
            const uint32_t i = i0 + (lane >> 1);
            float2 sc = make_float2(0.f, 0.f);
            float fa = 0.f, fr = 0.f;
            if (i < m) {
              const uint32_t g = cid[i];
              if (h == 0) {
                const uint32_t* r = reinterpret_cast<const uint32_t*>(rec_row(ix, g));
                fa = __uint_as_float(__ldg(r + ix.code_words));
                fr = __uint_as_float(__ldg(r + ix.code_words + 1));
              }
              sc = estimate_pair_chains<BITS, kPairBatch>(ix, g, qh, h);
            }
            const float o0 = __shfl_xor_sync(kFull, sc.x, 1), o1 = __shfl_xor_sync(kFull, sc.y, 1);
            if (h == 0 && i < m)
              cd[i] = rabitq_finish(__fadd_rn(__fadd_rn(sc.x, o0), __fadd_rn(sc.y, o1)), fa, fr, q_add, q_k1,
                                    float((1u << BITS) - 1u));
          }
        }
        // the guessed next row's records, one hop ahead
#pragma unroll
        for (int s = 0; s < NPL; ++s)
          if (pf[s] != kEmptySlot) prefetch_record_l2(ix, pf[s]);
      }
      __syncwarp();

      // ---- insert_into_beam for all m candidates (vamana.hh:347-352, 1014-1030) ----
      // A full beam drops every candidate farther than its last entry; those can
      // neither survive nor move a survivor, so they leave the merge first.  The
      // survivors are ranked by (distance, later insertion first); survivor i
      // lands at rank_i + ins_i (ins_i = beam entries strictly closer) and beam
      // entry p moves down by #{i : ins_i <= p} (candidates not farther than it).
      const float worst = nb == a.cap ? bd[a.cap - 1] : kInf;
      uint32_t ms = 0;
#pragma unroll
      for (int h = 0; h < NPL; ++h) {
        const uint32_t i = 32u * h + lane;
        const float d = i < m ? cd[i] : 0.f;
        const bool keep = i < m && d <= worst;
        const uint32_t bal = __ballot_sync(kFull, keep);
        if (keep) {
          sd[ms + __popc(bal & lanemask_lt())] = d;
          sid[ms + __popc(bal & lanemask_lt())] = cid[i];
        }
        ms += __popc(bal);
      }
      if (ms == 0) {
        scan_from = best + 1;
        continue;
      }
      __syncwarp();
      float nd[NPL];
      uint32_t nid[NPL], rank[NPL], ins[NPL];
#pragma unroll
      for (int h = 0; h < NPL; ++h) {
        const uint32_t i = 32u * h + lane;
        nd[h] = i < ms ? sd[i] : kInf;
        nid[h] = i < ms ? sid[i] : 0u;
        rank[h] = 0;
        ins[h] = i < ms ? lower_bound_smem(bd, nb, nd[h]) : 0xFFFFFFFFu;
      }
#pragma unroll 4
      for (uint32_t j = 0; j < ms; ++j) {
        const float dj = __shfl_sync(kFull, nd[j >> 5], j & 31);
#pragma unroll
        for (int h = 0; h < NPL; ++h) {
          const uint32_t i = 32u * h + lane;
          rank[h] += (dj < nd[h]) || (dj == nd[h] && j > i);
        }
      }
      uint32_t first_pos = 0xFFFFFFFFu;
#pragma unroll
      for (int h = 0; h < NPL; ++h)
        if (32u * h + lane < ms) first_pos = min(first_pos, rank[h] + ins[h]);
      first_pos = __reduce_min_sync(kFull, first_pos);
      // beam entry p moves down by #{survivors with ins <= p}.  ins depends on
      // the distance alone, so in rank order it never decreases: the count is
      // an upper-bound search of the insertion points laid out by rank (in sd,
      // whose distances were read into nd above).
      uint32_t* sins = reinterpret_cast<uint32_t*>(sd);
      __syncwarp();
#pragma unroll
      for (int h = 0; h < NPL; ++h)
        if (32u * h + lane < ms) sins[rank[h]] = ins[h];
      __syncwarp();
      // The beam moves in place, from its last 32-entry chunk down to the chunk
      // of the first insertion point (entries before it do not move): every
      // lane of a chunk reads its entry before any lane writes, and an entry
      // lands at or after its own position, in chunks already read.
      const uint32_t low_chunk = sins[0] & ~31u;
      for (uint32_t p0 = (nb - 1) & ~31u;; p0 -= 32) {
        const uint32_t p = p0 + lane;
        uint32_t shift = 0;
        float dv = 0.f;
        uint32_t iv = 0;
        if (p < nb) {
          uint32_t lo = 0, hi = ms;
          while (lo < hi) {
            const uint32_t mid = (lo + hi) >> 1;
            if (sins[mid] <= p)
              lo = mid + 1;
            else
              hi = mid;
          }
          shift = lo;
          dv = bd[p];
          iv = bi[p];
        }
        __syncwarp();
        if (shift && p + shift < a.cap) {
          bd[p + shift] = dv;
          bi[p + shift] = iv;
        }
        __syncwarp();
        if (p0 <= low_chunk) break;
      }
      // the survivors fill the positions the moves left
#pragma unroll
      for (int h = 0; h < NPL; ++h) {
        if (32u * h + lane < ms) {
          const uint32_t pos = rank[h] + ins[h];
          if (pos < a.cap) {
            bd[pos] = nd[h];
            bi[pos] = nid[h];
          }
        }
      }
      scan_from = min(first_pos, uint32_t(best) + 1);
      nb = min(a.cap, nb + ms);
      __syncwarp();
    }

    // ---- rerank (vamana.hh:358-422) and final order (vamana.hh:424-446) ----
    uint32_t Cr = 0;
    if (rabitq && nb > 0) {
      // the query goes into the visited table's words, dead once the search ends
      float* qx = reinterpret_cast<float*>(htab);
      __syncwarp();
      for (uint32_t j = lane; j < a.dim_pad; j += 32) qx[j] = j < dim ? qg[j] : 0.f;
      __syncwarp();
      l2_rows_warp<true>(ix, qx, bi, nb, bd, lane, ~kExpandedBit, pol_stream);
      Cr = nb;
      __syncwarp();
      for (uint32_t p = lane; p < nb; p += 32) {
        const float d = bd[p];
        uint32_t r = 0;
        for (uint32_t q = 0; q < nb; ++q) {
          const float dq = bd[q];
          r += (dq < d) || (dq == d && q < p);
        }
        if (r < a.k) {
          a.out_ids[size_t(qi) * a.k + r] = ix.ids[bi[p] & ~kExpandedBit];
          a.out_dist[size_t(qi) * a.k + r] = d;
        }
      }
    } else {
      for (uint32_t p = lane; p < nb && p < a.k; p += 32) {
        const uint32_t slot = bi[p] & ~kExpandedBit;
        a.out_ids[size_t(qi) * a.k + p] = a.out_slots ? slot : ix.ids[slot];
        a.out_dist[size_t(qi) * a.k + p] = bd[p];
      }
    }
    for (uint32_t r = nb + lane; r < a.k; r += 32) {
      a.out_ids[size_t(qi) * a.k + r] = kEmptySlot;
      a.out_dist[size_t(qi) * a.k + r] = kInf;
    }
    if (lane == 0) {
      if (a.counters) {
        a.counters[size_t(qi) * 4 + 0] = H;
        a.counters[size_t(qi) * 4 + 1] = E;
        a.counters[size_t(qi) * 4 + 2] = Cr;
        a.counters[size_t(qi) * 4 + 3] = min(nb, a.k) | (err << 16);
      }
      if (err) atomicOr(a.work + 1, err);
      if (overflow) atomicAdd(a.work + 2, 1u);
    }
    __syncwarp();
  }
}

// batch_rabitq_distance_kernel on the reference's staged layout (records back
// to back, rabitq_size bytes each, factors possibly unaligned): one thread per
// record, byte-wise reads, same chain order.
__global__ void estimate_ref_kernel(const float* __restrict__ qr, const float* __restrict__ f3,
                                    const uint8_t* __restrict__ rec, float* __restrict__ out, uint32_t n,
                                    uint32_t dim, uint32_t bits) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint32_t packed = (bits * dim + 7) / 8;
  const uint8_t* r = rec + size_t(i) * (packed + 8);
  const uint32_t mask = (1u << bits) - 1u;
  float s[4] = {0.f, 0.f, 0.f, 0.f};
  if (bits == 8) {
    // batch_rabitq_8bit_distance_kernel: char4 steps, chain i & 3, dims past 4*floor(dim/4) unused
    for (uint32_t c = 0; c < dim / 4; ++c) {
      const uint32_t word = uint32_t(r[4 * c]) | uint32_t(r[4 * c + 1]) << 8 | uint32_t(r[4 * c + 2]) << 16 |
                            uint32_t(r[4 * c + 3]) << 24;
      const float4 q4 = make_float4(qr[4 * c], qr[4 * c + 1], qr[4 * c + 2], qr[4 * c + 3]);
      s[c & 3] = __fadd_rn(s[c & 3], rabitq_char4(word, q4));
    }
  } else {
    for (uint32_t j = 0; j < dim; ++j) {
      const uint32_t bit_idx = j * bits, byte_idx = bit_idx >> 3, bit_off = bit_idx & 7;
      uint32_t chunk = r[byte_idx];
      if (bit_off + bits > 8 && byte_idx + 1 < packed) chunk |= uint32_t(r[byte_idx + 1]) << 8;
      s[j & 3] = __fmaf_rn(small_u2f((chunk >> bit_off) & mask), qr[j], s[j & 3]);
    }
  }
  uint32_t a_bits = 0, r_bits = 0;
  for (int b = 0; b < 4; ++b) {
    a_bits |= uint32_t(r[packed + b]) << (8 * b);
    r_bits |= uint32_t(r[packed + 4 + b]) << (8 * b);
  }
  out[i] = rabitq_finish(tile4_sum(s[0], s[1], s[2], s[3]), __uint_as_float(a_bits), __uint_as_float(r_bits), f3[0],
                         f3[1], float((1u << bits) - 1u));
}

// batch_l2_squared_distance_kernel<4> on contiguous rows: 4 lanes per row.
__global__ void l2_rows_kernel(const float* __restrict__ q, const float* __restrict__ cand, float* __restrict__ out,
                               uint32_t n, uint32_t dim) {
  const uint32_t gtid = blockIdx.x * blockDim.x + threadIdx.x;
  const uint32_t row = gtid >> 2, t = gtid & 3;
  float acc = 0.f;
  if (row < n) {
    const float* x = cand + size_t(row) * dim;
    const uint32_t n4 = dim >> 2;
    for (uint32_t i = t; i < n4; i += 4) {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float d = __fsub_rn(q[4 * i + k], x[4 * i + k]);
        acc = __fmaf_rn(d, d, acc);
      }
    }
    const uint32_t tail = (n4 << 2) + t;
    if (tail < dim) {
      const float d = __fsub_rn(q[tail], x[tail]);
      acc = __fmaf_rn(d, d, acc);
    }
  }
  acc = quad_butterfly(acc);
  if (row < n && t == 0) out[row] = acc;
}

template <int BITS, int NPL, int RCH, bool EXACT>
cudaError_t occ(uint32_t wpb, size_t smem, int* bps) {
  // the largest allowance once for all shapes (a block's static and dynamic
  // shared memory together at most kMaxBlockSmem), so concurrent searches of
  // other shapes never find it lowered under them
  auto* k = search_kernel<BITS, NPL, RCH, EXACT>;
  cudaFuncAttributes fa;
  cudaError_t e = cudaFuncGetAttributes(&fa, k);
  if (e != cudaSuccess) return e;
  const size_t max_dynamic = size_t(kMaxBlockSmem) - fa.sharedSizeBytes;
  e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(max_dynamic));
  if (e != cudaSuccess) return e;
  if (smem > max_dynamic) {
    *bps = 0;
    return cudaSuccess;
  }
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(bps, k, int(wpb * 32), smem);
}

template <int BITS, int NPL, int RCH, bool EXACT>
void launch(const SearchArgs& a, dim3 grid, dim3 block, size_t smem, cudaStream_t st) {
  search_kernel<BITS, NPL, RCH, EXACT><<<grid, block, smem, st>>>(a);
}

// Record chunks a lane keeps in registers: 4 (<= 64-byte records) or 8
// (<= 128 bytes); larger records are loaded after the visited check.
inline int record_chunks(uint32_t code_words) {
  const uint32_t nch = (code_words + 2 + 3) / 4;
  return nch <= 4 ? 4 : nch <= 8 ? 8 : 0;
}

template <int BITS, int NPL>
cudaError_t occ_rch(int rch, uint32_t wpb, size_t smem, int* bps) {
  return rch == 4 ? occ<BITS, NPL, 4, false>(wpb, smem, bps)
         : rch == 8 ? occ<BITS, NPL, 8, false>(wpb, smem, bps)
                    : occ<BITS, NPL, 0, false>(wpb, smem, bps);
}

template <int BITS, int NPL>
void launch_rch(int rch, const SearchArgs& a, dim3 g, dim3 b, size_t smem, cudaStream_t st) {
  if (rch == 4)
    launch<BITS, NPL, 4, false>(a, g, b, smem, st);
  else if (rch == 8)
    launch<BITS, NPL, 8, false>(a, g, b, smem, st);
  else
    launch<BITS, NPL, 0, false>(a, g, b, smem, st);
}

}  // namespace

uint32_t search_query_layout(bool exact, uint32_t bits, uint32_t code_words) {
  if (exact) return kQueryRaw;
  return record_chunks(code_words) == 0 && bits != 8 ? kQueryPair : kQueryRot;
}

bool search_wide_records(bool exact, uint32_t code_words) { return !exact && record_chunks(code_words) == 0; }

cudaError_t search_occupancy(uint32_t bits, uint32_t R, uint32_t code_words, bool exact, uint32_t wpb, size_t smem,
                             int* bps) {
  const bool two = R > 32;
  if (exact) return two ? occ<1, 2, 0, true>(wpb, smem, bps) : occ<1, 1, 0, true>(wpb, smem, bps);
  const int rch = record_chunks(code_words);
  switch (bits) {
    case 1: return two ? occ_rch<1, 2>(rch, wpb, smem, bps) : occ_rch<1, 1>(rch, wpb, smem, bps);
    case 2: return two ? occ_rch<2, 2>(rch, wpb, smem, bps) : occ_rch<2, 1>(rch, wpb, smem, bps);
    case 4: return two ? occ_rch<4, 2>(rch, wpb, smem, bps) : occ_rch<4, 1>(rch, wpb, smem, bps);
    case 8: return two ? occ_rch<8, 2>(rch, wpb, smem, bps) : occ_rch<8, 1>(rch, wpb, smem, bps);
    default: return cudaErrorInvalidValue;
  }
}

size_t search_block_smem(uint32_t cap_pad, uint32_t dim_pad, uint32_t hcap, uint32_t R, bool exact, uint32_t bits,
                         uint32_t code_words, uint32_t wpb) {
  return size_t(wpb) * search_warp_words(cap_pad, dim_pad, hcap, R, search_query_layout(exact, bits, code_words)) * 4;
}

cudaError_t launch_search(const SearchArgs& a, uint32_t wpb, uint32_t blocks, cudaStream_t stream) {
  const size_t smem = search_block_smem(a.cap_pad, a.dim_pad, a.hcap, a.ix.R, a.mode == 1, a.ix.bits,
                                        a.ix.code_words, wpb);
  const bool two = a.ix.R > 32;
  const int rch = record_chunks(a.ix.code_words);
  const dim3 grid(blocks), block(wpb * 32);
  if (a.mode == 1) {
    two ? launch<1, 2, 0, true>(a, grid, block, smem, stream) : launch<1, 1, 0, true>(a, grid, block, smem, stream);
    return cudaGetLastError();
  }
  switch (a.ix.bits) {
    case 1:
      two ? launch_rch<1, 2>(rch, a, grid, block, smem, stream) : launch_rch<1, 1>(rch, a, grid, block, smem, stream);
      break;
    case 2:
      two ? launch_rch<2, 2>(rch, a, grid, block, smem, stream) : launch_rch<2, 1>(rch, a, grid, block, smem, stream);
      break;
    case 4:
      two ? launch_rch<4, 2>(rch, a, grid, block, smem, stream) : launch_rch<4, 1>(rch, a, grid, block, smem, stream);
      break;
    case 8:
      two ? launch_rch<8, 2>(rch, a, grid, block, smem, stream) : launch_rch<8, 1>(rch, a, grid, block, smem, stream);
      break;
    default:
      return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_estimate_ref_layout(const float* qrot, const float* f3, const uint8_t* records, float* out,
                                       uint32_t n, uint32_t dim, uint32_t bits, cudaStream_t stream) {
  if (n == 0) return cudaSuccess;
  estimate_ref_kernel<<<(n + 127) / 128, 128, 0, stream>>>(qrot, f3, records, out, n, dim, bits);
  return cudaGetLastError();
}

__global__ void fill_f32_kernel(float* p, size_t n, float v) {
  const size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) p[i] = v;
}

cudaError_t launch_fill_f32(float* p, size_t n, float v, cudaStream_t stream) {
  if (n == 0) return cudaSuccess;
  fill_f32_kernel<<<uint32_t((n + 255) / 256), 256, 0, stream>>>(p, n, v);
  return cudaGetLastError();
}

cudaError_t launch_l2_rows(const float* q, const float* cand, float* out, uint32_t n, uint32_t dim,
                           cudaStream_t stream) {
  if (n == 0) return cudaSuccess;
  const uint64_t threads = uint64_t(n) * 4;
  l2_rows_kernel<<<uint32_t((threads + 255) / 256), 256, 0, stream>>>(q, cand, out, n, dim);
  return cudaGetLastError();
}

}  // namespace dvs
