// Seeded noise, perturbation and momentum rebuild for MuZO-Clip on sm_100a.
//
// The noise of a parameter block is the stream torch's CUDA generator produces for
// make_zo_noise_like (muzo_clip/prng.py:39-81): a fresh Philox4x32-10 generator keyed by
// hash64(step seed, name, shape, block), drawn by a grid-stride launch in which thread t of S
// fills elements t + S*(4c + j) from the j-th word of its c-th Philox block. The kernels here
// regenerate exactly those words (Philox4x32-10 below, from its publication) and, for normal
// noise, pass them through cuRAND's own Box-Muller transform (_curand_box_muller, called, not
// re-implemented), but organise the work for HBM: one work item is 8
// consecutive threads t..t+7 of one loop trip c, i.e. four 16-byte vectors (j = 0..3) of 8
// consecutive elements. Warps therefore read and write contiguous 512-byte runs, and the noise
// never touches memory.
#include <curand_kernel.h>

#include "muzo_common.cuh"

namespace muzo {
namespace {

// Philox4x32 with 10 rounds (Salmon, Moraes, Dror, Shaw, "Parallel Random Numbers: As Easy as
// 1, 2, 3", SC'11): per round two 32x32->64 multiplies of counter words 0 and 2 by the published
// multipliers, a swap-and-xor with the round key, and a Weyl increment of the key.
__device__ __forceinline__ uint4 philox4x32_10(uint4 c, uint32_t k0, uint32_t k1) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t hi0 = __umulhi(0xD2511F53u, c.x), lo0 = 0xD2511F53u * c.x;
    const uint32_t hi1 = __umulhi(0xCD9E8D57u, c.z), lo1 = 0xCD9E8D57u * c.z;
    c = make_uint4(hi1 ^ c.y ^ k0, lo1, hi0 ^ c.w ^ k1, lo0);
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return c;
}

// The four 32-bit words torch's generator gives launch thread t on loop trip `trip`: the Philox
// block whose counter holds (trip + offset/4) in its low 64 bits and t in its high 64 bits.
__device__ __forceinline__ uint4 thread_words(uint64_t key, uint64_t t, uint64_t word_offset, uint64_t trip) {
  const uint64_t blk = trip + (word_offset >> 2);
  return philox4x32_10(make_uint4(static_cast<uint32_t>(blk), static_cast<uint32_t>(blk >> 32),
                                  static_cast<uint32_t>(t), static_cast<uint32_t>(t >> 32)),
                       static_cast<uint32_t>(key), static_cast<uint32_t>(key >> 32));
}

// curand_normal4 of a Philox state positioned at the block `thread_words` returns: cuRAND's own
// Box-Muller transform (_curand_box_muller, called, not restated) on the four words, without
// the state set-up of curand_init.
__device__ __forceinline__ float4 normal4_from_words(uint4 r) {
  const float2 a = _curand_box_muller(r.x, r.y);
  const float2 b = _curand_box_muller(r.z, r.w);
  return make_float4(a.x, a.y, b.x, b.y);
}

// Noise of 8 consecutive launch threads t0..t0+7 for loop trip `trip`: z[j][k] is element
// t0 + k + S*(4*trip + j). `word_offset` is the launch's Philox offset (32-bit words). Normal
// noise applies cuRAND's Box-Muller transform to the same Philox words (curand_normal4).
template <int DIST>
__device__ __forceinline__ void noise8x4(uint64_t key, uint64_t t0, uint64_t word_offset,
                                         uint64_t trip, float (&z)[4][8]) {
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    if (DIST == MUZO_NORMAL) {
      const float4 n = normal4_from_words(thread_words(key, t0 + k, word_offset, trip));
      // randn's transform is rand * std + mean with std = 1, mean = 0
      z[0][k] = n.x; z[1][k] = n.y; z[2][k] = n.z; z[3][k] = n.w;
    } else {
      const uint4 r = thread_words(key, t0 + k, word_offset, trip);
      // randint(0, 2) keeps word % 2; the reference maps it to 2*b - 1
      z[0][k] = (r.x & 1u) ? 1.0f : -1.0f;
      z[1][k] = (r.y & 1u) ? 1.0f : -1.0f;
      z[2][k] = (r.z & 1u) ? 1.0f : -1.0f;
      z[3][k] = (r.w & 1u) ? 1.0f : -1.0f;
    }
  }
}

__device__ __forceinline__ int elem_size(int dtype) { return dtype == MUZO_F32 ? 4 : 2; }

__device__ __forceinline__ bool vec_ok(const void* base, int64_t elem_start, int dtype) {
  uintptr_t a = reinterpret_cast<uintptr_t>(base) + static_cast<uintptr_t>(elem_start) * elem_size(dtype);
  return (a & 15u) == 0;
}

struct SegView {
  char* param;
  char* out;
  char* kept;           // the block's kept noise (parameter dtype), or NULL
  int64_t numel;
  int64_t local_item0;  // first item of this CTA relative to the segment
  uint64_t philox_offset;
  uint32_t threads;
  int block;
};

// Every CTA handles MUZO_ITEMS_PER_CTA consecutive items of exactly one segment.
__device__ __forceinline__ SegView cta_segment(const muzo_segment* segs, int nsegs, int pdtype, int odtype,
                                               int64_t chunk = -1) {
  const int64_t item0 = (chunk < 0 ? static_cast<int64_t>(blockIdx.x) : chunk) * MUZO_ITEMS_PER_CTA;
  const int s = find_segment(segs, nsegs, item0);
  const muzo_segment& g = segs[s];
  SegView v;
  v.param = g.param ? static_cast<char*>(g.param) + g.elem_start * elem_size(pdtype) : nullptr;
  v.out = g.out ? static_cast<char*>(g.out) + g.elem_start * elem_size(odtype) : nullptr;
  v.kept = g.kept ? static_cast<char*>(g.kept) + g.elem_start * elem_size(pdtype) : nullptr;
  v.numel = g.numel;
  v.local_item0 = item0 - g.item_begin;
  v.philox_offset = g.philox_offset;
  v.threads = g.threads;
  v.block = g.block_index;
  return v;
}

constexpr int kItemsPerThread = MUZO_ITEMS_PER_CTA / kElemThreads;

// --------------------------------------------------------------------------- fill noise

template <int DIST>
__global__ void __launch_bounds__(kElemThreads)
fill_noise_kernel(const muzo_segment* __restrict__ segs, int nsegs, uint64_t key, int odtype) {
  const SegView sv = cta_segment(segs, nsegs, MUZO_F32, odtype);
  const uint32_t octets = sv.threads / 8;
  const bool vec = vec_ok(sv.out, 0, odtype);
#pragma unroll 1
  for (int it = 0; it < kItemsPerThread; ++it) {
    const uint32_t local = static_cast<uint32_t>(sv.local_item0) + it * kElemThreads + threadIdx.x;
    const uint32_t trip = local / octets;
    const uint32_t oct = local - trip * octets;
    const int64_t li0 = static_cast<int64_t>(sv.threads) * (4ll * trip) + 8ll * oct;
    if (li0 >= sv.numel) continue;
    float z[4][8];
    noise8x4<DIST>(key, 8ull * oct, sv.philox_offset, trip, z);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t li = li0 + static_cast<int64_t>(sv.threads) * j;
      if (li >= sv.numel) break;
      if (vec && li + 8 <= sv.numel) {
        store8(sv.out, li, odtype, z[j]);
      } else {
#pragma unroll
        for (int k = 0; k < 8; ++k)  // static indices keep the arrays in registers
          if (li + k < sv.numel) store_elem(sv.out, li + k, odtype, z[j][k]);
      }
    }
  }
}

// --------------------------------------------------------------------------- perturb

// W <- dtype(W + alpha * dtype(Z)). torch's add_(noise, alpha) evaluates a + alpha * b in fp32,
// which nvcc contracts to one fused multiply-add; for Rademacher noise (z = +-1, exact) that is
// w +- alpha. The weights of an item are loaded (still packed) before the Philox work so their
// latency overlaps it; Rademacher noise is kept as one sign bit per element.
template <int DTYPE>
struct Packed8 {
  uint4 a, b;  // 8 elements: 16 bytes for 16-bit types, 32 bytes for fp32
  __device__ __forceinline__ void load(const void* base, int64_t i) {
    if (DTYPE == MUZO_F32) {
      const uint4* p = reinterpret_cast<const uint4*>(reinterpret_cast<const float*>(base) + i);
      a = p[0]; b = p[1];
    } else {
      a = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(base) + i);
    }
  }
  __device__ __forceinline__ void unpack(float (&v)[8]) const {
    if (DTYPE == MUZO_F32) {
      v[0] = __uint_as_float(a.x); v[1] = __uint_as_float(a.y); v[2] = __uint_as_float(a.z); v[3] = __uint_as_float(a.w);
      v[4] = __uint_as_float(b.x); v[5] = __uint_as_float(b.y); v[6] = __uint_as_float(b.z); v[7] = __uint_as_float(b.w);
    } else {
      const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        if (DTYPE == MUZO_BF16) { v[2 * q] = bf16_lo(w[q]); v[2 * q + 1] = bf16_hi(w[q]); }
        else { v[2 * q] = half_lo(w[q]); v[2 * q + 1] = half_hi(w[q]); }
      }
    }
  }
};

// KEEP (normal noise only): also store the rounded noise dtype(Z) of every element to segs[i].out,
// laid out like the block, so that the other passes of the same projection can read it back
// instead of regenerating it.
template <int DIST, int DTYPE, bool KEEP = false>
__global__ void __launch_bounds__(kElemThreads, 4)
perturb_kernel(const muzo_segment* __restrict__ segs, int nsegs, const uint64_t* __restrict__ keys,
               float alpha) {
  static_assert(!KEEP || DIST == MUZO_NORMAL, "only normal noise is kept");
  const SegView sv = cta_segment(segs, nsegs, DTYPE, DTYPE);
  const uint32_t octets = sv.threads / 8;
  const bool keep = KEEP && sv.out != nullptr;  // a segment without a noise buffer only perturbs
  const bool vec = vec_ok(sv.param, 0, DTYPE) && (!keep || vec_ok(sv.out, 0, DTYPE));
  const uint64_t key = keys[sv.block];
#pragma unroll 1
  for (int it = 0; it < kItemsPerThread; ++it) {
    const uint32_t local = static_cast<uint32_t>(sv.local_item0) + it * kElemThreads + threadIdx.x;
    const uint32_t trip = local / octets;
    const uint32_t oct = local - trip * octets;
    const int64_t li0 = static_cast<int64_t>(sv.threads) * (4ll * trip) + 8ll * oct;
    if (li0 >= sv.numel) continue;
    if constexpr (DIST == MUZO_RADEMACHER) {
      // memory-bound: the packed weight loads go out before the Philox work (16-bit types)
      constexpr bool kHoist = DTYPE != MUZO_F32;
      Packed8<DTYPE> raw[4];
      if (kHoist) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int64_t li = li0 + static_cast<int64_t>(sv.threads) * j;
          if (vec && li + 8 <= sv.numel) raw[j].load(sv.param, li);
        }
      }
      uint32_t sbits[4] = {0u, 0u, 0u, 0u};  // one sign bit per element
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const uint4 r = thread_words(key, 8ull * oct + k, sv.philox_offset, trip);
        sbits[0] |= (r.x & 1u) << k; sbits[1] |= (r.y & 1u) << k;
        sbits[2] |= (r.z & 1u) << k; sbits[3] |= (r.w & 1u) << k;
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int64_t li = li0 + static_cast<int64_t>(sv.threads) * j;
        if (li >= sv.numel) break;
        const int cnt = li + 8 <= sv.numel ? 8 : static_cast<int>(sv.numel - li);
        float w[8];
        if (vec && cnt == 8) {
          if (!kHoist) raw[j].load(sv.param, li);
          raw[j].unpack(w);
        } else {
#pragma unroll
          for (int k = 0; k < 8; ++k) w[k] = k < cnt ? load_elem(sv.param, li + k, DTYPE) : 0.0f;
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) w[k] = __fadd_rn(w[k], ((sbits[j] >> k) & 1u) ? alpha : -alpha);
        if (vec && cnt == 8) {
          store8(sv.param, li, DTYPE, w);
        } else {
#pragma unroll
          for (int k = 0; k < 8; ++k)  // static indices keep w in registers
            if (k < cnt) store_elem(sv.param, li + k, DTYPE, w[k]);
        }
      }
    } else {
      // normal noise: bound by the Box-Muller arithmetic; weights loaded after it
      float z[4][8];
      noise8x4<DIST>(key, 8ull * oct, sv.philox_offset, trip, z);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int64_t li = li0 + static_cast<int64_t>(sv.threads) * j;
        if (li >= sv.numel) break;
        if (vec && li + 8 <= sv.numel) {
          float w[8];
          load8(sv.param, li, DTYPE, w);
#pragma unroll
          for (int k = 0; k < 8; k += 2) round2_to(z[j][k], z[j][k + 1], DTYPE);
          if (keep) store8(sv.out, li, DTYPE, z[j]);  // exact: z is already rounded to DTYPE
#pragma unroll
          for (int k = 0; k < 8; ++k) w[k] = __fmaf_rn(alpha, z[j][k], w[k]);
          store8(sv.param, li, DTYPE, w);
        } else {
#pragma unroll
          for (int k = 0; k < 8; ++k) {  // static indices keep z in registers
            if (li + k < sv.numel) {
              const float w = load_elem(sv.param, li + k, DTYPE);
              const float zr = round_to(z[j][k], DTYPE);
              if (keep) store_elem(sv.out, li + k, DTYPE, zr);
              store_elem(sv.param, li + k, DTYPE, __fmaf_rn(alpha, zr, w));
            }
          }
        }
      }
    }
  }
}

// --------------------------------------------------------------------------- rebuild

// The rebuild runs 512-thread CTAs in which two threads share a work item: each takes four of
// its eight launch threads (a quad), so a thread holds 16 accumulators instead of 32 and an SM
// keeps twice as many warps in flight to hide the Philox / Box-Muller latency.
constexpr int kRebuildThreads = 2 * kElemThreads;

template <int N>
__device__ __forceinline__ void block_accumulate3(double a, double b, double c, double* dst_a, double* dst_b,
                                                  double* dst_c) {
  __shared__ double red[3][N / 32];
  a = warp_sum(a); b = warp_sum(b); c = warp_sum(c);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) { red[0][warp] = a; red[1][warp] = b; red[2][warp] = c; }
  __syncthreads();
  if (warp == 0) {
    a = lane < N / 32 ? red[0][lane] : 0.0;
    b = lane < N / 32 ? red[1][lane] : 0.0;
    c = lane < N / 32 ? red[2][lane] : 0.0;
    a = warp_sum(a); b = warp_sum(b); c = warp_sum(c);
    if (lane == 0) {
      if (a != 0.0) atomicAdd(dst_a, a);
      if (b != 0.0) atomicAdd(dst_b, b);
      if (c != 0.0) atomicAdd(dst_c, c);
    }
  }
  __syncthreads();  // red is reused by the next chunk
}

// acc[j][k] += alpha * float(dtype(z)) for launch threads t0..t0+3 of loop trip `trip`.
template <int DIST, int PDTYPE>
__device__ __forceinline__ void accumulate4x4(uint64_t key, uint64_t t0, uint64_t word_offset, uint64_t trip,
                                              float alpha, float (&acc)[4][4]) {
  // normal noise: one Box-Muller block at a time (its temporaries are large; warps, not
  // unrolling, hide the latency); Rademacher: fully unrolled
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    if (DIST == MUZO_NORMAL && k > 0) asm volatile("" ::: "memory");
    if (DIST == MUZO_NORMAL) {
      float4 n = normal4_from_words(thread_words(key, t0 + k, word_offset, trip));
      round2_to(n.x, n.y, PDTYPE);
      round2_to(n.z, n.w, PDTYPE);
      acc[0][k] = __fmaf_rn(alpha, n.x, acc[0][k]);
      acc[1][k] = __fmaf_rn(alpha, n.y, acc[1][k]);
      acc[2][k] = __fmaf_rn(alpha, n.z, acc[2][k]);
      acc[3][k] = __fmaf_rn(alpha, n.w, acc[3][k]);
    } else {
      // z = +-1 is exact in every dtype and alpha * z is exact: acc + alpha*z == acc +- alpha
      const uint4 r = thread_words(key, t0 + k, word_offset, trip);
      acc[0][k] = __fadd_rn(acc[0][k], (r.x & 1u) ? alpha : -alpha);
      acc[1][k] = __fadd_rn(acc[1][k], (r.y & 1u) ? alpha : -alpha);
      acc[2][k] = __fadd_rn(acc[2][k], (r.z & 1u) ? alpha : -alpha);
      acc[3][k] = __fadd_rn(acc[3][k], (r.w & 1u) ? alpha : -alpha);
    }
  }
}

__device__ __forceinline__ void load4(const void* base, int64_t i, int dtype, float (&v)[4]) {
  if (dtype == MUZO_F32) {
    const float4 a = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(base) + i);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  } else {
    const uint2 u = *reinterpret_cast<const uint2*>(reinterpret_cast<const uint16_t*>(base) + i);
    if (dtype == MUZO_BF16) { v[0] = bf16_lo(u.x); v[1] = bf16_hi(u.x); v[2] = bf16_lo(u.y); v[3] = bf16_hi(u.y); }
    else { v[0] = half_lo(u.x); v[1] = half_hi(u.x); v[2] = half_lo(u.y); v[3] = half_hi(u.y); }
  }
}

// acc[j][k] += alpha * zk for the kept noise zk (already dtype(Z)) of elements li0 + S*j + k:
// the arithmetic of accumulate4x4's normal branch on values read from memory.
template <int PDTYPE>
__device__ __forceinline__ void accumulate_kept4x4(const char* kept, int64_t li0, uint32_t threads, int64_t numel,
                                                   bool vec, float alpha, float (&acc)[4][4]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int64_t li = li0 + static_cast<int64_t>(threads) * j;
    if (li >= numel) break;
    float z[4];
    if (vec && li + 4 <= numel) {
      load4(kept, li, PDTYPE, z);
    } else {
#pragma unroll
      for (int k = 0; k < 4; ++k) z[k] = li + k < numel ? load_elem(kept, li + k, PDTYPE) : 0.0f;
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) acc[j][k] = __fmaf_rn(alpha, z[k], acc[j][k]);
  }
}

__device__ __forceinline__ void store4_bf16(void* base, int64_t i, const float (&v)[4]) {
  uint2 u;
  u.x = pack_bf16(v[0], v[1]);
  u.y = pack_bf16(v[2], v[3]);
  *reinterpret_cast<uint2*>(reinterpret_cast<uint16_t*>(base) + i) = u;
}

// M = sum_h alphas[h] * float(dtype(Z_h)) (h = age, newest first, as the reference walks
// reversed(history)); M *= inv_coeff_sum; out = bf16(M). Also sums M^2, bf16(M)^2 and W^2.
// KEPT: Z_0 is read from the segment's kept noise (when it has one) instead of regenerated.
template <int DIST, int PDTYPE, bool KEPT = false>
__device__ __forceinline__ void rebuild_chunk(const muzo_segment* __restrict__ segs, int nsegs,
                                              const uint64_t* __restrict__ keys, const float* __restrict__ alphas,
                                              int horizon, int normalize, float inv_coeff_sum,
                                              double* __restrict__ sums, int32_t* __restrict__ flags,
                                              int64_t chunk) {
  const SegView sv = cta_segment(segs, nsegs, PDTYPE, MUZO_BF16, chunk);
  const uint32_t octets = sv.threads / 8;
  const bool vec = vec_ok(sv.out, 0, MUZO_BF16) && vec_ok(sv.param, 0, PDTYPE);
  const bool use_kept = KEPT && sv.kept != nullptr;
  const bool kept_vec = use_kept && vec_ok(sv.kept, 0, PDTYPE);
  const int h_first = use_kept ? 1 : 0;
  const uint64_t* bkeys = keys + static_cast<int64_t>(sv.block) * horizon;
  const int half = threadIdx.x & 1;          // which quad of the item's eight launch threads
  const int slot = threadIdx.x >> 1;         // item slot within the CTA's 256-item stride
  double m2 = 0.0, x2 = 0.0, w2 = 0.0;
  bool finite = true;
#pragma unroll 1
  for (int it = 0; it < kItemsPerThread; ++it) {
    const uint32_t local = static_cast<uint32_t>(sv.local_item0) + it * kElemThreads + slot;
    const uint32_t trip = local / octets;
    const uint32_t oct = local - trip * octets;
    const int64_t li0 = static_cast<int64_t>(sv.threads) * (4ll * trip) + 8ll * oct + 4 * half;
    if (li0 >= sv.numel) continue;
    float acc[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int k = 0; k < 4; ++k) acc[j][k] = 0.0f;
    if (use_kept) accumulate_kept4x4<PDTYPE>(sv.kept, li0, sv.threads, sv.numel, kept_vec, alphas[0], acc);
#pragma unroll 1
    for (int h = h_first; h < horizon; ++h)
      accumulate4x4<DIST, PDTYPE>(bkeys[h], 8ull * oct + 4 * half, sv.philox_offset, trip, alphas[h], acc);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t li = li0 + static_cast<int64_t>(sv.threads) * j;
      if (li >= sv.numel) break;
      float m[4], w[4];
      const int cnt = li + 4 <= sv.numel ? 4 : static_cast<int>(sv.numel - li);
#pragma unroll
      for (int k = 0; k < 4; ++k) m[k] = normalize ? acc[j][k] * inv_coeff_sum : acc[j][k];
      if (vec && cnt == 4) {
        load4(sv.param, li, PDTYPE, w);
        store4_bf16(sv.out, li, m);
      } else {
#pragma unroll
        for (int k = 0; k < 4; ++k) w[k] = k < cnt ? load_elem(sv.param, li + k, PDTYPE) : 0.0f;
#pragma unroll
        for (int k = 0; k < 4; ++k)  // static indices keep m in registers
          if (k < cnt) store_elem(sv.out, li + k, MUZO_BF16, m[k]);
      }
      float pm = 0.0f, px = 0.0f, pw = 0.0f;
      float mb[4] = {m[0], m[1], m[2], m[3]};
      bf16r2(mb[0], mb[1]);
      bf16r2(mb[2], mb[3]);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        if (k < cnt) {
          finite = finite && isfinite(m[k]);
          const float xb = mb[k];
          pm = __fmaf_rn(m[k], m[k], pm);
          px = __fmaf_rn(xb, xb, px);
          pw = __fmaf_rn(w[k], w[k], pw);
        }
      }
      m2 += pm; x2 += px; w2 += pw;
    }
  }
  double* bs = sums + static_cast<int64_t>(sv.block) * MUZO_NSUMS;
  block_accumulate3<kRebuildThreads>(m2, x2, w2, bs + MUZO_SUM_M2, bs + MUZO_SUM_X2, bs + MUZO_SUM_W2);
  if (!finite) atomicOr(flags + sv.block, MUZO_FLAG_NONFINITE_INPUT);
}

// M of the history rebuild in which history entry h is read from slot_base[h] + segs[i].kept
// (the block's byte offset inside a slot, in the block's dtype and layout) when slot_base[h] is
// nonzero and regenerated otherwise; the same arithmetic, in the same order, as rebuild_chunk.
template <int PDTYPE>
__device__ __forceinline__ void rebuild_history_chunk(const muzo_segment* __restrict__ segs, int nsegs,
                                                      const uint64_t* __restrict__ keys,
                                                      const float* __restrict__ alphas,
                                                      const uint64_t* __restrict__ slot_base, int horizon,
                                                      int normalize, float inv_coeff_sum, double* __restrict__ sums,
                                                      int32_t* __restrict__ flags, int64_t chunk) {
  const int64_t item0 = chunk * MUZO_ITEMS_PER_CTA;
  const muzo_segment& g = segs[find_segment(segs, nsegs, item0)];
  const SegView sv = cta_segment(segs, nsegs, PDTYPE, MUZO_BF16, chunk);
  const uint64_t kept_off = reinterpret_cast<uint64_t>(g.kept) + static_cast<uint64_t>(g.elem_start) * elem_size(PDTYPE);
  const uint32_t octets = sv.threads / 8;
  const bool vec = vec_ok(sv.out, 0, MUZO_BF16) && vec_ok(sv.param, 0, PDTYPE);
  const uint64_t* bkeys = keys + static_cast<int64_t>(sv.block) * horizon;
  const int half = threadIdx.x & 1;
  const int slot = threadIdx.x >> 1;
  double m2 = 0.0, x2 = 0.0, w2 = 0.0;
  bool finite = true;
#pragma unroll 1
  for (int it = 0; it < kItemsPerThread; ++it) {
    const uint32_t local = static_cast<uint32_t>(sv.local_item0) + it * kElemThreads + slot;
    const uint32_t trip = local / octets;
    const uint32_t oct = local - trip * octets;
    const int64_t li0 = static_cast<int64_t>(sv.threads) * (4ll * trip) + 8ll * oct + 4 * half;
    if (li0 >= sv.numel) continue;
    float acc[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int k = 0; k < 4; ++k) acc[j][k] = 0.0f;
#pragma unroll 1
    for (int h = 0; h < horizon; ++h) {
      const uint64_t base = slot_base[h];
      if (base != 0) {
        const char* kp = reinterpret_cast<const char*>(base + kept_off);
        accumulate_kept4x4<PDTYPE>(kp, li0, sv.threads, sv.numel, vec_ok(kp, 0, PDTYPE), alphas[h], acc);
      } else {
        accumulate4x4<MUZO_NORMAL, PDTYPE>(bkeys[h], 8ull * oct + 4 * half, sv.philox_offset, trip, alphas[h], acc);
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t li = li0 + static_cast<int64_t>(sv.threads) * j;
      if (li >= sv.numel) break;
      float m[4], w[4];
      const int cnt = li + 4 <= sv.numel ? 4 : static_cast<int>(sv.numel - li);
#pragma unroll
      for (int k = 0; k < 4; ++k) m[k] = normalize ? acc[j][k] * inv_coeff_sum : acc[j][k];
      if (vec && cnt == 4) {
        load4(sv.param, li, PDTYPE, w);
        store4_bf16(sv.out, li, m);
      } else {
#pragma unroll
        for (int k = 0; k < 4; ++k) w[k] = k < cnt ? load_elem(sv.param, li + k, PDTYPE) : 0.0f;
#pragma unroll
        for (int k = 0; k < 4; ++k)
          if (k < cnt) store_elem(sv.out, li + k, MUZO_BF16, m[k]);
      }
      float pm = 0.0f, px = 0.0f, pw = 0.0f;
      float mb[4] = {m[0], m[1], m[2], m[3]};
      bf16r2(mb[0], mb[1]);
      bf16r2(mb[2], mb[3]);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        if (k < cnt) {
          finite = finite && isfinite(m[k]);
          pm = __fmaf_rn(m[k], m[k], pm);
          px = __fmaf_rn(mb[k], mb[k], px);
          pw = __fmaf_rn(w[k], w[k], pw);
        }
      }
      m2 += pm; x2 += px; w2 += pw;
    }
  }
  double* bs = sums + static_cast<int64_t>(sv.block) * MUZO_NSUMS;
  block_accumulate3<kRebuildThreads>(m2, x2, w2, bs + MUZO_SUM_M2, bs + MUZO_SUM_X2, bs + MUZO_SUM_W2);
  if (!finite) atomicOr(flags + sv.block, MUZO_FLAG_NONFINITE_INPUT);
}

template <int PDTYPE>
__global__ void __launch_bounds__(kRebuildThreads, 2)
rebuild_history_kernel(const muzo_segment* __restrict__ segs, int nsegs, const uint64_t* __restrict__ keys,
                       const float* __restrict__ alphas, const uint64_t* __restrict__ slot_base, int horizon,
                       int normalize, float inv_coeff_sum, double* __restrict__ sums, int32_t* __restrict__ flags,
                       int64_t nchunks) {
  for (int64_t chunk = blockIdx.x; chunk < nchunks; chunk += gridDim.x)
    rebuild_history_chunk<PDTYPE>(segs, nsegs, keys, alphas, slot_base, horizon, normalize, inv_coeff_sum, sums,
                                  flags, chunk);
}

// The rebuild when every history entry is kept: a plain stream over linear segments (param = the
// block, out = bf16(M), kept = the block's byte offset inside a slot). Per 8 elements it reads
// the H kept vectors and the weights and writes bf16(M): 2H + 4 bytes per element for 16-bit
// weights. Accumulation order and arithmetic are rebuild_chunk's: acc = fma(alpha_h, z_h, acc)
// for h = 0 (newest) .. H-1, then the normalisation multiply.
constexpr int kKeptLoadsInFlight = 4;

template <int PDTYPE>
__global__ void __launch_bounds__(kElemThreads)
rebuild_kept_linear_kernel(const muzo_segment* __restrict__ segs, int nsegs, const float* __restrict__ alphas,
                           const uint64_t* __restrict__ slot_base, int horizon, int normalize, float inv_coeff_sum,
                           double* __restrict__ sums, int32_t* __restrict__ flags) {
  const int64_t item0 = static_cast<int64_t>(blockIdx.x) * MUZO_ITEMS_PER_CTA;
  const muzo_segment& g = segs[find_segment(segs, nsegs, item0)];
  const char* param = static_cast<const char*>(g.param);
  char* out = static_cast<char*>(g.out);
  const uint64_t kept_off = reinterpret_cast<uint64_t>(g.kept);
  const int64_t numel = g.numel;
  const int64_t local_item0 = item0 - g.item_begin;
  const bool vec = vec_ok(out, 0, MUZO_BF16) && vec_ok(param, 0, PDTYPE) && (kept_off & 15u) == 0;
  double m2 = 0.0, x2 = 0.0, w2 = 0.0;
  bool finite = true;
#pragma unroll 1
  for (int it = 0; it < kItemsPerThread; ++it) {
    const int64_t li = (local_item0 + it * kElemThreads + threadIdx.x) * 8;
    if (li >= numel) break;
    const int cnt = li + 8 <= numel ? 8 : static_cast<int>(numel - li);
    float acc[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) acc[k] = 0.0f;
    if (vec && cnt == 8) {
      // loads of several entries go out before their multiply-adds (memory-level parallelism)
#pragma unroll 1
      for (int h0 = 0; h0 < horizon; h0 += kKeptLoadsInFlight) {
        Packed8<PDTYPE> z[kKeptLoadsInFlight];
#pragma unroll
        for (int q = 0; q < kKeptLoadsInFlight; ++q)
          if (h0 + q < horizon) z[q].load(reinterpret_cast<const char*>(slot_base[h0 + q] + kept_off), li);
#pragma unroll
        for (int q = 0; q < kKeptLoadsInFlight; ++q) {
          if (h0 + q < horizon) {
            float v[8];
            z[q].unpack(v);
            const float a = alphas[h0 + q];
#pragma unroll
            for (int k = 0; k < 8; ++k) acc[k] = __fmaf_rn(a, v[k], acc[k]);
          }
        }
      }
    } else {
#pragma unroll 1
      for (int h = 0; h < horizon; ++h) {
        const char* kp = reinterpret_cast<const char*>(slot_base[h] + kept_off);
        const float a = alphas[h];
#pragma unroll
        for (int k = 0; k < 8; ++k)
          if (k < cnt) acc[k] = __fmaf_rn(a, load_elem(kp, li + k, PDTYPE), acc[k]);
      }
    }
    float m[8], w[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) m[k] = normalize ? acc[k] * inv_coeff_sum : acc[k];
    if (vec && cnt == 8) {
      load8(param, li, PDTYPE, w);
      store8(out, li, MUZO_BF16, m);
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k) w[k] = k < cnt ? load_elem(param, li + k, PDTYPE) : 0.0f;
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if (k < cnt) store_elem(out, li + k, MUZO_BF16, m[k]);
    }
    // the sums in the rebuild kernel's grouping: fp32 chains over 4 elements, added in fp64
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      float pm = 0.0f, px = 0.0f, pw = 0.0f;
      float mb[4] = {m[4 * q], m[4 * q + 1], m[4 * q + 2], m[4 * q + 3]};
      bf16r2(mb[0], mb[1]);
      bf16r2(mb[2], mb[3]);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        if (4 * q + k < cnt) {
          finite = finite && isfinite(m[4 * q + k]);
          pm = __fmaf_rn(m[4 * q + k], m[4 * q + k], pm);
          px = __fmaf_rn(mb[k], mb[k], px);
          pw = __fmaf_rn(w[4 * q + k], w[4 * q + k], pw);
        }
      }
      m2 += pm; x2 += px; w2 += pw;
    }
  }
  double* bs = sums + static_cast<int64_t>(g.block_index) * MUZO_NSUMS;
  block_accumulate3<kElemThreads>(m2, x2, w2, bs + MUZO_SUM_M2, bs + MUZO_SUM_X2, bs + MUZO_SUM_W2);
  if (!finite) atomicOr(flags + g.block_index, MUZO_FLAG_NONFINITE_INPUT);
}

template <int DIST, int PDTYPE, bool KEPT = false>
__global__ void __launch_bounds__(kRebuildThreads, 2)
rebuild_kernel(const muzo_segment* __restrict__ segs, int nsegs, const uint64_t* __restrict__ keys,
               const float* __restrict__ alphas, int horizon, int normalize, float inv_coeff_sum,
               double* __restrict__ sums, int32_t* __restrict__ flags, int64_t nchunks) {
  // a CTA walks chunks blockIdx.x, blockIdx.x + gridDim.x, ... (grid may be smaller than the
  // number of chunks, e.g. one CTA per SM next to a concurrently running GEMM)
  for (int64_t chunk = blockIdx.x; chunk < nchunks; chunk += gridDim.x)
    rebuild_chunk<DIST, PDTYPE, KEPT>(segs, nsegs, keys, alphas, horizon, normalize, inv_coeff_sum, sums, flags,
                                      chunk);
}

bool valid_dtype(int d) { return d == MUZO_F32 || d == MUZO_BF16 || d == MUZO_F16; }

template <typename F>
int dispatch_dtype(int dtype, F&& f) {
  switch (dtype) {
    case MUZO_F32: f(std::integral_constant<int, MUZO_F32>()); return MUZO_OK;
    case MUZO_BF16: f(std::integral_constant<int, MUZO_BF16>()); return MUZO_OK;
    case MUZO_F16: f(std::integral_constant<int, MUZO_F16>()); return MUZO_OK;
    default: return MUZO_ERR_DTYPE;
  }
}

int check_table(const muzo_segment* segs, int nsegs, int64_t total_items) {
  if (segs == nullptr || nsegs <= 0 || total_items <= 0 || total_items % MUZO_ITEMS_PER_CTA != 0)
    return MUZO_ERR_ARG;
  if (total_items / MUZO_ITEMS_PER_CTA > 0x7fffffffLL) return MUZO_ERR_UNSUPPORTED;
  return MUZO_OK;
}

}  // namespace
}  // namespace muzo

using namespace muzo;

extern "C" {

int muzo_fill_noise(const muzo_segment* d_segs, int nsegs, int64_t total_items, uint64_t key,
                    int dist, int out_dtype, void* stream) {
  if (nsegs == 0 || total_items == 0) return MUZO_OK;
  int st = check_table(d_segs, nsegs, total_items);
  if (st != MUZO_OK) return st;
  if (!valid_dtype(out_dtype)) return MUZO_ERR_DTYPE;
  const dim3 grid(static_cast<unsigned>(total_items / MUZO_ITEMS_PER_CTA));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dist == MUZO_NORMAL)
    fill_noise_kernel<MUZO_NORMAL><<<grid, kElemThreads, 0, s>>>(d_segs, nsegs, key, out_dtype);
  else if (dist == MUZO_RADEMACHER)
    fill_noise_kernel<MUZO_RADEMACHER><<<grid, kElemThreads, 0, s>>>(d_segs, nsegs, key, out_dtype);
  else
    return MUZO_ERR_ARG;
  return launch_status();
}

int muzo_perturb_segments(const muzo_segment* d_segs, int nsegs, int64_t total_items,
                          const uint64_t* d_keys, int dtype, int dist, float alpha, void* stream) {
  if (nsegs == 0 || total_items == 0) return MUZO_OK;
  int st = check_table(d_segs, nsegs, total_items);
  if (st != MUZO_OK) return st;
  if (d_keys == nullptr || (dist != MUZO_NORMAL && dist != MUZO_RADEMACHER)) return MUZO_ERR_ARG;
  const dim3 grid(static_cast<unsigned>(total_items / MUZO_ITEMS_PER_CTA));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  st = dispatch_dtype(dtype, [&](auto d) {
    constexpr int D = decltype(d)::value;
    if (dist == MUZO_NORMAL)
      perturb_kernel<MUZO_NORMAL, D><<<grid, kElemThreads, 0, s>>>(d_segs, nsegs, d_keys, alpha);
    else
      perturb_kernel<MUZO_RADEMACHER, D><<<grid, kElemThreads, 0, s>>>(d_segs, nsegs, d_keys, alpha);
  });
  if (st != MUZO_OK) return st;
  return launch_status();
}

int muzo_perturb_segments_keep_noise(const muzo_segment* d_segs, int nsegs, int64_t total_items,
                                     const uint64_t* d_keys, int dtype, float alpha, void* stream) {
  if (nsegs == 0 || total_items == 0) return MUZO_OK;
  int st = check_table(d_segs, nsegs, total_items);
  if (st != MUZO_OK) return st;
  if (d_keys == nullptr) return MUZO_ERR_ARG;
  const dim3 grid(static_cast<unsigned>(total_items / MUZO_ITEMS_PER_CTA));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  st = dispatch_dtype(dtype, [&](auto d) {
    constexpr int D = decltype(d)::value;
    perturb_kernel<MUZO_NORMAL, D, true><<<grid, kElemThreads, 0, s>>>(d_segs, nsegs, d_keys, alpha);
  });
  if (st != MUZO_OK) return st;
  return launch_status();
}

int muzo_rebuild_segments_kept(const muzo_segment* d_segs, int nsegs, int64_t total_items,
                               const uint64_t* d_keys, const float* d_alphas, int horizon,
                               int param_dtype, int normalize, float inv_coeff_sum, double* d_sums,
                               int32_t* d_flags, int max_ctas, void* stream) {
  if (nsegs == 0 || total_items == 0) return MUZO_OK;
  int st = check_table(d_segs, nsegs, total_items);
  if (st != MUZO_OK) return st;
  if (d_keys == nullptr || d_alphas == nullptr || d_sums == nullptr || d_flags == nullptr || horizon <= 0)
    return MUZO_ERR_ARG;
  const int64_t nchunks = total_items / MUZO_ITEMS_PER_CTA;
  const int64_t ctas = (max_ctas > 0 && max_ctas < nchunks) ? max_ctas : nchunks;
  const dim3 grid(static_cast<unsigned>(ctas));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  st = dispatch_dtype(param_dtype, [&](auto d) {
    constexpr int D = decltype(d)::value;
    rebuild_kernel<MUZO_NORMAL, D, true><<<grid, kRebuildThreads, 0, s>>>(
        d_segs, nsegs, d_keys, d_alphas, horizon, normalize, inv_coeff_sum, d_sums, d_flags, nchunks);
  });
  if (st != MUZO_OK) return st;
  return launch_status();
}

int muzo_rebuild_segments_history(const muzo_segment* d_segs, int nsegs, int64_t total_items,
                                  const uint64_t* d_keys, const float* d_alphas, const uint64_t* d_slot_base,
                                  int horizon, int param_dtype, int normalize, float inv_coeff_sum,
                                  double* d_sums, int32_t* d_flags, int max_ctas, void* stream) {
  if (nsegs == 0 || total_items == 0) return MUZO_OK;
  int st = check_table(d_segs, nsegs, total_items);
  if (st != MUZO_OK) return st;
  if (d_keys == nullptr || d_alphas == nullptr || d_slot_base == nullptr || d_sums == nullptr ||
      d_flags == nullptr || horizon <= 0)
    return MUZO_ERR_ARG;
  const int64_t nchunks = total_items / MUZO_ITEMS_PER_CTA;
  const int64_t ctas = (max_ctas > 0 && max_ctas < nchunks) ? max_ctas : nchunks;
  const dim3 grid(static_cast<unsigned>(ctas));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  st = dispatch_dtype(param_dtype, [&](auto d) {
    constexpr int D = decltype(d)::value;
    rebuild_history_kernel<D><<<grid, kRebuildThreads, 0, s>>>(d_segs, nsegs, d_keys, d_alphas, d_slot_base, horizon,
                                                              normalize, inv_coeff_sum, d_sums, d_flags, nchunks);
  });
  if (st != MUZO_OK) return st;
  return launch_status();
}

int muzo_rebuild_kept_linear(const muzo_segment* d_segs, int nsegs, int64_t total_items,
                             const float* d_alphas, const uint64_t* d_slot_base, int horizon, int param_dtype,
                             int normalize, float inv_coeff_sum, double* d_sums, int32_t* d_flags,
                             void* stream) {
  if (nsegs == 0 || total_items == 0) return MUZO_OK;
  int st = check_table(d_segs, nsegs, total_items);
  if (st != MUZO_OK) return st;
  if (d_alphas == nullptr || d_slot_base == nullptr || d_sums == nullptr || d_flags == nullptr || horizon <= 0)
    return MUZO_ERR_ARG;
  const dim3 grid(static_cast<unsigned>(total_items / MUZO_ITEMS_PER_CTA));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  st = dispatch_dtype(param_dtype, [&](auto d) {
    constexpr int D = decltype(d)::value;
    rebuild_kept_linear_kernel<D><<<grid, kElemThreads, 0, s>>>(d_segs, nsegs, d_alphas, d_slot_base, horizon,
                                                               normalize, inv_coeff_sum, d_sums, d_flags);
  });
  if (st != MUZO_OK) return st;
  return launch_status();
}

int muzo_rebuild_segments(const muzo_segment* d_segs, int nsegs, int64_t total_items,
                          const uint64_t* d_keys, const float* d_alphas, int horizon, int dist,
                          int param_dtype, int normalize, float inv_coeff_sum, double* d_sums,
                          int32_t* d_flags, int max_ctas, void* stream) {
  if (nsegs == 0 || total_items == 0) return MUZO_OK;
  int st = check_table(d_segs, nsegs, total_items);
  if (st != MUZO_OK) return st;
  if (d_keys == nullptr || d_alphas == nullptr || d_sums == nullptr || d_flags == nullptr ||
      horizon <= 0 || (dist != MUZO_NORMAL && dist != MUZO_RADEMACHER))
    return MUZO_ERR_ARG;
  const int64_t nchunks = total_items / MUZO_ITEMS_PER_CTA;
  const int64_t ctas = (max_ctas > 0 && max_ctas < nchunks) ? max_ctas : nchunks;
  const dim3 grid(static_cast<unsigned>(ctas));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  st = dispatch_dtype(param_dtype, [&](auto d) {
    constexpr int D = decltype(d)::value;
    if (dist == MUZO_NORMAL)
      rebuild_kernel<MUZO_NORMAL, D><<<grid, kRebuildThreads, 0, s>>>(
          d_segs, nsegs, d_keys, d_alphas, horizon, normalize, inv_coeff_sum, d_sums, d_flags, nchunks);
    else
      rebuild_kernel<MUZO_RADEMACHER, D><<<grid, kRebuildThreads, 0, s>>>(
          d_segs, nsegs, d_keys, d_alphas, horizon, normalize, inv_coeff_sum, d_sums, d_flags, nchunks);
  });
  if (st != MUZO_OK) return st;
  return launch_status();
}

}  // extern "C"
