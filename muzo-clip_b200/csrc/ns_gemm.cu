// Newton-Schulz GEMMs for MuZO-Clip on sm_100a: tcgen05.mma with fp32 accumulators in TMEM,
// operands staged in shared memory by TMA tensor copies (each CTA fills only its own tiles), and the
// element-wise parts of the quintic iteration (newton_schulz.py:55-58) fused into the epilogue.
//
// Three kernels share the tile enumeration and the epilogue arithmetic: the wide CTA-pair kernel
// (256 x 512 tiles as two 256 x 256 halves, tcgen05.mma.cta_group::2 over two SMs; default when
// the output has >= 256 rows and >= 512 columns), the CTA-pair kernel (256 x 256 tiles; outputs
// of 256 x 256 and more with fewer than 512 columns) and the one-SM kernel below (128 x 256
// tiles; small outputs). Per flop, the pair kernel stages two thirds of the one-SM kernel's
// operand bytes from L2 (32 instead of 48 KB per SM and k-block of 64) and the wide kernel half
// (48 KB per SM for twice the flops), which is what keeps the tensor pipe fed. Output tiles of
// the pair kernels are handed out in order by an atomic counter kept in the caller's status
// buffer, so pairs delayed by other kernels on the GPU take fewer tiles.
//
// One-SM kernel: one persistent CTA per SM (grid = min(tiles, SMs)), 6 warps:
//   warp 0      TMA producer (one thread): A/B k-blocks into a 4-stage shared-memory ring;
//   warp 1      TMEM owner and MMA issuer (one thread): 128x256x16 bf16 MMAs into one of two
//               256-column TMEM accumulators, so the epilogue of tile i overlaps tile i+1;
//   warps 2..5  epilogue: tcgen05.ld 32 columns at a time, apply the fused op, store bf16.
// Every wait is bounded; on timeout the kernel records an error code, drains and returns.
#include <atomic>
#include <cstdlib>

#include "tcgen05_common.cuh"

namespace muzo {
namespace {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 64;                  // one 128-byte swizzle row of bf16
constexpr int UMMA_K = 16;
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;    // 16 KB
constexpr int B_BYTES = BN * BK * 2;    // 32 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int MN_CHUNK_BYTES = 64 * BK * 2;  // one 64(MN) x 64(K) box of an MN-major operand
constexpr int NUM_THREADS = 192;
constexpr int TMEM_COLS = 2 * BN;       // two accumulators of BN fp32 columns
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 512 /*barriers, flags*/;

using namespace tc;

// Descriptor of one UMMA_K slice (k-th, 16 elements) of a stage operand with `rows` MN rows.
// K-major tile: rows of 128 bytes (64 K elements), 8-row groups 1024 bytes apart; advancing K
// by 16 moves the start 32 bytes inside the swizzle atom. MN-major tile: boxes of 64 MN x 64 K
// (8 KB each) side by side along MN; K rows 128 bytes apart, 8-row groups 1024 bytes apart;
// advancing K by 16 moves the start 16 rows (2048 bytes).
template <bool MN_MAJOR>
__device__ __forceinline__ uint64_t operand_desc(uint32_t tile_base, int k) {
  if (MN_MAJOR) return make_sdesc(tile_base + k * (UMMA_K * 128), MN_CHUNK_BYTES, 1024);
  return make_sdesc(tile_base + k * (UMMA_K * 2), 16, 1024);
}

// Instruction descriptor of kind::f16: fp32 accumulator, bf16 A and B, majors, N and M.
__host__ __device__ constexpr uint32_t make_idesc(int m, int n, bool a_mn, bool b_mn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(a_mn) << 15) |
         (static_cast<uint32_t>(b_mn) << 16) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(m >> 4) << 24);
}

struct GemmArgs {
  int64_t m, n, k, batch;
  int tiles_m, tiles_n;
  int tile_m, tile_n;      // output tile of one CTA (1-SM kernel) or of one CTA pair (2-SM)
  int sym;                 // symmetric output: only tiles meeting the upper triangle, mirrored
  int m_fastest;           // tile order walks M first: the (larger) N-side operand streams once
  int64_t tiles_per_batch;
  int64_t num_tiles;
  int num_kb;
  __nv_bfloat16* d;
  int64_t ldd, d_bs;
  const __nv_bfloat16* e;
  float c1, c2;
  int32_t* status;
  int32_t* sched;          // CTA-pair kernel: [0] next tile, [1] pairs finished (zero between launches)
  // update epilogue of the last iteration: per batch index b, sums[b * MUZO_NSUMS + MUZO_SUM_U2]
  // += sum of (fp32(D) * scales[b])^2 and flags[b] |= MUZO_FLAG_NONFINITE_OUTPUT (null: off)
  double* sums;
  const float* scales;
  int32_t* flags;
};

// Stall request read from status word 3 at kernel start (test use), see kStallLimitCycles.

// Sum of squares of the stored (bf16-rounded) values times `scale`, in the order of the separate
// update_sumsq pass: an fp32 chain over each 8 values, added in fp64.
struct U2Acc {
  double sum = 0.0;
  bool finite = true;
  __device__ __forceinline__ void add8(const float* v, float scale, int count) {
    float p = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      if (k < count) {
        finite = finite && isfinite(v[k]);
        const float u = v[k] * scale;
        p = __fmaf_rn(u, u, p);
      }
    }
    sum += p;
  }
  // One atomic per warp and tile; `b` is the tile's batch index.
  __device__ __forceinline__ void flush(const GemmArgs& g, int64_t b, int lane) {
    const double t = warp_sum(sum);
    const bool all_finite = __all_sync(0xffffffffu, finite) != 0;
    if (lane == 0) {
      if (t != 0.0) atomicAdd(g.sums + b * MUZO_NSUMS + MUZO_SUM_U2, t);
      if (!all_finite) atomicOr(g.flags + b, MUZO_FLAG_NONFINITE_OUTPUT);
    }
    sum = 0.0;
    finite = true;
  }
};

// A chunk of 32 output columns the epilogue stores nothing for: outside the matrix, or strictly
// below the diagonal of a symmetric output (written there by the mirror of the upper triangle).
__device__ __forceinline__ bool chunk_skipped(const GemmArgs& g, int64_t row, int64_t col0) {
  return row >= g.m || col0 >= g.n || (g.sym && col0 + 31 < row);
}

// The epilogue's element-wise operand E (laid out like D) for one chunk of 32 columns, as 16
// packed bf16 pairs; zeros past the last column.
__device__ __forceinline__ void load_e_chunk(const GemmArgs& g, int64_t b, int64_t row, int64_t col0,
                                             uint32_t (&ew)[16]) {
  const int64_t base = b * g.d_bs + row * g.ldd + col0;
  if (col0 + 32 <= g.n) {
    const uint4* ep = reinterpret_cast<const uint4*>(g.e + base);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint4 u = ep[q];
      ew[4 * q] = u.x; ew[4 * q + 1] = u.y; ew[4 * q + 2] = u.z; ew[4 * q + 3] = u.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const uint32_t lo = col0 + 2 * i < g.n ? __bfloat16_as_ushort(g.e[base + 2 * i]) : 0u;
      const uint32_t hi = col0 + 2 * i + 1 < g.n ? __bfloat16_as_ushort(g.e[base + 2 * i + 1]) : 0u;
      ew[i] = lo | (hi << 16);
    }
  }
}

// Epilogue of one chunk of 32 accumulator columns with E already loaded (unused for the plain
// store).
template <int EPI>
__device__ __forceinline__ void epilogue_chunk_e(const GemmArgs& g, int64_t b, int64_t row, int64_t col0,
                                                 const uint32_t (&acc)[32], const uint32_t (&ew)[16], U2Acc& u2,
                                                 float u2_scale) {
  if (chunk_skipped(g, row, col0)) return;
  const int64_t base = b * g.d_bs + row * g.ldd + col0;
  float o[32];
  if (EPI == MUZO_EPI_STORE) {
#pragma unroll
    for (int i = 0; i < 32; ++i) o[i] = __uint_as_float(acc[i]);
  } else {
    float e[32];
#pragma unroll
    for (int h = 0; h < 16; ++h) { e[2 * h] = bf16_lo(ew[h]); e[2 * h + 1] = bf16_hi(ew[h]); }
    // roundings in pairs (one packed conversion per two values)
#pragma unroll
    for (int i = 0; i < 32; i += 2) {
      float a0 = __uint_as_float(acc[i]), a1 = __uint_as_float(acc[i + 1]);
      float t0 = g.c1 * e[i], t1 = g.c1 * e[i + 1];
      bf16r2(t0, t1);                                  // c1 * E, rounded to bf16
      bf16r2(a0, a1);                                  // bf16(A @ A) or bf16(B @ X)
      if (EPI == MUZO_EPI_POLY) {
        float u0 = g.c2 * a0, u1 = g.c2 * a1;
        bf16r2(u0, u1);                                // c2 * bf16(A @ A)
        o[i] = t0 + u0;
        o[i + 1] = t1 + u1;
      } else {
        o[i] = t0 + a0;                                // a*X + bf16(B @ X)
        o[i + 1] = t1 + a1;
      }
    }
  }
  if (g.sym) {
    // mirror (j, row) of every element with j >= row: for a fixed j the 32 lanes of a warp hold
    // 32 consecutive rows, so each mirrored store is one contiguous 64-byte run
    const int64_t mbase = b * g.d_bs + row;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int64_t j = col0 + i;
      if (j < g.n && j >= row) g.d[mbase + j * g.ldd] = __float2bfloat16_rn(o[i]);
    }
    if (col0 < row) {  // chunk crosses the diagonal: direct stores of its upper part only
      for (int i = 0; i < 32; ++i) {
        const int64_t j = col0 + i;
        if (j < g.n && j >= row) g.d[base + i] = __float2bfloat16_rn(o[i]);
      }
      return;
    }
  }
  if (col0 + 32 <= g.n) {
    uint4* dp = reinterpret_cast<uint4*>(g.d + base);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint4 u;
      u.x = pack_bf16(o[8 * q + 0], o[8 * q + 1]);
      u.y = pack_bf16(o[8 * q + 2], o[8 * q + 3]);
      u.z = pack_bf16(o[8 * q + 4], o[8 * q + 5]);
      u.w = pack_bf16(o[8 * q + 6], o[8 * q + 7]);
      dp[q] = u;
      if (EPI == MUZO_EPI_UPDATE && g.sums != nullptr) {
        const float r[8] = {bf16_lo(u.x), bf16_hi(u.x), bf16_lo(u.y), bf16_hi(u.y),
                            bf16_lo(u.z), bf16_hi(u.z), bf16_lo(u.w), bf16_hi(u.w)};
        u2.add8(r, u2_scale, 8);
      }
    }
  } else {
    for (int i = 0; i < 32 && col0 + i < g.n; ++i) g.d[base + i] = __float2bfloat16_rn(o[i]);
    if (EPI == MUZO_EPI_UPDATE && g.sums != nullptr) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float r[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) r[k] = bf16r(o[8 * q + k]);
        const int64_t left = g.n - (col0 + 8 * q);
        if (left > 0) u2.add8(r, u2_scale, left >= 8 ? 8 : static_cast<int>(left));
      }
    }
  }
}

template <int EPI>
__device__ __forceinline__ void epilogue_chunk(const GemmArgs& g, int64_t b, int64_t row, int64_t col0,
                                               const uint32_t (&acc)[32], U2Acc& u2, float u2_scale) {
  if (chunk_skipped(g, row, col0)) return;
  uint32_t ew[16];
  if (EPI != MUZO_EPI_STORE) load_e_chunk(g, b, row, col0, ew);
  epilogue_chunk_e<EPI>(g, b, row, col0, acc, ew, u2, u2_scale);
}

// Epilogue of one chunk of 32 columns from bf16-rounded accumulator pairs `ap` (16 words) and E
// pairs `ew` (16 words), eight values at a time: the same arithmetic, stores and sum-of-squares
// order as epilogue_chunk_e (whose first step rounds the accumulator to bf16 in pairs).
template <int EPI>
__device__ __forceinline__ void epilogue_chunk_packed(const GemmArgs& g, int64_t b, int64_t row, int64_t col0,
                                                      const uint32_t* ap, const uint32_t* ew, U2Acc& u2,
                                                      float u2_scale) {
  if (chunk_skipped(g, row, col0)) return;
  const int64_t base = b * g.d_bs + row * g.ldd + col0;
  const int64_t mbase = b * g.d_bs + row;
  const bool full = col0 + 32 <= g.n;
  const bool crosses = g.sym && col0 < row;  // chunk crosses the diagonal: upper part stored directly
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    float o[8];
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float a0 = bf16_lo(ap[4 * q + w]), a1 = bf16_hi(ap[4 * q + w]);
      if (EPI == MUZO_EPI_STORE) {
        o[2 * w] = a0;
        o[2 * w + 1] = a1;
      } else {
        float t0 = g.c1 * bf16_lo(ew[4 * q + w]), t1 = g.c1 * bf16_hi(ew[4 * q + w]);
        bf16r2(t0, t1);                                // c1 * E, rounded to bf16
        if (EPI == MUZO_EPI_POLY) {
          float u0 = g.c2 * a0, u1 = g.c2 * a1;
          bf16r2(u0, u1);                              // c2 * bf16(A @ A)
          o[2 * w] = t0 + u0;
          o[2 * w + 1] = t1 + u1;
        } else {
          o[2 * w] = t0 + a0;                          // a*X + bf16(B @ X)
          o[2 * w + 1] = t1 + a1;
        }
      }
    }
    if (g.sym) {
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int64_t j = col0 + 8 * q + k;
        if (j < g.n && j >= row) g.d[mbase + j * g.ldd] = __float2bfloat16_rn(o[k]);
      }
      if (crosses) {
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const int64_t j = col0 + 8 * q + k;
          if (j < g.n && j >= row) g.d[base + 8 * q + k] = __float2bfloat16_rn(o[k]);
        }
        continue;
      }
    }
    if (full) {
      uint4 u;
      u.x = pack_bf16(o[0], o[1]);
      u.y = pack_bf16(o[2], o[3]);
      u.z = pack_bf16(o[4], o[5]);
      u.w = pack_bf16(o[6], o[7]);
      reinterpret_cast<uint4*>(g.d + base)[q] = u;
      if (EPI == MUZO_EPI_UPDATE && g.sums != nullptr) {
        const float r[8] = {bf16_lo(u.x), bf16_hi(u.x), bf16_lo(u.y), bf16_hi(u.y),
                            bf16_lo(u.z), bf16_hi(u.z), bf16_lo(u.w), bf16_hi(u.w)};
        u2.add8(r, u2_scale, 8);
      }
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if (col0 + 8 * q + k < g.n) g.d[base + 8 * q + k] = __float2bfloat16_rn(o[k]);
      if (EPI == MUZO_EPI_UPDATE && g.sums != nullptr) {
        float r[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) r[k] = bf16r(o[k]);
        const int64_t left = g.n - (col0 + 8 * q);
        if (left > 0) u2.add8(r, u2_scale, left >= 8 ? 8 : static_cast<int>(left));
      }
    }
  }
}

// Tile t -> (batch, tile row, tile column). Symmetric outputs enumerate, per tile row tm, only
// the columns tn >= tm * tile_m / tile_n (tiles that hold an element on or above the diagonal).
__device__ __forceinline__ void tile_coords(const GemmArgs& g, int64_t t, int64_t& b, int& tm, int& tn) {
  b = t / g.tiles_per_batch;
  int64_t r = t - b * g.tiles_per_batch;
  if (!g.sym) {
    if (g.m_fastest) {
      tn = static_cast<int>(r / g.tiles_m);
      tm = static_cast<int>(r - static_cast<int64_t>(tn) * g.tiles_m);
    } else {
      tm = static_cast<int>(r / g.tiles_n);
      tn = static_cast<int>(r - static_cast<int64_t>(tm) * g.tiles_n);
    }
    return;
  }
  int row = 0;
  while (true) {
    const int64_t width = g.tiles_n - (row * g.tile_m) / g.tile_n;
    if (r < width) break;
    r -= width;
    ++row;
  }
  tm = row;
  tn = static_cast<int>((row * g.tile_m) / g.tile_n + r);
}

template <bool A_MN, bool B_MN, int EPI>
__global__ void __launch_bounds__(NUM_THREADS, 1)
ns_gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
               GemmArgs g) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* stall_bar = tempty + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(stall_bar + 1);
  int* abort_flag = reinterpret_cast<int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int stall = *reinterpret_cast<volatile int*>(g.status + 3);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) { mbar_init(full + s, 1); mbar_init(empty + s, 1); }
    for (int a = 0; a < 2; ++a) { mbar_init(tfull + a, 1); mbar_init(tempty + a, 4); }
    mbar_init(stall_bar, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_holder)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_a)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_b)) : "memory");
      int stage = 0;
      uint32_t phase = 0;
      bool ok = stall != kErrTimeoutProducer || mbar_wait(stall_bar, 0, kStallLimitCycles);
      uint32_t armed = 0;            // bit s: stage s received at least one load
      uint32_t armed_parity = 0;     // bit s: phase parity of the last load into stage s
      for (int64_t t = blockIdx.x; t < g.num_tiles && ok; t += gridDim.x) {
        int64_t b; int tm, tn;
        tile_coords(g, t, b, tm, tn);
        const int m0 = tm * BM, n0 = tn * BN, bz = static_cast<int>(b);
        for (int kb = 0; kb < g.num_kb; ++kb) {
          if (!mbar_wait(empty + stage, phase ^ 1)) { ok = false; break; }
          if (*reinterpret_cast<volatile int*>(abort_flag)) { ok = false; break; }
          uint8_t* sa = smem + stage * STAGE_BYTES;
          uint8_t* sb = sa + A_BYTES;
          mbar_arrive_expect_tx(full + stage, STAGE_BYTES);
          armed |= 1u << stage;
          armed_parity = (armed_parity & ~(1u << stage)) | (phase << stage);
          const int k0 = kb * BK;
          if (A_MN) {
#pragma unroll
            for (int c = 0; c < BM / 64; ++c) tma_load_3d(&map_a, full + stage, sa + c * MN_CHUNK_BYTES, m0 + 64 * c, k0, bz);
          } else {
            tma_load_3d(&map_a, full + stage, sa, k0, m0, bz);
          }
          if (B_MN) {
#pragma unroll
            for (int c = 0; c < BN / 64; ++c) tma_load_3d(&map_b, full + stage, sb + c * MN_CHUNK_BYTES, n0 + 64 * c, k0, bz);
          } else {
            tma_load_3d(&map_b, full + stage, sb, k0, n0, bz);
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      if (!ok) {
        atomicCAS(g.status, kErrNone, kErrTimeoutProducer);
        atomicExch(abort_flag, 1);
      }
      // Every load this thread issued must have landed before the CTA may exit (bounded).
      for (int s2 = 0; s2 < STAGES; ++s2)
        if (armed & (1u << s2)) mbar_wait(full + s2, (armed_parity >> s2) & 1u);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc(BM, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = stall != kErrTimeoutMma || mbar_wait(stall_bar, 0, kStallLimitCycles);
      int64_t local = 0;
      for (int64_t t = blockIdx.x; t < g.num_tiles && ok; t += gridDim.x, ++local) {
        const int acc = static_cast<int>(local & 1);
        const uint32_t acc_phase = static_cast<uint32_t>((local >> 1) & 1);
        if (!mbar_wait(tempty + acc, acc_phase ^ 1)) { ok = false; break; }
        tc_fence_after();
        const uint32_t tmem_d = tmem_base + acc * BN;
        for (int kb = 0; kb < g.num_kb; ++kb) {
          if (!mbar_wait(full + stage, phase)) { ok = false; break; }
          if (*reinterpret_cast<volatile int*>(abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * STAGE_BYTES);
          const uint32_t sb = sa + A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / UMMA_K; ++k) {
            umma_f16(tmem_d, operand_desc<A_MN>(sa, k), operand_desc<B_MN>(sb, k), idesc,
                     (kb > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit(empty + stage);  // frees the stage once these MMAs have read it
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        umma_commit(tfull + acc);      // accumulator ready for the epilogue
      }
      if (!ok) {
        atomicCAS(g.status, kErrNone, kErrTimeoutMma);
        atomicExch(abort_flag, 1);
      }
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------------- epilogue (warps 2..5)
    const int lane_base = 32 * (warp & 3);  // TMEM lanes this warp may access
    int64_t local = 0;
    bool ok = true;
    if (stall == kErrTimeoutEpilogue) {
      bool waited = true;
      if (lane == 0) waited = mbar_wait(stall_bar, 0, kStallLimitCycles);
      ok = __shfl_sync(0xffffffffu, waited ? 1 : 0, 0) != 0;
    }
    U2Acc u2;
    for (int64_t t = blockIdx.x; t < g.num_tiles && ok; t += gridDim.x, ++local) {
      int64_t b; int tm, tn;
      tile_coords(g, t, b, tm, tn);
      const int acc = static_cast<int>(local & 1);
      const uint32_t acc_phase = static_cast<uint32_t>((local >> 1) & 1);
      bool ready = true;
      if (lane == 0) ready = mbar_wait(tfull + acc, acc_phase);
      ready = __shfl_sync(0xffffffffu, ready ? 1 : 0, 0) != 0;
      if (!ready || *reinterpret_cast<volatile int*>(abort_flag)) { ok = ready; break; }
      tc_fence_after();
      const int64_t row = static_cast<int64_t>(tm) * BM + lane_base + lane;
      const float u2_scale = (EPI == MUZO_EPI_UPDATE && g.sums != nullptr) ? g.scales[b] : 0.0f;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(tmem_base + (static_cast<uint32_t>(lane_base) << 16) + acc * BN + c * 32, r);
        epilogue_chunk<EPI>(g, b, row, static_cast<int64_t>(tn) * BN + c * 32, r, u2, u2_scale);
      }
      if (EPI == MUZO_EPI_UPDATE && g.sums != nullptr) u2.flush(g, b, lane);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty + acc);
    }
    if (!ok && lane == 0) {
      atomicCAS(g.status, kErrNone, kErrTimeoutEpilogue);
      atomicExch(abort_flag, 1);
    }
  }

  // Drain: make sure every issued MMA has completed before TMEM is released. The last commit of
  // this CTA arrives on tfull of its last tile; an aborted CTA waits (bounded) on a fresh commit.
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    if (lane == 0 && *reinterpret_cast<volatile int*>(abort_flag)) {
      // drain outstanding MMAs of an aborted CTA: commit once more and wait (bounded)
      uint64_t* drain = tempty;  // reuse: re-init a barrier no longer in use
      mbar_init(drain, 1);
      asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
      umma_commit(drain);
      mbar_wait(drain, 0);
    }
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS)
                 : "memory");
  }
}

// ------------------------------------------------------------------ 2-SM (CTA pair) kernel
// A cluster of two CTAs computes a 256 x 256 output tile with tcgen05.mma.cta_group::2: each CTA
// stages its own 128 rows of A and 128 columns of B (32 KB per k-block instead of 48 KB for a
// 128 x 256 tile on one SM), the leader CTA issues the MMAs, and each CTA's TMEM holds its 128
// rows of the accumulator. Both CTAs' TMA loads complete on the leader's stage barrier and each
// fills only its own CTA's shared memory; one MMA commit signals the same barrier in both CTAs;
// both CTAs' epilogues release the accumulator on the leader's barrier.
constexpr int PM = 256, PN = 256, PHALF = 128;
constexpr int P_STAGES = 6;
constexpr int PA_BYTES = PHALF * BK * 2;   // 16 KB
constexpr int PB_BYTES = PHALF * BK * 2;   // 16 KB
constexpr int P_STAGE_BYTES = PA_BYTES + PB_BYTES;
constexpr int P_SMEM_BYTES = P_STAGES * P_STAGE_BYTES + 1024 + 512;
constexpr int TILE_SLOTS = 4;   // tile-index ring from the leader's producer to every other role
constexpr int TILE_READERS = 10;  // leader MMA + 4 epilogue warps per CTA + the peer's producer

// Tile ring: the leader's producer takes tile indices from a global counter (atomicAdd), so a
// pair that starts late or runs slower — SMs held by a concurrent kernel such as an NCCL
// transfer — simply takes fewer tiles. Slot k % TILE_SLOTS of both CTAs receives the index of the
// pair's k-th tile (-1 when the counter passed the last tile); every other role reads it there
// and releases the slot on the leader.
__device__ __forceinline__ void publish_tile(int* slot, uint64_t* full, int t) {
#pragma unroll
  for (uint32_t r = 0; r < 2; ++r) {
    asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(map_to_rank(smem_u32(slot), r)), "r"(t) : "memory");
    mbar_arrive_cluster(map_to_rank(smem_u32(full), r));
  }
}

// Wait for the pair's k-th tile index; false when the wait expired.
__device__ __forceinline__ bool read_tile(const int* slots, uint64_t* full, int64_t k, int& t) {
  const int s = static_cast<int>(k % TILE_SLOTS);
  if (!mbar_wait_cluster(full + s, static_cast<uint32_t>((k / TILE_SLOTS) & 1))) return false;
  t = *reinterpret_cast<const volatile int*>(slots + s);
  return true;
}

__device__ __forceinline__ void release_tile(uint64_t* empty, int64_t k) {
  mbar_arrive_cluster(map_to_rank(smem_u32(empty + k % TILE_SLOTS), 0));
}

template <bool A_MN, bool B_MN, int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NUM_THREADS, 1)
ns_gemm_pair_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                    GemmArgs g) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + P_STAGES * P_STAGE_BYTES);
  uint64_t* empty = full + P_STAGES;
  uint64_t* tfull = empty + P_STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* tile_full = drain + 1;
  uint64_t* tile_empty = tile_full + TILE_SLOTS;
  uint64_t* stall_bar = tile_empty + TILE_SLOTS;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(stall_bar + 1);
  int* abort_flag = reinterpret_cast<int*>(tmem_holder + 1);
  int* tile_slots = abort_flag + 1;
  // phases of each stage this CTA's producer loaded into (leader: armed), read by the leader
  // after both producers have stopped
  uint32_t* issued = reinterpret_cast<uint32_t*>(tile_slots + TILE_SLOTS);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int64_t npairs = gridDim.x >> 1;
  const int stall = *reinterpret_cast<volatile int*>(g.status + 3);

  if (threadIdx.x == 0) {
    for (int s = 0; s < P_STAGES; ++s) { mbar_init(full + s, 1); mbar_init(empty + s, 1); issued[s] = 0; }
    for (int a = 0; a < 2; ++a) { mbar_init(tfull + a, 1); mbar_init(tempty + a, 8); }
    for (int s = 0; s < TILE_SLOTS; ++s) { mbar_init(tile_full + s, 1); mbar_init(tile_empty + s, TILE_READERS); }
    mbar_init(drain, 1);
    mbar_init(stall_bar, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_holder)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  cluster_sync_all();  // barriers of both CTAs initialised, TMEM allocated
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer (both CTAs)
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_a)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_b)) : "memory");
      int stage = 0;
      uint32_t phase = 0;
      bool ok = !(leader && stall == kErrTimeoutProducer) || mbar_wait(stall_bar, 0, kStallLimitCycles);
      uint32_t count[P_STAGES] = {};         // phases loaded into (leader: armed) per stage
      for (int64_t k = 0; ok; ++k) {
        int t = -1;
        if (leader) {
          if (!mbar_wait(tile_empty + k % TILE_SLOTS, static_cast<uint32_t>(((k / TILE_SLOTS) & 1) ^ 1))) {
            ok = false;
            break;
          }
          t = atomicAdd(g.sched, 1);
          if (t >= g.num_tiles) t = -1;
          publish_tile(tile_slots + k % TILE_SLOTS, tile_full + k % TILE_SLOTS, t);
        } else {
          if (!read_tile(tile_slots, tile_full, k, t)) { ok = false; break; }
          release_tile(tile_empty, k);
        }
        if (t < 0) break;
        int64_t b; int tm, tn;
        tile_coords(g, t, b, tm, tn);
        const int m0 = tm * PM + static_cast<int>(rank) * PHALF;
        const int n0 = tn * PN + static_cast<int>(rank) * PHALF;
        const int bz = static_cast<int>(b);
        for (int kb = 0; kb < g.num_kb; ++kb) {
          if (!mbar_wait(empty + stage, phase ^ 1)) { ok = false; break; }
          if (*reinterpret_cast<volatile int*>(abort_flag)) { ok = false; break; }
          uint8_t* sa = smem + stage * P_STAGE_BYTES;
          uint8_t* sb = sa + PA_BYTES;
          const uint32_t bar = map_to_rank(smem_u32(full + stage), 0);
          if (leader) mbar_arrive_expect_tx_u32(smem_u32(full + stage), 2 * P_STAGE_BYTES);
#pragma unroll
          for (int s2 = 0; s2 < P_STAGES; ++s2) count[s2] += s2 == stage ? 1u : 0u;
          const int k0 = kb * BK;
          if (A_MN) {
#pragma unroll
            for (int c = 0; c < PHALF / 64; ++c) tma_load_3d_pair(&map_a, bar, sa + c * MN_CHUNK_BYTES, m0 + 64 * c, k0, bz);
          } else {
            tma_load_3d_pair(&map_a, bar, sa, k0, m0, bz);
          }
          if (B_MN) {
#pragma unroll
            for (int c = 0; c < PHALF / 64; ++c) tma_load_3d_pair(&map_b, bar, sb + c * MN_CHUNK_BYTES, n0 + 64 * c, k0, bz);
          } else {
            tma_load_3d_pair(&map_b, bar, sb, k0, n0, bz);
          }
          if (++stage == P_STAGES) { stage = 0; phase ^= 1; }
        }
      }
      if (!ok) { atomicCAS(g.status, kErrNone, kErrTimeoutProducer); pair_abort(abort_flag); }
      // the loads still in flight are waited for after both producers have stopped (below)
#pragma unroll
      for (int s2 = 0; s2 < P_STAGES; ++s2) issued[s2] = count[s2];
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer (leader only)
    if (lane == 0 && leader) {
      constexpr uint32_t idesc = make_idesc(PM, PN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = stall != kErrTimeoutMma || mbar_wait(stall_bar, 0, kStallLimitCycles);
      for (int64_t local = 0; ok; ++local) {
        int t = -1;
        if (!read_tile(tile_slots, tile_full, local, t)) { ok = false; break; }
        release_tile(tile_empty, local);
        if (t < 0) break;
        const int acc = static_cast<int>(local & 1);
        const uint32_t acc_phase = static_cast<uint32_t>((local >> 1) & 1);
        if (!mbar_wait(tempty + acc, acc_phase ^ 1)) { ok = false; break; }
        tc_fence_after();
        const uint32_t tmem_d = tmem_base + acc * BN;
        for (int kb = 0; kb < g.num_kb; ++kb) {
          if (!mbar_wait(full + stage, phase)) { ok = false; break; }
          if (*reinterpret_cast<volatile int*>(abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * P_STAGE_BYTES);
          const uint32_t sb = sa + PA_BYTES;
#pragma unroll
          for (int k = 0; k < BK / UMMA_K; ++k)
            umma_f16_pair(tmem_d, operand_desc<A_MN>(sa, k), operand_desc<B_MN>(sb, k), idesc,
                          (kb > 0 || k > 0) ? 1u : 0u);
          umma_commit_pair(empty + stage);  // frees this stage in both CTAs
          if (++stage == P_STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        umma_commit_pair(tfull + acc);      // accumulator ready in both CTAs
      }
      if (!ok) { atomicCAS(g.status, kErrNone, kErrTimeoutMma); pair_abort(abort_flag); }
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------------- epilogue (both CTAs)
    const int lane_base = 32 * (warp & 3);
    const uint32_t leader_tempty0 = map_to_rank(smem_u32(tempty), 0);
    bool ok = true;
    if (stall == kErrTimeoutEpilogue) {
      bool waited = true;
      if (lane == 0) waited = mbar_wait(stall_bar, 0, kStallLimitCycles);
      ok = __shfl_sync(0xffffffffu, waited ? 1 : 0, 0) != 0;
    }
    U2Acc u2;
    for (int64_t local = 0; ok; ++local) {
      int t = -1;
      bool got = true;
      if (lane == 0) {
        got = read_tile(tile_slots, tile_full, local, t);
        if (got) release_tile(tile_empty, local);
      }
      got = __shfl_sync(0xffffffffu, got ? 1 : 0, 0) != 0;
      t = __shfl_sync(0xffffffffu, t, 0);
      if (!got) { ok = false; break; }
      if (t < 0) break;
      int64_t b; int tm, tn;
      tile_coords(g, t, b, tm, tn);
      const int acc = static_cast<int>(local & 1);
      const uint32_t acc_phase = static_cast<uint32_t>((local >> 1) & 1);
      bool ready = true;
      if (lane == 0) ready = mbar_wait(tfull + acc, acc_phase);
      ready = __shfl_sync(0xffffffffu, ready ? 1 : 0, 0) != 0;
      if (!ready || *reinterpret_cast<volatile int*>(abort_flag)) { ok = ready; break; }
      tc_fence_after();
      const int64_t row = static_cast<int64_t>(tm) * PM + static_cast<int64_t>(rank) * PHALF + lane_base + lane;
      const float u2_scale = (EPI == MUZO_EPI_UPDATE && g.sums != nullptr) ? g.scales[b] : 0.0f;
#pragma unroll 1
      for (int c = 0; c < PN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(tmem_base + (static_cast<uint32_t>(lane_base) << 16) + acc * BN + c * 32, r);
        epilogue_chunk<EPI>(g, b, row, static_cast<int64_t>(tn) * PN + c * 32, r, u2, u2_scale);
      }
      if (EPI == MUZO_EPI_UPDATE && g.sums != nullptr) u2.flush(g, b, lane);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(leader_tempty0 + acc * 8);
    }
    if (!ok && lane == 0) { atomicCAS(g.status, kErrNone, kErrTimeoutEpilogue); pair_abort(abort_flag); }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // both CTAs past their loops: the abort flag and the load records are final
  if (warp == 0 && leader && lane == 0) {
    // Every load of both CTAs counts on the leader's stage barriers, and both CTAs must outlive
    // them. A producer loads a stage's phase only once the previous phase was consumed, which
    // needs both CTAs' loads, so the two records differ by at most one phase per stage: after an
    // abort, the leader supplies the missing arrival (a phase the peer loaded but the leader did
    // not arm) or the missing bytes (a phase the leader armed but the peer did not load) so that
    // every phase with a load in flight completes, then waits for it (bounded).
    const uint32_t peer = map_to_rank(smem_u32(issued), 1);
    for (int s2 = 0; s2 < P_STAGES; ++s2) {
      uint32_t np;
      asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(np) : "r"(peer + 4u * s2) : "memory");
      const uint32_t nl = issued[s2];
      if (np == nl + 1) mbar_arrive_expect_tx_u32(smem_u32(full + s2), P_STAGE_BYTES);
      else if (nl == np + 1) mbar_complete_tx(full + s2, P_STAGE_BYTES);
      const uint32_t n = np > nl ? np : nl;
      if (n > 0) mbar_wait(full + s2, (n - 1) & 1u);
    }
  }
  if (warp == 1 && leader && lane == 0 && *reinterpret_cast<volatile int*>(abort_flag)) {
    // an aborted pair drains its in-flight MMAs before the accumulators are released (bounded)
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(drain))
                 : "memory");
    mbar_wait(drain, 0);
  }
  cluster_sync_all();  // no CTA leaves while its peer may still signal its barriers
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS) : "memory");
  }
  if (leader && threadIdx.x == 0) {
    // the last pair to finish (every pair has taken its final index by now) rewinds the counter
    // for the next launch that uses this status buffer
    __threadfence();
    if (atomicAdd(g.sched + 1, 1) == static_cast<int>(npairs) - 1) {
      atomicExch(g.sched, 0);
      atomicExch(g.sched + 1, 0);
    }
  }
}

// ------------------------------------------------------------------ wide CTA-pair kernel
// A pair computes a 256 x 512 output tile as two 256 x 256 halves (two tcgen05.mma.cta_group::2
// per K step into two accumulators that fill all 512 TMEM columns): each CTA stages its 128 rows
// of A once for both halves, so a k-block moves 48 KB per SM for twice the flops of the 32 KB
// k-block of the 256 x 256 tile — 48 instead of 64 bytes from L2 per 128 x 256 x 16 MMA step,
// which is what the L2-to-SM path sustains next to full tensor-pipe rate.
//
// With TMEM full, tile i+1 can only start where tile i has been drained, so the MMA issuer
// reorders the first and last W_EDGE k-blocks of each tile: the tail issues the half-0 MMAs of
// its last k-blocks first and signals half 0 ready, then their half-1 MMAs; the head of the next
// tile issues its first k-blocks' half-0 MMAs as soon as the epilogue has released half 0, and
// their half-1 MMAs once half 1 is released. Stages of those k-blocks are released after both
// halves have read them. Eight epilogue warps per CTA (two per TMEM lane quarter, 128 columns of
// each half apiece) load the fused operand E before the accumulator is ready and release each
// half as soon as its last TMEM load has completed.
//
// Epilogue traffic goes through TMA: each epilogue warp owns two 2 KB shared-memory boxes of
// 32 x 32 bf16 (64-byte swizzle). E of the warp's next 32-column chunk is loaded into one by a
// TMA load issued ahead of time; the chunk's result is written into the other and stored by a
// TMA store, so rows of 64 bytes leave as whole lines instead of one 16-byte piece per thread
// and row. Symmetric outputs mirror through the same box: the transposed block is read out of it
// column by column and stored by a second TMA store; a diagonal block is made symmetric there.
//
// Symmetric outputs: a tile whose left half lies strictly below the diagonal computes only its
// right half; columns past the matrix likewise drop a half.
constexpr int WN = 512;
constexpr int W_STAGES = 4;
constexpr int WB_HALF_BYTES = PHALF * BK * 2;                      // 16 KB: one half's B columns of a CTA
constexpr int W_STAGE_BYTES = PA_BYTES + 2 * WB_HALF_BYTES;        // 48 KB
constexpr int W_THREADS = 320;   // warp 0 producer, warp 1 MMA issuer, warps 2..9 epilogue
constexpr int W_EPI_WARPS = 8;
constexpr int W_EPI_BOX = 32 * 32 * 2;                             // one 32 x 32 bf16 box
constexpr int W_EPI_BYTES = W_EPI_WARPS * 2 * W_EPI_BOX;           // 32 KB: an E box and a D box per warp
constexpr int W_SMEM_BYTES = W_STAGES * W_STAGE_BYTES + W_EPI_BYTES + 1024 + 512;
constexpr int W_TILE_READERS = 1 + 2 * W_EPI_WARPS + 1;  // leader MMA + both CTAs' epilogues + peer producer
constexpr int W_EDGE = 2;        // k-blocks reordered at each end of a tile

// Byte offset of 16-byte unit u of row r in a 32 x 32 bf16 box staged with the 64-byte TMA
// swizzle (address bits 5:4 XOR bits 8:7); box bases are 512-byte aligned.
__device__ __forceinline__ uint32_t sw64(int r, int u) {
  return static_cast<uint32_t>(r * 64 + ((u ^ ((r >> 1) & 3)) << 4));
}

// Results of one chunk of 32 columns as bf16 pairs, from bf16-rounded accumulator pairs `ap` and
// E pairs `ew`: the arithmetic of epilogue_chunk_e (whose first step rounds the accumulator).
template <int EPI>
__device__ __forceinline__ void chunk_results(const GemmArgs& g, const uint32_t* ap, const uint32_t* ew,
                                              uint32_t (&out)[16]) {
#pragma unroll
  for (int w = 0; w < 16; ++w) {
    if (EPI == MUZO_EPI_STORE) {
      out[w] = ap[w];
    } else {
      const float a0 = bf16_lo(ap[w]), a1 = bf16_hi(ap[w]);
      float t0 = g.c1 * bf16_lo(ew[w]), t1 = g.c1 * bf16_hi(ew[w]);
      bf16r2(t0, t1);                                  // c1 * E, rounded to bf16
      if (EPI == MUZO_EPI_POLY) {
        float u0 = g.c2 * a0, u1 = g.c2 * a1;
        bf16r2(u0, u1);                                // c2 * bf16(A @ A)
        out[w] = pack_bf16(t0 + u0, t1 + u1);
      } else {
        out[w] = pack_bf16(t0 + a0, t1 + a1);          // a*X + bf16(B @ X)
      }
    }
  }
}

// Halves of tile (tm, tn) that hold an output element: bit h for columns [512 tn + 256 h, +256).
__device__ __forceinline__ int wide_halves(const GemmArgs& g, int tm, int tn) {
  int mask = 0;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int64_t lo = static_cast<int64_t>(tn) * WN + 256 * h;
    if (lo >= g.n) continue;
    if (g.sym && lo + 255 < static_cast<int64_t>(tm) * PM) continue;
    mask |= 1 << h;
  }
  return mask;
}

template <bool A_MN, bool B_MN, int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(W_THREADS, 1)
ns_gemm_wide_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                    const __grid_constant__ CUtensorMap map_d, const __grid_constant__ CUtensorMap map_e, GemmArgs g) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint8_t* epi_smem = smem + W_STAGES * W_STAGE_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(epi_smem + W_EPI_BYTES);
  uint64_t* empty = full + W_STAGES;
  uint64_t* tfull = empty + W_STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* tile_full = drain + 1;
  uint64_t* tile_empty = tile_full + TILE_SLOTS;
  uint64_t* stall_bar = tile_empty + TILE_SLOTS;
  uint64_t* ebars = stall_bar + 1;  // per epilogue warp: its E box loaded
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(ebars + W_EPI_WARPS);
  int* abort_flag = reinterpret_cast<int*>(tmem_holder + 1);
  int* tile_slots = abort_flag + 1;
  // per stage: phases this CTA's producer loaded into (leader: armed), and the bytes this CTA
  // loaded for the last of them; read by the leader after both producers have stopped
  uint32_t* issued = reinterpret_cast<uint32_t*>(tile_slots + TILE_SLOTS);
  uint32_t* issued_bytes = issued + W_STAGES;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int64_t npairs = gridDim.x >> 1;
  const int stall = *reinterpret_cast<volatile int*>(g.status + 3);

  if (threadIdx.x == 0) {
    for (int s = 0; s < W_STAGES; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
      issued[s] = 0;
      issued_bytes[s] = 0;
    }
    for (int a = 0; a < 2; ++a) { mbar_init(tfull + a, 1); mbar_init(tempty + a, 2 * W_EPI_WARPS); }
    for (int s = 0; s < TILE_SLOTS; ++s) { mbar_init(tile_full + s, 1); mbar_init(tile_empty + s, W_TILE_READERS); }
    for (int w = 0; w < W_EPI_WARPS; ++w) mbar_init(ebars + w, 1);
    mbar_init(drain, 1);
    mbar_init(stall_bar, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_holder)),
                 "r"(512)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  cluster_sync_all();  // barriers of both CTAs initialised, TMEM allocated
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer (both CTAs)
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_a)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_b)) : "memory");
      int stage = 0;
      uint32_t phase = 0;
      bool ok = !(leader && stall == kErrTimeoutProducer) || mbar_wait(stall_bar, 0, kStallLimitCycles);
      uint32_t count[W_STAGES] = {};
      uint32_t bytes_of[W_STAGES] = {};
      for (int64_t k = 0; ok; ++k) {
        int t = -1;
        if (leader) {
          if (!mbar_wait(tile_empty + k % TILE_SLOTS, static_cast<uint32_t>(((k / TILE_SLOTS) & 1) ^ 1))) {
            ok = false;
            break;
          }
          t = atomicAdd(g.sched, 1);
          if (t >= g.num_tiles) t = -1;
          publish_tile(tile_slots + k % TILE_SLOTS, tile_full + k % TILE_SLOTS, t);
        } else {
          if (!read_tile(tile_slots, tile_full, k, t)) { ok = false; break; }
          release_tile(tile_empty, k);
        }
        if (t < 0) break;
        int64_t b; int tm, tn;
        tile_coords(g, t, b, tm, tn);
        const int mask = wide_halves(g, tm, tn);
        const uint32_t cta_bytes = PA_BYTES + WB_HALF_BYTES * static_cast<uint32_t>(__popc(mask));
        const int m0 = tm * PM + static_cast<int>(rank) * PHALF;
        const int bz = static_cast<int>(b);
        for (int kb = 0; kb < g.num_kb; ++kb) {
          if (!mbar_wait(empty + stage, phase ^ 1)) { ok = false; break; }
          if (*reinterpret_cast<volatile int*>(abort_flag)) { ok = false; break; }
          uint8_t* sa = smem + stage * W_STAGE_BYTES;
          const uint32_t bar = map_to_rank(smem_u32(full + stage), 0);
          if (leader) mbar_arrive_expect_tx_u32(smem_u32(full + stage), 2 * cta_bytes);
#pragma unroll
          for (int s2 = 0; s2 < W_STAGES; ++s2) {
            count[s2] += s2 == stage ? 1u : 0u;
            bytes_of[s2] = s2 == stage ? cta_bytes : bytes_of[s2];
          }
          const int k0 = kb * BK;
          if (A_MN) {
#pragma unroll
            for (int c = 0; c < PHALF / 64; ++c) tma_load_3d_pair(&map_a, bar, sa + c * MN_CHUNK_BYTES, m0 + 64 * c, k0, bz);
          } else {
            tma_load_3d_pair(&map_a, bar, sa, k0, m0, bz);
          }
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            if (!((mask >> h) & 1)) continue;
            uint8_t* sb = sa + PA_BYTES + h * WB_HALF_BYTES;
            const int n0 = tn * WN + 256 * h + static_cast<int>(rank) * PHALF;
            if (B_MN) {
#pragma unroll
              for (int c = 0; c < PHALF / 64; ++c) tma_load_3d_pair(&map_b, bar, sb + c * MN_CHUNK_BYTES, n0 + 64 * c, k0, bz);
            } else {
              tma_load_3d_pair(&map_b, bar, sb, k0, n0, bz);
            }
          }
          if (++stage == W_STAGES) { stage = 0; phase ^= 1; }
        }
      }
      if (!ok) { atomicCAS(g.status, kErrNone, kErrTimeoutProducer); pair_abort(abort_flag); }
#pragma unroll
      for (int s2 = 0; s2 < W_STAGES; ++s2) { issued[s2] = count[s2]; issued_bytes[s2] = bytes_of[s2]; }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer (leader only)
    if (lane == 0 && leader) {
      constexpr uint32_t idesc = make_idesc(PM, 256, A_MN, B_MN);
      int64_t done = 0;  // k-blocks consumed by earlier tiles: k-block j of this tile is ring slot done + j
      bool ok = stall != kErrTimeoutMma || mbar_wait(stall_bar, 0, kStallLimitCycles);
      for (int64_t local = 0; ok; ++local) {
        int t = -1;
        if (!read_tile(tile_slots, tile_full, local, t)) { ok = false; break; }
        release_tile(tile_empty, local);
        if (t < 0) break;
        int64_t b; int tm, tn;
        tile_coords(g, t, b, tm, tn);
        const int mask = wide_halves(g, tm, tn);
        const uint32_t tphase = static_cast<uint32_t>(local & 1);  // tfull / tempty complete once per tile
        const int nk = g.num_kb;
        const int edge = nk >= 2 * W_EDGE ? W_EDGE : 0;
        // wait for stage j's operands (false: expired or aborted)
        auto wait_full = [&](int j) -> bool {
          const int64_t q = done + j;
          if (!mbar_wait(full + q % W_STAGES, static_cast<uint32_t>((q / W_STAGES) & 1))) return false;
          if (*reinterpret_cast<volatile int*>(abort_flag)) return false;
          tc_fence_after();
          return true;
        };
        auto issue = [&](int j, int h) {
          if (!((mask >> h) & 1)) return;
          const uint32_t sa = smem_u32(smem + ((done + j) % W_STAGES) * W_STAGE_BYTES);
          const uint32_t sb = sa + PA_BYTES + h * WB_HALF_BYTES;
#pragma unroll
          for (int k = 0; k < BK / UMMA_K; ++k)
            umma_f16_pair(tmem_base + 256 * h, operand_desc<A_MN>(sa, k), operand_desc<B_MN>(sb, k), idesc,
                          (j > 0 || k > 0) ? 1u : 0u);
        };
        auto release = [&](int j) { umma_commit_pair(empty + (done + j) % W_STAGES); };
        if (!mbar_wait(tempty + 0, tphase ^ 1)) { ok = false; break; }
        tc_fence_after();
        // head: half 0 of the first `edge` k-blocks, then half 1 of them once it is released
        for (int j = 0; j < edge && ok; ++j) {
          if (!wait_full(j)) { ok = false; break; }
          issue(j, 0);
        }
        if (!ok) break;
        if (!mbar_wait(tempty + 1, tphase ^ 1)) { ok = false; break; }
        tc_fence_after();
        for (int j = 0; j < edge; ++j) issue(j, 1);
        for (int j = 0; j < edge; ++j) release(j);
        // middle: both halves per k-block
        for (int j = edge; j < nk - edge && ok; ++j) {
          if (!wait_full(j)) { ok = false; break; }
          issue(j, 0);
          issue(j, 1);
          release(j);
        }
        if (!ok) break;
        // tail: half 0 of the last `edge` k-blocks and its ready signal, then their half 1
        for (int j = nk - edge; j < nk && ok; ++j) {
          if (!wait_full(j)) { ok = false; break; }
          issue(j, 0);
        }
        if (!ok) break;
        umma_commit_pair(tfull + 0);
        for (int j = nk - edge; j < nk; ++j) issue(j, 1);
        for (int j = nk - edge; j < nk; ++j) release(j);
        umma_commit_pair(tfull + 1);
        done += nk;
      }
      if (!ok) { atomicCAS(g.status, kErrNone, kErrTimeoutMma); pair_abort(abort_flag); }
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------------- epilogue (both CTAs)
    const int quarter = warp & 3;                 // TMEM lanes 32 * quarter .. + 32
    const int col_part = (warp - 2) >> 2;         // columns 128 * col_part .. + 128 of each half
    const uint32_t lane_addr = static_cast<uint32_t>(32 * quarter) << 16;
    const uint32_t leader_tempty = map_to_rank(smem_u32(tempty), 0);
    uint8_t* ebox = epi_smem + (warp - 2) * (2 * W_EPI_BOX);
    uint8_t* dbox = ebox + W_EPI_BOX;
    uint64_t* ebar = ebars + (warp - 2);
    uint32_t ephase = 0;
    bool e_pending = false;
    bool ok = true;
    if (stall == kErrTimeoutEpilogue) {
      bool waited = true;
      if (lane == 0) waited = mbar_wait(stall_bar, 0, kStallLimitCycles);
      ok = __shfl_sync(0xffffffffu, waited ? 1 : 0, 0) != 0;
    }
    U2Acc u2;
    for (int64_t local = 0; ok; ++local) {
      int t = -1;
      bool got = true;
      if (lane == 0) {
        got = read_tile(tile_slots, tile_full, local, t);
        if (got) release_tile(tile_empty, local);
      }
      got = __shfl_sync(0xffffffffu, got ? 1 : 0, 0) != 0;
      t = __shfl_sync(0xffffffffu, t, 0);
      if (!got) { ok = false; break; }
      if (t < 0) break;
      int64_t b; int tm, tn;
      tile_coords(g, t, b, tm, tn);
      const int mask = wide_halves(g, tm, tn);
      const uint32_t tphase = static_cast<uint32_t>(local & 1);
      const int r0 = tm * PM + static_cast<int>(rank) * PHALF + 32 * quarter;  // the warp's first row
      const int64_t row = r0 + lane;
      const float u2_scale = (EPI == MUZO_EPI_UPDATE && g.sums != nullptr) ? g.scales[b] : 0.0f;
      // chunk s = 4 h + c of this warp: columns c0(s) .. + 32 of half h; live when it holds an
      // element the epilogue stores (warp-uniform)
      auto c0_of = [&](int s) -> int { return tn * WN + 256 * (s >> 2) + 128 * col_part + 32 * (s & 3); };
      auto live = [&](int s) -> bool {
        if (((mask >> (s >> 2)) & 1) == 0) return false;
        const int c0 = c0_of(s);
        return r0 < g.m && c0 < g.n && !(g.sym && c0 < r0);
      };
      // TMA load of E for the first live chunk at or after `from` (lane 0 issues)
      auto issue_e = [&](int from) {
        if constexpr (EPI != MUZO_EPI_STORE) {
          for (int s2 = from; s2 < 8; ++s2) {
            if (!live(s2)) continue;
            if (lane == 0) {
              mbar_arrive_expect_tx(ebar, W_EPI_BOX);
              tma_load_3d(&map_e, ebar, ebox, c0_of(s2), r0, static_cast<int>(b));
            }
            e_pending = true;
            return;
          }
        }
      };
      issue_e(0);
      bool stop = false;
#pragma unroll 1
      for (int h = 0; h < 2 && !stop; ++h) {
        const bool active = ((mask >> h) & 1) != 0;
        bool ready = true;
        if (lane == 0) ready = mbar_wait(tfull + h, tphase);
        ready = __shfl_sync(0xffffffffu, ready ? 1 : 0, 0) != 0;
        if (!ready || *reinterpret_cast<volatile int*>(abort_flag)) { ok = ready; stop = true; break; }
        tc_fence_after();
        if (!active) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(leader_tempty + h * 8);
          continue;
        }
        // the warp's 128 columns of this half in one TMEM load; the half is released before any
        // other work and the values are rounded to bf16 pairs (every epilogue's first step)
        uint32_t accp[64];
        {
          uint32_t r[128];
          tmem_ld128(tmem_base + lane_addr + 256 * h + 128 * col_part, r);
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(leader_tempty + h * 8);
#pragma unroll
          for (int i = 0; i < 64; ++i) accp[i] = pack_bf16(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1]));
        }
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int s2 = 4 * h + c;
          if (!live(s2)) continue;
          const int c0 = c0_of(s2);
          uint32_t ew[16];
          if (EPI != MUZO_EPI_STORE) {
            bool landed = true;
            if (lane == 0) landed = mbar_wait(ebar, ephase);
            landed = __shfl_sync(0xffffffffu, landed ? 1 : 0, 0) != 0;
            if (!landed) { ok = false; stop = true; break; }
            ephase ^= 1;
            e_pending = false;
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const uint4 v = *reinterpret_cast<const uint4*>(ebox + sw64(lane, u));
              ew[4 * u] = v.x; ew[4 * u + 1] = v.y; ew[4 * u + 2] = v.z; ew[4 * u + 3] = v.w;
            }
            // The next E box is written by the TMA unit (async proxy) over these plain shared
            // loads, which a warp barrier alone does not wait for: a late load once returned the
            // next chunk's values. A store that depends on every load issues only after all of
            // them have landed (it writes into this lane's own row of the box, which the next
            // load overwrites), and the proxy fence orders it before the async write.
            *reinterpret_cast<volatile uint32_t*>(ebox + sw64(lane, 0)) = ew[3] ^ ew[7] ^ ew[11] ^ ew[15];
            fence_proxy_async_smem();
            __syncwarp();
            issue_e(s2 + 1);
          }
          uint32_t out[16];
          chunk_results<EPI>(g, accp + 16 * c, ew, out);
          if (EPI == MUZO_EPI_UPDATE && g.sums != nullptr && row < g.m) {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const int left = g.n - (c0 + 8 * q) < 8 ? static_cast<int>(g.n - (c0 + 8 * q)) : 8;
              const float v8[8] = {bf16_lo(out[4 * q]), bf16_hi(out[4 * q]), bf16_lo(out[4 * q + 1]),
                                   bf16_hi(out[4 * q + 1]), bf16_lo(out[4 * q + 2]), bf16_hi(out[4 * q + 2]),
                                   bf16_lo(out[4 * q + 3]), bf16_hi(out[4 * q + 3])};
              if (left > 0) u2.add8(v8, u2_scale, left);
            }
          }
          // this lane's row into the D box once the previous store has read it
          if (lane == 0) bulk_wait_read_all();
          __syncwarp();
#pragma unroll
          for (int u = 0; u < 4; ++u)
            *reinterpret_cast<uint4*>(dbox + sw64(lane, u)) = make_uint4(out[4 * u], out[4 * u + 1], out[4 * u + 2],
                                                                        out[4 * u + 3]);
          if (g.sym) {
            // column `lane` of the block: element (j, lane) of every row j
            __syncwarp();
            uint32_t col[16];
#pragma unroll
            for (int k = 0; k < 16; ++k) {
              const uint32_t lo = *reinterpret_cast<const uint16_t*>(dbox + sw64(2 * k, lane >> 3) + (lane & 7) * 2);
              const uint32_t hi = *reinterpret_cast<const uint16_t*>(dbox + sw64(2 * k + 1, lane >> 3) + (lane & 7) * 2);
              col[k] = lo | (hi << 16);
            }
            __syncwarp();
            if (c0 == r0) {
              // diagonal block: row `lane` keeps its elements on and above the diagonal and takes
              // the mirror of the upper triangle below it
#pragma unroll
              for (int k = 0; k < 16; ++k) {
                const uint32_t lo = 2 * k >= lane ? (out[k] & 0xffffu) : (col[k] & 0xffffu);
                const uint32_t hi = 2 * k + 1 >= lane ? (out[k] & 0xffff0000u) : (col[k] & 0xffff0000u);
                out[k] = lo | hi;
              }
#pragma unroll
              for (int u = 0; u < 4; ++u)
                *reinterpret_cast<uint4*>(dbox + sw64(lane, u)) = make_uint4(out[4 * u], out[4 * u + 1],
                                                                            out[4 * u + 2], out[4 * u + 3]);
              fence_proxy_async_smem();
              __syncwarp();
              if (lane == 0) { tma_store_3d(&map_d, dbox, c0, r0, static_cast<int>(b)); bulk_commit(); }
              continue;
            }
            // above the diagonal: the block, then its transpose at the mirrored position
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              tma_store_3d(&map_d, dbox, c0, r0, static_cast<int>(b));
              bulk_commit();
              bulk_wait_read_all();
            }
            __syncwarp();
#pragma unroll
            for (int u = 0; u < 4; ++u)
              *reinterpret_cast<uint4*>(dbox + sw64(lane, u)) = make_uint4(col[4 * u], col[4 * u + 1], col[4 * u + 2],
                                                                          col[4 * u + 3]);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) { tma_store_3d(&map_d, dbox, r0, c0, static_cast<int>(b)); bulk_commit(); }
            continue;
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) { tma_store_3d(&map_d, dbox, c0, r0, static_cast<int>(b)); bulk_commit(); }
        }
      }
      if (stop) break;
      if (EPI == MUZO_EPI_UPDATE && g.sums != nullptr) u2.flush(g, b, lane);
    }
    // no TMA load may still be writing this warp's box, and every store has completed
    if (lane == 0) {
      if (e_pending) mbar_wait(ebar, ephase);
      bulk_wait_all();
    }
    __syncwarp();
    if (!ok && lane == 0) { atomicCAS(g.status, kErrNone, kErrTimeoutEpilogue); pair_abort(abort_flag); }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // both CTAs past their loops: the abort flag and the load records are final
  if (warp == 0 && leader && lane == 0) {
    // Every load of both CTAs counts on the leader's stage barriers (see the 256 x 256 kernel):
    // after an abort the leader supplies a missing arrival or the missing bytes of the last phase
    // of each stage (both CTAs load the same bytes for a phase) and waits for it (bounded).
    const uint32_t peer = map_to_rank(smem_u32(issued), 1);
    const uint32_t peer_bytes = map_to_rank(smem_u32(issued_bytes), 1);
    for (int s2 = 0; s2 < W_STAGES; ++s2) {
      uint32_t np, nbytes;
      asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(np) : "r"(peer + 4u * s2) : "memory");
      asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(nbytes) : "r"(peer_bytes + 4u * s2) : "memory");
      const uint32_t nl = issued[s2];
      if (np == nl + 1) mbar_arrive_expect_tx_u32(smem_u32(full + s2), nbytes);
      else if (nl == np + 1) mbar_complete_tx(full + s2, issued_bytes[s2]);
      const uint32_t n = np > nl ? np : nl;
      if (n > 0) mbar_wait(full + s2, (n - 1) & 1u);
    }
  }
  if (warp == 1 && leader && lane == 0 && *reinterpret_cast<volatile int*>(abort_flag)) {
    // an aborted pair drains its in-flight MMAs before the accumulators are released (bounded)
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(drain))
                 : "memory");
    mbar_wait(drain, 0);
  }
  cluster_sync_all();  // no CTA leaves while its peer may still signal its barriers
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(512) : "memory");
  }
  if (leader && threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(g.sched + 1, 1) == static_cast<int>(npairs) - 1) {
      atomicExch(g.sched, 0);
      atomicExch(g.sched + 1, 0);
    }
  }
}

// ------------------------------------------------------------------ host side

// 3-D bf16 tensor map over [batch][rows][inner] with leading dim `ld` and batch stride `bs`
// (elements); box = box_inner x box_rows x 1 with 128-byte swizzle and zero fill out of bounds.
int encode_map(CUtensorMap* map, const void* base, int64_t inner, int64_t rows, int64_t batch, int64_t ld,
               int64_t bs, int box_inner, int box_rows,
               CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  auto fn = encode_fn();
  if (fn == nullptr) return MUZO_ERR_UNSUPPORTED;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(rows),
                        static_cast<cuuint64_t>(batch)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(ld * 2), static_cast<cuuint64_t>(bs * 2)};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(box_inner), static_cast<cuuint32_t>(box_rows), 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box,
                  estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? MUZO_OK : MUZO_ERR_ARG;
}

template <bool A_MN, bool B_MN, int EPI>
int launch_gemm(const CUtensorMap& ma, const CUtensorMap& mb, const GemmArgs& g, cudaStream_t s) {
  auto kern = ns_gemm_kernel<A_MN, B_MN, EPI>;
  static std::atomic<bool> configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev].load(std::memory_order_acquire)) {
    MUZO_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
    configured[dev].store(true, std::memory_order_release);
  }
  int64_t grid = g.num_tiles < device_sm_count() ? g.num_tiles : device_sm_count();
  kern<<<static_cast<unsigned>(grid), NUM_THREADS, SMEM_BYTES, s>>>(ma, mb, g);
  return launch_status();
}

// CTA-pair launch: grid = 2 x min(tiles, co-resident pairs). The number of pairs the device can
// hold at once is queried once per device and instantiation.
template <bool A_MN, bool B_MN, int EPI>
int launch_pair(const CUtensorMap& ma, const CUtensorMap& mb, const GemmArgs& g, cudaStream_t s) {
  auto kern = ns_gemm_pair_kernel<A_MN, B_MN, EPI>;
  static std::atomic<int> max_pairs[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return MUZO_ERR_UNSUPPORTED;
  if (max_pairs[dev].load(std::memory_order_acquire) == 0) {
    MUZO_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, P_SMEM_BYTES));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(2 * (device_sm_count() / 2)), 1, 1);
    cfg.blockDim = dim3(NUM_THREADS, 1, 1);
    cfg.dynamicSmemBytes = P_SMEM_BYTES;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) != cudaSuccess || clusters <= 0) {
      cudaGetLastError();
      clusters = device_sm_count() / 2;
    }
    max_pairs[dev].store(clusters, std::memory_order_release);
  }
  const int64_t cap = max_pairs[dev].load(std::memory_order_acquire);
  const int64_t pairs = g.num_tiles < cap ? g.num_tiles : cap;
  kern<<<static_cast<unsigned>(2 * pairs), NUM_THREADS, P_SMEM_BYTES, s>>>(ma, mb, g);
  return launch_status();
}

// Wide-pair launch: grid = 2 x min(tiles, SMs / 2) (one CTA per SM by its shared memory).
template <bool A_MN, bool B_MN, int EPI>
int launch_wide(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& md, const CUtensorMap& me,
                const GemmArgs& g, cudaStream_t s) {
  auto kern = ns_gemm_wide_kernel<A_MN, B_MN, EPI>;
  static std::atomic<int> max_pairs[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return MUZO_ERR_UNSUPPORTED;
  if (max_pairs[dev].load(std::memory_order_acquire) == 0) {
    MUZO_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, W_SMEM_BYTES));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(2 * (device_sm_count() / 2)), 1, 1);
    cfg.blockDim = dim3(W_THREADS, 1, 1);
    cfg.dynamicSmemBytes = W_SMEM_BYTES;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) != cudaSuccess || clusters <= 0) {
      cudaGetLastError();
      clusters = device_sm_count() / 2;
    }
    max_pairs[dev].store(clusters, std::memory_order_release);
  }
  const int64_t cap = max_pairs[dev].load(std::memory_order_acquire);
  const int64_t pairs = g.num_tiles < cap ? g.num_tiles : cap;
  kern<<<static_cast<unsigned>(2 * pairs), W_THREADS, W_SMEM_BYTES, s>>>(ma, mb, md, me, g);
  return launch_status();
}

enum class Kernel { kOneSm, kPair, kWide };

template <int EPI>
int launch_epi(Kernel kind, bool a_mn, bool b_mn, const CUtensorMap& ma, const CUtensorMap& mb,
               const CUtensorMap& md, const CUtensorMap& me, const GemmArgs& g, cudaStream_t s) {
  if (kind == Kernel::kWide) {
    if (!a_mn && !b_mn) return launch_wide<false, false, EPI>(ma, mb, md, me, g, s);
    if (!a_mn && b_mn) return launch_wide<false, true, EPI>(ma, mb, md, me, g, s);
    if (a_mn && !b_mn) return launch_wide<true, false, EPI>(ma, mb, md, me, g, s);
    return launch_wide<true, true, EPI>(ma, mb, md, me, g, s);
  }
  if (kind == Kernel::kPair) {
    if (!a_mn && !b_mn) return launch_pair<false, false, EPI>(ma, mb, g, s);
    if (!a_mn && b_mn) return launch_pair<false, true, EPI>(ma, mb, g, s);
    if (a_mn && !b_mn) return launch_pair<true, false, EPI>(ma, mb, g, s);
    return launch_pair<true, true, EPI>(ma, mb, g, s);
  }
  if (!a_mn && !b_mn) return launch_gemm<false, false, EPI>(ma, mb, g, s);
  if (!a_mn && b_mn) return launch_gemm<false, true, EPI>(ma, mb, g, s);
  if (a_mn && !b_mn) return launch_gemm<true, false, EPI>(ma, mb, g, s);
  return launch_gemm<true, true, EPI>(ma, mb, g, s);
}

// Kernel choice: the wide CTA-pair kernel (256 x 512 tiles) when the output has at least 256
// rows and 512 columns, the CTA-pair kernel (256 x 256) when it has 256 of each, else the one-SM
// kernel (128 x 256). MUZO_GEMM_PAIR=0 forces the one-SM kernel, MUZO_GEMM_WIDE=0 the 256 x 256
// pair kernel wherever the wide one would run.
Kernel choose_kernel(int64_t m, int64_t n) {
  const char* v = std::getenv("MUZO_GEMM_PAIR");
  if (v != nullptr && v[0] == '0') return Kernel::kOneSm;
  if (m < PM || n < PN) return Kernel::kOneSm;
  const char* w = std::getenv("MUZO_GEMM_WIDE");
  if (n >= WN && !(w != nullptr && w[0] == '0')) return Kernel::kWide;
  return Kernel::kPair;
}

__device__ int32_t g_default_status[4];

bool aligned16h(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace
}  // namespace muzo

using namespace muzo;

extern "C" {

int muzo_ns_gemm(const void* a, int64_t lda, int64_t a_batch_stride, int a_mn, const void* b, int64_t ldb,
                 int64_t b_batch_stride, int b_mn, void* d, int64_t ldd, int64_t d_batch_stride,
                 const void* e, int epilogue, float c1, float c2, int64_t m, int64_t n, int64_t k,
                 int64_t batch, int symmetric, double* d_sums, const float* d_scales, int32_t* d_flags,
                 int32_t* d_status, void* stream) {
  if (a == nullptr || b == nullptr || d == nullptr || m <= 0 || n <= 0 || k <= 0 || batch <= 0)
    return MUZO_ERR_ARG;
  if (d_sums != nullptr && (epilogue != MUZO_EPI_UPDATE || d_scales == nullptr || d_flags == nullptr))
    return MUZO_ERR_ARG;
  if (epilogue != MUZO_EPI_STORE && e == nullptr) return MUZO_ERR_ARG;
  if (epilogue < MUZO_EPI_STORE || epilogue > MUZO_EPI_UPDATE) return MUZO_ERR_ARG;
  if (symmetric && (m != n || epilogue == MUZO_EPI_UPDATE)) return MUZO_ERR_ARG;
  if (lda % 8 || ldb % 8 || ldd % 8 || a_batch_stride % 8 || b_batch_stride % 8 || d_batch_stride % 8 ||
      !aligned16h(a) || !aligned16h(b) || !aligned16h(d) || (e && !aligned16h(e)))
    return MUZO_ERR_ALIGN;
  if (m > 0x7fffffffLL || n > 0x7fffffffLL || k > 0x7fffffffLL || batch > 0x7fffffffLL)
    return MUZO_ERR_UNSUPPORTED;
  // logical extents of the stored operands
  const int64_t a_rows = a_mn ? k : m, a_inner = a_mn ? m : k;
  const int64_t b_rows = b_mn ? k : n, b_inner = b_mn ? n : k;
  if (lda < a_inner || ldb < b_inner || ldd < n) return MUZO_ERR_ARG;
  const Kernel kind = choose_kernel(m, n);
  const bool pair = kind != Kernel::kOneSm;
  const int tile_m = pair ? PM : BM, tile_n = kind == Kernel::kWide ? WN : pair ? PN : BN;
  // rows of one CTA's K-major box: A holds BM (= PHALF) rows either way; B holds BN columns on
  // one SM and PHALF columns per CTA of a pair
  const int b_box_rows = pair ? PHALF : BN;
  CUtensorMap ma, mb;
  int st = a_mn ? encode_map(&ma, a, a_inner, a_rows, batch, lda, a_batch_stride ? a_batch_stride : lda * a_rows, 64, BK)
                : encode_map(&ma, a, a_inner, a_rows, batch, lda, a_batch_stride ? a_batch_stride : lda * a_rows, BK, BM);
  if (st != MUZO_OK) return st;
  st = b_mn ? encode_map(&mb, b, b_inner, b_rows, batch, ldb, b_batch_stride ? b_batch_stride : ldb * b_rows, 64, BK)
            : encode_map(&mb, b, b_inner, b_rows, batch, ldb, b_batch_stride ? b_batch_stride : ldb * b_rows, BK,
                         b_box_rows);
  if (st != MUZO_OK) return st;
  GemmArgs g;
  g.m = m; g.n = n; g.k = k; g.batch = batch;
  g.tile_m = tile_m; g.tile_n = tile_n;
  g.tiles_m = static_cast<int>((m + tile_m - 1) / tile_m);
  g.tiles_n = static_cast<int>((n + tile_n - 1) / tile_n);
  g.sym = symmetric ? 1 : 0;
  // Concurrent CTAs share the operand of the fast tile index: walking M first keeps the N-side
  // operand's column block hot and streams it from DRAM once when it is the larger operand
  // (B X with X = m x n, n > m); otherwise N first.
  g.m_fastest = (!g.sym && n > m) ? 1 : 0;
  if (g.sym) {
    g.tiles_per_batch = 0;
    for (int tm = 0; tm < g.tiles_m; ++tm) g.tiles_per_batch += g.tiles_n - (tm * tile_m) / tile_n;
  } else {
    g.tiles_per_batch = static_cast<int64_t>(g.tiles_m) * g.tiles_n;
  }
  g.num_tiles = g.tiles_per_batch * batch;
  g.num_kb = static_cast<int>((k + BK - 1) / BK);
  g.d = static_cast<__nv_bfloat16*>(d);
  g.ldd = ldd;
  g.d_bs = d_batch_stride ? d_batch_stride : ldd * m;
  g.e = static_cast<const __nv_bfloat16*>(e);
  g.c1 = c1; g.c2 = c2;
  g.sums = d_sums;
  g.scales = d_scales;
  g.flags = d_flags;
  if (d_status == nullptr) {
    void* p = nullptr;
    MUZO_CUDA_CHECK(cudaGetSymbolAddress(&p, g_default_status));
    d_status = static_cast<int32_t*>(p);
  }
  if (g.num_tiles >= (1ll << 30)) return MUZO_ERR_UNSUPPORTED;
  g.status = d_status;
  g.sched = d_status + 1;
  // the wide kernel's epilogue boxes: 32 x 32 of D (and of E, laid out like D), 64-byte swizzle
  CUtensorMap md = {}, me = {};
  if (kind == Kernel::kWide) {
    st = encode_map(&md, d, n, m, batch, ldd, g.d_bs, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B);
    if (st != MUZO_OK) return st;
    st = encode_map(&me, e != nullptr ? e : d, n, m, batch, ldd, g.d_bs, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B);
    if (st != MUZO_OK) return st;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (epilogue) {
    case MUZO_EPI_STORE: return launch_epi<MUZO_EPI_STORE>(kind, a_mn, b_mn, ma, mb, md, me, g, s);
    case MUZO_EPI_POLY: return launch_epi<MUZO_EPI_POLY>(kind, a_mn, b_mn, ma, mb, md, me, g, s);
    default: return launch_epi<MUZO_EPI_UPDATE>(kind, a_mn, b_mn, ma, mb, md, me, g, s);
  }
}

}  // extern "C"
