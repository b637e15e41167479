// Newton-Schulz GEMMs for MuZO-Clip on sm_100a: tcgen05.mma with fp32 accumulators in TMEM,
// operands staged in shared memory by TMA (cp.async.bulk.tensor, no multicast), and the
// element-wise parts of the quintic iteration (newton_schulz.py:55-58) fused into the epilogue.
//
// One persistent CTA per SM (grid = min(tiles, SMs)), 6 warps:
//   warp 0      TMA producer (one thread): A/B k-blocks into a 4-stage shared-memory ring;
//   warp 1      TMEM owner and MMA issuer (one thread): 128x256x16 bf16 MMAs into one of two
//               256-column TMEM accumulators, so the epilogue of tile i overlaps tile i+1;
//   warps 2..5  epilogue: tcgen05.ld 32 columns at a time, apply the fused op, store bf16.
// Every wait is bounded; on timeout the kernel records an error code, drains and returns.
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
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;

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
};

template <int EPI>
__device__ __forceinline__ void epilogue_chunk(const GemmArgs& g, int64_t b, int64_t row, int64_t col0,
                                               const uint32_t (&acc)[32]) {
  if (row >= g.m || col0 >= g.n) return;
  if (g.sym && col0 + 31 < row) return;  // strictly below the diagonal: written by the mirror
  const int64_t base = b * g.d_bs + row * g.ldd + col0;
  float o[32];
  if (EPI == MUZO_EPI_STORE) {
#pragma unroll
    for (int i = 0; i < 32; ++i) o[i] = __uint_as_float(acc[i]);
  } else {
    float e[32];
    if (col0 + 32 <= g.n) {
      const uint4* ep = reinterpret_cast<const uint4*>(g.e + base);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint4 u = ep[q];
        uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int h = 0; h < 4; ++h) { e[8 * q + 2 * h] = bf16_lo(w[h]); e[8 * q + 2 * h + 1] = bf16_hi(w[h]); }
      }
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) e[i] = col0 + i < g.n ? __bfloat162float(g.e[base + i]) : 0.0f;
    }
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const float a = __uint_as_float(acc[i]);
      const float t1 = bf16r(g.c1 * e[i]);           // c1 * E, rounded to bf16
      if (EPI == MUZO_EPI_POLY) {
        const float t2 = bf16r(g.c2 * bf16r(a));     // c2 * bf16(A @ A)
        o[i] = t1 + t2;
      } else {
        o[i] = t1 + bf16r(a);                        // a*X + bf16(B @ X)
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
    }
  } else {
    for (int i = 0; i < 32 && col0 + i < g.n; ++i) g.d[base + i] = __float2bfloat16_rn(o[i]);
  }
}

// Tile t -> (batch, tile row, tile column). Symmetric outputs enumerate, per tile row tm, only
// the columns tn >= tm * BM / BN (tiles that hold an element on or above the diagonal).
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
    const int64_t width = g.tiles_n - (row * BM) / BN;
    if (r < width) break;
    r -= width;
    ++row;
  }
  tm = row;
  tn = static_cast<int>((row * BM) / BN + r);
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
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(tempty + 2);
  int* abort_flag = reinterpret_cast<int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) { mbar_init(full + s, 1); mbar_init(empty + s, 1); }
    for (int a = 0; a < 2; ++a) { mbar_init(tfull + a, 1); mbar_init(tempty + a, 4); }
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
      bool ok = true;
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
      bool ok = true;
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
    for (int64_t t = blockIdx.x; t < g.num_tiles; t += gridDim.x, ++local) {
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
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(tmem_base + (static_cast<uint32_t>(lane_base) << 16) + acc * BN + c * 32, r);
        epilogue_chunk<EPI>(g, b, row, static_cast<int64_t>(tn) * BN + c * 32, r);
      }
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

// ------------------------------------------------------------------ host side

// 3-D bf16 tensor map over [batch][rows][inner] with leading dim `ld` and batch stride `bs`
// (elements); box = box_inner x box_rows x 1 with 128-byte swizzle and zero fill out of bounds.
int encode_map(CUtensorMap* map, const void* base, int64_t inner, int64_t rows, int64_t batch, int64_t ld,
               int64_t bs, int box_inner, int box_rows) {
  auto fn = encode_fn();
  if (fn == nullptr) return MUZO_ERR_UNSUPPORTED;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(rows),
                        static_cast<cuuint64_t>(batch)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(ld * 2), static_cast<cuuint64_t>(bs * 2)};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(box_inner), static_cast<cuuint32_t>(box_rows), 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box,
                  estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? MUZO_OK : MUZO_ERR_ARG;
}

template <bool A_MN, bool B_MN, int EPI>
int launch_gemm(const CUtensorMap& ma, const CUtensorMap& mb, const GemmArgs& g, cudaStream_t s) {
  auto kern = ns_gemm_kernel<A_MN, B_MN, EPI>;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    MUZO_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
    configured[dev] = true;
  }
  int64_t grid = g.num_tiles < device_sm_count() ? g.num_tiles : device_sm_count();
  kern<<<static_cast<unsigned>(grid), NUM_THREADS, SMEM_BYTES, s>>>(ma, mb, g);
  return launch_status();
}

template <int EPI>
int launch_epi(bool a_mn, bool b_mn, const CUtensorMap& ma, const CUtensorMap& mb, const GemmArgs& g,
               cudaStream_t s) {
  if (!a_mn && !b_mn) return launch_gemm<false, false, EPI>(ma, mb, g, s);
  if (!a_mn && b_mn) return launch_gemm<false, true, EPI>(ma, mb, g, s);
  if (a_mn && !b_mn) return launch_gemm<true, false, EPI>(ma, mb, g, s);
  return launch_gemm<true, true, EPI>(ma, mb, g, s);
}

__device__ int32_t g_default_status;

bool aligned16h(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace
}  // namespace muzo

using namespace muzo;

extern "C" {

int muzo_ns_gemm(const void* a, int64_t lda, int64_t a_batch_stride, int a_mn, const void* b, int64_t ldb,
                 int64_t b_batch_stride, int b_mn, void* d, int64_t ldd, int64_t d_batch_stride,
                 const void* e, int epilogue, float c1, float c2, int64_t m, int64_t n, int64_t k,
                 int64_t batch, int symmetric, int32_t* d_status, void* stream) {
  if (a == nullptr || b == nullptr || d == nullptr || m <= 0 || n <= 0 || k <= 0 || batch <= 0)
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
  CUtensorMap ma, mb;
  int st = a_mn ? encode_map(&ma, a, a_inner, a_rows, batch, lda, a_batch_stride ? a_batch_stride : lda * a_rows, 64, BK)
                : encode_map(&ma, a, a_inner, a_rows, batch, lda, a_batch_stride ? a_batch_stride : lda * a_rows, BK, BM);
  if (st != MUZO_OK) return st;
  st = b_mn ? encode_map(&mb, b, b_inner, b_rows, batch, ldb, b_batch_stride ? b_batch_stride : ldb * b_rows, 64, BK)
            : encode_map(&mb, b, b_inner, b_rows, batch, ldb, b_batch_stride ? b_batch_stride : ldb * b_rows, BK, BN);
  if (st != MUZO_OK) return st;
  GemmArgs g;
  g.m = m; g.n = n; g.k = k; g.batch = batch;
  g.tiles_m = static_cast<int>((m + BM - 1) / BM);
  g.tiles_n = static_cast<int>((n + BN - 1) / BN);
  g.sym = symmetric ? 1 : 0;
  // Concurrent CTAs share the operand of the fast tile index: walking M first keeps the N-side
  // operand's column block hot and streams it from DRAM once when it is the larger operand
  // (B X with X = m x n, n > m); otherwise N first.
  g.m_fastest = (!g.sym && n > m) ? 1 : 0;
  if (g.sym) {
    g.tiles_per_batch = 0;
    for (int tm = 0; tm < g.tiles_m; ++tm) g.tiles_per_batch += g.tiles_n - (tm * BM) / BN;
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
  if (d_status == nullptr) {
    void* p = nullptr;
    MUZO_CUDA_CHECK(cudaGetSymbolAddress(&p, g_default_status));
    d_status = static_cast<int32_t*>(p);
  }
  g.status = d_status;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (epilogue) {
    case MUZO_EPI_STORE: return launch_epi<MUZO_EPI_STORE>(a_mn, b_mn, ma, mb, g, s);
    case MUZO_EPI_POLY: return launch_epi<MUZO_EPI_POLY>(a_mn, b_mn, ma, mb, g, s);
    default: return launch_epi<MUZO_EPI_UPDATE>(a_mn, b_mn, ma, mb, g, s);
  }
}

}  // extern "C"
