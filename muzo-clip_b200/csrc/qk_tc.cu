// Per-head maximum of the pre-softmax logits on the tensor cores (qk_clip.py:173-196).
//
// S = Q K^T is never stored: every 128-query x 256-key tile is accumulated in TMEM by
// tcgen05.mma (bf16 or fp16 operands, fp32 accumulation) and reduced to a maximum by the
// epilogue warps, which fold it into the head's running maximum with one atomicMax per warp
// and tile. Q [B, Hq, Sq, D] and K [B, Hkv, Sk, D] are read in place through 4-D tensor maps
// (transformers keeps them as transposed views of [B, S, H, D]); GQA maps query head h to key
// head h / (Hq / Hkv). Causal masking skips the key tiles entirely above a query tile's last row
// and masks the diagonal tiles in the epilogue.
//
// Layout of the kernel follows the Newton-Schulz GEMM: persistent CTAs (one per SM), warp 0 TMA
// producer into a 4-stage ring, warp 1 TMEM owner and MMA issuer with two 256-column
// accumulators, warps 2-5 epilogue; every wait is bounded.
#include "tcgen05_common.cuh"

namespace muzo {
namespace {

using namespace tc;

constexpr int QM = 128;    // queries per tile (UMMA M)
constexpr int QN = 256;    // keys per tile (UMMA N)
constexpr int QBK = 64;    // head-dim slice per stage (128-byte swizzle row)
constexpr int Q_STAGES = 4;
constexpr int QA_BYTES = QM * QBK * 2;
constexpr int QB_BYTES = QN * QBK * 2;
constexpr int Q_STAGE_BYTES = QA_BYTES + QB_BYTES;
constexpr int Q_THREADS = 192;
constexpr int Q_TMEM_COLS = 2 * QN;
constexpr int Q_SMEM_BYTES = Q_STAGES * Q_STAGE_BYTES + 1024 + 256;

struct QkArgs {
  int64_t sq, sk, shift;
  int hq, hkv, group, nqt, causal, num_kb;
  int64_t tiles_per_bh, num_tiles;
  int* enc;
  int32_t* valid;
  int32_t* status;
};

__device__ __forceinline__ int encode_max(float f) {
  const int b = __float_as_int(f);
  return b >= 0 ? b : b ^ 0x7fffffff;
}

__device__ __forceinline__ int kv_tiles(const QkArgs& g, int qt) {
  int64_t end = g.sk;
  if (g.causal) {
    const int64_t last = static_cast<int64_t>(qt + 1) * QM + g.shift;  // keys visible to the tile's last row
    end = last < g.sk ? last : g.sk;
    if (end < 0) end = 0;
  }
  return static_cast<int>((end + QN - 1) / QN);
}

// flat tile -> (batch*head, query tile, key tile)
__device__ __forceinline__ void qk_tile(const QkArgs& g, int64_t t, int64_t& bh, int& qt, int& kv) {
  bh = t / g.tiles_per_bh;
  int64_t r = t - bh * g.tiles_per_bh;
  int q = 0;
  while (q < g.nqt) {
    const int w = kv_tiles(g, q);
    if (r < w) break;
    r -= w;
    ++q;
  }
  qt = q;
  kv = static_cast<int>(r);
}

template <int FMT>
__global__ void __launch_bounds__(Q_THREADS, 1)
qk_max_tc_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k, QkArgs g) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Q_STAGES * Q_STAGE_BYTES);
  uint64_t* empty = full + Q_STAGES;
  uint64_t* tfull = empty + Q_STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(tempty + 2);
  int* abort_flag = reinterpret_cast<int*>(tmem_holder + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < Q_STAGES; ++s) { mbar_init(full + s, 1); mbar_init(empty + s, 1); }
    for (int a = 0; a < 2; ++a) { mbar_init(tfull + a, 1); mbar_init(tempty + a, 4); }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_holder)),
                 "r"(Q_TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 0) {
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_q)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_k)) : "memory");
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      uint32_t armed = 0, armed_parity = 0;
      for (int64_t t = blockIdx.x; t < g.num_tiles && ok; t += gridDim.x) {
        int64_t bh; int qt, kv;
        qk_tile(g, t, bh, qt, kv);
        const int b = static_cast<int>(bh / g.hq), h = static_cast<int>(bh % g.hq);
        const int kvh = h / g.group;
        for (int kb = 0; kb < g.num_kb; ++kb) {
          if (!mbar_wait(empty + stage, phase ^ 1)) { ok = false; break; }
          if (*reinterpret_cast<volatile int*>(abort_flag)) { ok = false; break; }
          uint8_t* sa = smem + stage * Q_STAGE_BYTES;
          mbar_arrive_expect_tx(full + stage, Q_STAGE_BYTES);
          armed |= 1u << stage;
          armed_parity = (armed_parity & ~(1u << stage)) | (phase << stage);
          tma_load_4d(&map_q, full + stage, sa, kb * QBK, qt * QM, h, b);
          tma_load_4d(&map_k, full + stage, sa + QA_BYTES, kb * QBK, kv * QN, kvh, b);
          if (++stage == Q_STAGES) { stage = 0; phase ^= 1; }
        }
      }
      if (!ok) { atomicCAS(g.status, kErrNone, kErrTimeoutProducer); atomicExch(abort_flag, 1); atomicExch(g.valid, 0); }
      for (int s2 = 0; s2 < Q_STAGES; ++s2)
        if (armed & (1u << s2)) mbar_wait(full + s2, (armed_parity >> s2) & 1u);
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_fmt(QM, QN, false, false, FMT);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int64_t local = 0;
      for (int64_t t = blockIdx.x; t < g.num_tiles && ok; t += gridDim.x, ++local) {
        const int acc = static_cast<int>(local & 1);
        const uint32_t acc_phase = static_cast<uint32_t>((local >> 1) & 1);
        if (!mbar_wait(tempty + acc, acc_phase ^ 1)) { ok = false; break; }
        tc_fence_after();
        const uint32_t tmem_d = tmem_base + acc * QN;
        for (int kb = 0; kb < g.num_kb; ++kb) {
          if (!mbar_wait(full + stage, phase)) { ok = false; break; }
          if (*reinterpret_cast<volatile int*>(abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * Q_STAGE_BYTES);
          const uint32_t sb = sa + QA_BYTES;
#pragma unroll
          for (int k = 0; k < QBK / 16; ++k)
            umma_f16(tmem_d, make_sdesc(sa + k * 32, 16, 1024), make_sdesc(sb + k * 32, 16, 1024), idesc,
                     (kb > 0 || k > 0) ? 1u : 0u);
          umma_commit(empty + stage);
          if (++stage == Q_STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        umma_commit(tfull + acc);
      }
      if (!ok) { atomicCAS(g.status, kErrNone, kErrTimeoutMma); atomicExch(abort_flag, 1); atomicExch(g.valid, 0); }
    }
    __syncwarp();
  } else {
    const int lane_base = 32 * (warp & 3);
    int64_t local = 0;
    bool ok = true;
    bool finite = true;
    for (int64_t t = blockIdx.x; t < g.num_tiles; t += gridDim.x, ++local) {
      int64_t bh; int qt, kv;
      qk_tile(g, t, bh, qt, kv);
      const int h = static_cast<int>(bh % g.hq);
      const int acc = static_cast<int>(local & 1);
      const uint32_t acc_phase = static_cast<uint32_t>((local >> 1) & 1);
      bool ready = true;
      if (lane == 0) ready = mbar_wait(tfull + acc, acc_phase);
      ready = __shfl_sync(0xffffffffu, ready ? 1 : 0, 0) != 0;
      if (!ready || *reinterpret_cast<volatile int*>(abort_flag)) { ok = ready; break; }
      tc_fence_after();
      const int64_t row = static_cast<int64_t>(qt) * QM + lane_base + lane;
      const int64_t jlim_causal = row + g.shift;  // last visible key of this row
      float best = -INFINITY;
#pragma unroll 1
      for (int c = 0; c < QN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(tmem_base + (static_cast<uint32_t>(lane_base) << 16) + acc * QN + c * 32, r);
        const int64_t j0 = static_cast<int64_t>(kv) * QN + c * 32;
        const bool row_ok = row < g.sq;
        const bool all_ok = row_ok && j0 + 31 < g.sk && (!g.causal || j0 + 31 <= jlim_causal);
        if (all_ok) {
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const float x = __uint_as_float(r[e]);
            finite = finite && isfinite(x);
            best = fmaxf(best, x);
          }
        } else if (row_ok) {
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const int64_t j = j0 + e;
            if (j < g.sk && (!g.causal || j <= jlim_causal)) {
              const float x = __uint_as_float(r[e]);
              finite = finite && isfinite(x);
              best = fmaxf(best, x);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty + acc);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) best = fmaxf(best, __shfl_xor_sync(0xffffffffu, best, o));
      if (lane == 0 && best > -INFINITY) atomicMax(g.enc + h, encode_max(best));
    }
    if (!finite) atomicExch(g.valid, 0);
    if (!ok && lane == 0) {
      atomicCAS(g.status, kErrNone, kErrTimeoutEpilogue);
      atomicExch(abort_flag, 1);
      atomicExch(g.valid, 0);  // a capture whose wait expired is dropped like a non-finite one
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    if (lane == 0 && *reinterpret_cast<volatile int*>(abort_flag)) {
      uint64_t* drain = tempty;
      mbar_init(drain, 1);
      asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
      umma_commit(drain);
      mbar_wait(drain, 0);
    }
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(Q_TMEM_COLS)
                 : "memory");
  }
}

// 4-D tensor map over [B][H][S][D] with element strides (sb, sh, ss) and box QBK x rows x 1 x 1.
int encode_qk_map(CUtensorMap* map, const void* base, int dtype, int64_t d, int64_t s, int64_t h, int64_t b,
                  int64_t ss, int64_t sh, int64_t sb, int rows) {
  auto fn = encode_fn();
  if (fn == nullptr) return MUZO_ERR_UNSUPPORTED;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(d), static_cast<cuuint64_t>(s), static_cast<cuuint64_t>(h),
                        static_cast<cuuint64_t>(b)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(ss * 2), static_cast<cuuint64_t>(sh * 2),
                           static_cast<cuuint64_t>(sb * 2)};
  cuuint32_t box[4] = {QBK, static_cast<cuuint32_t>(rows), 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUtensorMapDataType dt = dtype == MUZO_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = fn(map, dt, 4, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? MUZO_OK : MUZO_ERR_ARG;
}

__device__ int32_t g_qk_status;

}  // namespace

// Tensor-core path of muzo_qk_max (bf16 / fp16, strides multiple of 8 elements). enc holds the
// head maxima as ordered integers, already initialised by the caller.
int qk_max_tensor_cores(const void* q, const void* k, int dtype, int64_t batch, int64_t hq, int64_t hkv, int64_t sq,
                        int64_t sk, int64_t d, int64_t qsb, int64_t qsh, int64_t qss, int64_t ksb, int64_t ksh,
                        int64_t kss, int causal, int* enc, int32_t* valid, cudaStream_t stream) {
  CUtensorMap mq, mk;
  int st = encode_qk_map(&mq, q, dtype, d, sq, hq, batch, qss, qsh, qsb, QM);
  if (st != MUZO_OK) return st;
  st = encode_qk_map(&mk, k, dtype, d, sk, hkv, batch, kss, ksh, ksb, QN);
  if (st != MUZO_OK) return st;
  QkArgs g;
  g.sq = sq; g.sk = sk; g.shift = sk - sq;
  g.hq = static_cast<int>(hq); g.hkv = static_cast<int>(hkv); g.group = static_cast<int>(hq / hkv);
  g.nqt = static_cast<int>((sq + QM - 1) / QM);
  g.causal = causal;
  g.num_kb = static_cast<int>((d + QBK - 1) / QBK);
  int64_t per = 0;
  for (int qt = 0; qt < g.nqt; ++qt) {
    int64_t end = sk;
    if (causal) {
      const int64_t last = static_cast<int64_t>(qt + 1) * QM + g.shift;
      end = last < sk ? last : sk;
      if (end < 0) end = 0;
    }
    per += (end + QN - 1) / QN;
  }
  g.tiles_per_bh = per;
  g.num_tiles = per * batch * hq;
  g.enc = enc;
  g.valid = valid;
  void* p = nullptr;
  MUZO_CUDA_CHECK(cudaGetSymbolAddress(&p, g_qk_status));
  g.status = static_cast<int32_t*>(p);
  if (g.num_tiles == 0) return MUZO_OK;
  auto kern = dtype == MUZO_BF16 ? qk_max_tc_kernel<1> : qk_max_tc_kernel<0>;
  static bool configured[2][64] = {{false}};
  int dev = 0;
  cudaGetDevice(&dev);
  const int fi = dtype == MUZO_BF16 ? 1 : 0;
  if (dev >= 0 && dev < 64 && !configured[fi][dev]) {
    MUZO_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Q_SMEM_BYTES));
    configured[fi][dev] = true;
  }
  const int64_t grid = g.num_tiles < device_sm_count() ? g.num_tiles : device_sm_count();
  kern<<<static_cast<unsigned>(grid), Q_THREADS, Q_SMEM_BYTES, stream>>>(mq, mk, g);
  return launch_status();
}

}  // namespace muzo
