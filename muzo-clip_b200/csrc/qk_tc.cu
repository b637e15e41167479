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
#include <atomic>
#include <cstdlib>

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
  const int32_t* key_lo;   // per batch: visible keys [key_lo[b], key_hi[b]); NULL: all keys
  const int32_t* key_hi;
  int* enc;
  int32_t* valid;
  int32_t* status;
};

__device__ __forceinline__ int encode_max(float f) {
  const int b = __float_as_int(f);
  return b >= 0 ? b : b ^ 0x7fffffff;
}

// The visible key range [lo, hi) of batch row b, clamped to [0, sk].
__device__ __forceinline__ void key_range(const int32_t* key_lo, const int32_t* key_hi, int64_t b, int64_t sk,
                                          int64_t& lo, int64_t& hi) {
  lo = 0;
  hi = sk;
  if (key_lo != nullptr) {
    const int64_t l = __ldg(key_lo + b), h = __ldg(key_hi + b);
    lo = l > 0 ? l : 0;
    hi = h < sk ? h : sk;
  }
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
      int64_t jmin, jend;
      key_range(g.key_lo, g.key_hi, bh / g.hq, g.sk, jmin, jend);
      int64_t jmax = jend - 1;                     // last visible key of this row
      if (g.causal && row + g.shift < jmax) jmax = row + g.shift;
      float best = -INFINITY;
#pragma unroll 1
      for (int c = 0; c < QN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(tmem_base + (static_cast<uint32_t>(lane_base) << 16) + acc * QN + c * 32, r);
        const int64_t j0 = static_cast<int64_t>(kv) * QN + c * 32;
        const bool row_ok = row < g.sq;
        const bool all_ok = row_ok && j0 >= jmin && j0 + 31 <= jmax;
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
            if (j >= jmin && j <= jmax) {
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

// ------------------------------------------------------------------ CTA-pair kernel
// A 2-CTA cluster takes a contiguous range of (batch*head, 256-query block, 256-key block) tiles.
// Each CTA keeps its 128 query rows of the current query block resident in shared memory
// (two buffers, so the next block loads while the current one computes) and streams its 128
// keys of each key block: per SM
// 16 KB of K per 64-deep slice for a 256 x 256 MMA tile (tcgen05.mma.cta_group::2, M = N = 256).
// Eight epilogue warps per CTA (two per TMEM lane quarter, 128 columns each) fold the tile into
// per-thread running max / min registers with NaN-propagating max, and flush them with one
// atomicMax per warp when the head changes.
constexpr int PQ_ROWS = 128;                         // queries per CTA; a pair covers 256
constexpr int PK_ROWS = 128;                         // keys per CTA per tile; a pair tile covers 256
constexpr int PQ_MAX_KB = 4;                         // head dim up to 256 = 4 slices of 64
constexpr int PQ_SUB_BYTES = PQ_ROWS * QBK * 2;      // 16 KB per slice
constexpr int PK_STAGE_BYTES = PK_ROWS * QBK * 2;    // 16 KB
constexpr int PK_MAX_STAGES = 12;
constexpr int PQ_SLOTS = 2;                          // query-block buffers
constexpr int PQK_TILE_BYTES = 192 * 1024;           // query buffers + key stages
constexpr int PQK_THREADS = 320;                     // warp 0 TMA, warp 1 TMEM + MMA, warps 2..9 epilogue
constexpr int PQK_EPI_WARPS = 8;
constexpr int PQK_SMEM_BYTES = PQK_TILE_BYTES + 1024 + 512;

struct QkPairArgs {
  int64_t sq, sk, shift;
  int hq, group, nqb, causal, num_kb;
  int k_stages;            // key stages in the shared memory the query buffers leave
  int64_t tiles_per_bh, num_tiles;
  const int32_t* key_lo;   // per batch: visible keys [key_lo[b], key_hi[b]); NULL: all keys
  const int32_t* key_hi;
  int* enc;
  int32_t* valid;
  int32_t* status;
};

__device__ __forceinline__ int pair_kv_tiles(const QkPairArgs& g, int qb) {
  int64_t end = g.sk;
  if (g.causal) {
    const int64_t last = static_cast<int64_t>(qb + 1) * 2 * PQ_ROWS + g.shift;  // keys visible to the block's last row
    end = last < g.sk ? last : g.sk;
    if (end < 0) end = 0;
  }
  return static_cast<int>((end + 2 * PK_ROWS - 1) / (2 * PK_ROWS));
}

// flat tile -> (batch*head, query block, key block)
__device__ __forceinline__ void pair_qk_tile(const QkPairArgs& g, int64_t t, int64_t& bh, int& qb, int& kv) {
  bh = t / g.tiles_per_bh;
  int64_t r = t - bh * g.tiles_per_bh;
  int q = 0;
  while (q < g.nqb) {
    const int w = pair_kv_tiles(g, q);
    if (r < w) break;
    r -= w;
    ++q;
  }
  qb = q;
  kv = static_cast<int>(r);
}

// Sequential walk over a contiguous tile range: decoded once, then advanced without divisions
// (a 64-bit division per tile on every role's critical path costs more than the tile's MMAs).
struct PairTileCursor {
  int64_t bh;
  int qb, kv, nkv;
  __device__ __forceinline__ void start(const QkPairArgs& g, int64_t t) {
    pair_qk_tile(g, t, bh, qb, kv);
    nkv = pair_kv_tiles(g, qb);
  }
  // true when the next tile starts a new query block
  __device__ __forceinline__ bool last_of_block() const { return kv + 1 >= nkv; }
  __device__ __forceinline__ void advance(const QkPairArgs& g) {
    if (++kv < nkv) return;
    kv = 0;
    do {  // query blocks without visible keys hold no tiles
      if (++qb == g.nqb) { qb = 0; ++bh; }
      nkv = pair_kv_tiles(g, qb);
    } while (nkv == 0);
  }
};

__device__ __forceinline__ float max_nan(float a, float b) {
  float d;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
  return d;
}

template <int FMT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(PQK_THREADS, 1)
qk_max_pair_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                   QkPairArgs g) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  const int PQ_SLOT_BYTES = g.num_kb * PQ_SUB_BYTES;
  const int PK_STAGES = g.k_stages;
  uint8_t* sq_slots = smem;                                        // [PQ_SLOTS][num_kb][128 x 64]
  uint8_t* sk_stages = smem + PQ_SLOTS * PQ_SLOT_BYTES;            // [k_stages][128 x 64]
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + PQK_TILE_BYTES);
  uint64_t* empty = full + PK_MAX_STAGES;
  uint64_t* tfull = empty + PK_STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* q_full = tempty + 2;
  uint64_t* q_empty = q_full + PQ_SLOTS;
  uint64_t* drain = q_empty + PQ_SLOTS;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);
  int* abort_flag = reinterpret_cast<int*>(tmem_holder + 1);
  // phases this CTA's producer loaded into (leader: armed): key stages, then query buffers; read
  // by the leader once both producers have stopped
  uint32_t* issued = reinterpret_cast<uint32_t*>(abort_flag + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int64_t pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int64_t t_begin = pair * g.num_tiles / npairs, t_end = (pair + 1) * g.num_tiles / npairs;

  if (threadIdx.x == 0) {
    for (int s = 0; s < PK_STAGES; ++s) { mbar_init(full + s, 1); mbar_init(empty + s, 1); }
    for (int a = 0; a < 2; ++a) { mbar_init(tfull + a, 1); mbar_init(tempty + a, 2 * PQK_EPI_WARPS); }
    for (int q = 0; q < PQ_SLOTS; ++q) { mbar_init(q_full + q, 1); mbar_init(q_empty + q, 1); }
    mbar_init(drain, 1);
    *abort_flag = 0;
    for (int s = 0; s < PK_MAX_STAGES + PQ_SLOTS; ++s) issued[s] = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_holder)),
                 "r"(Q_TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer (both CTAs)
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_q)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_k)) : "memory");
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int64_t useq = -1;                      // sequence number of the current query block
      PairTileCursor cur;
      cur.start(g, t_begin);
      int64_t cur_bh = -1;
      int b = 0, h = 0;
      for (int64_t t = t_begin; t < t_end && ok; ++t, cur.advance(g)) {
        const int qb = cur.qb, kv = cur.kv;
        if (cur.bh != cur_bh) {
          cur_bh = cur.bh;
          b = static_cast<int>(cur_bh / g.hq);
          h = static_cast<int>(cur_bh - static_cast<int64_t>(b) * g.hq);
        }
        if (t == t_begin || kv == 0) {         // a new query block
          ++useq;
          // the MMAs of the block that used this buffer two blocks ago must be done with it
          const int qs = static_cast<int>(useq % PQ_SLOTS);
          if (!mbar_wait(q_empty + qs, static_cast<uint32_t>(((useq / PQ_SLOTS) & 1) ^ 1))) { ok = false; break; }
          if (leader) mbar_arrive_expect_tx_u32(smem_u32(q_full + qs), 2u * g.num_kb * PQ_SUB_BYTES);
          const uint32_t qbar = map_to_rank(smem_u32(q_full + qs), 0);
          for (int kb = 0; kb < g.num_kb; ++kb)
            tma_load_4d_pair(&map_q, qbar, sq_slots + qs * PQ_SLOT_BYTES + kb * PQ_SUB_BYTES, kb * QBK,
                             qb * 2 * PQ_ROWS + static_cast<int>(rank) * PQ_ROWS, h, b);
          issued[PK_MAX_STAGES + qs] += 1;
        }
        const int kvh = h / g.group;
        for (int kb = 0; kb < g.num_kb; ++kb) {
          if (!mbar_wait(empty + stage, phase ^ 1)) { ok = false; break; }
          if (*reinterpret_cast<volatile int*>(abort_flag)) { ok = false; break; }
          if (leader) mbar_arrive_expect_tx_u32(smem_u32(full + stage), 2u * PK_STAGE_BYTES);
          tma_load_4d_pair(&map_k, map_to_rank(smem_u32(full + stage), 0), sk_stages + stage * PK_STAGE_BYTES,
                           kb * QBK, kv * 2 * PK_ROWS + static_cast<int>(rank) * PK_ROWS, kvh, b);
          issued[stage] += 1;
          if (++stage == PK_STAGES) { stage = 0; phase ^= 1; }
        }
      }
      if (!ok) { atomicCAS(g.status, kErrNone, kErrTimeoutProducer); pair_abort(abort_flag); atomicExch(g.valid, 0); }
      // the loads still in flight are waited for after both producers have stopped (below)
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer (leader only)
    if (lane == 0 && leader) {
      constexpr uint32_t idesc = make_idesc_fmt(2 * PQ_ROWS, 2 * PK_ROWS, false, false, FMT);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int64_t useq = -1, local = 0;
      PairTileCursor cur;
      cur.start(g, t_begin);
      for (int64_t t = t_begin; t < t_end && ok; ++t, ++local, cur.advance(g)) {
        if (t == t_begin || cur.kv == 0) {     // a new query block
          ++useq;
          if (!mbar_wait(q_full + useq % PQ_SLOTS, static_cast<uint32_t>((useq / PQ_SLOTS) & 1))) { ok = false; break; }
          tc_fence_after();
        }
        const int acc = static_cast<int>(local & 1);
        if (!mbar_wait(tempty + acc, static_cast<uint32_t>(((local >> 1) & 1) ^ 1))) { ok = false; break; }
        tc_fence_after();
        const uint32_t tmem_d = tmem_base + acc * QN;
        for (int kb = 0; kb < g.num_kb; ++kb) {
          if (!mbar_wait(full + stage, phase)) { ok = false; break; }
          if (*reinterpret_cast<volatile int*>(abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(sq_slots + (useq % PQ_SLOTS) * PQ_SLOT_BYTES + kb * PQ_SUB_BYTES);
          const uint32_t sb = smem_u32(sk_stages + stage * PK_STAGE_BYTES);
#pragma unroll
          for (int k = 0; k < QBK / 16; ++k)
            umma_f16_pair(tmem_d, make_sdesc(sa + k * 32, 16, 1024), make_sdesc(sb + k * 32, 16, 1024), idesc,
                          (kb > 0 || k > 0) ? 1u : 0u);
          umma_commit_pair(empty + stage);
          if (++stage == PK_STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        umma_commit_pair(tfull + acc);
        // the last tile of this query block in the range: Q may be replaced once its MMAs finish
        if (t + 1 >= t_end || cur.last_of_block()) umma_commit_pair(q_empty + useq % PQ_SLOTS);
      }
      if (!ok) { atomicCAS(g.status, kErrNone, kErrTimeoutMma); pair_abort(abort_flag); atomicExch(g.valid, 0); }
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------------- epilogue (warps 2..9, both CTAs)
    const int quarter = warp & 3;                    // TMEM lanes this warp may access
    const int colh = (warp - 2) >> 2;                // which 128 of the tile's 256 key columns
    const uint32_t leader_tempty0 = map_to_rank(smem_u32(tempty), 0);
    bool ok = true;
    int64_t cur_bh = -1;
    float best = -INFINITY, low = INFINITY;
    auto flush = [&](int64_t bh) {
      float m = best;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = max_nan(m, __shfl_xor_sync(0xffffffffu, m, o));
      float l = low;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) l = fminf(l, __shfl_xor_sync(0xffffffffu, l, o));
      if (lane == 0) {
        if (m != m || m == INFINITY || l == -INFINITY) atomicExch(g.valid, 0);
        else if (m > -INFINITY) atomicMax(g.enc + static_cast<int>(bh % g.hq), encode_max(m));
      }
      best = -INFINITY;
      low = INFINITY;
    };
    int64_t local = 0;
    int64_t key_begin = 0, key_end = g.sk;
    PairTileCursor cur;
    cur.start(g, t_begin);
    for (int64_t t = t_begin; t < t_end; ++t, ++local, cur.advance(g)) {
      const int64_t bh = cur.bh;
      const int qb = cur.qb, kv = cur.kv;
      if (bh != cur_bh) {
        if (cur_bh >= 0) flush(cur_bh);
        cur_bh = bh;
        key_range(g.key_lo, g.key_hi, bh / g.hq, g.sk, key_begin, key_end);
      }
      const int acc = static_cast<int>(local & 1);
      bool ready = true;
      if (lane == 0) ready = mbar_wait(tfull + acc, static_cast<uint32_t>((local >> 1) & 1));
      ready = __shfl_sync(0xffffffffu, ready ? 1 : 0, 0) != 0;
      if (!ready || *reinterpret_cast<volatile int*>(abort_flag)) { ok = ready; break; }
      tc_fence_after();
      const int64_t row = static_cast<int64_t>(qb) * 2 * PQ_ROWS + static_cast<int64_t>(rank) * PQ_ROWS +
                          32 * quarter + lane;
      int64_t jmax = key_end - 1;                  // last visible key of this row
      if (g.causal && row + g.shift < jmax) jmax = row + g.shift;
      const int64_t j0 = static_cast<int64_t>(kv) * 2 * PK_ROWS + colh * 128;
      uint32_t r[128];
      tmem_ld128(tmem_base + (static_cast<uint32_t>(32 * quarter) << 16) + acc * QN + colh * 128, r);
      // the accumulator is in registers: hand it back to the MMA issuer before reducing it
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(leader_tempty0 + acc * 8);
      if (row < g.sq && j0 >= key_begin && j0 + 127 <= jmax) {
        // eight independent max / min chains instead of one 128-long dependency chain
        float m[8], n[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) { m[e] = __uint_as_float(r[e]); n[e] = m[e]; }
#pragma unroll
        for (int e = 8; e < 128; ++e) {
          const float x = __uint_as_float(r[e]);
          m[e & 7] = max_nan(m[e & 7], x);
          n[e & 7] = fminf(n[e & 7], x);
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) { best = max_nan(best, m[e]); low = fminf(low, n[e]); }
      } else if (row < g.sq && j0 <= jmax && j0 + 127 >= key_begin) {
#pragma unroll
        for (int e = 0; e < 128; ++e) {
          if (j0 + e <= jmax && j0 + e >= key_begin) {
            const float x = __uint_as_float(r[e]);
            best = max_nan(best, x);
            low = fminf(low, x);
          }
        }
      }
    }
    if (cur_bh >= 0 && ok) flush(cur_bh);
    if (!ok && lane == 0) {
      atomicCAS(g.status, kErrNone, kErrTimeoutEpilogue);
      pair_abort(abort_flag);
      atomicExch(g.valid, 0);
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // both producers stopped: the load records are final
  if (warp == 0 && leader && lane == 0) {
    // Both CTAs' loads count on the leader's barriers. A producer loads a stage's (or query
    // buffer's) next phase only once the previous one was consumed, which needs both CTAs' loads,
    // so the two records differ by at most one phase: after an abort the leader supplies the
    // missing arrival (peer loaded, leader did not arm) or the missing bytes (leader armed, peer
    // did not load), then waits (bounded) until every phase with a load in flight has landed.
    const uint32_t peer = map_to_rank(smem_u32(issued), 1);
    for (int s2 = 0; s2 < PK_STAGES + PQ_SLOTS; ++s2) {
      const bool qslot = s2 >= PK_STAGES;
      const int idx = qslot ? PK_MAX_STAGES + (s2 - PK_STAGES) : s2;
      uint64_t* bar = qslot ? q_full + (s2 - PK_STAGES) : full + s2;
      const uint32_t bytes = qslot ? static_cast<uint32_t>(g.num_kb * PQ_SUB_BYTES) : PK_STAGE_BYTES;
      uint32_t np;
      asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(np) : "r"(peer + 4u * idx) : "memory");
      const uint32_t nl = issued[idx];
      if (np == nl + 1) mbar_arrive_expect_tx_u32(smem_u32(bar), bytes);
      else if (nl == np + 1) mbar_complete_tx(bar, bytes);
      const uint32_t n = np > nl ? np : nl;
      if (n > 0) mbar_wait(bar, (n - 1) & 1u);
    }
  }
  if (warp == 1 && leader && lane == 0 && *reinterpret_cast<volatile int*>(abort_flag)) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(drain))
                 : "memory");
    mbar_wait(drain, 0);
  }
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(Q_TMEM_COLS) : "memory");
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
// CTA-pair launch (head dim up to 256): contiguous tile ranges over min(tiles, co-resident pairs).
int qk_max_pair(const void* q, const void* k, int dtype, int64_t batch, int64_t hq, int64_t hkv, int64_t sq,
                int64_t sk, int64_t d, int64_t qsb, int64_t qsh, int64_t qss, int64_t ksb, int64_t ksh, int64_t kss,
                int causal, const int32_t* key_lo, const int32_t* key_hi, int* enc, int32_t* valid,
                cudaStream_t stream) {
  CUtensorMap mq, mk;
  int st = encode_qk_map(&mq, q, dtype, d, sq, hq, batch, qss, qsh, qsb, PQ_ROWS);
  if (st != MUZO_OK) return st;
  st = encode_qk_map(&mk, k, dtype, d, sk, hkv, batch, kss, ksh, ksb, PK_ROWS);
  if (st != MUZO_OK) return st;
  QkPairArgs g;
  g.sq = sq; g.sk = sk; g.shift = sk - sq;
  g.hq = static_cast<int>(hq); g.group = static_cast<int>(hq / hkv);
  g.nqb = static_cast<int>((sq + 2 * PQ_ROWS - 1) / (2 * PQ_ROWS));
  g.causal = causal;
  g.num_kb = static_cast<int>((d + QBK - 1) / QBK);
  g.k_stages = (PQK_TILE_BYTES - PQ_SLOTS * g.num_kb * PQ_SUB_BYTES) / PK_STAGE_BYTES;
  if (g.k_stages > PK_MAX_STAGES) g.k_stages = PK_MAX_STAGES;
  int64_t per = 0;
  for (int qb = 0; qb < g.nqb; ++qb) {
    int64_t end = sk;
    if (causal) {
      const int64_t last = static_cast<int64_t>(qb + 1) * 2 * PQ_ROWS + g.shift;
      end = last < sk ? last : sk;
      if (end < 0) end = 0;
    }
    per += (end + 2 * PK_ROWS - 1) / (2 * PK_ROWS);
  }
  g.tiles_per_bh = per;
  g.num_tiles = per * batch * hq;
  g.key_lo = key_lo;
  g.key_hi = key_hi;
  g.enc = enc;
  g.valid = valid;
  void* p = nullptr;
  MUZO_CUDA_CHECK(cudaGetSymbolAddress(&p, g_qk_status));
  g.status = static_cast<int32_t*>(p);
  if (g.num_tiles == 0) return MUZO_OK;
  auto kern = dtype == MUZO_BF16 ? qk_max_pair_kernel<1> : qk_max_pair_kernel<0>;
  static std::atomic<int> max_pairs[2][64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return MUZO_ERR_UNSUPPORTED;
  const int fi = dtype == MUZO_BF16 ? 1 : 0;
  if (max_pairs[fi][dev].load(std::memory_order_acquire) == 0) {
    MUZO_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, PQK_SMEM_BYTES));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(2 * (device_sm_count() / 2)), 1, 1);
    cfg.blockDim = dim3(PQK_THREADS, 1, 1);
    cfg.dynamicSmemBytes = PQK_SMEM_BYTES;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) != cudaSuccess || clusters <= 0) {
      cudaGetLastError();
      clusters = device_sm_count() / 2;
    }
    max_pairs[fi][dev].store(clusters, std::memory_order_release);
  }
  const int64_t cap = max_pairs[fi][dev].load(std::memory_order_acquire);
  const int64_t pairs = g.num_tiles < cap ? g.num_tiles : cap;
  kern<<<static_cast<unsigned>(2 * pairs), PQK_THREADS, PQK_SMEM_BYTES, stream>>>(mq, mk, g);
  return launch_status();
}

int qk_max_tensor_cores(const void* q, const void* k, int dtype, int64_t batch, int64_t hq, int64_t hkv, int64_t sq,
                        int64_t sk, int64_t d, int64_t qsb, int64_t qsh, int64_t qss, int64_t ksb, int64_t ksh,
                        int64_t kss, int causal, const int32_t* key_lo, const int32_t* key_hi, int* enc,
                        int32_t* valid, cudaStream_t stream) {
  const char* pv = std::getenv("MUZO_QK_PAIR");
  if (d <= PQ_MAX_KB * QBK && !(pv != nullptr && pv[0] == '0'))
    return qk_max_pair(q, k, dtype, batch, hq, hkv, sq, sk, d, qsb, qsh, qss, ksb, ksh, kss, causal, key_lo, key_hi,
                       enc, valid, stream);
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
  g.key_lo = key_lo;
  g.key_hi = key_hi;
  g.enc = enc;
  g.valid = valid;
  void* p = nullptr;
  MUZO_CUDA_CHECK(cudaGetSymbolAddress(&p, g_qk_status));
  g.status = static_cast<int32_t*>(p);
  if (g.num_tiles == 0) return MUZO_OK;
  auto kern = dtype == MUZO_BF16 ? qk_max_tc_kernel<1> : qk_max_tc_kernel<0>;
  static std::atomic<bool> configured[2][64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  const int fi = dtype == MUZO_BF16 ? 1 : 0;
  if (dev >= 0 && dev < 64 && !configured[fi][dev].load(std::memory_order_acquire)) {
    MUZO_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Q_SMEM_BYTES));
    configured[fi][dev].store(true, std::memory_order_release);
  }
  const int64_t grid = g.num_tiles < device_sm_count() ? g.num_tiles : device_sm_count();
  kern<<<static_cast<unsigned>(grid), Q_THREADS, Q_SMEM_BYTES, stream>>>(mq, mk, g);
  return launch_status();
}

}  // namespace muzo
