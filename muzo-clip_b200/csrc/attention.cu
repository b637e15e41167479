// Attention forward on the tensor cores with the per-head maximum of the pre-softmax logits as a
// side output: QK-Clip's capture (qk_clip.py:173-196) computed by the attention that the forward
// runs anyway, so Q K^T is formed once. Forward only (MuZO's forwards run without gradients).
//
// One CTA per (batch, query head, block of 256 queries), 11 warps. The block is two query tiles
// of 128 rows that share every K / V tile of 128 keys, so each K / V byte loaded serves 256 rows:
//   warp 0      TMA producer (one thread): both query tiles once, then K tiles (K-major) into a
//               1-stage ring, refilled once both tiles' S = Q K^T has read it (a stream's next S
//               waits for its softmax anyway, so the load hides behind the softmax);
//   warp 10     TMA producer (one thread): V tiles (MN-major, the second operand of P V) into a
//               2-stage ring, refilled once both tiles' P V has read it;
//   warp 1      TMEM owner and MMA issuer (one thread): per query tile s, S_s = Q_s K_j^T into
//               its S buffer (fp32 in TMEM), then O_s += P_s V_j into its fp32 accumulator, which
//               stays in TMEM;
//   warps 2..9  two softmax streams of four warps, stream s for query tile s, one warp per TMEM
//               lane quarter, one query row per thread, all 128 keys of each tile: the raw
//               logits' maximum (the side output, over visible logits only), the online softmax
//               in base 2 with a lazy rescale (O and the row sum are rescaled only when the row
//               maximum grows by more than 2^8), P in bf16/fp16 written to shared memory in the
//               128-byte swizzled K-major layout the MMA reads, and at the end O / l stored to
//               [B, Sq, Hq, D]. The streams run side by side without waiting for each other.
// Visibility: key j of batch b is visible to query i when key_lo[b] <= j < key_hi[b] (padding)
// and, when causal, j <= i + Sk - Sq. Rows without a visible key are written as zeros.
// Every wait is bounded; on timeout the kernel records a code in the status word, raises its
// abort flag, drains its loads and MMAs, frees TMEM and returns.
#include <atomic>
#include <cstdlib>

#include "tcgen05_common.cuh"

namespace muzo {
namespace {

using namespace tc;

constexpr int AM = 128;          // query rows per query tile (UMMA M)
constexpr int AMB = 2 * AM;      // query rows per CTA: two query tiles share each K / V tile
constexpr int AN = 128;          // keys per tile: UMMA N of S, the K of P V
constexpr int ABK = 64;          // 128-byte swizzle row of 16-bit elements
constexpr int A_THREADS = 352;   // warp 0 TMA of Q and K, warp 1 MMA, warps 2..9 softmax (two streams
                                 // of four warps, one warp per TMEM lane quarter), warp 10 TMA of V
constexpr int K_STAGES = 1;      // K ring depth (tile j uses K stage j % K_STAGES)
constexpr int SUB_BYTES = 128 * ABK * 2;     // one swizzled block of 128 rows x 64 elements (16 KB)
constexpr int BOX_BYTES = 64 * ABK * 2;      // one 64 x 64 box of the MN-major V operand (8 KB)
constexpr uint32_t TMEM_COLS = 512;          // S of each stream at 0 and 128, O of each stream from 256
constexpr float kRescaleLog2 = 8.0f;          // lazy rescale threshold: P stays below 2^8

template <int D>
struct AttnLayout {
  static constexpr int Q_BYTES = (D / ABK) * SUB_BYTES;
  static constexpr int K_BYTES = (D / ABK) * SUB_BYTES;
  static constexpr int V_BYTES = 2 * (D / ABK) * BOX_BYTES;
  static constexpr int P_BYTES = 2 * SUB_BYTES;   // one 128 x 128 P tile per stream
  // V ring depth: two stages next to two Q tiles, one K stage and two P tiles (224 KB for D = 128)
  static constexpr int V_STAGES = 2;
  static constexpr int TILES_BYTES = 2 * Q_BYTES + K_STAGES * K_BYTES + V_STAGES * V_BYTES + 2 * P_BYTES;
  static constexpr int BAR_BYTES = 256;           // barriers, TMEM address, flags
  // tiles, barriers and 1 KB of alignment (225.25 KB for D = 128, within the 227 KB a CTA may
  // use); at least 116 KB so that one CTA holds an SM (every CTA allocates all 512 TMEM columns)
  static constexpr int NEED = TILES_BYTES + BAR_BYTES + 1024;
  static constexpr int SMEM_BYTES = NEED > 116 * 1024 ? NEED : 116 * 1024;
};

struct AttnArgs {
  int64_t sq, sk, shift;       // shift = Sk - Sq: causal key j is visible to query i when j <= i + shift
  int hq, group, nqb, causal, batch;
  int64_t num_items;           // batch * hq * nqb
  float scale_log2;            // softmax scale * log2(e)
  const int32_t* key_lo;       // per batch, or null (0)
  const int32_t* key_hi;       // per batch, or null (Sk)
  void* out;
  int64_t o_sb, o_sh, o_ss;    // output strides in elements; D contiguous
  int* enc;                    // per-head running maximum of the raw logits (order-preserving ints), or null
  int32_t* valid;
  int32_t* status;
};

__device__ __forceinline__ int encode_max(float f) {
  const int b = __float_as_int(f);
  return b >= 0 ? b : b ^ 0x7fffffff;
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Work item -> (batch, head, block of 256 queries); the longest query blocks (last, when causal) first.
__device__ __forceinline__ void attn_item(const AttnArgs& g, int64_t t, int& b, int& h, int& qb) {
  const int64_t bh_count = static_cast<int64_t>(g.batch) * g.hq;
  qb = g.nqb - 1 - static_cast<int>(t / bh_count);
  const int64_t bh = t % bh_count;
  b = static_cast<int>(bh / g.hq);
  h = static_cast<int>(bh % g.hq);
}

// First key tile of a work item and the tile counts of its two query tiles (zero for a tile with
// no row inside the sequence or no visible key).
__device__ __forceinline__ void attn_tiles(const AttnArgs& g, int b, int qb, int64_t& lo, int64_t& hi, int& t0,
                                           int& n0, int& n1) {
  lo = g.key_lo ? g.key_lo[b] : 0;
  hi = g.key_hi ? g.key_hi[b] : g.sk;
  if (lo < 0) lo = 0;
  if (hi > g.sk) hi = g.sk;
  t0 = static_cast<int>(lo / AN);
  int n[2];
  for (int t = 0; t < 2; ++t) {
    const int64_t first = static_cast<int64_t>(qb) * AMB + t * AM;   // first row of query tile t
    n[t] = 0;
    if (first >= g.sq) continue;
    const int64_t last_row = first + AM - 1 < g.sq - 1 ? first + AM - 1 : g.sq - 1;
    int64_t end = hi;
    if (g.causal && last_row + g.shift + 1 < end) end = last_row + g.shift + 1;  // keys the tile's last row sees
    if (end > lo) n[t] = static_cast<int>((end + AN - 1) / AN) - t0;
  }
  n0 = n[0];
  n1 = n[1];
}

// Three-input maximum (NaN-propagating) and minimum (sm_100).
__device__ __forceinline__ float max3_nan(float a, float b, float c) {
  float d;
  asm("max.NaN.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
__device__ __forceinline__ float min3(float a, float b, float c) {
  float d;
  asm("min.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

template <int FMT, int D>
__global__ void __launch_bounds__(A_THREADS, 1)
attn_fwd_max_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                    const __grid_constant__ CUtensorMap map_v, AttnArgs g) {
  using L = AttnLayout<D>;
  constexpr int NKB = D / ABK;   // 64-wide slices of the head dimension
  constexpr int VS = L::V_STAGES;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  // Two query tiles of 128 rows (streams 0 and 1) share every K / V tile of 128 keys: K through a
  // 2-stage ring (a stage is free once both tiles' S has read it), V through a VS-stage ring (free
  // once both tiles' P V has read it). Each stream owns an S buffer and an O accumulator in TMEM
  // and a P tile in shared memory.
  uint8_t* sQ = smem;                                   // [2][NKB][128 x 64]
  uint8_t* sK = sQ + 2 * L::Q_BYTES;
  uint8_t* sV = sK + K_STAGES * L::K_BYTES;
  uint8_t* sP = sV + VS * L::V_BYTES;
  uint64_t* q_full = reinterpret_cast<uint64_t*>(smem + L::TILES_BYTES);
  uint64_t* k_full = q_full + 1;
  uint64_t* k_empty = k_full + K_STAGES;
  uint64_t* v_full = k_empty + K_STAGES;
  uint64_t* v_empty = v_full + VS;
  uint64_t* s_full = v_empty + VS;          // [stream]: S of the stream's next tile computed
  uint64_t* p_full = s_full + 2;            // [stream]: P written (and S read) by the stream's 4 warps
  uint64_t* o_done = p_full + 2;            // [stream]: P V of the stream's last tile done
  uint64_t* drain = o_done + 2;
  uint64_t* stall_bar = drain + 1;          // nothing arrives here: a stall request waits on it
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(stall_bar + 1);
  int* abort_flag = reinterpret_cast<int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int b, h, qb;
  attn_item(g, blockIdx.x, b, h, qb);
  int64_t lo, hi;
  int t0, n0, n1;
  attn_tiles(g, b, qb, lo, hi, t0, n0, n1);
  const int ntiles = n0 > n1 ? n0 : n1;   // K / V tiles loaded (stream 1's rows come later: n1 >= n0)
  const int kvh = h / g.group;
  // status word 1: a role (1 producer, 2 MMA, 3 softmax) whose first wait is made to expire
  const int stall = *reinterpret_cast<volatile int*>(g.status + 1);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < K_STAGES; ++s) { mbar_init(k_full + s, 1); mbar_init(k_empty + s, 1); }
    for (int s = 0; s < VS; ++s) { mbar_init(v_full + s, 1); mbar_init(v_empty + s, 1); }
    for (int s = 0; s < 2; ++s) { mbar_init(s_full + s, 1); mbar_init(p_full + s, 4); mbar_init(o_done + s, 1); }
    mbar_init(drain, 1);
    mbar_init(stall_bar, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_holder)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  const uint32_t tmem_o = tmem_base + 2 * AN;   // O of stream s at tmem_o + s * D

  if (warp == 0 || warp == 10) {
    // ------------------------------------------------------------------ TMA producers
    // warp 0: both query tiles once, then K_j into K stage j % 2 once S_{j-2} of both streams has
    // read it; warp 10: V_j into V stage j % VS once P_{j-VS} V_{j-VS} of both streams has read it
    if (lane == 0 && ntiles > 0) {
      const bool keys = warp == 0;
      const int stages = keys ? K_STAGES : VS;
      uint64_t* full = keys ? k_full : v_full;
      uint64_t* empty = keys ? k_empty : v_empty;
      const uint32_t stage_bytes = keys ? L::K_BYTES : L::V_BYTES;
      bool ok = !(keys && stall == kErrTimeoutProducer && !mbar_wait(stall_bar, 0, kStallLimitCycles));
      if (keys && ok) {
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_q)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_k)) : "memory");
        mbar_arrive_expect_tx(q_full, 2 * L::Q_BYTES);
        for (int t = 0; t < 2; ++t)
          for (int kb = 0; kb < NKB; ++kb)
            tma_load_4d(&map_q, q_full, sQ + t * L::Q_BYTES + kb * SUB_BYTES, kb * ABK, qb * AMB + t * AM, h, b);
      } else if (!keys) {
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_v)) : "memory");
      }
      const bool q_armed = keys && ok;
      uint32_t armed = 0, armed_parity = 0;
      for (int j = 0; j < ntiles && ok; ++j) {
        const int stage = j % stages;
        const uint32_t phase = static_cast<uint32_t>((j / stages) & 1);
        if (!mbar_wait(empty + stage, phase ^ 1)) { ok = false; break; }
        if (*reinterpret_cast<volatile int*>(abort_flag)) { ok = false; break; }
        mbar_arrive_expect_tx(full + stage, stage_bytes);
        armed |= 1u << stage;
        armed_parity = (armed_parity & ~(1u << stage)) | (phase << stage);
        const int key0 = (t0 + j) * AN;
        if (keys) {
          uint8_t* dst = sK + stage * L::K_BYTES;
          for (int kb = 0; kb < NKB; ++kb) tma_load_4d(&map_k, full + stage, dst + kb * SUB_BYTES, kb * ABK, key0, kvh, b);
        } else {
          uint8_t* dst = sV + stage * L::V_BYTES;
          for (int kc = 0; kc < 2; ++kc)
            for (int dc = 0; dc < NKB; ++dc)
              tma_load_4d(&map_v, full + stage, dst + (kc * NKB + dc) * BOX_BYTES, dc * ABK, key0 + kc * 64, kvh, b);
        }
      }
      if (!ok) {
        atomicCAS(g.status, kErrNone, kErrTimeoutProducer);
        atomicExch(abort_flag, 1);
        if (g.valid) atomicExch(g.valid, 0);
      }
      // every load of this CTA must have landed before it may exit (bounded)
      if (q_armed) mbar_wait(q_full, 0);
      for (int s2 = 0; s2 < stages; ++s2)
        if (armed & (1u << s2)) mbar_wait(full + s2, (armed_parity >> s2) & 1u);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    // S_s(0) for both streams; then per tile j and stream s (in that order): once P_s(j) is
    // written (S buffer s read), S_s(j + 1) and then O_s += P_s(j) V_j. A K stage is released after
    // the last S that reads it, a V stage after the last P V.
    if (lane == 0 && ntiles > 0) {
      constexpr uint32_t idesc_s = make_idesc_fmt(AM, AN, false, false, FMT);
      constexpr uint32_t idesc_pv = make_idesc_fmt(AM, D, false, true, FMT);
      const int nt[2] = {n0, n1};
      auto issue_s = [&](int s, int j) -> bool {
        const int stage = j % K_STAGES;
        if (!mbar_wait(k_full + stage, static_cast<uint32_t>((j / K_STAGES) & 1))) return false;
        if (*reinterpret_cast<volatile int*>(abort_flag)) return false;
        tc_fence_after();
        const uint32_t sq_ = smem_u32(sQ + s * L::Q_BYTES);
        const uint32_t sk_ = smem_u32(sK + stage * L::K_BYTES);
#pragma unroll
        for (int kb = 0; kb < NKB; ++kb)
#pragma unroll
          for (int k = 0; k < ABK / 16; ++k)
            umma_f16(tmem_base + s * AN, make_sdesc(sq_ + kb * SUB_BYTES + k * 32, 16, 1024),
                     make_sdesc(sk_ + kb * SUB_BYTES + k * 32, 16, 1024), idesc_s, (kb > 0 || k > 0) ? 1u : 0u);
        umma_commit(s_full + s);
        // the last stream that reads K_j (stream 1 whenever it has tile j) releases the stage
        if (s == 1 || j >= nt[1]) umma_commit(k_empty + stage);
        return true;
      };
      auto issue_pv = [&](int s, int j) -> bool {
        const int stage = j % VS;
        if (!mbar_wait(v_full + stage, static_cast<uint32_t>((j / VS) & 1))) return false;
        if (*reinterpret_cast<volatile int*>(abort_flag)) return false;
        tc_fence_after();
        const uint32_t sv = smem_u32(sV + stage * L::V_BYTES);
        const uint32_t sp = smem_u32(sP + s * L::P_BYTES);
#pragma unroll
        for (int kc = 0; kc < 2; ++kc)
#pragma unroll
          for (int k = 0; k < ABK / 16; ++k)
            umma_f16(tmem_o + s * D, make_sdesc(sp + kc * SUB_BYTES + k * 32, 16, 1024),
                     make_sdesc(sv + kc * NKB * BOX_BYTES + k * (16 * 128), BOX_BYTES, 1024), idesc_pv,
                     (j > 0 || kc > 0 || k > 0) ? 1u : 0u);
        if (s == 1 || j >= nt[1]) umma_commit(v_empty + stage);   // V_j read by both streams
        umma_commit(o_done + s);        // P buffer of the stream free, O_s holds its tiles up to j
        return true;
      };
      bool ok = stall != kErrTimeoutMma || mbar_wait(stall_bar, 0, kStallLimitCycles);
      ok = ok && mbar_wait(q_full, 0);
      for (int s = 0; s < 2 && ok; ++s)
        if (nt[s] > 0) ok = issue_s(s, 0);
      for (int j = 0; j < ntiles && ok; ++j) {
        for (int s = 0; s < 2 && ok; ++s) {
          if (j >= nt[s]) continue;
          if (!mbar_wait(p_full + s, static_cast<uint32_t>(j & 1))) { ok = false; break; }
          tc_fence_after();
          if (j + 1 < nt[s] && !issue_s(s, j + 1)) { ok = false; break; }
          if (!issue_pv(s, j)) { ok = false; break; }
        }
      }
      if (!ok) {
        atomicCAS(g.status, kErrNone, kErrTimeoutMma);
        atomicExch(abort_flag, 1);
        if (g.valid) atomicExch(g.valid, 0);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ softmax streams and epilogue
    // Stream s (warps 2..5: s = 0, warps 6..9: s = 1) owns query tile s of the block: one warp per
    // TMEM lane quarter, one query row per thread, all 128 keys of each tile. The two streams run
    // side by side on the same K / V tiles without waiting for each other.
    const int quarter = warp & 3;
    const int stream = (warp - 2) >> 2;
    const int r = 32 * quarter + lane;                 // row of the tile == TMEM lane
    const int64_t row = static_cast<int64_t>(qb) * AMB + stream * AM + r;
    const bool row_in = row < g.sq;
    const int64_t jmax = g.causal ? row + g.shift : g.sk - 1;  // last key visible by causality
    const uint32_t lane_addr = static_cast<uint32_t>(32 * quarter) << 16;
    const uint32_t s_cols = tmem_base + lane_addr + stream * AN;
    const uint32_t o_cols = tmem_o + lane_addr + stream * D;
    uint8_t* my_p = sP + stream * L::P_BYTES;
    const int n_mine = stream == 0 ? n0 : n1;
    float m_run = -INFINITY;    // running maximum of the scaled logits (log2 units) used by P
    float l_run = 0.0f;         // running sum of P
    float raw_max = -INFINITY;  // side output: maximum of the visible raw logits q . k (NaN-propagating)
    float raw_min = INFINITY;   // a visible -inf logit shows here
    bool ok = true;
    if (stall == kErrTimeoutEpilogue) {
      bool waited = true;
      if (lane == 0) waited = mbar_wait(stall_bar, 0, kStallLimitCycles);
      ok = __shfl_sync(0xffffffffu, waited ? 1 : 0, 0) != 0;
    }
    for (int u = 0; u < n_mine && ok; ++u) {
      bool ready = true;
      if (lane == 0) ready = mbar_wait(s_full + stream, static_cast<uint32_t>(u & 1));
      ready = __shfl_sync(0xffffffffu, ready ? 1 : 0, 0) != 0;
      if (!ready || *reinterpret_cast<volatile int*>(abort_flag)) { ok = false; break; }
      tc_fence_after();
      // visible key columns [c_lo, c_hi) of this tile for this row
      const int64_t key0 = static_cast<int64_t>(t0 + u) * AN;
      const int64_t end = hi < jmax + 1 ? hi : jmax + 1;
      int c_lo = 0, c_hi = 0;
      if (row_in) {
        const int64_t a0 = lo - key0, a1 = end - key0;
        c_lo = a0 < 0 ? 0 : (a0 > AN ? AN : static_cast<int>(a0));
        c_hi = a1 < 0 ? 0 : (a1 > AN ? AN : static_cast<int>(a1));
        if (c_hi < c_lo) c_hi = c_lo;
      }
      const bool all_visible = c_lo == 0 && c_hi == AN;
      // pass 1: the tile's maximum and minimum over the visible logits
      float mx[4], mn[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) { mx[q] = -INFINITY; mn[q] = INFINITY; }
#pragma unroll
      for (int ch = 0; ch < 2; ++ch) {
        uint32_t v[64];
        tmem_ld64(s_cols + ch * 64, v);
        if (all_visible) {
#pragma unroll
          for (int c = 0; c < 64; c += 2) {
            const float x0 = __uint_as_float(v[c]), x1 = __uint_as_float(v[c + 1]);
            mx[(c >> 1) & 3] = max3_nan(mx[(c >> 1) & 3], x0, x1);
            mn[(c >> 1) & 3] = min3(mn[(c >> 1) & 3], x0, x1);
          }
        } else {
#pragma unroll
          for (int c = 0; c < 64; c += 2) {
            const int k0 = ch * 64 + c;
            const bool v0 = k0 >= c_lo && k0 < c_hi, v1 = k0 + 1 >= c_lo && k0 + 1 < c_hi;
            const float x0 = __uint_as_float(v[c]), x1 = __uint_as_float(v[c + 1]);
            mx[(c >> 1) & 3] = max3_nan(mx[(c >> 1) & 3], v0 ? x0 : -INFINITY, v1 ? x1 : -INFINITY);
            mn[(c >> 1) & 3] = min3(mn[(c >> 1) & 3], v0 ? x0 : INFINITY, v1 ? x1 : INFINITY);
          }
        }
      }
      const float mt = max3_nan(max3_nan(mx[0], mx[1], mx[2]), mx[3], -INFINITY);
      raw_max = max3_nan(raw_max, mt, -INFINITY);
      raw_min = min3(min3(raw_min, mn[0], mn[1]), mn[2], mn[3]);
      // lazy online softmax in base 2
      const float mt2 = mt * g.scale_log2;
      float alpha = 1.0f;
      bool rescale = false;
      if (mt2 > m_run + kRescaleLog2) {
        alpha = m_run == -INFINITY ? 0.0f : fast_exp2(m_run - mt2);
        rescale = u > 0;
        m_run = mt2;
      }
      // P V of this stream's previous tile must be done: its P buffer is reused and O may be rescaled
      if (u > 0) {
        bool done = true;
        if (lane == 0) done = mbar_wait(o_done + stream, static_cast<uint32_t>((u - 1) & 1));
        done = __shfl_sync(0xffffffffu, done ? 1 : 0, 0) != 0;
        if (!done) { ok = false; break; }
        tc_fence_after();
      }
      if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t v[32];
          tmem_ld32(o_cols + c * 32, v);
          if (rescale) {
#pragma unroll
            for (int e = 0; e < 32; ++e) v[e] = __float_as_uint(__uint_as_float(v[e]) * alpha);
          }
          tmem_st32(o_cols + c * 32, v);
        }
      }
      // pass 2: P = 2^(s * scale_log2 - m_run), its row sum, and P in the 128-byte swizzled K-major
      // layout (chunk c16 of 8 keys of K block ch sits at row * 128 + ((c16 ^ (row & 7)) * 16))
      const float nm = -m_run;
      float lsum[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) lsum[q] = 0.0f;
#pragma unroll
      for (int ch = 0; ch < 2; ++ch) {
        uint32_t v[64];
        tmem_ld64(s_cols + ch * 64, v);
        uint32_t packed[32];
        if (m_run == -INFINITY) {
#pragma unroll
          for (int c = 0; c < 32; ++c) packed[c] = 0u;
        } else if (all_visible) {
#pragma unroll
          for (int c = 0; c < 64; c += 2) {
            const float p0 = fast_exp2(fmaf(__uint_as_float(v[c]), g.scale_log2, nm));
            const float p1 = fast_exp2(fmaf(__uint_as_float(v[c + 1]), g.scale_log2, nm));
            lsum[(c >> 1) & 3] += p0;
            lsum[((c >> 1) & 3) + 4] += p1;
            packed[c >> 1] = FMT == 1 ? pack_bf16(p0, p1) : pack_half(p0, p1);
          }
        } else {
#pragma unroll
          for (int c = 0; c < 64; c += 2) {
            const int k0 = ch * 64 + c;
            const float x0 = (k0 >= c_lo && k0 < c_hi) ? __uint_as_float(v[c]) : -INFINITY;
            const float x1 = (k0 + 1 >= c_lo && k0 + 1 < c_hi) ? __uint_as_float(v[c + 1]) : -INFINITY;
            const float p0 = fast_exp2(fmaf(x0, g.scale_log2, nm));
            const float p1 = fast_exp2(fmaf(x1, g.scale_log2, nm));
            lsum[(c >> 1) & 3] += p0;
            lsum[((c >> 1) & 3) + 4] += p1;
            packed[c >> 1] = FMT == 1 ? pack_bf16(p0, p1) : pack_half(p0, p1);
          }
        }
#pragma unroll
        for (int c16 = 0; c16 < 8; ++c16) {
          uint8_t* dst = my_p + ch * SUB_BYTES + r * 128 + ((c16 ^ (r & 7)) << 4);
          *reinterpret_cast<uint4*>(dst) =
              make_uint4(packed[4 * c16], packed[4 * c16 + 1], packed[4 * c16 + 2], packed[4 * c16 + 3]);
        }
      }
      l_run = l_run * alpha + (((lsum[0] + lsum[1]) + (lsum[2] + lsum[3])) + ((lsum[4] + lsum[5]) + (lsum[6] + lsum[7])));
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full + stream);
    }
    // this stream's last P V must be done before O_s is read
    if (ok && n_mine > 0) {
      bool done = true;
      if (lane == 0) done = mbar_wait(o_done + stream, static_cast<uint32_t>((n_mine - 1) & 1));
      done = __shfl_sync(0xffffffffu, done ? 1 : 0, 0) != 0;
      if (!done) ok = false;
      tc_fence_after();
    }
    if (ok) {
      // O / l of this row (zeros for a row without a visible key or a tile without one)
      const float inv = l_run > 0.0f ? 1.0f / l_run : 0.0f;
      uint16_t* orow = reinterpret_cast<uint16_t*>(g.out) + static_cast<int64_t>(b) * g.o_sb +
                       static_cast<int64_t>(h) * g.o_sh + row * g.o_ss;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t v[32];
        if (n_mine > 0) {
          tmem_ld32(o_cols + c * 32, v);
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) v[e] = 0u;
        }
        if (row_in) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint32_t w[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float o0 = __uint_as_float(v[8 * q + 2 * e]) * inv;
              const float o1 = __uint_as_float(v[8 * q + 2 * e + 1]) * inv;
              w[e] = FMT == 1 ? pack_bf16(o0, o1) : pack_half(o0, o1);
            }
            *reinterpret_cast<uint4*>(orow + c * 32 + 8 * q) = make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
      }
      if (g.enc != nullptr) {
        float m = raw_max;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = max3_nan(m, __shfl_xor_sync(0xffffffffu, m, o), -INFINITY);
        float mnv = raw_min;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mnv = fminf(mnv, __shfl_xor_sync(0xffffffffu, mnv, o));
        if (lane == 0) {
          if (m != m || m == INFINITY || mnv == -INFINITY) atomicExch(g.valid, 0);
          else if (m > -INFINITY) atomicMax(g.enc + h, encode_max(m));
        }
      }
    } else if (lane == 0) {
      atomicCAS(g.status, kErrNone, kErrTimeoutEpilogue);
      atomicExch(abort_flag, 1);
      if (g.valid) atomicExch(g.valid, 0);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    if (lane == 0 && *reinterpret_cast<volatile int*>(abort_flag)) {
      // drain the MMAs an aborted CTA issued before its TMEM is released (bounded)
      umma_commit(drain);
      mbar_wait(drain, 0);
    }
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS)
                 : "memory");
  }
}

// 4-D tensor map over [B][H][S][D] (element strides ss, sh, sb; D contiguous), box 64 x rows.
int encode_attn_map(CUtensorMap* map, const void* base, int dtype, int64_t d, int64_t s, int64_t h, int64_t b,
                    int64_t ss, int64_t sh, int64_t sb, int rows) {
  auto fn = encode_fn();
  if (fn == nullptr) return MUZO_ERR_UNSUPPORTED;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(d), static_cast<cuuint64_t>(s), static_cast<cuuint64_t>(h),
                        static_cast<cuuint64_t>(b)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(ss * 2), static_cast<cuuint64_t>(sh * 2),
                           static_cast<cuuint64_t>(sb * 2)};
  cuuint32_t box[4] = {ABK, static_cast<cuuint32_t>(rows), 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUtensorMapDataType dt = dtype == MUZO_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult res = fn(map, dt, 4, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return res == CUDA_SUCCESS ? MUZO_OK : MUZO_ERR_ARG;
}

template <int FMT, int D>
int launch_attn(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const AttnArgs& g,
                cudaStream_t s) {
  auto kern = attn_fwd_max_kernel<FMT, D>;
  static std::atomic<bool> configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return MUZO_ERR_UNSUPPORTED;
  if (!configured[dev].load(std::memory_order_acquire)) {
    MUZO_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, AttnLayout<D>::SMEM_BYTES));
    configured[dev].store(true, std::memory_order_release);
  }
  kern<<<static_cast<unsigned>(g.num_items), A_THREADS, AttnLayout<D>::SMEM_BYTES, s>>>(mq, mk, mv, g);
  return launch_status();
}

__global__ void init_attn_max_kernel(int* enc, int n, int32_t* valid) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) enc[i] = encode_max(-INFINITY);
  if (i == 0) *valid = 1;
}

// smax[h] = dtype(dtype(max raw logit) * scale), the eager logit's rounding (monotonic, so the
// rounded maximum is the maximum of the rounded logits); heads without a visible logit stay -inf.
__global__ void finalize_attn_max_kernel(int* enc, int n, int dtype, float scale) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int e = enc[i];
  float v = __int_as_float(e >= 0 ? e : e ^ 0x7fffffff);
  if (v > -INFINITY) v = round_to(round_to(v, dtype) * scale, dtype);
  reinterpret_cast<float*>(enc)[i] = v;
}

bool aligned16p(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace
}  // namespace muzo

using namespace muzo;

extern "C" {

int muzo_attention_max(const void* q, const void* k, const void* v, void* out, int dtype, int64_t batch,
                       int64_t hq, int64_t hkv, int64_t seq_q, int64_t seq_k, int64_t head_dim,
                       int64_t q_stride_b, int64_t q_stride_h, int64_t q_stride_s,
                       int64_t k_stride_b, int64_t k_stride_h, int64_t k_stride_s,
                       int64_t v_stride_b, int64_t v_stride_h, int64_t v_stride_s,
                       int64_t o_stride_b, int64_t o_stride_h, int64_t o_stride_s, int causal, float scale,
                       const int32_t* d_key_lo, const int32_t* d_key_hi, float* smax, int32_t* d_valid,
                       int32_t* d_status, void* stream) {
  if (q == nullptr || k == nullptr || v == nullptr || out == nullptr || d_status == nullptr || batch < 0 ||
      hq <= 0 || hkv <= 0 || hq % hkv != 0 || seq_q < 0 || seq_k < 0 || (smax != nullptr && d_valid == nullptr))
    return MUZO_ERR_ARG;
  if (dtype != MUZO_BF16 && dtype != MUZO_F16) return MUZO_ERR_DTYPE;
  if (head_dim != 64 && head_dim != 128) return MUZO_ERR_UNSUPPORTED;
  const int64_t strides[12] = {q_stride_b, q_stride_h, q_stride_s, k_stride_b, k_stride_h, k_stride_s,
                               v_stride_b, v_stride_h, v_stride_s, o_stride_b, o_stride_h, o_stride_s};
  for (int64_t st : strides)
    if (st % 8 != 0) return MUZO_ERR_ALIGN;
  if (!aligned16p(q) || !aligned16p(k) || !aligned16p(v) || !aligned16p(out)) return MUZO_ERR_ALIGN;
  if (batch > 0x7fffffffLL || hq > 0x7fffffffLL || seq_q > 0x7fffffffLL || seq_k > 0x7fffffffLL)
    return MUZO_ERR_UNSUPPORTED;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int* enc = reinterpret_cast<int*>(smax);
  if (enc != nullptr)
    init_attn_max_kernel<<<static_cast<unsigned>((hq + 255) / 256), 256, 0, s>>>(enc, static_cast<int>(hq), d_valid);
  const int64_t nqb = (seq_q + AMB - 1) / AMB;
  const int64_t items = batch * hq * nqb;
  if (items > 0) {
    if (items > 0x7fffffffLL) return MUZO_ERR_UNSUPPORTED;
    CUtensorMap mq, mk, mv;
    int st = encode_attn_map(&mq, q, dtype, head_dim, seq_q, hq, batch, q_stride_s, q_stride_h, q_stride_b, AM);
    if (st != MUZO_OK) return st;
    st = encode_attn_map(&mk, k, dtype, head_dim, seq_k, hkv, batch, k_stride_s, k_stride_h, k_stride_b, AN);
    if (st != MUZO_OK) return st;
    st = encode_attn_map(&mv, v, dtype, head_dim, seq_k, hkv, batch, v_stride_s, v_stride_h, v_stride_b, 64);
    if (st != MUZO_OK) return st;
    AttnArgs g;
    g.sq = seq_q; g.sk = seq_k; g.shift = seq_k - seq_q;
    g.hq = static_cast<int>(hq); g.group = static_cast<int>(hq / hkv); g.nqb = static_cast<int>(nqb);
    g.causal = causal ? 1 : 0; g.batch = static_cast<int>(batch);
    g.num_items = items;
    g.scale_log2 = scale * 1.4426950408889634f;
    g.key_lo = d_key_lo; g.key_hi = d_key_hi;
    g.out = out; g.o_sb = o_stride_b; g.o_sh = o_stride_h; g.o_ss = o_stride_s;
    g.enc = enc; g.valid = d_valid; g.status = d_status;
    if (dtype == MUZO_BF16)
      st = head_dim == 64 ? launch_attn<1, 64>(mq, mk, mv, g, s) : launch_attn<1, 128>(mq, mk, mv, g, s);
    else
      st = head_dim == 64 ? launch_attn<0, 64>(mq, mk, mv, g, s) : launch_attn<0, 128>(mq, mk, mv, g, s);
    if (st != MUZO_OK) return st;
  }
  if (enc != nullptr)
    finalize_attn_max_kernel<<<static_cast<unsigned>((hq + 255) / 256), 256, 0, s>>>(enc, static_cast<int>(hq), dtype,
                                                                                     scale);
  return launch_status();
}

}  // extern "C"
