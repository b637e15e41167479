// Attention forward on the tensor cores with the per-head maximum of the pre-softmax logits as a
// side output: QK-Clip's capture (qk_clip.py:173-196) computed by the attention that the forward
// runs anyway, so Q K^T is formed once. Forward only (MuZO's forwards run without gradients).
//
// One CTA per (batch, query head, block of 128 queries), 6 warps:
//   warp 0      TMA producer (one thread): the Q block once, then K and V tiles of 128 keys into a
//               2-stage ring (K K-major, V MN-major as the second operand of P V);
//   warp 1      TMEM owner and MMA issuer (one thread): S_j = Q K_j^T (tcgen05.mma, fp32 in TMEM,
//               two S buffers so S_{j+1} is computed while the softmax reads S_j), then
//               O += P_j V_j into an fp32 accumulator that stays in TMEM;
//   warps 2..5  softmax and epilogue, one query row per thread: the raw logits' running maximum
//               (the side output, over visible logits only), the online softmax in base 2 with
//               a lazy rescale (O and the row sum are rescaled only when the row maximum grows by
//               more than 2^8), P in bf16/fp16 written to shared memory in the 128-byte swizzled
//               K-major layout the MMA reads, and at the end O / l stored to [B, Sq, Hq, D].
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

constexpr int AM = 128;          // query rows per CTA (UMMA M)
constexpr int AN = 128;          // keys per tile: UMMA N of S, the K of P V
constexpr int ABK = 64;          // 128-byte swizzle row of 16-bit elements
constexpr int A_THREADS = 320;   // warp 0 TMA, warp 1 MMA, warps 2..9 softmax (two per TMEM lane quarter)
constexpr int KV_STAGES = 2;
constexpr int SUB_BYTES = 128 * ABK * 2;     // one swizzled block of 128 rows x 64 elements (16 KB)
constexpr int BOX_BYTES = 64 * ABK * 2;      // one 64 x 64 box of the MN-major V operand (8 KB)
constexpr uint32_t TMEM_COLS = 512;          // S buffers at 0 and 128, O at 256
constexpr float kRescaleLog2 = 8.0f;          // lazy rescale threshold: P stays below 2^8

template <int D>
struct AttnLayout {
  static constexpr int Q_BYTES = (D / ABK) * SUB_BYTES;
  static constexpr int K_BYTES = (D / ABK) * SUB_BYTES;
  static constexpr int V_BYTES = 2 * (D / ABK) * BOX_BYTES;
  static constexpr int P_BYTES = 2 * SUB_BYTES;
  static constexpr int STAGE_BYTES = K_BYTES + V_BYTES;
  static constexpr int TILES_BYTES = Q_BYTES + KV_STAGES * STAGE_BYTES + P_BYTES;
  // tiles, 1 KB of barriers and flags, 3 KB + 96 B of softmax exchange, 1 KB of alignment; at
  // least 116 KB so that one CTA holds an SM (every CTA allocates all 512 TMEM columns)
  static constexpr int NEED = TILES_BYTES + 1024 + 6 * AM * 4 + 24 * 4 + 1024;
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

// Work item -> (batch, head, query block); the longest query blocks (last, when causal) first.
__device__ __forceinline__ void attn_item(const AttnArgs& g, int64_t t, int& b, int& h, int& qb) {
  const int64_t bh_count = static_cast<int64_t>(g.batch) * g.hq;
  qb = g.nqb - 1 - static_cast<int>(t / bh_count);
  const int64_t bh = t % bh_count;
  b = static_cast<int>(bh / g.hq);
  h = static_cast<int>(bh % g.hq);
}

// First key tile and tile count of a work item.
__device__ __forceinline__ void attn_tiles(const AttnArgs& g, int b, int qb, int64_t& lo, int64_t& hi, int& t0,
                                           int& ntiles) {
  lo = g.key_lo ? g.key_lo[b] : 0;
  hi = g.key_hi ? g.key_hi[b] : g.sk;
  if (lo < 0) lo = 0;
  if (hi > g.sk) hi = g.sk;
  int64_t end = hi;
  if (g.causal) {
    const int64_t last = static_cast<int64_t>(qb) * AM + AM - 1 + g.shift + 1;  // keys the block's last row sees
    if (last < end) end = last;
  }
  if (end <= lo) {
    t0 = 0;
    ntiles = 0;
    return;
  }
  t0 = static_cast<int>(lo / AN);
  ntiles = static_cast<int>((end + AN - 1) / AN) - t0;
}

template <int FMT, int D>
__global__ void __launch_bounds__(A_THREADS, 1)
attn_fwd_max_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                    const __grid_constant__ CUtensorMap map_v, AttnArgs g) {
  using L = AttnLayout<D>;
  constexpr int NKB = D / ABK;   // 64-wide slices of the head dimension
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  uint8_t* sQ = smem;
  uint8_t* sKV = sQ + L::Q_BYTES;
  uint8_t* sP = sKV + KV_STAGES * L::STAGE_BYTES;
  uint64_t* q_full = reinterpret_cast<uint64_t*>(smem + L::TILES_BYTES);
  uint64_t* kv_full = q_full + 1;
  uint64_t* kv_empty = kv_full + KV_STAGES;
  uint64_t* s_full = kv_empty + KV_STAGES;
  uint64_t* s_empty = s_full + 2;
  uint64_t* p_full = s_empty + 2;
  uint64_t* o_done = p_full + 1;
  uint64_t* drain = o_done + 1;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);
  int* abort_flag = reinterpret_cast<int*>(tmem_holder + 1);
  // softmax pair exchange: row maxima [2 tile parities][2 halves][128 rows], then the row sums
  // [2 halves][128 rows]; each warp's "still running" word [2 parities][2 halves][4 quarters],
  // then the final one [2 halves][4 quarters]
  float* red_max = reinterpret_cast<float*>(smem + L::TILES_BYTES + 1024);
  int* red_ok = reinterpret_cast<int*>(red_max + 6 * AM);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int b, h, qb;
  attn_item(g, blockIdx.x, b, h, qb);
  int64_t lo, hi;
  int t0, ntiles;
  attn_tiles(g, b, qb, lo, hi, t0, ntiles);
  const int kvh = h / g.group;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < KV_STAGES; ++s) { mbar_init(kv_full + s, 1); mbar_init(kv_empty + s, 1); }
    for (int s = 0; s < 2; ++s) { mbar_init(s_full + s, 1); mbar_init(s_empty + s, 8); }
    mbar_init(p_full, 8);
    mbar_init(o_done, 1);
    mbar_init(drain, 1);
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
  const uint32_t tmem_o = tmem_base + 2 * AN;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0 && ntiles > 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_q)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_k)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_v)) : "memory");
      mbar_arrive_expect_tx(q_full, L::Q_BYTES);
      for (int kb = 0; kb < NKB; ++kb) tma_load_4d(&map_q, q_full, sQ + kb * SUB_BYTES, kb * ABK, qb * AM, h, b);
      bool ok = true;
      uint32_t armed = 0, armed_parity = 0;
      for (int j = 0; j < ntiles; ++j) {
        const int stage = j % KV_STAGES;
        const uint32_t phase = static_cast<uint32_t>((j / KV_STAGES) & 1);
        if (!mbar_wait(kv_empty + stage, phase ^ 1)) { ok = false; break; }
        if (*reinterpret_cast<volatile int*>(abort_flag)) { ok = false; break; }
        uint8_t* sK = sKV + stage * L::STAGE_BYTES;
        uint8_t* sV = sK + L::K_BYTES;
        mbar_arrive_expect_tx(kv_full + stage, L::STAGE_BYTES);
        armed |= 1u << stage;
        armed_parity = (armed_parity & ~(1u << stage)) | (phase << stage);
        const int key0 = (t0 + j) * AN;
        for (int kb = 0; kb < NKB; ++kb) tma_load_4d(&map_k, kv_full + stage, sK + kb * SUB_BYTES, kb * ABK, key0, kvh, b);
        for (int kc = 0; kc < 2; ++kc)
          for (int dc = 0; dc < NKB; ++dc)
            tma_load_4d(&map_v, kv_full + stage, sV + (kc * NKB + dc) * BOX_BYTES, dc * ABK, key0 + kc * 64, kvh, b);
      }
      if (!ok) {
        atomicCAS(g.status, kErrNone, kErrTimeoutProducer);
        atomicExch(abort_flag, 1);
        if (g.valid) atomicExch(g.valid, 0);
      }
      // every load of this CTA must have landed before it may exit (bounded)
      mbar_wait(q_full, 0);
      for (int s2 = 0; s2 < KV_STAGES; ++s2)
        if (armed & (1u << s2)) mbar_wait(kv_full + s2, (armed_parity >> s2) & 1u);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0 && ntiles > 0) {
      constexpr uint32_t idesc_s = make_idesc_fmt(AM, AN, false, false, FMT);
      constexpr uint32_t idesc_pv = make_idesc_fmt(AM, D, false, true, FMT);
      bool ok = mbar_wait(q_full, 0);
      auto issue_pv = [&](int t) -> bool {
        if (!mbar_wait(p_full, static_cast<uint32_t>(t & 1))) return false;
        if (*reinterpret_cast<volatile int*>(abort_flag)) return false;
        tc_fence_after();
        const int stage = t % KV_STAGES;
        const uint32_t sv = smem_u32(sKV + stage * L::STAGE_BYTES + L::K_BYTES);
        const uint32_t sp = smem_u32(sP);
#pragma unroll
        for (int kc = 0; kc < 2; ++kc)
#pragma unroll
          for (int k = 0; k < ABK / 16; ++k)
            umma_f16(tmem_o, make_sdesc(sp + kc * SUB_BYTES + k * 32, 16, 1024),
                     make_sdesc(sv + kc * NKB * BOX_BYTES + k * (16 * 128), BOX_BYTES, 1024), idesc_pv,
                     (t > 0 || kc > 0 || k > 0) ? 1u : 0u);
        umma_commit(kv_empty + stage);  // K_t and V_t read
        umma_commit(o_done);            // P buffer free, O holds tiles 0..t
        return true;
      };
      for (int j = 0; j < ntiles && ok; ++j) {
        const int stage = j % KV_STAGES;
        const uint32_t phase = static_cast<uint32_t>((j / KV_STAGES) & 1);
        const int sb = j & 1;
        const uint32_t sp = static_cast<uint32_t>((j >> 1) & 1);
        if (!mbar_wait(kv_full + stage, phase) || !mbar_wait(s_empty + sb, sp ^ 1)) { ok = false; break; }
        if (*reinterpret_cast<volatile int*>(abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t sq_ = smem_u32(sQ);
        const uint32_t sk_ = smem_u32(sKV + stage * L::STAGE_BYTES);
#pragma unroll
        for (int kb = 0; kb < NKB; ++kb)
#pragma unroll
          for (int k = 0; k < ABK / 16; ++k)
            umma_f16(tmem_base + sb * AN, make_sdesc(sq_ + kb * SUB_BYTES + k * 32, 16, 1024),
                     make_sdesc(sk_ + kb * SUB_BYTES + k * 32, 16, 1024), idesc_s, (kb > 0 || k > 0) ? 1u : 0u);
        umma_commit(s_full + sb);
        if (j > 0 && !issue_pv(j - 1)) { ok = false; break; }
      }
      if (ok) ok = issue_pv(ntiles - 1);
      if (!ok) {
        atomicCAS(g.status, kErrNone, kErrTimeoutMma);
        atomicExch(abort_flag, 1);
        if (g.valid) atomicExch(g.valid, 0);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ softmax and epilogue
    // Two warps per TMEM lane quarter: warp half h takes keys [64 h, 64 h + 64) of every tile,
    // and columns [h D/2, (h + 1) D/2) of O. The pair exchanges its row maxima once per tile
    // through shared memory (named barrier 1 + quarter, 64 threads).
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int r = 32 * quarter + lane;                 // row of the block == TMEM lane
    const int64_t row = static_cast<int64_t>(qb) * AM + r;
    const bool row_in = row < g.sq;
    const int64_t jmax = g.causal ? row + g.shift : g.sk - 1;  // last key visible by causality
    const uint32_t lane_addr = static_cast<uint32_t>(32 * quarter) << 16;
    constexpr int HN = AN / 2;         // keys per warp and tile
    constexpr int HD = D / 2;          // O columns per warp
    float m_run = -INFINITY;    // running maximum of the scaled logits (log2 units) used by P
    float l_run = 0.0f;         // running sum of this warp's half of P
    float raw_max = -INFINITY;  // side output: maximum of the visible raw logits q . k
    bool finite = true;
    bool ok = true;
    auto pair_sync = [&]() { asm volatile("bar.sync %0, 64;" ::"r"(1 + quarter) : "memory"); };
    // The pair leaves the loop together: every failure (an expired wait, an abort) is noted in
    // `ok` and exchanged at the next per-tile barrier (or the final one), never acted on alone.
    for (int j = 0; j < ntiles; ++j) {
      const int sb = j & 1;
      const uint32_t sp = static_cast<uint32_t>((j >> 1) & 1);
      bool ready = ok;
      if (lane == 0 && ready) ready = mbar_wait(s_full + sb, sp);
      ready = __shfl_sync(0xffffffffu, ready ? 1 : 0, 0) != 0;
      ready = ready && !*reinterpret_cast<volatile int*>(abort_flag);
      red_ok[(j & 1) * 8 + half * 4 + quarter] = ready ? 1 : 0;
      float s[HN];
      if (ready) {
        tc_fence_after();
        uint32_t v[HN];
        tmem_ld64(tmem_base + lane_addr + sb * AN + half * HN, v);
#pragma unroll
        for (int e = 0; e < HN; ++e) s[e] = __uint_as_float(v[e]);
        tc_fence_before();
      }
      __syncwarp();
      if (lane == 0 && ready) mbar_arrive(s_empty + sb);  // S buffer (this half) free for S_{j+2}
      // visibility of this half tile's keys for this row; partial maxima and the non-finite test
      const int64_t key0 = static_cast<int64_t>(t0 + j) * AN + half * HN;
      const bool all_visible = row_in && key0 >= lo && key0 + HN <= hi && key0 + HN - 1 <= jmax;
      float mp[8];
      uint32_t badp[8];   // a visible logit with all exponent bits set: +-inf or NaN
#pragma unroll
      for (int q = 0; q < 8; ++q) { mp[q] = -INFINITY; badp[q] = 0u; }
      if (all_visible) {
#pragma unroll
        for (int c = 0; c < HN; ++c) badp[c & 7] |= (__float_as_uint(s[c]) & 0x7fffffffu) >= 0x7f800000u ? 1u : 0u;
      } else {
        const int64_t vis_lo = lo - key0, vis_hi_excl = (hi < jmax + 1 ? hi : jmax + 1) - key0;
#pragma unroll
        for (int c = 0; c < HN; ++c) {
          if (!row_in || c < vis_lo || c >= vis_hi_excl) s[c] = -INFINITY;
          else badp[c & 7] |= (__float_as_uint(s[c]) & 0x7fffffffu) >= 0x7f800000u ? 1u : 0u;
        }
      }
#pragma unroll
      for (int c = 0; c < HN; ++c) mp[c & 7] = fmaxf(mp[c & 7], s[c]);
      const float mine = fmaxf(fmaxf(fmaxf(mp[0], mp[1]), fmaxf(mp[2], mp[3])), fmaxf(fmaxf(mp[4], mp[5]), fmaxf(mp[6], mp[7])));
      finite = finite && (badp[0] | badp[1] | badp[2] | badp[3] | badp[4] | badp[5] | badp[6] | badp[7]) == 0u;
      raw_max = fmaxf(raw_max, mine);
      // exchange the half-row maxima (double-buffered by tile parity)
      red_max[((j & 1) * 2 + half) * AM + r] = mine;
      pair_sync();
      const float other = red_max[((j & 1) * 2 + (half ^ 1)) * AM + r];
      const bool pair_ok = red_ok[(j & 1) * 8 + (half ^ 1) * 4 + quarter] != 0;
      if (!ready || !pair_ok) { ok = false; break; }
      const float mt = fmaxf(mine, other);
      // lazy online softmax in base 2 (both halves reach the same m_run and alpha)
      const float mt2 = mt * g.scale_log2;
      float alpha = 1.0f;
      bool rescale = false;
      if (mt2 > m_run + kRescaleLog2) {
        alpha = m_run == -INFINITY ? 0.0f : fast_exp2(m_run - mt2);
        rescale = j > 0;
        m_run = mt2;
      }
      float lp[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) lp[q] = 0.0f;
      uint32_t packed[HN / 2];
      if (m_run == -INFINITY) {
#pragma unroll
        for (int c = 0; c < HN / 2; ++c) packed[c] = 0u;
      } else {
#pragma unroll
        for (int c = 0; c < HN; c += 2) {
          const float p0 = fast_exp2(fmaf(s[c], g.scale_log2, -m_run));
          const float p1 = fast_exp2(fmaf(s[c + 1], g.scale_log2, -m_run));
          lp[(c >> 1) & 7] += p0 + p1;
          if (FMT == 1) packed[c / 2] = pack_bf16(p0, p1);
          else packed[c / 2] = pack_half(p0, p1);
        }
      }
      const float lsum = ((lp[0] + lp[1]) + (lp[2] + lp[3])) + ((lp[4] + lp[5]) + (lp[6] + lp[7]));
      l_run = l_run * alpha + lsum;
      // P V of the previous tile must be done: the P buffer is reused and O may be rescaled
      if (j > 0) {
        bool done = true;
        if (lane == 0) done = mbar_wait(o_done, static_cast<uint32_t>((j - 1) & 1));
        done = __shfl_sync(0xffffffffu, done ? 1 : 0, 0) != 0;
        if (!done) { ok = false; continue; }   // the next barrier ends the pair's loop
        tc_fence_after();
      }
      if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll 1
        for (int c = 0; c < HD / 32; ++c) {
          uint32_t v[32];
          tmem_ld32(tmem_o + lane_addr + half * HD + c * 32, v);
          if (rescale) {
#pragma unroll
            for (int e = 0; e < 32; ++e) v[e] = __float_as_uint(__uint_as_float(v[e]) * alpha);
          }
          tmem_st32(tmem_o + lane_addr + half * HD + c * 32, v);
        }
      }
      // this half of the P row into K block `half` of the swizzled K-major layout: chunk c16 of
      // 8 keys sits at row * 128 + ((c16 ^ (row & 7)) * 16)
#pragma unroll
      for (int c16 = 0; c16 < HN / 8; ++c16) {
        uint8_t* dst = sP + half * SUB_BYTES + r * 128 + ((c16 ^ (r & 7)) << 4);
        *reinterpret_cast<uint4*>(dst) =
            make_uint4(packed[4 * c16], packed[4 * c16 + 1], packed[4 * c16 + 2], packed[4 * c16 + 3]);
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
    }
    // epilogue: O / l of this row, this warp's half of the columns
    if (ok && ntiles > 0) {
      bool done = true;
      if (lane == 0) done = mbar_wait(o_done, static_cast<uint32_t>((ntiles - 1) & 1));
      done = __shfl_sync(0xffffffffu, done ? 1 : 0, 0) != 0;
      if (!done) ok = false;
      tc_fence_after();
    }
    // the row sum is the two halves' sums (both warps of the pair reach this barrier together:
    // a failed wait ends both loops at the same tile)
    red_max[(4 + half) * AM + r] = l_run;
    red_ok[16 + half * 4 + quarter] = ok;
    pair_sync();
    const float l_total = l_run + red_max[(4 + (half ^ 1)) * AM + r];
    ok = ok && red_ok[16 + (half ^ 1) * 4 + quarter] != 0;
    if (ok) {
      const float inv = l_total > 0.0f ? 1.0f / l_total : 0.0f;
      uint16_t* orow = reinterpret_cast<uint16_t*>(g.out) + static_cast<int64_t>(b) * g.o_sb +
                       static_cast<int64_t>(h) * g.o_sh + row * g.o_ss + half * HD;
#pragma unroll 1
      for (int c = 0; c < HD / 32; ++c) {
        uint32_t v[32];
        if (ntiles > 0) tmem_ld32(tmem_o + lane_addr + half * HD + c * 32, v);
        else {
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
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (lane == 0 && m > -INFINITY) atomicMax(g.enc + h, encode_max(m));
        if (!finite) atomicExch(g.valid, 0);
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
  const int64_t nqb = (seq_q + AM - 1) / AM;
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
