// Element-wise step kernels around the Newton-Schulz GEMMs: normalisation of the rebuilt
// momentum, the update's sum of squares, the fused scale / ratio-clip / apply / weight-decay
// write-back, and the QK-Clip row scaling. All are HBM-bound streams over linear segments
// (muzo_plan_linear), 8 elements (one 16-byte vector of bf16) per work item.
#include "muzo_common.cuh"

namespace muzo {
namespace {

constexpr int kItemsPerThread = MUZO_ITEMS_PER_CTA / kElemThreads;

struct LinView {
  char* param;
  char* out;
  int64_t numel;
  int64_t local_item0;
  int block;
};

__device__ __forceinline__ LinView cta_linear(const muzo_segment* segs, int nsegs) {
  const int64_t item0 = static_cast<int64_t>(blockIdx.x) * MUZO_ITEMS_PER_CTA;
  const int s = find_segment(segs, nsegs, item0);
  const muzo_segment& g = segs[s];
  LinView v;
  v.param = static_cast<char*>(g.param);
  v.out = static_cast<char*>(g.out);
  v.numel = g.numel;
  v.local_item0 = item0 - g.item_begin;
  v.block = g.block_index;
  return v;
}

__device__ __forceinline__ bool aligned16(const void* p) {
  return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

__device__ __forceinline__ double block_sum(double v) {
  __shared__ double red[kElemThreads / 32];
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  double r = 0.0;
  if (warp == 0) {
    r = lane < kElemThreads / 32 ? red[lane] : 0.0;
    r = warp_sum(r);
  }
  return r;  // valid in thread 0
}

// ------------------------------------------------------------------ normalisation
// bf16(x / d) for the IEEE round-to-nearest quotient, through the product with the correctly
// rounded reciprocal r = 1/d: |x * r - x / d| stays within 2 fp32 ulps of the quotient, so both
// round to the same bf16 value unless the product lies within 4 ulps of a bf16 rounding midpoint
// (low 16 bits of the fp32 pattern near 0x8000) or is not finite; those few take the division.
__device__ __forceinline__ float bf16_quotient(float x, float d, float r) {
  const float q = x * r;
  const uint32_t low = __float_as_uint(q) & 0xffffu;
  if (low - 0x7ffcu <= 8u || !isfinite(q)) return __fdiv_rn(x, d);
  return q;
}

// X <- bf16(X / (||X||_F + 1e-7)) (newton_schulz.py:46-53): the norm is the fp32 Frobenius norm
// of the bf16 values, 1e-7 is added in fp32 and the division is IEEE round-to-nearest.
__global__ void __launch_bounds__(kElemThreads)
ns_normalize_kernel(const muzo_segment* __restrict__ segs, int nsegs, const double* __restrict__ sums,
                    int32_t* __restrict__ flags) {
  const LinView v = cta_linear(segs, nsegs);
  const double* bs = sums + static_cast<int64_t>(v.block) * MUZO_NSUMS;
  const double m2 = bs[MUZO_SUM_M2];
  const float nrm = static_cast<float>(sqrt(bs[MUZO_SUM_X2]));
  const float denom = __fadd_rn(nrm, 1e-7f);
  const float recip = __frcp_rn(denom);
  // zeropower_via_newtonschulz5 returns zeros for a zero or non-finite fp32 norm (35-43)
  if (v.local_item0 == 0 && threadIdx.x == 0 && (!(m2 > 0.0) || !isfinite(m2)))
    atomicOr(flags + v.block, MUZO_FLAG_ZERO_NORM);
  const bool vec = aligned16(v.out);
  // two vectors per trip, both loaded before either is stored: two 16-byte loads in flight per
  // thread instead of one
#pragma unroll 1
  for (int it = 0; it < kItemsPerThread; it += 2) {
    const int64_t li0 = (v.local_item0 + it * kElemThreads + threadIdx.x) * 8;
    const int64_t li1 = li0 + static_cast<int64_t>(kElemThreads) * 8;
    if (li0 >= v.numel) break;
    if (vec && li1 + 8 <= v.numel) {
      float x0[8], x1[8];
      load8(v.out, li0, MUZO_BF16, x0);
      load8(v.out, li1, MUZO_BF16, x1);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        x0[k] = bf16_quotient(x0[k], denom, recip);
        x1[k] = bf16_quotient(x1[k], denom, recip);
      }
      store8(v.out, li0, MUZO_BF16, x0);
      store8(v.out, li1, MUZO_BF16, x1);
      continue;
    }
#pragma unroll 1
    for (int j = 0; j < 2; ++j) {
      const int64_t li = j == 0 ? li0 : li1;
      if (li >= v.numel) break;
      if (vec && li + 8 <= v.numel) {
        float x[8];
        load8(v.out, li, MUZO_BF16, x);
#pragma unroll
        for (int k = 0; k < 8; ++k) x[k] = bf16_quotient(x[k], denom, recip);
        store8(v.out, li, MUZO_BF16, x);
      } else {
#pragma unroll
        for (int k = 0; k < 8; ++k)
          if (li + k < v.numel)
            store_elem(v.out, li + k, MUZO_BF16, __fdiv_rn(load_elem(v.out, li + k, MUZO_BF16), denom));
      }
    }
  }
}

// ------------------------------------------------------------------ prepare
// Newton-Schulz input from an arbitrary matrix G (newton_schulz.py:35-46): X = bf16(G) and the
// sums of fp32(G)^2 and X^2; a non-finite G sets MUZO_FLAG_NONFINITE_INPUT.
template <int DTYPE>
__global__ void __launch_bounds__(kElemThreads)
ns_prepare_kernel(const muzo_segment* __restrict__ segs, int nsegs, double* __restrict__ sums,
                  int32_t* __restrict__ flags) {
  const LinView v = cta_linear(segs, nsegs);
  const bool vec = aligned16(v.out) && aligned16(v.param);
  double m2 = 0.0, x2 = 0.0;
  bool finite = true;
#pragma unroll 1
  for (int it = 0; it < kItemsPerThread; ++it) {
    const int64_t item = v.local_item0 + it * kElemThreads + threadIdx.x;
    const int64_t li = item * 8;
    if (li >= v.numel) break;
    const int cnt = li + 8 <= v.numel ? 8 : static_cast<int>(v.numel - li);
    float g[8];
    if (vec && cnt == 8) load8(v.param, li, DTYPE, g);
    else for (int k = 0; k < 8; ++k) g[k] = k < cnt ? load_elem(v.param, li + k, DTYPE) : 0.0f;
    float pm = 0.0f, px = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      finite = finite && isfinite(g[k]);
      const float xb = bf16r(g[k]);
      pm = __fmaf_rn(g[k], g[k], pm);
      px = __fmaf_rn(xb, xb, px);
    }
    m2 += pm; x2 += px;
    if (vec && cnt == 8) store8(v.out, li, MUZO_BF16, g);
    else {
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if (k < cnt) store_elem(v.out, li + k, MUZO_BF16, g[k]);
    }
  }
  double* bs = sums + static_cast<int64_t>(v.block) * MUZO_NSUMS;
  const double tm = block_sum(m2);
  const double tx = block_sum(x2);
  if (threadIdx.x == 0) {
    if (tm != 0.0) atomicAdd(bs + MUZO_SUM_M2, tm);
    if (tx != 0.0) atomicAdd(bs + MUZO_SUM_X2, tx);
  }
  if (!finite) atomicOr(flags + v.block, MUZO_FLAG_NONFINITE_INPUT);
}

// ------------------------------------------------------------------ sum of U^2
// U = fp32(X) * scale (muzo_optimizer.py:340); sums U^2 and flags a non-finite X
// (newton_schulz.py:63-65).
__global__ void __launch_bounds__(kElemThreads)
update_sumsq_kernel(const muzo_segment* __restrict__ segs, int nsegs, const float* __restrict__ scales,
                    double* __restrict__ sums, int32_t* __restrict__ flags) {
  const LinView v = cta_linear(segs, nsegs);
  const float scale = scales[v.block];
  const bool vec = aligned16(v.out);
  double acc = 0.0;
  bool finite = true;
#pragma unroll 1
  for (int it = 0; it < kItemsPerThread; ++it) {
    const int64_t item = v.local_item0 + it * kElemThreads + threadIdx.x;
    const int64_t li = item * 8;
    if (li >= v.numel) break;
    float x[8];
    const int cnt = li + 8 <= v.numel ? 8 : static_cast<int>(v.numel - li);
    if (vec && cnt == 8) load8(v.out, li, MUZO_BF16, x);
    else for (int k = 0; k < 8; ++k) x[k] = k < cnt ? load_elem(v.out, li + k, MUZO_BF16) : 0.0f;
    float p = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      finite = finite && isfinite(x[k]);
      const float u = x[k] * scale;
      p = __fmaf_rn(u, u, p);
    }
    acc += p;
  }
  const double tot = block_sum(acc);
  if (threadIdx.x == 0 && tot != 0.0)
    atomicAdd(sums + static_cast<int64_t>(v.block) * MUZO_NSUMS + MUZO_SUM_U2, tot);
  if (!finite) atomicOr(flags + v.block, MUZO_FLAG_NONFINITE_OUTPUT);
}

// ------------------------------------------------------------------ perturbation from kept noise
// W <- dtype(W + alpha * Zk) with Zk (segs[i].out, the block's dtype and layout) the rounded noise
// a normal-noise pass of the same key kept: the arithmetic of the regenerating pass
// (add_(noise, alpha) as one fp32 fused multiply-add, then the rounding to the weight dtype) on
// values read from memory, 6 B per 16-bit element instead of a Philox + Box-Muller evaluation.
template <int DTYPE>
__global__ void __launch_bounds__(kElemThreads)
perturb_kept_kernel(const muzo_segment* __restrict__ segs, int nsegs, float alpha) {
  const LinView v = cta_linear(segs, nsegs);
  if (v.param == nullptr || v.out == nullptr) return;
  const bool vec = aligned16(v.param) && aligned16(v.out);
#pragma unroll 1
  for (int it = 0; it < kItemsPerThread; ++it) {
    const int64_t item = v.local_item0 + it * kElemThreads + threadIdx.x;
    const int64_t li = item * 8;
    if (li >= v.numel) break;
    if (vec && li + 8 <= v.numel) {
      float w[8], z[8];
      load8(v.out, li, DTYPE, z);
      load8(v.param, li, DTYPE, w);
#pragma unroll
      for (int k = 0; k < 8; ++k) w[k] = __fmaf_rn(alpha, z[k], w[k]);
      store8(v.param, li, DTYPE, w);
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if (li + k < v.numel)
          store_elem(v.param, li + k, DTYPE,
                     __fmaf_rn(alpha, load_elem(v.out, li + k, DTYPE), load_elem(v.param, li + k, DTYPE)));
    }
  }
}

// ------------------------------------------------------------------ apply
struct ApplyScalars {
  float clip;     // multiplier applied to U
  bool clipped;
  bool zeroed;
  float ratio;    // ratio before the clip
};

// Per-block scalars of muzo_optimizer.py:342-349, recomputed by every CTA of the block.
__device__ __forceinline__ ApplyScalars block_scalars(const double* bs, int32_t flag, int64_t numel,
                                                      float lr, double ratio_clip) {
  ApplyScalars s;
  s.zeroed = (flag & (MUZO_FLAG_NONFINITE_INPUT | MUZO_FLAG_ZERO_NORM | MUZO_FLAG_NONFINITE_OUTPUT)) != 0;
  const double n = static_cast<double>(numel);
  const float rms_u = s.zeroed ? 0.0f : static_cast<float>(sqrt(bs[MUZO_SUM_U2] / n));
  const float rms_w = static_cast<float>(sqrt(bs[MUZO_SUM_W2] / n));
  const float update_rms = rms_u * lr;
  const float ratio = __fdiv_rn(update_rms, __fadd_rn(rms_w, 1e-12f));
  s.ratio = ratio;
  s.clipped = static_cast<double>(ratio) > ratio_clip;
  s.clip = s.clipped ? static_cast<float>(ratio_clip / static_cast<double>(ratio)) : 1.0f;
  return s;
}

// One element of the apply: U = x * scale (times the clip factor), W = dtype(W - lr * dtype(U)),
// then the decay multiply, each rounding as the reference's tensor ops.
template <int DTYPE>
__device__ __forceinline__ void apply8(float (&x)[8], float (&w)[8], const ApplyScalars& sc, float scale, float neg_lr,
                                       int apply_decay, float decay) {
  float u[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    u[k] = sc.zeroed ? 0.0f : x[k] * scale;           // U.mul_(sqrt(max)*muon_scale)
    if (sc.clipped) u[k] = u[k] * sc.clip;             // U.mul_(clip / ratio)
  }
#pragma unroll
  for (int k = 0; k < 8; k += 2) round2_to(u[k], u[k + 1], DTYPE);       // U.to(block.dtype)
#pragma unroll
  for (int k = 0; k < 8; ++k) w[k] = __fmaf_rn(neg_lr, u[k], w[k]);      // block.add_(U, alpha=-lr)
#pragma unroll
  for (int k = 0; k < 8; k += 2) round2_to(w[k], w[k + 1], DTYPE);
  if (apply_decay) {
#pragma unroll
    for (int k = 0; k < 8; ++k) w[k] = w[k] * decay;                     // block.mul_(1 - lr*wd)
#pragma unroll
    for (int k = 0; k < 8; k += 2) round2_to(w[k], w[k + 1], DTYPE);
  }
}

// Apply of every block (muzo_optimizer.py:340-353). The sum of the clipped update's squares
// (the reported update_rms) is clip^2 times the sum of U^2 the last Newton-Schulz GEMM
// accumulated: written once per block by its first CTA instead of summed per element.
template <int DTYPE>
__global__ void __launch_bounds__(kElemThreads)
apply_update_kernel(const muzo_segment* __restrict__ segs, int nsegs, const float* __restrict__ scales,
                    float lr, double ratio_clip, int apply_decay, float decay,
                    double* __restrict__ sums, const int32_t* __restrict__ flags,
                    float* __restrict__ stats) {
  const LinView v = cta_linear(segs, nsegs);
  double* bs = sums + static_cast<int64_t>(v.block) * MUZO_NSUMS;
  const ApplyScalars sc = block_scalars(bs, flags[v.block], v.numel, lr, ratio_clip);
  const float scale = scales[v.block];
  const float neg_lr = -lr;
  if (v.local_item0 == 0 && threadIdx.x == 0) {
    float* st = stats + static_cast<int64_t>(v.block) * MUZO_NSTATS;
    st[MUZO_STAT_RATIO_BEFORE] = sc.ratio;
    st[MUZO_STAT_CLIP_FACTOR] = sc.clip;
    st[MUZO_STAT_ZEROED] = sc.zeroed ? 1.0f : 0.0f;
    const double c = sc.clipped ? static_cast<double>(sc.clip) : 1.0;
    bs[MUZO_SUM_U2_CLIPPED] = sc.zeroed ? 0.0 : c * c * bs[MUZO_SUM_U2];
  }
  const bool vec = aligned16(v.out) && aligned16(v.param);
#pragma unroll 1
  for (int it = 0; it < kItemsPerThread; ++it) {
    const int64_t item = v.local_item0 + it * kElemThreads + threadIdx.x;
    const int64_t li = item * 8;
    if (li >= v.numel) break;
    float x[8], w[8];
    const int64_t li1 = li + static_cast<int64_t>(kElemThreads) * 8;
    if (vec && (it & 1) == 0 && it + 1 < kItemsPerThread && li1 + 8 <= v.numel) {
      // two items per trip, all four vectors loaded before either result is stored
      float x1[8], w1[8];
      load8(v.out, li, MUZO_BF16, x);
      load8(v.param, li, DTYPE, w);
      load8(v.out, li1, MUZO_BF16, x1);
      load8(v.param, li1, DTYPE, w1);
      apply8<DTYPE>(x, w, sc, scale, neg_lr, apply_decay, decay);
      apply8<DTYPE>(x1, w1, sc, scale, neg_lr, apply_decay, decay);
      store8(v.param, li, DTYPE, w);
      store8(v.param, li1, DTYPE, w1);
      ++it;
      continue;
    }
    if (vec && li + 8 <= v.numel) {
      load8(v.out, li, MUZO_BF16, x);
      load8(v.param, li, DTYPE, w);
      apply8<DTYPE>(x, w, sc, scale, neg_lr, apply_decay, decay);
      store8(v.param, li, DTYPE, w);
    } else {
      const int cnt = static_cast<int>(v.numel - li < 8 ? v.numel - li : 8);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        x[k] = k < cnt ? load_elem(v.out, li + k, MUZO_BF16) : 0.0f;
        w[k] = k < cnt ? load_elem(v.param, li + k, DTYPE) : 0.0f;
      }
      apply8<DTYPE>(x, w, sc, scale, neg_lr, apply_decay, decay);
#pragma unroll
      for (int k = 0; k < 8; ++k)  // static indices keep w in registers
        if (k < cnt) store_elem(v.param, li + k, DTYPE, w[k]);
    }
  }
}

// ------------------------------------------------------------------ QK-Clip row scaling
template <int DTYPE>
__global__ void qk_scale_rows_kernel(char* __restrict__ w, int64_t groups, int64_t rows_per_group,
                                     int64_t cols, const float* __restrict__ factors,
                                     const int32_t* __restrict__ mask) {
  const int64_t total = groups * rows_per_group * cols;
  const int64_t per_group = rows_per_group * cols;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t g = i / per_group;
    if (mask[g] == 0) continue;
    store_elem(w, i, DTYPE, load_elem(w, i, DTYPE) * factors[g]);
  }
}

int check_linear(const muzo_segment* segs, int nsegs, int64_t total_items) {
  if (segs == nullptr || nsegs <= 0 || total_items <= 0 || total_items % MUZO_ITEMS_PER_CTA != 0)
    return MUZO_ERR_ARG;
  if (total_items / MUZO_ITEMS_PER_CTA > 0x7fffffffLL) return MUZO_ERR_UNSUPPORTED;
  return MUZO_OK;
}

}  // namespace
}  // namespace muzo

using namespace muzo;

extern "C" {

int muzo_ns_normalize(const muzo_segment* d_segs, int nsegs, int64_t total_items,
                      const double* d_sums, int32_t* d_flags, void* stream) {
  if (nsegs == 0 || total_items == 0) return MUZO_OK;
  int st = check_linear(d_segs, nsegs, total_items);
  if (st != MUZO_OK) return st;
  if (d_sums == nullptr || d_flags == nullptr) return MUZO_ERR_ARG;
  ns_normalize_kernel<<<static_cast<unsigned>(total_items / MUZO_ITEMS_PER_CTA), kElemThreads, 0,
                        static_cast<cudaStream_t>(stream)>>>(d_segs, nsegs, d_sums, d_flags);
  return launch_status();
}

int muzo_ns_prepare(const muzo_segment* d_segs, int nsegs, int64_t total_items, int dtype,
                    double* d_sums, int32_t* d_flags, void* stream) {
  if (nsegs == 0 || total_items == 0) return MUZO_OK;
  int st = check_linear(d_segs, nsegs, total_items);
  if (st != MUZO_OK) return st;
  if (d_sums == nullptr || d_flags == nullptr) return MUZO_ERR_ARG;
  const unsigned grid = static_cast<unsigned>(total_items / MUZO_ITEMS_PER_CTA);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case MUZO_BF16: ns_prepare_kernel<MUZO_BF16><<<grid, kElemThreads, 0, s>>>(d_segs, nsegs, d_sums, d_flags); break;
    case MUZO_F16: ns_prepare_kernel<MUZO_F16><<<grid, kElemThreads, 0, s>>>(d_segs, nsegs, d_sums, d_flags); break;
    case MUZO_F32: ns_prepare_kernel<MUZO_F32><<<grid, kElemThreads, 0, s>>>(d_segs, nsegs, d_sums, d_flags); break;
    default: return MUZO_ERR_DTYPE;
  }
  return launch_status();
}

int muzo_update_sumsq(const muzo_segment* d_segs, int nsegs, int64_t total_items,
                      const float* d_scales, double* d_sums, int32_t* d_flags, void* stream) {
  if (nsegs == 0 || total_items == 0) return MUZO_OK;
  int st = check_linear(d_segs, nsegs, total_items);
  if (st != MUZO_OK) return st;
  if (d_scales == nullptr || d_sums == nullptr || d_flags == nullptr) return MUZO_ERR_ARG;
  update_sumsq_kernel<<<static_cast<unsigned>(total_items / MUZO_ITEMS_PER_CTA), kElemThreads, 0,
                        static_cast<cudaStream_t>(stream)>>>(d_segs, nsegs, d_scales, d_sums, d_flags);
  return launch_status();
}

int muzo_perturb_kept_noise(const muzo_segment* d_segs, int nsegs, int64_t total_items, int dtype,
                            float alpha, void* stream) {
  if (nsegs == 0 || total_items == 0) return MUZO_OK;
  int st = check_linear(d_segs, nsegs, total_items);
  if (st != MUZO_OK) return st;
  const unsigned grid = static_cast<unsigned>(total_items / MUZO_ITEMS_PER_CTA);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case MUZO_BF16: perturb_kept_kernel<MUZO_BF16><<<grid, kElemThreads, 0, s>>>(d_segs, nsegs, alpha); break;
    case MUZO_F16: perturb_kept_kernel<MUZO_F16><<<grid, kElemThreads, 0, s>>>(d_segs, nsegs, alpha); break;
    case MUZO_F32: perturb_kept_kernel<MUZO_F32><<<grid, kElemThreads, 0, s>>>(d_segs, nsegs, alpha); break;
    default: return MUZO_ERR_DTYPE;
  }
  return launch_status();
}

int muzo_apply_update(const muzo_segment* d_segs, int nsegs, int64_t total_items, int dtype,
                      const float* d_scales, float lr, double ratio_clip, int apply_decay,
                      float decay, double* d_sums, const int32_t* d_flags, float* d_stats,
                      void* stream) {
  if (nsegs == 0 || total_items == 0) return MUZO_OK;
  int st = check_linear(d_segs, nsegs, total_items);
  if (st != MUZO_OK) return st;
  if (d_scales == nullptr || d_sums == nullptr || d_flags == nullptr || d_stats == nullptr)
    return MUZO_ERR_ARG;
  const unsigned grid = static_cast<unsigned>(total_items / MUZO_ITEMS_PER_CTA);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case MUZO_BF16:
      apply_update_kernel<MUZO_BF16><<<grid, kElemThreads, 0, s>>>(
          d_segs, nsegs, d_scales, lr, ratio_clip, apply_decay, decay, d_sums, d_flags, d_stats);
      break;
    case MUZO_F16:
      apply_update_kernel<MUZO_F16><<<grid, kElemThreads, 0, s>>>(
          d_segs, nsegs, d_scales, lr, ratio_clip, apply_decay, decay, d_sums, d_flags, d_stats);
      break;
    case MUZO_F32:
      apply_update_kernel<MUZO_F32><<<grid, kElemThreads, 0, s>>>(
          d_segs, nsegs, d_scales, lr, ratio_clip, apply_decay, decay, d_sums, d_flags, d_stats);
      break;
    default:
      return MUZO_ERR_DTYPE;
  }
  return launch_status();
}

int muzo_qk_scale_rows(void* w, int dtype, int64_t groups, int64_t rows_per_group, int64_t cols,
                       const float* d_factors, const int32_t* d_mask, void* stream) {
  if (w == nullptr || d_factors == nullptr || d_mask == nullptr || groups < 0 ||
      rows_per_group < 0 || cols < 0)
    return MUZO_ERR_ARG;
  const int64_t total = groups * rows_per_group * cols;
  if (total == 0) return MUZO_OK;
  int64_t blocks = (total + 255) / 256;
  const int64_t cap = static_cast<int64_t>(device_sm_count()) * 8;
  if (blocks > cap) blocks = cap;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  char* p = static_cast<char*>(w);
  switch (dtype) {
    case MUZO_BF16:
      qk_scale_rows_kernel<MUZO_BF16><<<static_cast<unsigned>(blocks), 256, 0, s>>>(
          p, groups, rows_per_group, cols, d_factors, d_mask);
      break;
    case MUZO_F16:
      qk_scale_rows_kernel<MUZO_F16><<<static_cast<unsigned>(blocks), 256, 0, s>>>(
          p, groups, rows_per_group, cols, d_factors, d_mask);
      break;
    case MUZO_F32:
      qk_scale_rows_kernel<MUZO_F32><<<static_cast<unsigned>(blocks), 256, 0, s>>>(
          p, groups, rows_per_group, cols, d_factors, d_mask);
      break;
    default:
      return MUZO_ERR_DTYPE;
  }
  return launch_status();
}

}  // extern "C"
