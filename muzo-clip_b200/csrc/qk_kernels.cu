// QK-Clip reductions: the per-head maximum of the eager pre-softmax logits (qk_clip.py:173-196)
// computed straight from Q and K without materialising the S x S logits, the same reduction over
// already materialised logits (softmax capture), and the guarded running-max merge.
//
// Maxima are accumulated as order-preserving integers with atomicMax, then decoded; the eager
// rounding of the logits, round(round(q.k) * scale) in the model dtype, is monotonic, so it is
// applied once to the maximum dot product instead of to every logit.
#include <cstdlib>

#include "muzo_common.cuh"

namespace muzo {

int qk_max_tensor_cores(const void* q, const void* k, int dtype, int64_t batch, int64_t hq, int64_t hkv, int64_t sq,
                        int64_t sk, int64_t d, int64_t qsb, int64_t qsh, int64_t qss, int64_t ksb, int64_t ksh,
                        int64_t kss, int causal, const int32_t* key_lo, const int32_t* key_hi, int* enc,
                        int32_t* valid, cudaStream_t stream);

namespace {

__device__ __forceinline__ int encode_max(float f) {
  const int b = __float_as_int(f);
  return b >= 0 ? b : b ^ 0x7fffffff;
}
__device__ __forceinline__ float decode_max(int e) { return __int_as_float(e >= 0 ? e : e ^ 0x7fffffff); }

__global__ void init_max_kernel(int* enc, int n, int32_t* valid) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) enc[i] = encode_max(-INFINITY);
  if (i == 0 && valid) *valid = 1;
}

// smax[h] = round(round(max_dot) * scale) in the logits dtype.
__global__ void finalize_max_kernel(int* enc, int n, int dtype, float scale, int apply_scale) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float v = decode_max(enc[i]);
  if (apply_scale && isfinite(v)) v = round_to(round_to(v, dtype) * scale, dtype);
  reinterpret_cast<float*>(enc)[i] = v;
}

// ------------------------------------------------------------------ max over Q.K^T (SIMT)
// One CTA per (batch, head, 64-query tile); K streams through shared memory in 64-key tiles.
// 256 threads, each owning a 4 x 4 block of logits of the 64 x 64 tile. Exact fp32 products
// of the dtype's values, fp32 accumulation.
constexpr int QT = 64, KT = 64, DCHUNK = 32;

template <int DTYPE>
__global__ void __launch_bounds__(256)
qk_max_simt_kernel(const char* __restrict__ q, const char* __restrict__ k, int64_t hq, int64_t hkv,
                   int64_t sq, int64_t sk, int64_t d, int64_t qsb, int64_t qsh, int64_t qss,
                   int64_t ksb, int64_t ksh, int64_t kss, int causal, const int32_t* __restrict__ key_lo,
                   const int32_t* __restrict__ key_hi, int* __restrict__ enc, int32_t* __restrict__ valid) {
  __shared__ float qs[DCHUNK][QT + 1];
  __shared__ float ks[DCHUNK][KT + 1];
  const int64_t qtiles = (sq + QT - 1) / QT;
  const int64_t unit = blockIdx.x;
  const int64_t bh = unit / qtiles;
  const int64_t qt = unit - bh * qtiles;
  const int64_t b = bh / hq, h = bh - b * hq;
  const int64_t kvh = h / (hq / hkv);
  const int esz = DTYPE == MUZO_F32 ? 4 : 2;
  const char* qbase = q + (b * qsb + h * qsh) * esz;
  const char* kbase = k + (b * ksb + kvh * ksh) * esz;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int64_t i0 = qt * QT;
  const int64_t shift = sk - sq;  // causal: key j visible to query i when j <= i + shift
  int64_t kbegin = 0, kend = sk;   // visible keys of this batch row: [kbegin, kend)
  if (key_lo != nullptr) {
    kbegin = max(static_cast<int64_t>(key_lo[b]), static_cast<int64_t>(0));
    kend = min(static_cast<int64_t>(key_hi[b]), sk);
  }
  const int64_t kstop = causal ? min(kend, i0 + QT + shift) : kend;
  float best = -INFINITY;
  bool finite = true;
  for (int64_t j0 = kbegin - kbegin % KT; j0 < kstop; j0 += KT) {
    float acc[4][4] = {};
    for (int64_t c0 = 0; c0 < d; c0 += DCHUNK) {
      for (int e = threadIdx.x; e < DCHUNK * QT; e += 256) {
        const int r = e / DCHUNK, c = e % DCHUNK;
        const int64_t qi = i0 + r, dc = c0 + c;
        qs[c][r] = (qi < sq && dc < d) ? load_elem(qbase, qi * qss + dc, DTYPE) : 0.0f;
        const int64_t kj = j0 + r;
        ks[c][r] = (kj < sk && dc < d) ? load_elem(kbase, kj * kss + dc, DTYPE) : 0.0f;
      }
      __syncthreads();
#pragma unroll 4
      for (int c = 0; c < DCHUNK; ++c) {
        float a[4], bb[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) { a[u] = qs[c][ty * 4 + u]; bb[u] = ks[c][tx * 4 + u]; }
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
          for (int v = 0; v < 4; ++v) acc[u][v] = __fmaf_rn(a[u], bb[v], acc[u][v]);
      }
      __syncthreads();
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int64_t i = i0 + ty * 4 + u;
#pragma unroll
      for (int v = 0; v < 4; ++v) {
        const int64_t j = j0 + tx * 4 + v;
        if (i < sq && j >= kbegin && j < kend && (!causal || j <= i + shift)) {
          const float x = acc[u][v];
          finite = finite && isfinite(x);
          best = fmaxf(best, x);
        }
      }
    }
  }
  // block max
  __shared__ float red[8];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) best = fmaxf(best, __shfl_xor_sync(0xffffffffu, best, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    float m = red[0];
    for (int w = 1; w < 8; ++w) m = fmaxf(m, red[w]);
    if (m > -INFINITY) atomicMax(enc + h, encode_max(m));
  }
  if (!finite) atomicExch(valid, 0);
}

// ------------------------------------------------------------------ max over logits
template <int DTYPE>
__global__ void __launch_bounds__(256)
logits_head_max_kernel(const char* __restrict__ logits, int64_t bsz, int64_t heads, int64_t sq, int64_t sk,
                       int64_t sb, int64_t sh, int64_t sqs, int64_t sks, int* __restrict__ enc,
                       int32_t* __restrict__ valid) {
  const int64_t h = blockIdx.y;
  const int64_t per_head = bsz * sq * sk;
  float best = -INFINITY;
  bool finite = true;
  for (int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; e < per_head;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t b = e / (sq * sk);
    const int64_t r = e - b * sq * sk;
    const int64_t i = r / sk, j = r - i * sk;
    const float x = load_elem(logits, b * sb + h * sh + i * sqs + j * sks, DTYPE);
    finite = finite && isfinite(x);
    best = fmaxf(best, x);
  }
  __shared__ float red[8];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) best = fmaxf(best, __shfl_xor_sync(0xffffffffu, best, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    float m = red[0];
    for (int w = 1; w < 8; ++w) m = fmaxf(m, red[w]);
    if (m > -INFINITY) atomicMax(enc + h, encode_max(m));
  }
  if (!finite) atomicExch(valid, 0);
}

// The tensor-core path can be turned off for comparison runs (MUZO_QK_SIMT=1).
bool qk_tensor_cores_enabled() {
  static const bool enabled = [] {
    const char* e = getenv("MUZO_QK_SIMT");
    return !(e != nullptr && e[0] == '1');
  }();
  return enabled;
}

__global__ void max_merge_kernel(float* running, const float* fresh, const int32_t* valid, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  if (valid != nullptr && *valid == 0) return;
  running[i] = fmaxf(running[i], fresh[i]);
}

}  // namespace
}  // namespace muzo

using namespace muzo;

extern "C" {

int muzo_qk_max(const void* q, const void* k, int dtype, int64_t batch, int64_t hq, int64_t hkv,
                int64_t seq_q, int64_t seq_k, int64_t head_dim, int64_t q_stride_b, int64_t q_stride_h,
                int64_t q_stride_s, int64_t k_stride_b, int64_t k_stride_h, int64_t k_stride_s,
                int causal, float scale, float* smax, int32_t* d_valid, void* stream) {
  return muzo_qk_max_ranges(q, k, dtype, batch, hq, hkv, seq_q, seq_k, head_dim, q_stride_b, q_stride_h, q_stride_s,
                            k_stride_b, k_stride_h, k_stride_s, causal, nullptr, nullptr, scale, smax, d_valid,
                            stream);
}

int muzo_qk_max_ranges(const void* q, const void* k, int dtype, int64_t batch, int64_t hq, int64_t hkv,
                       int64_t seq_q, int64_t seq_k, int64_t head_dim, int64_t q_stride_b, int64_t q_stride_h,
                       int64_t q_stride_s, int64_t k_stride_b, int64_t k_stride_h, int64_t k_stride_s,
                       int causal, const int32_t* d_key_lo, const int32_t* d_key_hi, float scale, float* smax,
                       int32_t* d_valid, void* stream) {
  if (q == nullptr || k == nullptr || smax == nullptr || d_valid == nullptr || batch < 0 || hq <= 0 ||
      hkv <= 0 || hq % hkv != 0 || seq_q < 0 || seq_k < 0 || head_dim <= 0 ||
      (d_key_lo == nullptr) != (d_key_hi == nullptr))
    return MUZO_ERR_ARG;
  if (dtype != MUZO_BF16 && dtype != MUZO_F16 && dtype != MUZO_F32) return MUZO_ERR_DTYPE;  // before any launch
  if (hq > 0x7fffffffLL) return MUZO_ERR_UNSUPPORTED;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int* enc = reinterpret_cast<int*>(smax);
  init_max_kernel<<<static_cast<unsigned>((hq + 255) / 256), 256, 0, s>>>(enc, static_cast<int>(hq), d_valid);
  const int64_t units = batch * hq * ((seq_q + QT - 1) / QT);
  // bf16 / fp16 with TMA-compatible strides (multiples of 8 elements, 16-byte aligned bases)
  // run on the tensor cores; fp32 (exact fp32 products, as the reference's fp32 matmul) and
  // other layouts on the CUDA cores
  const bool tensor_path = (dtype == MUZO_BF16 || dtype == MUZO_F16) && head_dim % 8 == 0 &&
                           q_stride_b % 8 == 0 && q_stride_h % 8 == 0 && q_stride_s % 8 == 0 &&
                           k_stride_b % 8 == 0 && k_stride_h % 8 == 0 && k_stride_s % 8 == 0 &&
                           (reinterpret_cast<uintptr_t>(q) & 15u) == 0 && (reinterpret_cast<uintptr_t>(k) & 15u) == 0 &&
                           batch <= 0x7fffffffLL && hq <= 0x7fffffffLL && seq_q <= 0x7fffffffLL &&
                           seq_k <= 0x7fffffffLL && qk_tensor_cores_enabled();
  if (tensor_path && units > 0 && seq_k > 0) {
    const int st = qk_max_tensor_cores(q, k, dtype, batch, hq, hkv, seq_q, seq_k, head_dim, q_stride_b, q_stride_h,
                                       q_stride_s, k_stride_b, k_stride_h, k_stride_s, causal, d_key_lo, d_key_hi, enc,
                                       d_valid, s);
    if (st != MUZO_OK) return st;
  } else if (units > 0 && seq_k > 0) {
    if (units > 0x7fffffffLL) return MUZO_ERR_UNSUPPORTED;
    const unsigned grid = static_cast<unsigned>(units);
    const char* qp = static_cast<const char*>(q);
    const char* kp = static_cast<const char*>(k);
    switch (dtype) {
      case MUZO_BF16:
        qk_max_simt_kernel<MUZO_BF16><<<grid, 256, 0, s>>>(qp, kp, hq, hkv, seq_q, seq_k, head_dim, q_stride_b,
                                                           q_stride_h, q_stride_s, k_stride_b, k_stride_h,
                                                           k_stride_s, causal, d_key_lo, d_key_hi, enc, d_valid);
        break;
      case MUZO_F16:
        qk_max_simt_kernel<MUZO_F16><<<grid, 256, 0, s>>>(qp, kp, hq, hkv, seq_q, seq_k, head_dim, q_stride_b,
                                                          q_stride_h, q_stride_s, k_stride_b, k_stride_h,
                                                          k_stride_s, causal, d_key_lo, d_key_hi, enc, d_valid);
        break;
      case MUZO_F32:
        qk_max_simt_kernel<MUZO_F32><<<grid, 256, 0, s>>>(qp, kp, hq, hkv, seq_q, seq_k, head_dim, q_stride_b,
                                                          q_stride_h, q_stride_s, k_stride_b, k_stride_h,
                                                          k_stride_s, causal, d_key_lo, d_key_hi, enc, d_valid);
        break;
      default:
        return MUZO_ERR_DTYPE;
    }
  }
  finalize_max_kernel<<<static_cast<unsigned>((hq + 255) / 256), 256, 0, s>>>(enc, static_cast<int>(hq), dtype,
                                                                               scale, 1);
  return launch_status();
}

int muzo_logits_head_max(const void* logits, int dtype, int64_t batch, int64_t heads, int64_t seq_q,
                         int64_t seq_k, int64_t stride_b, int64_t stride_h, int64_t stride_q,
                         int64_t stride_k, float* out, int32_t* d_valid, void* stream) {
  if (logits == nullptr || out == nullptr || d_valid == nullptr || batch < 0 || heads <= 0 || seq_q < 0 ||
      seq_k < 0 || heads > 65535)
    return MUZO_ERR_ARG;
  if (dtype != MUZO_BF16 && dtype != MUZO_F16 && dtype != MUZO_F32) return MUZO_ERR_DTYPE;  // before any launch
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int* enc = reinterpret_cast<int*>(out);
  init_max_kernel<<<static_cast<unsigned>((heads + 255) / 256), 256, 0, s>>>(enc, static_cast<int>(heads), d_valid);
  const int64_t per_head = batch * seq_q * seq_k;
  if (per_head > 0) {
    int64_t gx = (per_head + 255) / 256;
    const int64_t cap = (static_cast<int64_t>(device_sm_count()) * 8 + heads - 1) / heads;
    if (gx > cap) gx = cap;
    if (gx < 1) gx = 1;
    const dim3 grid(static_cast<unsigned>(gx), static_cast<unsigned>(heads));
    const char* lp = static_cast<const char*>(logits);
    switch (dtype) {
      case MUZO_BF16:
        logits_head_max_kernel<MUZO_BF16><<<grid, 256, 0, s>>>(lp, batch, heads, seq_q, seq_k, stride_b, stride_h,
                                                               stride_q, stride_k, enc, d_valid);
        break;
      case MUZO_F16:
        logits_head_max_kernel<MUZO_F16><<<grid, 256, 0, s>>>(lp, batch, heads, seq_q, seq_k, stride_b, stride_h,
                                                              stride_q, stride_k, enc, d_valid);
        break;
      case MUZO_F32:
        logits_head_max_kernel<MUZO_F32><<<grid, 256, 0, s>>>(lp, batch, heads, seq_q, seq_k, stride_b, stride_h,
                                                              stride_q, stride_k, enc, d_valid);
        break;
      default:
        return MUZO_ERR_DTYPE;
    }
  }
  finalize_max_kernel<<<static_cast<unsigned>((heads + 255) / 256), 256, 0, s>>>(enc, static_cast<int>(heads),
                                                                                 dtype, 1.0f, 0);
  return launch_status();
}

int muzo_max_merge(float* running, const float* fresh, const int32_t* d_valid, int64_t n, void* stream) {
  if (running == nullptr || fresh == nullptr || n < 0) return MUZO_ERR_ARG;
  if (n == 0) return MUZO_OK;
  if (n > 0x7fffffffLL) return MUZO_ERR_UNSUPPORTED;
  max_merge_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      running, fresh, d_valid, static_cast<int>(n));
  return launch_status();
}

}  // extern "C"
