// Newton-Schulz input normalisation that allocates nothing.
//
// muzo_ns_prepare + muzo_ns_normalize need scratch between their two passes: a segment table
// and per-matrix sums of squares, which their callers allocate. Some callers cannot: a runtime
// that reserves the whole device memory pool at start-up and forbids cudaMalloc afterwards, or a
// plugin running inside another framework whose allocator owns every device byte. For them this
// file keeps that scratch in one file-scope device array of fixed size.
//
// The array lives in every GPU that loads the library until the process exits. Every call uses
// the same array and leaves its contents behind; each call clears the sums it accumulates before
// using them. Calls whose kernels overlap on the GPU (different streams, or different host
// threads, on one device) race on the array: serialise them.
#include "muzo_common.cuh"

namespace muzo {
namespace {

constexpr int kNoallocMaxBlocks = MUZO_NOALLOC_MAX_BLOCKS;

struct NoallocScratch {
  muzo_segment segs[kNoallocMaxBlocks];
  double sums[kNoallocMaxBlocks][MUZO_NSUMS];
};

// The scratch: 64 segments (4 KB) and 64 x 8 fp64 sums (4 KB).
static __device__ __align__(256) unsigned char g_noalloc_scratch[sizeof(NoallocScratch)];

struct TableParam {
  muzo_segment segs[kNoallocMaxBlocks];
  int nsegs;
};

// Copies the caller's table into the scratch and clears the sums and the caller's flags.
__global__ void noalloc_setup_kernel(const TableParam t, NoallocScratch* s, int32_t* flags) {
  const int i = threadIdx.x;
  if (i < t.nsegs) {
    s->segs[i] = t.segs[i];
#pragma unroll
    for (int k = 0; k < MUZO_NSUMS; ++k) s->sums[i][k] = 0.0;
    flags[i] = 0;
  }
}

constexpr int kItemsPerThread = MUZO_ITEMS_PER_CTA / kElemThreads;

__device__ __forceinline__ bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

__device__ __forceinline__ double cta_sum(double v) {
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
  return r;
}

// X = bf16(G), sums of fp32(G)^2 and X^2, non-finite flag (newton_schulz.py:35-46).
template <int DTYPE>
__global__ void __launch_bounds__(kElemThreads)
noalloc_prepare_kernel(NoallocScratch* s, int nsegs, int32_t* flags) {
  const int64_t item0 = static_cast<int64_t>(blockIdx.x) * MUZO_ITEMS_PER_CTA;
  const int sidx = find_segment(s->segs, nsegs, item0);
  const muzo_segment& g = s->segs[sidx];
  const char* in = static_cast<const char*>(g.param);
  char* out = static_cast<char*>(g.out);
  const int64_t numel = g.numel;
  const int64_t local0 = item0 - g.item_begin;
  const bool vec = aligned16(in) && aligned16(out);
  double m2 = 0.0, x2 = 0.0;
  bool finite = true;
#pragma unroll 1
  for (int it = 0; it < kItemsPerThread; ++it) {
    const int64_t li = (local0 + it * kElemThreads + threadIdx.x) * 8;
    if (li >= numel) break;
    const int cnt = li + 8 <= numel ? 8 : static_cast<int>(numel - li);
    float v[8];
    if (vec && cnt == 8) {
      load8(in, li, DTYPE, v);
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k) v[k] = k < cnt ? load_elem(in, li + k, DTYPE) : 0.0f;
    }
    float pm = 0.0f, px = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      finite = finite && isfinite(v[k]);
      const float xb = bf16r(v[k]);
      pm = __fmaf_rn(v[k], v[k], pm);
      px = __fmaf_rn(xb, xb, px);
    }
    m2 += pm; x2 += px;
    if (vec && cnt == 8) {
      store8(out, li, MUZO_BF16, v);
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if (k < cnt) store_elem(out, li + k, MUZO_BF16, v[k]);
    }
  }
  const double tm = cta_sum(m2);
  const double tx = cta_sum(x2);
  if (threadIdx.x == 0) {
    if (tm != 0.0) atomicAdd(&s->sums[g.block_index][MUZO_SUM_M2], tm);
    if (tx != 0.0) atomicAdd(&s->sums[g.block_index][MUZO_SUM_X2], tx);
  }
  if (!finite) atomicOr(flags + g.block_index, MUZO_FLAG_NONFINITE_INPUT);
}

// X = bf16(X / (||X||_F + 1e-7)); zero or non-finite fp32 norm sets MUZO_FLAG_ZERO_NORM.
__global__ void __launch_bounds__(kElemThreads)
noalloc_normalize_kernel(NoallocScratch* s, int nsegs, int32_t* flags) {
  const int64_t item0 = static_cast<int64_t>(blockIdx.x) * MUZO_ITEMS_PER_CTA;
  const int sidx = find_segment(s->segs, nsegs, item0);
  const muzo_segment& g = s->segs[sidx];
  char* x = static_cast<char*>(g.out);
  const int64_t numel = g.numel;
  const int64_t local0 = item0 - g.item_begin;
  const double m2 = s->sums[g.block_index][MUZO_SUM_M2];
  const float denom = __fadd_rn(static_cast<float>(sqrt(s->sums[g.block_index][MUZO_SUM_X2])), 1e-7f);
  if (local0 == 0 && threadIdx.x == 0 && (!(m2 > 0.0) || !isfinite(m2)))
    atomicOr(flags + g.block_index, MUZO_FLAG_ZERO_NORM);
  const bool vec = aligned16(x);
#pragma unroll 1
  for (int it = 0; it < kItemsPerThread; ++it) {
    const int64_t li = (local0 + it * kElemThreads + threadIdx.x) * 8;
    if (li >= numel) break;
    if (vec && li + 8 <= numel) {
      float v[8];
      load8(x, li, MUZO_BF16, v);
#pragma unroll
      for (int k = 0; k < 8; ++k) v[k] = __fdiv_rn(v[k], denom);
      store8(x, li, MUZO_BF16, v);
    } else {
      for (int k = 0; k < 8 && li + k < numel; ++k)
        store_elem(x, li + k, MUZO_BF16, __fdiv_rn(load_elem(x, li + k, MUZO_BF16), denom));
    }
  }
}

// Device address of the scratch array in the current context, looked up on every call: a cached
// address would dangle after the context is torn down and re-created (the module is reloaded
// elsewhere), and the lookup costs little next to the three launches.
NoallocScratch* scratch_for_current_device(int* status) {
  void* p = nullptr;
  const cudaError_t err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (err != cudaSuccess || p == nullptr) {
    set_last_cuda_error(err);
    *status = MUZO_ERR_CUDA;
    return nullptr;
  }
  *status = MUZO_OK;
  return static_cast<NoallocScratch*>(p);
}

}  // namespace
}  // namespace muzo

using namespace muzo;

extern "C" {

int muzo_ns_normalize_noalloc(const void* const* inputs, void* const* outputs, const int64_t* numels,
                              int nblocks, int dtype, int32_t* d_flags, void* stream) {
  if (nblocks < 0 || (nblocks > 0 && (inputs == nullptr || outputs == nullptr || numels == nullptr)))
    return MUZO_ERR_ARG;
  if (nblocks > kNoallocMaxBlocks) return MUZO_ERR_CAPACITY;  // the scratch holds 64 matrices
  if (dtype != MUZO_F32 && dtype != MUZO_BF16 && dtype != MUZO_F16) return MUZO_ERR_DTYPE;
  if (nblocks == 0) return MUZO_OK;
  if (d_flags == nullptr) return MUZO_ERR_ARG;
  for (int i = 0; i < nblocks; ++i)
    if (inputs[i] == nullptr || outputs[i] == nullptr || numels[i] < 0) return MUZO_ERR_ARG;

  TableParam table;
  int nsegs = 0;
  int64_t total_items = 0;
  int st = muzo_plan_linear(numels, const_cast<void* const*>(inputs), outputs, nblocks, table.segs,
                            kNoallocMaxBlocks, &nsegs, &total_items);
  if (st != MUZO_OK) return st;
  table.nsegs = nsegs;
  if (total_items / MUZO_ITEMS_PER_CTA > 0x7fffffffLL) return MUZO_ERR_UNSUPPORTED;

  NoallocScratch* scratch = scratch_for_current_device(&st);
  if (st != MUZO_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  noalloc_setup_kernel<<<1, kNoallocMaxBlocks, 0, s>>>(table, scratch, d_flags);
  st = launch_status();
  if (st != MUZO_OK || total_items == 0) return st;
  const unsigned grid = static_cast<unsigned>(total_items / MUZO_ITEMS_PER_CTA);
  switch (dtype) {
    case MUZO_BF16: noalloc_prepare_kernel<MUZO_BF16><<<grid, kElemThreads, 0, s>>>(scratch, nsegs, d_flags); break;
    case MUZO_F16: noalloc_prepare_kernel<MUZO_F16><<<grid, kElemThreads, 0, s>>>(scratch, nsegs, d_flags); break;
    default: noalloc_prepare_kernel<MUZO_F32><<<grid, kElemThreads, 0, s>>>(scratch, nsegs, d_flags); break;
  }
  st = launch_status();
  if (st != MUZO_OK) return st;
  noalloc_normalize_kernel<<<grid, kElemThreads, 0, s>>>(scratch, nsegs, d_flags);
  return launch_status();
}

}  // extern "C"
