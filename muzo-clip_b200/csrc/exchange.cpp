// Host side of the weight exchange between the ranks of one node: interprocess handles of the
// allocations that hold the parameters, and the copy-engine pushes of updated blocks into the
// peers' parameter memory. No kernel runs here: every push is one cudaMemcpyAsync (device to
// device through the peer mapping), so the transfer takes no SM from the Newton-Schulz GEMMs.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdint>
#include <cstring>

#include "muzo_b200.h"

namespace muzo {
void set_last_cuda_error(cudaError_t err);
}

namespace {

// cuMemGetAddressRange through the runtime's driver entry point (no link against libcuda).
PFN_cuMemGetAddressRange_v3020 address_range_fn() {
  static const PFN_cuMemGetAddressRange_v3020 fn = []() -> PFN_cuMemGetAddressRange_v3020 {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &p, 3020, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(p);
    return nullptr;
  }();
  return fn;
}

int fail(cudaError_t err) {
  muzo::set_last_cuda_error(err);
  return MUZO_ERR_CUDA;
}

}  // namespace

extern "C" {

int muzo_ipc_export(const void* d_ptr, void* handle_out, uint64_t* offset_out, uint64_t* alloc_bytes_out) {
  if (d_ptr == nullptr || handle_out == nullptr || offset_out == nullptr) return MUZO_ERR_ARG;
  auto range = address_range_fn();
  if (range == nullptr) return MUZO_ERR_UNSUPPORTED;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(d_ptr)) != CUDA_SUCCESS) return MUZO_ERR_UNSUPPORTED;
  cudaIpcMemHandle_t h;
  cudaError_t err = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (err != cudaSuccess) {
    cudaGetLastError();
    muzo::set_last_cuda_error(err);
    return MUZO_ERR_UNSUPPORTED;  // e.g. memory from a virtual-memory or stream-ordered pool
  }
  static_assert(sizeof(h) == MUZO_IPC_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle_out, &h, sizeof(h));
  *offset_out = static_cast<uint64_t>(reinterpret_cast<CUdeviceptr>(d_ptr) - base);
  if (alloc_bytes_out != nullptr) *alloc_bytes_out = static_cast<uint64_t>(size);
  return MUZO_OK;
}

int muzo_ipc_import(const void* handle, void** d_base_out) {
  if (handle == nullptr || d_base_out == nullptr) return MUZO_ERR_ARG;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  cudaError_t err = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (err != cudaSuccess) {
    cudaGetLastError();
    return fail(err);
  }
  *d_base_out = p;
  return MUZO_OK;
}

int muzo_ipc_close(void* d_base) {
  if (d_base == nullptr) return MUZO_ERR_ARG;
  cudaError_t err = cudaIpcCloseMemHandle(d_base);
  if (err != cudaSuccess) {
    cudaGetLastError();
    return fail(err);
  }
  return MUZO_OK;
}

int muzo_push_blocks(void* const* dst, const void* const* src, const uint64_t* bytes, int n, void* stream) {
  if (n < 0 || (n > 0 && (dst == nullptr || src == nullptr || bytes == nullptr))) return MUZO_ERR_ARG;
  for (int i = 0; i < n; ++i)
    if (dst[i] == nullptr || src[i] == nullptr) return MUZO_ERR_ARG;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  for (int i = 0; i < n; ++i) {
    if (bytes[i] == 0) continue;
    cudaError_t err = cudaMemcpyAsync(dst[i], src[i], static_cast<size_t>(bytes[i]), cudaMemcpyDeviceToDevice, s);
    if (err != cudaSuccess) return fail(err);
  }
  return MUZO_OK;
}

}  // extern "C"
