// Peer-memory plumbing of the multi-GPU chunk pipeline: export a device
// buffer to the other ranks' processes (CUDA IPC), map theirs, and copy a
// shard with the copy engines.  Host code only - no kernel here - so a shard
// moving over NVLink takes no SM time from the layer kernels running beside
// it.
//
// Reference: the config-4 all-gather of the encoder-norm outputs has no
// counterpart in the reference (its engine runs on one GPU,
// native/asr/src/engine.cu:1166-1616); this is the exchange step of the
// chunk-sharded run.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstring>

#include "vl_common.cuh"

namespace vl {
namespace {

using MemGetAddressRange = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

// cuMemGetAddressRange through the runtime's driver entry point table, so the
// library does not link libcuda directly (it still loads on a host without a
// driver, where only argument checks run).
cudaError_t allocation_base(const void* ptr, void** base, size_t* size) {
  static MemGetAddressRange fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    const cudaError_t err = cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q);
    if (err != cudaSuccess) return err;
    if (q != cudaDriverEntryPointSuccess || p == nullptr) return cudaErrorNotSupported;
    fn = reinterpret_cast<MemGetAddressRange>(p);
  }
  CUdeviceptr b = 0;
  size_t n = 0;
  if (fn(&b, &n, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) return cudaErrorInvalidValue;
  *base = reinterpret_cast<void*>(b);
  *size = n;
  return cudaSuccess;
}

}  // namespace

cudaError_t ipc_export(const void* ptr, void* handle_out, uint64_t* offset_out) {
  void* base = nullptr;
  size_t size = 0;
  cudaError_t err = allocation_base(ptr, &base, &size);
  if (err != cudaSuccess) return err;
  cudaIpcMemHandle_t h;
  err = cudaIpcGetMemHandle(&h, base);
  if (err != cudaSuccess) return err;
  static_assert(sizeof(h) == VL_IPC_HANDLE_BYTES, "cudaIpcMemHandle_t size");
  std::memcpy(handle_out, &h, sizeof(h));
  *offset_out = static_cast<uint64_t>(static_cast<const char*>(ptr) - static_cast<char*>(base));
  return cudaSuccess;
}

cudaError_t ipc_open(const void* handle, void** base_out) {
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  return cudaIpcOpenMemHandle(base_out, h, cudaIpcMemLazyEnablePeerAccess);
}

cudaError_t ipc_close(void* base) { return cudaIpcCloseMemHandle(base); }

cudaError_t copy_async(void* dst, const void* src, size_t bytes, cudaStream_t stream) {
  return cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, stream);
}

}  // namespace vl
