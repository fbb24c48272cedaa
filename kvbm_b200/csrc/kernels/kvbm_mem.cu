// Host-side memory plumbing for the block manager's tiers, exported through
// the same C ABI as the kernels:
//   * G1 pools allocated with cudaMalloc outside the framework allocator, so
//     a CUDA IPC handle maps exactly the pool (no sub-allocation offsets);
//   * CUDA IPC export/import of G1 pools and of completion-flag pages between
//     the processes of one node (the prefill -> decode data path);
//   * G2 pinned host memory, mapped into the device address space so SM
//     kernels can gather/scatter it directly over PCIe / C2C.
//
// Parity: the reference allocates and registers tiers through dynamo-memory
// and NIXL (crates/kvbm-physical/src/layout/builder.rs, allocate_device /
// allocate_pinned); here the same roles are plain CUDA runtime calls.
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

extern "C" {

int kvbm_device_alloc(uint64_t bytes, void** out) {
  if (!out) return cudaErrorInvalidValue;
  return cudaMalloc(out, bytes);
}

int kvbm_device_free(void* p) { return cudaFree(p); }

int kvbm_memset_async(void* p, int value, uint64_t bytes, cudaStream_t stream) {
  return cudaMemsetAsync(p, value, bytes, stream);
}

// 64-byte opaque IPC handle of a cudaMalloc'd base pointer.
int kvbm_ipc_get_handle(void* p, uint8_t* out64) {
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) return e;
  memcpy(out64, &h, sizeof(h));
  return cudaSuccess;
}

int kvbm_ipc_open_handle(const uint8_t* in64, void** out) {
  cudaIpcMemHandle_t h;
  memcpy(&h, in64, sizeof(h));
  return cudaIpcOpenMemHandle(out, h, cudaIpcMemLazyEnablePeerAccess);
}

int kvbm_ipc_close(void* p) { return cudaIpcCloseMemHandle(p); }

int kvbm_ipc_handle_size(void) { return static_cast<int>(sizeof(cudaIpcMemHandle_t)); }

// Pinned host allocation mapped into the device address space (portable to
// every device). With UVA the returned pointer is valid on host and device.
int kvbm_host_alloc_mapped(uint64_t bytes, void** out) {
  if (!out) return cudaErrorInvalidValue;
  return cudaHostAlloc(out, bytes, cudaHostAllocMapped | cudaHostAllocPortable);
}

int kvbm_host_free(void* p) { return cudaFreeHost(p); }

// Page-lock and map an existing host range (e.g. a hugepage mmap).
int kvbm_host_register(void* p, uint64_t bytes) {
  return cudaHostRegister(p, bytes, cudaHostRegisterMapped | cudaHostRegisterPortable);
}

int kvbm_host_unregister(void* p) { return cudaHostUnregister(p); }

int kvbm_host_device_pointer(void* host, void** dev) { return cudaHostGetDevicePointer(dev, host, 0); }

int kvbm_can_access_peer(int dev, int peer, int* out) { return cudaDeviceCanAccessPeer(out, dev, peer); }

int kvbm_enable_peer_access(int peer) {
  cudaError_t e = cudaDeviceEnablePeerAccess(peer, 0);
  if (e == cudaErrorPeerAccessAlreadyEnabled) {
    cudaGetLastError();
    return cudaSuccess;
  }
  return e;
}

// One async copy of `bytes` (direction inferred through UVA). This is the
// copy-engine baseline the SM kernels are measured against.
int kvbm_memcpy_async(void* dst, const void* src, uint64_t bytes, cudaStream_t stream) {
  return cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, stream);
}

// Copy-engine baseline for a batch of equal-size regions: one
// cudaMemcpyAsync per region, issued from host pointer tables.
int kvbm_memcpy_pairs_ce(const uint64_t* src, const uint64_t* dst, uint64_t n, uint64_t bytes, cudaStream_t stream) {
  for (uint64_t i = 0; i < n; ++i) {
    cudaError_t e = cudaMemcpyAsync(reinterpret_cast<void*>(dst[i]), reinterpret_cast<const void*>(src[i]), bytes,
                                    cudaMemcpyDefault, stream);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

// Copy-engine baseline for a strided batch: `height` rows of `width` bytes,
// `spitch` / `dpitch` bytes apart (one request's layer of KV blocks).
int kvbm_memcpy_2d_async(void* dst, uint64_t dpitch, const void* src, uint64_t spitch, uint64_t width,
                         uint64_t height, cudaStream_t stream) {
  return cudaMemcpy2DAsync(dst, dpitch, src, spitch, width, height, cudaMemcpyDefault, stream);
}

int kvbm_get_device(int* dev) { return cudaGetDevice(dev); }

const char* kvbm_error_string(int code) { return cudaGetErrorString(static_cast<cudaError_t>(code)); }

}  // extern "C"
