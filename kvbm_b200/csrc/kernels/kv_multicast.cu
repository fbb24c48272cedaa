// One-to-many KV fan-out through NVSwitch multicast (NVLS).
//
// Every rank of a replicated-data group holds its G1 pool inside one
// multicast object (the same geometry at the same offset on every rank). The
// source rank reads each (block, layer, K/V) chunk of its own pool once and
// writes it with `multimem.st` to the multicast address of the destination
// chunk: the switch delivers every 16-byte store to every member's pool, so
// the source GPU sends each byte over NVLink once whatever the group size
// (one store per peer would send it world_size - 1 times). The last CTA to
// finish then adds 1 to the group's completion counter, also through the
// multicast address, with release semantics at system scope; each receiving
// rank orders its compute stream behind the counter with a bounded wait.
//
// Ordering: each CTA makes its stores visible with a system-scope fence
// before it bumps the launch's CTA counter; the last CTA fences again after
// reading the counter, so its release-add is ordered after every CTA's
// stores (the fence/atomic/fence pattern of the threadfence-reduction
// sample). The local CTA counter resets itself for the next launch.
//
// Parity: crates/kvbm-engine/src/collectives/mod.rs:75-113 (broadcast of G1
// blocks from rank 0 to every rank for replicated-data / MLA workers) and
// worker/physical/replicated.rs:50-150; the reference broadcasts with NCCL.
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "kvbm_kernels.h"

namespace {

struct McParams {
  uint64_t src_layer_base[KVBM_MAX_LAYERS];  // this rank's pool, absolute per-layer addresses
  uint64_t dst_layer_off[KVBM_MAX_LAYERS];   // per-layer offsets from the pool base (same on every rank)
  uint64_t mc_base;                          // multicast address of the pool base
  int64_t block_stride, outer_stride;
  int64_t chunk_units;                       // 16-byte units per (block, layer, outer) chunk
  const int32_t* src_ids;
  const int32_t* dst_ids;
  int32_t num_blocks, num_layers, outer;
  int32_t pool_blocks;                       // ids must lie in [0, pool_blocks) on both sides
  int* status;                               // kStatusBadIndex when an id is out of range (chunk skipped)
  uint64_t flag_mc;                          // multicast address of the group's u64 completion counter
  unsigned int* cta_done;                    // this rank's CTA counter (zero between launches)
};

__device__ __forceinline__ void multimem_st_v4(uint64_t addr, uint4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

__device__ __forceinline__ void multimem_add_release_u64(uint64_t addr, uint64_t v) {
  asm volatile("multimem.red.release.sys.global.add.u64 [%0], %1;" ::"l"(addr), "l"(v) : "memory");
}

__device__ __forceinline__ uint4 ld_nc_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

constexpr int kThreads = 512;
constexpr int kUnroll = 4;

__global__ void __launch_bounds__(kThreads) kv_multicast_kernel(const __grid_constant__ McParams P) {
  const int64_t L = P.num_layers, O = P.outer;
  const int64_t total = int64_t(P.num_blocks) * L * O;
  const int64_t G = gridDim.x, b = blockIdx.x;
  const int64_t per = total / G, rem = total % G;
  const int64_t count = per + (b < rem ? 1 : 0);
  const int64_t begin = b * per + (b < rem ? b : rem);
  const int64_t U = P.chunk_units;
  for (int64_t c = begin; c < begin + count; ++c) {
    int64_t r = c;
    const int64_t o = r % O;
    r /= O;
    const int64_t l = r % L;
    const int64_t i = r / L;
    const int64_t sb = P.src_ids[i], db = P.dst_ids[i];
    if (sb < 0 || db < 0 || sb >= P.pool_blocks || db >= P.pool_blocks) {
      if (threadIdx.x == 0 && P.status) atomicExch(P.status, kvbm::kStatusBadIndex);
      continue;
    }
    const uint4* src = reinterpret_cast<const uint4*>(P.src_layer_base[l] + sb * P.block_stride + o * P.outer_stride);
    const uint64_t dst = P.mc_base + P.dst_layer_off[l] + uint64_t(db * P.block_stride + o * P.outer_stride);
    int64_t u = threadIdx.x;
    for (; u + (kUnroll - 1) * kThreads < U; u += kUnroll * kThreads) {
      uint4 v[kUnroll];
#pragma unroll
      for (int k = 0; k < kUnroll; ++k) v[k] = ld_nc_v4(src + u + k * kThreads);
#pragma unroll
      for (int k = 0; k < kUnroll; ++k) multimem_st_v4(dst + 16 * uint64_t(u + k * kThreads), v[k]);
    }
    for (; u < U; u += kThreads) multimem_st_v4(dst + 16 * uint64_t(u), ld_nc_v4(src + u));
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const unsigned int prev = atomicAdd(P.cta_done, 1u);
    if (prev == gridDim.x - 1) {
      __threadfence_system();
      *reinterpret_cast<volatile unsigned int*>(P.cta_done) = 0u;
      multimem_add_release_u64(P.flag_mc, 1ull);
    }
  }
}

__global__ void multicast_signal_kernel(uint64_t flag_mc) {
  __threadfence_system();
  multimem_add_release_u64(flag_mc, 1ull);
}

}  // namespace

extern "C" int kvbm_signal_multicast(uint64_t flag_mc, cudaStream_t stream) {
  if (!flag_mc || flag_mc % 8) return cudaErrorInvalidValue;
  multicast_signal_kernel<<<1, 1, 0, stream>>>(flag_mc);
  return cudaGetLastError();
}

extern "C" int kvbm_kv_multicast(const uint64_t* src_layer_base, const uint64_t* dst_layer_off, int num_layers,
                                 uint64_t mc_base, int64_t block_stride, int64_t outer_stride, int64_t chunk_bytes,
                                 int outer, const int32_t* src_ids, const int32_t* dst_ids, int num_blocks,
                                 int pool_blocks, uint64_t flag_mc, unsigned int* cta_done, int* status,
                                 int max_ctas, cudaStream_t stream) {
  if (num_layers <= 0 || num_layers > KVBM_MAX_LAYERS || num_blocks < 0 || outer <= 0) return cudaErrorInvalidValue;
  if (!mc_base || !flag_mc || !cta_done || !src_ids || !dst_ids) return cudaErrorInvalidValue;
  // every chunk start and size must be 16-byte aligned for the vector stores
  if (chunk_bytes <= 0 || chunk_bytes % 16 || block_stride % 16 || outer_stride % 16 || mc_base % 16 ||
      flag_mc % 8)
    return cudaErrorInvalidValue;
  McParams P{};
  for (int l = 0; l < num_layers; ++l) {
    if (src_layer_base[l] % 16 || dst_layer_off[l] % 16) return cudaErrorInvalidValue;
    P.src_layer_base[l] = src_layer_base[l];
    P.dst_layer_off[l] = dst_layer_off[l];
  }
  P.mc_base = mc_base;
  P.block_stride = block_stride;
  P.outer_stride = outer_stride;
  P.chunk_units = chunk_bytes / 16;
  P.src_ids = src_ids;
  P.dst_ids = dst_ids;
  P.num_blocks = num_blocks;
  P.pool_blocks = pool_blocks;
  P.status = status;
  P.num_layers = num_layers;
  P.outer = outer;
  P.flag_mc = flag_mc;
  P.cta_done = cta_done;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t chunks = int64_t(num_blocks) * num_layers * outer;
  int64_t grid = max_ctas > 0 ? max_ctas : 2 * sms;
  if (grid > chunks) grid = chunks > 0 ? chunks : 1;
  kv_multicast_kernel<<<static_cast<unsigned>(grid), kThreads, 0, stream>>>(P);
  return cudaGetLastError();
}
