// C ABI of the kvbm_b200 sm_100a kernel library (libkvbm_cuda.so).
//
// Every entry point returns a cudaError_t value as int (0 = success) and is
// asynchronous on the given stream. Pointer tables passed to kernels must be
// device-accessible (device memory or mapped pinned host memory).
//
// Behavioural parity (not code) with the reference kernel ABI:
//   kvbm_universal_from_block   <-> crates/kvbm-kernels/cuda/tensor_kernels.cu:347 (K1)
//   kvbm_block_from_universal   <-> crates/kvbm-kernels/cuda/tensor_kernels.cu:376 (K2)
//   kvbm_nhd_hnd_transpose      <-> crates/kvbm-kernels/cuda/tensor_kernels.cu:502 (K3)
//   kvbm_copy_pairs             <-> crates/kvbm-kernels/cuda/tensor_kernels.cu:724 (K4)
// Dtype codes keep the reference's numbering (crates/kvbm-kernels/src/tensor_kernels.rs:40)
// and the block layout codes keep NHD=0 / HND=1 (tensor_kernels.rs:51).
#pragma once
#include <stdint.h>
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KVBM_MAX_LAYERS 128

enum KvbmDtype { KVBM_F16 = 0, KVBM_BF16 = 1, KVBM_F32 = 2, KVBM_F64 = 3, KVBM_FP8_E4M3 = 4 };
enum KvbmBlockLayout { KVBM_NHD = 0, KVBM_HND = 1 };

// How one side of a tile transfer turns (pair p, layer i, outer o) into a
// base address. A tile is the [page_size, head_dim] slab of one head.
enum KvbmAddrMode {
  // layer_base[i] + ids[p] * block_stride + o * outer_stride
  KVBM_ADDR_LAYER_BASES = 0,
  // table[p] + (layer_offset + i) * layer_stride + o * outer_stride
  KVBM_ADDR_BLOCK_TABLE = 1,
  // table[(p * chunk_layers + i) * chunk_outer + o]
  KVBM_ADDR_CHUNK_TABLE = 2,
};

typedef struct KvbmSide {
  int32_t mode;
  int32_t head_offset;     // added to the tile's head index on this side
  int32_t chunk_layers;    // CHUNK_TABLE: layers per block in the table
  int32_t chunk_outer;     // CHUNK_TABLE: outer chunks per layer in the table
  const uint64_t* table;   // BLOCK_TABLE / CHUNK_TABLE pointer table (device-accessible)
  const int32_t* ids;      // LAYER_BASES block ids (device-accessible), one per pair
  int64_t block_stride;    // bytes
  int64_t layer_stride;    // bytes (BLOCK_TABLE)
  int64_t layer_offset;    // layers (BLOCK_TABLE)
  int64_t outer_stride;    // bytes
  int64_t token_stride;    // bytes
  int64_t head_stride;     // bytes
  // Optional fp32 scales for fp8 data, one per (block, layer, outer, head):
  // scales[blk * s_block + (s_layer_offset + i) * s_layer + o * s_outer + head * s_head]
  // where blk = ids[p] in LAYER_BASES mode and p otherwise.
  float* scales;
  int64_t s_block, s_layer, s_outer, s_head, s_layer_offset;
  uint64_t layer_base[KVBM_MAX_LAYERS];
} KvbmSide;

typedef struct KvbmTileShape {
  int32_t num_pairs;
  int32_t num_layers;
  int32_t num_outer;
  int32_t num_heads;   // heads moved per tile set
  int32_t page_size;   // tokens per block
  int32_t head_dim;    // elements
  int32_t src_dtype;
  int32_t dst_dtype;
} KvbmTileShape;

// Generic fused gather -> (layout transform, head reshard, fp8 quant/dequant)
// -> scatter. The destination may be local HBM, mapped pinned host memory or
// a peer GPU's memory mapped through CUDA IPC. One warp per tile.
int kvbm_kv_tile_xfer(const KvbmSide* src, const KvbmSide* dst, const KvbmTileShape* shape, int max_ctas,
                      cudaStream_t stream);

// Same contract, staged through shared memory: one elected thread issues 1-D
// bulk async copies (TMA engine, local source only) of whole contiguous
// (pair, layer, outer) chunks into a multi-stage ring; consumer warps convert
// and store. Requires the source chunk [page, heads, head_dim] (or its HND
// transpose) to be contiguous and 16-byte aligned; returns
// cudaErrorInvalidValue otherwise so callers fall back to kvbm_kv_tile_xfer.
int kvbm_kv_chunk_xfer_tma(const KvbmSide* src, const KvbmSide* dst, const KvbmTileShape* shape, int max_ctas,
                           cudaStream_t stream);

// One entry point for both engines. `engine`: 0 auto (a TMA engine when the
// source chunks allow it, else the tile kernel), 1 tile, 2 TMA (returns
// cudaErrorInvalidValue instead of falling back when the TMA engines cannot
// take the transfer). Among the TMA engines, the bulk copy (TMA loads and TMA
// stores only, no SM data path) runs when the destination chunk is the
// source chunk's byte image and `flags` allows TMA stores to the destination
// (KVBM_XFER_DST_LOCAL: this GPU's memory; KVBM_XFER_BULK_PEER: a peer GPU's
// memory); otherwise the staged pipeline with consumer warps. `*ran` (may be
// null) receives which kernel was launched: 1 tile, 2 TMA pipeline, 3 TMA
// bulk copy.
#define KVBM_XFER_DST_LOCAL 1
#define KVBM_XFER_BULK_PEER 2
#define KVBM_XFER_NO_BULK 4
int kvbm_kv_xfer(const KvbmSide* src, const KvbmSide* dst, const KvbmTileShape* shape, int engine, int max_ctas,
                 int flags, int* ran, cudaStream_t stream);

// Status word the TMA engines write when a bounded wait gives up (3) or a
// chunk address is misaligned (2); 0 = no error since the last reset. It
// lives in mapped host memory, so reading it needs no device synchronization
// (read it after the transfer's stream has passed the launch).
int kvbm_xfer_status(int device, int reset);

// Test hook: the limit of the TMA engines' pipeline waits for launches made
// after the call (0 restores the default of 2 s; 1 makes every pipeline wait
// give up at once). Waits that drain copies already issued keep the full
// limit, so no copy is in flight when a CTA exits.
void kvbm_xfer_set_wait_limit_ns(uint64_t ns);
// 1 (default): fp8 casts whose head tile fits one register batch per lane run
// the software-pipelined persistent cast kernel; 0: the one-tile-at-a-time kernel.
void kvbm_xfer_set_cast_pipeline(int on);
// Quarters (0, 1, 2 or 4) of the pipelined cast kernel's bf16 -> fp8 and
// fp8 -> bf16 conversions done on the integer / FMA pipes (bit-identical for
// finite values) instead of with the conversion instructions. Defaults: 0 for
// quantise, 1 for dequantise.
void kvbm_xfer_set_cast_softconv(int quant_quarters, int dequant_quarters);

// Split-by-bytes batched copy of num_pairs (src, dst) regions of equal size.
// `align` is the alignment (16, 8, 4, 2 or 1) that every pointer and
// `bytes_per_pair` is guaranteed to have.
int kvbm_copy_pairs(const uint64_t* src_ptrs, const uint64_t* dst_ptrs, uint64_t num_pairs, uint64_t bytes_per_pair,
                    int align, int max_ctas, cudaStream_t stream);

// Reference-compatible permutes over pointer tables.
int kvbm_universal_from_block(void* const* universal_ptrs, const void* const* block_ptrs, size_t num_blocks, size_t nh,
                              size_t nl, size_t no, size_t nt, size_t hd, size_t nl_full, size_t nl_offset,
                              int dtype, int layout, cudaStream_t stream);
int kvbm_block_from_universal(const void* const* universal_ptrs, void* const* block_ptrs, size_t num_blocks,
                              size_t nh, size_t nl, size_t no, size_t nt, size_t hd, size_t nl_full,
                              size_t nl_offset, int dtype, int layout, cudaStream_t stream);
int kvbm_nhd_hnd_transpose(const void* const* src_chunks, void* const* dst_chunks, size_t num_blocks, size_t nl,
                           size_t no, size_t nt, size_t nh, size_t hd, int dtype, int src_layout,
                           cudaStream_t stream);

// Completion flags at system scope. signal: release-store `value` into
// `flag` (which may live on a peer GPU). wait: spin (bounded by timeout_ns of
// %globaltimer) until *flag >= expected; on timeout writes 1 to *status and
// returns so the context stays usable.
int kvbm_signal_flag(uint64_t* flag, uint64_t value, cudaStream_t stream);
int kvbm_wait_flag(const uint64_t* flag, uint64_t expected, uint64_t timeout_ns, int* status, cudaStream_t stream);

// Fan-out of (block, layer, K/V) chunks from this rank's pool into every
// member of an NVLink multicast group (multimem stores through `mc_base`, the
// multicast address of the pool base); the last CTA adds 1 to the group's
// u64 counter at multicast address `flag_mc`. `cta_done` is a zeroed device
// u32 of this rank. Geometry must match on every rank; ids outside
// [0, pool_blocks) are skipped and reported in `status` (kStatusBadIndex).
int kvbm_kv_multicast(const uint64_t* src_layer_base, const uint64_t* dst_layer_off, int num_layers,
                      uint64_t mc_base, int64_t block_stride, int64_t outer_stride, int64_t chunk_bytes, int outer,
                      const int32_t* src_ids, const int32_t* dst_ids, int num_blocks, int pool_blocks,
                      uint64_t flag_mc, unsigned int* cta_done, int* status, int max_ctas, cudaStream_t stream);
// Add 1 (release, system scope) to the u64 counter at multicast address `flag_mc`.
int kvbm_signal_multicast(uint64_t flag_mc, cudaStream_t stream);

// Layout-independent 64-bit checksum per block: the wrapping sum over every
// 4-byte word w of the block's selected layers/heads of mix64(w, i), with i
// the word's index in canonical [layer, outer, token, head, word] order.
// Blocks holding the same values hash equal whatever their physical layout
// (NHD / HND, fully contiguous / layer separate / universal). `out` gets
// shape->num_pairs values; src_dtype gives the element size.
int kvbm_kv_checksum(const KvbmSide* side, const KvbmTileShape* shape, uint64_t* out, cudaStream_t stream);

// Number of SMs of the current device (cached).
int kvbm_sm_count(void);

// ---- Llama driver harness: paged decode attention (llama_ops.cu) ----------
//
// Split-KV paged decode attention over a block table, grouped-query heads
// (hq = group * hkv), head_dim 128, bf16 q / K / V / out. The caller provides
// the split partials: part_acc (batch * hq * splits * 128 floats) and
// part_ml (batch * hq * splits * 2 floats). Two launches (split kernel, then
// combine).
int kvbm_paged_decode_attn(const void* q, const void* k_base, const void* v_base, int64_t block_stride,
                           int64_t token_stride, int64_t head_stride, int page, const int32_t* block_table,
                           int max_blocks, const int32_t* seq_lens, int batch, int hq, int hkv, int hd,
                           float softmax_scale, int splits, float* part_acc, float* part_ml, void* out,
                           cudaStream_t stream);

// The same attention for callers that cannot allocate device memory when they
// call in (an application that owns all device memory in its own arena, code
// running inside an allocator callback, a path that cannot absorb the device
// synchronization cudaMalloc / cudaFree may cause). No counterpart in the
// reference block manager: an addition of this library.
//
// The split partials live in a fixed array of device memory inside this
// library (kvbm_paged_decode_attn_noalloc_max_rows() rows of 130 floats,
// about 4.3 MB, held by every GPU that loads the library until the process
// exits). The first call on a device, with that device current, looks the
// array's address up once (cudaGetSymbolAddress) and caches it: make that
// first call before any stream capture. batch * hq * splits above the
// capacity is rejected with cudaErrorInvalidValue. All calls on a device share
// the array: calls whose kernels can overlap on the GPU race on it, so order
// them on one stream or with events. After cudaDeviceReset the cached address
// is stale: do not call this entry point on a device after resetting it.
// On failure kvbm_last_error_message() says why (per calling thread).
int kvbm_paged_decode_attn_noalloc(const void* q, const void* k_base, const void* v_base, int64_t block_stride,
                                   int64_t token_stride, int64_t head_stride, int page, const int32_t* block_table,
                                   int max_blocks, const int32_t* seq_lens, int batch, int hq, int hkv, int hd,
                                   float softmax_scale, int splits, void* out, cudaStream_t stream);
int kvbm_paged_decode_attn_noalloc_max_rows(void);
const char* kvbm_last_error_message(void);

#ifdef __cplusplus
}
#endif
