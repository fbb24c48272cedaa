// Skinny GEMM on the 5th-generation tensor cores (tcgen05 + TMEM + TMA):
//   Y[m, n] = sum_k X[m, k] * W[n, k]      (Y = X W^T, bf16 in, fp32 accumulate, bf16 out)
// for a handful of rows m (a decode batch, M <= 128) against a large weight W
// [N, K] - the projections of a decode step, which are bound by streaming W
// once from HBM.
//
// Roles are swapped so the big operand fills the 128-row MMA: each CTA
// computes D = W_tile X^T for 128 consecutive weight rows (UMMA M = 128)
// against all tokens (UMMA N = BN, the token count rounded up to 16), with D
// accumulating in TMEM (128 lanes x BN fp32 columns).
//
// * TMA: per K chunk of 64 elements (128 bytes), one tiled 2-D bulk tensor
//   load of the 128 x 64 weight tile and one of the BN x 64 activation tile,
//   128-byte swizzled, into a ring of kStages shared-memory stages. Both are
//   this GPU's own memory; no cluster multicast.
// * MMA: one thread issues 4 tcgen05.mma (K = 16 each, the descriptor start
//   advanced 32 bytes within the 128-byte swizzle atom) per stage and
//   tcgen05.commit's the stage's "empty" mbarrier, so the producer refills a
//   stage as soon as the tensor cores are done reading it.
// * Split-K: grid = (N / 128) x splits. A single split writes bf16 directly;
//   otherwise each split adds its fp32 tile into a workspace with red.add and
//   the last split of a tile (ticket counter) converts the tile to bf16 and
//   re-zeroes the workspace and counter for the next launch.
// * Every mbarrier wait is bounded (%globaltimer); a CTA that gives up records
//   kStatusPipelineTimeout in g_gemm_status, waits (bounded) for its own copies
//   and MMAs, frees its TMEM and returns.
#include "common.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstring>
#include <mutex>

using namespace kvbm;

namespace {

constexpr int kThreads = 128;         // 4 warps: warp w reads TMEM lanes [32w, 32w + 32)
constexpr int kTileN = 128;           // weight rows per CTA (UMMA M)
constexpr int kChunkK = 64;           // K elements per stage (128 bytes of bf16: one swizzle atom row)
constexpr uint64_t kWaitNs = 2000000000ull;

// Ring depth: as many stages of (128 + BN) x 128 bytes as fit in ~200 KiB, at most 8.
template <int BN>
struct Ring {
  static constexpr uint32_t kStageBytes = (kTileN + BN) * kChunkK * 2;
  static constexpr int kStages = (200 * 1024) / kStageBytes < 8 ? (200 * 1024) / kStageBytes : 8;
};

__device__ int g_gemm_status = 0;

// ---- tcgen05 / TMA wrappers ----------------------------------------------------
KVBM_DEVICE void tma_load_2d(void* smem_dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

KVBM_DEVICE void tmem_alloc(uint32_t* smem_slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_slot)),
               "r"(ncols)
               : "memory");
}
KVBM_DEVICE void tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::); }
KVBM_DEVICE void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
KVBM_DEVICE void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
KVBM_DEVICE void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (bf16 x bf16 -> fp32)
KVBM_DEVICE void umma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
}
KVBM_DEVICE void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 32 TMEM lanes (one per thread of the warp) x 16 consecutive 32-bit columns.
KVBM_DEVICE void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor, K-major, 128-byte swizzle: rows of 128
// bytes, 8-row groups 1024 bytes apart (stride byte offset), leading byte
// offset unused (1), version 1, layout type 2 (SWIZZLE_128B).
KVBM_DEVICE uint64_t smem_desc_k128(const void* p) {
  const uint64_t addr = smem_u32(p);
  return ((addr >> 4) & 0x3FFFull) | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}

// Instruction descriptor: D fp32, A and B bf16, both K-major, M = 128, N = n.
__host__ __device__ constexpr uint32_t idesc_bf16(int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) | ((128u >> 4) << 24);
}

struct GemmParams {
  int M, N, K;
  int chunks_per_split;  // K chunks handled by one split
  int splits;
  __nv_bfloat16* y;      // [M, N] row stride ldy
  int ldy;
  float* ws;             // [M, N] fp32 zeros (splits > 1)
  unsigned int* tickets;  // [N / 128] zeros (splits > 1)
};

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
    skinny_gemm_tc_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_x,
                          const __grid_constant__ GemmParams P) {
  constexpr uint32_t kBytesW = kTileN * kChunkK * 2;  // 16 KiB
  constexpr uint32_t kStageBytes = Ring<BN>::kStageBytes;
  constexpr int kStages = Ring<BN>::kStages;
  constexpr uint32_t kTmemCols = BN < 32 ? 32 : BN;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte alignment for the swizzle atoms
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t full[kStages], empty[kStages], done;
  __shared__ uint32_t tmem_base;
  __shared__ int failed;
  __shared__ unsigned int ticket;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, split = blockIdx.y;
  const int n0 = tile * kTileN;
  const int kc0 = split * P.chunks_per_split;
  const int total_chunks = (P.K + kChunkK - 1) / kChunkK;
  const int nchunks = max(0, min(P.chunks_per_split, total_chunks - kc0));

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&done, 1);
    fence_mbar_init();
    failed = 0;
  }
  if (warp == 0) {
    tmem_alloc(&tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_d = tmem_base;

  // ---- producer + MMA issuer: one thread -----------------------------------
  int issued = 0, consumed = 0;
  if (threadIdx.x == 0 && nchunks > 0) {
    bool ok = true;
    auto produce = [&](int c) {
      const int s = c % kStages;
      uint8_t* st = smem + s * kStageBytes;
      mbar_arrive_expect_tx(&full[s], kStageBytes);
      tma_load_2d(st, &map_w, (kc0 + c) * kChunkK, n0, &full[s]);
      tma_load_2d(st + kBytesW, &map_x, (kc0 + c) * kChunkK, 0, &full[s]);
    };
    for (; issued < min(kStages, nchunks); ++issued) produce(issued);
    for (int c = 0; c < nchunks && ok; ++c) {
      const int s = c % kStages;
      if (!mbar_wait_bounded(&full[s], (c / kStages) & 1, kWaitNs)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint8_t* st = smem + s * kStageBytes;
      const uint64_t da = smem_desc_k128(st), db = smem_desc_k128(st + kBytesW);
#pragma unroll
      for (int k = 0; k < kChunkK / 16; ++k)  // +32 bytes per K=16 step: +2 in 16-byte units
        umma_bf16(tmem_d, da + 2 * k, db + 2 * k, idesc_bf16(BN), (c > 0 || k > 0) ? 1u : 0u);
      umma_commit(&empty[s]);
      consumed = c + 1;
      if (issued < nchunks) {
        // refill this stage once the MMAs above have read it
        if (!mbar_wait_bounded(&empty[s], (c / kStages) & 1, kWaitNs)) {
          ok = false;
          break;
        }
        produce(issued++);
      }
    }
    if (ok) {
      umma_commit(&done);
    } else {
      failed = 1;
      atomicExch(&g_gemm_status, kStatusPipelineTimeout);
      // let every copy issued into this CTA's shared memory land before leaving
      for (int c = consumed; c < issued; ++c) mbar_wait_bounded(&full[c % kStages], (c / kStages) & 1, kWaitNs);
      umma_commit(&done);
    }
  }
  __syncthreads();

  // ---- epilogue: TMEM -> registers -> Y (or the split-K workspace) ----------
  bool mine = nchunks > 0 && !failed;
  if (nchunks > 0 && !mbar_wait_bounded(&done, 0, kWaitNs)) {
    mine = false;
    atomicExch(&g_gemm_status, kStatusPipelineTimeout);
  }
  // tcgen05.ld is warp-collective: every thread takes the same branch
  const bool have = __syncthreads_and(mine) != 0;
  tc_fence_after();
  const int row = n0 + warp * 32 + lane;  // weight row = output column of Y
  if (have) {
#pragma unroll
    for (int c0 = 0; c0 < BN; c0 += 16) {
      float v[16];
      tmem_ld16(tmem_d + (static_cast<uint32_t>(warp * 32) << 16) + c0, v);
      if (row < P.N) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int m = c0 + j;
          if (m < P.M) {
            if (P.splits == 1)
              P.y[static_cast<int64_t>(m) * P.ldy + row] = __float2bfloat16(v[j]);
            else
              atomicAdd(&P.ws[static_cast<int64_t>(m) * P.N + row], v[j]);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem_d, kTmemCols);

  if (P.splits > 1) {
    // the last split of this tile turns the fp32 sum into bf16 and re-arms the workspace
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) ticket = atomicAdd(&P.tickets[tile], 1u);
    __syncthreads();
    if (ticket == static_cast<unsigned int>(P.splits - 1)) {
      __threadfence();
      if (row < P.N) {
        for (int m = 0; m < P.M; ++m) {
          float* w = &P.ws[static_cast<int64_t>(m) * P.N + row];
          P.y[static_cast<int64_t>(m) * P.ldy + row] = __float2bfloat16(__ldcg(w));
          *w = 0.f;
        }
      }
      if (threadIdx.x == 0) P.tickets[tile] = 0u;
    }
  }
}

// ---- host side ------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2-D bf16 tensor [rows, cols] (row stride ld elements), box [box_rows, 64 cols], 128-byte swizzle.
bool make_map(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {ld * 2};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(kChunkK), box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int sm_count_cached() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

template <int BN>
int launch(const CUtensorMap& mw, const CUtensorMap& mx, const GemmParams& P, int tiles, cudaStream_t stream) {
  constexpr size_t smem = 1024 + static_cast<size_t>(Ring<BN>::kStages) * Ring<BN>::kStageBytes;
  static int configured = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured != dev) {
    cudaError_t e = cudaFuncSetAttribute(skinny_gemm_tc_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    configured = dev;
  }
  skinny_gemm_tc_kernel<BN><<<dim3(tiles, P.splits), kThreads, smem, stream>>>(mw, mx, P);
  return cudaGetLastError();
}

}  // namespace

// Split count the launcher would use for an (N, K) weight on this GPU.
extern "C" int kvbm_skinny_gemm_splits(int n, int k) {
  const int tiles = (n + kTileN - 1) / kTileN;
  const int chunks = (k + kChunkK - 1) / kChunkK;
  const int sms = sm_count_cached();  // one CTA per SM is resident (the ring takes most of shared memory)
  // time ~ waves of CTAs x K chunks per CTA; the fewest splits that minimise it, >= 4 chunks each
  int best = 1;
  long best_cost = -1;
  for (int s = 1; s <= 16 && (chunks + s - 1) / s >= 4; ++s) {
    const long waves = (static_cast<long>(tiles) * s + sms - 1) / sms;
    const long cost = waves * ((chunks + s - 1) / s);
    if (best_cost < 0 || cost < best_cost) {
      best = s;
      best_cost = cost;
    }
  }
  return best;
}

// Y[M, N] (row stride ldy) = X[M, K] (row stride ldx) * W[N, K]^T (row stride ldw).
// bf16, M <= 128, K % 8 == 0, all base pointers and row strides 16-byte aligned.
// With splits > 1, `ws` is an fp32 [M, N] buffer of zeros and `tickets`
// (N / 128 rounded up) 32-bit zeros; the kernel leaves both zeroed again.
extern "C" int kvbm_skinny_gemm(const void* x, int ldx, const void* w, int ldw, void* y, int ldy, int M, int N, int K,
                                int splits, float* ws, unsigned int* tickets, cudaStream_t stream) {
  if (M == 0 || N == 0) return cudaSuccess;
  if (!x || !w || !y || M < 0 || M > 128 || N < 0 || K <= 0 || K % 8 != 0) return cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w)) & 15) return cudaErrorInvalidValue;
  if ((ldx % 8) || (ldw % 8) || ldx < K || ldw < K || ldy < N) return cudaErrorInvalidValue;
  if (splits <= 0) splits = kvbm_skinny_gemm_splits(N, K);
  if (splits > 1 && (!ws || !tickets)) return cudaErrorInvalidValue;
  const int bn = M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : 128;
  CUtensorMap mw, mx;
  if (!make_map(&mw, w, static_cast<uint64_t>(N), static_cast<uint64_t>(K), static_cast<uint64_t>(ldw), kTileN))
    return cudaErrorInvalidValue;
  if (!make_map(&mx, x, static_cast<uint64_t>(M), static_cast<uint64_t>(K), static_cast<uint64_t>(ldx),
                static_cast<uint32_t>(bn)))
    return cudaErrorInvalidValue;
  const int tiles = (N + kTileN - 1) / kTileN;
  const int chunks = (K + kChunkK - 1) / kChunkK;
  GemmParams P;
  P.M = M;
  P.N = N;
  P.K = K;
  P.splits = std::min(splits, chunks);
  P.chunks_per_split = (chunks + P.splits - 1) / P.splits;
  P.splits = (chunks + P.chunks_per_split - 1) / P.chunks_per_split;  // no empty splits
  P.y = static_cast<__nv_bfloat16*>(y);
  P.ldy = ldy;
  P.ws = ws;
  P.tickets = tickets;
  switch (bn) {
    case 16: return launch<16>(mw, mx, P, tiles, stream);
    case 32: return launch<32>(mw, mx, P, tiles, stream);
    case 64: return launch<64>(mw, mx, P, tiles, stream);
    default: return launch<128>(mw, mx, P, tiles, stream);
  }
}

// 0, or the status a launch recorded (3 = a pipeline wait gave up); synchronizes.
extern "C" int kvbm_skinny_gemm_status(int reset) {
  int v = -1;
  if (cudaMemcpyFromSymbol(&v, g_gemm_status, sizeof(int)) != cudaSuccess) return -1;
  if (reset) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_gemm_status, &zero, sizeof(int));
  }
  return v;
}
