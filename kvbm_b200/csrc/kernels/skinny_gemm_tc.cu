// Skinny GEMM on the 5th-generation tensor cores (tcgen05 + TMEM + TMA):
//   Y[m, n] = sum_k X[m, k] * W[n, k]      (Y = X W^T, bf16 in, fp32 accumulate, bf16 out)
// for a handful of rows m (a decode batch, M <= 128) against a large weight W
// [N, K] - the projections of a decode step, which are bound by streaming W
// once from HBM.
//
// Roles are swapped so the big operand fills the 128-row MMA: a work unit is
// one K chunk (64 elements) of one 128-row weight tile, and the MMA computes
// D = W_tile X^T (UMMA M = 128, N = BN = the token count rounded up to 16)
// into a TMEM accumulator of 128 lanes x BN fp32 columns.
//
// Persistent stream-K schedule: one CTA per SM; the tiles x chunks units are
// cut into equal contiguous ranges, one per CTA, so every SM streams the same
// number of weight bytes whatever N and K are (no wave quantisation, no split
// count to tune). A CTA walks its range as segments (the part of one tile
// inside the range). A segment that covers a whole tile stores bf16 directly;
// partial segments add fp32 into a workspace with red.add, and the last
// contributor of the tile (ticket counter) converts it to bf16 and re-zeroes
// workspace and ticket for the next launch.
//
// Warp roles (192 threads):
// * warp 0, one lane: TMA producer - per unit, a tiled 2-D bulk tensor load of
//   the 128 x 64 weight tile and one of the BN x 64 activation tile (128-byte
//   swizzle) into a ring of shared-memory stages. Both operands are in this
//   GPU's own memory; every CTA loads its own tiles.
// * warp 1, one lane: MMA issuer - 4 tcgen05.mma (K = 16 each, descriptor
//   start advanced 32 bytes inside the 128-byte swizzle atom) per unit, then
//   tcgen05.commit to the stage's "empty" barrier; tcgen05.commit to the
//   accumulator's "full" barrier after a segment's last unit. Two TMEM
//   accumulators alternate between segments, so the next segment's MMAs run
//   while the epilogue drains the previous one.
// * warps 2-5: epilogue - tcgen05.ld (warp w reads TMEM lanes 32 (w % 4) ..
//   +31), stores or red.add, ticket, conversion.
// Every wait is bounded (%globaltimer) and also gives up when another role has
// given up; the CTA then records kStatusPipelineTimeout in g_gemm_status, lets
// its copies and MMAs drain (bounded), frees its TMEM and returns. Such a
// launch leaves the workspace and tickets dirty; the host zeroes them
// (ops/llama_ops.py skinny_gemm_status).
//
// The stream-K schedule (SegIter, the rounds / per-CTA split and the grid
// shrink in the host launcher, the ticket rule) is restated as a Python model
// in tests/test_gemm_cluster_protocol.py and model-checked there: change both
// together.
#include "common.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstring>
#include <mutex>

using namespace kvbm;

namespace {

constexpr int kThreads = 192;         // producer warp, MMA warp, 4 epilogue warps
constexpr int kEpiThreads = 128;
constexpr int kTileN = 128;           // weight rows per tile (UMMA M)
constexpr int kChunkK = 64;           // K elements per unit (128 bytes of bf16: one swizzle atom row)
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

// Bounded mbarrier wait that also gives up once another role of the CTA has.
KVBM_DEVICE bool wait_or_abort(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (globaltimer_ns() - t0 > kWaitNs) {
      *abort_flag = 1;
      atomicExch(&g_gemm_status, kStatusPipelineTimeout);
      return false;
    }
  }
}

// Programmatic dependent launch: wait until the preceding kernel in the stream
// has completed and its writes are visible (a no-op without the launch attribute).
KVBM_DEVICE void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
KVBM_DEVICE void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Named barrier of the 4 epilogue warps. bar.sync is warp-aligned: reconverge the
// warp first (code before it may have run on one lane only).
KVBM_DEVICE void epi_bar() {
  __syncwarp();
  asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory");
}

struct GemmParams {
  int M, N, K;
  int chunks;             // K chunks per tile
  int tiles;              // 128-row weight tiles
  int rounds;             // whole tiles per CTA before the stream-K part
  int per;                // stream-K units per CTA
  __nv_bfloat16* y;       // [M, N] row stride ldy
  int ldy;
  float* ws;              // [M, N] fp32 zeros
  unsigned int* tickets;  // [tiles] zeros
  unsigned long long* timeline;  // optional: 8 %globaltimer stamps per CTA (see kvbm_skinny_gemm_set_timeline)
};

KVBM_DEVICE void stamp(unsigned long long* tl, int slot) {
  if (tl) tl[blockIdx.x * 8 + slot] = globaltimer_ns();
}

// The segments of CTA b, in order. First `rounds` whole tiles (b, b + grid,
// ...), written straight to Y; then the CTA's equal share of the remaining
// tiles' units (stream-K), whose tiles several CTAs may share.
struct SegIter {
  int r, rounds, grid, b, u, u1, chunks, tile0;
  KVBM_DEVICE SegIter(const GemmParams& P, int b_, int grid_)
      : r(0), rounds(P.rounds), grid(grid_), b(b_), chunks(P.chunks), tile0(P.rounds * grid_) {
    const int total = (P.tiles - tile0) * P.chunks;
    u = min(b * P.per, total);
    u1 = min((b + 1) * P.per, total);
  }
  KVBM_DEVICE bool next(int& tile, int& c0, int& c1) {
    if (r < rounds) {
      tile = r * grid + b;
      c0 = 0;
      c1 = chunks;
      ++r;
      return true;
    }
    if (u >= u1) return false;
    const int t = u / chunks;
    c0 = u - t * chunks;
    const int end = min(u1, (t + 1) * chunks);
    c1 = end - t * chunks;
    u = end;
    tile = tile0 + t;
    return true;
  }
};

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
    skinny_gemm_tc_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_x,
                          const __grid_constant__ GemmParams P) {
  constexpr uint32_t kBytesW = kTileN * kChunkK * 2;  // 16 KiB
  constexpr uint32_t kStageBytes = Ring<BN>::kStageBytes;
  constexpr int kStages = Ring<BN>::kStages;
  constexpr uint32_t kTmemCols = 2 * BN < 32 ? 32 : 2 * BN;  // two accumulators
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte alignment for the swizzle atoms
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t full[kStages], empty[kStages], acc_full[2], acc_empty[2], mma_done, teardown;
  __shared__ uint32_t tmem_base;
  __shared__ volatile int abort_flag;
  __shared__ unsigned int ticket;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  unsigned long long* tl = P.timeline;

  if (threadIdx.x == 32) {
    prefetch_tmap(&map_w);
    prefetch_tmap(&map_x);
  }
  if (threadIdx.x == 0) {
    stamp(tl, 0);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 4);  // one arrival per epilogue warp
    }
    mbar_init(&mma_done, 1);
    mbar_init(&teardown, 5);  // the MMA thread and the 4 epilogue warps, once done with TMEM
    fence_mbar_init();
    abort_flag = 0;
  }
  if (warp == 0) {
    tmem_alloc(&tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_d = tmem_base;
  if (threadIdx.x == 0) stamp(tl, 1);

  if (warp == 0) {
    // ---- TMA producer ------------------------------------------------------
    if (lane == 0) {
      // The weight tiles of the first ring's worth of units do not depend on
      // the preceding kernel: start streaming them before waiting for it.
      int tile, c0, c1, it = 0;
      {
        SegIter segs(P, blockIdx.x, gridDim.x);
        while (it < kStages && segs.next(tile, c0, c1)) {
          for (int c = c0; c < c1 && it < kStages; ++c, ++it) {
            mbar_arrive_expect_tx(&full[it], kStageBytes);
            tma_load_2d(smem + it * kStageBytes, &map_w, c * kChunkK, tile * kTileN, &full[it]);
          }
        }
      }
      const int early = it;
      grid_dep_wait();  // the activations are the preceding kernel's output
      stamp(tl, 2);
      SegIter segs(P, blockIdx.x, gridDim.x);
      it = 0;
      bool ok = true;
      while (ok && segs.next(tile, c0, c1)) {
        for (int c = c0; c < c1; ++c, ++it) {
          const int s = it % kStages;
          uint8_t* st = smem + s * kStageBytes;
          if (it >= early) {
            if (it >= kStages && !wait_or_abort(&empty[s], ((it / kStages) - 1) & 1, &abort_flag)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&full[s], kStageBytes);
            tma_load_2d(st, &map_w, c * kChunkK, tile * kTileN, &full[s]);
          }
          tma_load_2d(st + kBytesW, &map_x, c * kChunkK, 0, &full[s]);
        }
      }
      // every copy issued into this CTA's shared memory lands before the CTA leaves
      for (int i = max(0, it - kStages); i < it; ++i)
        mbar_wait_bounded(&full[i % kStages], (i / kStages) & 1, kWaitNs);
    }
  } else if (warp == 1) {
    // ---- MMA issuer --------------------------------------------------------
    if (lane == 0) {
      SegIter segs(P, blockIdx.x, gridDim.x);
      int tile, c0, c1, it = 0, j = 0;
      bool ok = true;
      while (ok && segs.next(tile, c0, c1)) {
        const int a = j & 1;
        if (j >= 2 && !wait_or_abort(&acc_empty[a], ((j >> 1) - 1) & 1, &abort_flag)) break;
        tc_fence_after();
        const uint32_t acc = tmem_d + a * BN;
        for (int c = c0; c < c1; ++c, ++it) {
          const int s = it % kStages;
          if (!wait_or_abort(&full[s], (it / kStages) & 1, &abort_flag)) {
            ok = false;
            break;
          }
          if (it == 0) stamp(tl, 3);
          tc_fence_after();
          const uint8_t* st = smem + s * kStageBytes;
          const uint64_t da = smem_desc_k128(st), db = smem_desc_k128(st + kBytesW);
#pragma unroll
          for (int k = 0; k < kChunkK / 16; ++k)  // +32 bytes per K=16 step: +2 in 16-byte units
            umma_bf16(acc, da + 2 * k, db + 2 * k, idesc_bf16(BN), (c > c0 || k > 0) ? 1u : 0u);
          umma_commit(&empty[s]);
        }
        if (ok) umma_commit(&acc_full[a]);
        ++j;
      }
      stamp(tl, 4);
      // all MMAs complete before TMEM is freed
      umma_commit(&mma_done);
      mbar_wait_bounded(&mma_done, 0, kWaitNs);
      tc_fence_before();
      mbar_arrive(&teardown);
    }
  } else {
    // ---- epilogue: TMEM -> registers -> Y, or the workspace -----------------
    const int lane_grp = warp & 3;  // TMEM lanes this warp may read
    const int et = threadIdx.x - 64;
    grid_dep_wait();  // Y and the workspace may still be in use by the preceding kernel
    SegIter segs(P, blockIdx.x, gridDim.x);
    int tile, c0, c1, j = 0;
    // every epilogue warp runs the same sequence of named barriers, aborted or not
    while (segs.next(tile, c0, c1)) {
      const int a = j & 1;
      const bool ok = __all_sync(0xffffffffu, wait_or_abort(&acc_full[a], (j >> 1) & 1, &abort_flag));
      const bool whole = c0 == 0 && c1 == P.chunks;
      const int row = tile * kTileN + lane_grp * 32 + lane;  // weight row = output column of Y
      if (ok) {  // warp-uniform: tcgen05.ld is warp-collective
        tc_fence_after();
#pragma unroll
        for (int m0 = 0; m0 < BN; m0 += 16) {
          float v[16];
          tmem_ld16(tmem_d + (static_cast<uint32_t>(lane_grp * 32) << 16) + a * BN + m0, v);
          if (row < P.N) {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int m = m0 + i;
              if (m < P.M) {
                if (whole)
                  P.y[static_cast<int64_t>(m) * P.ldy + row] = __float2bfloat16(v[i]);
                else
                  atomicAdd(&P.ws[static_cast<int64_t>(m) * P.N + row], v[i]);
              }
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[a]);  // the MMA warp may reuse this accumulator
      }
      if (et == 0) stamp(tl, 5);  // last accumulator of this CTA drained (overwritten per segment)
      if (!whole) {
        // the tile's last contributor turns the fp32 sum into bf16 and re-arms the workspace
        const int t = tile - P.rounds * static_cast<int>(gridDim.x);  // a stream-K tile
        const int first = (t * P.chunks) / P.per;
        const int last = ((t + 1) * P.chunks - 1) / P.per;
        // The barrier orders every epilogue thread's red.add before thread 0's
        // gpu-scope fence (cumulative), which orders them before the ticket.
        epi_bar();
        if (et == 0) {
          __threadfence();
          ticket = abort_flag ? ~0u : atomicAdd(&P.tickets[tile], 1u);
        }
        epi_bar();
        if (ticket == static_cast<unsigned int>(last - first)) {
          __threadfence();
          const int r = tile * kTileN + et;  // thread et converts row r of this tile
          if (r < P.N) {
            for (int m0 = 0; m0 < P.M; m0 += 32) {
              float v[32];
#pragma unroll
              for (int i = 0; i < 32; ++i)  // all loads in flight before the first store
                v[i] = m0 + i < P.M ? __ldcg(&P.ws[static_cast<int64_t>(m0 + i) * P.N + r]) : 0.f;
#pragma unroll
              for (int i = 0; i < 32; ++i) {
                if (m0 + i < P.M) {
                  P.y[static_cast<int64_t>(m0 + i) * P.ldy + r] = __float2bfloat16(v[i]);
                  __stcg(&P.ws[static_cast<int64_t>(m0 + i) * P.N + r], 0.f);
                }
              }
            }
          }
          if (et == 0) P.tickets[tile] = 0u;
        }
      }
      ++j;
    }
    if (et == 0) stamp(tl, 6);
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&teardown);
  }
  // TMEM is freed once the MMA thread and every epilogue warp said they are done
  // with it (an explicit count, independent of how the role warps reconverge).
  __syncwarp();
  if (warp == 0) {
    mbar_wait_bounded(&teardown, 0, kWaitNs);
    tc_fence_after();
    if (lane == 0) stamp(tl, 7);
    tmem_dealloc(tmem_d, kTmemCols);
  }
}

// ---- cluster split-K variant ------------------------------------------------------
// For weights with fewer 128-row tiles than SMs: a cluster of S CTAs (S <= 8)
// shares each tile, CTA rank r streaming K chunks [r C / S, (r + 1) C / S).
// Each CTA leaves its fp32 partial tile in its own shared memory and the S
// partials are summed through distributed shared memory (ld.shared::cluster),
// each rank converting an equal slice of the tile to bf16: no workspace, no
// global atomics, no last-arrival round trip through L2. Clusters walk tiles
// c, c + clusters, ...
//
// Per-tile handshake, one mbarrier pair in every CTA, S arrivals per phase
// (one per rank, release/acquire at cluster scope):
//   red_ready - "my partial of this tile is in my shared memory"
//   red_done  - "I have finished reading your partial of this tile"
// A rank overwrites its partial (next tile) or exits only after its own
// red_done phase for the previous tile completed, so no peer reads shared
// memory that has been reused or released.

template <int BN>
struct ClusterRing {
  static constexpr uint32_t kPartialBytes = kTileN * BN * 4;
  static constexpr uint32_t kStageBytes = (kTileN + BN) * kChunkK * 2;
  static constexpr int kFit = static_cast<int>((200 * 1024 - kPartialBytes) / kStageBytes);
  static constexpr int kStages = kFit < 8 ? kFit : 8;
  static constexpr size_t kSmem = 1024 + static_cast<size_t>(kStages) * kStageBytes + kPartialBytes;
};

KVBM_DEVICE uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// address of this CTA's shared variable `p` in the shared memory of cluster rank `rank`
KVBM_DEVICE uint32_t map_to_rank(const void* p, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(smem_u32(p)), "r"(rank));
  return out;
}
KVBM_DEVICE void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
KVBM_DEVICE bool mbar_try_wait_acq_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// every thread of every CTA in the cluster; used once, right after barrier initialisation
KVBM_DEVICE void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
KVBM_DEVICE bool wait_cluster_or_abort(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  if (mbar_try_wait_acq_cluster(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (mbar_try_wait_acq_cluster(bar, parity)) return true;
    if (*abort_flag) return false;
    if (globaltimer_ns() - t0 > kWaitNs) {
      *abort_flag = 1;
      atomicExch(&g_gemm_status, kStatusPipelineTimeout);
      return false;
    }
  }
}

struct ClusterParams {
  int M, N, K;
  int chunks;  // K chunks per tile
  int tiles;   // 128-row weight tiles
  int S;       // cluster size = CTAs per tile
  __nv_bfloat16* y;
  int ldy;
};

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
    skinny_gemm_cluster_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_x,
                               const __grid_constant__ ClusterParams P) {
  constexpr uint32_t kBytesW = kTileN * kChunkK * 2;
  constexpr uint32_t kStageBytes = ClusterRing<BN>::kStageBytes;
  constexpr int kStages = ClusterRing<BN>::kStages;
  constexpr uint32_t kTmemCols = 2 * BN < 32 ? 32 : 2 * BN;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* partial = reinterpret_cast<float*>(smem + kStages * kStageBytes);  // [M][128] fp32
  __shared__ uint64_t full[kStages], empty[kStages], acc_full[2], acc_empty[2], mma_done, red_ready, red_done,
      teardown;
  __shared__ uint32_t tmem_base;
  __shared__ volatile int abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = P.S;
  const uint32_t rank = cluster_rank();
  const int c_lo = static_cast<int>(rank) * P.chunks / S, c_hi = (static_cast<int>(rank) + 1) * P.chunks / S;
  const int clusters = gridDim.y;

  if (threadIdx.x == 32) {
    prefetch_tmap(&map_w);
    prefetch_tmap(&map_x);
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 4);
    }
    mbar_init(&mma_done, 1);
    mbar_init(&red_ready, S);
    mbar_init(&red_done, S);
    mbar_init(&teardown, 5);
    fence_mbar_init();
    abort_flag = 0;
  }
  if (warp == 0) {
    tmem_alloc(&tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  cluster_sync_all();  // every rank's barriers exist before the first remote arrival
  const uint32_t tmem_d = tmem_base;

  if (warp == 0) {
    // ---- TMA producer (weight stages before the grid dependency, as above) --
    if (lane == 0) {
      int it = 0;
      for (int tile = blockIdx.y; tile < P.tiles && it < kStages; tile += clusters)
        for (int c = c_lo; c < c_hi && it < kStages; ++c, ++it) {
          mbar_arrive_expect_tx(&full[it], kStageBytes);
          tma_load_2d(smem + it * kStageBytes, &map_w, c * kChunkK, tile * kTileN, &full[it]);
        }
      const int early = it;
      grid_dep_wait();
      it = 0;
      bool ok = true;
      for (int tile = blockIdx.y; ok && tile < P.tiles; tile += clusters) {
        for (int c = c_lo; c < c_hi; ++c, ++it) {
          const int s = it % kStages;
          uint8_t* st = smem + s * kStageBytes;
          if (it >= early) {
            if (it >= kStages && !wait_or_abort(&empty[s], ((it / kStages) - 1) & 1, &abort_flag)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&full[s], kStageBytes);
            tma_load_2d(st, &map_w, c * kChunkK, tile * kTileN, &full[s]);
          }
          tma_load_2d(st + kBytesW, &map_x, c * kChunkK, 0, &full[s]);
        }
      }
      for (int i = max(0, it - kStages); i < it; ++i)
        mbar_wait_bounded(&full[i % kStages], (i / kStages) & 1, kWaitNs);
    }
  } else if (warp == 1) {
    // ---- MMA issuer ----------------------------------------------------------
    if (lane == 0) {
      int it = 0, j = 0;
      bool ok = true;
      for (int tile = blockIdx.y; ok && tile < P.tiles; tile += clusters, ++j) {
        const int a = j & 1;
        if (j >= 2 && !wait_or_abort(&acc_empty[a], ((j >> 1) - 1) & 1, &abort_flag)) break;
        tc_fence_after();
        const uint32_t acc = tmem_d + a * BN;
        for (int c = c_lo; c < c_hi; ++c, ++it) {
          const int s = it % kStages;
          if (!wait_or_abort(&full[s], (it / kStages) & 1, &abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint8_t* st = smem + s * kStageBytes;
          const uint64_t da = smem_desc_k128(st), db = smem_desc_k128(st + kBytesW);
#pragma unroll
          for (int k = 0; k < kChunkK / 16; ++k)
            umma_bf16(acc, da + 2 * k, db + 2 * k, idesc_bf16(BN), (c > c_lo || k > 0) ? 1u : 0u);
          umma_commit(&empty[s]);
        }
        if (ok) umma_commit(&acc_full[a]);
      }
      umma_commit(&mma_done);
      mbar_wait_bounded(&mma_done, 0, kWaitNs);
      tc_fence_before();
      mbar_arrive(&teardown);
    }
  } else {
    // ---- epilogue: TMEM -> own partial -> cluster sum of a slice -> Y ---------
    const int lane_grp = warp & 3;
    const int et = threadIdx.x - 64;
    const int rowl = lane_grp * 32 + lane;  // tile row this thread reads from TMEM
    grid_dep_wait();
    const int E = P.M * kTileN;  // partial elements that matter, e = m * 128 + row
    const int e0 = static_cast<int>(rank) * E / S, e1 = (static_cast<int>(rank) + 1) * E / S;
    int j = 0;
    for (int tile = blockIdx.y; tile < P.tiles; tile += clusters, ++j) {
      const int a = j & 1;
      const bool ok = __all_sync(0xffffffffu, wait_or_abort(&acc_full[a], (j >> 1) & 1, &abort_flag));
      // the partial buffer is free once every rank has read the previous tile's
      if (j > 0) wait_cluster_or_abort(&red_done, (j - 1) & 1, &abort_flag);
      if (ok) {
        tc_fence_after();
#pragma unroll
        for (int m0 = 0; m0 < BN; m0 += 16) {
          if (m0 < P.M) {  // uniform across the warp
            float v[16];
            tmem_ld16(tmem_d + (static_cast<uint32_t>(lane_grp * 32) << 16) + a * BN + m0, v);
#pragma unroll
            for (int i = 0; i < 16; ++i)
              if (m0 + i < P.M) partial[(m0 + i) * kTileN + rowl] = v[i];
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[a]);
      }
      // bar.sync orders all 128 writes before thread 0's cluster-scope release
      epi_bar();
      if (et == 0)
        for (int q = 0; q < S; ++q) mbar_arrive_cluster(map_to_rank(&red_ready, q));
      wait_cluster_or_abort(&red_ready, j & 1, &abort_flag);
      // this rank's slice of the tile: sum the S partials, convert, store
      const uint32_t base = smem_u32(partial);
      for (int e = e0 + et; e < e1; e += 4 * kEpiThreads) {
        // issue every load (4 elements x the other ranks) before the first add
        float v[4][8];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int ee = e + u * kEpiThreads;
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            v[u][q] = 0.f;
            if (q < S && ee < e1) {
              if (q == static_cast<int>(rank)) {
                v[u][q] = partial[ee];
              } else {
                uint32_t ra;
                asm("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(base + ee * 4u), "r"(q));
                asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v[u][q]) : "r"(ra));
              }
            }
          }
        }
        float acc4[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          acc4[u] = 0.f;
#pragma unroll
          for (int q = 0; q < 8; ++q) acc4[u] += v[u][q];
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int ee = e + u * kEpiThreads;
          const int r = tile * kTileN + (ee & (kTileN - 1));
          if (ee < e1 && r < P.N) P.y[static_cast<int64_t>(ee / kTileN) * P.ldy + r] = __float2bfloat16(acc4[u]);
        }
      }
      epi_bar();
      if (et == 0)
        for (int q = 0; q < S; ++q) mbar_arrive_cluster(map_to_rank(&red_done, q));
    }
    // leave only when no rank still reads this CTA's partial
    if (j > 0) wait_cluster_or_abort(&red_done, (j - 1) & 1, &abort_flag);
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&teardown);
  }
  __syncwarp();
  if (warp == 0) {  // as in the stream-K kernel
    mbar_wait_bounded(&teardown, 0, kWaitNs);
    tc_fence_after();
    tmem_dealloc(tmem_d, kTmemCols);
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

int g_pdl = 1;  // launch with programmatic stream serialization

template <int BN>
int launch(const CUtensorMap& mw, const CUtensorMap& mx, const GemmParams& P, int grid, cudaStream_t stream) {
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
  // With programmatic dependent launch the CTAs may start while the previous
  // kernel in the stream drains: they allocate TMEM and stream their first
  // weight tiles, then wait (griddepcontrol.wait) before reading activations.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = g_pdl;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, skinny_gemm_tc_kernel<BN>, mw, mx, P);
}

template <int BN>
int set_cluster_smem() {
  static int configured = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured != dev) {
    cudaError_t e = cudaFuncSetAttribute(skinny_gemm_cluster_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(ClusterRing<BN>::kSmem));
    if (e != cudaSuccess) return e;
    configured = dev;
  }
  return cudaSuccess;
}

// Clusters of S CTAs that can be resident at once (0 if none).
template <int BN>
int cluster_capacity(int S) {
  static int cap[9] = {-1, -1, -1, -1, -1, -1, -1, -1, -1};
  static int cap_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (cap_dev != dev) {
    for (int& c : cap) c = -1;
    cap_dev = dev;
  }
  if (cap[S] < 0) {
    cap[S] = 0;
    if (set_cluster_smem<BN>() == cudaSuccess) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(S);
      cfg.blockDim = dim3(kThreads);
      cfg.dynamicSmemBytes = ClusterRing<BN>::kSmem;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = S;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, skinny_gemm_cluster_kernel<BN>, &cfg) == cudaSuccess) cap[S] = n;
      else cudaGetLastError();
    }
  }
  return cap[S];
}

template <int BN>
int launch_cluster(const CUtensorMap& mw, const CUtensorMap& mx, const ClusterParams& P, int clusters,
                   cudaStream_t stream) {
  if (int e = set_cluster_smem<BN>()) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(P.S, clusters);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = ClusterRing<BN>::kSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = P.S;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = g_pdl;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, skinny_gemm_cluster_kernel<BN>, mw, mx, P);
}

int g_mode = 0;  // 0: pick by estimated time, 1: stream-K only, 2: cluster split-K only
unsigned long long* g_timeline = nullptr;  // stream-K launches stamp phases here when set

struct ClusterChoice {
  int S = 0, clusters = 0;
  long cost = -1;
};

// Estimated time, in K-chunk loads per CTA, of the best cluster split-K launch.
template <int BN>
ClusterChoice best_cluster(int tiles, int chunks) {
  ClusterChoice best;
  for (int S = 1; S <= 8 && S <= chunks; ++S) {
    const int cap = cluster_capacity<BN>(S);
    if (cap <= 0) continue;
    const int clusters = std::min(tiles, cap);
    const long rounds = (tiles + clusters - 1) / clusters;
    const long cost = rounds * ((chunks + S - 1) / S + (S > 1 ? 3 : 0));  // + the cluster reduction
    if (best.cost < 0 || cost < best.cost) {
      best.S = S;
      best.clusters = clusters;
      best.cost = cost;
    }
  }
  return best;
}

template <int BN>
int run(const CUtensorMap& mw, const CUtensorMap& mx, GemmParams& P, int ctas, cudaStream_t stream) {
  long grid = ctas > 0 ? ctas : sm_count_cached();
  P.rounds = static_cast<int>(P.tiles / grid);  // whole tiles every CTA takes first
  const long rest = (P.tiles - P.rounds * grid) * static_cast<long>(P.chunks);
  P.per = rest > 0 ? static_cast<int>((rest + grid - 1) / grid) : 1;
  if (P.rounds == 0) grid = (rest + P.per - 1) / P.per;  // no CTA without work
  if (g_mode == 2 || (g_mode == 0 && ctas <= 0)) {
    // stream-K: the largest share, plus the fix-up tail when some tile is split
    const bool split = rest > 0 && P.per % P.chunks != 0;
    const long sk_cost = static_cast<long>(P.rounds) * P.chunks + P.per + (split ? 10 + P.M / 8 : 0);
    const ClusterChoice c = best_cluster<BN>(P.tiles, P.chunks);
    if (c.cost >= 0 && (g_mode == 2 || c.cost < sk_cost)) {
      ClusterParams C;
      C.M = P.M;
      C.N = P.N;
      C.K = P.K;
      C.chunks = P.chunks;
      C.tiles = P.tiles;
      C.S = c.S;
      C.y = P.y;
      C.ldy = P.ldy;
      return launch_cluster<BN>(mw, mx, C, c.clusters, stream);
    }
    if (g_mode == 2) return cudaErrorLaunchOutOfResources;
  }
  return launch<BN>(mw, mx, P, static_cast<int>(grid), stream);
}

}  // namespace

// Device buffer of 8 x 64-bit words per CTA (one per SM is enough) that the
// stream-K kernel fills with %globaltimer stamps: entry, prologue done, grid
// dependency resolved, first stage landed, last MMA issued, last accumulator
// drained, fix-ups done, exit. nullptr turns it off (the default).
extern "C" int kvbm_skinny_gemm_set_timeline(void* buf) {
  g_timeline = static_cast<unsigned long long*>(buf);
  return 0;
}

// 0: choose stream-K or cluster split-K by estimated time (default); 1: stream-K
// only; 2: cluster split-K only. Returns the previous mode.
extern "C" int kvbm_skinny_gemm_set_mode(int mode) {
  const int prev = g_mode;
  g_mode = (mode >= 0 && mode <= 2) ? mode : 0;
  return prev;
}

// Programmatic dependent launch on (1, the default) or off (0); returns the previous setting.
extern "C" int kvbm_skinny_gemm_set_pdl(int on) {
  const int prev = g_pdl;
  g_pdl = on ? 1 : 0;
  return prev;
}

// Number of persistent CTAs a launch uses by default (one per SM).
extern "C" int kvbm_skinny_gemm_ctas() { return sm_count_cached(); }

// Y[M, N] (row stride ldy) = X[M, K] (row stride ldx) * W[N, K]^T (row stride ldw).
// bf16, M <= 128, K % 8 == 0, x and w 16-byte aligned, ldx and ldw multiples
// of 8. `ctas` > 0 forces a stream-K launch of that many persistent CTAs
// (unless the mode is cluster-only); otherwise the launcher picks stream-K
// over all SMs or cluster split-K. `ws` is an fp32 [M, N] buffer of zeros and
// `tickets` (N / 128 rounded up) 32-bit zeros; the kernel leaves both zeroed.
extern "C" int kvbm_skinny_gemm(const void* x, int ldx, const void* w, int ldw, void* y, int ldy, int M, int N, int K,
                                int ctas, float* ws, unsigned int* tickets, cudaStream_t stream) {
  if (M == 0 || N == 0) return cudaSuccess;
  if (!x || !w || !y || !ws || !tickets || M < 0 || M > 128 || N < 0 || K <= 0 || K % 8 != 0)
    return cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w)) & 15) return cudaErrorInvalidValue;
  if ((ldx % 8) || (ldw % 8) || ldx < K || ldw < K || ldy < N) return cudaErrorInvalidValue;
  const int bn = M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : 128;
  CUtensorMap mw, mx;
  if (!make_map(&mw, w, static_cast<uint64_t>(N), static_cast<uint64_t>(K), static_cast<uint64_t>(ldw), kTileN))
    return cudaErrorInvalidValue;
  if (!make_map(&mx, x, static_cast<uint64_t>(M), static_cast<uint64_t>(K), static_cast<uint64_t>(ldx),
                static_cast<uint32_t>(bn)))
    return cudaErrorInvalidValue;
  GemmParams P;
  P.M = M;
  P.N = N;
  P.K = K;
  P.tiles = (N + kTileN - 1) / kTileN;
  P.chunks = (K + kChunkK - 1) / kChunkK;
  if (static_cast<long>(P.tiles) * P.chunks > (1l << 30)) return cudaErrorInvalidValue;
  P.y = static_cast<__nv_bfloat16*>(y);
  P.ldy = ldy;
  P.ws = ws;
  P.tickets = tickets;
  P.timeline = g_timeline;
  switch (bn) {
    case 16: return run<16>(mw, mx, P, ctas, stream);
    case 32: return run<32>(mw, mx, P, ctas, stream);
    case 64: return run<64>(mw, mx, P, ctas, stream);
    default: return run<128>(mw, mx, P, ctas, stream);
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
