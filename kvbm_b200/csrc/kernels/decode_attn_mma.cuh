// Paged decode attention on tensor cores (warp-level mma.sync, bf16 in,
// fp32 accumulate), for head_dim 128 and up to 8 query heads per KV head.
//
// Per warp, KV is consumed in 16-token units (one paged block, or a 16-token
// slice of a larger block). A unit's K and V rows for this KV head (16 x 256
// bytes each) are staged into a 3-deep per-warp ring in shared memory with
// 16-byte cp.async copies; rows past seq_len are zero-filled by the copy
// (src-size 0), so masked tokens contribute exact zeros. Rows are stored
// with the 16-byte chunk index XOR-swizzled by (row & 7), which makes every
// ldmatrix below bank-conflict free.
//
//   S = Q K^T : A = Q (16 rows, GROUP used), B = K tile via ldmatrix (K rows
//               are the column-major B operand), 8 k-steps x 2 n-tiles;
//   online softmax in base 2 on the S fragments (row max/sum across the 4
//   lanes of a row group);
//   O += P V  : A = P re-packed from the S fragments (bf16), B = V tile via
//               ldmatrix.trans, 16 n-tiles of 8 head dims.
//
// Each warp owns every 4th unit of the split's block range and keeps its own
// (m, l, O); the CTA merges its 4 warps and writes one partial per split,
// merged across splits by attn_combine_kernel.
#pragma once

#include "common.cuh"

namespace kvbm {
namespace attn {

constexpr int kHD = 128;
constexpr int kWarps = 4;
constexpr int kStages = 3;
constexpr int kRowBytes = kHD * 2;              // 256 B per token row
constexpr int kTileBytes = 16 * kRowBytes;      // 4 KiB: 16 tokens
constexpr int kStageBytes = 2 * kTileBytes;     // K + V

__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  return static_cast<uint32_t>(row * kRowBytes + ((chunk ^ (row & 7)) << 4));
}

__device__ __forceinline__ void cp_async16(uint32_t smem, const void* gmem, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem), "l"(gmem), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// D += A(16x16 bf16, row) * B(16x8 bf16, col), fp32 accumulators.
__device__ __forceinline__ void mma_bf16(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

template <int GROUP>
__global__ void __launch_bounds__(kWarps * 32) paged_decode_mma_kernel(
    const __nv_bfloat16* __restrict__ q, const uint8_t* __restrict__ k_base, const uint8_t* __restrict__ v_base,
    int64_t block_stride, int64_t token_stride, int64_t head_stride, int page, const int32_t* __restrict__ block_table,
    int max_blocks, const int32_t* __restrict__ seq_lens, float qscale, int splits, float* __restrict__ part_acc,
    float* __restrict__ part_ml, unsigned int* __restrict__ counters, __nv_bfloat16* __restrict__ out) {
  static_assert(GROUP == 1 || GROUP == 2 || GROUP == 4 || GROUP == 8, "GROUP must be 1, 2, 4 or 8");
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ float red_m[kWarps][8];
  __shared__ float red_l[kWarps][8];
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int Hkv = gridDim.y;
  const int Hq = Hkv * GROUP;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gid = lane >> 2, tig = lane & 3;
  const uint32_t ring = static_cast<uint32_t>(__cvta_generic_to_shared(smem)) + warp * kStages * kStageBytes;

  // ---- Q fragments (rows = query heads of this KV head; scaled, bf16) ----
  uint32_t qa[8][4];
  {
    const bool row_ok = gid < GROUP;
    const __nv_bfloat16* qrow = q + (static_cast<int64_t>(b) * Hq + kvh * GROUP + (row_ok ? gid : 0)) * kHD;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      const int k0 = ks * 16 + tig * 2;
      float x0 = 0.f, x1 = 0.f, x2 = 0.f, x3 = 0.f;
      if (row_ok) {
        x0 = __bfloat162float(qrow[k0]) * qscale;
        x1 = __bfloat162float(qrow[k0 + 1]) * qscale;
        x2 = __bfloat162float(qrow[k0 + 8]) * qscale;
        x3 = __bfloat162float(qrow[k0 + 9]) * qscale;
      }
      qa[ks][0] = pack_bf16x2(x0, x1);
      qa[ks][1] = 0u;  // rows 8..15 unused
      qa[ks][2] = pack_bf16x2(x2, x3);
      qa[ks][3] = 0u;
    }
  }

  const int seq = seq_lens[b];
  const int nblk = (seq + page - 1) / page;
  const int per = (nblk + splits - 1) / splits;
  const int b0 = split * per;
  const int b1 = min(nblk, b0 + per);
  const int upb = page / 16;  // 16-token units per block
  const int mine = (b1 - b0 - warp > 0) ? (b1 - b0 - warp + kWarps - 1) / kWarps : 0;
  const int units = mine * upb;

  auto issue = [&](int u) {
    if (u < units) {
      const int blk = b0 + warp + (u / upb) * kWarps;
      const int sub = (u % upb) * 16;
      const int64_t phys = block_table[static_cast<int64_t>(b) * max_blocks + blk];
      const uint8_t* kb = k_base + phys * block_stride + static_cast<int64_t>(kvh) * head_stride;
      const uint8_t* vb = v_base + phys * block_stride + static_cast<int64_t>(kvh) * head_stride;
      const uint32_t st = ring + (u % kStages) * kStageBytes;
      const int tok0 = blk * page + sub;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int c = lane + 32 * i;  // 256 chunks of 16 B per tile
        const int row = c >> 4, chunk = c & 15;
        const int ok = (tok0 + row < seq) ? 16 : 0;
        const int64_t off = static_cast<int64_t>(sub + row) * token_stride + chunk * 16;
        cp_async16(st + swz(row, chunk), kb + off, ok);
        cp_async16(st + kTileBytes + swz(row, chunk), vb + off, ok);
      }
    }
    cp_async_commit();
  };

  float m_run = -INFINITY, l_run = 0.f;  // for row gid (valid when gid < GROUP)
  float o[16][4];
#pragma unroll
  for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;

#pragma unroll
  for (int s = 0; s < kStages - 1; ++s) issue(s);

  for (int u = 0; u < units; ++u) {
    cp_async_wait<kStages - 2>();
    __syncwarp();
    const uint32_t st = ring + (u % kStages) * kStageBytes;
    const int tok0 = (b0 + warp + (u / upb) * kWarps) * page + (u % upb) * 16;

    // ---- S = Q K^T : two n-tiles of 8 tokens ----
    float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
      for (int ks = 0; ks < 8; ks += 2) {
        const int mtx = lane >> 3;
        const int row = nt * 8 + (lane & 7);
        uint32_t r0, r1, r2, r3;
        ldsm_x4(st + swz(row, 2 * ks + mtx), r0, r1, r2, r3);
        mma_bf16(s[nt], qa[ks], r0, r1);
        mma_bf16(s[nt], qa[ks + 1], r2, r3);
      }
    }
    // ---- online softmax on rows gid (entries 0,1 of each n-tile) ----
    float v4[4] = {s[0][0], s[0][1], s[1][0], s[1][1]};
    const int tk[4] = {tig * 2, tig * 2 + 1, 8 + tig * 2, 9 + tig * 2};
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (tok0 + tk[i] >= seq) v4[i] = -INFINITY;
      mx = fmaxf(mx, v4[i]);
    }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float m_new = fmaxf(m_run, mx);
    float p[4];
    float alpha = 1.f;
    if (m_new == -INFINITY) {
      p[0] = p[1] = p[2] = p[3] = 0.f;
    } else {
      alpha = exp2f(m_run - m_new);
#pragma unroll
      for (int i = 0; i < 4; ++i) p[i] = exp2f(v4[i] - m_new);
      m_run = m_new;
    }
    float ps = p[0] + p[1] + p[2] + p[3];
    ps += __shfl_xor_sync(0xffffffffu, ps, 1);
    ps += __shfl_xor_sync(0xffffffffu, ps, 2);
    l_run = l_run * alpha + ps;
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      o[n][0] *= alpha;
      o[n][1] *= alpha;
    }
    // ---- O += P V ----
    uint32_t pa[4];
    pa[0] = pack_bf16x2(p[0], p[1]);
    pa[1] = 0u;
    pa[2] = pack_bf16x2(p[2], p[3]);
    pa[3] = 0u;
#pragma unroll
    for (int dn = 0; dn < 16; dn += 2) {
      const int mtx = lane >> 3;
      const int row = (mtx & 1) * 8 + (lane & 7);
      uint32_t r0, r1, r2, r3;
      ldsm_x4_t(st + kTileBytes + swz(row, dn + (mtx >> 1)), r0, r1, r2, r3);
      mma_bf16(o[dn], pa, r0, r1);
      mma_bf16(o[dn + 1], pa, r2, r3);
    }
    __syncwarp();
    issue(u + kStages - 1);
  }
  cp_async_wait<0>();

  // ---- merge the 4 warps (rows gid < GROUP hold data in o[n][0..1]) ----
  float* red_o = reinterpret_cast<float*>(smem);  // reuse the ring: [warps][GROUP][128]
  __syncthreads();
  if (gid < GROUP) {
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      red_o[(warp * GROUP + gid) * kHD + n * 8 + tig * 2] = o[n][0];
      red_o[(warp * GROUP + gid) * kHD + n * 8 + tig * 2 + 1] = o[n][1];
    }
    if (tig == 0) {
      red_m[warp][gid] = m_run;
      red_l[warp][gid] = l_run;
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < GROUP * kHD; i += blockDim.x) {
    const int g = i / kHD, d = i - g * kHD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, red_m[w][g]);
    float L = 0.f, A = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        const float f = exp2f(red_m[w][g] - M);
        L += red_l[w][g] * f;
        A += red_o[(w * GROUP + g) * kHD + d] * f;
      }
    }
    const int64_t row = (static_cast<int64_t>(b) * Hq + kvh * GROUP + g) * splits + split;
    part_acc[row * kHD + d] = A;
    if (d == 0) {
      part_ml[row * 2] = M;
      part_ml[row * 2 + 1] = L;
    }
  }
  if (counters == nullptr) return;  // a separate combine kernel merges the splits

  // ---- split combine in the last CTA of this (request, KV head) ----
  // Every CTA publishes its partials (fence, then a ticket); the CTA that draws
  // the last ticket merges all splits of its GROUP query heads and re-arms the
  // counter for the next launch.
  __shared__ unsigned int ticket;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) ticket = atomicAdd(&counters[static_cast<int64_t>(b) * Hkv + kvh], 1u);
  __syncthreads();
  if (ticket != static_cast<unsigned int>(splits - 1)) return;
  __threadfence();
  for (int i = threadIdx.x; i < GROUP * kHD; i += blockDim.x) {
    const int g = i / kHD, d = i - g * kHD;
    const int64_t bh = static_cast<int64_t>(b) * Hq + kvh * GROUP + g;
    float M = -INFINITY;
    for (int sp = 0; sp < splits; ++sp) M = fmaxf(M, __ldcg(&part_ml[(bh * splits + sp) * 2]));
    float L = 0.f, A = 0.f;
    if (M != -INFINITY) {
      for (int sp = 0; sp < splits; ++sp) {
        const float f = exp2f(__ldcg(&part_ml[(bh * splits + sp) * 2]) - M);
        L += __ldcg(&part_ml[(bh * splits + sp) * 2 + 1]) * f;
        A += __ldcg(&part_acc[(bh * splits + sp) * kHD + d]) * f;
      }
    }
    out[bh * kHD + d] = __float2bfloat16(L > 0.f ? A / L : 0.f);
  }
  if (threadIdx.x == 0) counters[static_cast<int64_t>(b) * Hkv + kvh] = 0u;
}

constexpr size_t kSmemBytes = static_cast<size_t>(kWarps) * kStages * kStageBytes;  // 96 KiB

}  // namespace attn
}  // namespace kvbm
