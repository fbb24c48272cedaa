// Fused Llama-architecture ops for the prefill/decode driver harness
// (sm_100a): RMSNorm with fused residual add, RoPE fused with the paged KV
// cache write, SiLU-and-multiply, and split-KV paged decode attention with
// grouped-query heads.
//
// The reference (crates/kvbm-kernels) ships no model kernels; vLLM computes
// attention there. These exist so the block manager can be exercised end to
// end on a PyTorch Llama model whose KV cache lives in the block manager's
// paged layout. The decode projections run on the tcgen05 skinny GEMM
// (skinny_gemm_tc.cu) or cuBLAS; prefill GEMMs on cuBLAS.
#include "common.cuh"
#include "decode_attn_mma.cuh"
#include "kvbm_kernels.h"

#include <algorithm>

using namespace kvbm;

namespace {

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }
__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  const int nw = blockDim.x >> 5;
  float t = (lane < nw) ? red[lane] : 0.f;
  t = warp_sum(t);
  __syncthreads();
  return t;
}

// ---------------------------------------------------------------------------
// RMSNorm (+ residual). If `residual` is given: residual <- x + residual
// (rounded to bf16, as the unfused model does) and out <- norm(residual) * w.
// One CTA per row; each thread owns 8-element (16-byte) vectors.
// ---------------------------------------------------------------------------
constexpr int kNormMaxVec = 4;  // up to 4 x 8 = 32 elements per thread

__global__ void __launch_bounds__(256) rmsnorm_kernel(const __nv_bfloat16* __restrict__ x,
                                                      __nv_bfloat16* __restrict__ residual,
                                                      const __nv_bfloat16* __restrict__ w,
                                                      __nv_bfloat16* __restrict__ out, int D, float eps) {
  // a GEMM launched after this kernel with programmatic dependent launch may
  // start streaming its weights now (it waits for this grid before reading `out`)
  asm volatile("griddepcontrol.launch_dependents;");
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const int nvec = D / 8;
  const int4* xr = reinterpret_cast<const int4*>(x + row * D);
  int4* rr = residual ? reinterpret_cast<int4*>(residual + row * D) : nullptr;
  float vals[kNormMaxVec][8];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < kNormMaxVec; ++k) {
    const int v = threadIdx.x + k * blockDim.x;
    if (v < nvec) {
      int4 a = xr[v];
      uint32_t wa[4] = {(uint32_t)a.x, (uint32_t)a.y, (uint32_t)a.z, (uint32_t)a.w};
      if (rr) {
        const int4 b = rr[v];
        const uint32_t wb[4] = {(uint32_t)b.x, (uint32_t)b.y, (uint32_t)b.z, (uint32_t)b.w};
#pragma unroll
        for (int j = 0; j < 4; ++j)
          wa[j] = pack_bf16(bf16_lo(wa[j]) + bf16_lo(wb[j]), bf16_hi(wa[j]) + bf16_hi(wb[j]));
        rr[v] = make_int4(wa[0], wa[1], wa[2], wa[3]);
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        vals[k][2 * j] = bf16_lo(wa[j]);
        vals[k][2 * j + 1] = bf16_hi(wa[j]);
        ss += vals[k][2 * j] * vals[k][2 * j] + vals[k][2 * j + 1] * vals[k][2 * j + 1];
      }
    }
  }
  ss = block_sum(ss, red);
  const float inv = rsqrtf(ss / D + eps);
  const int4* wr = reinterpret_cast<const int4*>(w);
  int4* orow = reinterpret_cast<int4*>(out + row * D);
#pragma unroll
  for (int k = 0; k < kNormMaxVec; ++k) {
    const int v = threadIdx.x + k * blockDim.x;
    if (v < nvec) {
      const int4 g = wr[v];
      const uint32_t wg[4] = {(uint32_t)g.x, (uint32_t)g.y, (uint32_t)g.z, (uint32_t)g.w};
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        // round the normalised value to bf16 before the weight multiply, as
        // the reference model does
        const float n0 = __bfloat162float(__float2bfloat16(vals[k][2 * j] * inv));
        const float n1 = __bfloat162float(__float2bfloat16(vals[k][2 * j + 1] * inv));
        o[j] = pack_bf16(n0 * bf16_lo(wg[j]), n1 * bf16_hi(wg[j]));
      }
      orow[v] = make_int4(o[0], o[1], o[2], o[3]);
    }
  }
}

// ---------------------------------------------------------------------------
// RoPE (rotate-half convention) applied in place to the q and k heads of a
// packed qkv row [Hq + 2*Hkv, hd], fused with the write of k (rotated) and v
// into the paged cache at slot_mapping[t] (slot = block * page + offset).
// One warp per (token, head); cos/sin come from a [max_pos, hd] fp32 table
// holding cos in [0, hd/2) and sin in [hd/2, hd).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) rope_kv_write_kernel(
    __nv_bfloat16* __restrict__ qkv, int T, int Hq, int Hkv, int hd, const int32_t* __restrict__ positions,
    const float* __restrict__ cos_sin, uint8_t* k_base, uint8_t* v_base, int64_t block_stride, int64_t token_stride,
    int64_t head_stride, int page, const int64_t* __restrict__ slots) {
  const int lane = threadIdx.x & 31;
  const int64_t w = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int H = Hq + 2 * Hkv;
  if (w >= static_cast<int64_t>(T) * H) return;
  const int64_t t = w / H;
  const int h = static_cast<int>(w - t * H);
  __nv_bfloat16* row = qkv + (t * H + h) * hd;
  const int64_t slot = slots ? slots[t] : -1;
  uint8_t* cache_row = nullptr;
  if (h >= Hq && slot >= 0) {
    const int64_t blk = slot / page, off = slot - blk * page;
    const int kvh = (h < Hq + Hkv) ? (h - Hq) : (h - Hq - Hkv);
    uint8_t* base = (h < Hq + Hkv) ? k_base : v_base;
    cache_row = base + blk * block_stride + off * token_stride + kvh * head_stride;
  }
  if (h < Hq + Hkv) {
    const int half = hd / 2;
    const float* cs = cos_sin + static_cast<int64_t>(positions[t]) * hd;
    for (int i = lane; i < half; i += 32) {
      const float x1 = __bfloat162float(row[i]);
      const float x2 = __bfloat162float(row[i + half]);
      const float c = cs[i], s = cs[half + i];
      const __nv_bfloat16 y1 = __float2bfloat16(x1 * c - x2 * s);
      const __nv_bfloat16 y2 = __float2bfloat16(x2 * c + x1 * s);
      row[i] = y1;
      row[i + half] = y2;
      if (cache_row) {
        reinterpret_cast<__nv_bfloat16*>(cache_row)[i] = y1;
        reinterpret_cast<__nv_bfloat16*>(cache_row)[i + half] = y2;
      }
    }
  } else if (cache_row) {
    const int nv = hd / 8;
    for (int i = lane; i < nv; i += 32)
      reinterpret_cast<int4*>(cache_row)[i] = reinterpret_cast<const int4*>(row)[i];
  }
}

// ---------------------------------------------------------------------------
// Fused RoPE + KV write + KV push (head_dim 128).
//
// One half-warp per head row: lane l of the half holds elements [8l, 8l+8)
// (one 16-byte load). Rotate-half RoPE pairs element i with i+64, i.e. lane
// l with lane l^8 of the same half, exchanged with one shuffle. Q and K rows
// are rotated in place (the attention that follows reads them from qkv);
// K and V rows are stored to the local paged cache (``slots``, optional)
// and to a second paged cache (``rslots``, optional) that may live in a
// peer GPU's memory: the prefill -> decode KV transfer happens inside the
// kernel that produces the KV, so the bytes cross NVLink while the rest of
// the grid is still rotating Q heads, and there is no separate copy kernel
// competing with the next GEMM for SMs. Work items are token-major, so the
// peer stores are spread evenly over the whole launch.
// Parity: the per-layer save path of the reference's connector
// (crates/kvbm-connector/src/connector/worker/mod.rs, save_kv_layer) fused
// with the write that produces the layer's KV.
// ---------------------------------------------------------------------------
struct RopeKvParams {
  __nv_bfloat16* qkv;
  int T, Hq, Hkv;
  const int32_t* positions;
  const float* cos_sin;
  uint8_t* k_base;
  uint8_t* v_base;
  int64_t block_stride, token_stride, head_stride;
  int page;
  const int64_t* slots;
  uint8_t* rk_base;
  uint8_t* rv_base;
  int64_t r_block_stride, r_token_stride, r_head_stride;
  int r_page;
  int r_head_offset;
  const int64_t* rslots;
  int group;          // head pairs per work item
  int q_per_kv;       // query pairs visited after each K/V pair (0: K/V pairs first)
  __nv_bfloat16* q_out;  // optional [T, Hq, 128]: rotated query rows go here instead of back into qkv
  int pair_base;      // head-pair subset in K,V-first order: [pair_base, pair_base + npairs)
  int npairs;         // 0: all pairs
  FastDiv pairs_div;  // divides by the number of groups per token
  FastDiv page_div;
  FastDiv r_page_div;
};

__device__ __forceinline__ uint8_t* cache_base(uint8_t* kb, int64_t slot, const FastDiv& pd, int64_t bs, int64_t ts) {
  const uint32_t blk = pd.div(static_cast<uint32_t>(slot));
  const uint32_t off = pd.mod(static_cast<uint32_t>(slot), blk);
  return kb + static_cast<int64_t>(blk) * bs + static_cast<int64_t>(off) * ts;
}

// Work item = (token, group of `P.group` head pairs). With GQA (Hq/2 query
// pairs a multiple of the Hkv K/V pairs) the visiting order interleaves one
// K/V pair with every (Hq/2)/Hkv query pairs, so the stores that may cross
// NVLink are spread evenly over the launch instead of arriving in bursts;
// otherwise K/V pairs come first (pair j covers heads (Hq + 2j + {0,1}) mod H).
// The warp loads the token's cos/sin once and keeps kRopeUnroll pairs of
// rows in flight per lane.
constexpr int kRopeUnroll = 4;  // head pairs in flight per lane (64 registers: 32 warps per SM)

template <int kUnroll>
__global__ void __launch_bounds__(256) rope_kv_fused_kernel(const __grid_constant__ RopeKvParams P) {
  const int lane = threadIdx.x & 31;
  const int hl = lane & 15;  // lane within the half-warp: elements [8*hl, 8*hl+8)
  const int half = lane >> 4;
  const int H = P.Hq + 2 * P.Hkv;
  const int pairs = P.npairs > 0 ? P.npairs : (H + 1) >> 1;
  const int groups = static_cast<int>(P.pairs_div.d);  // head-pair groups per token
  const uint32_t items = static_cast<uint32_t>(P.T) * static_cast<uint32_t>(groups);
  const uint32_t stride = gridDim.x * (blockDim.x >> 5);
  const float sign = hl < 8 ? -1.f : 1.f;
  for (uint32_t w = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); w < items; w += stride) {
    const uint32_t t = P.pairs_div.div(w);
    const int g = static_cast<int>(P.pairs_div.mod(w, t));
    const int j_begin = g * P.group, j_end = min(pairs, j_begin + P.group);
    // per-token state: rotation table row and cache row bases
    const float* cs = P.cos_sin + static_cast<int64_t>(P.positions[t]) * 128 + (hl & 7) * 8;
    const float4 c0 = reinterpret_cast<const float4*>(cs)[0], c1 = reinterpret_cast<const float4*>(cs)[1];
    const float4 s0 = reinterpret_cast<const float4*>(cs + 64)[0];
    const float4 s1 = reinterpret_cast<const float4*>(cs + 64)[1];
    const float c[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
    const float sn[8] = {sign * s0.x, sign * s0.y, sign * s0.z, sign * s0.w,
                         sign * s1.x, sign * s1.y, sign * s1.z, sign * s1.w};
    uint8_t* lrow = nullptr;
    uint8_t* rrow = nullptr;
    if (P.slots) {
      const int64_t slot = P.slots[t];
      if (slot >= 0) lrow = cache_base(P.k_base, slot, P.page_div, P.block_stride, P.token_stride);
    }
    if (P.rslots) {
      const int64_t slot = P.rslots[t];
      if (slot >= 0) rrow = cache_base(P.rk_base, slot, P.r_page_div, P.r_block_stride, P.r_token_stride);
    }
    __nv_bfloat16* trow = P.qkv + static_cast<int64_t>(t) * H * 128 + hl * 8;
    for (int j0 = j_begin; j0 < j_end; j0 += kUnroll) {
      int4 x[kUnroll];
      int hh[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int j = j0 + u;
        int h;
        if (P.q_per_kv > 0) {  // interleaved: [KV, Q x q_per_kv] repeated
          const int b = j / (P.q_per_kv + 1), r = j - b * (P.q_per_kv + 1);
          h = (r == 0 ? P.Hq + 2 * b : 2 * (b * P.q_per_kv + r - 1)) + half;
        } else {
          h = 2 * (P.pair_base + j) + half + P.Hq;
          if (h >= H) h -= H;
        }
        const bool valid = j < j_end && h < H && (P.q_per_kv > 0 || 2 * (P.pair_base + j) + half < H);
        hh[u] = valid ? h : -1;
        x[u] = valid ? *reinterpret_cast<const int4*>(trow + static_cast<int64_t>(h) * 128) : make_int4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        int4 p;  // rotation partner: lane ^ 8 of the same half-warp
        p.x = __shfl_xor_sync(0xffffffffu, x[u].x, 8);
        p.y = __shfl_xor_sync(0xffffffffu, x[u].y, 8);
        p.z = __shfl_xor_sync(0xffffffffu, x[u].z, 8);
        p.w = __shfl_xor_sync(0xffffffffu, x[u].w, 8);
        const int h = hh[u];
        if (h < 0) continue;
        __nv_bfloat16* row = trow + static_cast<int64_t>(h) * 128;
        if (h < P.Hq + P.Hkv) {
          const uint32_t xm[4] = {(uint32_t)x[u].x, (uint32_t)x[u].y, (uint32_t)x[u].z, (uint32_t)x[u].w};
          const uint32_t xp[4] = {(uint32_t)p.x, (uint32_t)p.y, (uint32_t)p.z, (uint32_t)p.w};
          uint32_t y[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            // first half: x*c - partner*s ; second half: x*c + partner*s (sign folded into sn)
            y[k] = pack_bf16(bf16_lo(xm[k]) * c[2 * k] + bf16_lo(xp[k]) * sn[2 * k],
                             bf16_hi(xm[k]) * c[2 * k + 1] + bf16_hi(xp[k]) * sn[2 * k + 1]);
          }
          x[u] = make_int4((int)y[0], (int)y[1], (int)y[2], (int)y[3]);
          if (P.q_out != nullptr && h < P.Hq)
            reinterpret_cast<int4*>(P.q_out + (static_cast<int64_t>(t) * P.Hq + h) * 128)[hl] = x[u];
          else
            *reinterpret_cast<int4*>(row) = x[u];
        }
        if (h >= P.Hq) {
          const bool is_k = h < P.Hq + P.Hkv;
          const int kvh = is_k ? h - P.Hq : h - P.Hq - P.Hkv;
          if (lrow)
            reinterpret_cast<int4*>(lrow + (is_k ? 0 : P.v_base - P.k_base) +
                                    static_cast<int64_t>(kvh) * P.head_stride)[hl] = x[u];
          if (rrow)
            reinterpret_cast<int4*>(rrow + (is_k ? 0 : P.rv_base - P.rk_base) +
                                    static_cast<int64_t>(kvh + P.r_head_offset) * P.r_head_stride)[hl] = x[u];
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// out[t, i] = silu(gate_up[t, i]) * gate_up[t, I + i]
// ---------------------------------------------------------------------------
constexpr int kSiluUnroll = 4;

__device__ __forceinline__ int4 silu_mul_vec(const int4 g, const int4 u) {
  const uint32_t wg[4] = {(uint32_t)g.x, (uint32_t)g.y, (uint32_t)g.z, (uint32_t)g.w};
  const uint32_t wu[4] = {(uint32_t)u.x, (uint32_t)u.y, (uint32_t)u.z, (uint32_t)u.w};
  uint32_t o[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float a = bf16_lo(wg[j]), b = bf16_hi(wg[j]);
    const float sa = __bfloat162float(__float2bfloat16(a / (1.f + __expf(-a))));
    const float sb = __bfloat162float(__float2bfloat16(b / (1.f + __expf(-b))));
    o[j] = pack_bf16(sa * bf16_lo(wu[j]), sb * bf16_hi(wu[j]));
  }
  return make_int4(o[0], o[1], o[2], o[3]);
}

// Each thread keeps kSiluUnroll gate/up vector pairs in flight: all loads of
// a batch are issued before any math, so a thread has 8 x 16 B outstanding.
__global__ void __launch_bounds__(256) silu_mul_kernel(const __nv_bfloat16* __restrict__ gu,
                                                       __nv_bfloat16* __restrict__ out, int64_t T, int I) {
  asm volatile("griddepcontrol.launch_dependents;");  // as in rmsnorm_kernel
  const int nv = I / 8;
  const int64_t total = T * nv;
  const int64_t step = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t base = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; base < total;
       base += step * kSiluUnroll) {
    int4 g[kSiluUnroll], u[kSiluUnroll];
    int64_t t[kSiluUnroll];
    int c[kSiluUnroll];
#pragma unroll
    for (int k = 0; k < kSiluUnroll; ++k) {
      const int64_t v = base + k * step;
      t[k] = v / nv;
      c[k] = static_cast<int>(v - t[k] * nv);
      if (v < total) {
        g[k] = reinterpret_cast<const int4*>(gu + t[k] * 2 * I)[c[k]];
        u[k] = reinterpret_cast<const int4*>(gu + t[k] * 2 * I + I)[c[k]];
      }
    }
#pragma unroll
    for (int k = 0; k < kSiluUnroll; ++k) {
      if (base + k * step < total) reinterpret_cast<int4*>(out + t[k] * I)[c[k]] = silu_mul_vec(g[k], u[k]);
    }
  }
}

// ---------------------------------------------------------------------------
// Paged decode attention, split over the KV sequence (flash-decoding).
//
// grid = (splits, Hkv, B), 4 warps per CTA. A CTA owns the GROUP query heads
// that share one KV head, so each K/V row is loaded once for GROUP heads.
// Within a 16-token sub-block, lane (t = lane % 16, half = lane / 16) loads
// half of token t's key (64 dims, 8 x 16 B) for the score, and for P.V lane
// (c = lane % 16, parity = lane / 16) loads dims [8c, 8c+8) of the value rows
// of its token parity. Online softmax in base 2 (q pre-scaled by
// softmax_scale * log2 e). Each split writes unnormalised partials
// (acc[hd], m, l) into the caller's scratch; attn_combine merges them.
// ---------------------------------------------------------------------------
constexpr int kHD = 128;
constexpr int kAttnWarps = 4;

template <int GROUP>
__global__ void __launch_bounds__(kAttnWarps * 32) paged_decode_kernel(
    const __nv_bfloat16* __restrict__ q, const uint8_t* __restrict__ k_base, const uint8_t* __restrict__ v_base,
    int64_t block_stride, int64_t token_stride, int64_t head_stride, int page, const int32_t* __restrict__ block_table,
    int max_blocks, const int32_t* __restrict__ seq_lens, float qscale, int splits, float* __restrict__ part_acc,
    float* __restrict__ part_ml) {
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int Hkv = gridDim.y;
  const int Hq = Hkv * GROUP;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __shared__ float q_s[GROUP][kHD + 4];
  __shared__ float red_m[kAttnWarps][GROUP];
  __shared__ float red_l[kAttnWarps][GROUP];
  __shared__ float red_acc[kAttnWarps][GROUP][kHD];

  for (int i = threadIdx.x; i < GROUP * kHD; i += blockDim.x) {
    const int g = i / kHD, d = i - g * kHD;
    q_s[g][d] = __bfloat162float(q[(static_cast<int64_t>(b) * Hq + kvh * GROUP + g) * kHD + d]) * qscale;
  }
  __syncthreads();

  const int seq = seq_lens[b];
  const int nblk = (seq + page - 1) / page;
  const int per = (nblk + splits - 1) / splits;
  const int b0 = split * per;
  const int b1 = min(nblk, b0 + per);

  float m[GROUP], l[GROUP], acc[GROUP][8];
#pragma unroll
  for (int g = 0; g < GROUP; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[g][e] = 0.f;
  }
  const int tl = lane & 15, half = lane >> 4;
  // All K and V loads of a 16-token sub-block are issued before any use, so
  // each warp keeps 8 KiB in flight per sub-block (one memory round trip).
  // Rows past seq_len are still inside the allocated block: they are loaded
  // and then masked (score -inf, value zeroed).
  for (int blk = b0 + warp; blk < b1; blk += kAttnWarps) {
    const int64_t phys = block_table[static_cast<int64_t>(b) * max_blocks + blk];
    const uint8_t* kb = k_base + phys * block_stride + static_cast<int64_t>(kvh) * head_stride;
    const uint8_t* vb = v_base + phys * block_stride + static_cast<int64_t>(kvh) * head_stride;
    for (int sub = 0; sub < page; sub += 16) {
      const int tok0 = blk * page + sub;
      int4 kv[8], vv[8];
      const uint8_t* kr = kb + static_cast<int64_t>(sub + tl) * token_stride + half * 128;
#pragma unroll
      for (int j = 0; j < 8; ++j) kv[j] = ld_v4_stream(kr + j * 16);
#pragma unroll
      for (int j = 0; j < 8; ++j)
        vv[j] = ld_v4_stream(vb + static_cast<int64_t>(sub + 2 * j + half) * token_stride + tl * 16);
      const bool valid = tok0 + tl < seq;
      float s[GROUP];
#pragma unroll
      for (int g = 0; g < GROUP; ++g) s[g] = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint32_t w4[4] = {(uint32_t)kv[j].x, (uint32_t)kv[j].y, (uint32_t)kv[j].z, (uint32_t)kv[j].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float k0 = bf16_lo(w4[e]), k1 = bf16_hi(w4[e]);
          const int d = half * 64 + j * 8 + e * 2;
#pragma unroll
          for (int g = 0; g < GROUP; ++g) s[g] += q_s[g][d] * k0 + q_s[g][d + 1] * k1;
        }
      }
      float p[GROUP];
#pragma unroll
      for (int g = 0; g < GROUP; ++g) {
        s[g] += __shfl_xor_sync(0xffffffffu, s[g], 16);
        if (!valid) s[g] = -INFINITY;
        float mx = s[g];
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        const float m_new = fmaxf(m[g], mx);
        if (m_new == -INFINITY) {
          p[g] = 0.f;
          continue;
        }
        const float alpha = exp2f(m[g] - m_new);
        p[g] = valid ? exp2f(s[g] - m_new) : 0.f;
        float ps = p[g];
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
        l[g] = l[g] * alpha + ps;
        m[g] = m_new;
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[g][e] *= alpha;
      }
      // P.V: lane (c = tl, parity = half) holds value rows 2j + parity.
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int tt = 2 * j + half;
        float pt[GROUP];
#pragma unroll
        for (int g = 0; g < GROUP; ++g) pt[g] = __shfl_sync(0xffffffffu, p[g], tt);
        const bool vvalid = tok0 + tt < seq;
        const uint32_t w4[4] = {vvalid ? (uint32_t)vv[j].x : 0u, vvalid ? (uint32_t)vv[j].y : 0u,
                                vvalid ? (uint32_t)vv[j].z : 0u, vvalid ? (uint32_t)vv[j].w : 0u};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float v0 = bf16_lo(w4[e]), v1 = bf16_hi(w4[e]);
#pragma unroll
          for (int g = 0; g < GROUP; ++g) {
            acc[g][2 * e] += pt[g] * v0;
            acc[g][2 * e + 1] += pt[g] * v1;
          }
        }
      }
    }
  }
  // Merge the two token parities, then the warps.
#pragma unroll
  for (int g = 0; g < GROUP; ++g)
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[g][e] += __shfl_xor_sync(0xffffffffu, acc[g][e], 16);
  if (half == 0) {
#pragma unroll
    for (int g = 0; g < GROUP; ++g)
#pragma unroll
      for (int e = 0; e < 8; ++e) red_acc[warp][g][tl * 8 + e] = acc[g][e];
  }
  if (lane == 0) {
#pragma unroll
    for (int g = 0; g < GROUP; ++g) {
      red_m[warp][g] = m[g];
      red_l[warp][g] = l[g];
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < GROUP * kHD; i += blockDim.x) {
    const int g = i / kHD, d = i - g * kHD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, red_m[w][g]);
    float L = 0.f, A = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kAttnWarps; ++w) {
        const float f = exp2f(red_m[w][g] - M);
        L += red_l[w][g] * f;
        A += red_acc[w][g][d] * f;
      }
    }
    const int64_t row = (static_cast<int64_t>(b) * Hq + kvh * GROUP + g) * splits + split;
    part_acc[row * kHD + d] = A;
    if (d == 0) {
      part_ml[row * 2] = M;
      part_ml[row * 2 + 1] = L;
    }
  }
}

// out[b, h, :] = sum_s acc_s * 2^(m_s - M) / sum_s l_s * 2^(m_s - M)
__global__ void __launch_bounds__(kHD) attn_combine_kernel(const float* __restrict__ part_acc,
                                                           const float* __restrict__ part_ml, int splits,
                                                           __nv_bfloat16* __restrict__ out) {
  const int64_t bh = blockIdx.x;
  const int d = threadIdx.x;
  float M = -INFINITY;
  for (int s = 0; s < splits; ++s) M = fmaxf(M, part_ml[(bh * splits + s) * 2]);
  float L = 0.f, A = 0.f;
  if (M != -INFINITY) {
    for (int s = 0; s < splits; ++s) {
      const float f = exp2f(part_ml[(bh * splits + s) * 2] - M);
      L += part_ml[(bh * splits + s) * 2 + 1] * f;
      A += part_acc[(bh * splits + s) * kHD + d] * f;
    }
  }
  out[bh * kHD + d] = __float2bfloat16(L > 0.f ? A / L : 0.f);
}

// The decode GEMM that follows rmsnorm / silu_mul (programmatic dependent
// launch) needs most of the SM's unified L1 / shared memory; with the same
// carve-out its CTAs can become resident beside these small kernels' CTAs
// instead of waiting for the SM to drain and be reconfigured.
template <typename K>
void prefer_max_shared(K kernel) {
  static bool done = false;
  if (!done) {
    cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    done = true;
  }
}

}  // namespace

extern "C" int kvbm_rmsnorm(const void* x, void* residual, const void* weight, void* out, int64_t rows, int dim,
                            float eps, cudaStream_t stream) {
  if (rows == 0) return cudaSuccess;
  if (!x || !weight || !out || dim % 8 != 0 || dim / 8 > 256 * kNormMaxVec) return cudaErrorInvalidValue;
  const int threads = std::min(256, std::max(32, (dim / 8 + 31) / 32 * 32));
  prefer_max_shared(rmsnorm_kernel);
  rmsnorm_kernel<<<static_cast<unsigned>(rows), threads, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(x), static_cast<__nv_bfloat16*>(residual),
      static_cast<const __nv_bfloat16*>(weight), static_cast<__nv_bfloat16*>(out), dim, eps);
  return cudaGetLastError();
}

namespace {
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

int g_rope_unroll = kRopeUnroll;  // head pairs in flight per lane: 2, 4 (default) or 8

int launch_rope_fused(RopeKvParams& P, cudaStream_t stream) {
  const int H = P.Hq + 2 * P.Hkv;
  const int pairs = P.npairs > 0 ? P.npairs : (H + 1) / 2;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  // whole tokens per warp when there are enough tokens to fill the GPU,
  // otherwise split each token's heads over several warps (decode)
  const int unroll = g_rope_unroll;
  const int groups_max = (pairs + unroll - 1) / unroll;
  int groups = 1;
  while (groups < groups_max && static_cast<int64_t>(P.T) * groups < int64_t{sms} * 64) groups *= 2;
  groups = std::min(groups, groups_max);
  P.q_per_kv = (P.npairs == 0 && P.Hq % 2 == 0 && P.Hkv > 0 && (P.Hq / 2) % P.Hkv == 0) ? (P.Hq / 2) / P.Hkv : 0;
  P.group = (pairs + groups - 1) / groups;
  groups = (pairs + P.group - 1) / P.group;
  const int64_t items = static_cast<int64_t>(P.T) * groups;
  if (items >= (int64_t{1} << 31)) return cudaErrorInvalidValue;
  P.pairs_div = FastDiv(static_cast<uint32_t>(groups));
  P.page_div = FastDiv(static_cast<uint32_t>(P.page > 0 ? P.page : 1));
  P.r_page_div = FastDiv(static_cast<uint32_t>(P.r_page > 0 ? P.r_page : 1));
  const int64_t ctas = (items + 7) / 8;
  // one item per warp (a grid capped at one resident wave measured 6% slower on prefill batches)
  const unsigned grid = static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>(ctas, int64_t{sms} * 32)));
  switch (g_rope_unroll) {
    case 2: rope_kv_fused_kernel<2><<<grid, 256, 0, stream>>>(P); break;
    case 8: rope_kv_fused_kernel<8><<<grid, 256, 0, stream>>>(P); break;
    default: rope_kv_fused_kernel<kRopeUnroll><<<grid, 256, 0, stream>>>(P); break;
  }
  return cudaGetLastError();
}

bool cache_ok(const void* kb, const void* vb, int64_t bs, int64_t ts, int64_t hs, int page) {
  return kb && vb && page > 0 && aligned16(kb) && aligned16(vb) && bs % 16 == 0 && ts % 16 == 0 && hs % 16 == 0;
}
}  // namespace

extern "C" int kvbm_rope_kv_write(void* qkv, int64_t tokens, int hq, int hkv, int hd, const int32_t* positions,
                                  const float* cos_sin, void* k_base, void* v_base, int64_t block_stride,
                                  int64_t token_stride, int64_t head_stride, int page, const int64_t* slots,
                                  cudaStream_t stream) {
  if (tokens == 0) return cudaSuccess;
  if (!qkv || !positions || !cos_sin || hd % 8 != 0) return cudaErrorInvalidValue;
  if (slots && (!k_base || !v_base || page <= 0)) return cudaErrorInvalidValue;
  if (hd == 128 && aligned16(qkv) && aligned16(cos_sin) &&
      (!slots || cache_ok(k_base, v_base, block_stride, token_stride, head_stride, page))) {
    RopeKvParams P{};
    P.qkv = static_cast<__nv_bfloat16*>(qkv);
    P.T = static_cast<int>(tokens);
    P.Hq = hq;
    P.Hkv = hkv;
    P.positions = positions;
    P.cos_sin = cos_sin;
    P.k_base = static_cast<uint8_t*>(k_base);
    P.v_base = static_cast<uint8_t*>(v_base);
    P.block_stride = block_stride;
    P.token_stride = token_stride;
    P.head_stride = head_stride;
    P.page = page;
    P.slots = slots;
    return launch_rope_fused(P, stream);
  }
  const int64_t warps = tokens * (hq + 2 * hkv);
  const unsigned grid = static_cast<unsigned>((warps + 7) / 8);
  rope_kv_write_kernel<<<grid, 256, 0, stream>>>(static_cast<__nv_bfloat16*>(qkv), static_cast<int>(tokens), hq, hkv,
                                                 hd, positions, cos_sin, static_cast<uint8_t*>(k_base),
                                                 static_cast<uint8_t*>(v_base), block_stride, token_stride,
                                                 head_stride, page, slots);
  return cudaGetLastError();
}

// Head pairs each lane keeps in flight in the RoPE/KV kernel (2, 4 or 8; more
// loads in flight cost registers and so resident warps). Returns the previous
// value, or -1 for an unsupported one. For tuning; the default is 4.
extern "C" int kvbm_rope_set_unroll(int unroll) {
  if (unroll != 2 && unroll != 4 && unroll != 8) return -1;
  const int prev = g_rope_unroll;
  g_rope_unroll = unroll;
  return prev;
}

// Decode form: RoPE + paged KV write, with the rotated query rows written to
// a separate contiguous q_out [tokens, hq, 128] (the attention's input), so
// no copy of the strided q slice follows; head_dim 128.
extern "C" int kvbm_rope_kv_write_qout(void* qkv, int64_t tokens, int hq, int hkv, const int32_t* positions,
                                       const float* cos_sin, void* k_base, void* v_base, int64_t block_stride,
                                       int64_t token_stride, int64_t head_stride, int page, const int64_t* slots,
                                       void* q_out, cudaStream_t stream) {
  if (tokens == 0) return cudaSuccess;
  if (!qkv || !positions || !cos_sin || !q_out || !aligned16(qkv) || !aligned16(cos_sin) || !aligned16(q_out))
    return cudaErrorInvalidValue;
  if (slots && !cache_ok(k_base, v_base, block_stride, token_stride, head_stride, page)) return cudaErrorInvalidValue;
  RopeKvParams P{};
  P.qkv = static_cast<__nv_bfloat16*>(qkv);
  P.T = static_cast<int>(tokens);
  P.Hq = hq;
  P.Hkv = hkv;
  P.positions = positions;
  P.cos_sin = cos_sin;
  P.k_base = static_cast<uint8_t*>(k_base);
  P.v_base = static_cast<uint8_t*>(v_base);
  P.block_stride = block_stride;
  P.token_stride = token_stride;
  P.head_stride = head_stride;
  P.page = page;
  P.slots = slots;
  P.q_out = static_cast<__nv_bfloat16*>(q_out);
  return launch_rope_fused(P, stream);
}

// Head subsets for kvbm_rope_kv_push_heads: 0 = every head, 1 = the K and
// V heads only (requires an even Hq), 2 = the query heads only.
namespace {
int set_subset(RopeKvParams& P, int subset) {
  if (subset == 0) return cudaSuccess;
  if (P.Hq % 2 != 0) return cudaErrorInvalidValue;
  if (subset == 1) {
    P.pair_base = 0;
    P.npairs = P.Hkv;
  } else if (subset == 2) {
    P.pair_base = P.Hkv;
    P.npairs = P.Hq / 2;
  } else {
    return cudaErrorInvalidValue;
  }
  return P.npairs > 0 ? cudaSuccess : cudaErrorInvalidValue;
}
}  // namespace

// RoPE + KV write into the local cache (optional) and a second cache that
// may be a peer GPU's (mapped through CUDA IPC or peer access); head_dim 128.
extern "C" int kvbm_rope_kv_push_heads(void* qkv, int64_t tokens, int hq, int hkv, const int32_t* positions,
                                       const float* cos_sin, void* k_base, void* v_base, int64_t block_stride,
                                       int64_t token_stride, int64_t head_stride, int page, const int64_t* slots,
                                       void* rk_base, void* rv_base, int64_t r_block_stride, int64_t r_token_stride,
                                       int64_t r_head_stride, int r_page, int r_head_offset, const int64_t* rslots,
                                       int subset, cudaStream_t stream) {
  if (tokens == 0) return cudaSuccess;
  if (!qkv || !positions || !cos_sin || !aligned16(qkv) || !aligned16(cos_sin)) return cudaErrorInvalidValue;
  if (slots && !cache_ok(k_base, v_base, block_stride, token_stride, head_stride, page)) return cudaErrorInvalidValue;
  if (rslots && !cache_ok(rk_base, rv_base, r_block_stride, r_token_stride, r_head_stride, r_page))
    return cudaErrorInvalidValue;
  if (r_head_offset < 0) return cudaErrorInvalidValue;
  RopeKvParams P{};
  P.qkv = static_cast<__nv_bfloat16*>(qkv);
  P.T = static_cast<int>(tokens);
  P.Hq = hq;
  P.Hkv = hkv;
  P.positions = positions;
  P.cos_sin = cos_sin;
  P.k_base = static_cast<uint8_t*>(k_base);
  P.v_base = static_cast<uint8_t*>(v_base);
  P.block_stride = block_stride;
  P.token_stride = token_stride;
  P.head_stride = head_stride;
  P.page = page;
  P.slots = slots;
  P.rk_base = static_cast<uint8_t*>(rk_base);
  P.rv_base = static_cast<uint8_t*>(rv_base);
  P.r_block_stride = r_block_stride;
  P.r_token_stride = r_token_stride;
  P.r_head_stride = r_head_stride;
  P.r_page = r_page;
  P.r_head_offset = r_head_offset;
  P.rslots = rslots;
  const int e = set_subset(P, subset);
  if (e != cudaSuccess) return e;
  return launch_rope_fused(P, stream);
}

extern "C" int kvbm_rope_kv_push(void* qkv, int64_t tokens, int hq, int hkv, const int32_t* positions,
                                 const float* cos_sin, void* k_base, void* v_base, int64_t block_stride,
                                 int64_t token_stride, int64_t head_stride, int page, const int64_t* slots,
                                 void* rk_base, void* rv_base, int64_t r_block_stride, int64_t r_token_stride,
                                 int64_t r_head_stride, int r_page, int r_head_offset, const int64_t* rslots,
                                 cudaStream_t stream) {
  return kvbm_rope_kv_push_heads(qkv, tokens, hq, hkv, positions, cos_sin, k_base, v_base, block_stride,
                                 token_stride, head_stride, page, slots, rk_base, rv_base, r_block_stride,
                                 r_token_stride, r_head_stride, r_page, r_head_offset, rslots, 0, stream);
}

extern "C" int kvbm_silu_mul(const void* gate_up, void* out, int64_t tokens, int inter, cudaStream_t stream) {
  if (tokens == 0) return cudaSuccess;
  if (!gate_up || !out || inter % 8 != 0) return cudaErrorInvalidValue;
  int sms = 148;
  int dev = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t work = tokens * (inter / 8);
  const unsigned grid = static_cast<unsigned>(
      std::max<int64_t>(1, std::min<int64_t>((work + 256 * kSiluUnroll - 1) / (256 * kSiluUnroll),
                                             static_cast<int64_t>(sms) * 8)));
  prefer_max_shared(silu_mul_kernel);
  silu_mul_kernel<<<grid, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(gate_up),
                                            static_cast<__nv_bfloat16*>(out), tokens, inter);
  return cudaGetLastError();
}

// Scratch: part_acc holds batch*hq*splits*128 floats, part_ml batch*hq*splits*2.
extern "C" int kvbm_paged_decode_attn_simt(const void* q, const void* k_base, const void* v_base, int64_t block_stride,
                                      int64_t token_stride, int64_t head_stride, int page, const int32_t* block_table,
                                      int max_blocks, const int32_t* seq_lens, int batch, int hq, int hkv, int hd,
                                      float softmax_scale, int splits, float* part_acc, float* part_ml, void* out,
                                      cudaStream_t stream) {
  if (batch == 0) return cudaSuccess;
  if (!q || !k_base || !v_base || !block_table || !seq_lens || !part_acc || !part_ml || !out)
    return cudaErrorInvalidValue;
  if (hd != kHD || hkv <= 0 || hq % hkv != 0 || page % 16 != 0 || splits <= 0 || splits > 65535)
    return cudaErrorInvalidValue;
  if (token_stride % 16 != 0 || head_stride % 16 != 0 || block_stride % 16 != 0) return cudaErrorInvalidValue;
  const float qscale = softmax_scale * 1.4426950408889634f;  // log2(e)
  dim3 grid(splits, hkv, batch);
  const int group = hq / hkv;
  const auto* qq = static_cast<const __nv_bfloat16*>(q);
  const auto* kb = static_cast<const uint8_t*>(k_base);
  const auto* vb = static_cast<const uint8_t*>(v_base);
  switch (group) {
    case 1:
      paged_decode_kernel<1><<<grid, kAttnWarps * 32, 0, stream>>>(qq, kb, vb, block_stride, token_stride, head_stride,
                                                                   page, block_table, max_blocks, seq_lens, qscale,
                                                                   splits, part_acc, part_ml);
      break;
    case 2:
      paged_decode_kernel<2><<<grid, kAttnWarps * 32, 0, stream>>>(qq, kb, vb, block_stride, token_stride, head_stride,
                                                                   page, block_table, max_blocks, seq_lens, qscale,
                                                                   splits, part_acc, part_ml);
      break;
    case 4:
      paged_decode_kernel<4><<<grid, kAttnWarps * 32, 0, stream>>>(qq, kb, vb, block_stride, token_stride, head_stride,
                                                                   page, block_table, max_blocks, seq_lens, qscale,
                                                                   splits, part_acc, part_ml);
      break;
    case 8:
      paged_decode_kernel<8><<<grid, kAttnWarps * 32, 0, stream>>>(qq, kb, vb, block_stride, token_stride, head_stride,
                                                                   page, block_table, max_blocks, seq_lens, qscale,
                                                                   splits, part_acc, part_ml);
      break;
    default:
      return cudaErrorInvalidValue;
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  attn_combine_kernel<<<static_cast<unsigned>(batch) * hq, kHD, 0, stream>>>(part_acc, part_ml, splits,
                                                                            static_cast<__nv_bfloat16*>(out));
  return cudaGetLastError();
}

namespace {
int decode_attn_mma(const void* q, const void* k_base, const void* v_base, int64_t block_stride,
                    int64_t token_stride, int64_t head_stride, int page, const int32_t* block_table, int max_blocks,
                    const int32_t* seq_lens, int batch, int hq, int hkv, int hd, float softmax_scale, int splits,
                    float* part_acc, float* part_ml, unsigned int* counters, void* out, cudaStream_t stream);
}  // namespace

// Tensor-core paged decode attention (mma.sync + cp.async staging); falls
// back to the SIMT kernel for shapes it does not cover. Same scratch layout.
// Two launches: the split-KV kernel, then the combine kernel.
extern "C" int kvbm_paged_decode_attn(const void* q, const void* k_base, const void* v_base, int64_t block_stride,
                                      int64_t token_stride, int64_t head_stride, int page, const int32_t* block_table,
                                      int max_blocks, const int32_t* seq_lens, int batch, int hq, int hkv, int hd,
                                      float softmax_scale, int splits, float* part_acc, float* part_ml, void* out,
                                      cudaStream_t stream) {
  return decode_attn_mma(q, k_base, v_base, block_stride, token_stride, head_stride, page, block_table, max_blocks,
                         seq_lens, batch, hq, hkv, hd, softmax_scale, splits, part_acc, part_ml, nullptr, out, stream);
}

// One launch: the split-KV kernel's last CTA per (request, KV head) merges the
// splits itself. `counters` holds batch * hkv zero-initialised words; every
// launch leaves them zero again, so one buffer serves every layer and every
// replay of a captured graph. Shapes the tensor-core kernel does not cover
// take the two-launch SIMT path.
extern "C" int kvbm_paged_decode_attn_fused(const void* q, const void* k_base, const void* v_base,
                                            int64_t block_stride, int64_t token_stride, int64_t head_stride, int page,
                                            const int32_t* block_table, int max_blocks, const int32_t* seq_lens,
                                            int batch, int hq, int hkv, int hd, float softmax_scale, int splits,
                                            float* part_acc, float* part_ml, unsigned int* counters, void* out,
                                            cudaStream_t stream) {
  if (!counters) return cudaErrorInvalidValue;
  return decode_attn_mma(q, k_base, v_base, block_stride, token_stride, head_stride, page, block_table, max_blocks,
                         seq_lens, batch, hq, hkv, hd, softmax_scale, splits, part_acc, part_ml, counters, out, stream);
}

namespace {
int decode_attn_mma(const void* q, const void* k_base, const void* v_base, int64_t block_stride,
                    int64_t token_stride, int64_t head_stride, int page, const int32_t* block_table, int max_blocks,
                    const int32_t* seq_lens, int batch, int hq, int hkv, int hd, float softmax_scale, int splits,
                    float* part_acc, float* part_ml, unsigned int* counters, void* out, cudaStream_t stream) {
  const int group = hkv > 0 ? hq / hkv : 0;
  const bool mma_ok = hd == kvbm::attn::kHD && hkv > 0 && hq % hkv == 0 &&
                      (group == 1 || group == 2 || group == 4 || group == 8) && page % 16 == 0 &&
                      token_stride % 16 == 0 && head_stride % 16 == 0 && block_stride % 16 == 0 &&
                      (reinterpret_cast<uintptr_t>(k_base) % 16) == 0 && (reinterpret_cast<uintptr_t>(v_base) % 16) == 0;
  if (!mma_ok)
    return kvbm_paged_decode_attn_simt(q, k_base, v_base, block_stride, token_stride, head_stride, page, block_table,
                                       max_blocks, seq_lens, batch, hq, hkv, hd, softmax_scale, splits, part_acc,
                                       part_ml, out, stream);
  if (batch == 0) return cudaSuccess;
  if (!q || !block_table || !seq_lens || !part_acc || !part_ml || !out || splits <= 0 || splits > 65535)
    return cudaErrorInvalidValue;
  const float qscale = softmax_scale * 1.4426950408889634f;
  dim3 grid(splits, hkv, batch);
  const auto* qq = static_cast<const __nv_bfloat16*>(q);
  const auto* kb = static_cast<const uint8_t*>(k_base);
  const auto* vb = static_cast<const uint8_t*>(v_base);
  const size_t smem = kvbm::attn::kSmemBytes;
  cudaError_t e = cudaSuccess;
#define KVBM_LAUNCH_MMA(G)                                                                                      \
  e = cudaFuncSetAttribute(kvbm::attn::paged_decode_mma_kernel<G>, cudaFuncAttributeMaxDynamicSharedMemorySize,  \
                           static_cast<int>(smem));                                                              \
  if (e != cudaSuccess) return e;                                                                                \
  kvbm::attn::paged_decode_mma_kernel<G><<<grid, kvbm::attn::kWarps * 32, smem, stream>>>(                      \
      qq, kb, vb, block_stride, token_stride, head_stride, page, block_table, max_blocks, seq_lens, qscale, splits, \
      part_acc, part_ml, counters, static_cast<__nv_bfloat16*>(out));
  switch (group) {
    case 1: KVBM_LAUNCH_MMA(1) break;
    case 2: KVBM_LAUNCH_MMA(2) break;
    case 4: KVBM_LAUNCH_MMA(4) break;
    default: KVBM_LAUNCH_MMA(8) break;
  }
#undef KVBM_LAUNCH_MMA
  e = cudaGetLastError();
  if (e != cudaSuccess || counters != nullptr) return e;
  attn_combine_kernel<<<static_cast<unsigned>(batch) * hq, kHD, 0, stream>>>(part_acc, part_ml, splits,
                                                                            static_cast<__nv_bfloat16*>(out));
  return cudaGetLastError();
}
}  // namespace

// ===========================================================================
// Allocation-free paged decode attention.
//
// This entry point is an addition of this library; the reference block
// manager has no counterpart to it.
//
// kvbm_paged_decode_attn_noalloc returns exactly what kvbm_paged_decode_attn
// returns, but it takes no scratch buffers: the per-split partial results it
// needs live in one fixed array in device global memory that belongs to this
// library (kNoAllocMaxRows rows of 130 floats, about 4.3 MB). Every GPU that
// loads the library holds that array until the process exits.
//
// Who needs it: callers that cannot allocate device memory when they call in.
// For example, a host application that owns all device memory through its own
// arena and does not allow other components to call cudaMalloc; code that runs
// inside an allocator's callback, where allocating again would re-enter (or
// deadlock) that allocator; or a latency-critical path that cannot afford the
// device-wide synchronization cudaMalloc and cudaFree may perform. The caller
// still provides q, the KV pool, the block table, the sequence lengths and the
// output buffer.
//
// Set-up: the first call on each device, made while that device is current,
// looks up the array's device address with cudaGetSymbolAddress and caches
// it (the array's name in host code is only a host-side stand-in, never a
// device address). Make that first call before any stream capture starts.
// After set-up a call performs no allocation and calls no allocating routine.
//
// Limit: batch * hq * splits must not exceed kNoAllocMaxRows; a larger request
// is rejected with cudaErrorInvalidValue, and kvbm_last_error_message() says
// why.
//
// Reset: after cudaDeviceReset the address cached for that device is stale;
// the entry point must not be called on a device after resetting it.
//
// Sharing: all calls on one device use the same array, which still holds the
// previous call's partials. Nothing has to be cleared first, because each
// call's split kernel writes every partial row its combine kernel reads. Two
// calls whose kernels can overlap on the GPU (different streams with no
// ordering between them) race on the array and give wrong results: order them
// on one stream or with events.
// ===========================================================================

#include <cstdio>
#include <mutex>

namespace {

constexpr int kNoAllocMaxRows = 8192;
constexpr int kNoAllocMaxDevices = 64;
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocMaxRows * (kHD + 2)];
std::mutex g_noalloc_mu;
float* g_noalloc_ptr[kNoAllocMaxDevices] = {};
thread_local char g_last_error[256] = "";

}  // namespace

extern "C" const char* kvbm_last_error_message(void) { return g_last_error; }

extern "C" int kvbm_paged_decode_attn_noalloc_max_rows(void) { return kNoAllocMaxRows; }

extern "C" int kvbm_paged_decode_attn_noalloc(const void* q, const void* k_base, const void* v_base,
                                              int64_t block_stride, int64_t token_stride, int64_t head_stride,
                                              int page, const int32_t* block_table, int max_blocks,
                                              const int32_t* seq_lens, int batch, int hq, int hkv, int hd,
                                              float softmax_scale, int splits, void* out, cudaStream_t stream) {
  g_last_error[0] = '\0';
  if (batch < 0 || hq < 0 || splits <= 0) {
    std::snprintf(g_last_error, sizeof(g_last_error), "kvbm_paged_decode_attn_noalloc: invalid batch/hq/splits");
    return cudaErrorInvalidValue;
  }
  const int64_t rows = static_cast<int64_t>(batch) * hq * splits;
  if (rows > kNoAllocMaxRows) {
    std::snprintf(g_last_error, sizeof(g_last_error),
                  "kvbm_paged_decode_attn_noalloc: batch*hq*splits = %lld exceeds the static scratch capacity of %d "
                  "rows; use fewer splits or kvbm_paged_decode_attn with caller-provided scratch",
                  static_cast<long long>(rows), kNoAllocMaxRows);
    return cudaErrorInvalidValue;
  }
  if (hd != kHD) {
    std::snprintf(g_last_error, sizeof(g_last_error), "kvbm_paged_decode_attn_noalloc: head_dim must be %d", kHD);
    return cudaErrorInvalidValue;
  }
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kNoAllocMaxDevices) {
    std::snprintf(g_last_error, sizeof(g_last_error), "kvbm_paged_decode_attn_noalloc: device %d unsupported", dev);
    return cudaErrorInvalidDevice;
  }
  float* base = nullptr;
  {
    std::lock_guard<std::mutex> g(g_noalloc_mu);
    if (g_noalloc_ptr[dev] == nullptr) {
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
      if (e != cudaSuccess) {
        std::snprintf(g_last_error, sizeof(g_last_error),
                      "kvbm_paged_decode_attn_noalloc: cudaGetSymbolAddress failed (%s)", cudaGetErrorString(e));
        return e;
      }
      g_noalloc_ptr[dev] = static_cast<float*>(p);
    }
    base = g_noalloc_ptr[dev];
  }
  float* part_acc = base;
  float* part_ml = base + rows * kHD;
  e = static_cast<cudaError_t>(kvbm_paged_decode_attn(q, k_base, v_base, block_stride, token_stride, head_stride,
                                                      page, block_table, max_blocks, seq_lens, batch, hq, hkv, hd,
                                                      softmax_scale, splits, part_acc, part_ml, out, stream));
  if (e != cudaSuccess)
    std::snprintf(g_last_error, sizeof(g_last_error), "kvbm_paged_decode_attn_noalloc: attention launch failed (%s)",
                  cudaGetErrorString(e));
  return e;
}
