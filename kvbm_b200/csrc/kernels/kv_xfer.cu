// Fused KV block transfer kernels for sm_100a.
//
// One kernel family covers every KV movement the block manager needs:
// layout permutes (block stack <-> universal <-> operational, NHD <-> HND),
// KV-head resharding for heterogeneous tensor parallelism, block-scaled fp8
// e4m3 quantisation / dequantisation, and the destination being local HBM,
// mapped pinned host memory (G2) or a peer GPU's HBM mapped through CUDA IPC
// (the prefill -> decode path over NVLink 5 / NVSwitch).
//
// The unit of work is a tile: the [page_size, head_dim] slab of one KV head
// of one (block pair, layer, outer) chunk. Rows of a tile (one token's
// head_dim vector) are contiguous on both sides for every layout the block
// manager uses, so every access is a 16-byte vector and a row maps to
// head_dim*elem/16 consecutive lanes.
//
// Parity: behaviour of crates/kvbm-kernels/cuda/tensor_kernels.cu:171-259
// (universal <-> block), :416-461 (NHD <-> HND) and :667-714 (vectorized
// copy), re-designed as one tiled, warp-per-tile kernel family with
// fusion of the transforms the reference performs in separate passes or not
// at all (fp8 arithmetic, head resharding, peer stores).
#include "common.cuh"
#include "kvbm_kernels.h"

#include <algorithm>
#include <cstdio>
#include <cstring>

using namespace kvbm;

namespace {

constexpr int kWarpsPerCta = 8;
constexpr int kThreads = kWarpsPerCta * 32;
constexpr float kE4M3Max = 448.0f;

enum TileKind : int {
  kCopy = 0,
  kQuantBf16 = 1,
  kQuantF16 = 2,
  kQuantF32 = 3,
  kDequantBf16 = 4,
  kDequantF16 = 5,
  kDequantF32 = 6,
};

struct XferParams {
  KvbmSide src;
  KvbmSide dst;
  KvbmTileShape shape;
  int64_t total_tiles;
  int32_t src_row_bytes;
  int32_t dst_row_bytes;
  FastDiv fd_heads, fd_outer, fd_layers;
  FastDiv fd_upr;  // 16-byte (or U-byte for copies) source units per row
};

__device__ __forceinline__ const uint8_t* chunk_addr(const KvbmSide& s, int64_t p, int64_t i, int64_t o) {
  switch (s.mode) {
    case KVBM_ADDR_LAYER_BASES:
      return reinterpret_cast<const uint8_t*>(s.layer_base[i]) + static_cast<int64_t>(s.ids[p]) * s.block_stride +
             o * s.outer_stride;
    case KVBM_ADDR_BLOCK_TABLE:
      return reinterpret_cast<const uint8_t*>(s.table[p]) + (s.layer_offset + i) * s.layer_stride +
             o * s.outer_stride;
    default:
      return reinterpret_cast<const uint8_t*>(s.table[(p * s.chunk_layers + i) * s.chunk_outer + o]);
  }
}

__device__ __forceinline__ float* scale_addr(const KvbmSide& s, int64_t p, int64_t i, int64_t o, int64_t head) {
  if (s.scales == nullptr) return nullptr;
  const int64_t blk = (s.mode == KVBM_ADDR_LAYER_BASES) ? static_cast<int64_t>(s.ids[p]) : p;
  return s.scales + blk * s.s_block + (s.s_layer_offset + i) * s.s_layer + o * s.s_outer + head * s.s_head;
}

template <int U>
struct UnitT;
template <>
struct UnitT<16> { using T = int4; };
template <>
struct UnitT<8> { using T = int2; };
template <>
struct UnitT<4> { using T = int; };
template <>
struct UnitT<2> { using T = short; };
template <>
struct UnitT<1> { using T = char; };

// ---- per-tile bodies (one warp) --------------------------------------------
//
// `src` / `dst` point at row 0 of the tile; rows are `*_rs` bytes apart.

template <int U>
__device__ __forceinline__ void tile_copy(const uint8_t* src, int64_t src_rs, uint8_t* dst, int64_t dst_rs, int rows,
                                          const FastDiv& upr, int lane) {
  using V = typename UnitT<U>::T;
  constexpr int kBatch = 8;
  const int n = rows * static_cast<int>(upr.d);
  for (int base = 0; base < n; base += 32 * kBatch) {
    V v[kBatch];
#pragma unroll
    for (int k = 0; k < kBatch; ++k) {
      const int u = base + k * 32 + lane;
      if (u < n) {
        const int r = upr.div(u), c = upr.mod(u, r);
        v[k] = *reinterpret_cast<const V*>(src + r * src_rs + c * U);
      }
    }
#pragma unroll
    for (int k = 0; k < kBatch; ++k) {
      const int u = base + k * 32 + lane;
      if (u < n) {
        const int r = upr.div(u), c = upr.mod(u, r);
        *reinterpret_cast<V*>(dst + r * dst_rs + c * U) = v[k];
      }
    }
  }
}

__device__ __forceinline__ uint16_t pack_fp8x2(float a, float b) {
  return static_cast<uint16_t>(__nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3));
}

// Two IEEE fp32 products a*s, b*s in one packed instruction (sm_100 f32x2 SIMD);
// per lane the same rounding as two mul.rn.f32, so results are bit-identical.
__device__ __forceinline__ float2 mul2(float a, float b, float s) {
  uint64_t x, y, r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(x) : "f"(a), "f"(b));
  asm("mov.b64 %0, {%1, %1};" : "=l"(y) : "f"(s));
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(x), "l"(y));
  float2 o;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(o.x), "=f"(o.y) : "l"(r));
  return o;
}

__device__ __forceinline__ float2 unpack_fp8x2(uint16_t x) {
  __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(x), __NV_E4M3);
  __half2 h = *reinterpret_cast<__half2*>(&hr);
  return __half22float2(h);
}

// ---- fp8 e4m3 block scaling ------------------------------------------------
//
// One fp32 scale per tile (per block, layer, outer, head): scale = amax / 448,
// q = satfinite_rn(x * (448 / amax)); x = q * scale on the way back. The
// tile is read once: every lane keeps its share of the tile in registers
// (8 x 16 bytes for a [16 x 128] 16-bit head tile), the warp reduces amax,
// then each lane converts and stores. amax of 16-bit data is taken on the
// raw bits: with the sign bit cleared, non-negative IEEE / bfloat16 values
// order like unsigned integers, so a SIMD unsigned max over the packed
// halves finds the largest magnitude without unpacking (NaN inputs are not
// filtered). Unit index -> (row, column) uses shifts when the units per row
// are a power of two (every head_dim the block manager uses).

struct UnitMap {
  FastDiv upr;
  int shift;  // log2(units per row), or -1
  __device__ __forceinline__ void rc(int u, int& r, int& c) const {
    if (shift >= 0) {
      r = u >> shift;
      c = u & ((1 << shift) - 1);
    } else {
      r = static_cast<int>(upr.div(static_cast<uint32_t>(u)));
      c = static_cast<int>(upr.mod(static_cast<uint32_t>(u), static_cast<uint32_t>(r)));
    }
  }
};

__device__ __forceinline__ UnitMap unit_map(const FastDiv& upr) {
  UnitMap m{upr, -1};
  if ((upr.d & (upr.d - 1)) == 0) m.shift = __ffs(static_cast<int>(upr.d)) - 1;
  return m;
}

template <int KIND>
__device__ __forceinline__ uint32_t unit_amax_bits(const int4& v) {
  if (KIND == kQuantF32) {
    const uint32_t a = static_cast<uint32_t>(v.x) & 0x7fffffffu, b = static_cast<uint32_t>(v.y) & 0x7fffffffu;
    const uint32_t c = static_cast<uint32_t>(v.z) & 0x7fffffffu, d = static_cast<uint32_t>(v.w) & 0x7fffffffu;
    return max(max(a, b), max(c, d));
  }
  const uint32_t m = 0x7fff7fffu;
  const uint32_t a = __vmaxu2(static_cast<uint32_t>(v.x) & m, static_cast<uint32_t>(v.y) & m);
  const uint32_t b = __vmaxu2(static_cast<uint32_t>(v.z) & m, static_cast<uint32_t>(v.w) & m);
  return __vmaxu2(a, b);
}

// Combine two amax words: per 16-bit half for 16-bit data (the halves are
// independent maxima until the very end), as one value for f32.
template <int KIND>
__device__ __forceinline__ uint32_t amax_combine(uint32_t a, uint32_t b) {
  return KIND == kQuantF32 ? max(a, b) : __vmaxu2(a, b);
}

template <int KIND>
__device__ __forceinline__ float amax_bits_to_float(uint32_t bits) {
  if (KIND == kQuantF32) return __uint_as_float(bits);
  const uint32_t h = max(bits & 0xffffu, bits >> 16);
  if (KIND == kQuantBf16) return __uint_as_float(h << 16);
  return __half2float(__ushort_as_half(static_cast<unsigned short>(h)));
}

// ---- fp8 conversions on the integer / FMA pipes ------------------------------
//
// The hardware conversions (f32 -> e4m3x2, e4m3x2 -> f16x2, f32 -> bf16x2)
// issue on the SM's narrow conversion pipe, which the casts saturate; these
// produce the same bits with integer and FMA instructions, for finite inputs:
//   f32 -> e4m3 (round to nearest even, saturating to 448): normal results
//     round the fp32 bits at 3 mantissa bits and rebias the exponent (127 ->
//     7); results below 2^-6 are multiples of 2^-9, rounded by adding
//     1.5 * 2^14 (whose ulp is 2^-9) in fp32 and reading the low bits (the
//     round-by-addition method: an fp32 add rounds to the ulp of the larger
//     operand, to nearest even).
//   e4m3 -> f32: normal codes rebias the exponent; subnormal codes m give
//     m * 2^-9 = (1.5 * 2^14 + m * 2^-9) - 1.5 * 2^14, exact in fp32.
//   f32 -> bf16 (round to nearest even): add 0x7fff plus the kept lsb, keep
//     the top 16 bits.
// The quantiser never writes the e4m3 NaN codes (0x7f / 0xff), so the
// dequantiser does not special-case them.
__device__ __forceinline__ uint32_t f32_to_e4m3_sw(float v) {
  const uint32_t b = __float_as_uint(v);
  const uint32_t a = b & 0x7fffffffu;
  const uint32_t r = a + 0x7ffffu + ((a >> 20) & 1u);
  const uint32_t normal = min((r >> 20) - (120u << 3), 0x7eu);
  const uint32_t sub = __float_as_uint(__uint_as_float(a) + 24576.0f) - 0x46c00000u;
  return ((b >> 24) & 0x80u) | (a >= 0x3c800000u ? normal : sub);
}

__device__ __forceinline__ float e4m3_to_f32_sw(uint32_t c) {
  const uint32_t em = c & 0x7fu;
  const uint32_t normal = (em + (120u << 3)) << 20;
  const uint32_t sub = __float_as_uint(__uint_as_float(0x46c00000u | em) - 24576.0f);
  return __uint_as_float(((c & 0x80u) << 24) | (em >= 8u ? normal : sub));
}

__device__ __forceinline__ uint32_t f32_to_bf16_bits_sw(float v) {
  const uint32_t u = __float_as_uint(v);
  return (u + 0x7fffu + ((u >> 16) & 1u)) >> 16;
}

// 16-byte source unit -> its fp8 bytes (8 for 16-bit sources, 4 for f32), as 32-bit words.
// SWQ: for bf16 sources, this many of every four converted pairs go through the integer / FMA
// pipes (same bits as the hardware path), the rest through the conversion instructions.
template <int KIND, int SWQ = 0>
__device__ __forceinline__ void unit_to_fp8(const int4& v, float inv, uint32_t* out) {
  const uint32_t w[4] = {(uint32_t)v.x, (uint32_t)v.y, (uint32_t)v.z, (uint32_t)v.w};
  if (KIND == kQuantF32) {
    const uint16_t a = pack_fp8x2(__uint_as_float(w[0]) * inv, __uint_as_float(w[1]) * inv);
    const uint16_t b = pack_fp8x2(__uint_as_float(w[2]) * inv, __uint_as_float(w[3]) * inv);
    out[0] = (uint32_t)a | ((uint32_t)b << 16);
    return;
  }
  float f[8];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if (KIND == kQuantBf16) {
      f[2 * j] = __uint_as_float(w[j] << 16);
      f[2 * j + 1] = __uint_as_float(w[j] & 0xffff0000u);
    } else {
      const float2 p = __half22float2(*reinterpret_cast<const __half2*>(&w[j]));
      f[2 * j] = p.x;
      f[2 * j + 1] = p.y;
    }
  }
  float2 p[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) p[j] = mul2(f[2 * j], f[2 * j + 1], inv);
  uint32_t h16[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if (KIND == kQuantBf16 && j < SWQ)
      h16[j] = f32_to_e4m3_sw(p[j].x) | (f32_to_e4m3_sw(p[j].y) << 8);
    else
      h16[j] = pack_fp8x2(p[j].x, p[j].y);
  }
  out[0] = h16[0] | (h16[1] << 16);
  out[1] = h16[2] | (h16[3] << 16);
}

// Quantise one head tile. Lanes take pairs of adjacent 16-byte source units
// (units per row are even for every head_dim that is a multiple of 16), so
// 16-bit sources store 16 fp8 bytes per lane and pair.
template <int KIND>
__device__ __forceinline__ void tile_quant(const uint8_t* src, int64_t src_rs, uint8_t* dst, int64_t dst_rs,
                                           int rows, const FastDiv& upr, float* scale_out, int lane) {
  constexpr int kOut = (KIND == kQuantF32) ? 4 : 8;  // fp8 bytes per source unit
  constexpr int kCache = 4;                           // pairs per lane kept in registers
  const UnitMap um = unit_map(upr);
  const int pairs = rows * static_cast<int>(upr.d) / 2;
  int4 va[kCache], vb[kCache];
  uint32_t mx = 0;
#pragma unroll
  for (int k = 0; k < kCache; ++k) {
    const int q = k * 32 + lane;
    if (q < pairs) {
      int r, c;
      um.rc(2 * q, r, c);
      const int4* p = reinterpret_cast<const int4*>(src + r * src_rs + c * 16);
      va[k] = p[0];
      vb[k] = p[1];
    }
  }
#pragma unroll
  for (int k = 0; k < kCache; ++k) {
    if (k * 32 + lane < pairs)
      mx = amax_combine<KIND>(mx, amax_combine<KIND>(unit_amax_bits<KIND>(va[k]), unit_amax_bits<KIND>(vb[k])));
  }
  for (int q = kCache * 32 + lane; q < pairs; q += 32) {  // tiles larger than the register share
    int r, c;
    um.rc(2 * q, r, c);
    const int4* p = reinterpret_cast<const int4*>(src + r * src_rs + c * 16);
    mx = amax_combine<KIND>(mx, amax_combine<KIND>(unit_amax_bits<KIND>(p[0]), unit_amax_bits<KIND>(p[1])));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = amax_combine<KIND>(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  const float amax = amax_bits_to_float<KIND>(mx);
  const float scale = amax > 0.f ? amax / kE4M3Max : 1.0f;
  const float inv = amax > 0.f ? kE4M3Max / amax : 1.0f;
  auto store_pair = [&](const int4& a, const int4& b, int q) {
    int r, c;
    um.rc(2 * q, r, c);
    uint8_t* d = dst + r * dst_rs + c * kOut;
    uint32_t w[4];
    unit_to_fp8<KIND>(a, inv, w);
    unit_to_fp8<KIND>(b, inv, w + kOut / 4);
    if (KIND == kQuantF32) {
      *reinterpret_cast<uint2*>(d) = make_uint2(w[0], w[1]);
    } else {
      *reinterpret_cast<int4*>(d) = make_int4((int)w[0], (int)w[1], (int)w[2], (int)w[3]);
    }
  };
#pragma unroll
  for (int k = 0; k < kCache; ++k) {
    const int q = k * 32 + lane;
    if (q < pairs) store_pair(va[k], vb[k], q);
  }
  for (int q = kCache * 32 + lane; q < pairs; q += 32) {
    int r, c;
    um.rc(2 * q, r, c);
    const int4* p = reinterpret_cast<const int4*>(src + r * src_rs + c * 16);
    store_pair(p[0], p[1], q);
  }
  if (lane == 0 && scale_out != nullptr) *scale_out = scale;
}

// Dequantise an e4m3 tile into 16-bit or f32 values: x = q * scale. All of a
// lane's loads are issued before its first conversion.
template <int KIND>
__device__ __forceinline__ void tile_dequant(const uint8_t* src, int64_t src_rs, uint8_t* dst, int64_t dst_rs,
                                             int rows, const FastDiv& upr, const float* scale_in, int lane) {
  const float scale = scale_in ? *scale_in : 1.0f;
  const UnitMap um = unit_map(upr);
  const int n = rows * static_cast<int>(upr.d);  // 16 fp8 per source unit
  constexpr int kBatch = 4;
  for (int base = 0; base < n; base += 32 * kBatch) {
    int4 v[kBatch];
#pragma unroll
    for (int k = 0; k < kBatch; ++k) {
      const int u = base + k * 32 + lane;
      if (u < n) {
        int r, c;
        um.rc(u, r, c);
        v[k] = *reinterpret_cast<const int4*>(src + r * src_rs + c * 16);
      }
    }
#pragma unroll
    for (int k = 0; k < kBatch; ++k) {
      const int u = base + k * 32 + lane;
      if (u >= n) continue;
      int r, c;
      um.rc(u, r, c);
      const uint32_t w[4] = {(uint32_t)v[k].x, (uint32_t)v[k].y, (uint32_t)v[k].z, (uint32_t)v[k].w};
      float f[16];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 a = unpack_fp8x2(static_cast<uint16_t>(w[j] & 0xffffu));
        const float2 b = unpack_fp8x2(static_cast<uint16_t>(w[j] >> 16));
        f[4 * j + 0] = a.x * scale;
        f[4 * j + 1] = a.y * scale;
        f[4 * j + 2] = b.x * scale;
        f[4 * j + 3] = b.y * scale;
      }
      uint8_t* d = dst + r * dst_rs;
      if (KIND == kDequantF32) {
#pragma unroll
        for (int q = 0; q < 4; ++q)
          *reinterpret_cast<float4*>(d + c * 64 + q * 16) =
              make_float4(f[4 * q], f[4 * q + 1], f[4 * q + 2], f[4 * q + 3]);
      } else {
        uint32_t o[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (KIND == kDequantBf16) {
            __nv_bfloat162 bb = __floats2bfloat162_rn(f[2 * j], f[2 * j + 1]);
            o[j] = *reinterpret_cast<uint32_t*>(&bb);
          } else {
            __half2 hh = __floats2half2_rn(f[2 * j], f[2 * j + 1]);
            o[j] = *reinterpret_cast<uint32_t*>(&hh);
          }
        }
        *reinterpret_cast<int4*>(d + c * 32) = make_int4(o[0], o[1], o[2], o[3]);
        *reinterpret_cast<int4*>(d + c * 32 + 16) = make_int4(o[4], o[5], o[6], o[7]);
      }
    }
  }
}

// ---- software-pipelined fp8 tiles ------------------------------------------
//
// When a head tile fits one batch per lane (16 x 16-byte source units for a
// quantise, 4 fp8 units for a dequantise: every [16 x 128] head tile), a
// persistent warp keeps the copies of its next tiles in flight (cp.async
// into a per-warp shared-memory ring) while it reduces, converts and stores
// the current one, so DRAM reads overlap the cast math without costing
// registers. Larger tiles take the one-tile-at-a-time path.

constexpr int kQPairs = 4;   // source unit pairs per lane held per tile
constexpr int kDqUnits = 4;  // fp8 source units per lane held per tile

template <int KIND, int SWQ = 0>
__device__ __forceinline__ void quant_store(const int4 (&va)[kQPairs], const int4 (&vb)[kQPairs], uint8_t* dst,
                                            int64_t rs, int pairs, const UnitMap& um, float* scale_out, int lane) {
  constexpr int kOut = (KIND == kQuantF32) ? 4 : 8;
  uint32_t mx = 0;
#pragma unroll
  for (int k = 0; k < kQPairs; ++k)
    if (k * 32 + lane < pairs)
      mx = amax_combine<KIND>(mx, amax_combine<KIND>(unit_amax_bits<KIND>(va[k]), unit_amax_bits<KIND>(vb[k])));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = amax_combine<KIND>(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  const float amax = amax_bits_to_float<KIND>(mx);
  const float inv = amax > 0.f ? kE4M3Max / amax : 1.0f;
#pragma unroll
  for (int k = 0; k < kQPairs; ++k) {
    const int q = k * 32 + lane;
    if (q >= pairs) continue;
    int r, c;
    um.rc(2 * q, r, c);
    uint8_t* d = dst + r * rs + c * kOut;
    uint32_t w[4];
    unit_to_fp8<KIND, SWQ>(va[k], inv, w);
    unit_to_fp8<KIND, SWQ>(vb[k], inv, w + kOut / 4);
    if (KIND == kQuantF32) {
      *reinterpret_cast<uint2*>(d) = make_uint2(w[0], w[1]);
    } else {
      *reinterpret_cast<int4*>(d) = make_int4((int)w[0], (int)w[1], (int)w[2], (int)w[3]);
    }
  }
  if (lane == 0 && scale_out != nullptr) *scale_out = amax > 0.f ? amax / kE4M3Max : 1.0f;
}

template <int KIND, int SWQ = 0>
__device__ __forceinline__ void dequant_store(const int4 (&v)[kDqUnits], uint8_t* dst, int64_t rs, int n,
                                              const UnitMap& um, float scale, int lane) {
#pragma unroll
  for (int k = 0; k < kDqUnits; ++k) {
    const int u = k * 32 + lane;
    if (u >= n) continue;
    int r, c;
    um.rc(u, r, c);
    const uint32_t w[4] = {(uint32_t)v[k].x, (uint32_t)v[k].y, (uint32_t)v[k].z, (uint32_t)v[k].w};
    if constexpr (SWQ > 0 && KIND == kDequantBf16) {
      // word j (4 fp8 values): the first SWQ words on the integer / FMA pipes, the rest in hardware
      uint32_t o[8];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (j < SWQ) {
          const float2 pa = mul2(e4m3_to_f32_sw(w[j]), e4m3_to_f32_sw(w[j] >> 8), scale);
          const float2 pb = mul2(e4m3_to_f32_sw(w[j] >> 16), e4m3_to_f32_sw(w[j] >> 24), scale);
          o[2 * j] = __byte_perm(f32_to_bf16_bits_sw(pa.x), f32_to_bf16_bits_sw(pa.y), 0x5410);
          o[2 * j + 1] = __byte_perm(f32_to_bf16_bits_sw(pb.x), f32_to_bf16_bits_sw(pb.y), 0x5410);
        } else {
          const float2 a = unpack_fp8x2(static_cast<uint16_t>(w[j] & 0xffffu));
          const float2 b = unpack_fp8x2(static_cast<uint16_t>(w[j] >> 16));
          const float2 pa = mul2(a.x, a.y, scale), pb = mul2(b.x, b.y, scale);
          __nv_bfloat162 ba = __floats2bfloat162_rn(pa.x, pa.y), bb = __floats2bfloat162_rn(pb.x, pb.y);
          o[2 * j] = *reinterpret_cast<uint32_t*>(&ba);
          o[2 * j + 1] = *reinterpret_cast<uint32_t*>(&bb);
        }
      }
      uint8_t* d = dst + r * rs;
      *reinterpret_cast<int4*>(d + c * 32) = make_int4(o[0], o[1], o[2], o[3]);
      *reinterpret_cast<int4*>(d + c * 32 + 16) = make_int4(o[4], o[5], o[6], o[7]);
      continue;
    }
    float f[16];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 a = unpack_fp8x2(static_cast<uint16_t>(w[j] & 0xffffu));
      const float2 b = unpack_fp8x2(static_cast<uint16_t>(w[j] >> 16));
      const float2 pa = mul2(a.x, a.y, scale), pb = mul2(b.x, b.y, scale);
      f[4 * j + 0] = pa.x;
      f[4 * j + 1] = pa.y;
      f[4 * j + 2] = pb.x;
      f[4 * j + 3] = pb.y;
    }
    uint8_t* d = dst + r * rs;
    if (KIND == kDequantF32) {
#pragma unroll
      for (int q = 0; q < 4; ++q)
        *reinterpret_cast<float4*>(d + c * 64 + q * 16) = make_float4(f[4 * q], f[4 * q + 1], f[4 * q + 2], f[4 * q + 3]);
    } else {
      uint32_t o[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (KIND == kDequantBf16) {
          __nv_bfloat162 bb = __floats2bfloat162_rn(f[2 * j], f[2 * j + 1]);
          o[j] = *reinterpret_cast<uint32_t*>(&bb);
        } else {
          __half2 hh = __floats2half2_rn(f[2 * j], f[2 * j + 1]);
          o[j] = *reinterpret_cast<uint32_t*>(&hh);
        }
      }
      *reinterpret_cast<int4*>(d + c * 32) = make_int4(o[0], o[1], o[2], o[3]);
      *reinterpret_cast<int4*>(d + c * 32 + 16) = make_int4(o[4], o[5], o[6], o[7]);
    }
  }
}

struct TilePtrs {
  const uint8_t* s;
  uint8_t* d;
  float* scale;
};

template <int KIND>
__device__ __forceinline__ TilePtrs tile_ptrs(const XferParams& P, int64_t t) {
  const uint32_t t32 = static_cast<uint32_t>(t);
  const uint32_t q1 = P.fd_heads.div(t32);
  const int h = static_cast<int>(P.fd_heads.mod(t32, q1));
  const uint32_t q2 = P.fd_outer.div(q1);
  const int64_t o = P.fd_outer.mod(q1, q2);
  const uint32_t q3 = P.fd_layers.div(q2);
  const int64_t i = P.fd_layers.mod(q2, q3);
  const int64_t p = q3;
  TilePtrs r;
  r.s = chunk_addr(P.src, p, i, o) + static_cast<int64_t>(h + P.src.head_offset) * P.src.head_stride;
  r.d = const_cast<uint8_t*>(chunk_addr(P.dst, p, i, o)) + static_cast<int64_t>(h + P.dst.head_offset) * P.dst.head_stride;
  r.scale = (KIND <= kQuantF32) ? scale_addr(P.dst, p, i, o, h + P.dst.head_offset)
                                : scale_addr(P.src, p, i, o, h + P.src.head_offset);
  return r;
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const uint32_t sa = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(sa), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Copy one source tile densely into a warp's shared-memory slot (unit u at byte 16 u).
__device__ __forceinline__ void tile_fetch(const uint8_t* src, int64_t rs, int units, const UnitMap& um, int lane,
                                           uint8_t* slot) {
  for (int u = lane; u < units; u += 32) {
    int r, c;
    um.rc(u, r, c);
    cp_async16(slot + u * 16, src + r * rs + c * 16);
  }
}

// Each warp walks its tiles (warp, warp + nwarps, ...) through a ring of S
// shared-memory slots filled by cp.async: the copies of the next S - 1 tiles
// are in flight while the warp reduces, converts and stores the current one,
// without holding them in registers.
template <int KIND, int S, int SWQ>
__device__ __forceinline__ void cast_tiles_async(const XferParams& P, uint8_t* ring, int tile_bytes, int64_t warp,
                                                 int64_t nwarps, int lane) {
  const UnitMap um = unit_map(P.fd_upr);
  const int units = P.shape.page_size * static_cast<int>(P.fd_upr.d);
  const int64_t srs = P.src.token_stride, drs = P.dst.token_stride;
  const int64_t total = P.total_tiles;
#pragma unroll
  for (int k = 0; k < S - 1; ++k) {
    const int64_t t = warp + k * nwarps;
    if (t < total) tile_fetch(tile_ptrs<KIND>(P, t).s, srs, units, um, lane, ring + k * tile_bytes);
    cp_async_commit();
  }
  for (int64_t k = 0;; ++k) {
    const int64_t t = warp + k * nwarps;
    if (t >= total) break;
    const int64_t tn = t + (S - 1) * nwarps;
    if (tn < total) tile_fetch(tile_ptrs<KIND>(P, tn).s, srs, units, um, lane, ring + ((k + S - 1) % S) * tile_bytes);
    cp_async_commit();
    cp_async_wait<S - 1>();  // this tile's group has landed (S - 1 younger groups may still fly)
    __syncwarp();
    const uint8_t* slot = ring + (k % S) * tile_bytes;
    const TilePtrs cur = tile_ptrs<KIND>(P, t);
    if constexpr (KIND <= kQuantF32) {
      const int pairs = units / 2;
      int4 a[kQPairs], b[kQPairs];
#pragma unroll
      for (int j = 0; j < kQPairs; ++j) {
        const int q = j * 32 + lane;
        if (q < pairs) {
          a[j] = *reinterpret_cast<const int4*>(slot + 32 * q);
          b[j] = *reinterpret_cast<const int4*>(slot + 32 * q + 16);
        }
      }
      quant_store<KIND, SWQ>(a, b, cur.d, drs, pairs, um, cur.scale, lane);
    } else {
      int4 v[kDqUnits];
#pragma unroll
      for (int j = 0; j < kDqUnits; ++j) {
        const int u = j * 32 + lane;
        if (u < units) v[j] = *reinterpret_cast<const int4*>(slot + 16 * u);
      }
      dequant_store<KIND, SWQ>(v, cur.d, drs, units, um, cur.scale ? *cur.scale : 1.0f, lane);
    }
    __syncwarp();  // every lane is done with the slot before it is refilled
  }
  cp_async_wait<0>();
}

template <int KIND, int U>
__device__ __forceinline__ void run_tile(const XferParams& P, const uint8_t* s, int64_t s_rs, uint8_t* d,
                                         int64_t d_rs, int64_t p, int64_t i, int64_t o, int h, int lane) {
  const int rows = P.shape.page_size;
  if constexpr (KIND == kCopy) {
    tile_copy<U>(s, s_rs, d, d_rs, rows, P.fd_upr, lane);
    // fp8 -> fp8 copies carry their scales along.
    if (lane == 0 && P.src.scales != nullptr && P.dst.scales != nullptr) {
      *scale_addr(P.dst, p, i, o, h + P.dst.head_offset) = *scale_addr(P.src, p, i, o, h + P.src.head_offset);
    }
  } else if constexpr (KIND == kQuantBf16 || KIND == kQuantF16 || KIND == kQuantF32) {
    tile_quant<KIND>(s, s_rs, d, d_rs, rows, P.fd_upr, scale_addr(P.dst, p, i, o, h + P.dst.head_offset), lane);
  } else {
    tile_dequant<KIND>(s, s_rs, d, d_rs, rows, P.fd_upr, scale_addr(P.src, p, i, o, h + P.src.head_offset), lane);
  }
}

// Warp-per-tile kernel. Tiles are ordered (pair, layer, outer, head) with
// head fastest so the warps of one CTA sweep one contiguous chunk together.
// Ring depth of the pipelined cast kernels: 3 x 4 KiB slots per warp for a
// quantise (two CTAs of 96 KiB per SM), 4 x 2 KiB for a dequantise.
__host__ __device__ constexpr int cast_stages(int kind) { return kind <= kQuantF32 ? 3 : 4; }

template <int KIND, int SWQ>
__global__ void __launch_bounds__(kThreads) kv_cast_pipe_kernel(const __grid_constant__ XferParams P, int tile_bytes) {
  extern __shared__ __align__(128) uint8_t cast_smem[];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  constexpr int S = cast_stages(KIND);
  const int64_t warp = static_cast<int64_t>(blockIdx.x) * kWarpsPerCta + w;
  cast_tiles_async<KIND, S, SWQ>(P, cast_smem + static_cast<size_t>(w) * S * tile_bytes, tile_bytes, warp,
                            static_cast<int64_t>(gridDim.x) * kWarpsPerCta, lane);
}

template <int KIND, int U>
__global__ void __launch_bounds__(kThreads, KIND == kCopy ? 1 : 4) kv_tile_xfer_kernel(const __grid_constant__ XferParams P) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = static_cast<int64_t>(blockIdx.x) * kWarpsPerCta + (threadIdx.x >> 5);
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * kWarpsPerCta;
  for (int64_t t = warp; t < P.total_tiles; t += nwarps) {
    // 32-bit decode through precomputed reciprocals (total_tiles < 2^31)
    const uint32_t t32 = static_cast<uint32_t>(t);
    const uint32_t q1 = P.fd_heads.div(t32);
    const int h = static_cast<int>(P.fd_heads.mod(t32, q1));
    const uint32_t q2 = P.fd_outer.div(q1);
    const int64_t o = P.fd_outer.mod(q1, q2);
    const uint32_t q3 = P.fd_layers.div(q2);
    const int64_t i = P.fd_layers.mod(q2, q3);
    const int64_t p = q3;
    const uint8_t* s = chunk_addr(P.src, p, i, o) + static_cast<int64_t>(h + P.src.head_offset) * P.src.head_stride;
    uint8_t* d = const_cast<uint8_t*>(chunk_addr(P.dst, p, i, o)) +
                 static_cast<int64_t>(h + P.dst.head_offset) * P.dst.head_stride;
    run_tile<KIND, U>(P, s, P.src.token_stride, d, P.dst.token_stride, p, i, o, h, lane);
  }
}

int g_sm_count = 0;

int sm_count() {
  if (g_sm_count == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_sm_count, cudaDevAttrMultiProcessorCount, dev);
    if (g_sm_count <= 0) g_sm_count = 148;
  }
  return g_sm_count;
}

int dtype_bytes(int dt) {
  switch (dt) {
    case KVBM_F16:
    case KVBM_BF16:
      return 2;
    case KVBM_F32:
      return 4;
    case KVBM_F64:
      return 8;
    case KVBM_FP8_E4M3:
      return 1;
    default:
      return 0;
  }
}

int pick_kind(int sdt, int ddt) {
  if (sdt == ddt) return kCopy;
  if (ddt == KVBM_FP8_E4M3) {
    if (sdt == KVBM_BF16) return kQuantBf16;
    if (sdt == KVBM_F16) return kQuantF16;
    if (sdt == KVBM_F32) return kQuantF32;
  }
  if (sdt == KVBM_FP8_E4M3) {
    if (ddt == KVBM_BF16) return kDequantBf16;
    if (ddt == KVBM_F16) return kDequantF16;
    if (ddt == KVBM_F32) return kDequantF32;
  }
  return -1;
}

bool side_ok(const KvbmSide& s, int layers) {
  if (s.mode == KVBM_ADDR_LAYER_BASES) {
    if (s.ids == nullptr || layers > KVBM_MAX_LAYERS) return false;
    for (int i = 0; i < layers; ++i)
      if (s.layer_base[i] == 0) return false;
    return true;
  }
  if (s.mode == KVBM_ADDR_BLOCK_TABLE) return s.table != nullptr;
  if (s.mode == KVBM_ADDR_CHUNK_TABLE) return s.table != nullptr && s.chunk_layers > 0 && s.chunk_outer > 0;
  return false;
}

// Largest power-of-two unit (<= 16) dividing every byte quantity given.
int common_align(std::initializer_list<int64_t> xs) {
  int a = 16;
  for (int64_t x : xs) {
    while (a > 1 && (x % a) != 0) a >>= 1;
  }
  return a;
}

bool g_cast_pipe = true;
// Quarters (0, 1, 2, 4) of the bf16 <-> fp8 conversions done on the integer / FMA pipes. Measured on
// B200 (128 Llama-3-8B blocks): quantise is fastest all in hardware (software conversion costs more
// than the conversion pipe saves); dequantise is fastest with one quarter in software (+8 %), which
// offloads the saturated conversion pipe without saturating the integer pipe.
int g_cast_soft_quant = 0;
int g_cast_soft_dequant = 1;

template <int KIND, int U>
cudaError_t launch_tile(const XferParams& P, int max_ctas, cudaStream_t stream) {
  const int64_t ctas_needed = (P.total_tiles + kWarpsPerCta - 1) / kWarpsPerCta;
  if constexpr (KIND != kCopy) {
    const int units = P.shape.page_size * static_cast<int>(P.fd_upr.d);
    const bool fits = (KIND <= kQuantF32) ? units / 2 <= kQPairs * 32 : units <= kDqUnits * 32;
    if (g_cast_pipe && fits) {
      // persistent: every warp walks many tiles, so the next tiles' copies overlap this one's math
      const int tile_bytes = units * 16;
      const size_t smem = static_cast<size_t>(kWarpsPerCta) * cast_stages(KIND) * tile_bytes;
      auto kern = kv_cast_pipe_kernel<KIND, 0>;
      if constexpr (KIND == kQuantBf16 || KIND == kDequantBf16) {
        const int q = KIND == kQuantBf16 ? g_cast_soft_quant : g_cast_soft_dequant;
        if (q == 1) kern = kv_cast_pipe_kernel<KIND, 1>;
        if (q == 2) kern = kv_cast_pipe_kernel<KIND, 2>;
        if (q >= 4) kern = kv_cast_pipe_kernel<KIND, 4>;
      }
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
      if (e != cudaSuccess) return e;
      int per_sm = 1;
      e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, smem);
      if (e != cudaSuccess) return e;
      const int64_t pcap = max_ctas > 0 ? max_ctas : static_cast<int64_t>(sm_count()) * std::max(1, per_sm);
      const int pgrid = static_cast<int>(std::max<int64_t>(1, std::min(ctas_needed, pcap)));
      kern<<<pgrid, kThreads, smem, stream>>>(P, tile_bytes);
      return cudaGetLastError();
    }
  }
  int64_t cap = max_ctas > 0 ? max_ctas : static_cast<int64_t>(sm_count()) * 8;
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min(ctas_needed, cap)));
  kv_tile_xfer_kernel<KIND, U><<<grid, kThreads, 0, stream>>>(P);
  return cudaGetLastError();
}

cudaError_t dispatch_tile(const XferParams& P, int kind, int unit, int max_ctas, cudaStream_t stream) {
  switch (kind) {
    case kCopy:
      switch (unit) {
        case 16: return launch_tile<kCopy, 16>(P, max_ctas, stream);
        case 8: return launch_tile<kCopy, 8>(P, max_ctas, stream);
        case 4: return launch_tile<kCopy, 4>(P, max_ctas, stream);
        case 2: return launch_tile<kCopy, 2>(P, max_ctas, stream);
        default: return launch_tile<kCopy, 1>(P, max_ctas, stream);
      }
    case kQuantBf16: return launch_tile<kQuantBf16, 16>(P, max_ctas, stream);
    case kQuantF16: return launch_tile<kQuantF16, 16>(P, max_ctas, stream);
    case kQuantF32: return launch_tile<kQuantF32, 16>(P, max_ctas, stream);
    case kDequantBf16: return launch_tile<kDequantBf16, 16>(P, max_ctas, stream);
    case kDequantF16: return launch_tile<kDequantF16, 16>(P, max_ctas, stream);
    case kDequantF32: return launch_tile<kDequantF32, 16>(P, max_ctas, stream);
    default: return cudaErrorInvalidValue;
  }
}

// Validates the request and fills P; returns the tile kind or -1.
int prepare(const KvbmSide* src, const KvbmSide* dst, const KvbmTileShape* shape, XferParams& P, int* unit_out) {
  if (!src || !dst || !shape) return -1;
  const KvbmTileShape& S = *shape;
  if (S.num_pairs < 0 || S.num_layers < 0 || S.num_outer <= 0 || S.num_heads <= 0 || S.page_size <= 0 ||
      S.head_dim <= 0)
    return -1;
  if (S.num_layers > KVBM_MAX_LAYERS && (src->mode == KVBM_ADDR_LAYER_BASES || dst->mode == KVBM_ADDR_LAYER_BASES))
    return -1;
  if (src->head_offset < 0 || dst->head_offset < 0) return -1;
  const int kind = pick_kind(S.src_dtype, S.dst_dtype);
  if (kind < 0) return -1;
  const int sb = dtype_bytes(S.src_dtype), db = dtype_bytes(S.dst_dtype);
  std::memcpy(&P.src, src, sizeof(KvbmSide));
  std::memcpy(&P.dst, dst, sizeof(KvbmSide));
  P.shape = S;
  P.total_tiles = static_cast<int64_t>(S.num_pairs) * S.num_layers * S.num_outer * S.num_heads;
  P.src_row_bytes = S.head_dim * sb;
  P.dst_row_bytes = S.head_dim * db;
  if (P.total_tiles >= (int64_t(1) << 31)) return -1;  // callers split larger batches
  P.fd_heads = FastDiv(static_cast<uint32_t>(S.num_heads));
  P.fd_outer = FastDiv(static_cast<uint32_t>(S.num_outer));
  P.fd_layers = FastDiv(static_cast<uint32_t>(std::max(1, S.num_layers)));
  if (P.total_tiles == 0) {
    *unit_out = 16;
    return kind;
  }
  if (!side_ok(P.src, S.num_layers) || !side_ok(P.dst, S.num_layers)) return -1;
  if (kind == kCopy) {
    int64_t a = common_align({P.src_row_bytes, P.src.token_stride, P.src.head_stride, P.dst.token_stride,
                              P.dst.head_stride, P.src.block_stride, P.dst.block_stride, P.src.outer_stride,
                              P.dst.outer_stride, P.src.layer_stride, P.dst.layer_stride});
    for (int i = 0; i < S.num_layers && P.src.mode == KVBM_ADDR_LAYER_BASES; ++i)
      a = std::min<int64_t>(a, common_align({static_cast<int64_t>(P.src.layer_base[i])}));
    for (int i = 0; i < S.num_layers && P.dst.mode == KVBM_ADDR_LAYER_BASES; ++i)
      a = std::min<int64_t>(a, common_align({static_cast<int64_t>(P.dst.layer_base[i])}));
    // Table-mode base pointers are device-resident; the caller guarantees the
    // element alignment, so the unit never drops below the element size.
    *unit_out = static_cast<int>(std::max<int64_t>(a, sb));
    if (*unit_out > 16) *unit_out = 16;
  } else {
    // Conversions work on 16-byte source units and need 16 fp8 / 8 x 16-bit
    // elements per unit, with every row start 16-byte aligned on both sides.
    if (S.head_dim % 16 != 0) return -1;
    const int64_t a = common_align({P.src.token_stride, P.src.head_stride, P.dst.token_stride, P.dst.head_stride,
                                    P.src.block_stride, P.dst.block_stride, P.src.outer_stride, P.dst.outer_stride,
                                    P.src.layer_stride, P.dst.layer_stride});
    if (a < 16) return -1;
    *unit_out = 16;
  }
  P.fd_upr = FastDiv(static_cast<uint32_t>(P.src_row_bytes / *unit_out));
  return kind;
}

// ---- checksums ---------------------------------------------------------------
// splitmix64 finalizer (Steele, Lea, Flood: "Fast splittable pseudorandom
// number generators", OOPSLA 2014), applied to (word, index) pairs.
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}

__global__ void __launch_bounds__(kThreads) kv_checksum_kernel(const __grid_constant__ XferParams P,
                                                                unsigned long long* out) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = static_cast<int64_t>(blockIdx.x) * kWarpsPerCta + (threadIdx.x >> 5);
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * kWarpsPerCta;
  const int wpr = P.src_row_bytes / 4;  // 4-byte words per row
  const int page = P.shape.page_size, H = P.shape.num_heads, O = P.shape.num_outer;
  const int n = page * wpr;
  for (int64_t t = warp; t < P.total_tiles; t += nwarps) {
    const uint32_t t32 = static_cast<uint32_t>(t);
    const uint32_t q1 = P.fd_heads.div(t32);
    const int h = static_cast<int>(P.fd_heads.mod(t32, q1));
    const uint32_t q2 = P.fd_outer.div(q1);
    const int64_t o = P.fd_outer.mod(q1, q2);
    const uint32_t q3 = P.fd_layers.div(q2);
    const int64_t i = P.fd_layers.mod(q2, q3);
    const int64_t p = q3;
    const uint8_t* s = chunk_addr(P.src, p, i, o) + static_cast<int64_t>(h + P.src.head_offset) * P.src.head_stride;
    uint64_t acc = 0;
    for (int u = lane; u < n; u += 32) {
      const int r = P.fd_upr.div(static_cast<uint32_t>(u)), c = P.fd_upr.mod(static_cast<uint32_t>(u), r);
      const uint32_t wv = *reinterpret_cast<const uint32_t*>(s + r * P.src.token_stride + c * 4);
      const uint64_t idx = ((static_cast<uint64_t>(i * O + o) * page + r) * H + h) * wpr + c;
      acc += mix64((idx << 32) ^ wv ^ 0x9e3779b97f4a7c15ull);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (lane == 0) atomicAdd(out + p, static_cast<unsigned long long>(acc));
  }
}

}  // namespace

extern "C" int kvbm_kv_checksum(const KvbmSide* side, const KvbmTileShape* shape, uint64_t* out,
                                cudaStream_t stream) {
  if (!side || !shape || !out) return cudaErrorInvalidValue;
  KvbmTileShape S = *shape;
  S.dst_dtype = S.src_dtype;
  XferParams P;
  int unit = 16;
  if (prepare(side, side, &S, P, &unit) < 0) return cudaErrorInvalidValue;
  if (P.src_row_bytes % 4 != 0 || P.src.token_stride % 4 != 0 || P.src.head_stride % 4 != 0)
    return cudaErrorInvalidValue;
  if (S.num_pairs == 0) return cudaSuccess;
  cudaError_t e = cudaMemsetAsync(out, 0, sizeof(uint64_t) * S.num_pairs, stream);
  if (e != cudaSuccess) return e;
  P.fd_upr = FastDiv(static_cast<uint32_t>(P.src_row_bytes / 4));
  const int64_t ctas = (P.total_tiles + kWarpsPerCta - 1) / kWarpsPerCta;
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(ctas, int64_t{sm_count()} * 8)));
  kv_checksum_kernel<<<grid, kThreads, 0, stream>>>(P, reinterpret_cast<unsigned long long*>(out));
  return cudaGetLastError();
}

extern "C" int kvbm_sm_count(void) { return sm_count(); }

extern "C" int kvbm_kv_tile_xfer(const KvbmSide* src, const KvbmSide* dst, const KvbmTileShape* shape, int max_ctas,
                                 cudaStream_t stream) {
  XferParams P;
  int unit = 16;
  const int kind = prepare(src, dst, shape, P, &unit);
  if (kind < 0) return cudaErrorInvalidValue;
  if (P.total_tiles == 0) return cudaSuccess;
  return dispatch_tile(P, kind, unit, max_ctas, stream);
}

// ---------------------------------------------------------------------------
// TMA-staged chunk pipeline.
//
// One CTA = 1 producer warp + 8 consumer warps. The producer's elected lane
// issues 1-D bulk async copies (cp.async.bulk, local source) of a whole
// (pair, layer, outer) chunk, or of its per-token / per-head contiguous runs,
// into a ring of shared-memory stages; completion is counted in bytes on a
// "full" mbarrier per stage. Consumer warps take one head tile each from the
// staged chunk, convert it and store it to the destination, then arrive on
// the stage's "empty" mbarrier. Every wait is bounded by %globaltimer.
// ---------------------------------------------------------------------------

namespace {

constexpr int kConsumerWarps = 8;
constexpr int kPipeThreads = (kConsumerWarps + 1) * 32;
constexpr uint64_t kPipeWaitNs = 2000000000ull;  // 2 s

struct PipeParams {
  XferParams x;
  int32_t stages;
  int32_t stage_bytes;
  int32_t chunk_bytes;      // bytes copied per chunk
  int32_t run_bytes;        // bytes per contiguous run
  int32_t num_runs;         // runs per chunk
  int32_t src_nhd;          // 1: smem rows ordered [token][head], 0: [head][token]
  int64_t run_stride;       // global-memory stride between runs
  int64_t total_chunks;
  int* status;              // status word in mapped host memory (may be null)
  uint64_t wait_ns;         // limit of every pipeline wait
};

// This CTA's contiguous range of chunks. Chunks are ordered (pair, layer,
// outer), so a contiguous range walks one block's layers before the next
// block's: each CTA touches a few memory pages at a time on both sides
// (fewer address-translation misses than a grid-strided walk over pools
// that span tens of GiB).
__device__ __forceinline__ void cta_chunks(int64_t total, int64_t& begin, int64_t& count) {
  const int64_t G = gridDim.x, b = blockIdx.x;
  const int64_t per = total / G, rem = total % G;
  count = per + (b < rem ? 1 : 0);
  begin = b * per + (b < rem ? b : rem);
}

// A pipeline wait bounded by `limit_ns`. A limit of 1 ns or less gives up at
// once, before the first try (mbarrier.try_wait may itself block for a while,
// so a tiny limit alone would not make the give-up path run reliably): the
// test hook that exercises the timeout path without any fault.
__device__ __forceinline__ bool pipe_wait(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
  if (limit_ns <= 1) return false;
  return mbar_wait_bounded(bar, parity, limit_ns);
}

template <int KIND>
__global__ void __launch_bounds__(kPipeThreads, 1) kv_chunk_pipe_kernel(const __grid_constant__ PipeParams Q) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  const XferParams& P = Q.x;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem_raw);
  uint64_t* empty_bar = full_bar + Q.stages;
  uint8_t* stage_base = smem_raw + 1024;  // barriers live in the first 1 KiB
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int H = P.shape.num_heads, O = P.shape.num_outer, L = P.shape.num_layers;
  // Consumer warps form groups of wc warps; each group takes every groups-th
  // staged chunk and splits its head tiles, so chunks with fewer heads than
  // consumer warps (KV-head slices of a TP rank) keep every warp busy.
  const int wc = H < kConsumerWarps ? H : kConsumerWarps;
  const int groups = kConsumerWarps / wc;
  if (threadIdx.x == 0) {
    for (int s = 0; s < Q.stages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], wc);
    }
    fence_mbar_init();
  }
  __syncthreads();

  const int T = P.shape.page_size;
  const int64_t row = P.src_row_bytes;

  if (warp == kConsumerWarps) {
    // ---------------- producer ----------------
    if (lane == 0) {
      int64_t k = 0;
      bool ok = true;
      int64_t begin, count;
      cta_chunks(Q.total_chunks, begin, count);
      for (; k < count && ok; ++k) {
        const int64_t c = begin + k;
        const int s = static_cast<int>(k % Q.stages);
        const uint32_t phase = static_cast<uint32_t>((k / Q.stages) & 1);
        if (k >= Q.stages && !pipe_wait(&empty_bar[s], phase ^ 1u, Q.wait_ns)) {
          ok = false;
          break;
        }
        int64_t r = c;
        const int64_t o = r % O;
        r /= O;
        const int64_t i = r % L;
        const int64_t p = r / L;
        const uint8_t* base = chunk_addr(P.src, p, i, o) +
                              (Q.src_nhd ? static_cast<int64_t>(P.src.head_offset) * row
                                         : static_cast<int64_t>(P.src.head_offset) * P.src.head_stride);
        if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) {
          // Never issue a misaligned bulk copy: record it and stop.
          report_status(Q.status, kStatusBadIndex);
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&full_bar[s], static_cast<uint32_t>(Q.chunk_bytes));
        uint8_t* dst = stage_base + static_cast<int64_t>(s) * Q.stage_bytes;
        for (int j = 0; j < Q.num_runs; ++j)
          bulk_g2s(dst + static_cast<int64_t>(j) * Q.run_bytes, base + j * Q.run_stride,
                   static_cast<uint32_t>(Q.run_bytes), &full_bar[s]);
      }
      if (!ok) {
        report_status(Q.status, kStatusPipelineTimeout);
        // Drain: wait (bounded by the full 2 s, whatever the pipeline's own
        // limit) for the copies already issued so none are in flight when
        // the CTA exits.
        const int64_t issued = k;
        const int64_t first = issued > Q.stages ? issued - Q.stages : 0;
        for (int64_t kk = first; kk < issued; ++kk) {
          const int s = static_cast<int>(kk % Q.stages);
          mbar_wait_bounded(&full_bar[s], static_cast<uint32_t>((kk / Q.stages) & 1), kPipeWaitNs);
        }
      }
    }
    return;
  }

  // ---------------- consumers ----------------
  const int group = warp / wc, gw = warp - group * wc;
  if (group >= groups) return;  // H does not divide the consumer warps: the remainder idles
  int64_t begin, count;
  cta_chunks(Q.total_chunks, begin, count);
  for (int64_t k = group; k < count; k += groups) {
    const int64_t c = begin + k;
    const int s = static_cast<int>(k % Q.stages);
    const uint32_t phase = static_cast<uint32_t>((k / Q.stages) & 1);
    if (!pipe_wait(&full_bar[s], phase, Q.wait_ns)) {
      if (lane == 0) report_status(Q.status, kStatusPipelineTimeout);
      break;
    }
    int64_t r = c;
    const int64_t o = r % O;
    r /= O;
    const int64_t i = r % L;
    const int64_t p = r / L;
    const uint8_t* sbuf = stage_base + static_cast<int64_t>(s) * Q.stage_bytes;
    uint8_t* dchunk = const_cast<uint8_t*>(chunk_addr(P.dst, p, i, o));
    for (int h = gw; h < H; h += wc) {
      const uint8_t* srow = Q.src_nhd ? sbuf + h * row : sbuf + static_cast<int64_t>(h) * T * row;
      const int64_t s_rs = Q.src_nhd ? static_cast<int64_t>(H) * row : row;
      uint8_t* d = dchunk + static_cast<int64_t>(h + P.dst.head_offset) * P.dst.head_stride;
      run_tile<KIND, 16>(P, srow, s_rs, d, P.dst.token_stride, p, i, o, h, lane);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty_bar[s]);
  }
}

template <int KIND>
cudaError_t launch_pipe(PipeParams& Q, int max_ctas, cudaStream_t stream) {
  const size_t smem = 1024 + static_cast<size_t>(Q.stages) * Q.stage_bytes;
  cudaError_t e = cudaFuncSetAttribute(kv_chunk_pipe_kernel<KIND>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  const int64_t cap = max_ctas > 0 ? max_ctas : sm_count();
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(Q.total_chunks, cap)));
  kv_chunk_pipe_kernel<KIND><<<grid, kPipeThreads, smem, stream>>>(Q);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Bulk copy engine: same-layout, same-dtype chunks moved entirely by the TMA
// unit. One thread per CTA keeps stages-1 bulk loads (global -> shared) in
// flight ahead of the bulk stores (shared -> global) that drain them; no SM
// load/store instruction touches the data, so the copy rate does not follow
// the SM clock down when the GPU runs at its power cap.
// ---------------------------------------------------------------------------

__device__ __forceinline__ const uint8_t* src_chunk(const XferParams& P, int64_t c) {
  const int O = P.shape.num_outer, L = P.shape.num_layers;
  int64_t r = c;
  const int64_t o = r % O;
  r /= O;
  const int64_t i = r % L;
  return chunk_addr(P.src, r / L, i, o);
}

__device__ __forceinline__ uint8_t* dst_chunk(const XferParams& P, int64_t c) {
  const int O = P.shape.num_outer, L = P.shape.num_layers;
  int64_t r = c;
  const int64_t o = r % O;
  r /= O;
  const int64_t i = r % L;
  return const_cast<uint8_t*>(chunk_addr(P.dst, r / L, i, o));
}

__global__ void __launch_bounds__(32, 1) kv_bulk_copy_kernel(const __grid_constant__ PipeParams Q) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  if (threadIdx.x != 0) return;
  const XferParams& P = Q.x;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem_raw);
  uint8_t* stage0 = smem_raw + 1024;
  const int S = Q.stages;
  for (int s = 0; s < S; ++s) mbar_init(&full[s], 1);
  fence_mbar_init();
  int64_t begin, n;
  cta_chunks(Q.total_chunks, begin, n);
  const uint32_t bytes = static_cast<uint32_t>(Q.chunk_bytes);
  int64_t issued = 0;  // loads issued so far (chunk j of this CTA = begin + j)
  bool ok = true;
  auto load = [&](int64_t j) -> bool {
    const uint8_t* src = src_chunk(P, begin + j);
    if ((reinterpret_cast<uintptr_t>(src) & 15) != 0) return false;
    const int s = static_cast<int>(j % S);
    mbar_arrive_expect_tx(&full[s], bytes);
    bulk_g2s(stage0 + static_cast<int64_t>(s) * Q.stage_bytes, src, bytes, &full[s]);
    return true;
  };
  for (; issued < n && issued < S; ++issued) {
    if (!load(issued)) {
      report_status(Q.status, kStatusBadIndex);
      ok = false;
      break;
    }
  }
  int64_t j = 0;
  for (; ok && j < n; ++j) {
    const int s = static_cast<int>(j % S);
    if (!pipe_wait(&full[s], static_cast<uint32_t>((j / S) & 1), Q.wait_ns)) {
      report_status(Q.status, kStatusPipelineTimeout);
      ok = false;
      break;
    }
    uint8_t* dst = dst_chunk(P, begin + j);
    if ((reinterpret_cast<uintptr_t>(dst) & 15) != 0) {
      report_status(Q.status, kStatusBadIndex);
      ok = false;
      break;
    }
    fence_proxy_async_smem();
    bulk_s2g(dst, stage0 + static_cast<int64_t>(s) * Q.stage_bytes, bytes);
    bulk_commit();
    // refill the previous chunk's stage: its store had this iteration to read shared memory
    if (j >= 1 && issued < n) {
      bulk_wait_read<1>();
      if (!load(issued)) {
        report_status(Q.status, kStatusBadIndex);
        ok = false;
        break;
      }
      ++issued;
    }
  }
  if (!ok) {
    // loads issued but not consumed: wait (bounded) so none lands after the CTA exits
    for (int64_t k = j; k < issued; ++k)
      mbar_wait_bounded(&full[k % S], static_cast<uint32_t>((k / S) & 1), kPipeWaitNs);
  }
  bulk_wait_all<0>();  // every store complete before the kernel ends
}

int* g_status_host = nullptr;  // one status word per device, in mapped pinned memory
uint64_t g_wait_ns_override = 0;
constexpr int kMaxDevices = 64;

int* status_word() {
  if (g_status_host == nullptr) {
    void* p = nullptr;
    if (cudaHostAlloc(&p, sizeof(int) * kMaxDevices, cudaHostAllocMapped | cudaHostAllocPortable) != cudaSuccess)
      return nullptr;
    std::memset(p, 0, sizeof(int) * kMaxDevices);
    g_status_host = static_cast<int*>(p);
  }
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= kMaxDevices) return nullptr;
  void* d = nullptr;
  if (cudaHostGetDevicePointer(&d, g_status_host + dev, 0) != cudaSuccess) return nullptr;
  return static_cast<int*>(d);
}

enum XferEngine { kEngineAuto = 0, kEngineTile = 1, kEngineTma = 2 };
enum XferRan { kRanNone = 0, kRanTile = 1, kRanTmaPipe = 2, kRanTmaBulk = 3 };

// Fills Q for the TMA engines; returns the tile kind, or -1 when the source
// chunks are not contiguous / aligned (the TMA engines cannot take them).
int tma_setup(const KvbmSide* src, const KvbmSide* dst, const KvbmTileShape* shape, PipeParams& Q) {
  std::memset(&Q, 0, sizeof(Q));
  int unit = 16;
  const int kind = prepare(src, dst, shape, Q.x, &unit);
  if (kind < 0) return -1;
  const KvbmTileShape& S = Q.x.shape;
  const int64_t row = Q.x.src_row_bytes;
  const KvbmSide& s = Q.x.src;
  if (row % 16 != 0 || (kind == kCopy && Q.x.dst_row_bytes % 16 != 0)) return -1;
  // Find the contiguous runs of one chunk on the source side.
  if (s.head_stride == row) {
    // NHD-like: each token holds its heads back to back.
    Q.src_nhd = 1;
    if (s.token_stride == row * S.num_heads) {
      Q.num_runs = 1;
      Q.run_bytes = static_cast<int32_t>(row * S.num_heads * S.page_size);
    } else {
      Q.num_runs = S.page_size;
      Q.run_bytes = static_cast<int32_t>(row * S.num_heads);
      Q.run_stride = s.token_stride;
    }
  } else if (s.token_stride == row) {
    // HND-like: each head holds its tokens back to back.
    Q.src_nhd = 0;
    if (s.head_stride == row * S.page_size) {
      Q.num_runs = 1;
      Q.run_bytes = static_cast<int32_t>(row * S.num_heads * S.page_size);
    } else {
      Q.num_runs = S.num_heads;
      Q.run_bytes = static_cast<int32_t>(row * S.page_size);
      Q.run_stride = s.head_stride;
    }
  } else {
    return -1;
  }
  if (Q.run_bytes % 16 != 0 || Q.run_stride % 16 != 0) return -1;
  Q.chunk_bytes = Q.run_bytes * Q.num_runs;
  Q.stage_bytes = (Q.chunk_bytes + 127) / 128 * 128;
  const int budget = 200 * 1024;
  Q.stages = std::min(16, budget / Q.stage_bytes);
  if (Q.stages < 2) return -1;
  Q.total_chunks = static_cast<int64_t>(S.num_pairs) * S.num_layers * S.num_outer;
  Q.status = status_word();
  Q.wait_ns = g_wait_ns_override ? g_wait_ns_override : kPipeWaitNs;
  return kind;
}

// Whether the destination chunk is the source chunk's exact byte image (a
// whole contiguous chunk in the same layout and dtype).
bool bulk_eligible(const PipeParams& Q, int kind) {
  const KvbmSide& s = Q.x.src;
  const KvbmSide& d = Q.x.dst;
  return kind == kCopy && Q.num_runs == 1 && s.head_offset == 0 && d.head_offset == 0 &&
         d.token_stride == s.token_stride && d.head_stride == s.head_stride && Q.x.dst_row_bytes == Q.x.src_row_bytes &&
         s.scales == nullptr && d.scales == nullptr;
}

cudaError_t launch_bulk(PipeParams& Q, int max_ctas, cudaStream_t stream) {
  const size_t smem = 1024 + static_cast<size_t>(Q.stages) * Q.stage_bytes;
  cudaError_t e =
      cudaFuncSetAttribute(kv_bulk_copy_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  const int64_t cap = max_ctas > 0 ? max_ctas : sm_count();
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(Q.total_chunks, cap)));
  kv_bulk_copy_kernel<<<grid, 32, smem, stream>>>(Q);
  return cudaGetLastError();
}

cudaError_t dispatch_pipe(PipeParams& Q, int kind, int max_ctas, cudaStream_t stream) {
  switch (kind) {
    case kCopy: return launch_pipe<kCopy>(Q, max_ctas, stream);
    case kQuantBf16: return launch_pipe<kQuantBf16>(Q, max_ctas, stream);
    case kQuantF16: return launch_pipe<kQuantF16>(Q, max_ctas, stream);
    case kQuantF32: return launch_pipe<kQuantF32>(Q, max_ctas, stream);
    case kDequantBf16: return launch_pipe<kDequantBf16>(Q, max_ctas, stream);
    case kDequantF16: return launch_pipe<kDequantF16>(Q, max_ctas, stream);
    case kDequantF32: return launch_pipe<kDequantF32>(Q, max_ctas, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

extern "C" int kvbm_kv_chunk_xfer_tma(const KvbmSide* src, const KvbmSide* dst, const KvbmTileShape* shape,
                                      int max_ctas, cudaStream_t stream) {
  PipeParams Q;
  const int kind = tma_setup(src, dst, shape, Q);
  if (kind < 0) return cudaErrorInvalidValue;
  if (Q.x.total_tiles == 0) return cudaSuccess;
  return dispatch_pipe(Q, kind, max_ctas, stream);
}

extern "C" int kvbm_kv_xfer(const KvbmSide* src, const KvbmSide* dst, const KvbmTileShape* shape, int engine,
                            int max_ctas, int flags, int* ran, cudaStream_t stream) {
  if (ran) *ran = kRanNone;
  if (engine != kEngineTile) {
    PipeParams Q;
    const int kind = tma_setup(src, dst, shape, Q);
    if (kind >= 0) {
      if (Q.x.total_tiles == 0) return cudaSuccess;
      const bool dst_bulk_ok = (flags & KVBM_XFER_DST_LOCAL) || (flags & KVBM_XFER_BULK_PEER);
      if (dst_bulk_ok && !(flags & KVBM_XFER_NO_BULK) && bulk_eligible(Q, kind)) {
        if (ran) *ran = kRanTmaBulk;
        return launch_bulk(Q, max_ctas, stream);
      }
      if (ran) *ran = kRanTmaPipe;
      return dispatch_pipe(Q, kind, max_ctas, stream);
    }
    if (engine == kEngineTma) return cudaErrorInvalidValue;  // asked for the TMA engine: never a silent fallback
  }
  XferParams P;
  int unit = 16;
  const int kind = prepare(src, dst, shape, P, &unit);
  if (kind < 0) return cudaErrorInvalidValue;
  if (P.total_tiles == 0) return cudaSuccess;
  if (ran) *ran = kRanTile;
  return dispatch_tile(P, kind, unit, max_ctas, stream);
}

extern "C" int kvbm_xfer_status(int device, int reset) {
  if (g_status_host == nullptr || device < 0 || device >= kMaxDevices) return 0;
  const int v = *reinterpret_cast<volatile int*>(g_status_host + device);
  if (reset) *reinterpret_cast<volatile int*>(g_status_host + device) = 0;
  return v;
}

// 1 (default): fp8 casts whose head tile fits one register batch run the
// software-pipelined persistent kernel; 0: the one-tile-at-a-time kernel.
extern "C" void kvbm_xfer_set_cast_pipeline(int on) { g_cast_pipe = on != 0; }

// Quarters (0, 1, 2 or 4) of the pipelined cast kernel's bf16 -> fp8 and
// fp8 -> bf16 conversions done on the integer / FMA pipes (same bits) instead
// of with the conversion instructions, to balance the two pipes. Defaults:
// 0 for quantise, 1 for dequantise.
extern "C" void kvbm_xfer_set_cast_softconv(int quant_quarters, int dequant_quarters) {
  g_cast_soft_quant = quant_quarters < 0 ? 0 : quant_quarters;
  g_cast_soft_dequant = dequant_quarters < 0 ? 0 : dequant_quarters;
}

extern "C" void kvbm_xfer_set_wait_limit_ns(uint64_t ns) { g_wait_ns_override = ns; }

// ---------------------------------------------------------------------------
// Reference-compatible permutes (pointer-table API), expressed as tile
// transfers.
// ---------------------------------------------------------------------------

namespace {

void fill_universal(KvbmSide& u, const void* const* ptrs, size_t nh, size_t no, size_t nt, size_t hd, size_t nl_full,
                    size_t nl_offset, int eb) {
  std::memset(&u, 0, sizeof(u));
  u.mode = KVBM_ADDR_BLOCK_TABLE;
  u.table = reinterpret_cast<const uint64_t*>(ptrs);
  u.token_stride = static_cast<int64_t>(hd) * eb;
  u.outer_stride = static_cast<int64_t>(nt * hd) * eb;
  u.layer_stride = static_cast<int64_t>(no * nt * hd) * eb;
  u.head_stride = static_cast<int64_t>(nl_full * no * nt * hd) * eb;
  u.layer_offset = static_cast<int64_t>(nl_offset);
  (void)nh;
}

void fill_stack(KvbmSide& b, const void* const* ptrs, size_t nl, size_t no, size_t nt, size_t nh, size_t hd,
                int layout, int eb) {
  std::memset(&b, 0, sizeof(b));
  b.mode = KVBM_ADDR_CHUNK_TABLE;
  b.table = reinterpret_cast<const uint64_t*>(ptrs);
  b.chunk_layers = static_cast<int32_t>(nl);
  b.chunk_outer = static_cast<int32_t>(no);
  if (layout == KVBM_NHD) {
    b.token_stride = static_cast<int64_t>(nh * hd) * eb;
    b.head_stride = static_cast<int64_t>(hd) * eb;
  } else {
    b.token_stride = static_cast<int64_t>(hd) * eb;
    b.head_stride = static_cast<int64_t>(nt * hd) * eb;
  }
}

int permute_common(const KvbmSide& src, const KvbmSide& dst, size_t num_blocks, size_t nh, size_t nl, size_t no,
                   size_t nt, size_t hd, int dtype, cudaStream_t stream) {
  if (dtype_bytes(dtype) == 0) return cudaErrorInvalidValue;
  if (num_blocks == 0 || nh == 0 || nl == 0 || no == 0 || nt == 0 || hd == 0) return cudaSuccess;
  KvbmTileShape S;
  S.num_pairs = static_cast<int32_t>(num_blocks);
  S.num_layers = static_cast<int32_t>(nl);
  S.num_outer = static_cast<int32_t>(no);
  S.num_heads = static_cast<int32_t>(nh);
  S.page_size = static_cast<int32_t>(nt);
  S.head_dim = static_cast<int32_t>(hd);
  S.src_dtype = dtype;
  S.dst_dtype = dtype;
  return kvbm_kv_tile_xfer(&src, &dst, &S, 0, stream);
}

}  // namespace

extern "C" int kvbm_universal_from_block(void* const* universal_ptrs, const void* const* block_ptrs,
                                         size_t num_blocks, size_t nh, size_t nl, size_t no, size_t nt, size_t hd,
                                         size_t nl_full, size_t nl_offset, int dtype, int layout,
                                         cudaStream_t stream) {
  if (num_blocks == 0) return cudaSuccess;
  if (!universal_ptrs || !block_ptrs || nl_offset + nl > nl_full) return cudaErrorInvalidValue;
  if (layout != KVBM_NHD && layout != KVBM_HND) return cudaErrorInvalidValue;
  const int eb = dtype_bytes(dtype);
  if (eb == 0) return cudaErrorInvalidValue;
  KvbmSide src, dst;
  fill_stack(src, block_ptrs, nl, no, nt, nh, hd, layout, eb);
  fill_universal(dst, const_cast<const void* const*>(universal_ptrs), nh, no, nt, hd, nl_full, nl_offset, eb);
  return permute_common(src, dst, num_blocks, nh, nl, no, nt, hd, dtype, stream);
}

extern "C" int kvbm_block_from_universal(const void* const* universal_ptrs, void* const* block_ptrs,
                                         size_t num_blocks, size_t nh, size_t nl, size_t no, size_t nt, size_t hd,
                                         size_t nl_full, size_t nl_offset, int dtype, int layout,
                                         cudaStream_t stream) {
  if (num_blocks == 0) return cudaSuccess;
  if (!universal_ptrs || !block_ptrs || nl_offset + nl > nl_full) return cudaErrorInvalidValue;
  if (layout != KVBM_NHD && layout != KVBM_HND) return cudaErrorInvalidValue;
  const int eb = dtype_bytes(dtype);
  if (eb == 0) return cudaErrorInvalidValue;
  KvbmSide src, dst;
  fill_universal(src, universal_ptrs, nh, no, nt, hd, nl_full, nl_offset, eb);
  fill_stack(dst, const_cast<const void* const*>(block_ptrs), nl, no, nt, nh, hd, layout, eb);
  return permute_common(src, dst, num_blocks, nh, nl, no, nt, hd, dtype, stream);
}

extern "C" int kvbm_nhd_hnd_transpose(const void* const* src_chunks, void* const* dst_chunks, size_t num_blocks,
                                      size_t nl, size_t no, size_t nt, size_t nh, size_t hd, int dtype,
                                      int src_layout, cudaStream_t stream) {
  if (num_blocks == 0) return cudaSuccess;
  if (!src_chunks || !dst_chunks) return cudaErrorInvalidValue;
  if (src_layout != KVBM_NHD && src_layout != KVBM_HND) return cudaErrorInvalidValue;
  const int eb = dtype_bytes(dtype);
  if (eb == 0) return cudaErrorInvalidValue;
  KvbmSide src, dst;
  fill_stack(src, src_chunks, nl, no, nt, nh, hd, src_layout, eb);
  fill_stack(dst, const_cast<const void* const*>(dst_chunks), nl, no, nt, nh, hd,
             src_layout == KVBM_NHD ? KVBM_HND : KVBM_NHD, eb);
  return permute_common(src, dst, num_blocks, nh, nl, no, nt, hd, dtype, stream);
}

// ---------------------------------------------------------------------------
// Split-by-bytes batched copy (replaces one-CTA-per-pair copying).
// ---------------------------------------------------------------------------

namespace {

template <int U>
__global__ void __launch_bounds__(kThreads) copy_pairs_kernel(const uint64_t* __restrict__ src_ptrs,
                                                             const uint64_t* __restrict__ dst_ptrs,
                                                             uint64_t num_pairs, uint64_t bytes,
                                                             uint64_t chunks_per_pair) {
  using V = typename UnitT<U>::T;
  constexpr int kBatch = 8;
  constexpr uint64_t kChunk = 32ull * kBatch * U;  // bytes per warp work item
  const int lane = threadIdx.x & 31;
  const uint64_t warp = static_cast<uint64_t>(blockIdx.x) * kWarpsPerCta + (threadIdx.x >> 5);
  const uint64_t nwarps = static_cast<uint64_t>(gridDim.x) * kWarpsPerCta;
  const uint64_t total = num_pairs * chunks_per_pair;
  for (uint64_t w = warp; w < total; w += nwarps) {
    const uint64_t p = w / chunks_per_pair;
    const uint64_t off = (w - p * chunks_per_pair) * kChunk;
    const uint8_t* s = reinterpret_cast<const uint8_t*>(src_ptrs[p]) + off;
    uint8_t* d = reinterpret_cast<uint8_t*>(dst_ptrs[p]) + off;
    const uint64_t n = min(kChunk, bytes - off) / U;
    V v[kBatch];
#pragma unroll
    for (int k = 0; k < kBatch; ++k) {
      const uint64_t u = k * 32 + lane;
      if (u < n) v[k] = *reinterpret_cast<const V*>(s + u * U);
    }
#pragma unroll
    for (int k = 0; k < kBatch; ++k) {
      const uint64_t u = k * 32 + lane;
      if (u < n) *reinterpret_cast<V*>(d + u * U) = v[k];
    }
  }
}

template <int U>
cudaError_t launch_copy(const uint64_t* s, const uint64_t* d, uint64_t n, uint64_t bytes, int max_ctas,
                        cudaStream_t stream) {
  constexpr uint64_t kChunk = 32ull * 8 * U;
  const uint64_t cpp = (bytes + kChunk - 1) / kChunk;
  const uint64_t work = n * cpp;
  const uint64_t need = (work + kWarpsPerCta - 1) / kWarpsPerCta;
  const uint64_t cap = max_ctas > 0 ? static_cast<uint64_t>(max_ctas) : static_cast<uint64_t>(sm_count()) * 8;
  const int grid = static_cast<int>(std::max<uint64_t>(1, std::min(need, cap)));
  copy_pairs_kernel<U><<<grid, kThreads, 0, stream>>>(s, d, n, bytes, cpp);
  return cudaGetLastError();
}

}  // namespace

extern "C" int kvbm_copy_pairs(const uint64_t* src_ptrs, const uint64_t* dst_ptrs, uint64_t num_pairs,
                               uint64_t bytes_per_pair, int align, int max_ctas, cudaStream_t stream) {
  if (num_pairs == 0 || bytes_per_pair == 0) return cudaSuccess;
  if (!src_ptrs || !dst_ptrs) return cudaErrorInvalidValue;
  int a = 16;
  while (a > 1 && (align % a != 0 || bytes_per_pair % a != 0)) a >>= 1;
  switch (a) {
    case 16: return launch_copy<16>(src_ptrs, dst_ptrs, num_pairs, bytes_per_pair, max_ctas, stream);
    case 8: return launch_copy<8>(src_ptrs, dst_ptrs, num_pairs, bytes_per_pair, max_ctas, stream);
    case 4: return launch_copy<4>(src_ptrs, dst_ptrs, num_pairs, bytes_per_pair, max_ctas, stream);
    case 2: return launch_copy<2>(src_ptrs, dst_ptrs, num_pairs, bytes_per_pair, max_ctas, stream);
    default: return launch_copy<1>(src_ptrs, dst_ptrs, num_pairs, bytes_per_pair, max_ctas, stream);
  }
}

// ---------------------------------------------------------------------------
// System-scope completion flags.
// ---------------------------------------------------------------------------

namespace {

__global__ void signal_kernel(uint64_t* flag, uint64_t value) {
  fence_acq_rel_sys();
  st_release_sys_u64(flag, value);
}

// Copy `n` 64-bit payload words (e.g. the first generated token) to the
// peer, then publish the flag with release semantics at system scope.
__global__ void signal_payload_kernel(uint64_t* flag, uint64_t value, uint64_t* dst, const uint64_t* src, int n) {
  for (int i = 0; i < n; ++i) dst[i] = src[i];
  fence_acq_rel_sys();
  st_release_sys_u64(flag, value);
}

// Wait until every flags[i] >= expected (one thread, bounded by timeout_ns).
__global__ void wait_all_kernel(const uint64_t* flags, int n, uint64_t expected, uint64_t timeout_ns, int* status) {
  const uint64_t t0 = globaltimer_ns();
  for (int i = 0; i < n; ++i) {
    while (ld_acquire_sys_u64(flags + i) < expected) {
      if (globaltimer_ns() - t0 > timeout_ns) {
        if (status) atomicExch(status, kStatusWaitTimeout);
        return;
      }
      __nanosleep(256);
    }
  }
}

__global__ void wait_kernel(const uint64_t* flag, uint64_t expected, uint64_t timeout_ns, int* status) {
  const uint64_t t0 = globaltimer_ns();
  while (ld_acquire_sys_u64(flag) < expected) {
    if (globaltimer_ns() - t0 > timeout_ns) {
      if (status) atomicExch(status, kStatusWaitTimeout);
      return;
    }
    __nanosleep(256);
  }
}

}  // namespace

extern "C" int kvbm_signal_flag(uint64_t* flag, uint64_t value, cudaStream_t stream) {
  if (!flag) return cudaErrorInvalidValue;
  signal_kernel<<<1, 1, 0, stream>>>(flag, value);
  return cudaGetLastError();
}

extern "C" int kvbm_signal_flag_payload(uint64_t* flag, uint64_t value, uint64_t* payload_dst,
                                        const uint64_t* payload_src, int n_words, cudaStream_t stream) {
  if (!flag || n_words < 0 || (n_words > 0 && (!payload_dst || !payload_src))) return cudaErrorInvalidValue;
  signal_payload_kernel<<<1, 1, 0, stream>>>(flag, value, payload_dst, payload_src, n_words);
  return cudaGetLastError();
}

extern "C" int kvbm_wait_flags_all(const uint64_t* flags, int n, uint64_t expected, uint64_t timeout_ns, int* status,
                                   cudaStream_t stream) {
  if (!flags || n < 0) return cudaErrorInvalidValue;
  if (n == 0) return cudaSuccess;
  wait_all_kernel<<<1, 1, 0, stream>>>(flags, n, expected, timeout_ns, status);
  return cudaGetLastError();
}

extern "C" int kvbm_wait_flag(const uint64_t* flag, uint64_t expected, uint64_t timeout_ns, int* status,
                              cudaStream_t stream) {
  if (!flag) return cudaErrorInvalidValue;
  wait_kernel<<<1, 1, 0, stream>>>(flag, expected, timeout_ns, status);
  return cudaGetLastError();
}
