// Hashing for the block manager: token-block hashes and positional lineage
// sequence hashes.
//
// A SequenceHash identifies a full block of tokens *and* everything before it
// in the sequence. It carries three fields:
//   position (u32) - block index in the sequence, 0-based
//   parent   (u64) - the parent block's lineage hash (0 for the first block)
//   lineage  (u64) - hash chained over (parent lineage, salt, tokens)
// Python sees it as one integer: position << 128 | parent << 64 | lineage.
// The position and parent link let the hub index and the lineage
// eviction policy navigate the prefix tree from a single hash, the role the
// reference's PositionalLineageHash plays (an external dynamo-tokens type that
// is not available here; crates/kvbm-common/src/lib.rs:23). The hash function
// is MurmurHash3 x64-128 (Austin Appleby, public domain algorithm),
// implemented here from its published description.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cstring>
#include <functional>
#include <string>

namespace kvbm {

inline uint64_t rotl64(uint64_t x, int r) { return (x << r) | (x >> (64 - r)); }

inline uint64_t fmix64(uint64_t k) {
  k ^= k >> 33;
  k *= 0xff51afd7ed558ccdULL;
  k ^= k >> 33;
  k *= 0xc4ceb9fe1a85ec53ULL;
  k ^= k >> 33;
  return k;
}

// MurmurHash3 x64 128-bit over `len` bytes.
inline void murmur3_128(const void* key, size_t len, uint64_t seed, uint64_t out[2]) {
  const uint8_t* data = static_cast<const uint8_t*>(key);
  const size_t nblocks = len / 16;
  uint64_t h1 = seed, h2 = seed;
  const uint64_t c1 = 0x87c37b91114253d5ULL;
  const uint64_t c2 = 0x4cf5ad432745937fULL;
  for (size_t i = 0; i < nblocks; ++i) {
    uint64_t k1, k2;
    std::memcpy(&k1, data + i * 16, 8);
    std::memcpy(&k2, data + i * 16 + 8, 8);
    k1 *= c1;
    k1 = rotl64(k1, 31);
    k1 *= c2;
    h1 ^= k1;
    h1 = rotl64(h1, 27);
    h1 += h2;
    h1 = h1 * 5 + 0x52dce729;
    k2 *= c2;
    k2 = rotl64(k2, 33);
    k2 *= c1;
    h2 ^= k2;
    h2 = rotl64(h2, 31);
    h2 += h1;
    h2 = h2 * 5 + 0x38495ab5;
  }
  const uint8_t* tail = data + nblocks * 16;
  uint64_t k1 = 0, k2 = 0;
  switch (len & 15) {
    case 15: k2 ^= uint64_t(tail[14]) << 48; [[fallthrough]];
    case 14: k2 ^= uint64_t(tail[13]) << 40; [[fallthrough]];
    case 13: k2 ^= uint64_t(tail[12]) << 32; [[fallthrough]];
    case 12: k2 ^= uint64_t(tail[11]) << 24; [[fallthrough]];
    case 11: k2 ^= uint64_t(tail[10]) << 16; [[fallthrough]];
    case 10: k2 ^= uint64_t(tail[9]) << 8; [[fallthrough]];
    case 9:
      k2 ^= uint64_t(tail[8]);
      k2 *= c2;
      k2 = rotl64(k2, 33);
      k2 *= c1;
      h2 ^= k2;
      [[fallthrough]];
    case 8: k1 ^= uint64_t(tail[7]) << 56; [[fallthrough]];
    case 7: k1 ^= uint64_t(tail[6]) << 48; [[fallthrough]];
    case 6: k1 ^= uint64_t(tail[5]) << 40; [[fallthrough]];
    case 5: k1 ^= uint64_t(tail[4]) << 32; [[fallthrough]];
    case 4: k1 ^= uint64_t(tail[3]) << 24; [[fallthrough]];
    case 3: k1 ^= uint64_t(tail[2]) << 16; [[fallthrough]];
    case 2: k1 ^= uint64_t(tail[1]) << 8; [[fallthrough]];
    case 1:
      k1 ^= uint64_t(tail[0]);
      k1 *= c1;
      k1 = rotl64(k1, 31);
      k1 *= c2;
      h1 ^= k1;
      break;
    default:
      break;
  }
  h1 ^= len;
  h2 ^= len;
  h1 += h2;
  h2 += h1;
  h1 = fmix64(h1);
  h2 = fmix64(h2);
  h1 += h2;
  h2 += h1;
  out[0] = h1;
  out[1] = h2;
}

inline uint64_t splitmix64(uint64_t x) {
  x += 0x9e3779b97f4a7c15ULL;
  x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ULL;
  x = (x ^ (x >> 27)) * 0x94d049bb133111ebULL;
  return x ^ (x >> 31);
}

struct SeqHash {
  uint64_t lineage = 0;  // chained hash of (parent lineage, salt, tokens)
  uint64_t parent = 0;   // parent block's lineage (0 for the first block)
  uint32_t position = 0; // block index in the sequence, 0-based

  bool operator==(const SeqHash& o) const {
    return lineage == o.lineage && parent == o.parent && position == o.position;
  }
  bool operator!=(const SeqHash& o) const { return !(*this == o); }
};

struct SeqHashHasher {
  size_t operator()(const SeqHash& h) const {
    // lineage is already a well-mixed hash
    return static_cast<size_t>(h.lineage ^ (uint64_t(h.position) * 0x9e3779b97f4a7c15ULL));
  }
};

// Hash of one block's tokens (independent of position), seeded by the salt.
inline uint64_t block_hash(const int32_t* tokens, size_t n, uint64_t salt) {
  uint64_t out[2];
  murmur3_128(tokens, n * sizeof(int32_t), salt, out);
  return out[0];
}

// Salt derived from a string (LoRA name, cache salt); empty string -> 0.
inline uint64_t string_salt(const std::string& s) {
  if (s.empty()) return 0;
  uint64_t out[2];
  murmur3_128(s.data(), s.size(), 0x73616c74ULL, out);
  return out[0];
}

// Chain a block onto its parent (nullptr parent = first block).
inline SeqHash chain(const SeqHash* parent, uint64_t blk_hash, uint64_t salt) {
  uint64_t buf[3] = {parent ? parent->lineage : 0x6b76626d5f726f6fULL, blk_hash, salt};
  uint64_t out[2];
  murmur3_128(buf, sizeof(buf), 0x5eedULL, out);
  SeqHash h;
  h.lineage = out[0] == 0 ? 1 : out[0];  // 0 is reserved for "no parent"
  h.position = parent ? parent->position + 1 : 0;
  h.parent = parent ? parent->lineage : 0;
  return h;
}

}  // namespace kvbm
