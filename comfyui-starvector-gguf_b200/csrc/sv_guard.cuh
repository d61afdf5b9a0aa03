// sv_guard.cuh -- the incremental loop guard's window hash and occurrence table,
// shared by sv_loop_guard.cu (insert + probe) and sv_advance.cu (the beam loop's
// per-step inserts).
//
// A window of `w` tokens ending at position e hashes to
//   h(e) = sum_{k<w} tok(x[e-w+1+k]) * B^(w-1-k)   (mod 2^32, x[<0] contributing 0),
// which rolls as h(e) = h(e-1) * B + tok(x[e]) - tok(x[e-w]) * B^w.  The table holds
// one 64-bit entry (hash << 32 | start) per distinct (window hash, start) pair,
// open addressing with linear probing from fmix32(hash) (MurmurHash3's finalizer,
// Austin Appleby, public domain); an all-ones word is an empty slot.  Every match of
// the hash is verified token by token, so the table only narrows the candidates.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace sv {

constexpr uint32_t kGuardBase = 0x9E3779B1u;
constexpr unsigned long long kGuardEmpty = ~0ull;

__device__ __forceinline__ uint32_t guard_tok(int32_t x) { return (uint32_t)x; }
__device__ __forceinline__ uint32_t guard_tok(int64_t x) { return (uint32_t)x ^ ((uint32_t)(x >> 32) * 0x85EBCA6Bu); }

__device__ __forceinline__ uint32_t guard_pow(uint32_t b, int e) {
  uint32_t r = 1;
  for (; e; e >>= 1, b *= b)
    if (e & 1) r *= b;
  return r;
}

__device__ __forceinline__ uint32_t guard_mix(uint32_t h) {
  h ^= h >> 16;
  h *= 0x85EBCA6Bu;
  h ^= h >> 13;
  h *= 0xC2B2AE35u;
  h ^= h >> 16;
  return h;
}

// Inserts (h, start) unless present; false when the table is full.
__device__ __forceinline__ bool guard_insert(unsigned long long* table, int64_t mask, uint32_t h, uint32_t start) {
  const unsigned long long e = ((unsigned long long)h << 32) | start;
  int64_t slot = guard_mix(h) & mask;
  for (int64_t i = 0; i <= mask; ++i) {
    const unsigned long long old = atomicCAS(&table[slot], kGuardEmpty, e);
    if (old == kGuardEmpty || old == e) return true;
    slot = (slot + 1) & mask;
  }
  return false;
}

}  // namespace sv
