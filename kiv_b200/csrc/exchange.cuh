// Peer-memory exchange between the ranks of a sharded layer-step.
//
// Every rank owns an arena that all ranks map (CUDA IPC over NVLink).  Arena
// layout (identical on every rank):
//   header  [4 types][16] u64: word 0 the type's epoch (exchanges done),
//           word 1 a CTA counter (last CTA of a launch);
//   regions one per type, two parities each (epoch & 1), holding the lists
//           of every rank at slot [src], as 64-bit words (flag << 32 | data);
//           the candidate region (X_CAND) instead holds one word per
//           candidate position, written by the rank that owns its page.
// A merge launch of epoch e: each CTA stores its part of this rank's lists
// into slot [rank] of parity e & 1 of every arena, each 32-bit value in one
// 64-bit store together with the flag e + 1 (a single-copy atomic access, so
// no fence is needed: a reader that sees the flag sees the value); it then
// reads every rank's lists from its own arena, waiting (bounded) on each word
// until its flag is e + 1, merges, and the launch's last CTA sets the epoch
// to e + 1.  Two parities suffice: a rank can only start epoch e + 2 after it
// has read every rank's epoch e + 1 lists, which each rank sends only after
// finishing its merge of epoch e.
#pragma once

#include "../../include/kiv_b200.h"
#include "common.cuh"

namespace kiv {

enum XType { X_COARSE = 0, X_FINE = 1, X_ATTN = 2, X_CAND = 3 };
constexpr int X_TYPES = 4;
constexpr int64_t X_HDR_BYTES = 1024;

struct XArgs {
  int32_t world, rank;
  char *arena[KIV_MAX_PEERS];
  int64_t off;        // byte offset of this type's region (parity 0)
  int64_t par_bytes;  // bytes of one parity of the region
  int64_t budget;     // SM clock cycles a wait may spin before it gives up
};

// default bound of every wait: 2^31 cycles, about 1.1 s at 1965 MHz
constexpr int64_t X_DEFAULT_WAIT_CYCLES = 1ll << 31;

// byte offsets of the regions and the arena size for per-rank payloads
// (bytes of one rank's lists) cb, fb, ab and the candidate payload xb (bytes
// of all ranks' candidates together)
struct XLayout {
  int64_t off[X_TYPES], par[X_TYPES], total;
};
__host__ __device__ inline XLayout x_layout(int64_t cb, int64_t fb, int64_t ab, int64_t xb, int world) {
  XLayout L;
  const int64_t pay[X_TYPES] = {cb * world, fb * world, ab * world, xb};
  int64_t o = X_HDR_BYTES;
  for (int t = 0; t < X_TYPES; ++t) {
    L.par[t] = (pay[t] + 255) / 256 * 256;
    L.off[t] = o;
    o += 2 * L.par[t];
  }
  L.total = o;
  return L;
}

__device__ __forceinline__ unsigned long long *x_word(char *arena, int t, int i) {
  return reinterpret_cast<unsigned long long *>(arena) + t * 16 + i;
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys(const unsigned long long *p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned long long x_epoch(const XArgs &x, int t) {
  return *reinterpret_cast<volatile unsigned long long *>(x_word(x.arena[x.rank], t, 0));
}
// region (parity of epoch e) of rank d's arena, as 64-bit words
__device__ __forceinline__ unsigned long long *x_region(const XArgs &x, int d, unsigned long long e) {
  return reinterpret_cast<unsigned long long *>(x.arena[d] + x.off + (int64_t)(e & 1ull) * x.par_bytes);
}
__device__ __forceinline__ uint32_t x_flag(unsigned long long e) { return (uint32_t)(e + 1ull); }
// one value with its flag, in one single-copy atomic 64-bit store
__device__ __forceinline__ void ll_store(unsigned long long *p, uint32_t data, uint32_t flag) {
  const unsigned long long v = ((unsigned long long)flag << 32) | data;
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
// v was loaded from p: if its flag is not `flag` yet, reload until it is (a
// wait bounded by `budget` cycles, after which ok turns false and later
// checks stop waiting); returns the value.  Callers load a batch of words
// first (independent loads, one round trip) and check them afterwards.
__device__ __forceinline__ uint32_t ll_check(const unsigned long long *p, unsigned long long v, uint32_t flag,
                                             bool &ok, int64_t budget) {
  if ((uint32_t)(v >> 32) != flag && ok) {
    const long long t0 = clock64();
    do {
      v = ld_relaxed_sys(p);
      if (clock64() - t0 > budget) {
        ok = false;
        break;
      }
    } while ((uint32_t)(v >> 32) != flag);
  }
  return (uint32_t)v;
}
// the launch's last CTA moves the epoch of type t past e
__device__ __forceinline__ void x_advance(const XArgs &x, int t, unsigned long long e) {
  if (last_block(x_word(x.arena[x.rank], t, 1), gridDim.x) && threadIdx.x == 0)
    *reinterpret_cast<volatile unsigned long long *>(x_word(x.arena[x.rank], t, 0)) = e + 1;
}

}  // namespace kiv
