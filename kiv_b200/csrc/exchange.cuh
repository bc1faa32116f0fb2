// Peer-memory exchange between the ranks of a sharded layer-step.
//
// Every rank owns an arena that all ranks map (CUDA IPC over NVLink).  Arena
// layout (identical on every rank):
//   header  [3 types][16] u64: word 0 the type's epoch (exchanges done),
//           word 1 a CTA counter (last CTA of a launch), words 8 + src the
//           number of CTAs of rank src that have delivered into this arena;
//   regions one per type, two parities each (epoch & 1), holding the lists
//           of every rank at slot [src].
// A merge launch of epoch e: each CTA stores its part of this rank's lists
// into slot [rank] of parity e & 1 of every arena, fences at system scope and
// adds 1 to counter [rank] of every arena (release); then it waits until
// every counter of its own arena reaches (e + 1) x CTAs (acquire, bounded),
// merges from its own arena, and the launch's last CTA sets the epoch to
// e + 1.  Two parities suffice: a rank can only start epoch e + 2 after it
// has received every rank's epoch e + 1 lists, which each rank sends only
// after finishing its merge of epoch e.
#pragma once

#include "../../include/kiv_b200.h"
#include "common.cuh"

namespace kiv {

enum XType { X_COARSE = 0, X_FINE = 1, X_ATTN = 2 };
constexpr int64_t X_HDR_BYTES = 1024;

struct XArgs {
  int32_t world, rank;
  char *arena[KIV_MAX_PEERS];
  int64_t off;        // byte offset of this type's region (parity 0)
  int64_t par_bytes;  // bytes of one parity of the region
};

// byte offsets of the three regions and the arena size for per-rank payloads
// (bytes of one rank's lists) cb, fb, ab
struct XLayout {
  int64_t off[3], par[3], total;
};
__host__ __device__ inline XLayout x_layout(int64_t cb, int64_t fb, int64_t ab, int world) {
  XLayout L;
  const int64_t pay[3] = {cb, fb, ab};
  int64_t o = X_HDR_BYTES;
  for (int t = 0; t < 3; ++t) {
    L.par[t] = (pay[t] * world + 255) / 256 * 256;
    L.off[t] = o;
    o += 2 * L.par[t];
  }
  L.total = o;
  return L;
}

__device__ __forceinline__ unsigned long long *x_word(char *arena, int t, int i) {
  return reinterpret_cast<unsigned long long *>(arena) + t * 16 + i;
}
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long *p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_sys_add(unsigned long long *p, unsigned long long v) {
  asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long x_epoch(const XArgs &x, int t) {
  return *reinterpret_cast<volatile unsigned long long *>(x_word(x.arena[x.rank], t, 0));
}
// region (parity of epoch e) of rank d's arena
__device__ __forceinline__ char *x_region(const XArgs &x, int d, unsigned long long e) {
  return x.arena[d] + x.off + (int64_t)(e & 1ull) * x.par_bytes;
}
// after this CTA's stores into the arenas: count the CTA in every arena
__device__ __forceinline__ void x_signal(const XArgs &x, int t) {
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0)
    for (int d = 0; d < x.world; ++d) red_release_sys_add(x_word(x.arena[d], t, 8 + x.rank), 1ull);
}
// wait until every rank has counted `target` CTAs in this rank's arena;
// false after a bounded wait without it
__device__ __forceinline__ bool x_wait(const XArgs &x, int t, unsigned long long target) {
  __shared__ int s_ok;
  if (threadIdx.x == 0) s_ok = 1;
  __syncthreads();
  if ((int)threadIdx.x < x.world) {
    const unsigned long long *f = x_word(x.arena[x.rank], t, 8 + threadIdx.x);
    if (ld_acquire_sys(f) < target) {
      const long long t0 = clock64();
      while (ld_acquire_sys(f) < target) {
        if (clock64() - t0 > (1ll << 31)) {
          s_ok = 0;
          break;
        }
        __nanosleep(32);
      }
    }
  }
  __syncthreads();
  __threadfence();
  return s_ok != 0;
}
// the launch's last CTA moves the epoch of type t past e
__device__ __forceinline__ void x_advance(const XArgs &x, int t, unsigned long long e) {
  if (last_block(x_word(x.arena[x.rank], t, 1), gridDim.x) && threadIdx.x == 0)
    *reinterpret_cast<volatile unsigned long long *>(x_word(x.arena[x.rank], t, 0)) = e + 1;
}

}  // namespace kiv
