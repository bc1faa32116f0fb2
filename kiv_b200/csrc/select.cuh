// Exact top-k selection over 32-bit order-preserving keys.
//
// The k largest keys are found with three 11-bit radix passes (bits 31..21,
// 20..10, 10..0): each pass builds a histogram of the keys that still match
// the known prefix, and the bin holding the k-th largest key extends the
// prefix.  After the passes the threshold key T and the number `need_eq` of
// keys equal to T that belong to the top-k are known; the selected set is
// then every key > T plus the first `need_eq` keys == T in index order.  This
// is the total order (score descending, index ascending) the oracle uses.
//
// The keys of one selection may be spread over the CTAs of a thread-block
// cluster (each CTA owns a contiguous index range, in cluster-rank order);
// histograms and counts are combined through distributed shared memory.
#pragma once

#include <cooperative_groups.h>
#include <cub/block/block_scan.cuh>

#include "common.cuh"

namespace kiv {

namespace cg = cooperative_groups;

constexpr int SEL_BINS = 2048;

constexpr int SEL_MAX_CL = 16;

template <int BLOCK>
struct SelectSmem {
  uint32_t hist[2][SEL_BINS];   // local histograms, double-buffered across passes
  uint64_t cnt;                 // this CTA's packed (gt << 32 | eq) counts
  uint64_t rank_cnt[SEL_MAX_CL];
  uint32_t bin;                 // chosen bin of the current pass
  uint32_t above;               // keys strictly above the chosen bin
  union {
    typename cub::BlockScan<uint32_t, BLOCK>::TempStorage scan32;
    typename cub::BlockScan<unsigned long long, BLOCK>::TempStorage scan64;
  };
};

template <int CL>
__device__ __forceinline__ void cl_sync() {
  if constexpr (CL > 1) {
    cg::this_cluster().sync();
  } else {
    __syncthreads();
  }
}

template <int CL, typename P>
__device__ __forceinline__ P *cl_map(P *p, int rank) {
  if constexpr (CL > 1) {
    return cg::this_cluster().map_shared_rank(p, rank);
  } else {
    return p;
  }
}

template <int CL>
__device__ __forceinline__ int cl_rank() {
  if constexpr (CL > 1) {
    return (int)cg::this_cluster().block_rank();
  } else {
    return 0;
  }
}

// warp-aggregated histogram increment (shared or global memory).  Lanes are
// grouped by target address, so lanes may update different histograms.
__device__ __forceinline__ void hist_add(uint32_t *h, uint32_t bin) {
  const unsigned act = __activemask();
  const unsigned peers = __match_any_sync(act, reinterpret_cast<unsigned long long>(h + bin));
  const int leader = __ffs(peers) - 1;
  if ((int)(threadIdx.x & 31) == leader) atomicAdd(&h[bin], (uint32_t)__popc(peers));
}

// Find the threshold key T of the k largest keys among all CTAs of the
// cluster (1 <= k <= total keys); every CTA returns the same T and need_eq.
// `keys` may point to shared or global memory.  pre0, when given, is the
// histogram of (key >> 21) over all keys of the selection (global memory),
// built by the kernel that produced the keys; it replaces the first pass.
// Later passes count only keys matching the known prefix -- a small set --
// into this CTA's histogram; every CTA then reads the histograms of all
// cluster ranks (one cluster barrier per pass).
template <int BLOCK, int CL>
__device__ void radix_threshold(const uint32_t *keys, int n_local, uint32_t k, SelectSmem<BLOCK> &sm,
                                uint32_t &T, uint32_t &need_eq, const uint32_t *pre0 = nullptr) {
  static_assert(SEL_BINS % BLOCK == 0 || BLOCK % SEL_BINS == 0, "block size");
  constexpr int IPT = SEL_BINS >= BLOCK ? SEL_BINS / BLOCK : 1;
  uint32_t prefix = 0, pmask = 0, remaining = k;
  const int shifts[3] = {21, 10, 0};
#pragma unroll 1
  for (int pass = 0; pass < 3; ++pass) {
    const int sh = shifts[pass];
    const bool from_pre = pass == 0 && pre0 != nullptr;
    uint32_t *h = sm.hist[pass & 1];
    if (!from_pre) {
      for (int i = threadIdx.x; i < SEL_BINS; i += BLOCK) h[i] = 0;
      __syncthreads();
      for (int i = threadIdx.x; i < n_local; i += BLOCK) {
        const uint32_t key = keys[i];
        if ((key & pmask) == prefix) {
          const uint32_t bin = (key >> sh) & (SEL_BINS - 1);
          if (pass == 0) hist_add(h, bin);      // every key: aggregate within the warp
          else atomicAdd(&h[bin], 1u);           // few keys, spread bins
        }
      }
      cl_sync<CL>();
    }
    // totals in descending bin order: item j of thread t is bin (SEL_BINS-1) - (t*IPT + j)
    uint32_t items[IPT];
#pragma unroll
    for (int j = 0; j < IPT; ++j) {
      const int idx = threadIdx.x * IPT + j;
      uint32_t t = 0;
      if (idx < SEL_BINS) {
        const int bin = SEL_BINS - 1 - idx;
        if (from_pre) {
          t = __ldcg(pre0 + bin);
        } else {
#pragma unroll
          for (int r = 0; r < CL; ++r) t += cl_map<CL>(h, r)[bin];
        }
      }
      items[j] = t;
    }
    uint32_t incl[IPT];
    cub::BlockScan<uint32_t, BLOCK>(sm.scan32).InclusiveSum(items, incl);
#pragma unroll
    for (int j = 0; j < IPT; ++j) {
      const int idx = threadIdx.x * IPT + j;
      const uint32_t above = incl[j] - items[j];   // keys in bins above this one
      if (idx < SEL_BINS && above < remaining && incl[j] >= remaining) {
        sm.bin = (uint32_t)(SEL_BINS - 1 - idx);
        sm.above = above;
      }
    }
    __syncthreads();
    const uint32_t bin = sm.bin;
    remaining -= sm.above;
    prefix |= bin << sh;
    pmask |= (uint32_t)(SEL_BINS - 1) << sh;
    __syncthreads();
  }
  T = prefix;
  need_eq = remaining;
}

// Emit the selected keys (key > T, plus the first need_eq keys == T in
// cluster index order) in ascending index order.  emit(local_index, out_pos)
// is called once per selected key; out_pos counts over the whole cluster.
// With take_all, every key is selected.  Each thread owns a contiguous
// segment; one 64-bit block scan gives both counts before the thread, and the
// CTAs exchange their totals in one cluster round trip.
template <int BLOCK, int CL, typename Emit>
__device__ void ordered_emit(const uint32_t *keys, int n_local, uint32_t T, uint32_t need_eq,
                             bool take_all, SelectSmem<BLOCK> &sm, Emit emit) {
  using Scan = cub::BlockScan<unsigned long long, BLOCK>;
  const int seg = (n_local + BLOCK - 1) / BLOCK;
  const int lo = min(n_local, (int)threadIdx.x * seg);
  const int hi = min(n_local, lo + seg);
  uint32_t gt = 0, eq = 0;
  for (int i = lo; i < hi; ++i) {
    const uint32_t key = keys[i];
    gt += (take_all || key > T) ? 1u : 0u;
    eq += (!take_all && key == T) ? 1u : 0u;
  }
  unsigned long long before, total;
  Scan(sm.scan64).ExclusiveSum(((unsigned long long)gt << 32) | eq, before, total);
  if (threadIdx.x == 0) sm.cnt = total;
  cl_sync<CL>();
  const int me = cl_rank<CL>();
  if ((int)threadIdx.x < CL) sm.rank_cnt[threadIdx.x] = *cl_map<CL>(&sm.cnt, (int)threadIdx.x);
  __syncthreads();
  uint32_t eq_before_cta = 0, out_before_cta = 0;
  for (int r = 0; r < me; ++r) {
    const uint32_t g = (uint32_t)(sm.rank_cnt[r] >> 32), e = (uint32_t)sm.rank_cnt[r];
    const uint32_t take = need_eq > eq_before_cta ? min(e, need_eq - eq_before_cta) : 0u;
    out_before_cta += g + take;
    eq_before_cta += e;
  }
  const uint32_t gt_before = (uint32_t)(before >> 32), eq_before = (uint32_t)before;
  const uint32_t room = need_eq > eq_before_cta ? need_eq - eq_before_cta : 0u;
  uint32_t pos = out_before_cta + gt_before + min(eq_before, room);
  uint32_t eq_rank = eq_before_cta + eq_before;
  for (int i = lo; i < hi; ++i) {
    const uint32_t key = keys[i];
    bool s = false;
    if (take_all || key > T) {
      s = true;
    } else if (key == T) {
      s = eq_rank < need_eq;
      ++eq_rank;
    }
    if (s) emit(i, pos++);
  }
  // no CTA may leave while others still read its shared memory
  cl_sync<CL>();
}

// Largest key and float sum of keys[0, n) of this CTA, added into two state
// words (atomicMax on the key, atomicAdd on a double).
template <int BLOCK>
__device__ void block_stats(const uint32_t *keys, int n, int64_t *max_word, int64_t *sum_word) {
  __shared__ uint32_t wmax[BLOCK / 32];
  __shared__ float wsum[BLOCK / 32];
  uint32_t mk = 0;
  float sm = 0.f;
  for (int i = threadIdx.x; i < n; i += BLOCK) {
    const uint32_t k = keys[i];
    mk = k > mk ? k : mk;
    sm += key2f(k);
  }
  mk = __reduce_max_sync(KIV_FULL_MASK, mk);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sm += __shfl_xor_sync(KIV_FULL_MASK, sm, o);
  if ((threadIdx.x & 31) == 0) {
    wmax[threadIdx.x >> 5] = mk;
    wsum[threadIdx.x >> 5] = sm;
  }
  __syncthreads();
  if (threadIdx.x == 0 && n > 0) {
    uint32_t m = 0;
    double t = 0.0;
    for (int w = 0; w < BLOCK / 32; ++w) {
      m = wmax[w] > m ? wmax[w] : m;
      t += wsum[w];
    }
    atomicMax(reinterpret_cast<unsigned long long *>(max_word), (unsigned long long)m);
    atomicAdd(reinterpret_cast<double *>(sum_word), t);
  }
  __syncthreads();
}

// Compact the set flags of flags[0, n) into out (ascending), zero the flags,
// and return the count (valid in thread 0).  Local index i maps to global id
// i * stride + offset.  Single CTA.
template <int BLOCK>
__device__ int64_t compact_flags(uint8_t *flags, int64_t n, int32_t *out, int64_t cap, int stride,
                                 int offset, typename cub::BlockScan<uint32_t, BLOCK>::TempStorage &tmp) {
  using Scan = cub::BlockScan<uint32_t, BLOCK>;
  constexpr int IPT = 4;
  int64_t base = 0;
  for (int64_t t0 = 0; t0 < n; t0 += (int64_t)BLOCK * IPT) {
    uint32_t f[IPT], c = 0;
#pragma unroll
    for (int j = 0; j < IPT; ++j) {
      const int64_t i = t0 + (int64_t)threadIdx.x * IPT + j;
      f[j] = (i < n) ? (uint32_t)__ldcg(reinterpret_cast<const unsigned char *>(flags + i)) : 0u;
      c += f[j] ? 1u : 0u;
    }
    uint32_t before, total;
    Scan(tmp).ExclusiveSum(c, before, total);
    int64_t pos = base + before;
#pragma unroll
    for (int j = 0; j < IPT; ++j) {
      const int64_t i = t0 + (int64_t)threadIdx.x * IPT + j;
      if (f[j]) {
        if (pos < cap) out[pos] = (int32_t)(i * stride + offset);
        ++pos;
        flags[i] = 0;
      }
    }
    base += total;
    __syncthreads();
  }
  return base < cap ? base : cap;
}

}  // namespace kiv
