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

template <int BLOCK>
struct SelectSmem {
  uint32_t hist[3][SEL_BINS];   // rotating; with a cluster only rank 0's are used
  uint32_t cnt[2];          // this CTA's (gt, eq) counts
  uint32_t bin;             // chosen bin of the current pass
  uint32_t above;           // keys strictly above the chosen bin
  typename cub::BlockScan<uint32_t, BLOCK>::TempStorage scan;
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

// warp-aggregated shared-memory histogram increment (h may be another
// cluster CTA's shared memory)
__device__ __forceinline__ void hist_add(uint32_t *h, uint32_t bin) {
  const unsigned act = __activemask();
  const unsigned peers = __match_any_sync(act, bin);
  const int leader = __ffs(peers) - 1;
  if ((int)(threadIdx.x & 31) == leader) atomicAdd(&h[bin], (uint32_t)__popc(peers));
}

// Find the threshold key T of the k largest keys among all CTAs of the
// cluster (k >= 1 and k <= total keys).  Every CTA returns the same T and
// need_eq.  `keys` may point to shared or global memory.  With a cluster,
// every CTA adds its counts into rank 0's histogram (shared::cluster
// atomics, warp-aggregated); the three histograms rotate so that each pass
// needs a single cluster barrier.
template <int BLOCK, int CL>
__device__ void radix_threshold(const uint32_t *keys, int n_local, uint32_t k, SelectSmem<BLOCK> &sm,
                                uint32_t &T, uint32_t &need_eq, const uint32_t *pre0 = nullptr) {
  constexpr int IPT = SEL_BINS / BLOCK;
  uint32_t prefix = 0, pmask = 0, remaining = k;
  const int shifts[3] = {21, 10, 0};
  const bool leader = cl_rank<CL>() == 0;
  if (leader || CL == 1) {
    for (int i = threadIdx.x; i < 3 * SEL_BINS; i += BLOCK) (&sm.hist[0][0])[i] = 0;
  }
  cl_sync<CL>();
#pragma unroll 1
  for (int pass = 0; pass < 3; ++pass) {
    const uint32_t *h = cl_map<CL>(sm.hist[pass], 0);
    const int sh = shifts[pass];
    if (pass == 0 && pre0 != nullptr) {
      h = pre0;   // the producer of the keys already built the first histogram
    } else {
      for (int i = threadIdx.x; i < n_local; i += BLOCK) {
        const uint32_t key = keys[i];
        if ((key & pmask) == prefix) hist_add(cl_map<CL>(sm.hist[pass], 0), (key >> sh) & (SEL_BINS - 1));
      }
      cl_sync<CL>();
    }
    // totals, in descending bin order: item j of thread t is bin (SEL_BINS-1) - (t*IPT + j)
    uint32_t items[IPT];
#pragma unroll
    for (int j = 0; j < IPT; ++j)
      items[j] = (pass == 0 && pre0 != nullptr) ? __ldcg(h + SEL_BINS - 1 - (threadIdx.x * IPT + j))
                                                : h[SEL_BINS - 1 - (threadIdx.x * IPT + j)];
    uint32_t incl[IPT];
    cub::BlockScan<uint32_t, BLOCK>(sm.scan).InclusiveSum(items, incl);
#pragma unroll
    for (int j = 0; j < IPT; ++j) {
      const int bin = SEL_BINS - 1 - (threadIdx.x * IPT + j);
      const uint32_t above = incl[j] - items[j];   // keys in bins > bin
      if (above < remaining && incl[j] >= remaining) {
        sm.bin = (uint32_t)bin;
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
// cluster index order) in ascending index order.  `emit(local_index, out_pos)`
// is called once per selected key; out_pos counts over the whole cluster.
// With take_all, every key is selected.
template <int BLOCK, int CL, typename Emit>
__device__ void ordered_emit(const uint32_t *keys, int n_local, uint32_t T, uint32_t need_eq,
                             bool take_all, SelectSmem<BLOCK> &sm, Emit emit) {
  using Scan = cub::BlockScan<uint32_t, BLOCK>;
  const int seg = (n_local + BLOCK - 1) / BLOCK;
  const int lo = min(n_local, (int)threadIdx.x * seg);
  const int hi = min(n_local, lo + seg);
  uint32_t gt = 0, eq = 0;
  for (int i = lo; i < hi; ++i) {
    const uint32_t key = keys[i];
    gt += (take_all || key > T) ? 1u : 0u;
    eq += (!take_all && key == T) ? 1u : 0u;
  }
  uint32_t eq_before_thread, gt_before_thread, cta_gt, cta_eq;
  Scan(sm.scan).ExclusiveSum(eq, eq_before_thread, cta_eq);
  __syncthreads();
  Scan(sm.scan).ExclusiveSum(gt, gt_before_thread, cta_gt);
  if (threadIdx.x == 0) {
    sm.cnt[0] = cta_gt;
    sm.cnt[1] = cta_eq;
  }
  cl_sync<CL>();
  // ranks before mine in the cluster
  const int me = cl_rank<CL>();
  uint32_t eq_before_cta = 0, out_before_cta = 0;
  for (int r = 0; r < me; ++r) {
    const uint32_t *c = cl_map<CL>(sm.cnt, r);
    const uint32_t g = c[0], e = c[1];
    const uint32_t take = (need_eq > eq_before_cta) ? min(e, need_eq - eq_before_cta) : 0u;
    out_before_cta += g + take;
    eq_before_cta += e;
  }
  // selected count of this thread's segment
  uint32_t eq_rank = eq_before_cta + eq_before_thread;
  uint32_t mine = 0;
  {
    uint32_t er = eq_rank;
    for (int i = lo; i < hi; ++i) {
      const uint32_t key = keys[i];
      if (take_all || key > T) {
        ++mine;
      } else if (key == T) {
        if (er < need_eq) ++mine;
        ++er;
      }
    }
  }
  uint32_t out_before_thread;
  __syncthreads();
  Scan(sm.scan).ExclusiveSum(mine, out_before_thread);
  uint32_t pos = out_before_cta + out_before_thread;
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
