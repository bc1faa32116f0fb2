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
#include <cub/block/block_reduce.cuh>
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

// ---------------------------------------------------------------------------
// Candidate-set selection.  Given the first-pass histogram of all keys (bins
// of key >> 21), the threshold bin b0 and the count above it are known; only
// keys in bins >= b0 can be selected.  Those are compacted (in index order)
// into shared memory, one more histogram pass over the bin-b0 keys finds the
// bin b1 of bits 20..10, and the few keys of the boundary bin (b0, b1) are
// ranked exactly by comparison (score desc, index asc).
//
// Tiles are warp-contiguous: warp w of the CTA owns the 32 * CS_KEYS
// consecutive indices starting at tile + w * 32 * CS_KEYS, and its step j
// reads 32 consecutive keys (one per lane), so global loads are coalesced and
// shared-memory reads conflict-free; ballots give the in-warp order.
// ---------------------------------------------------------------------------
constexpr int CS_KEYS = 16;   // keys per lane per tile

template <int BLOCK>
struct CandSmem {
  uint32_t hist[SEL_BINS];
  uint32_t bin, above;
  int cnt[SEL_MAX_CL];
  int wcnt[BLOCK / 32];
  int total;
  union {
    typename cub::BlockScan<uint32_t, BLOCK>::TempStorage scan32;
    typename cub::BlockReduce<uint32_t, BLOCK>::TempStorage red;
  };
};

// Exclusive prefix over the warps of the per-warp counts `cnt` (same value
// in every lane): returns the count before this warp, *total the CTA total.
// Ends with a barrier after which sm.wcnt may be reused.
template <int BLOCK>
__device__ __forceinline__ int warp_prefix(int cnt, int *total, CandSmem<BLOCK> &sm) {
  const int warp = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) sm.wcnt[warp] = cnt;
  __syncthreads();
  int before = 0, all = 0;
#pragma unroll
  for (int w = 0; w < BLOCK / 32; ++w) {
    const int c = sm.wcnt[w];
    before += w < warp ? c : 0;
    all += c;
  }
  __syncthreads();
  *total = all;
  return before;
}

// Find the bin of the k-th largest count of a descending-order histogram:
// sets sm.bin and sm.above (count strictly above).  `load(bin)` gives counts.
// If the counts sum to less than k, bin 0 with above 0 is returned.
template <int BLOCK, typename Load>
__device__ void find_bin(uint32_t k, CandSmem<BLOCK> &sm, Load load) {
  constexpr int IPT = SEL_BINS / BLOCK;
  uint32_t items[IPT], incl[IPT];
#pragma unroll
  for (int j = 0; j < IPT; ++j) items[j] = load(SEL_BINS - 1 - (threadIdx.x * IPT + j));
  if (threadIdx.x == 0) {
    sm.bin = 0;
    sm.above = 0;
  }
  cub::BlockScan<uint32_t, BLOCK>(sm.scan32).InclusiveSum(items, incl);
#pragma unroll
  for (int j = 0; j < IPT; ++j) {
    const uint32_t above = incl[j] - items[j];
    if (above < k && incl[j] >= k) {
      sm.bin = (uint32_t)(SEL_BINS - 1 - (threadIdx.x * IPT + j));
      sm.above = above;
    }
  }
  __syncthreads();
}

// Ordered compaction: out[..] = (key, index) of the keys i in [0, n) with
// pred(key) true, in index order, starting at out position `base`; keys are
// read with get(i).  Returns the count (may exceed cap; writes stop at cap).
template <int BLOCK, typename Get, typename Pred>
__device__ int ordered_compact(int n, Get get, Pred pred, uint32_t *okey, int32_t *oidx, int base, int cap,
                               CandSmem<BLOCK> &sm) {
  constexpr int WT = 32 * CS_KEYS;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const unsigned below = (1u << lane) - 1u;
  int total = 0;
  for (int t0 = 0; t0 < n; t0 += BLOCK * CS_KEYS) {
    const int wb = t0 + warp * WT + lane;
    uint32_t k[CS_KEYS];
    unsigned m[CS_KEYS];
    int cnt = 0;
#pragma unroll
    for (int j = 0; j < CS_KEYS; ++j) k[j] = wb + j * 32 < n ? get(wb + j * 32) : 0u;
#pragma unroll
    for (int j = 0; j < CS_KEYS; ++j) {
      m[j] = __ballot_sync(KIV_FULL_MASK, wb + j * 32 < n && pred(k[j]));
      cnt += __popc(m[j]);
    }
    int tile_total;
    int pos = base + total + warp_prefix<BLOCK>(cnt, &tile_total, sm);
#pragma unroll
    for (int j = 0; j < CS_KEYS; ++j) {
      const int p = pos + __popc(m[j] & below);
      if (((m[j] >> lane) & 1u) && p < cap) {
        okey[p] = k[j];
        oidx[p] = wb + j * 32;
      }
      pos += __popc(m[j]);
    }
    total += tile_total;
  }
  return total;
}

// Calls emit(i, pos) for every i in [0, n) with pred(i) true, where pos is
// the rank of i among them in index order; returns their count.  Each warp
// owns a contiguous segment, walked 32 indices at a time (two passes: count,
// then place); compact code for shared-memory sources.
template <int BLOCK, typename Pred, typename Emit>
__device__ int ordered_emit_pred(int n, Pred pred, Emit emit, CandSmem<BLOCK> &sm) {
  constexpr int NW = BLOCK / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const unsigned below = (1u << lane) - 1u;
  const int seg = ((n + NW - 1) / NW + 31) & ~31;
  const int lo = min(n, warp * seg), hi = min(n, lo + seg);
  int cnt = 0;
#pragma unroll 1
  for (int i0 = lo; i0 < hi; i0 += 32) {
    const int i = i0 + lane;
    cnt += __popc(__ballot_sync(KIV_FULL_MASK, i < hi && pred(i)));
  }
  int total;
  int pos = warp_prefix<BLOCK>(cnt, &total, sm);
#pragma unroll 1
  for (int i0 = lo; i0 < hi; i0 += 32) {
    const int i = i0 + lane;
    const bool p = i < hi && pred(i);
    const unsigned m = __ballot_sync(KIV_FULL_MASK, p);
    if (p) emit(i, (uint32_t)(pos + __popc(m & below)));
    pos += __popc(m);
  }
  return total;
}

// Select from candidates ck[0, n) (index order, every key in a bin >= b0):
// all keys in bins > b0, plus the top need0 keys of bin b0.  Calls
// emit(candidate index, output position) in index order.  bnd_key / bnd_idx
// are scratch for the boundary bin (capacity bnd_cap), flag is n bytes of
// scratch (ck and flag in shared memory).  Falls back to the general radix
// threshold when the boundary bin is larger than bnd_cap.
template <int BLOCK, typename Emit>
__device__ void select_candidates(const uint32_t *ck, int n, uint32_t b0, uint32_t need0, uint32_t *bnd_key,
                                  int32_t *bnd_idx, uint8_t *flag, int bnd_cap, CandSmem<BLOCK> &sm,
                                  SelectSmem<BLOCK> &rs, Emit emit) {
  // pass 1 over the bin-b0 keys: bits 20..10
  for (int i = threadIdx.x; i < SEL_BINS; i += BLOCK) sm.hist[i] = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += BLOCK) {
    const uint32_t key = ck[i];
    flag[i] = 0;
    if ((key >> 21) == b0) atomicAdd(&sm.hist[(key >> 10) & (SEL_BINS - 1)], 1u);
  }
  __syncthreads();
  find_bin<BLOCK>(need0, sm, [&](int b) { return sm.hist[b]; });
  const uint32_t b1 = sm.bin;
  const uint32_t need1 = need0 - sm.above;
  const uint32_t bkey = (b0 << 11) | b1;          // key >> 10 of the boundary bin
  const uint32_t count1 = sm.hist[b1];
  __syncthreads();
  if ((int)count1 <= bnd_cap) {
    // boundary-bin keys (any order), ranked by comparison in the total order
    // (key descending, index ascending)
    if (threadIdx.x == 0) sm.total = 0;
    __syncthreads();
#pragma unroll 1
    for (int i = threadIdx.x; i < n; i += BLOCK) {
      const uint32_t key = ck[i];
      if ((key >> 10) == bkey) {
        const int slot = atomicAdd(&sm.total, 1);
        bnd_key[slot] = key;
        bnd_idx[slot] = i;
      }
    }
    __syncthreads();
    const int nb = sm.total;
#pragma unroll 1
    for (int i = threadIdx.x; i < nb; i += BLOCK) {
      const uint32_t ki = bnd_key[i];
      const int xi = bnd_idx[i];
      uint32_t rank = 0;
#pragma unroll 4
      for (int j = 0; j < nb; ++j) {
        const uint32_t kj = bnd_key[j];
        rank += (kj > ki || (kj == ki && bnd_idx[j] < xi)) ? 1u : 0u;
      }
      if (rank < need1) flag[xi] = 1;
    }
    __syncthreads();
    // emission in index order: every key above the boundary bin, plus the
    // flagged boundary keys
    ordered_emit_pred<BLOCK>(n, [&](int i) { return (ck[i] >> 10) > bkey || flag[i] != 0; }, emit, sm);
  } else {
    // many keys share the boundary bin: exact radix threshold over the candidates
    uint32_t T = 0, need = 0;
    uint32_t above0 = 0;
    for (int i = threadIdx.x; i < n; i += BLOCK) above0 += ((ck[i] >> 21) > b0) ? 1u : 0u;
    above0 = cub::BlockReduce<uint32_t, BLOCK>(sm.red).Sum(above0);
    if (threadIdx.x == 0) sm.above = above0;
    __syncthreads();
    radix_threshold<BLOCK, 1>(ck, n, sm.above + need0, rs, T, need);
    ordered_emit<BLOCK, 1>(ck, n, T, need, false, rs, emit);
  }
}

// Exclusive prefix sum of v over the CTA (compact code: warp shuffles plus
// one pass over the warp totals); *total gets the CTA sum.  wsum holds
// BLOCK / 32 ints of shared scratch.  Contains two barriers.
template <int BLOCK>
__device__ __forceinline__ int block_excl_sum(int v, int *total, int *wsum) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll 1
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(KIV_FULL_MASK, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) wsum[warp] = x;
  __syncthreads();
  int before = 0, all = 0;
#pragma unroll 1
  for (int w = 0; w < BLOCK / 32; ++w) {
    const int c = wsum[w];
    before += w < warp ? c : 0;
    all += c;
  }
  __syncthreads();
  *total = all;
  return before + x - v;
}

// Marks of word wi (pages 32 wi .. 32 wi + 31) that belong to shard `rank`
// of `count` (page % count == rank).
__device__ __forceinline__ uint32_t owner_mask(int64_t wi, int rank, int count) {
  if (count <= 1) return ~0u;
  uint32_t m = 0;
  for (int j = (int)((rank - (wi * 32) % count + count) % count); j < 32; j += count) m |= 1u << j;
  return m;
}

// Sorted union of the marked pages (bit i of bits[i / 32] set = local page i,
// i < np) as global page ids (local page i -> i * nshard + rank) into
// list[0, cap); returns the count.  With fcount > 1 the bitmap indexes global
// pages (nshard = 1) and only the pages of shard frank (page % fcount ==
// frank) are kept.  bits is shared memory when SMEM, else global.  Every
// thread of the CTA calls it.  Each thread owns UB_WORDS consecutive words
// (UB_WORDS * 32 pages) per tile; the code is kept small because it runs once
// per launch on cold instruction caches.
constexpr int UB_WORDS = 2;
template <int BLOCK, bool SMEM>
__device__ int union_from_bits(const uint32_t *bits, int64_t np, int32_t *list, int cap, int rank, int nshard,
                               int *wsum, int frank = 0, int fcount = 1) {
  const int64_t nw = (np + 31) / 32;
  int base = 0;
#pragma unroll 1
  for (int64_t t0 = 0; t0 < nw; t0 += (int64_t)BLOCK * UB_WORDS) {
    const int64_t w0 = t0 + (int64_t)threadIdx.x * UB_WORDS;
    uint32_t v[UB_WORDS];
    int c = 0;
#pragma unroll
    for (int j = 0; j < UB_WORDS; ++j) {
      const int64_t wi = w0 + j;
      uint32_t x = wi < nw ? (SMEM ? bits[wi] : __ldcg(bits + wi)) : 0u;
      const int64_t valid = np - wi * 32;            // pages of this word below np
      if (valid < 32) x &= valid > 0 ? (1u << valid) - 1u : 0u;
      if (fcount > 1) x &= owner_mask(wi, frank, fcount);
      v[j] = x;
      c += __popc(x);
    }
    int total;
    int pos = base + block_excl_sum<BLOCK>(c, &total, wsum);
#pragma unroll
    for (int j = 0; j < UB_WORDS; ++j) {
      uint32_t x = v[j];
#pragma unroll 1
      while (x) {
        const int bit = __ffs(x) - 1;
        if (pos < cap) list[pos] = (int32_t)(((w0 + j) * 32 + bit) * nshard + rank);
        ++pos;
        x &= x - 1;
      }
    }
    base += total;
  }
  __syncthreads();
  return base < cap ? base : cap;
}

// Positions g < n (ascending) of the pages list[g] that belong to shard
// `rank` of `count`, into out; returns their number.  Every thread of the CTA
// calls it; ends with a barrier.
template <int BLOCK>
__device__ int owned_positions(const int32_t *list, int n, int32_t *out, int rank, int count, int *wsum) {
  constexpr int IPT = 4;
  int base = 0;
#pragma unroll 1
  for (int t0 = 0; t0 < n; t0 += BLOCK * IPT) {
    const int i0 = t0 + threadIdx.x * IPT;
    bool f[IPT];
    int c = 0;
#pragma unroll
    for (int j = 0; j < IPT; ++j) {
      f[j] = i0 + j < n && list[i0 + j] % count == rank;
      c += f[j] ? 1 : 0;
    }
    int total;
    int pos = base + block_excl_sum<BLOCK>(c, &total, wsum);
#pragma unroll
    for (int j = 0; j < IPT; ++j)
      if (f[j]) out[pos++] = i0 + j;
    base += total;
  }
  __syncthreads();
  return base;
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

}  // namespace kiv
