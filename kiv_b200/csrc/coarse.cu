// Kernel (b): coarse page scoring fused with the per-row top-`top_pages`
// select and the page union.
//
// Reference behaviour restated (kiv/cold_store.py:203-230):
//   s[b,h,q,p] = scaling * <q[b,h,q], summary[b, h // G, p]>
//   per (b,h,q): the min(top_pages, Np) best pages; union over b, h, q, sorted.
// The reference materializes repeat_kv(summaries) (G copies) and runs a
// GEMM; here each summary row is read once per KV head and scored against all
// G*Q query rows of that head in registers.  Scores are written as 32-bit
// order-preserving keys for the radix select.
#include <algorithm>

#include "common.cuh"
#include "internal.h"
#include "exchange.cuh"
#include "select.cuh"

namespace kiv {

constexpr int CS_THREADS = 128;      // coarse scoring
constexpr int CS_PAGES = 16;         // pages per work item (one bulk copy)
constexpr int TK_THREADS = 512;      // per-row top-k
constexpr int TK_BND = 1024;         // boundary-bin capacity of the candidate select
constexpr int TK_SCAP = 16384;       // scores of a row staged in shared memory
constexpr int CM_THREADS = 256;      // merge of gathered per-row lists
constexpr int CM_RANK_MAX = 1024;   // merge by direct ranking up to this many entries
constexpr int UN_THREADS = 1024;     // page union from the page marks

// local finalized pages of this shard given the global finalized count
__device__ __forceinline__ int64_t local_pages(int64_t np_global, int rank, int n) {
  return np_global > rank ? (np_global - rank + n - 1) / n : 0;
}

template <typename T, int LPR, int VPL, int RCH>
__global__ void __launch_bounds__(CS_THREADS)
coarse_scores_kernel(kiv_store st, kiv_query q, Workspace w) {
  griddep_wait();
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    st.state[KIV_ST_COARSE_MAX] = 0;
    st.state[KIV_ST_COARSE_SUM] = 0;
  }
  extern __shared__ __align__(128) uint8_t cs_smem[];
  __shared__ uint64_t bar;
  __shared__ int s_fail;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane % LPR;                    // lane within its row group
  const int grp = lane / LPR;                  // row group within the warp
  constexpr int GPW = 32 / LPR;                // row groups per warp
  constexpr int NW = CS_THREADS / 32;
  const int D = st.head_dim, H = st.num_kv_heads, S = st.page_size;
  const int nv = D / Elem<T>::V;
  const int G = q.num_query_heads / H, Q = q.query_len;
  const int rows_kv = G * Q;
  const int nchunks = (rows_kv + RCH - 1) / RCH;
  const int64_t np_global = st_ld(st.state, KIV_ST_COLD_LEN) / S;
  const int64_t np = coarse_pages(st, np_global);
  clear_stale_marks(st, w, np);
  const int64_t nblk = (np + CS_PAGES - 1) / CS_PAGES;
  const int64_t items = (int64_t)st.batch * H * nchunks * nblk;
  const T *qb = reinterpret_cast<const T *>(q.q);
  const T *summ = reinterpret_cast<const T *>(st.summaries);
  T *tile = reinterpret_cast<T *>(cs_smem);    // [CS_PAGES][D]
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    mbar_fence_init();
    s_fail = 0;
  }
  __syncthreads();

  uint32_t kmax = 0;
  float ksum = 0.f;
  uint32_t phase = 0;
  for (int64_t it = blockIdx.x; it < items; it += gridDim.x, phase ^= 1) {
    const int64_t pb = it % nblk;
    const int64_t rest = it / nblk;
    const int ch = (int)(rest % nchunks);
    const int bh = (int)(rest / nchunks);
    const int b = bh / H, kvh = bh % H;
    const int64_t p0 = pb * CS_PAGES;
    const int npg = (int)std::min<int64_t>(CS_PAGES, np - p0);
    if (threadIdx.x == 0) {
      // one bulk copy: this block's summaries are contiguous
      const uint32_t bytes = (uint32_t)npg * D * sizeof(T);
      mbar_arrive_tx(&bar, bytes);
      bulk_g2s(tile, summ + ((int64_t)bh * w.np_cap + p0) * D, bytes, &bar);
    }
    RowDot<T, LPR, VPL, RCH> dot;
    const T *qrows[RCH];
#pragma unroll
    for (int r = 0; r < RCH; ++r) {
      const int rr = ch * RCH + r;
      if (rr < rows_kv) {
        const int h = kvh * G + rr / Q, t = rr % Q;
        qrows[r] = qb + b * q.stride_b + h * q.stride_h + t * q.stride_t;
      } else {
        qrows[r] = nullptr;
      }
    }
    dot.load_query(qrows, g, nv, 1.0f);
    if (!mbar_wait_bounded(&bar, phase)) s_fail = 1;
    __syncthreads();
    if (s_fail) break;
    for (int pi0 = 0; pi0 < npg; pi0 += NW * GPW) {
      const int pi = pi0 + warp * GPW + grp;
      const bool valid = pi < npg;
      float acc[RCH];
      dot.template partial<false>(valid ? tile + (size_t)pi * D : nullptr, g, nv, acc);
      int base = 0;
      tr_reduce<RCH, LPR / 2>(acc, lane, base);
      constexpr int NOUT = TrOut<RCH, LPR>::N;
      constexpr int REPL = TrOut<RCH, LPR>::REPL;
      if (valid && (g % REPL) == 0) {
#pragma unroll
        for (int i = 0; i < NOUT; ++i) {
          const int rr = ch * RCH + base + i;
          if (rr < rows_kv) {
            const int h = kvh * G + rr / Q, t = rr % Q;
            const int64_t R_idx = ((int64_t)b * q.num_query_heads + h) * Q + t;
            const float sc = acc[i] * q.scaling;
            w.scores[R_idx * w.np_cap + p0 + pi] = sc;
            const uint32_t key = f2key(sc);
            hist_add(w.chist + R_idx * SEL_BINS, key >> 21);
            kmax = key > kmax ? key : kmax;
            ksum += sc;
          }
        }
      }
    }
    __syncthreads();  // the tile is free for the next block
  }
  kmax = __reduce_max_sync(KIV_FULL_MASK, kmax);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ksum += __shfl_xor_sync(KIV_FULL_MASK, ksum, o);
  if (lane == 0 && kmax != 0) {
    atomicMax(reinterpret_cast<unsigned long long *>(&w.cstat[0]), (unsigned long long)kmax);
    atomicAdd(reinterpret_cast<double *>(&w.cstat[1]), (double)ksum);
  }
  if (s_fail && threadIdx.x == 0)
    atomicOr(reinterpret_cast<unsigned long long *>(st.state + KIV_ST_ERROR), (unsigned long long)KIV_ERRBIT_WAIT_TIMEOUT);
}

// Per-row top-k.  The scorer left each row's first-pass histogram (bins of
// key >> 21) in w.chist; only pages in bins at or above the threshold bin are
// compacted and resolved (select_candidates).  shard_count == 1: mark the
// selected pages in w.pbits (the fine pass builds the sorted union from
// them).  shard_count > 1: write the row's local list (score, page id) in
// page order for the all-gather.
__global__ void __launch_bounds__(TK_THREADS)
coarse_topk_kernel(kiv_store st, kiv_query q, Workspace w, float *row_scores, int32_t *row_pages, int cap,
                   int scap, int self_hist) {
  extern __shared__ uint4 dyn_smem[];
  __shared__ __align__(16) CandSmem<TK_THREADS> cs;
  __shared__ SelectSmem<TK_THREADS> rs;
  __shared__ uint64_t bar;
  __shared__ int s_fail;
  uint32_t *ckey = reinterpret_cast<uint32_t *>(dyn_smem);
  int32_t *cidx = reinterpret_cast<int32_t *>(ckey + cap);
  uint32_t *bkey = reinterpret_cast<uint32_t *>(cidx + cap);
  int32_t *bidx = reinterpret_cast<int32_t *>(bkey + TK_BND);
  int32_t *sel_ci = bidx + TK_BND;                 // [top_pages, padded to 4] chosen candidates
  float *sscore = reinterpret_cast<float *>(sel_ci + ((q.top_pages + 3) & ~3));   // [scap] staged scores
  uint8_t *flag = reinterpret_cast<uint8_t *>(sscore + scap);
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    mbar_fence_init();
    s_fail = 0;
  }
  // the cold length was published by the eviction, two kernels back
  const int S = st.page_size;
  const int64_t np_global = st_ld(st.state, KIV_ST_COLD_LEN) / S;
  const int64_t np = coarse_pages(st, np_global);
  __syncthreads();
  griddep_wait();
  const int row = blockIdx.x;
  const int K = q.top_pages;
  const int rank = st.shard_rank, nsh = st.shard_count;
  // self_hist: the scorer left no histogram (tcgen05 and prefill-shaped
  // scoring); it is built here from the staged scores
  const uint32_t *pre = self_hist ? nullptr : w.chist + (int64_t)row * SEL_BINS;
  float *src = w.scores + (int64_t)row * w.np_cap;
  float *ls = row_scores ? row_scores + (int64_t)row * K : nullptr;
  int32_t *lpg = row_pages ? row_pages + (int64_t)row * K : nullptr;
  const bool repl = repl_summaries(st);
  auto emit_page = [&](int64_t lp, uint32_t pos, uint32_t key) {
    if (nsh == 1) {
      atomicOr(&w.pbits[lp >> 5], 1u << (lp & 31));
    } else if (repl) {
      // lp is a global page; the marks index global pages (every shard holds the whole union)
      atomicOr(&w.pbits[lp >> 5], 1u << (lp & 31));
    } else if (pos < (uint32_t)K) {
      ls[pos] = key2f(key);
      lpg[pos] = (int32_t)(lp * nsh + rank);
    }
  };
  const uint32_t k = (uint32_t)(K < np ? (int64_t)K : np);
  // inputs -> shared memory in one round trip: the row's histogram and scores
  const bool staged = np > 0 && np <= scap && (reinterpret_cast<uintptr_t>(src) & 15) == 0;
  if (threadIdx.x == 0 && np > 0) {
    const uint32_t sb = staged ? (uint32_t)((np * 4 + 15) & ~15ll) : 0u;
    const uint32_t hb = pre ? SEL_BINS * 4 : 0u;
    if (hb + sb) {
      mbar_arrive_tx(&bar, hb + sb);
      if (hb) bulk_g2s(cs.hist, pre, hb, &bar);
      if (sb) bulk_g2s(sscore, src, sb, &bar);
    }
  }
  if (!pre)
    for (int i = threadIdx.x; i < SEL_BINS; i += TK_THREADS) cs.hist[i] = 0;
  if (np > 0 && (pre || staged) && !mbar_wait_bounded(&bar, 0)) s_fail = 1;
  auto score_at = [&](int64_t i) { return staged ? sscore[i] : __ldcg(src + i); };
  if (!pre && np > 0 && (int64_t)k < np) {
    __syncthreads();
    if (staged)
      for (int64_t i = threadIdx.x; i < np; i += TK_THREADS) atomicAdd(&cs.hist[f2key(sscore[i]) >> 21], 1u);
    else
      for (int64_t i = threadIdx.x; i < np; i += TK_THREADS) atomicAdd(&cs.hist[f2key(__ldcg(src + i)) >> 21], 1u);
    __syncthreads();
  }
  if (np > 0 && (int64_t)k >= np) {
    for (int64_t i = threadIdx.x; i < np; i += TK_THREADS) emit_page(i, (uint32_t)i, f2key(score_at(i)));
  } else if (np > 0) {
    find_bin<TK_THREADS>(k, cs, [&](int b) { return cs.hist[b]; });
    const uint32_t b0 = cs.bin, need0 = k - cs.above;
    __syncthreads();
    // (one instantiation per source: a load that may come from either memory
    // is issued as a generic load, slower than a shared-memory one)
    auto above_bin = [&](uint32_t key) { return (key >> 21) >= b0; };
    const int n = staged ? ordered_compact<TK_THREADS>((int)np, [&](int i) { return f2key(sscore[i]); }, above_bin,
                                                       ckey, cidx, 0, cap, cs)
                         : ordered_compact<TK_THREADS>((int)np, [&](int i) { return f2key(__ldcg(src + i)); },
                                                       above_bin, ckey, cidx, 0, cap, cs);
    if (n <= cap) {
      select_candidates<TK_THREADS>(ckey, n, b0, need0, bkey, bidx, flag, TK_BND, cs, rs,
                                    [&](int ci, uint32_t pos) {
                                      if (pos < k) sel_ci[pos] = ci;
                                    });
      __syncthreads();
      for (int p = threadIdx.x; p < (int)k; p += TK_THREADS) {
        const int ci = sel_ci[p];
        emit_page(cidx[ci], (uint32_t)p, ckey[ci]);
      }
    } else {
      // too many candidates for shared memory: exact radix select over the
      // row in global memory (keys written in place of the scores)
      uint32_t *gk = reinterpret_cast<uint32_t *>(src);
      for (int64_t i = threadIdx.x; i < np; i += TK_THREADS) gk[i] = f2key(src[i]);
      __syncthreads();
      uint32_t T = 0, need = 0;
      radix_threshold<TK_THREADS, 1>(gk, (int)np, k, rs, T, need, pre);
      ordered_emit<TK_THREADS, 1>(gk, (int)np, T, need, false, rs,
                                  [&](int i, uint32_t pos) { emit_page(i, pos, gk[i]); });
    }
  }
  if (nsh > 1 && !repl) {
    for (int j = (int)k + threadIdx.x; j < K; j += TK_THREADS) {
      ls[j] = 0.f;
      lpg[j] = -1;
    }
  }
  // this row's first-pass histogram has been used: clear it for the next pass
  __syncthreads();
  if (pre)
    for (int i = threadIdx.x; i < SEL_BINS; i += TK_THREADS) w.chist[(int64_t)row * SEL_BINS + i] = 0;
  if (row == 0 && threadIdx.x == 0) {
    if (nsh == 1 || repl) st.state[KIV_ST_UNION_PENDING] = 1;
    const unsigned long long mk = w.cstat[0], sb = w.cstat[1];
    if (mk) atomicMax(reinterpret_cast<unsigned long long *>(st.state + KIV_ST_COARSE_MAX), mk);
    atomicAdd(reinterpret_cast<double *>(st.state + KIV_ST_COARSE_SUM), __longlong_as_double((long long)sb));
    w.cstat[0] = 0;
    w.cstat[1] = 0;
  }
  if (s_fail && threadIdx.x == 0)
    atomicOr(reinterpret_cast<unsigned long long *>(st.state + KIV_ST_ERROR), (unsigned long long)KIV_ERRBIT_WAIT_TIMEOUT);
}

// Per-row top-k for prefill-shaped coarse scoring (thousands of query rows of
// a few thousand pages each): one warp per row, persistent CTAs.  Exact, with
// the same order as coarse_topk_kernel (score descending, lowest page first on
// ties): a radix select over the order-preserving keys finds the boundary --
// levels of 11, 11 and 10 bits, each a histogram in the warp's shared memory
// over the keys that match the levels so far, stopping once the boundary bin
// holds at most RT_CAND keys -- then one pass marks every key above the
// boundary and compacts the boundary keys (index order), which are ranked by
// comparison (or, when all of them are equal, taken lowest page first).
// Union marks collect in a CTA bitmap and reach w.pbits once per CTA.
constexpr int RT_THREADS = 256;
constexpr int RT_WARPS = RT_THREADS / 32;
constexpr int RT_CAND = 256;          // boundary keys resolved by ranking; also the largest top_pages
constexpr int RT_UNROLL = 16;         // independent loads in flight per lane
constexpr int RT_HWORDS = SEL_BINS + SEL_BINS / 64;   // histogram with one pad word per 64 bins
// bin -> word: lane l scans bins [64 l, 64 l + 64) of the 2048, which start 65 words apart
__device__ __forceinline__ int rt_hidx(int bin) { return bin + (bin >> 6); }

__global__ void __launch_bounds__(RT_THREADS)
coarse_rows_topk_kernel(kiv_store st, kiv_query q, Workspace w, float *row_scores, int32_t *row_pages,
                        int nwords) {
  extern __shared__ uint32_t rt_smem[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t *hist = rt_smem + warp * RT_HWORDS;
  uint32_t *ckey = rt_smem + RT_WARPS * RT_HWORDS + warp * RT_CAND;
  int32_t *cidx = reinterpret_cast<int32_t *>(rt_smem + RT_WARPS * (RT_HWORDS + RT_CAND)) + warp * RT_CAND;
  uint8_t *cflag = reinterpret_cast<uint8_t *>(rt_smem + RT_WARPS * (RT_HWORDS + 2 * RT_CAND)) + warp * RT_CAND;
  uint32_t *bits = rt_smem + RT_WARPS * (RT_HWORDS + 2 * RT_CAND) + RT_WARPS * RT_CAND / 4;   // [nwords]
  for (int i = threadIdx.x; i < nwords; i += RT_THREADS) bits[i] = 0;
  const int S = st.page_size;
  const int nsh = st.shard_count, rank = st.shard_rank;
  griddep_wait();
  const int64_t np_global = st_ld(st.state, KIV_ST_COLD_LEN) / S;
  const int64_t np = coarse_pages(st, np_global);
  const bool repl = repl_summaries(st);
  const bool marks = nsh == 1 || repl;
  const int K = q.top_pages;
  const uint32_t k = (uint32_t)(K < np ? (int64_t)K : np);
  const unsigned lt = (1u << lane) - 1u;
  __syncthreads();
  // i: a local page, or a global one with replicated summaries (marks index global pages)
  auto mark = [&](int64_t i) {
    if (nwords > 0) atomicOr(&bits[i >> 5], 1u << (i & 31));
    else atomicOr(&w.pbits[i >> 5], 1u << (i & 31));
  };
  for (int64_t row = (int64_t)blockIdx.x * RT_WARPS + warp; row < w.R; row += (int64_t)gridDim.x * RT_WARPS) {
    const float *src = w.scores + row * w.np_cap;
    float *ls = row_scores ? row_scores + row * K : nullptr;
    int32_t *lpg = row_pages ? row_pages + row * K : nullptr;
    uint32_t prefix = 0, mask = 0, remaining = k;
    bool all = (int64_t)k >= np;
    if (!all) {
#pragma unroll 1
      for (int level = 0; level < 3; ++level) {
        const int sh = level == 0 ? 21 : (level == 1 ? 10 : 0);
        const int nbins = level == 2 ? 1024 : 2048;
        for (int i = lane; i < RT_HWORDS; i += 32) hist[i] = 0;
        __syncwarp();
        for (int64_t base = 0; base < np; base += 32 * RT_UNROLL) {
          float v[RT_UNROLL];
#pragma unroll
          for (int x = 0; x < RT_UNROLL; ++x) {
            const int64_t i = base + x * 32 + lane;
            v[x] = i < np ? __ldcg(src + i) : 0.f;
          }
#pragma unroll
          for (int x = 0; x < RT_UNROLL; ++x) {
            const uint32_t key = f2key(v[x]);
            if (base + x * 32 + lane < np && (key & mask) == prefix) atomicAdd(&hist[rt_hidx((key >> sh) & (nbins - 1))], 1u);
          }
        }
        __syncwarp();
        // boundary bin: lane l owns bins [hi - per + 1, hi], lane 0 the highest
        const int per = nbins / 32;
        const int hi = nbins - 1 - lane * per;
        uint32_t tot = 0;
        for (int x = 0; x < per; ++x) tot += hist[rt_hidx(hi - x)];
        uint32_t incl = tot;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const uint32_t y = __shfl_up_sync(KIV_FULL_MASK, incl, o);
          if (lane >= o) incl += y;
        }
        const uint32_t excl = incl - tot;
        const unsigned own = __ballot_sync(KIV_FULL_MASK, excl < remaining && incl >= remaining);
        const int sl = own ? __ffs(own) - 1 : 0;
        int bin = 0;
        uint32_t above = 0, cnt = 0;
        if (lane == sl) {
          uint32_t acc = excl;
          for (int x = 0; x < per; ++x) {
            const uint32_t h = hist[rt_hidx(hi - x)];
            if (acc + h >= remaining) {
              bin = hi - x;
              above = acc;
              cnt = h;
              break;
            }
            acc += h;
          }
        }
        bin = __shfl_sync(KIV_FULL_MASK, bin, sl);
        above = __shfl_sync(KIV_FULL_MASK, above, sl);
        cnt = __shfl_sync(KIV_FULL_MASK, cnt, sl);
        __syncwarp();
        remaining -= above;
        prefix |= (uint32_t)bin << sh;
        mask |= (uint32_t)(nbins - 1) << sh;
        if (cnt <= RT_CAND) break;
      }
    }
    // keys above the boundary are selected; the boundary keys ((key & mask) ==
    // prefix) are compacted in index order
    int nb = 0;
    for (int64_t base = 0; base < np; base += 32 * RT_UNROLL) {
      float v[RT_UNROLL];
#pragma unroll
      for (int x = 0; x < RT_UNROLL; ++x) {
        const int64_t i = base + x * 32 + lane;
        v[x] = i < np ? __ldcg(src + i) : 0.f;
      }
#pragma unroll
      for (int x = 0; x < RT_UNROLL; ++x) {
        const int64_t i = base + x * 32 + lane;
        const uint32_t key = f2key(v[x]);
        const bool in = i < np;
        const bool up = in && (all || (key & mask) > prefix);
        const bool bnd = in && !all && (key & mask) == prefix;
        if (up && marks) mark(i);
        const unsigned bb = __ballot_sync(KIV_FULL_MASK, bnd);
        if (bnd) {
          const int pos = nb + __popc(bb & lt);
          if (pos < RT_CAND) {
            ckey[pos] = key;
            cidx[pos] = (int32_t)i;
          }
        }
        nb += __popc(bb);
      }
    }
    __syncwarp();
    // boundary: `remaining` of the nb keys, score descending then lowest page
    const int nbc = nb < RT_CAND ? nb : RT_CAND;
    for (int j = lane; j < nbc; j += 32) {
      bool take;
      if (mask == 0xFFFFFFFFu) {
        take = (uint32_t)j < remaining;             // all equal: index order
      } else {
        const uint32_t kj = ckey[j];
        uint32_t r = 0;
        for (int x = 0; x < nbc; ++x) {
          const uint32_t kx = ckey[x];
          r += (kx > kj) || (kx == kj && x < j);
        }
        take = r < remaining;
      }
      cflag[j] = take ? 1 : 0;
      if (take && marks) mark(cidx[j]);
    }
    __syncwarp();
    if (!marks) {
      // this rank's list of the row, (score, global page) in page order
      int pos = 0, bi = 0;
      for (int64_t base = 0; base < np; base += 32) {
        const int64_t i = base + lane;
        const bool in = i < np;
        const float sc = in ? __ldcg(src + i) : 0.f;
        const uint32_t key = f2key(sc);
        const bool up = in && (all || (key & mask) > prefix);
        const bool bnd = in && !all && (key & mask) == prefix;
        const unsigned bb = __ballot_sync(KIV_FULL_MASK, bnd);
        const int bpos = bi + __popc(bb & lt);
        const bool sel = up || (bnd && bpos < RT_CAND && cflag[bpos]);
        const unsigned sb = __ballot_sync(KIV_FULL_MASK, sel);
        if (sel) {
          const int p = pos + __popc(sb & lt);
          if (p < K) {
            ls[p] = sc;
            lpg[p] = (int32_t)(i * nsh + rank);
          }
        }
        pos += __popc(sb);
        bi += __popc(bb);
      }
      for (int j = (int)k + lane; j < K; j += 32) {
        ls[j] = 0.f;
        lpg[j] = -1;
      }
    }
    __syncwarp();
  }
  __syncthreads();
  if (nwords > 0)
    for (int i = threadIdx.x; i < nwords; i += RT_THREADS)
      if (bits[i]) atomicOr(&w.pbits[i], bits[i]);
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    if (marks) st.state[KIV_ST_UNION_PENDING] = 1;
    const unsigned long long mk = w.cstat[0], sb = w.cstat[1];
    if (mk) atomicMax(reinterpret_cast<unsigned long long *>(st.state + KIV_ST_COARSE_MAX), mk);
    atomicAdd(reinterpret_cast<double *>(st.state + KIV_ST_COARSE_SUM), __longlong_as_double((long long)sb));
    w.cstat[0] = 0;
    w.cstat[1] = 0;
  }
}

// Sorted page union from the marks the coarse pass set (single CTA): used
// ahead of the scorers that do not build it themselves.  Clears the marks and
// the pending word; a no-op when no coarse pass is pending (reused union).
__global__ void __launch_bounds__(UN_THREADS) union_kernel(kiv_store st, Workspace w) {
  griddep_wait();
  __shared__ int wsum[UN_THREADS / 32];
  if (st_ld(st.state, KIV_ST_UNION_PENDING) == 0) return;
  const int64_t np_global = st_ld(st.state, KIV_ST_COLD_LEN) / st.page_size;
  // marks: one per local page, or per global page with replicated summaries
  // (this shard's pages of the union kept)
  const int64_t np = coarse_pages(st, np_global);
  const bool repl = repl_summaries(st);
  const int u = union_from_bits<UN_THREADS, false>(w.pbits, np, w.uni, (int)w.u_cap, repl ? 0 : st.shard_rank,
                                                   repl ? 1 : st.shard_count, wsum, st.shard_rank,
                                                   repl ? st.shard_count : 1);
  for (int64_t i = threadIdx.x; i < (np + 31) / 32; i += UN_THREADS) w.pbits[i] = 0;
  if (threadIdx.x == 0) {
    st.state[KIV_ST_UNION] = u;
    st.state[KIV_ST_UNION_PENDING] = 0;
  }
}

kiv_status launch_union(const kiv_store *st, const Workspace &w, cudaStream_t s) {
  return cuda_status(launch_pdl(union_kernel, dim3(1), dim3(UN_THREADS), 0, s, 1, *st, w), "union");
}

// Merge gathered per-row lists [n][R][K] into the global per-row top-k and
// keep the union pages this shard owns.  Ties at the threshold are broken by
// the lowest page id.
template <bool X>
__global__ void __launch_bounds__(CM_THREADS)
coarse_merge_kernel(kiv_store st, kiv_query q, Workspace w, const float *ls, const int32_t *lp, int32_t n,
                    XArgs x, const float *mine_s, const int32_t *mine_p) {
  // the epoch was advanced by this type's previous exchange; read it after
  // the dependency wait, which also covers a merge of the same type right
  // before this one in the stream
  griddep_wait();
  const unsigned long long e = X ? x_epoch(x, X_COARSE) : 0ull;
  extern __shared__ uint4 dyn_smem[];
  __shared__ SelectSmem<CM_THREADS> sm;
  const int S = st.page_size;
  const int64_t np_global = st_ld(st.state, KIV_ST_COLD_LEN) / S;
  const int row = blockIdx.x;
  const int K = q.top_pages;
  const int64_t R = w.R;
  bool ok = true;
  uint32_t flag = 0;
  if (X) {
    // this rank's list of this row -> slot [rank] of every arena, as
    // (score, page) word pairs carrying the epoch's flag
    flag = x_flag(e);
    for (int d = 0; d < x.world; ++d) {
      unsigned long long *reg = x_region(x, d, e) + (((int64_t)x.rank * R + row) * K) * 2;
      for (int j = threadIdx.x; j < K; j += CM_THREADS) {
        ll_store(reg + 2 * j, __float_as_uint(mine_s[(int64_t)row * K + j]), flag);
        ll_store(reg + 2 * j + 1, (uint32_t)mine_p[(int64_t)row * K + j], flag);
      }
    }
    n = x.world;
  }
  const int m = n * K;
  uint32_t *keys = reinterpret_cast<uint32_t *>(dyn_smem);
  int32_t *ids = reinterpret_cast<int32_t *>(keys + m);
  const unsigned long long *mine = X ? x_region(x, x.rank, e) : nullptr;
  constexpr int CB = 4;   // entries per thread per batch (independent loads)
  for (int i0 = 0; i0 < m; i0 += CM_THREADS * CB) {
    unsigned long long wv[2 * CB];
    int64_t offs[CB];
#pragma unroll
    for (int k = 0; k < CB; ++k) {
      const int i = i0 + k * CM_THREADS + threadIdx.x;
      const int src = i / K, j = i % K;
      offs[k] = ((int64_t)src * R + row) * K + j;
      if (X && i < m) {
        wv[2 * k] = ld_relaxed_sys(mine + 2 * offs[k]);
        wv[2 * k + 1] = ld_relaxed_sys(mine + 2 * offs[k] + 1);
      }
    }
#pragma unroll
    for (int k = 0; k < CB; ++k) {
      const int i = i0 + k * CM_THREADS + threadIdx.x;
      if (i >= m) continue;
      int32_t pg;
      float sc;
      if (X) {
        sc = __uint_as_float(ll_check(mine + 2 * offs[k], wv[2 * k], flag, ok, x.budget));
        pg = (int32_t)ll_check(mine + 2 * offs[k] + 1, wv[2 * k + 1], flag, ok, x.budget);
      } else {
        sc = __ldcg(ls + offs[k]);
        pg = __ldcg(lp + offs[k]);
      }
      ids[i] = pg;
      keys[i] = pg >= 0 ? f2key(sc) : 0u;
    }
  }
  if (X && !ok)
    atomicOr(reinterpret_cast<unsigned long long *>(st.state + KIV_ST_ERROR),
             (unsigned long long)KIV_ERRBIT_WAIT_TIMEOUT);
  // a wait that gave up leaves some lists unread: mark no page
  if (__syncthreads_or(X && !ok)) {
    if (X) x_advance(x, X_COARSE, e);
    return;
  }
  const uint32_t k = (uint32_t)(K < np_global ? (int64_t)K : np_global);
  auto mark = [&](int32_t id) {
    if ((id % st.shard_count) == st.shard_rank) {
      const int32_t lpg = id / st.shard_count;
      atomicOr(&w.pbits[lpg >> 5], 1u << (lpg & 31));
    }
  };
  if (k > 0 && m <= CM_RANK_MAX) {
    // few entries: each one's rank in the total order (score desc, page asc)
    // by comparison with all of them, in one pass
    for (int i = threadIdx.x; i < m; i += CM_THREADS) {
      const int32_t pi = ids[i];
      if (pi < 0) continue;
      const uint32_t ki = keys[i];
      uint32_t rank = 0;
#pragma unroll 4
      for (int j = 0; j < m; ++j) {
        const uint32_t kj = keys[j];
        const int32_t pj = ids[j];
        rank += (pj >= 0 && (kj > ki || (kj == ki && pj < pi))) ? 1u : 0u;
      }
      if (rank < k) mark(pi);
    }
  } else if (k > 0) {
    uint32_t T = 0, need = 0;
    radix_threshold<CM_THREADS, 1>(keys, m, k, sm, T, need);
    // entries == T: take the `need` lowest page ids
    for (int i = threadIdx.x; i < m; i += CM_THREADS) {
      bool take = keys[i] > T;
      if (!take && keys[i] == T && ids[i] >= 0) {
        uint32_t rank = 0;
        for (int j = 0; j < m; ++j)
          rank += (keys[j] == T && ids[j] >= 0 && ids[j] < ids[i]) ? 1u : 0u;
        take = rank < need;
      }
      if (take && ids[i] >= 0) mark(ids[i]);
    }
  }
  if (row == 0 && threadIdx.x == 0) st.state[KIV_ST_UNION_PENDING] = 1;
  if (X) x_advance(x, X_COARSE, e);
}

template <typename T, int LPR, int VPL, int RCH>
static void launch_cs(const kiv_store *st, const kiv_query *q, const Workspace &w, cudaStream_t s) {
  const int H = st->num_kv_heads;
  const int rows_kv = (q->num_query_heads / H) * q->query_len;
  const int64_t nchunks = ceil_div(rows_kv, RCH);
  const int64_t items = (int64_t)st->batch * H * nchunks * ceil_div(w.np_cap, CS_PAGES);
  const int64_t grid = std::min<int64_t>(std::max<int64_t>(items, 1), (int64_t)sm_count() * 8);
  const size_t smem = (size_t)CS_PAGES * st->head_dim * sizeof(T);
  launch_pdl(coarse_scores_kernel<T, LPR, VPL, RCH>, dim3((unsigned)grid), dim3(CS_THREADS), smem, s, 1, *st, *q,
             w);
}

template <typename T>
static kiv_status dispatch_cs(const kiv_store *st, const kiv_query *q, const Workspace &w,
                              cudaStream_t s) {
  const int nv = st->head_dim / Elem<T>::V;
  const int rows_kv = (q->num_query_heads / st->num_kv_heads) * q->query_len;
  const bool small = rows_kv <= 4;
#define KIV_CS(LPR, VPL)                                          \
  do {                                                            \
    if (small) launch_cs<T, LPR, VPL, 4>(st, q, w, s);            \
    else launch_cs<T, LPR, VPL, 8>(st, q, w, s);                  \
  } while (0)
  if (nv <= 2) KIV_CS(2, 1);
  else if (nv <= 4) KIV_CS(4, 1);
  else if (nv <= 8) KIV_CS(8, 1);
  else if (nv <= 16) KIV_CS(16, 1);
  else if (nv <= 32) KIV_CS(32, 1);
  else if (nv <= 64) KIV_CS(32, 2);
  else return KIV_ERR_UNSUPPORTED;
#undef KIV_CS
  return KIV_OK;
}

kiv_status launch_coarse(const kiv_store *st, const kiv_query *q, const Workspace &w,
                         float *row_scores, int32_t *row_pages, cudaStream_t s) {
  kiv_status rc;
  // prefill-shaped queries: tensor-core scoring, no per-row histograms (the
  // workspace holds none for this shape)
  const int self_hist = prefill_shape(st, q) ? 1 : 0;
  if (self_hist && !prefill_tc_eligible(st, q)) {
    set_error("prefill-shaped query needs a 16-byte aligned base and strides that are multiples of 8 elements");
    return KIV_ERR_ARG;
  }
  // the per-row top-k builds its first histogram from the scores it stages,
  // except after the CUDA-core scorer (which writes the histograms itself)
  int topk_self_hist = 1;
  if (self_hist) {
    rc = launch_prefill_coarse_scores(st, q, w, s);
  } else if (fine_tc_eligible(st, q)) {
    rc = launch_coarse_score_tc(st, q, w, s);
  } else {
    topk_self_hist = 0;
    switch (st->dtype) {
      case KIV_DTYPE_F32: rc = dispatch_cs<float>(st, q, w, s); break;
      case KIV_DTYPE_BF16: rc = dispatch_cs<__nv_bfloat16>(st, q, w, s); break;
      case KIV_DTYPE_F16: rc = dispatch_cs<__half>(st, q, w, s); break;
      default: rc = KIV_ERR_UNSUPPORTED;
    }
  }
  if (rc != KIV_OK) return rc;
  if (q->top_pages > 8192) {
    set_error("coarse: top_pages %d exceeds the shared-memory select (max 8192)", q->top_pages);
    return KIV_ERR_CAPACITY;
  }
  if (self_hist && q->top_pages <= RT_CAND) {
    // prefill-shaped rows: one warp per row
    const int64_t words = ceil_div(w.np_cap, 32);
    const int nwords = words <= 4096 ? (int)words : 0;
    const size_t smem = 4 * (size_t)RT_WARPS * (RT_HWORDS + 2 * RT_CAND) + (size_t)RT_WARPS * RT_CAND +
                        4 * (size_t)nwords;
    const int64_t grid = std::max<int64_t>(1, std::min<int64_t>(ceil_div(w.R, RT_WARPS), 2 * (int64_t)sm_count()));
    cudaFuncSetAttribute(coarse_rows_topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    return cuda_status(launch_pdl(coarse_rows_topk_kernel, dim3((unsigned)grid), dim3(RT_THREADS), smem, s, 1, *st,
                                  *q, w, row_scores, row_pages, nwords),
                       "coarse_rows_topk");
  }
  // candidate buffer (key + index + flag per page), the boundary scratch, the
  // chosen list and the staged scores of the row
  const int64_t np_pad = align_up(w.np_cap, 16);
  const int scap = (int)std::min<int64_t>(np_pad, TK_SCAP);
  const int64_t fixed = 8 * TK_BND + 4 * align_up(q->top_pages, 4) + 4 * (int64_t)scap;
  const int64_t room = (176 * 1024 - fixed) / 9;
  const int cap = std::max(16, (int)std::min<int64_t>(np_pad, room & ~15ll));
  const size_t smem = (size_t)cap * 9 + (size_t)fixed;
  cudaFuncSetAttribute(coarse_topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  const cudaError_t e = launch_pdl(coarse_topk_kernel, dim3((unsigned)w.R), dim3(TK_THREADS), smem, s, 1, *st, *q,
                                   w, row_scores, row_pages, cap, scap, topk_self_hist);
  if (e != cudaSuccess) return cuda_status(e, "coarse_topk");
  return cuda_status(cudaGetLastError(), "coarse");
}

kiv_status launch_coarse_merge(const kiv_store *st, const kiv_query *q, const Workspace &w,
                               const float *ls, const int32_t *lp, int32_t n, cudaStream_t s,
                               const XArgs *x) {
  const int nl = x ? x->world : n;
  const size_t smem = (size_t)nl * q->top_pages * (sizeof(uint32_t) + sizeof(int32_t));
  if (smem > 200 * 1024) return KIV_ERR_CAPACITY;
  cudaError_t e;
  if (x) {
    cudaFuncSetAttribute(coarse_merge_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    e = launch_pdl(coarse_merge_kernel<true>, dim3((unsigned)w.R), dim3(CM_THREADS), smem, s, 1, *st, *q, w,
                   (const float *)nullptr, (const int32_t *)nullptr, nl, *x, ls, lp);
  } else {
    cudaFuncSetAttribute(coarse_merge_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    e = launch_pdl(coarse_merge_kernel<false>, dim3((unsigned)w.R), dim3(CM_THREADS), smem, s, 1, *st, *q, w, ls,
                   lp, n, XArgs{}, (const float *)nullptr, (const int32_t *)nullptr);
  }
  if (e != cudaSuccess) return cuda_status(e, "coarse_merge");
  return cuda_status(cudaGetLastError(), "coarse_merge");
}

}  // namespace kiv
