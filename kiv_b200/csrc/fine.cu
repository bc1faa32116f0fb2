// Kernel (c): fine token scoring fused with the top-`top_p` token select.
//
// Reference behaviour restated (kiv/cold_store.py:227-262, :301, :332-347):
//   candidates = every token of the union pages (ascending) + the partial page;
//   f[b,h,q,c] = scaling * <q[b,h,q], K[b, h // G, c]>;  agg[b,c] = max_{h,q} f;
//   keep the P = min(top_p, cold_len, C) best candidates per batch row.
// The reference gathers candidate K AND V of every union page from host
// memory over PCIe, materializes repeat_kv(K) and runs a GEMM.  Here the cold
// tier is HBM-resident: each candidate page tile (rows of one KV head) is
// staged into shared memory by a 1-D TMA bulk copy (4-stage mbarrier
// pipeline), scored against all G*Q rows of its KV head, and reduced to the
// max over heads and positions in shared memory; V is never touched.  The
// select runs on one thread-block cluster per batch row with the candidate
// keys spread over the cluster's shared memory.
#include <algorithm>

#include "common.cuh"
#include "internal.h"
#include "exchange.cuh"
#include "select.cuh"

namespace kiv {

constexpr int FS_THREADS = 256;
constexpr int FS_STAGES = 4;
constexpr int FS_TILE_BYTES = 16384;
constexpr int SL_THREADS = 512;
constexpr int SL_BND = 1024;      // boundary-bin capacity of the candidate select
constexpr int SL_CAP = 4096;      // candidates resolved in rank 0's shared memory
constexpr int SL_UCAP = 4096;     // union pages staged in shared memory
constexpr int SL_KCAP = 16384;    // keys per CTA staged in shared memory
constexpr int FM_THREADS = 512;

struct FineGeom {
  int64_t U, np_global, partial, per_b, items;
  bool part_owned;
};

__device__ __forceinline__ FineGeom fine_geom(const kiv_store &st) {
  FineGeom f;
  const int S = st.page_size;
  const int64_t cold = st_ld(st.state, KIV_ST_COLD_LEN);
  f.U = st_ld(st.state, KIV_ST_UNION);
  f.np_global = cold / S;
  f.partial = cold % S;
  f.part_owned = f.partial > 0 && (f.np_global % st.shard_count) == st.shard_rank;
  f.per_b = f.U + (f.part_owned ? 1 : 0);
  f.items = (int64_t)st.batch * f.per_b;
  return f;
}

// global token id of local candidate position c
__device__ __forceinline__ int32_t cand_token(const Workspace &w, const FineGeom &f, int S, int64_t c) {
  const int64_t uS = f.U * S;
  if (c < uS) return (int32_t)((int64_t)w.uni[c / S] * S + c % S);
  return (int32_t)(f.np_global * S + (c - uS));
}

template <typename T, int LPR, int VPL, int RCH>
__global__ void __launch_bounds__(FS_THREADS)
fine_scores_kernel(kiv_store st, kiv_query q, Workspace w, int tr, int stage_q) {
  griddep_wait();
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    st.state[KIV_ST_FINE_MAX] = 0;
    st.state[KIV_ST_FINE_SUM] = 0;
  }
  extern __shared__ __align__(128) uint8_t fs_smem[];
  __shared__ uint64_t bars[FS_STAGES];
  __shared__ int s_fail;
  __shared__ uint32_t s_hist[SEL_BINS];   // first-pass histogram of the batch row being processed
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane % LPR, grp = lane / LPR;
  constexpr int GPW = 32 / LPR;
  constexpr int NGROUPS = (FS_THREADS / 32) * GPW;
  constexpr int V = Elem<T>::V;
  const int D = st.head_dim, H = st.num_kv_heads, S = st.page_size;
  const int nv = D / V;
  const int Hq = q.num_query_heads, Q = q.query_len;
  const int G = Hq / H;
  const int rows_kv = G * Q;
  const int nchunks = (rows_kv + RCH - 1) / RCH;
  T *tiles = reinterpret_cast<T *>(fs_smem);
  float *mx = reinterpret_cast<float *>(fs_smem + (size_t)FS_STAGES * tr * D * sizeof(T));
  float *qs = mx + ((tr + 3) & ~3);   // [Hq*Q][D] fp32 query rows of the current batch row

  const FineGeom f = fine_geom(st);
  const int nrb = (S + tr - 1) / tr;
  // work unit = (b, candidate page u, row block rb); its tiles are the H KV heads
  const int64_t units = f.items * nrb;
  const int64_t my_units = units > blockIdx.x ? (units - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;
  const int64_t my_tiles = my_units * H;
  const T *cold_k = reinterpret_cast<const T *>(st.cold_k);
  const T *qb = reinterpret_cast<const T *>(q.q);

  if (threadIdx.x == 0) {
    for (int s = 0; s < FS_STAGES; ++s) mbar_init(&bars[s], 1);
    mbar_fence_init();
    s_fail = 0;
  }
  for (int i = threadIdx.x; i < tr; i += FS_THREADS) mx[i] = -INFINITY;
  for (int i = threadIdx.x; i < SEL_BINS; i += FS_THREADS) s_hist[i] = 0;
  __syncthreads();

  struct Unit { int b; int64_t u; int rb; int rows; };
  auto unit_of = [&](int64_t t) {
    Unit x;
    const int64_t un = blockIdx.x + (t / H) * gridDim.x;
    x.rb = (int)(un % nrb);
    const int64_t item = un / nrb;
    x.b = (int)(item / f.per_b);
    x.u = item % f.per_b;
    const int64_t limit = x.u < f.U ? S : f.partial;
    x.rows = (int)std::max<int64_t>(0, std::min<int64_t>(tr, limit - (int64_t)x.rb * tr));
    return x;
  };
  auto issue = [&](int64_t t) {
    const int stage = (int)(t % FS_STAGES);
    const Unit x = unit_of(t);
    const int kvh = (int)(t % H);
    const uint32_t bytes = (uint32_t)x.rows * D * sizeof(T);
    if (bytes > 0) {
      const int64_t page = x.u < f.U ? (int64_t)w.uni[x.u] : f.np_global;
      const int64_t lp = page_slot(st, w, page / st.shard_count);
      const T *src = cold_k + (((int64_t)x.b * H + kvh) * st.cold_capacity + lp * S + (int64_t)x.rb * tr) * D;
      mbar_arrive_tx(&bars[stage], bytes);
      bulk_g2s(tiles + (size_t)stage * tr * D, src, bytes, &bars[stage]);
    } else {
      mbar_arrive(&bars[stage]);
    }
  };
  if (threadIdx.x == 0) {
    for (int64_t t = 0; t < std::min<int64_t>(FS_STAGES, my_tiles); ++t) issue(t);
  }

  int staged_b = -1;
  // running stats and histogram of the batch row being processed (flushed
  // when it changes and at the end; every thread calls this, at the same
  // points).  The histogram collects in shared memory with plain atomics
  // and reaches the row's global histogram once, non-zero bins only.
  int stat_b = -1;
  uint32_t kmax = 0;
  float ksum = 0.f;
  auto flush_stats = [&]() {
    if (stat_b < 0) return;
    uint32_t mk = __reduce_max_sync(KIV_FULL_MASK, kmax);
    float sm = ksum;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sm += __shfl_xor_sync(KIV_FULL_MASK, sm, o);
    if (lane == 0 && mk != 0) {
      atomicMax(reinterpret_cast<unsigned long long *>(&w.fstat[2 * stat_b]), (unsigned long long)mk);
      atomicAdd(reinterpret_cast<double *>(&w.fstat[2 * stat_b + 1]), (double)sm);
    }
    kmax = 0;
    ksum = 0.f;
    __syncthreads();
    uint32_t *hb = w.fhist + (int64_t)stat_b * SEL_BINS;
    for (int i = threadIdx.x; i < SEL_BINS; i += FS_THREADS) {
      const uint32_t c = s_hist[i];
      if (c) {
        atomicAdd(&hb[i], c);
        s_hist[i] = 0;
      }
    }
    __syncthreads();
  };
  for (int64_t t = 0; t < my_tiles; ++t) {
    const Unit x = unit_of(t);
    const int kvh = (int)(t % H);
    if (stage_q && x.b != staged_b) {
      // stage this batch row's query rows (fp32) once; reused by every tile
      for (int e = threadIdx.x; e < Hq * Q * nv; e += FS_THREADS) {
        const int rq = e / nv, vi = e % nv;
        const int h = rq / Q, tq = rq % Q;
        float fv[V];
        Elem<T>::unpack(ld16(qb + x.b * q.stride_b + h * q.stride_h + tq * q.stride_t + vi * V), fv);
#pragma unroll
        for (int k = 0; k < V; ++k) qs[(size_t)rq * D + vi * V + k] = fv[k];
      }
      staged_b = x.b;
    }
    const int stage = (int)(t % FS_STAGES);
    const uint32_t parity = (uint32_t)((t / FS_STAGES) & 1);
    if (!mbar_wait_bounded(&bars[stage], parity)) s_fail = 1;
    __syncthreads();
    if (s_fail) break;
    const T *tile = tiles + (size_t)stage * tr * D;
    for (int ch = 0; ch < nchunks; ++ch) {
      RowDot<T, LPR, VPL, RCH> dot;
      if (stage_q) {
        const float *qrows[RCH];
#pragma unroll
        for (int r = 0; r < RCH; ++r) {
          const int rr = ch * RCH + r;
          // query row (h, tq) with h = kvh*G + rr/Q is staged at index h*Q + tq
          qrows[r] = rr < rows_kv ? qs + (size_t)((kvh * G + rr / Q) * Q + rr % Q) * D : nullptr;
        }
        dot.load_query_f32(qrows, g, nv);
      } else {
        const T *qrows[RCH];
#pragma unroll
        for (int r = 0; r < RCH; ++r) {
          const int rr = ch * RCH + r;
          qrows[r] = rr < rows_kv ? qb + x.b * q.stride_b + (kvh * G + rr / Q) * q.stride_h +
                                        (rr % Q) * q.stride_t
                                  : nullptr;
        }
        dot.load_query(qrows, g, nv, 1.0f);
      }
      const int my_group = warp * GPW + grp;
      for (int r0 = 0; r0 < x.rows; r0 += NGROUPS) {
        const int r = r0 + my_group;
        float acc[RCH];
        dot.template partial<false>(r < x.rows ? tile + (size_t)r * D : nullptr, g, nv, acc);
        int base = 0;
        tr_reduce<RCH, LPR / 2>(acc, lane, base);
        constexpr int NOUT = TrOut<RCH, LPR>::N;
        float m = -INFINITY;
#pragma unroll
        for (int i = 0; i < NOUT; ++i) {
          const int rr = ch * RCH + base + i;
          if (rr < rows_kv) m = fmaxf(m, acc[i] * q.scaling);
        }
        m = group_max<LPR / 2>(m);
        if (r < x.rows && g == 0) mx[r] = fmaxf(mx[r], m);
      }
    }
    __syncthreads();  // stage consumed, mx updated
    if (threadIdx.x == 0 && t + FS_STAGES < my_tiles) issue(t + FS_STAGES);
    if (kvh == H - 1) {
      // unit complete: publish its keys (+ first-pass histogram, stats), reset the running max
      if (x.b != stat_b) {
        flush_stats();
        stat_b = x.b;
      }
      uint32_t *dst = w.agg + (int64_t)x.b * w.c_cap + x.u * S + (int64_t)x.rb * tr;
      for (int i = threadIdx.x; i < tr; i += FS_THREADS) {
        if (i < x.rows) {
          const uint32_t key = f2key(mx[i]);
          dst[i] = key;
          atomicAdd(&s_hist[key >> 21], 1u);
          kmax = key > kmax ? key : kmax;
          ksum += mx[i];
        }
        mx[i] = -INFINITY;
      }
      __syncthreads();
    }
  }
  flush_stats();
  if (s_fail && threadIdx.x == 0)
    atomicOr(reinterpret_cast<unsigned long long *>(st.state + KIV_ST_ERROR), (unsigned long long)KIV_ERRBIT_WAIT_TIMEOUT);
}

// One cluster of CL CTAs per batch row: exact top-P over the C candidates.
// The scorer left the row's first-pass histogram (key >> 21) in w.fhist, so
// the threshold bin b0 is known up front.  Right after the dependency wait
// one bulk copy per input brings the histogram, this CTA's index range of
// keys and (rank 0) the union pages into shared memory, so the kernel pays
// one memory round trip for its inputs.  Each CTA compacts its keys in bins
// >= b0 (index order), the CTAs exchange their counts, push their candidates
// into rank 0's shared memory, and rank 0 resolves the top P among them
// (select_candidates).  When the candidates do not fit, the cluster runs the
// full radix select over the keys instead.
// shard_count == 1: sel[b, :P] = selected token ids (ascending).
// shard_count > 1: sel / scores hold this shard's local list (tail -1).
// XC (candidate exchange): the keys of every shard's candidates arrive in this
// shard's arena as flagged words (each read waits, bounded, for its flag);
// every CTA counts its keys into a histogram and the cluster sums them, then
// the select runs as above over all candidates.  sel gets the global top-P
// (ascending, tail -1) on every shard and sel_local this shard's part of it;
// a wait that gave up selects nothing.
template <int CL, bool XC>
__global__ void __launch_bounds__(SL_THREADS)
fine_select_kernel(kiv_store st, kiv_query q, Workspace w, int32_t *sel, float *scores, int cap, int ucap,
                   int kcap, int32_t *sel_local, const __grid_constant__ XArgs x) {
  extern __shared__ uint4 sl_dyn[];
  __shared__ __align__(16) CandSmem<SL_THREADS> cs;
  __shared__ SelectSmem<SL_THREADS> sm;
  __shared__ int s_cnt;
  __shared__ int s_fail;
  __shared__ int s_xfail;
  __shared__ int s_wsum[SL_THREADS / 32];
  __shared__ uint64_t bar;
  uint32_t *ckey = reinterpret_cast<uint32_t *>(sl_dyn);
  int32_t *cidx = reinterpret_cast<int32_t *>(ckey + cap);
  uint32_t *bkey = reinterpret_cast<uint32_t *>(cidx + cap);
  int32_t *bidx = reinterpret_cast<int32_t *>(bkey + SL_BND);
  int32_t *sel_ci = bidx + SL_BND;                        // [cap] chosen candidates
  int32_t *suni = sel_ci + cap;                            // [ucap] union pages (staged)
  uint32_t *skey = reinterpret_cast<uint32_t *>(suni + ucap);   // [kcap] this CTA's keys (staged)
  uint8_t *flag = reinterpret_cast<uint8_t *>(skey + kcap);
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    mbar_fence_init();
    s_fail = 0;
    s_xfail = 0;
  }
  if (XC)
    for (int i = threadIdx.x; i < SEL_BINS; i += SL_THREADS) sm.hist[0][i] = 0;
  __syncthreads();
  // the cold length was published by the eviction, kernels back
  const int64_t cold = st_ld(st.state, KIV_ST_COLD_LEN);
  griddep_wait();
  const int b = blockIdx.x / CL;
  const int r = cl_rank<CL>();
  const int S = st.page_size;
  // This CTA's index range is fixed by the candidate capacity, so the input
  // copies start before the candidate count is known (one round trip for
  // the copies and the state read together); keys past the count are unused.
  const int64_t chunk = ((w.c_cap + CL - 1) / CL + 15) / 16 * 16;
  const int64_t lo = std::min<int64_t>(w.c_cap, r * chunk);
  const int64_t n_cap = std::min<int64_t>(w.c_cap, lo + chunk) - lo;
  const uint32_t *src = w.agg + (int64_t)b * w.c_cap + lo;
  uint32_t *hb = w.fhist + (int64_t)b * SEL_BINS;
  const bool kstaged = n_cap > 0 && n_cap <= kcap && (reinterpret_cast<uintptr_t>(src) & 15) == 0;
  // XC: the keys come from the arena (below), the histogram is built here
  const uint32_t hbytes = XC ? 0u : SEL_BINS * 4;
  const uint32_t kb = kstaged && !XC ? (uint32_t)((n_cap * 4 + 15) & ~15ll) : 0u;
  const uint32_t ub = r == 0 && ucap > 0 ? (uint32_t)((ucap * 4 + 15) & ~15) : 0u;
  if (threadIdx.x == 0 && hbytes + kb + ub > 0) {
    mbar_arrive_tx(&bar, hbytes + kb + ub);
    if (hbytes) bulk_g2s(cs.hist, hb, hbytes, &bar);
    if (kb) bulk_g2s(skey, src, kb, &bar);
    if (ub) bulk_g2s(suni, w.uni, ub, &bar);
  }
  FineGeom f;
  f.U = st_ld(st.state, KIV_ST_UNION);
  f.np_global = cold / S;
  f.partial = cold % S;
  // XC: the partial page's candidates are in every shard's arena
  f.part_owned = f.partial > 0 && (XC || (f.np_global % st.shard_count) == st.shard_rank);
  f.per_b = f.U + (f.part_owned ? 1 : 0);
  f.items = (int64_t)st.batch * f.per_b;
  const int64_t C = f.U * S + (f.part_owned ? f.partial : 0);
  const int n_local = (int)std::max<int64_t>(0, std::min<int64_t>(C, lo + n_cap) - lo);
  const int64_t P = std::min<int64_t>(q.top_p, C);
  const bool all = P >= C;
  const bool ustaged = r == 0 && f.U > 0 && f.U <= ucap;
  int32_t *out = sel + (int64_t)b * q.top_p;
  float *osc = scores ? scores + (int64_t)b * q.top_p : nullptr;
  // cleanup inputs, loaded while the copies fly
  unsigned long long st_mk = 0, st_sb = 0;
  int64_t pending = 0;
  if (r == 0 && threadIdx.x == 0) {
    st_mk = w.fstat[2 * b];
    st_sb = w.fstat[2 * b + 1];
    pending = st_ld(st.state, KIV_ST_UNION_PENDING);
  }
  if (hbytes + kb + ub > 0 && !mbar_wait_bounded(&bar, 0)) s_fail = 1;
  const unsigned long long xe = XC ? x_epoch(x, X_CAND) : 0ull;
  if (XC) {
    // this CTA's candidates from the arena: independent loads first (one
    // round trip), then each word's flag checked (reloaded until it arrives)
    const unsigned long long *words = x_region(x, x.rank, xe) + (int64_t)b * w.c_cap + lo;
    uint32_t *kdst = kstaged ? skey : const_cast<uint32_t *>(src);
    const uint32_t flag = x_flag(xe);
    bool ok = true;
    constexpr int XB = 16;
#pragma unroll 1
    for (int i0 = 0; i0 < n_local; i0 += SL_THREADS * XB) {
      unsigned long long v[XB];
#pragma unroll
      for (int k = 0; k < XB; ++k) {
        const int i = i0 + k * SL_THREADS + threadIdx.x;
        v[k] = i < n_local ? ld_relaxed_sys(words + i) : 0ull;
      }
#pragma unroll
      for (int k = 0; k < XB; ++k) {
        const int i = i0 + k * SL_THREADS + threadIdx.x;
        if (i < n_local) {
          const uint32_t key = ll_check(words + i, v[k], flag, ok, x.budget);
          kdst[i] = key;
          atomicAdd(&sm.hist[0][key >> 21], 1u);
        }
      }
    }
    const int anyfail = __syncthreads_or(!ok);
    if (threadIdx.x == 0) s_xfail = anyfail;
    cl_sync<CL>();
    // one failed wait fails the whole cluster
    bool fail = false;
#pragma unroll 1
    for (int o = 0; o < CL; ++o) fail |= *cl_map<CL>(&s_xfail, o) != 0;
    if (!fail) {
      // the row's histogram = the sum of the cluster's: CTA r sums its share of
      // the bins over the cluster and writes the sums into every CTA's copy
      constexpr int BS = SEL_BINS / CL;
      for (int i = threadIdx.x; i < BS; i += SL_THREADS) {
        const int bin = r * BS + i;
        uint32_t t = 0;
#pragma unroll
        for (int o = 0; o < CL; ++o) t += cl_map<CL>(sm.hist[0], o)[bin];
#pragma unroll
        for (int o = 0; o < CL; ++o) cl_map<CL>(cs.hist, o)[bin] = t;
      }
      cl_sync<CL>();
    }
    if (fail) {
      // keep every CTA's shared memory alive until the cluster has read it
      cl_sync<CL>();
      if (threadIdx.x == 0) {
        if (r == 0) {
          w.selcnt[b] = 0;
          atomicOr(reinterpret_cast<unsigned long long *>(st.state + KIV_ST_ERROR),
                   (unsigned long long)KIV_ERRBIT_WAIT_TIMEOUT);
          if (b == 0) {
            st.state[KIV_ST_SEL] = 0;
            st.state[KIV_ST_SEL_LOCAL] = 0;
          }
        }
      }
      x_advance(x, X_CAND, xe);
      return;
    }
  }
  const uint32_t *keys = kstaged ? skey : src;
  auto key_at = [&](int i) { return kstaged ? skey[i] : __ldcg(src + i); };
  auto emit_global = [&](int i, uint32_t pos) {   // i: index within this CTA's range
    if (pos < P) {
      out[pos] = cand_token(w, f, S, lo + i);
      if (osc) osc[pos] = key2f(key_at(i));
    }
  };
  if (P > 0 && !all) {
    find_bin<SL_THREADS>((uint32_t)P, cs, [&](int bin) { return cs.hist[bin]; });
    const uint32_t b0 = cs.bin, need0 = (uint32_t)P - cs.above;
    __syncthreads();
    // (one instantiation per source: see coarse_topk_kernel)
    auto above_bin = [&](uint32_t key) { return (key >> 21) >= b0; };
    const int n_r = kstaged ? ordered_compact<SL_THREADS>(n_local, [&](int i) { return skey[i]; }, above_bin, ckey,
                                                          cidx, 0, cap, cs)
                            : ordered_compact<SL_THREADS>(n_local, [&](int i) { return __ldcg(src + i); }, above_bin,
                                                          ckey, cidx, 0, cap, cs);
    if (threadIdx.x == 0) s_cnt = n_r;
    cl_sync<CL>();
    int total = 0, off = 0;
#pragma unroll 1
    for (int o = 0; o < CL; ++o) {
      const int c = *cl_map<CL>(&s_cnt, o);
      off += o < r ? c : 0;
      total += c;
    }
    if (total <= cap) {
      if (r > 0) {
        uint32_t *rk = cl_map<CL>(ckey, 0);
        int32_t *ri = cl_map<CL>(cidx, 0);
        for (int i = threadIdx.x; i < n_r; i += SL_THREADS) {
          rk[off + i] = ckey[i];
          ri[off + i] = (int32_t)lo + cidx[i];
        }
      }
      cl_sync<CL>();
      if (r == 0) {
        select_candidates<SL_THREADS>(ckey, total, b0, need0, bkey, bidx, flag, SL_BND, cs, sm,
                                      [&](int ci, uint32_t pos) {
                                        if (pos < P) sel_ci[pos] = ci;
                                      });
        __syncthreads();
        const int64_t uS = f.U * S;
        for (int p = threadIdx.x; p < (int)P; p += SL_THREADS) {
          const int ci = sel_ci[p];
          const int64_t c = cidx[ci];
          int32_t tok;
          if (c < uS) tok = (int32_t)((int64_t)(ustaged ? suni[c / S] : __ldcg(w.uni + c / S)) * S + c % S);
          else tok = (int32_t)(f.np_global * S + (c - uS));
          out[p] = tok;
          if (osc) osc[p] = key2f(ckey[ci]);
        }
      }
    } else {
      uint32_t T = 0, need = 0;
      radix_threshold<SL_THREADS, CL>(keys, n_local, (uint32_t)P, sm, T, need, XC ? nullptr : hb);
      ordered_emit<SL_THREADS, CL>(keys, n_local, T, need, false, sm, emit_global);
    }
  } else if (P > 0) {
    ordered_emit<SL_THREADS, CL>(keys, n_local, 0u, 0u, true, sm, emit_global);
  }
  int n_mine = (int)P;
  if (XC && sel_local) {
    // this shard's rows of the global list, ascending (the list was written by
    // the whole cluster)
    cl_sync<CL>();
    if (r == 0) {
      int base = 0;
#pragma unroll 1
      for (int p0 = 0; p0 < (int)P; p0 += SL_THREADS) {
        const int p = p0 + threadIdx.x;
        const int32_t tok = p < (int)P ? __ldcg(out + p) : -1;
        const bool mine = tok >= 0 && (tok / S) % st.shard_count == st.shard_rank;
        int total;
        const int pos = base + block_excl_sum<SL_THREADS>(mine ? 1 : 0, &total, s_wsum);
        if (mine) sel_local[(int64_t)b * q.top_p + pos] = tok;
        base += total;
      }
      n_mine = base;
    }
  }
  // every CTA has read the histogram (first cluster barrier, or P == 0)
  if (r == 0) {
    __syncthreads();
    if (!XC)
      for (int i = threadIdx.x; i < SEL_BINS; i += SL_THREADS) hb[i] = 0;
    if (threadIdx.x == 0) {
      if (st_mk) atomicMax(reinterpret_cast<unsigned long long *>(st.state + KIV_ST_FINE_MAX), st_mk);
      atomicAdd(reinterpret_cast<double *>(st.state + KIV_ST_FINE_SUM), __longlong_as_double((long long)st_sb));
      w.fstat[2 * b] = 0;
      w.fstat[2 * b + 1] = 0;
      if (s_fail)
        atomicOr(reinterpret_cast<unsigned long long *>(st.state + KIV_ST_ERROR),
                 (unsigned long long)KIV_ERRBIT_WAIT_TIMEOUT);
    }
    if (st.shard_count > 1) {
      for (int64_t j = P + threadIdx.x; j < q.top_p; j += SL_THREADS) {
        out[j] = -1;
        if (osc) osc[j] = 0.f;
      }
    }
    if (b == 0) {
      // the scorer built the union from the coarse pass's page marks: consume them
      if (threadIdx.x == 0) s_cnt = (int)pending;
      __syncthreads();
      if (s_cnt) {
        const int64_t np = coarse_pages(st, f.np_global);   // bits of the marks
        for (int64_t i = threadIdx.x; i < (np + 31) / 32; i += SL_THREADS) w.pbits[i] = 0;
        if (threadIdx.x == 0) st.state[KIV_ST_UNION_PENDING] = 0;
      }
    }
    if (threadIdx.x == 0) {
      w.selcnt[b] = (int32_t)n_mine;
      if (b == 0) {
        st.state[KIV_ST_CAND] = C;
        st.state[KIV_ST_SEL] = P;
        st.state[KIV_ST_SEL_LOCAL] = n_mine;
      }
    }
  }
  // the arena's candidates of this epoch are read: the launch's last CTA moves the epoch on
  if (XC) x_advance(x, X_CAND, xe);
}

// lower_bound over the first n entries of an ascending id list
__device__ __forceinline__ int lower_bound_ids(const int32_t *ids, int n, int32_t x) {
  int lo = 0, hi = n;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (ids[mid] < x) lo = mid + 1;
    else hi = mid;
  }
  return lo;
}

// Per-list exclusive prefix of flags over the n concatenated lists of L
// entries, with one block-wide scan: gp[i] = flags in [0, i) overall, then
// pre[j*(L+1) + a] = flags of list j before a (a = L: the list's total).
// Ends with a barrier.
__device__ void list_prefix_block(const uint8_t *flag, int m, int n, int L, int32_t *gp, int32_t *pre,
                                  typename cub::BlockScan<int, FM_THREADS>::TempStorage &tmp) {
  constexpr int IPT = 4;
  int base = 0;
#pragma unroll 1
  for (int t0 = 0; t0 < m; t0 += FM_THREADS * IPT) {
    const int i0 = t0 + threadIdx.x * IPT;
    int f[IPT], c = 0;
#pragma unroll
    for (int k = 0; k < IPT; ++k) {
      f[k] = (i0 + k < m) ? flag[i0 + k] : 0;
      c += f[k];
    }
    int before, total;
    cub::BlockScan<int, FM_THREADS>(tmp).ExclusiveSum(c, before, total);
    int run = base + before;
#pragma unroll
    for (int k = 0; k < IPT; ++k) {
      if (i0 + k < m) gp[i0 + k] = run;
      run += f[k];
    }
    base += total;
    __syncthreads();
  }
  for (int e = threadIdx.x; e < n * (L + 1); e += FM_THREADS) {
    const int j = e / (L + 1), a = e % (L + 1);
    const int v = a < L ? gp[j * L + a] : ((j + 1) * L < m ? gp[(j + 1) * L] : base);
    pre[e] = v - gp[j * L];
  }
  __syncthreads();
}

// Merge n gathered lists [n][B][top_p] (ascending ids, tail -1) into the
// global top-P of each batch row; sel gets all of them (ascending ids),
// sel_local the ones this shard owns (list index == shard rank).
template <bool X>
__global__ void __launch_bounds__(FM_THREADS)
fine_merge_kernel(kiv_store st, kiv_query q, Workspace w, const float *ls, const int32_t *lt,
                  int32_t n, int32_t *sel, int32_t *sel_local, XArgs x, const float *mine_s,
                  const int32_t *mine_t) {
  // the epoch was advanced by this type's previous exchange; read it after
  // the dependency wait, which also covers a merge of the same type right
  // before this one in the stream
  griddep_wait();
  const unsigned long long e = X ? x_epoch(x, X_FINE) : 0ull;
  extern __shared__ uint4 fm_dyn[];
  __shared__ SelectSmem<FM_THREADS> sm;
  __shared__ typename cub::BlockScan<int, FM_THREADS>::TempStorage fm_scan;
  __shared__ int s_valid[64];
  const int b = blockIdx.x;
  const int L = q.top_p, B = st.batch;
  bool ok = true;
  uint32_t flag = 0;
  if (X) {
    // this rank's list of batch row b -> slot [rank] of every arena, as
    // (token, score) word pairs carrying the epoch's flag
    flag = x_flag(e);
    for (int d = 0; d < x.world; ++d) {
      unsigned long long *reg = x_region(x, d, e) + (((int64_t)x.rank * B + b) * L) * 2;
      for (int a = threadIdx.x; a < L; a += FM_THREADS) {
        ll_store(reg + 2 * a, (uint32_t)mine_t[(int64_t)b * L + a], flag);
        ll_store(reg + 2 * a + 1, __float_as_uint(mine_s[(int64_t)b * L + a]), flag);
      }
    }
    n = x.world;
  }
  const int m = n * L;
  uint32_t *keys = reinterpret_cast<uint32_t *>(fm_dyn);
  int32_t *ids = reinterpret_cast<int32_t *>(keys + m);
  int32_t *pre_eq = ids + m;
  int32_t *pre_sel = pre_eq + n * (L + 1);
  int32_t *gp = pre_sel + n * (L + 1);
  uint8_t *fl = reinterpret_cast<uint8_t *>(gp + m);
  const unsigned long long *mine = X ? x_region(x, x.rank, e) : nullptr;
  constexpr int CB = 4;   // entries per thread per batch (independent loads)
  for (int i0 = 0; i0 < m; i0 += FM_THREADS * CB) {
    unsigned long long wv[2 * CB];
    int64_t offs[CB];
#pragma unroll
    for (int k = 0; k < CB; ++k) {
      const int i = i0 + k * FM_THREADS + threadIdx.x;
      const int j = i / L, a = i % L;
      offs[k] = ((int64_t)j * B + b) * L + a;
      if (X && i < m) {
        wv[2 * k] = ld_relaxed_sys(mine + 2 * offs[k]);
        wv[2 * k + 1] = ld_relaxed_sys(mine + 2 * offs[k] + 1);
      }
    }
#pragma unroll
    for (int k = 0; k < CB; ++k) {
      const int i = i0 + k * FM_THREADS + threadIdx.x;
      if (i >= m) continue;
      int32_t id;
      float sc;
      if (X) {
        id = (int32_t)ll_check(mine + 2 * offs[k], wv[2 * k], flag, ok, x.budget);
        sc = __uint_as_float(ll_check(mine + 2 * offs[k] + 1, wv[2 * k + 1], flag, ok, x.budget));
      } else {
        id = __ldcg(lt + offs[k]);
        sc = __ldcg(ls + offs[k]);
      }
      ids[i] = id;
      keys[i] = id >= 0 ? f2key(sc) : 0u;
    }
  }
  if (X && !ok)
    atomicOr(reinterpret_cast<unsigned long long *>(st.state + KIV_ST_ERROR),
             (unsigned long long)KIV_ERRBIT_WAIT_TIMEOUT);
  if (threadIdx.x < 64) s_valid[threadIdx.x] = 0;
  // a wait that gave up leaves some lists unread: select nothing
  if (__syncthreads_or(X && !ok)) {
    if (threadIdx.x == 0) {
      w.selcnt[b] = 0;
      if (b == 0) {
        st.state[KIV_ST_SEL] = 0;
        st.state[KIV_ST_SEL_LOCAL] = 0;
      }
    }
    if (X) x_advance(x, X_FINE, e);
    return;
  }
  // valid entries per list, one shared atomic per warp and list
  for (int i0 = threadIdx.x & ~31; i0 < m; i0 += FM_THREADS) {
    const int i = i0 + (threadIdx.x & 31);
    const bool v = i < m && ids[i] >= 0;
    const int j = (i < m ? i : m - 1) / L;
    const unsigned grp = __match_any_sync(KIV_FULL_MASK, j);
    const int c = __popc(__ballot_sync(KIV_FULL_MASK, v) & grp);
    if ((int)(threadIdx.x & 31) == __ffs(grp) - 1 && c) atomicAdd(&s_valid[j], c);
  }
  __syncthreads();
  int valid = 0;
  for (int j = 0; j < n; ++j) valid += s_valid[j];
  const int P = min(L, valid);
  uint32_t T = 0, need = 0;
  const bool all = P >= valid;
  if (P > 0 && !all) radix_threshold<FM_THREADS, 1>(keys, m, (uint32_t)P, sm, T, need);
  // ties at T: rank among equal keys by token id across all lists
  for (int i = threadIdx.x; i < m; i += FM_THREADS)
    fl[i] = (ids[i] >= 0 && !all && keys[i] == T) ? 1 : 0;
  __syncthreads();
  list_prefix_block(fl, m, n, L, gp, pre_eq, fm_scan);
  uint8_t *take = fl + m;
  for (int i = threadIdx.x; i < m; i += FM_THREADS) {
    const int j = i / L, a = i % L;
    bool s = ids[i] >= 0 && (all || keys[i] > T);
    if (!s && fl[i]) {
      int rank = pre_eq[j * (L + 1) + a];
      for (int o = 0; o < n; ++o)
        if (o != j) rank += pre_eq[o * (L + 1) + lower_bound_ids(ids + o * L, s_valid[o], ids[i])];
      s = rank < (int)need;
    }
    take[i] = s ? 1 : 0;
  }
  __syncthreads();
  list_prefix_block(take, m, n, L, gp, pre_sel, fm_scan);
  for (int i = threadIdx.x; i < m; i += FM_THREADS) {
    if (!take[i]) continue;
    const int j = i / L, a = i % L;
    if (sel) {
      // global position: selected entries of every list with a smaller id
      int pos = pre_sel[j * (L + 1) + a];
      for (int o = 0; o < n; ++o)
        if (o != j) pos += pre_sel[o * (L + 1) + lower_bound_ids(ids + o * L, s_valid[o], ids[i])];
      sel[(int64_t)b * L + pos] = ids[i];
    }
    if (j == st.shard_rank) sel_local[(int64_t)b * L + pre_sel[j * (L + 1) + a]] = ids[i];
  }
  if (threadIdx.x == 0) {
    w.selcnt[b] = pre_sel[st.shard_rank * (L + 1) + L];
    if (b == 0) {
      st.state[KIV_ST_SEL] = P;
      st.state[KIV_ST_SEL_LOCAL] = pre_sel[st.shard_rank * (L + 1) + L];
    }
  }
  if (X) x_advance(x, X_FINE, e);
}

template <typename T, int LPR, int VPL, int RCH>
static kiv_status launch_fs(const kiv_store *st, const kiv_query *q, const Workspace &w,
                            cudaStream_t s) {
  const int D = st->head_dim, S = st->page_size;
  int tr = 1;
  while (tr * 2 <= S && (int64_t)tr * 2 * D * (int)sizeof(T) <= FS_TILE_BYTES) tr *= 2;
  const size_t qbytes = (size_t)q->num_query_heads * q->query_len * D * sizeof(float);
  const int stage_q = qbytes <= 64 * 1024 ? 1 : 0;
  const size_t smem = (size_t)FS_STAGES * tr * D * sizeof(T) + (size_t)((tr + 3) & ~3) * sizeof(float) +
                      (stage_q ? qbytes : 0);
  auto kern = fine_scores_kernel<T, LPR, VPL, RCH>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  int per_sm = 1;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, FS_THREADS, smem);
  per_sm = std::max(per_sm, 1);
  const int64_t units_cap = (int64_t)st->batch * (w.u_cap + 1) * ceil_div(S, tr);
  const int64_t grid = std::max<int64_t>(1, std::min<int64_t>(units_cap, (int64_t)sm_count() * per_sm));
  return cuda_status(launch_pdl(kern, dim3((unsigned)grid), dim3(FS_THREADS), smem, s, 1, *st, *q, w, tr, stage_q),
                     "fine_scores");
}

template <typename T>
static kiv_status dispatch_fs(const kiv_store *st, const kiv_query *q, const Workspace &w,
                              cudaStream_t s) {
  const int nv = st->head_dim / Elem<T>::V;
  const int rows_kv = (q->num_query_heads / st->num_kv_heads) * q->query_len;
  const bool small = rows_kv <= 4;
#define KIV_FS(LPR, VPL) \
  return small ? launch_fs<T, LPR, VPL, 4>(st, q, w, s) : launch_fs<T, LPR, VPL, 8>(st, q, w, s)
  if (nv <= 2) KIV_FS(2, 1);
  if (nv <= 4) KIV_FS(4, 1);
  if (nv <= 8) KIV_FS(8, 1);
  if (nv <= 16) KIV_FS(16, 1);
  if (nv <= 32) KIV_FS(32, 1);
  if (nv <= 64) KIV_FS(32, 2);
#undef KIV_FS
  return KIV_ERR_UNSUPPORTED;
}

kiv_status launch_fine_score(const kiv_store *st, const kiv_query *q, const Workspace &w, cudaStream_t s) {
  if (fine_tc_eligible(st, q)) return launch_fine_score_tc(st, q, w, s);
  if (prefill_tc_eligible(st, q)) return launch_prefill_fine_scores(st, q, w, s);
  KIV_CHECK(launch_union(st, w, s));
  KIV_CHECK(launch_stage_union(st, w, s));
  switch (st->dtype) {
    case KIV_DTYPE_F32: return dispatch_fs<float>(st, q, w, s);
    case KIV_DTYPE_BF16: return dispatch_fs<__nv_bfloat16>(st, q, w, s);
    case KIV_DTYPE_F16: return dispatch_fs<__half>(st, q, w, s);
  }
  return KIV_ERR_UNSUPPORTED;
}

kiv_status launch_fine(const kiv_store *st, const kiv_query *q, const Workspace &w, int32_t *sel,
                       float *sel_scores, cudaStream_t s) {
  const kiv_status rc = launch_fine_score(st, q, w, s);
  if (rc != KIV_OK) return rc;
  return launch_fine_topk(st, q, w, sel, sel_scores, s);
}

// select: one cluster of SEL_CLUSTER CTAs per batch row (x: candidate exchange)
static kiv_status launch_select(const kiv_store *st, const kiv_query *q, const Workspace &w, int32_t *sel,
                                float *sel_scores, int32_t *sel_local, cudaStream_t s, const XArgs *x) {
  const int cap = (int)std::max<int64_t>(16, std::min<int64_t>(SL_CAP, align_up(w.c_cap, 16)));
  const int ucap = (int)std::min<int64_t>(SL_UCAP, align_up(w.u_cap, 4));
  const int kcap = (int)std::min<int64_t>(SL_KCAP, align_up(ceil_div(w.c_cap, SEL_CLUSTER), 16) + 16);
  const size_t smem = (size_t)cap * 13 + (size_t)SL_BND * 8 + (size_t)ucap * 4 + (size_t)kcap * 4;
  cudaError_t e;
  if (x) {
    auto kern = fine_select_kernel<SEL_CLUSTER, true>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    e = launch_pdl(kern, dim3((unsigned)(st->batch * SEL_CLUSTER)), dim3(SL_THREADS), smem, s, SEL_CLUSTER, *st,
                   *q, w, sel, sel_scores, cap, ucap, kcap, sel_local, *x);
  } else {
    auto kern = fine_select_kernel<SEL_CLUSTER, false>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    e = launch_pdl(kern, dim3((unsigned)(st->batch * SEL_CLUSTER)), dim3(SL_THREADS), smem, s, SEL_CLUSTER, *st,
                   *q, w, sel, sel_scores, cap, ucap, kcap, (int32_t *)nullptr, XArgs{});
  }
  return cuda_status(e, "fine_select");
}

kiv_status launch_fine_topk(const kiv_store *st, const kiv_query *q, const Workspace &w, int32_t *sel,
                            float *sel_scores, cudaStream_t s) {
  return launch_select(st, q, w, sel, sel_scores, nullptr, s, nullptr);
}

bool fine_exchange_eligible(const kiv_store *st, const kiv_query *q) {
  const Workspace w = workspace_layout(st, q, nullptr);
  const int rows_kv = (q->num_query_heads / st->num_kv_heads) * q->query_len;
  // (<= 16 query rows per KV head: the shapes whose attention reads peer rows too)
  return repl_summaries(*st) && st->host_capacity == 0 && fine_tc_eligible(st, q) && rows_kv <= 16 &&
         w.u_cap <= 8192 && (int64_t)st->batch * SEL_CLUSTER <= sm_count();
}

kiv_status launch_fine_exchange_select(const kiv_store *st, const kiv_query *q, const Workspace &w, int32_t *sel,
                                       int32_t *sel_local, cudaStream_t s, const XArgs &x) {
  return launch_select(st, q, w, sel, nullptr, sel_local, s, &x);
}

kiv_status launch_fine_merge(const kiv_store *st, const kiv_query *q, const Workspace &w,
                             const float *ls, const int32_t *lt, int32_t n, int32_t *sel,
                             int32_t *sel_local, cudaStream_t s, const XArgs *x) {
  const int nl = x ? x->world : n;
  const int64_t m = (int64_t)nl * q->top_p;
  const size_t smem = (size_t)m * 12 + (size_t)nl * (q->top_p + 1) * 8 + (size_t)m * 2 + 16;
  if (smem > 200 * 1024 || nl > 64) {
    set_error("fine_merge: %d lists of %d entries exceed the shared-memory merge", nl, q->top_p);
    return KIV_ERR_CAPACITY;
  }
  cudaError_t e;
  if (x) {
    cudaFuncSetAttribute(fine_merge_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    e = launch_pdl(fine_merge_kernel<true>, dim3((unsigned)st->batch), dim3(FM_THREADS), smem, s, 1, *st, *q, w,
                   (const float *)nullptr, (const int32_t *)nullptr, nl, sel, sel_local, *x, ls, lt);
  } else {
    cudaFuncSetAttribute(fine_merge_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    e = launch_pdl(fine_merge_kernel<false>, dim3((unsigned)st->batch), dim3(FM_THREADS), smem, s, 1, *st, *q, w,
                   ls, lt, n, sel, sel_local, XArgs{}, (const float *)nullptr, (const int32_t *)nullptr);
  }
  if (e != cudaSuccess) return cuda_status(e, "fine_merge");
  return cuda_status(cudaGetLastError(), "fine_merge");
}

}  // namespace kiv
