// Kernels (b) and (c) for prefill-shaped queries (a chunk of Q positions,
// G*Q > 32 query rows per KV head): coarse and fine scoring as tensor-core
// contractions on tcgen05.
//
// Same results as the decode-shaped scorers (coarse.cu, fine.cu, fine_tc.cu),
// restating kiv/cold_store.py:203-230 (coarse: s = scaling * <q, summary> per
// query row and page) and :332-338 (fine: per candidate token, the max over
// all query rows of all KV heads of scaling * <q, k>).  With thousands of
// query rows per KV head the work is a dense GEMM (c4: 2*32*4096*C*96 FLOP
// per chunk), so the query rows are the resident operand:
//
//  * the G*Q rows of a KV head are cut into blocks of `nt` rows (one head,
//    nt consecutive positions; MMA N = nt <= 256); a CTA keeps `nres` blocks
//    in shared memory (one 4-D TMA box per block and 32-element slice of D,
//    SWIZZLE_64B) and streams 128-row tiles of keys (fine: one candidate page
//    of one KV head; coarse: 128 page summaries) through a TMA ring;
//  * one MMA chain (D/16 tcgen05.mma, M = 128, N = nt, K = D) per resident
//    block and tile, alternating between two TMEM accumulators so the
//    epilogue drains one while the next is computed;
//  * epilogue (4 warps, thread = tile row): fine -- max over the valid
//    columns of every chain, then one red.max of the order-preserving key
//    into the batch row's candidate keys (partial maxima from other CTAs,
//    blocks and KV heads meet there); coarse -- every score stored at
//    scores[row][page] (coalesced: a warp writes 32 consecutive pages).
//
// CTA i serves block group i % ngr of every KV head and tiles j, j + nj, ...
// (j = i / ngr) of it, so the ngr CTAs that read the same key tile do so at
// about the same time (one DRAM read, the rest from L2).  Every load targets
// only this CTA.
#include <algorithm>

#include "internal.h"
#include "select.cuh"
#include "tc.cuh"

namespace kiv {

constexpr int PF_EPI = 8;             // epilogue warps: two per TMEM lane quadrant (column halves)
constexpr int PF_THREADS = 32 * (PF_EPI + 2);   // + warp 8 TMA producer, warp 9 MMA issuer
constexpr int PF_TILE = 128;          // tile rows (MMA M): tokens of a page, or page summaries
constexpr int PF_BOX = 32;            // elements per TMA box along D (64 bytes, SWIZZLE_64B)
constexpr int PF_MAX_STAGES = 6;
constexpr int AH_THREADS = 512;       // histogram of the candidate keys

struct PfGeom {
  int nt;        // query rows per block (MMA N), multiple of 16
  int nres;      // blocks resident per CTA
  int tblocks;   // blocks per query head: ceil(Q / nt)
  int rb;        // blocks per KV head: G * tblocks
  int ngr;       // block groups per KV head: ceil(rb / nres)
  int nj;        // CTAs per block group
  int stages;    // key tile ring depth
  size_t smem;
};

template <bool BF16, bool COARSE>
__global__ void __launch_bounds__(PF_THREADS, 1)
prefill_scores_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap qmap,
                      kiv_store st, kiv_query q, Workspace w, PfGeom g) {
  extern __shared__ uint8_t pf_dyn[];
  __shared__ uint64_t full[PF_MAX_STAGES], empty[PF_MAX_STAGES], acc_full[2], acc_empty[2], q_full, q_empty;
  __shared__ uint32_t s_tmem;
  __shared__ int s_fail;
  __shared__ uint32_t s_wmax[PF_EPI];
  __shared__ float s_wsum[PF_EPI];
  __shared__ float s_half[2][PF_TILE];   // column-half maxima of the tile rows (two tiles in flight)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int D = st.head_dim, H = st.num_kv_heads, S = st.page_size;
  const int Hq = q.num_query_heads, Q = q.query_len, G = Hq / H;
  const int nbox = D / PF_BOX;
  const uint32_t box_q = (uint32_t)g.nt * (PF_BOX * 2);       // bytes of one query box
  const uint32_t box_k = (uint32_t)PF_TILE * (PF_BOX * 2);    // bytes of one key box
  const uint32_t tile_bytes = box_k * nbox;
  const uint32_t tcols = 2 * g.nt <= 32 ? 32u : (2 * g.nt <= 64 ? 64u : (2 * g.nt <= 128 ? 128u : (2 * g.nt <= 256 ? 256u : 512u)));
  const int grp = blockIdx.x % g.ngr, j = blockIdx.x / g.ngr;
  const int rb0 = grp * g.nres;
  const int nb = std::min(g.nres, g.rb - rb0);

  // 1024-byte aligned carve-up: [stages][nbox][128 x 64 B] [nres][nbox][nt x 64 B]
  const uint32_t base_addr = smem_u32(pf_dyn);
  uint8_t *smem = pf_dyn + ((1024 - (base_addr & 1023)) & 1023);
  uint8_t *stage_mem = smem;
  uint8_t *qmem = stage_mem + (size_t)g.stages * tile_bytes;

  // ---- prologue (overlaps the previous kernel's tail under PDL)
  if (threadIdx.x == 0) {
    for (int s = 0; s < g.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], PF_EPI);
    }
    mbar_init(&q_full, 1);
    mbar_init(&q_empty, 1);
    mbar_fence_init();
    s_fail = 0;
  }
  if (warp == 0) {
    tc::tmem_alloc(&s_tmem, tcols);
    tc::tmem_relinquish();
  }
  if (threadIdx.x == 32 * PF_EPI) {
    tc::prefetch_map(&kmap);
    tc::prefetch_map(&qmap);
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = s_tmem;
  griddep_wait();
  const int64_t cold = st_ld(st.state, KIV_ST_COLD_LEN);
  const int64_t np_global = cold / S;
  const int64_t partial = cold % S;
  const bool part_owned = partial > 0 && (np_global % st.shard_count) == st.shard_rank;
  int64_t U = 0;
  if (COARSE) {
    clear_stale_marks(st, w, coarse_pages(st, np_global));   // bits of the page marks
    if (blockIdx.x == 0 && threadIdx.x == 0) {
      st.state[KIV_ST_COARSE_MAX] = 0;
      st.state[KIV_ST_COARSE_SUM] = 0;
    }
  } else {
    U = st_ld(st.state, KIV_ST_UNION);
  }
  // units of one (batch row, KV head): coarse -- blocks of 128 local pages;
  // fine -- the union pages plus the partial page
  // coarse: the pages this shard scores (all of them with replicated summaries)
  const int64_t np_scored = coarse_pages(st, np_global);
  const int64_t units = COARSE ? (np_scored + PF_TILE - 1) / PF_TILE : U + (part_owned ? 1 : 0);
  const int64_t my_units = (nb > 0 && units > j) ? (units - j + g.nj - 1) / g.nj : 0;
  const int64_t BH = (int64_t)st.batch * H;

  bool ok = true;
  if (warp == PF_EPI) {
    if (lane == 0 && my_units > 0) {
      // ------------------------------------------------ TMA producer
      int64_t t = 0;
      for (int64_t bh = 0; bh < BH && ok; ++bh) {
        const int b = (int)(bh / H), kvh = (int)(bh % H);
        // this KV head's query blocks, once the MMAs on the previous ones are done
        if (bh > 0 && !mbar_wait_bounded(&q_empty, (uint32_t)((bh - 1) & 1))) { ok = false; break; }
        mbar_arrive_tx(&q_full, (uint32_t)nb * nbox * box_q);
        for (int i = 0; i < nb; ++i) {
          const int rbi = rb0 + i, gi = rbi / g.tblocks, tb = rbi % g.tblocks;
          for (int jb = 0; jb < nbox; ++jb)
            tc::tma_load_4d(qmem + ((size_t)i * nbox + jb) * box_q, &qmap, PF_BOX * jb, tb * g.nt, kvh * G + gi, b,
                            &q_full);
        }
        for (int64_t k = 0; k < my_units; ++k, ++t) {
          const int s = (int)(t % g.stages);
          if (t >= g.stages && !mbar_wait_bounded(&empty[s], (uint32_t)((t / g.stages - 1) & 1))) {
            ok = false;
            break;
          }
          const int64_t u = j + k * g.nj;
          int32_t y;
          if (COARSE) {
            y = (int32_t)(bh * w.np_cap + u * PF_TILE);
          } else {
            const int64_t page = u < U ? (int64_t)w.uni[u] : np_global;
            y = (int32_t)(bh * st.cold_capacity + page_slot(st, w, page / st.shard_count) * S);
          }
          mbar_arrive_tx(&full[s], tile_bytes);
          for (int jb = 0; jb < nbox; ++jb)
            tc::tma_load_2d(stage_mem + (size_t)s * tile_bytes + (size_t)jb * box_k, &kmap, PF_BOX * jb, y, &full[s]);
        }
      }
      if (!ok) s_fail = 1;
    }
  } else if (warp == PF_EPI + 1) {
    if (lane == 0 && my_units > 0) {
      // ------------------------------------------------ MMA issuer
      const uint32_t idesc = tc::idesc_f16(BF16, PF_TILE, g.nt);
      int64_t t = 0, c = 0;
      for (int64_t bh = 0; bh < BH && ok; ++bh) {
        if (!mbar_wait_bounded(&q_full, (uint32_t)(bh & 1))) { ok = false; break; }
        tc::fence_after_sync();
        for (int64_t k = 0; k < my_units && ok; ++k, ++t) {
          const int s = (int)(t % g.stages);
          if (!mbar_wait_bounded(&full[s], (uint32_t)((t / g.stages) & 1))) { ok = false; break; }
          tc::fence_after_sync();
          const uint32_t a0 = smem_u32(stage_mem + (size_t)s * tile_bytes);
          for (int i = 0; i < nb; ++i, ++c) {
            const int a = (int)(c & 1);
            if (c >= 2 && !mbar_wait_bounded(&acc_empty[a], (uint32_t)(((c >> 1) - 1) & 1))) { ok = false; break; }
            tc::fence_after_sync();
            const uint32_t b0 = smem_u32(qmem + (size_t)i * nbox * box_q);
            for (int kk = 0; kk < D / 16; ++kk) {
              const int jb = kk >> 1, sub = kk & 1;
              const uint64_t ad = tc::sdesc_k64(a0 + jb * box_k + sub * 32);
              const uint64_t bd = tc::sdesc_k64(b0 + jb * box_q + sub * 32);
              tc::mma_f16(tmem + (uint32_t)(a * g.nt), ad, bd, idesc, kk > 0 ? 1u : 0u);
            }
            tc::commit(&acc_full[a]);
          }
          tc::commit(&empty[s]);
        }
        tc::commit(&q_empty);
      }
      if (!ok) s_fail = 1;
    }
  } else {
    // ------------------------------------------ epilogue, warps 0..PF_EPI-1
    // warp e reads TMEM lanes 32 * (e % 4) .. (its tile rows) and the 16-column
    // chunks e / 4, e / 4 + 2, ... of every accumulator
    const int quad = warp & 3, half = warp >> 2;
    const int row = quad * 32 + lane;   // tile row: token of the page (fine), page of the block (coarse)
    uint32_t kmax = 0;
    float ksum = 0.f;
    int64_t c = 0, tile = 0;
    // A failed wait (a bug upstream) turns `ok` off: the loops still run to the
    // end, without waiting, so the two warps of a quadrant meet at every barrier.
    for (int64_t bh = 0; bh < BH; ++bh) {
      const int b = (int)(bh / H), kvh = (int)(bh % H);
      for (int64_t k = 0; k < my_units; ++k, ++tile) {
        const int64_t u = j + k * g.nj;
        // independent partial maxima: the fmax chain is not one long dependency
        float m[8];
#pragma unroll
        for (int x = 0; x < 8; ++x) m[x] = -INFINITY;
        for (int i = 0; i < nb; ++i, ++c) {
          const int a = (int)(c & 1);
          if (ok && !mbar_wait_bounded(&acc_full[a], (uint32_t)((c >> 1) & 1))) ok = false;
          if (!ok) continue;
          tc::fence_after_sync();
          const int rbi = rb0 + i, gi = rbi / g.tblocks, t0 = (rbi % g.tblocks) * g.nt;
          const int valid = min(g.nt, Q - t0);
          const uint32_t taddr = tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(a * g.nt);
          if (COARSE) {
            const int64_t p = u * PF_TILE + row;
            const bool live = p < np_scored;
            float *dst = w.scores + (((int64_t)b * Hq + kvh * G + gi) * Q + t0) * w.np_cap + p;
            for (int c0 = 16 * half; c0 < g.nt; c0 += 32) {
              uint32_t r[16];
              tc::ld_32x16(taddr + c0, r);
              tc::wait_ld();
              if (live) {
#pragma unroll
                for (int cc = 0; cc < 16; ++cc) {
                  if (c0 + cc < valid) {
                    const float sc = __uint_as_float(r[cc]) * q.scaling;
                    dst[(int64_t)(c0 + cc) * w.np_cap] = sc;
                    const uint32_t key = f2key(sc);
                    kmax = key > kmax ? key : kmax;
                    ksum += sc;
                  }
                }
              }
            }
          } else if (valid == g.nt) {
            // this half's chunks (half, half + 2, ...; at most 8) in two TMEM
            // round trips of four (the register file of one SM sub-partition
            // holds three warps of this kernel)
            const int nch = (g.nt / 16 + 1 - half) / 2;
#pragma unroll
            for (int x0 = 0; x0 < 8; x0 += 4) {
              if (x0 < nch) {
                uint32_t r[4][16];
#pragma unroll
                for (int x = 0; x < 4; ++x)
                  if (x0 + x < nch) tc::ld_32x16(taddr + (uint32_t)((half + 2 * (x0 + x)) * 16), r[x]);
                tc::wait_ld();
#pragma unroll
                for (int x = 0; x < 4; ++x) {
                  if (x0 + x < nch) {
#pragma unroll
                    for (int cc = 0; cc < 16; ++cc) m[cc & 7] = fmaxf(m[cc & 7], __uint_as_float(r[x][cc]));
                  }
                }
              }
            }
          } else {
            for (int c0 = 16 * half; c0 < g.nt; c0 += 32) {
              uint32_t r[16];
              tc::ld_32x16(taddr + c0, r);
              tc::wait_ld();
#pragma unroll
              for (int cc = 0; cc < 16; ++cc)
                if (c0 + cc < valid) m[cc & 7] = fmaxf(m[cc & 7], __uint_as_float(r[cc]));
            }
          }
          tc::fence_before_sync();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acc_empty[a]);
        }
        if (!COARSE) {
          float mx = fmaxf(fmaxf(fmaxf(m[0], m[1]), fmaxf(m[2], m[3])), fmaxf(fmaxf(m[4], m[5]), fmaxf(m[6], m[7])));
          // the two column halves of a row meet in shared memory (named barrier per quadrant)
          if (half == 1) s_half[tile & 1][row] = mx;
          asm volatile("bar.sync %0, 64;" ::"r"(1 + quad) : "memory");
          if (half == 0) {
            mx = fmaxf(mx, s_half[tile & 1][row]);
            // scaling > 0: the max of the scaled scores is the scaled max
            const int n_tok = u < U ? PF_TILE : (int)partial;
            if (ok && row < n_tok) atomicMax(&w.agg[(int64_t)b * w.c_cap + u * S + row], f2key(mx * q.scaling));
          }
        }
      }
    }
    if (!ok) s_fail = 1;
    kmax = __reduce_max_sync(KIV_FULL_MASK, kmax);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ksum += __shfl_xor_sync(KIV_FULL_MASK, ksum, o);
    if (lane == 0) {
      s_wmax[warp] = kmax;
      s_wsum[warp] = ksum;
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (threadIdx.x == 0) {
    if (COARSE && my_units > 0) {
      uint32_t mk = 0;
      double sm = 0.0;
      for (int i = 0; i < PF_EPI; ++i) {
        mk = s_wmax[i] > mk ? s_wmax[i] : mk;
        sm += s_wsum[i];
      }
      atomicMax(reinterpret_cast<unsigned long long *>(&w.cstat[0]), (unsigned long long)mk);
      atomicAdd(reinterpret_cast<double *>(&w.cstat[1]), sm);
    }
    if (s_fail)
      atomicOr(reinterpret_cast<unsigned long long *>(st.state + KIV_ST_ERROR),
               (unsigned long long)KIV_ERRBIT_WAIT_TIMEOUT);
  }
  if (warp == 0) tc::tmem_dealloc(tmem, tcols);
}

// candidates of this fine pass: C = U * S (+ the partial page on its owner)
__device__ __forceinline__ int64_t pf_candidates(const kiv_store &st) {
  const int64_t cold = st_ld(st.state, KIV_ST_COLD_LEN);
  const int S = st.page_size;
  const int64_t npg = cold / S, partial = cold % S;
  const bool part_owned = partial > 0 && (npg % st.shard_count) == st.shard_rank;
  return st_ld(st.state, KIV_ST_UNION) * S + (part_owned ? partial : 0);
}

// Zero the candidate keys before the scorer's red.max (key 0 is below the key
// of every float) and reset the fine score statistics of the step.
__global__ void agg_prep_kernel(kiv_store st, Workspace w) {
  griddep_wait();
  const int64_t C = pf_candidates(st);
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    st.state[KIV_ST_FINE_MAX] = 0;
    st.state[KIV_ST_FINE_SUM] = 0;
  }
  const int64_t n4 = C / 4;
  for (int b = 0; b < st.batch; ++b) {
    uint32_t *row = w.agg + (int64_t)b * w.c_cap;    // c_cap is a multiple of the page size: 16-byte rows
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x)
      reinterpret_cast<uint4 *>(row)[i] = make_uint4(0, 0, 0, 0);
    for (int64_t i = n4 * 4 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < C;
         i += (int64_t)gridDim.x * blockDim.x)
      row[i] = 0u;
  }
}

// First radix-select histogram (key >> 21) and score statistics of every
// batch row's candidate keys, which the select kernel expects from the scorer.
__global__ void __launch_bounds__(AH_THREADS) agg_hist_kernel(kiv_store st, Workspace w, int cpb) {
  __shared__ uint32_t hist[SEL_BINS];
  __shared__ uint32_t s_wmax[AH_THREADS / 32];
  __shared__ float s_wsum[AH_THREADS / 32];
  for (int i = threadIdx.x; i < SEL_BINS; i += AH_THREADS) hist[i] = 0;
  griddep_wait();
  const int64_t C = pf_candidates(st);
  const int b = blockIdx.x / cpb, cj = blockIdx.x % cpb;
  __syncthreads();
  uint32_t kmax = 0;
  float ksum = 0.f;
  const uint32_t *row = w.agg + (int64_t)b * w.c_cap;
  for (int64_t c = (int64_t)cj * AH_THREADS + threadIdx.x; c < C; c += (int64_t)cpb * AH_THREADS) {
    const uint32_t key = row[c];
    hist_add(hist, key >> 21);
    kmax = key > kmax ? key : kmax;
    ksum += key2f(key);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < SEL_BINS; i += AH_THREADS)
    if (hist[i]) atomicAdd(&w.fhist[(int64_t)b * SEL_BINS + i], hist[i]);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  kmax = __reduce_max_sync(KIV_FULL_MASK, kmax);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ksum += __shfl_xor_sync(KIV_FULL_MASK, ksum, o);
  if (lane == 0) {
    s_wmax[warp] = kmax;
    s_wsum[warp] = ksum;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t mk = 0;
    double sm = 0.0;
    for (int i = 0; i < AH_THREADS / 32; ++i) {
      mk = s_wmax[i] > mk ? s_wmax[i] : mk;
      sm += s_wsum[i];
    }
    if (mk) {
      atomicMax(reinterpret_cast<unsigned long long *>(&w.fstat[2 * b]), (unsigned long long)mk);
      atomicAdd(reinterpret_cast<double *>(&w.fstat[2 * b + 1]), sm);
    }
  }
}

// ------------------------------------------------------------------ host
bool prefill_shape(const kiv_store *st, const kiv_query *q) {
  const int64_t rows_kv = (int64_t)(q->num_query_heads / st->num_kv_heads) * q->query_len;
  const int D = st->head_dim;
  return (st->dtype == KIV_DTYPE_BF16 || st->dtype == KIV_DTYPE_F16) && st->page_size == PF_TILE &&
         D % PF_BOX == 0 && D >= PF_BOX && D <= 256 && rows_kv > 32 && q->query_len < (1 << 24) &&
         (int64_t)st->batch * st->num_kv_heads * st->cold_capacity < (1ll << 31) &&
         getenv("KIV_DISABLE_TCGEN05") == nullptr;
}

bool prefill_tc_eligible(const kiv_store *st, const kiv_query *q) {
  auto ok_stride = [](int64_t s) { return s > 0 && s % 8 == 0; };   // 16-byte multiples for TMA
  return prefill_shape(st, q) && (reinterpret_cast<uintptr_t>(q->q) & 15) == 0 && ok_stride(q->stride_b) &&
         ok_stride(q->stride_h) && ok_stride(q->stride_t);
}

// block size, residency and ring depth for this query shape (dynamic shared
// memory at most 220 KB, at least two key stages)
static kiv_status pf_geom(const kiv_store *st, const kiv_query *q, bool coarse, const Workspace &w, PfGeom &g) {
  const int D = st->head_dim, Q = q->query_len, G = q->num_query_heads / st->num_kv_heads;
  const size_t tile = (size_t)PF_TILE * D * 2, budget = 220 * 1024;
  int nt = (int)std::min<int64_t>(256, align_up(Q, 16));
  for (;;) {
    const int tblocks = (int)ceil_div(Q, nt), rb = G * tblocks;
    const size_t blk = (size_t)nt * D * 2;
    int nres = (int)std::max<size_t>(1, std::min<size_t>((size_t)rb, (128 * 1024) / blk));
    for (; nres >= 1; --nres) {
      const size_t fixed = 1024 + (size_t)nres * blk;
      if (fixed + 2 * tile > budget) continue;
      g.nt = nt;
      g.nres = nres;
      g.tblocks = tblocks;
      g.rb = rb;
      g.ngr = (int)ceil_div(rb, nres);
      g.stages = (int)std::min<size_t>(4, (budget - fixed) / tile);
      g.smem = fixed + (size_t)g.stages * tile;
      const int64_t units_cap = coarse ? ceil_div(w.np_cap, PF_TILE) : w.u_cap + 1;
      g.nj = (int)std::max<int64_t>(1, std::min<int64_t>(units_cap, sm_count() / g.ngr));
      return KIV_OK;
    }
    if (nt <= 16) return KIV_ERR_UNSUPPORTED;
    nt = std::max(16, nt / 32 * 16);
  }
}

static kiv_status launch_prefill_scores(const kiv_store *st, const kiv_query *q, const Workspace &w,
                                        cudaStream_t s, bool coarse) {
  PfGeom g;
  KIV_CHECK(pf_geom(st, q, coarse, w, g));
  const int D = st->head_dim;
  const bool bf = st->dtype == KIV_DTYPE_BF16;
  const int64_t bh = (int64_t)st->batch * st->num_kv_heads;
  CUtensorMap kmap, qmap;
  {
    const uint64_t dims[2] = {(uint64_t)D, (uint64_t)(bh * (coarse ? w.np_cap : st->cold_capacity))};
    const uint64_t strides[1] = {(uint64_t)D * 2};
    const uint32_t box[2] = {PF_BOX, PF_TILE};
    KIV_CHECK(encode_tiled(&kmap, st->dtype, 2, coarse ? st->summaries : st->cold_k, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_64B));
  }
  {
    const uint64_t dims[4] = {(uint64_t)D, (uint64_t)q->query_len, (uint64_t)q->num_query_heads,
                              (uint64_t)st->batch};
    const uint64_t strides[3] = {(uint64_t)q->stride_t * 2, (uint64_t)q->stride_h * 2, (uint64_t)q->stride_b * 2};
    const uint32_t box[4] = {PF_BOX, (uint32_t)g.nt, 1, 1};
    KIV_CHECK(encode_tiled(&qmap, st->dtype, 4, q->q, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_64B));
  }
  const int64_t grid = (int64_t)g.ngr * g.nj;
  cudaError_t e;
#define KIV_PF_LAUNCH(BF, CO)                                                                            \
  do {                                                                                                   \
    cudaFuncSetAttribute(prefill_scores_kernel<BF, CO>, cudaFuncAttributeMaxDynamicSharedMemorySize,       \
                         (int)g.smem);                                                                   \
    e = launch_pdl(prefill_scores_kernel<BF, CO>, dim3((unsigned)grid), dim3(PF_THREADS), g.smem, s, 1, kmap, \
                   qmap, *st, *q, w, g);                                                                 \
  } while (0)
  if (bf && coarse) KIV_PF_LAUNCH(true, true);
  else if (bf) KIV_PF_LAUNCH(true, false);
  else if (coarse) KIV_PF_LAUNCH(false, true);
  else KIV_PF_LAUNCH(false, false);
#undef KIV_PF_LAUNCH
  return cuda_status(e, coarse ? "prefill_coarse_scores" : "prefill_fine_scores");
}

kiv_status launch_prefill_coarse_scores(const kiv_store *st, const kiv_query *q, const Workspace &w,
                                        cudaStream_t s) {
  return launch_prefill_scores(st, q, w, s, true);
}

// union -> zeroed keys -> tensor-core scoring (red.max) -> histogram and stats
kiv_status launch_prefill_fine_scores(const kiv_store *st, const kiv_query *q, const Workspace &w,
                                      cudaStream_t s) {
  KIV_CHECK(launch_union(st, w, s));
  KIV_CHECK(launch_stage_union(st, w, s));
  const int64_t prep_grid = std::max<int64_t>(1, std::min<int64_t>(ceil_div(w.c_cap, 4 * 256), sm_count() * 4));
  KIV_CHECK(cuda_status(launch_pdl(agg_prep_kernel, dim3((unsigned)prep_grid), dim3(256), 0, s, 1, *st, w),
                        "agg_prep"));
  KIV_CHECK(launch_prefill_scores(st, q, w, s, false));
  const int cpb = (int)std::max<int64_t>(1, std::min<int64_t>(ceil_div(w.c_cap, AH_THREADS * 8),
                                                               std::max(1, 2 * sm_count() / st->batch)));
  return cuda_status(launch_pdl(agg_hist_kernel, dim3((unsigned)(st->batch * cpb)), dim3(AH_THREADS), 0, s, 1,
                                *st, w, cpb),
                     "agg_hist");
}

}  // namespace kiv
