// Kernel (c), tensor-core form: fine token scoring on tcgen05.
//
// Same result as fine_scores_kernel (fine.cu): for every candidate token of
// the union pages (and the partial page), key = f2key(max over the G*Q query
// rows of every KV head of scaling * <q, k>) -- restating kiv/cold_store.py:
// 332-338.  Here one candidate page (128 tokens) of one KV head is one MMA
// tile: M = 128 tokens, N = 16 or 32 query rows (zero-padded), K = head_dim.
//
//  warp 4 (one thread): TMA producer -- 2-D tensor-map loads (SWIZZLE_128B,
//          boxes of 64 elements x 128 rows) of the K tile into a 3/4-stage
//          shared-memory ring, completing on per-stage mbarriers;
//  warp 5 (one thread): MMA issuer -- head_dim/16 tcgen05.mma per tile into
//          one of two TMEM accumulators, tcgen05.commit to free the stage and
//          to publish the accumulator;
//  warps 0-3: epilogue -- tcgen05.ld of the accumulator (thread i = token i),
//          max over the valid query rows, running max over KV heads, key
//          store, and the first radix-select histogram + score stats of the
//          batch row (so the select kernel skips its first pass).
// The query rows are written once into shared memory in the same swizzled
// K-major layout.  Every load targets only this CTA.  CTAs are grouped by
// batch row (each group stages its row's queries once).  Used when the store
// is 16-bit, page_size == 128, head_dim is a multiple of 64 (<= 256) and
// G*Q <= 32; otherwise fine_scores_kernel runs.
//
// Candidate exchange (XC, page-sharded stores with replicated summaries):
// every shard holds the whole page union (the coarse pass is exact on each
// shard), scores the union pages it owns, and stores each key at its global
// candidate position (union position * S + token; the partial page after the
// union) into every shard's exchange arena, as a flagged 64-bit word.  Each
// shard's select then reads all candidates and takes the exact global top-P
// itself, so no list merge follows.
#include <algorithm>

#include "exchange.cuh"
#include "internal.h"
#include "select.cuh"
#include "tc.cuh"

namespace kiv {

constexpr int TC_THREADS = 192;
constexpr int TC_PAGE = 128;
constexpr int64_t TC_UNION_INLINE = 8192;   // largest union built inside the fine scorer

struct TcGeom {
  int64_t U, np_global, partial, per_b;
  bool part_owned;
};

// COARSE == false: fine scoring over candidate pages (key per token, max over rows)
// COARSE == true:  coarse scoring over page summaries (score per row and page;
//                  the per-row top-k builds the rows' histograms from them)
// XC: candidate exchange (fine only), keys to every shard's arena (see above)
template <bool BF16, bool COARSE, bool XC>
__global__ void __launch_bounds__(TC_THREADS, 1)
scores_tc_kernel(const __grid_constant__ CUtensorMap kmap, kiv_store st, kiv_query q, Workspace w,
                 int ncols, int stages, int union_inline, int cpb, const __grid_constant__ XArgs x) {
  using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  extern __shared__ uint8_t tc_dyn[];
  __shared__ uint64_t full[4], empty[4], acc_full[2], acc_empty[2], ubar;
  __shared__ uint32_t s_tmem;
  __shared__ int s_fail;
  __shared__ uint32_t s_wmax[4];
  __shared__ float s_wsum[4];
  __shared__ int s_psum[TC_THREADS / 32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int D = st.head_dim, H = st.num_kv_heads, S = st.page_size;
  const int Hq = q.num_query_heads, Q = q.query_len, G = Hq / H;
  const int rows_kv = G * Q;
  const int nbox = D / 64;
  const uint32_t tile_bytes = (uint32_t)TC_PAGE * D * sizeof(T);
  const uint32_t qbox_bytes = (uint32_t)ncols * 128;
  // CTAs are grouped by batch row: cpb consecutive CTAs serve batch row b,
  // whose query rows are staged once
  const int b = blockIdx.x / cpb, cj = blockIdx.x % cpb;

  // 1024-byte aligned carve-up: [stages][tile] [H][nbox][qbox] [hist 2048] [union list]
  // (XC: [own positions] after the union list)
  const uint32_t base_addr = smem_u32(tc_dyn);
  uint8_t *smem = tc_dyn + ((1024 - (base_addr & 1023)) & 1023);
  uint8_t *stage_mem = smem;
  uint8_t *qmem = stage_mem + (size_t)stages * tile_bytes;
  uint32_t *hist = reinterpret_cast<uint32_t *>(qmem + (size_t)H * nbox * qbox_bytes);
  int32_t *ulist = reinterpret_cast<int32_t *>(hist + SEL_BINS);
  int32_t *own = ulist + w.u_cap;

  // ---- prologue: independent of the previous kernel in the stream (with
  // programmatic dependent launch it overlaps that kernel's tail).  The
  // query was written before the layer-step's first kernel.
  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 4);
    }
    mbar_init(&ubar, 1);
    mbar_fence_init();
    s_fail = 0;
  }
  if (warp == 0) {
    tc::tmem_alloc(&s_tmem, (uint32_t)(2 * ncols < 32 ? 32 : 2 * ncols));
    tc::tmem_relinquish();
  }
  if (threadIdx.x == 32 * 4) tc::prefetch_map(&kmap);
  // query rows of batch row b -> swizzled K-major tiles [kvh][box][ncols x 128 B]
  const T *qb = reinterpret_cast<const T *>(q.q) + (int64_t)b * q.stride_b;
  for (int e = threadIdx.x; e < H * ncols * (D / 8); e += TC_THREADS) {
    const int chunk = e % (D / 8);            // 16-byte chunk along D
    const int n = (e / (D / 8)) % ncols;      // query row within the KV head
    const int kvh = e / ((D / 8) * ncols);
    uint4 v = make_uint4(0, 0, 0, 0);
    if (n < rows_kv) {
      const int h = kvh * G + n / Q, tq = n % Q;
      v = ld16(qb + h * q.stride_h + tq * q.stride_t + chunk * 8);
    }
    const int box = chunk / 8, c = chunk % 8;
    uint8_t *dst = qmem + ((size_t)kvh * nbox + box) * qbox_bytes + n * 128 + ((c ^ (n & 7)) * 16);
    *reinterpret_cast<uint4 *>(dst) = v;
  }
  for (int i = threadIdx.x; i < SEL_BINS; i += TC_THREADS) hist[i] = 0;
  tc::fence_proxy_async_smem();
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = s_tmem;
  // ---- the previous kernel's results (state, union) are needed from here on;
  // the cold length too (an eviction may be the kernel right before this one)
  griddep_wait();
  const int64_t bh0 = (int64_t)b * H;
  // coarse pass: this CTA's first tile (page block cj of KV head 0 -- inside
  // the summaries' capacity, cj < cpb <= blocks of np_cap) is loaded before
  // the cold length is known; pages past it are masked in the epilogue
  const bool coarse_first = COARSE && warp == 4 && lane == 0;
  if (coarse_first) {
    mbar_arrive_tx(&full[0], tile_bytes);
    for (int j = 0; j < nbox; ++j)
      tc::tma_load_2d(stage_mem + (size_t)j * TC_PAGE * 128, &kmap, 64 * j, (int32_t)(bh0 * w.np_cap + cj * TC_PAGE),
                      &full[0]);
  }
  // fine pass: the whole page-mark bitmap (its capacity, so the copy does not
  // wait for the cold length) comes in with one bulk copy into the still
  // unused stage ring, in flight while the state words load
  const uint32_t fbytes = (uint32_t)((((w.np_cap + 31) / 32) * 4 + 15) & ~15ll);
  const bool bulk = !COARSE && union_inline && (int64_t)fbytes <= (int64_t)stages * tile_bytes &&
                    fbytes < (1u << 20);
  if (bulk && threadIdx.x == 0) {
    mbar_arrive_tx(&ubar, fbytes);
    bulk_g2s(stage_mem, w.pbits, fbytes, &ubar);
  }
  const int64_t cold = st_ld(st.state, KIV_ST_COLD_LEN);
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    st.state[COARSE ? KIV_ST_COARSE_MAX : KIV_ST_FINE_MAX] = 0;
    st.state[COARSE ? KIV_ST_COARSE_SUM : KIV_ST_FINE_SUM] = 0;
  }

  TcGeom f;
  const int32_t *pages = w.uni;
  f.np_global = cold / S;
  f.partial = cold % S;
  f.part_owned = f.partial > 0 && (f.np_global % st.shard_count) == st.shard_rank;
  // page marks: one per local page, or per global page with replicated summaries
  const int64_t nmark = coarse_pages(st, f.np_global);
  const bool repl = repl_summaries(st);
  int64_t n_own = 0;   // XC: this shard's pages of the union
  if (COARSE) {
    clear_stale_marks(st, w, nmark);
    f.U = 0;
  } else if (union_inline) {
    // The page marks of a new coarse pass (copied above, before knowing
    // whether a coarse pass is pending, so that the reads share one round
    // trip): when one is, every CTA builds the sorted union from the marks
    // and CTA 0 also publishes it (the select kernel and the reuse path read
    // it from the workspace).
    // Global marks (replicated summaries) keep this shard's pages, or every
    // page with the candidate exchange.
    const int mrank = repl ? 0 : st.shard_rank, mcount = repl ? 1 : st.shard_count;
    const int fcount = repl && !XC ? st.shard_count : 1;
    const bool pending = st_ld(st.state, KIV_ST_UNION_PENDING) != 0;
    if (bulk && !mbar_wait_bounded(&ubar, 0)) s_fail = 1;
    if (pending) {
      if (bulk)
        f.U = union_from_bits<TC_THREADS, true>(reinterpret_cast<const uint32_t *>(stage_mem), nmark, ulist,
                                                (int)w.u_cap, mrank, mcount, s_psum, st.shard_rank, fcount);
      else
        f.U = union_from_bits<TC_THREADS, false>(w.pbits, nmark, ulist, (int)w.u_cap, mrank, mcount, s_psum,
                                                 st.shard_rank, fcount);
      if (blockIdx.x == 0) {
        for (int i = threadIdx.x; i < f.U; i += TC_THREADS) w.uni[i] = ulist[i];
        if (threadIdx.x == 0) st.state[KIV_ST_UNION] = f.U;
      }
      pages = ulist;
    } else {
      f.U = st_ld(st.state, KIV_ST_UNION);
      if (XC) {
        for (int i = threadIdx.x; i < f.U; i += TC_THREADS) ulist[i] = __ldcg(w.uni + i);
        __syncthreads();
        pages = ulist;
      }
    }
    if (XC) n_own = owned_positions<TC_THREADS>(ulist, (int)f.U, own, st.shard_rank, st.shard_count, s_psum);
    if (bulk) {
      // the stage ring is written by TMA next: order these generic reads first
      tc::fence_proxy_async_smem();
      __syncthreads();
    }
  } else {
    f.U = st_ld(st.state, KIV_ST_UNION);
  }
  f.per_b = (XC ? n_own : f.U) + (f.part_owned ? 1 : 0);
  // XC: the exchange epoch of the candidates (advanced by the select that reads them)
  const unsigned long long xe = XC ? x_epoch(x, X_CAND) : 0ull;
  // XC: global candidate position of unit u's first token
  auto unit_pos = [&](int64_t u) -> int64_t {
    if (!XC) return u * S;
    return u < n_own ? (int64_t)own[u] * S : f.U * S;
  };
  // per batch row b.  FINE: one unit per candidate page (tiles = its KV
  // heads); COARSE: one unit per block of 128 finalized local pages (tiles =
  // KV heads).  CTA cj of the row's cpb takes units cj, cj + cpb, ...
  // coarse: the pages this shard scores (all of them with replicated summaries)
  const int64_t np_scored = nmark;
  const int64_t units = COARSE ? (np_scored + TC_PAGE - 1) / TC_PAGE : f.per_b;
  const int64_t my_units = units > cj ? (units - cj + cpb - 1) / cpb : 0;
  const int64_t my_tiles = my_units * H;

  if (warp == 4) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer
      // (coarse: tile 0 is in flight already; with no tile to score, it is
      // waited for before the CTA exits)
      if (COARSE && my_tiles == 0 && !mbar_wait_bounded(&full[0], 0)) s_fail = 1;
      for (int64_t t = COARSE ? 1 : 0; t < my_tiles; ++t) {
        const int s = (int)(t % stages);
        if (t >= stages && !mbar_wait_bounded(&empty[s], (uint32_t)((t / stages - 1) & 1))) {
          s_fail = 1;
          break;
        }
        const int64_t u = cj + (t / H) * cpb;
        const int kvh = (int)(t % H);
        int32_t y;
        if (COARSE) {
          y = (int32_t)((bh0 + kvh) * w.np_cap + u * TC_PAGE);
        } else {
          const int64_t nu = XC ? n_own : f.U;
          const int64_t page = u < nu ? (int64_t)pages[XC ? own[u] : u] : f.np_global;
          const int64_t lp = page_slot(st, w, page / st.shard_count);
          y = (int32_t)((bh0 + kvh) * st.cold_capacity + lp * S);
        }
        mbar_arrive_tx(&full[s], tile_bytes);
        for (int j = 0; j < nbox; ++j)
          tc::tma_load_2d(stage_mem + (size_t)s * tile_bytes + (size_t)j * TC_PAGE * 128, &kmap, 64 * j, y,
                          &full[s]);
      }
    }
  } else if (warp == 5) {
    if (lane == 0) {
      // ------------------------------------------------ MMA issuer
      const uint32_t idesc = tc::idesc_f16(BF16, TC_PAGE, ncols);
      for (int64_t t = 0; t < my_tiles; ++t) {
        const int s = (int)(t % stages);
        const int a = (int)(t & 1);
        if (!mbar_wait_bounded(&full[s], (uint32_t)((t / stages) & 1))) { s_fail = 1; break; }
        if (t >= 2 && !mbar_wait_bounded(&acc_empty[a], (uint32_t)((t / 2 - 1) & 1))) { s_fail = 1; break; }
        tc::fence_after_sync();
        const int kvh = (int)(t % H);
        const uint32_t a0 = smem_u32(stage_mem + (size_t)s * tile_bytes);
        const uint32_t b0 = smem_u32(qmem + (size_t)kvh * nbox * qbox_bytes);
        for (int kk = 0; kk < D / 16; ++kk) {
          const int j = kk >> 2, sub = kk & 3;
          const uint64_t ad = tc::sdesc_k128(a0 + j * (TC_PAGE * 128) + sub * 32);
          const uint64_t bd = tc::sdesc_k128(b0 + j * qbox_bytes + sub * 32);
          tc::mma_f16(tmem + (uint32_t)(a * ncols), ad, bd, idesc, kk > 0 ? 1u : 0u);
        }
        tc::commit(&empty[s]);
        tc::commit(&acc_full[a]);
      }
    }
  } else {
    // -------------------------------------------------- epilogue, warps 0-3
    const int tok = warp * 32 + lane;
    float m = -INFINITY;
    uint32_t kmax = 0;
    float ksum = 0.f;
    for (int64_t t = 0; t < my_tiles; ++t) {
      const int a = (int)(t & 1);
      if (!mbar_wait_bounded(&acc_full[a], (uint32_t)((t / 2) & 1))) { s_fail = 1; break; }
      tc::fence_after_sync();
      const uint32_t taddr = tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(a * ncols);
      uint32_t r[16];
      if (COARSE) {
        // one score per (query row, page): thread tok holds page u*128 + tok
        const int64_t u = cj + (t / H) * cpb;
        const int kvh = (int)(t % H);
        const int64_t p = u * TC_PAGE + tok;
        for (int c0 = 0; c0 < ncols; c0 += 16) {
          tc::ld_32x16(taddr + c0, r);
          tc::wait_ld();
          if (p < np_scored) {
#pragma unroll
            for (int c = 0; c < 16; ++c) {
              const int rr = c0 + c;
              if (rr < rows_kv) {
                const float sc = __uint_as_float(r[c]) * q.scaling;
                const int h = kvh * G + rr / Q, tq = rr % Q;
                const int64_t R_idx = ((int64_t)b * Hq + h) * Q + tq;
                w.scores[R_idx * w.np_cap + p] = sc;
                const uint32_t key = f2key(sc);
                kmax = key > kmax ? key : kmax;
                ksum += sc;
              }
            }
          }
        }
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[a]);
        continue;
      }
      for (int c0 = 0; c0 < ncols; c0 += 16) {
        tc::ld_32x16(taddr + c0, r);
        tc::wait_ld();
#pragma unroll
        for (int c = 0; c < 16; ++c)
          if (c0 + c < rows_kv) m = fmaxf(m, __uint_as_float(r[c]) * q.scaling);
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[a]);
      if ((t % H) == H - 1) {
        const int64_t u = cj + (t / H) * cpb;
        const int n_tok = u < (XC ? n_own : f.U) ? TC_PAGE : (int)f.partial;
        if (tok < n_tok) {
          const uint32_t key = f2key(m);
          if (XC) {
            // this candidate into every shard's arena (the select builds the histogram)
            const int64_t c = (int64_t)b * w.c_cap + unit_pos(u) + tok;
            for (int d = 0; d < x.world; ++d) ll_store(x_region(x, d, xe) + c, key, x_flag(xe));
          } else {
            w.agg[(int64_t)b * w.c_cap + u * S + tok] = key;
            // shared-memory atomic: the warp's keys fall in a few bins, which
            // costs far less here than aggregating the lanes with a match
            atomicAdd(&hist[key >> 21], 1u);
          }
          kmax = key > kmax ? key : kmax;
          ksum += m;
        }
        m = -INFINITY;
      }
    }
    // per-warp stats
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
  // publish the histogram and the stats of batch row 0 for the select kernel
  if (!COARSE && !XC) {
    for (int i = threadIdx.x; i < SEL_BINS; i += TC_THREADS)
      if (hist[i]) atomicAdd(&w.fhist[(int64_t)b * SEL_BINS + i], hist[i]);
  }
  if (threadIdx.x == 0) {
    uint32_t mk = 0;
    double sm = 0.0;
    for (int i = 0; i < 4; ++i) {
      mk = s_wmax[i] > mk ? s_wmax[i] : mk;
      sm += s_wsum[i];
    }
    if (my_tiles > 0) {
      if (COARSE) {
        atomicMax(reinterpret_cast<unsigned long long *>(&w.cstat[0]), (unsigned long long)mk);
        atomicAdd(reinterpret_cast<double *>(&w.cstat[1]), sm);
      } else {
        atomicMax(reinterpret_cast<unsigned long long *>(&w.fstat[2 * b]), (unsigned long long)mk);
        atomicAdd(reinterpret_cast<double *>(&w.fstat[2 * b + 1]), sm);
      }
    }
    if (s_fail)
      atomicOr(reinterpret_cast<unsigned long long *>(st.state + KIV_ST_ERROR),
               (unsigned long long)KIV_ERRBIT_WAIT_TIMEOUT);
  }
  if (warp == 0) tc::tmem_dealloc(tmem, (uint32_t)(2 * ncols < 32 ? 32 : 2 * ncols));
}

// ------------------------------------------------------------------ host
static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

static kiv_status encode_fn() {
  if (g_encode) return KIV_OK;
  void *fn = nullptr;
  cudaDriverEntryPointQueryResult qr;
  cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &qr);
  if (e != cudaSuccess || qr != cudaDriverEntryPointSuccess || fn == nullptr) {
    set_error("cuTensorMapEncodeTiled unavailable");
    return KIV_ERR_CUDA;
  }
  g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  return KIV_OK;
}

kiv_status encode_tiled(CUtensorMap *map, int dtype, int rank, const void *base, const uint64_t *dims,
                        const uint64_t *strides, const uint32_t *box, CUtensorMapSwizzle swizzle) {
  KIV_CHECK(encode_fn());
  cuuint64_t d[5], st[4];
  cuuint32_t b[5], e[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
    if (i + 1 < rank) st[i] = strides[i];
  }
  const CUresult r = g_encode(map, dtype == KIV_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                              (cuuint32_t)rank, const_cast<void *>(base), d, st, b, e, CU_TENSOR_MAP_INTERLEAVE_NONE,
                              swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d)", (int)r);
    return KIV_ERR_CUDA;
  }
  return KIV_OK;
}

bool fine_tc_eligible(const kiv_store *st, const kiv_query *q) {
  const int rows_kv = (q->num_query_heads / st->num_kv_heads) * q->query_len;
  const int ncols = rows_kv <= 16 ? 16 : 32;
  const size_t qbytes = (size_t)st->num_kv_heads * ncols * st->head_dim * 2;
  return (st->dtype == KIV_DTYPE_BF16 || st->dtype == KIV_DTYPE_F16) && st->page_size == TC_PAGE &&
         st->head_dim % 64 == 0 && st->head_dim <= 256 && rows_kv <= 32 && qbytes <= 32 * 1024 &&
         (int64_t)st->batch * st->num_kv_heads * st->cold_capacity < (1ll << 31) &&
         getenv("KIV_DISABLE_TCGEN05") == nullptr;
}

// tensor-core scoring: coarse (summaries) or fine (candidate pages); x: the
// candidate exchange (fine only)
static kiv_status launch_scores_tc(const kiv_store *st, const kiv_query *q, const Workspace &w, cudaStream_t s,
                                   bool coarse, const XArgs *x = nullptr) {
  KIV_CHECK(encode_fn());
  const int D = st->head_dim;
  const int rows_kv = (q->num_query_heads / st->num_kv_heads) * q->query_len;
  const int ncols = rows_kv <= 16 ? 16 : 32;
  CUtensorMap map;
  const int64_t bh = (int64_t)st->batch * st->num_kv_heads;
  const int64_t rows = coarse ? bh * w.np_cap : bh * st->cold_capacity;
  const cuuint64_t dims[2] = {(cuuint64_t)D, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)D * 2};
  const cuuint32_t box[2] = {64, TC_PAGE};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = g_encode(&map, st->dtype == KIV_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                                : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                              2, coarse ? st->summaries : st->cold_k, dims, strides, box, estr,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d)", (int)r);
    return KIV_ERR_CUDA;
  }
  const size_t tile = (size_t)TC_PAGE * D * 2;
  const size_t qbytes = (size_t)st->num_kv_heads * ncols * D * 2;
  // fine pass: the union list is built in shared memory unless it is large
  // (with a host tier the union is staged before scoring: built separately)
  const int union_inline = !coarse && w.u_cap <= TC_UNION_INLINE && st->host_capacity == 0 ? 1 : 0;
  if (x && !union_inline) {
    set_error("candidate exchange needs the union built in the scorer (union cap %lld)", (long long)w.u_cap);
    return KIV_ERR_UNSUPPORTED;
  }
  if (!coarse && !union_inline) {
    KIV_CHECK(launch_union(st, w, s));
    KIV_CHECK(launch_stage_union(st, w, s));
  }
  const size_t fixed = 1024 + qbytes + SEL_BINS * 4 + (union_inline ? (size_t)w.u_cap * 4 * (x ? 2 : 1) : 0);
  const int stages = (int)std::min<size_t>(4, (200 * 1024 - fixed) / tile);
  if (stages < 2) return KIV_ERR_UNSUPPORTED;
  const size_t smem = fixed + (size_t)stages * tile;
  // per batch row: cpb CTAs (about the SMs shared out over the rows)
  const int64_t units_cap = coarse ? ceil_div(w.np_cap, TC_PAGE) : w.u_cap + 1;
  const int64_t cpb = std::max<int64_t>(1, std::min<int64_t>(units_cap, sm_count() / st->batch));
  const int64_t grid = (int64_t)st->batch * cpb;
  const XArgs xa = x ? *x : XArgs{};
#define KIV_TC_LAUNCH(BF, CO, XC)                                                                      \
  do {                                                                                                 \
    cudaFuncSetAttribute(scores_tc_kernel<BF, CO, XC>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); \
    e = launch_pdl(scores_tc_kernel<BF, CO, XC>, dim3((unsigned)grid), dim3(TC_THREADS), smem, s, 1, map, *st, *q, \
                   w, ncols, stages, union_inline, (int)cpb, xa);                                       \
  } while (0)
  const bool bf = st->dtype == KIV_DTYPE_BF16;
  cudaError_t e = cudaSuccess;
  if (bf && coarse) KIV_TC_LAUNCH(true, true, false);
  else if (bf && x) KIV_TC_LAUNCH(true, false, true);
  else if (bf) KIV_TC_LAUNCH(true, false, false);
  else if (coarse) KIV_TC_LAUNCH(false, true, false);
  else if (x) KIV_TC_LAUNCH(false, false, true);
  else KIV_TC_LAUNCH(false, false, false);
#undef KIV_TC_LAUNCH
  return cuda_status(e, coarse ? "coarse_scores_tc" : "fine_scores_tc");
}

kiv_status launch_fine_score_tc(const kiv_store *st, const kiv_query *q, const Workspace &w, cudaStream_t s) {
  return launch_scores_tc(st, q, w, s, false);
}

kiv_status launch_coarse_score_tc(const kiv_store *st, const kiv_query *q, const Workspace &w, cudaStream_t s) {
  return launch_scores_tc(st, q, w, s, true);
}

kiv_status launch_fine_score_tc_exchange(const kiv_store *st, const kiv_query *q, const Workspace &w,
                                         cudaStream_t s, const XArgs &x) {
  return launch_scores_tc(st, q, w, s, false, &x);
}

}  // namespace kiv
