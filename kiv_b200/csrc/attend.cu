// Kernels (d) and (e): gather of the selected rows, and attention over
// [selected cold ; hot] split over the keys with a log-sum-exp merge.
//
// Reference behaviour restated (kiv/middleware.py:330-352, kiv/mask_utils.py:8-38,
// HF eager_attention_forward):
//   keys = cat(cold_k[selected], hot_k), values likewise; the mask is the hot
//   mask with all-attendable columns prepended for the cold rows;
//   out = softmax(scaling * q k^T + mask) v, output layout [B, Q, Hq, D].
// Nothing is concatenated here: each split of the key range stages its K and
// V rows (cold rows straight from their token slots, hot rows from the ring)
// into shared memory with per-row 1-D TMA bulk copies, runs an online softmax
// for all G*Q query rows of its KV head, and writes a partial (out, max, sum);
// a second kernel merges the partials of all splits (and, sharded, of all
// GPUs) by log-sum-exp.
#include <algorithm>

#include "common.cuh"
#include "exchange.cuh"
#include "internal.h"

namespace kiv {

constexpr int AT_THREADS = 256;
constexpr int AT_STAGES = 2;
constexpr int CB_THREADS = 256;
constexpr int CB_COLS_SPLIT = 16;  // output columns per CTA, merge of one rank's splits
constexpr int CB_COLS_X = 64;      // output columns per CTA, merge across ranks

template <typename T>
struct AttnArgs {
  kiv_store st;
  kiv_query q;
  kiv_mask mask;
  Workspace w;
  const int32_t *sel;
  int32_t sel_stride;
  int32_t hot_slice, hot_slices;
  int32_t n_split;
  // page-sharded store, global selection: every shard's cold rows (the owner
  // of page p is shard p % shard_count), or null pointers for own rows only
  const void *peer_k[KIV_MAX_PEERS];
  const void *peer_v[KIV_MAX_PEERS];
  int32_t peers;
};

// reduced [RCH][D] outputs live after the key-subset partials
__device__ __forceinline__ float *sc_out_slot(float *ored, int pairs, int ksub, int V) {
  return ored + (size_t)pairs * ksub * V;
}

template <typename T, int LPR, int VPL, int RCH>
__global__ void __launch_bounds__(AT_THREADS)
attend_split_kernel(AttnArgs<T> a) {
  extern __shared__ __align__(128) uint8_t at_smem[];
  __shared__ uint64_t bars[AT_STAGES];
  __shared__ float s_m[RCH], s_l[RCH], s_alpha[RCH];
  __shared__ int s_fail;
  const kiv_store &st = a.st;
  const kiv_query &q = a.q;
  constexpr int V = Elem<T>::V;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane % LPR, grp = lane / LPR;
  constexpr int GPW = 32 / LPR;
  constexpr int NGROUPS = (AT_THREADS / 32) * GPW;
  const int D = st.head_dim, H = st.num_kv_heads, S = st.page_size;
  const int nv = D / V;
  const int G = q.num_query_heads / H, Q = q.query_len;
  const int rows_kv = G * Q;
  const int nchunks = (rows_kv + RCH - 1) / RCH;

  // work item -> (b, kvh, chunk, split)
  const int split = blockIdx.x % a.n_split;
  const int rest = blockIdx.x / a.n_split;
  const int ch = rest % nchunks;
  const int bh = rest / nchunks;
  const int b = bh / H, kvh = bh % H;

  // ---- prologue: inputs written before the retrieval's first kernel (the
  // hot window state, the query); with programmatic dependent launch it
  // overlaps the selection kernel's tail
  const int64_t hot_len = st_ld(st.state, KIV_ST_HOT_LEN);
  const int64_t hot_start = st_ld(st.state, KIV_ST_HOT_START);
  const int64_t hot_lo = hot_len * a.hot_slice / a.hot_slices;
  const int64_t hot_hi = hot_len * (a.hot_slice + 1) / a.hot_slices;
  if (threadIdx.x == 0) {
    for (int s = 0; s < AT_STAGES; ++s) mbar_init(&bars[s], 1);
    mbar_fence_init();
    s_fail = 0;
  }
  if (threadIdx.x < RCH) {
    s_m[threadIdx.x] = -INFINITY;
    s_l[threadIdx.x] = 0.f;
  }
  // query rows of this chunk (fp32 registers)
  const T *qb = reinterpret_cast<const T *>(q.q);
  int row_h[RCH], row_t[RCH];
  RowDot<T, LPR, VPL, RCH> dot;
  {
    const T *qrows[RCH];
#pragma unroll
    for (int r = 0; r < RCH; ++r) {
      const int rr = ch * RCH + r;
      if (rr < rows_kv) {
        row_h[r] = kvh * G + rr / Q;
        row_t[r] = rr % Q;
        qrows[r] = qb + b * q.stride_b + row_h[r] * q.stride_h + row_t[r] * q.stride_t;
      } else {
        row_h[r] = -1;
        row_t[r] = 0;
        qrows[r] = nullptr;
      }
    }
    dot.load_query(qrows, g, nv, 1.0f);
  }
  // Key order of the split: the hot window rows first, then the selected
  // cold rows.  The split size is fixed by the cold list capacity
  // (sel_stride bounds the selected count), so a split made only of hot rows
  // is known before the selection finishes and never waits for it.
  const int64_t hot_count = hot_hi - hot_lo;
  int64_t kps = (a.sel_stride + hot_count + a.n_split - 1) / a.n_split;
  kps = (kps + 7) / 8 * 8;
  const int64_t k_lo = split * kps;
  const bool hot_only = k_lo + kps <= hot_count;

  T *kt = reinterpret_cast<T *>(at_smem);                 // [STAGES][TILE][D]
  T *vt = kt + (size_t)AT_STAGES * ATT_TILE * D;          // [STAGES][TILE][D]
  float *sc = reinterpret_cast<float *>(vt + (size_t)AT_STAGES * ATT_TILE * D);  // [RCH][TILE]
  float *ored = sc + RCH * ATT_TILE;                       // [2*THREADS*V] key-subset partials + [RCH][D]

  const T *cold_k = reinterpret_cast<const T *>(st.cold_k);
  const T *cold_v = reinterpret_cast<const T *>(st.cold_v);
  const T *hot_k = reinterpret_cast<const T *>(st.hot_k);
  const T *hot_v = reinterpret_cast<const T *>(st.hot_v);
  const int32_t *selb = a.sel + (int64_t)b * a.sel_stride;
  const int64_t bhk = (int64_t)b * H + kvh;
  const uint32_t row_bytes = (uint32_t)D * sizeof(T);

  // tok_hint: the cold key's token when already loaded, else -1
  auto key_rows = [&](int64_t k, const T *&pk, const T *&pv, int32_t tok_hint) {
    if (k < hot_count) {
      const int64_t slot = (hot_start + hot_lo + k) % st.hot_capacity;
      pk = hot_k + (bhk * st.hot_capacity + slot) * D;
      pv = hot_v + (bhk * st.hot_capacity + slot) * D;
    } else {
      const int64_t tok = tok_hint >= 0 ? tok_hint : selb[k - hot_count];
      const int64_t p = tok / S;
      const int64_t slot = page_slot(st, a.w, p / st.shard_count) * S + tok % S;
      const T *bk = cold_k, *bv = cold_v;
      if (a.peers) {
        // the owner's cold tier (same layout on every shard; NVLink for another shard's)
        const int own = (int)(p % st.shard_count);
        bk = reinterpret_cast<const T *>(a.peer_k[own]);
        bv = reinterpret_cast<const T *>(a.peer_v[own]);
      }
      pk = bk + (bhk * st.cold_capacity + slot) * D;
      pv = bv + (bhk * st.cold_capacity + slot) * D;
    }
  };
  // warp 0 copies the rows of tile t with key index in [lo, hi): lane i takes
  // key k0 + i (K and V).  `arrive`: this is the tile's last part (completes
  // the barrier phase); otherwise only the expected bytes are added.
  auto issue_part = [&](int t, int64_t lo, int64_t hi, bool arrive, int32_t tok_hint) {
    const int stage = t % AT_STAGES;
    const int64_t k0 = k_lo + (int64_t)t * ATT_TILE;
    const int64_t a0 = std::max<int64_t>(k0, lo), a1 = std::min<int64_t>(k0 + ATT_TILE, hi);
    const uint32_t bytes = a1 > a0 ? 2u * (uint32_t)(a1 - a0) * row_bytes : 0u;
    if (lane == 0) {
      if (arrive) mbar_arrive_tx(&bars[stage], bytes);
      else if (bytes) mbar_expect_tx(&bars[stage], bytes);
    }
    __syncwarp();
    const int64_t k = k0 + lane;
    if (k >= a0 && k < a1) {
      const T *pk, *pv;
      key_rows(k, pk, pv, tok_hint);
      bulk_g2s(kt + ((size_t)stage * ATT_TILE + lane) * D, pk, row_bytes, &bars[stage]);
      bulk_g2s(vt + ((size_t)stage * ATT_TILE + lane) * D, pv, row_bytes, &bars[stage]);
    }
  };
  const int early_tiles = (int)std::min<int64_t>(AT_STAGES, (std::min<int64_t>(kps, hot_count - k_lo) +
                                                             ATT_TILE - 1) / ATT_TILE);
  __syncthreads();   // barriers initialized
  // hot rows of the first tiles: independent of the selection
  if (warp == 0)
    for (int t = 0; t < early_tiles; ++t)
      issue_part(t, k_lo, std::min<int64_t>(hot_count, k_lo + kps), hot_only, -1);
  int64_t ncold = 0;
  int32_t tok0 = -1, tok1 = -1;
  static_assert(AT_STAGES == 2, "two preloaded tiles");
  if (!hot_only) {
    // ---- the selection (previous kernel) is needed from here on.  The
    // selected count and the tokens of the first two tiles load together
    // (entries past the count are ignored).
    griddep_wait();
    if (warp == 0) {
      const int64_t c0 = k_lo + lane - hot_count, c1 = c0 + ATT_TILE;
      const int64_t lim = std::min<int64_t>((int64_t)a.sel_stride, k_lo + kps - hot_count);
      if (c0 >= 0 && c0 < lim) tok0 = selb[c0];
      if (c1 >= 0 && c1 < lim) tok1 = selb[c1];
    }
    ncold = a.w.selcnt[b];
  }
  const int64_t nkeys = hot_count + ncold;
  const int64_t k_hi = std::min<int64_t>(nkeys, k_lo + kps);
  const int ntile = k_hi > k_lo ? (int)((k_hi - k_lo + ATT_TILE - 1) / ATT_TILE) : 0;
  if (warp == 0 && !hot_only) {
    // cold rows of the first tiles (and the arrival that completes them)
    if (ntile > 0) issue_part(0, hot_count, k_hi, true, tok0);
    if (ntile > 1) issue_part(1, hot_count, k_hi, true, tok1);
  }
  auto issue = [&](int t) { issue_part(t, k_lo, k_hi, true, -1); };

  // P.V mapping: thread -> (vector dv, row r, key subset ks)
  const int nvp = nv;  // vectors per row
  const int pairs = nvp * RCH;
  const int ksub = std::max(1, AT_THREADS / pairs);
  float o[2][V];
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int e = 0; e < V; ++e) o[i][e] = 0.f;

  for (int t = 0; t < ntile; ++t) {
    const int stage = t % AT_STAGES;
    if (!mbar_wait_bounded(&bars[stage], (uint32_t)((t / AT_STAGES) & 1))) s_fail = 1;
    __syncthreads();
    if (s_fail) break;
    const int64_t k0 = k_lo + (int64_t)t * ATT_TILE;
    const int n = (int)std::min<int64_t>(ATT_TILE, k_hi - k0);
    const T *ktile = kt + (size_t)stage * ATT_TILE * D;
    const T *vtile = vt + (size_t)stage * ATT_TILE * D;
    // ---- scores ----
    for (int kk0 = 0; kk0 < ATT_TILE; kk0 += NGROUPS) {
      const int kk = kk0 + warp * GPW + grp;
      float acc[RCH];
      dot.template partial<false>(kk < n ? ktile + (size_t)kk * D : nullptr, g, nv, acc);
      int base = 0;
      tr_reduce<RCH, LPR / 2>(acc, lane, base);
      constexpr int NOUT = TrOut<RCH, LPR>::N;
      constexpr int REPL = TrOut<RCH, LPR>::REPL;
      if (kk < ATT_TILE && (g % REPL) == 0) {
#pragma unroll
        for (int i = 0; i < NOUT; ++i) {
          const int r = base + i;
          float s = -INFINITY;
          if (kk < n && row_h[r] >= 0) {
            s = acc[i] * q.scaling;
            if (q.softcap > 0.f) s = q.softcap * tanhf(s / q.softcap);
            const int64_t k = k0 + kk;
            if (k < hot_count) {
              const int64_t j = hot_lo + k;
              if (a.mask.causal && j > hot_len - Q + row_t[r]) s = -INFINITY;
              if (a.mask.add != nullptr)
                s += a.mask.add[b * a.mask.stride_b + row_h[r] * a.mask.stride_h +
                                row_t[r] * a.mask.stride_t + j];
            }
          }
          sc[r * ATT_TILE + kk] = s;
        }
      }
    }
    __syncthreads();
    // ---- online softmax: warp r owns query row r ----
    for (int r = warp; r < RCH; r += AT_THREADS / 32) {
      const float x = sc[r * ATT_TILE + lane];
      float mt = x;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) mt = fmaxf(mt, __shfl_xor_sync(KIV_FULL_MASK, mt, off));
      const float m_old = s_m[r];
      const float m_new = fmaxf(m_old, mt);
      const float alpha = (m_new == -INFINITY) ? 1.f : __expf(m_old - m_new);
      const float p = (m_new == -INFINITY) ? 0.f : __expf(x - m_new);
      float ps = p;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) ps += __shfl_xor_sync(KIV_FULL_MASK, ps, off);
      sc[r * ATT_TILE + lane] = p;
      __syncwarp();
      if (lane == 0) {
        s_alpha[r] = alpha;
        s_m[r] = m_new;
        s_l[r] = s_l[r] * alpha + ps;
      }
    }
    __syncthreads();
    // ---- o = o * alpha + p . V ----
    {
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int idx = threadIdx.x + i * AT_THREADS;
        if (idx >= pairs * ksub) continue;
        const int pair = idx % pairs;
        const int ks = idx / pairs;
        const int dv = pair % nvp, r = pair / nvp;
        const float al = s_alpha[r];
#pragma unroll
        for (int e = 0; e < V; ++e) o[i][e] *= al;
        for (int kk = ks; kk < n; kk += ksub) {
          const float p = sc[r * ATT_TILE + kk];
          float f[V];
          Elem<T>::unpack(ld16(vtile + (size_t)kk * D + dv * V), f);
#pragma unroll
          for (int e = 0; e < V; ++e) o[i][e] = fmaf(p, f[e], o[i][e]);
        }
      }
    }
    __syncthreads();
    if (warp == 0 && t + AT_STAGES < ntile) issue(t + AT_STAGES);
  }
  if (s_fail) {
    if (threadIdx.x == 0)
      atomicOr(reinterpret_cast<unsigned long long *>(st.state + KIV_ST_ERROR), 8ull);
    return;
  }
  const int Dp = partial_stride(D);
  if (ksub == 1) {
    // one thread per (row, vector): write the partial straight from registers
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int idx = threadIdx.x + i * AT_THREADS;
      if (idx >= pairs) continue;
      const int dv = idx % nvp, r = idx / nvp;
      if (row_h[r] < 0) continue;
      const int64_t R_idx = ((int64_t)b * q.num_query_heads + row_h[r]) * Q + row_t[r];
      float *dst = a.w.part + (R_idx * a.w.split_cap + split) * Dp;
#pragma unroll
      for (int e = 0; e < V; e += 4)
        *reinterpret_cast<float4 *>(dst + dv * V + e) = make_float4(o[i][e], o[i][e + 1], o[i][e + 2], o[i][e + 3]);
      if (dv == 0) {
        dst[D] = s_m[r];
        dst[D + 1] = s_l[r];
      }
    }
    return;
  }
  // reduce over key subsets in a fixed order (deterministic) and write the
  // partial (out, max, sum)
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int idx = threadIdx.x + i * AT_THREADS;
    if (idx >= pairs * ksub) continue;
#pragma unroll
    for (int e = 0; e < V; ++e) ored[(size_t)idx * V + e] = o[i][e];
  }
  __syncthreads();
  for (int pr = threadIdx.x; pr < pairs; pr += AT_THREADS) {
    const int dv = pr % nvp, r = pr / nvp;
    float acc[V];
#pragma unroll
    for (int e = 0; e < V; ++e) acc[e] = 0.f;
    for (int ks = 0; ks < ksub; ++ks)
#pragma unroll
      for (int e = 0; e < V; ++e) acc[e] += ored[((size_t)ks * pairs + pr) * V + e];
#pragma unroll
    for (int e = 0; e < V; ++e) sc_out_slot(ored, pairs, ksub, V)[(size_t)r * D + dv * V + e] = acc[e];
  }
  __syncthreads();
  for (int r = 0; r < RCH; ++r) {
    if (row_h[r] < 0) continue;
    const int64_t R_idx = ((int64_t)b * q.num_query_heads + row_h[r]) * Q + row_t[r];
    float *dst = a.w.part + (R_idx * a.w.split_cap + split) * Dp;
    const float *fin = sc_out_slot(ored, pairs, ksub, V);
    for (int d = threadIdx.x; d < D; d += AT_THREADS) dst[d] = fin[r * D + d];
    if (threadIdx.x == 0) {
      dst[D] = s_m[r];
      dst[D + 1] = s_l[r];
    }
  }
}

// ---------------------------------------------------------------------------
// Tensor-core decode attention for 16-bit stores with at most 16 query rows
// per KV head (the G*Q rows of a decode step).  Same splits, key order and
// partial format as attend_split_kernel; per 32-key tile S = Q K^T and
// O = P V run on warp-level MMAs (m16n8k16, fp32 accumulate): the query rows
// form a single 16-row tile, a quarter of the smallest tcgen05 tile, and
// this kernel is on the latency path of every decode step.  K and V rows are
// staged by per-row bulk copies into rows padded by 16 bytes, so the
// ldmatrix reads of 8 rows hit 8 distinct bank groups.  P is rounded to the
// store dtype before the P V product (as flash attention does).
// ---------------------------------------------------------------------------
constexpr int AM_THREADS = 128;    // 4 warps: 8 keys each for S, D/4 columns each for O
constexpr int AM_ROWS = 16;        // query rows per tile
constexpr int AM_PPITCH = 80;      // bytes per row of the P tile (32 keys + pad)

template <typename T> struct MmaOp;
template <> struct MmaOp<__nv_bfloat16> {
  __device__ __forceinline__ static void mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
  __device__ __forceinline__ static uint32_t pack2(float x, float y) {
    __nv_bfloat162 h = __floats2bfloat162_rn(x, y);
    return *reinterpret_cast<uint32_t *>(&h);
  }
};
template <> struct MmaOp<__half> {
  __device__ __forceinline__ static void mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
  __device__ __forceinline__ static uint32_t pack2(float x, float y) {
    __half2 h = __floats2half2_rn(x, y);
    return *reinterpret_cast<uint32_t *>(&h);
  }
};
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void *p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void *p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

template <typename T>
__global__ void __launch_bounds__(AM_THREADS)
attend_mma_kernel(AttnArgs<T> a) {
  extern __shared__ __align__(128) uint8_t am_smem[];
  __shared__ uint64_t bars[AT_STAGES];
  __shared__ float s_red[4][AM_ROWS], s_sum[4][AM_ROWS];
  __shared__ float s_m[AM_ROWS], s_l[AM_ROWS], s_mnew[AM_ROWS];
  __shared__ int s_fail;
  using Op = MmaOp<T>;
  const kiv_store &st = a.st;
  const kiv_query &q = a.q;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t4 = lane & 3;
  const int D = st.head_dim, H = st.num_kv_heads, S = st.page_size;
  const int G = q.num_query_heads / H, Q = q.query_len;
  const int rows_kv = G * Q;
  const int pitch = D * (int)sizeof(T) + 16;   // bytes per staged row
  const int split = blockIdx.x % a.n_split;
  const int bh = blockIdx.x / a.n_split;
  const int b = bh / H, kvh = bh % H;

  uint8_t *qs = am_smem;                                         // [16][pitch]
  uint8_t *ks = qs + AM_ROWS * pitch;                            // [STAGES][TILE][pitch]
  uint8_t *vs = ks + AT_STAGES * ATT_TILE * pitch;               // [STAGES][TILE][pitch]
  uint8_t *ps = vs + AT_STAGES * ATT_TILE * pitch;               // [16][AM_PPITCH]

  // ---- prologue: inputs written before the retrieval's first kernel
  const int64_t hot_len = st_ld(st.state, KIV_ST_HOT_LEN);
  const int64_t hot_start = st_ld(st.state, KIV_ST_HOT_START);
  const int64_t hot_lo = hot_len * a.hot_slice / a.hot_slices;
  const int64_t hot_hi = hot_len * (a.hot_slice + 1) / a.hot_slices;
  if (threadIdx.x == 0) {
    for (int s = 0; s < AT_STAGES; ++s) mbar_init(&bars[s], 1);
    mbar_fence_init();
    s_fail = 0;
  }
  if (threadIdx.x < AM_ROWS) {
    s_m[threadIdx.x] = -INFINITY;
    s_l[threadIdx.x] = 0.f;
  }
  {
    const T *qb = reinterpret_cast<const T *>(q.q);
    const int nc = D / 8;                                         // 16-byte chunks per row
    for (int e = threadIdx.x; e < AM_ROWS * nc; e += AM_THREADS) {
      const int rr = e / nc, c = e % nc;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (rr < rows_kv) {
        const int h = kvh * G + rr / Q, tq = rr % Q;
        v = ld16(qb + b * q.stride_b + h * q.stride_h + tq * q.stride_t + c * 8);
      }
      *reinterpret_cast<uint4 *>(qs + rr * pitch + c * 16) = v;
    }
  }
  const int64_t hot_count = hot_hi - hot_lo;
  int64_t kps = (a.sel_stride + hot_count + a.n_split - 1) / a.n_split;
  kps = (kps + 7) / 8 * 8;
  const int64_t k_lo = split * kps;
  const bool hot_only = k_lo + kps <= hot_count;

  const T *cold_k = reinterpret_cast<const T *>(st.cold_k);
  const T *cold_v = reinterpret_cast<const T *>(st.cold_v);
  const T *hot_k = reinterpret_cast<const T *>(st.hot_k);
  const T *hot_v = reinterpret_cast<const T *>(st.hot_v);
  const int32_t *selb = a.sel + (int64_t)b * a.sel_stride;
  const int64_t bhk = (int64_t)b * H + kvh;
  const uint32_t row_bytes = (uint32_t)D * sizeof(T);
  auto key_rows = [&](int64_t k, const T *&pk, const T *&pv, int32_t tok_hint) {
    if (k < hot_count) {
      const int64_t slot = (hot_start + hot_lo + k) % st.hot_capacity;
      pk = hot_k + (bhk * st.hot_capacity + slot) * D;
      pv = hot_v + (bhk * st.hot_capacity + slot) * D;
    } else {
      const int64_t tok = tok_hint >= 0 ? tok_hint : selb[k - hot_count];
      const int64_t p = tok / S;
      const int64_t slot = page_slot(st, a.w, p / st.shard_count) * S + tok % S;
      const T *bk = cold_k, *bv = cold_v;
      if (a.peers) {
        // the owner's cold tier (same layout on every shard; NVLink for another shard's)
        const int own = (int)(p % st.shard_count);
        bk = reinterpret_cast<const T *>(a.peer_k[own]);
        bv = reinterpret_cast<const T *>(a.peer_v[own]);
      }
      pk = bk + (bhk * st.cold_capacity + slot) * D;
      pv = bv + (bhk * st.cold_capacity + slot) * D;
    }
  };
  auto issue_part = [&](int t, int64_t lo, int64_t hi, bool arrive, int32_t tok_hint) {
    const int stage = t % AT_STAGES;
    const int64_t k0 = k_lo + (int64_t)t * ATT_TILE;
    const int64_t a0 = std::max<int64_t>(k0, lo), a1 = std::min<int64_t>(k0 + ATT_TILE, hi);
    const uint32_t bytes = a1 > a0 ? 2u * (uint32_t)(a1 - a0) * row_bytes : 0u;
    if (lane == 0) {
      if (arrive) mbar_arrive_tx(&bars[stage], bytes);
      else if (bytes) mbar_expect_tx(&bars[stage], bytes);
    }
    __syncwarp();
    const int64_t k = k0 + lane;
    if (k >= a0 && k < a1) {
      const T *pk, *pv;
      key_rows(k, pk, pv, tok_hint);
      bulk_g2s(ks + ((size_t)stage * ATT_TILE + lane) * pitch, pk, row_bytes, &bars[stage]);
      bulk_g2s(vs + ((size_t)stage * ATT_TILE + lane) * pitch, pv, row_bytes, &bars[stage]);
    }
  };
  const int early_tiles = (int)std::min<int64_t>(AT_STAGES, (std::min<int64_t>(kps, hot_count - k_lo) +
                                                             ATT_TILE - 1) / ATT_TILE);
  __syncthreads();   // barriers, statistics and query tile ready
  if (warp == 0)
    for (int t = 0; t < early_tiles; ++t)
      issue_part(t, k_lo, std::min<int64_t>(hot_count, k_lo + kps), hot_only, -1);
  int64_t ncold = 0;
  int32_t tok0 = -1, tok1 = -1;
  if (!hot_only) {
    // ---- the selection (previous kernel) is needed from here on
    griddep_wait();
    if (warp == 0) {
      const int64_t c0 = k_lo + lane - hot_count, c1 = c0 + ATT_TILE;
      const int64_t lim = std::min<int64_t>((int64_t)a.sel_stride, k_lo + kps - hot_count);
      if (c0 >= 0 && c0 < lim) tok0 = selb[c0];
      if (c1 >= 0 && c1 < lim) tok1 = selb[c1];
    }
    ncold = a.w.selcnt[b];
  }
  const int64_t nkeys = hot_count + ncold;
  const int64_t k_hi = std::min<int64_t>(nkeys, k_lo + kps);
  const int ntile = k_hi > k_lo ? (int)((k_hi - k_lo + ATT_TILE - 1) / ATT_TILE) : 0;
  if (warp == 0 && !hot_only) {
    if (ntile > 0) issue_part(0, hot_count, k_hi, true, tok0);
    if (ntile > 1) issue_part(1, hot_count, k_hi, true, tok1);
  }

  const int ntw = D / 32;           // 8-column output tiles per warp
  const int dbase = warp * (D / 4);
  float o[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;

  for (int t = 0; t < ntile; ++t) {
    const int stage = t % AT_STAGES;
    if (!mbar_wait_bounded(&bars[stage], (uint32_t)((t / AT_STAGES) & 1))) s_fail = 1;
    const int64_t k0 = k_lo + (int64_t)t * ATT_TILE;
    const int n = (int)std::min<int64_t>(ATT_TILE, k_hi - k0);
    uint8_t *kst = ks + (size_t)stage * ATT_TILE * pitch;
    uint8_t *vst = vs + (size_t)stage * ATT_TILE * pitch;
    if (n < ATT_TILE) {
      // rows past the tile's keys hold stale data: zero V there (P is 0 there)
      for (int e = threadIdx.x; e < (ATT_TILE - n) * (D / 8); e += AM_THREADS)
        *reinterpret_cast<uint4 *>(vst + (n + e / (D / 8)) * pitch + (e % (D / 8)) * 16) = make_uint4(0, 0, 0, 0);
    }
    __syncthreads();
    if (s_fail) break;
    // ---- S = Q K^T for keys [8 warp, 8 warp + 8)
    float sacc[4] = {0.f, 0.f, 0.f, 0.f};
    {
      const uint8_t *qrow = qs + (lane & 15) * pitch + 16 * (lane >> 4);
      const uint8_t *krow = kst + (8 * warp + (lane & 7)) * pitch + 16 * (lane >> 3);
#pragma unroll 2
      for (int d0 = 0; d0 < D; d0 += 32) {
        uint32_t qa[4], qb2[4], kb[4];
        ldsm_x4(qa, qrow + d0 * 2);
        ldsm_x4(qb2, qrow + d0 * 2 + 32);
        ldsm_x4(kb, krow + d0 * 2);
        Op::mma(sacc, qa, kb[0], kb[1]);
        Op::mma(sacc, qb2, kb[2], kb[3]);
      }
    }
    float sv[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int row = g + 8 * (i >> 1);
      const int kk = 8 * warp + 2 * t4 + (i & 1);
      float sc = -INFINITY;
      if (kk < n && row < rows_kv) {
        sc = sacc[i] * q.scaling;
        if (q.softcap > 0.f) sc = q.softcap * tanhf(sc / q.softcap);
        const int64_t k = k0 + kk;
        if (k < hot_count) {
          const int64_t j = hot_lo + k;
          const int h = kvh * G + row / Q, tq = row % Q;
          if (a.mask.causal && j > hot_len - Q + tq) sc = -INFINITY;
          if (a.mask.add != nullptr)
            sc += a.mask.add[b * a.mask.stride_b + h * a.mask.stride_h + tq * a.mask.stride_t + j];
        }
      }
      sv[i] = sc;
    }
    // ---- online softmax over the tile (rows g and g + 8 of this thread)
    float m0 = fmaxf(sv[0], sv[1]), m1 = fmaxf(sv[2], sv[3]);
#pragma unroll
    for (int off = 1; off < 4; off <<= 1) {
      m0 = fmaxf(m0, __shfl_xor_sync(KIV_FULL_MASK, m0, off));
      m1 = fmaxf(m1, __shfl_xor_sync(KIV_FULL_MASK, m1, off));
    }
    if (t4 == 0) {
      s_red[warp][g] = m0;
      s_red[warp][g + 8] = m1;
    }
    __syncthreads();
    float mn[2], al[2];
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int row = g + 8 * hh;
      float mt = s_red[0][row];
#pragma unroll
      for (int w2 = 1; w2 < 4; ++w2) mt = fmaxf(mt, s_red[w2][row]);
      const float mo = s_m[row];
      mn[hh] = fmaxf(mo, mt);
      al[hh] = (mn[hh] == -INFINITY || mo == -INFINITY) ? (mn[hh] == -INFINITY ? 1.f : 0.f) : __expf(mo - mn[hh]);
    }
    float pv[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float m = mn[i >> 1];
      pv[i] = (sv[i] == -INFINITY || m == -INFINITY) ? 0.f : __expf(sv[i] - m);
    }
    *reinterpret_cast<uint32_t *>(ps + g * AM_PPITCH + (8 * warp + 2 * t4) * 2) = Op::pack2(pv[0], pv[1]);
    *reinterpret_cast<uint32_t *>(ps + (g + 8) * AM_PPITCH + (8 * warp + 2 * t4) * 2) = Op::pack2(pv[2], pv[3]);
    float l0 = pv[0] + pv[1], l1 = pv[2] + pv[3];
#pragma unroll
    for (int off = 1; off < 4; off <<= 1) {
      l0 += __shfl_xor_sync(KIV_FULL_MASK, l0, off);
      l1 += __shfl_xor_sync(KIV_FULL_MASK, l1, off);
    }
    if (t4 == 0) {
      s_sum[warp][g] = l0;
      s_sum[warp][g + 8] = l1;
      if (warp == 0) {
        s_mnew[g] = mn[0];
        s_mnew[g + 8] = mn[1];
      }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      o[i][0] *= al[0];
      o[i][1] *= al[0];
      o[i][2] *= al[1];
      o[i][3] *= al[1];
    }
    __syncthreads();
    if (threadIdx.x < AM_ROWS) {
      const int row = threadIdx.x;
      const float mo = s_m[row], mnr = s_mnew[row];
      const float alr = (mnr == -INFINITY || mo == -INFINITY) ? (mnr == -INFINITY ? 1.f : 0.f) : __expf(mo - mnr);
      s_l[row] = s_l[row] * alr + s_sum[0][row] + s_sum[1][row] + s_sum[2][row] + s_sum[3][row];
      s_m[row] = mnr;
    }
    // ---- O += P V for columns [dbase, dbase + D/4)
#pragma unroll
    for (int kk0 = 0; kk0 < ATT_TILE; kk0 += 16) {
      uint32_t pa[4];
      ldsm_x4(pa, ps + (lane & 15) * AM_PPITCH + (kk0 + 8 * (lane >> 4)) * 2);
      const uint8_t *vrow = vst + (kk0 + (lane & 15)) * pitch + (dbase + 8 * (lane >> 4)) * 2;
#pragma unroll
      for (int nt = 0; nt < 8; nt += 2) {
        if (nt < ntw) {
          uint32_t vb[4];
          ldsm_x4_t(vb, vrow + nt * 16);
          Op::mma(o[nt], pa, vb[0], vb[1]);
          Op::mma(o[nt + 1], pa, vb[2], vb[3]);
        }
      }
    }
    __syncthreads();
    if (warp == 0 && t + AT_STAGES < ntile) issue_part(t + AT_STAGES, k_lo, k_hi, true, -1);
  }
  if (s_fail) {
    if (threadIdx.x == 0)
      atomicOr(reinterpret_cast<unsigned long long *>(st.state + KIV_ST_ERROR), 8ull);
    return;
  }
  // ---- partial (out, max, sum) of every query row
  const int Dp = partial_stride(D);
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    const int row = g + 8 * hh;
    if (row >= rows_kv) continue;
    const int h = kvh * G + row / Q, tq = row % Q;
    const int64_t R_idx = ((int64_t)b * q.num_query_heads + h) * Q + tq;
    float *dst = a.w.part + (R_idx * a.w.split_cap + split) * Dp;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
      if (nt < ntw)
        *reinterpret_cast<float2 *>(dst + dbase + nt * 8 + 2 * t4) = make_float2(o[nt][2 * hh], o[nt][2 * hh + 1]);
    if (warp == 0 && t4 == 0) {
      dst[D] = s_m[row];
      dst[D + 1] = s_l[row];
    }
  }
}

template <typename T>
static bool attend_mma_eligible(const kiv_store *st, const kiv_query *q) {
  const int rows_kv = (q->num_query_heads / st->num_kv_heads) * q->query_len;
  return sizeof(T) == 2 && rows_kv <= AM_ROWS && st->head_dim % 64 == 0 && st->head_dim <= 256 &&
         getenv("KIV_DISABLE_MMA_ATTN") == nullptr;
}

template <typename T>
static kiv_status launch_am(const AttnArgs<T> &a, cudaStream_t s) {
  const int pitch = a.st.head_dim * (int)sizeof(T) + 16;
  const size_t smem = (size_t)(AM_ROWS + 2 * AT_STAGES * ATT_TILE) * pitch + (size_t)AM_ROWS * AM_PPITCH;
  auto kern = attend_mma_kernel<T>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  const int64_t grid = (int64_t)a.st.batch * a.st.num_kv_heads * a.n_split;
  if (grid > 0x7fffffff) return KIV_ERR_ARG;
  return cuda_status(launch_pdl(kern, dim3((unsigned)grid), dim3(AM_THREADS), smem, s, 1, a), "attend_mma");
}

// Merge n partials per row.  Partial i of row r is at
// part + r*row_stride + i*pstride*PSTRIDE(D): (out[D], max, sum, pad, pad).
// One CTA per (row, CB_COLS-column chunk); thread (c4, grp) folds partials
// grp, grp + NG, ... into a running (max, sum, out) -- every load is
// independent of the others, so the partials stream in one round trip --
// and the NG groups are merged in a fixed order (deterministic).
// final_out != nullptr: write out/sum in the store dtype at [B, Q, Hq, D];
// otherwise write the merged (out, max, sum).
template <typename T, bool X, int CB_COLS>
__global__ void __launch_bounds__(CB_THREADS)
combine_kernel(const float *part, int64_t row_stride, int64_t pstride, int n, int D, int Hq, int Q,
               T *final_out, float *merged, XArgs x, const float *mine, int64_t rows, int64_t *state) {
  // the epoch was advanced by this type's previous exchange; read it after
  // the dependency wait, which also covers a merge of the same type right
  // before this one in the stream
  griddep_wait();
  const unsigned long long e = X ? x_epoch(x, X_ATTN) : 0ull;
  constexpr int C4 = CB_COLS / 4;              // float4 columns per chunk
  constexpr int NG = CB_THREADS / C4;          // partial groups
  constexpr int NW = CB_THREADS / 32;          // warps (each merges 32 / C4 groups)
  static_assert(32 % C4 == 0, "a warp holds whole groups");
  __shared__ float4 s_acc[NW][C4];
  __shared__ float s_m[NW][C4], s_l[NW][C4];
  const int nch = (D + CB_COLS - 1) / CB_COLS;
  const int64_t row = blockIdx.x / nch;        // (b*Hq + h)*Q + t
  const int chunk = blockIdx.x % nch;
  const int Dp = partial_stride(D);
  bool ok = true;
  uint32_t flag = 0;
  const unsigned long long *xin = nullptr;
  if (X) {
    // this rank's partial of this (row, column chunk) -> slot [rank] of every
    // arena, one flagged word per value
    flag = x_flag(e);
    const int c0 = chunk * CB_COLS, c1 = min(D, c0 + CB_COLS);
    const float *src = mine + row * Dp;
    for (int d = 0; d < x.world; ++d) {
      unsigned long long *dst = x_region(x, d, e) + ((int64_t)x.rank * rows + row) * Dp;
      for (int c = c0 + threadIdx.x; c < c1; c += CB_THREADS) ll_store(dst + c, __float_as_uint(src[c]), flag);
      if (threadIdx.x < 2) ll_store(dst + D + threadIdx.x, __float_as_uint(src[D + threadIdx.x]), flag);
    }
    xin = x_region(x, x.rank, e);
    row_stride = Dp;
    pstride = rows;
    n = x.world;
  }
  const float *p = X ? nullptr : part + row * row_stride;
  const int c4 = threadIdx.x % C4, grp = threadIdx.x / C4;
  const int col = chunk * CB_COLS + c4 * 4;
  const int colc = col < D ? col : 0;          // in-bounds column for the loads
  float m = -INFINITY, l = 0.f;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
  for (int i = grp; i < n; i += NG) {
    float4 v;
    float mi, li;
    if (X) {
      const unsigned long long *wi = xin + row * row_stride + (int64_t)i * pstride * Dp;
      const unsigned long long w0 = ld_relaxed_sys(wi + colc), w1 = ld_relaxed_sys(wi + colc + 1);
      const unsigned long long w2 = ld_relaxed_sys(wi + colc + 2), w3 = ld_relaxed_sys(wi + colc + 3);
      const unsigned long long wm = ld_relaxed_sys(wi + D), wl = ld_relaxed_sys(wi + D + 1);
      v.x = __uint_as_float(ll_check(wi + colc, w0, flag, ok, x.budget));
      v.y = __uint_as_float(ll_check(wi + colc + 1, w1, flag, ok, x.budget));
      v.z = __uint_as_float(ll_check(wi + colc + 2, w2, flag, ok, x.budget));
      v.w = __uint_as_float(ll_check(wi + colc + 3, w3, flag, ok, x.budget));
      mi = __uint_as_float(ll_check(wi + D, wm, flag, ok, x.budget));
      li = __uint_as_float(ll_check(wi + D + 1, wl, flag, ok, x.budget));
    } else {
      const float *pi = p + (int64_t)i * pstride * Dp;
      v = __ldcg(reinterpret_cast<const float4 *>(pi + colc));
      mi = __ldcg(pi + D);
      li = __ldcg(pi + D + 1);
    }
    if (mi == -INFINITY) continue;             // empty partial
    const float mn = fmaxf(m, mi);
    const float a = __expf(m - mn), bi = __expf(mi - mn);   // m == -inf: a = 0
    acc.x = acc.x * a + v.x * bi;
    acc.y = acc.y * a + v.y * bi;
    acc.z = acc.z * a + v.z * bi;
    acc.w = acc.w * a + v.w * bi;
    l = l * a + li * bi;
    m = mn;
  }
  // the warp's groups of this column quad (lanes c4, c4 + C4, ...) merge by
  // shuffles in a fixed tree; both lanes of a pair compute the same
  // (commutative) result, so every lane ends with the warp's merge
#pragma unroll
  for (int off = C4; off < 32; off <<= 1) {
    const float mo = __shfl_xor_sync(KIV_FULL_MASK, m, off);
    const float lo = __shfl_xor_sync(KIV_FULL_MASK, l, off);
    float4 ao;
    ao.x = __shfl_xor_sync(KIV_FULL_MASK, acc.x, off);
    ao.y = __shfl_xor_sync(KIV_FULL_MASK, acc.y, off);
    ao.z = __shfl_xor_sync(KIV_FULL_MASK, acc.z, off);
    ao.w = __shfl_xor_sync(KIV_FULL_MASK, acc.w, off);
    const float mn = fmaxf(m, mo);
    const float a = m == -INFINITY ? 0.f : __expf(m - mn);
    const float b = mo == -INFINITY ? 0.f : __expf(mo - mn);
    acc.x = acc.x * a + ao.x * b;
    acc.y = acc.y * a + ao.y * b;
    acc.z = acc.z * a + ao.z * b;
    acc.w = acc.w * a + ao.w * b;
    l = l * a + lo * b;
    m = mn;
  }
  const int warp = threadIdx.x >> 5;
  if ((threadIdx.x & 31) < C4) {
    s_acc[warp][c4] = acc;
    s_m[warp][c4] = m;
    s_l[warp][c4] = l;
  }
  if (X && !ok)
    atomicOr(reinterpret_cast<unsigned long long *>(state + KIV_ST_ERROR),
             (unsigned long long)KIV_ERRBIT_WAIT_TIMEOUT);
  // a wait that gave up leaves some inputs unread: write no output
  const bool failed = __syncthreads_or(X && !ok) != 0;
  if (X) x_advance(x, X_ATTN, e);   // every CTA has read its inputs from the arena
  if (failed || grp != 0) return;
  float M = -INFINITY;
#pragma unroll
  for (int gi = 0; gi < NW; ++gi) M = fmaxf(M, s_m[gi][c4]);
  float L = 0.f;
  float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int gi = 0; gi < NW; ++gi) {
    const float mg = s_m[gi][c4];
    const float w = mg == -INFINITY ? 0.f : __expf(mg - M);
    const float4 u = s_acc[gi][c4];
    t.x += u.x * w;
    t.y += u.y * w;
    t.z += u.z * w;
    t.w += u.w * w;
    L += s_l[gi][c4] * w;
  }
  if (col >= D) return;
  if (final_out) {
    const int64_t tq = row % Q, bh = row / Q;
    const int64_t h = bh % Hq, b = bh / Hq;
    T *dst = final_out + ((b * Q + tq) * Hq + h) * D + col;
    dst[0] = Elem<T>::from_f(L > 0.f ? t.x / L : 0.f);
    dst[1] = Elem<T>::from_f(L > 0.f ? t.y / L : 0.f);
    dst[2] = Elem<T>::from_f(L > 0.f ? t.z / L : 0.f);
    dst[3] = Elem<T>::from_f(L > 0.f ? t.w / L : 0.f);
  } else {
    *reinterpret_cast<float4 *>(merged + row * Dp + col) = t;
    if (chunk == 0 && c4 == 0) {
      merged[row * Dp + D] = M;
      merged[row * Dp + D + 1] = L;
    }
  }
}

template <typename T>
static void launch_combine(const float *part, int64_t row_stride, int64_t pstride, int n, int D, int Hq,
                           int Q, int64_t rows, T *final_out, float *merged, cudaStream_t s) {
  const int64_t nch = ceil_div(D, CB_COLS_SPLIT);
  launch_pdl(combine_kernel<T, false, CB_COLS_SPLIT>, dim3((unsigned)(rows * nch)), dim3(CB_THREADS), 0, s, 1, part, row_stride,
             pstride, n, D, Hq, Q, final_out, merged, XArgs{}, (const float *)nullptr, rows, (int64_t *)nullptr);
}

template <typename T>
__global__ void gather_kernel(kiv_store st, const int32_t *sel, int32_t stride, int32_t P, T *ok, T *ov) {
  griddep_wait();
  constexpr int V = Elem<T>::V;
  const int D = st.head_dim, H = st.num_kv_heads, S = st.page_size;
  const int nv = D / V;
  const int64_t cold_len = st_ld(st.state, KIV_ST_COLD_LEN);
  const int64_t ng = (cold_len + S - 1) / S;   // global pages with rows
  const int64_t started = ng > st.shard_rank ? (ng - st.shard_rank + st.shard_count - 1) / st.shard_count : 0;
  const int64_t total = (int64_t)st.batch * H * P * nv;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int vi = (int)(e % nv);
    const int64_t i = (e / nv) % P;
    const int64_t bh = e / ((int64_t)nv * P);
    const int b = (int)(bh / H);
    const int64_t tok = sel[(int64_t)b * stride + i];
    if (tok < 0 || tok >= cold_len) continue;
    const int64_t p = tok / S;
    if (p % st.shard_count != st.shard_rank) continue;
    const int64_t lp = p / st.shard_count;
    const int64_t dst = (bh * P + i) * D + vi * V;
    if (st.host_capacity > 0 && lp < started - ring_pages(st)) {
      // a page of the host tier: read it there (mapped host memory)
      const int64_t src = (bh * st.host_capacity + lp * S + tok % S) * D + vi * V;
      st16(ok + dst, ld16(reinterpret_cast<const T *>(st.host_k) + src));
      st16(ov + dst, ld16(reinterpret_cast<const T *>(st.host_v) + src));
      continue;
    }
    const int64_t slot = (st.host_capacity > 0 ? lp % ring_pages(st) : lp) * S + tok % S;
    const int64_t src = (bh * st.cold_capacity + slot) * D + vi * V;
    st16(ok + dst, ld16(reinterpret_cast<const T *>(st.cold_k) + src));
    st16(ov + dst, ld16(reinterpret_cast<const T *>(st.cold_v) + src));
  }
}

template <typename T, int LPR, int VPL, int RCH>
static kiv_status launch_at(const AttnArgs<T> &a, cudaStream_t s) {
  const int D = a.st.head_dim;
  const size_t smem = (size_t)2 * AT_STAGES * ATT_TILE * D * sizeof(T) +
                      (size_t)RCH * ATT_TILE * sizeof(float) +
                      ((size_t)2 * AT_THREADS * Elem<T>::V + (size_t)RCH * D) * sizeof(float);
  auto kern = attend_split_kernel<T, LPR, VPL, RCH>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  const int H = a.st.num_kv_heads;
  const int rows_kv = (a.q.num_query_heads / H) * a.q.query_len;
  const int64_t nchunks = ceil_div(rows_kv, RCH);
  const int64_t grid = (int64_t)a.st.batch * H * nchunks * a.n_split;
  if (grid > 0x7fffffff) return KIV_ERR_ARG;
  return cuda_status(launch_pdl(kern, dim3((unsigned)grid), dim3(AT_THREADS), smem, s, 1, a), "attend_split");
}

template <typename T>
static kiv_status dispatch_at(AttnArgs<T> a, cudaStream_t s) {
  const int nv = a.st.head_dim / Elem<T>::V;
  const int rows_kv = (a.q.num_query_heads / a.st.num_kv_heads) * a.q.query_len;
  const bool small = rows_kv <= 4;
  if (nv * (small ? 4 : 8) > 2 * AT_THREADS) return KIV_ERR_UNSUPPORTED;
#define KIV_AT(LPR, VPL) \
  return small ? launch_at<T, LPR, VPL, 4>(a, s) : launch_at<T, LPR, VPL, 8>(a, s)
  if (nv <= 2) KIV_AT(2, 1);
  if (nv <= 4) KIV_AT(4, 1);
  if (nv <= 8) KIV_AT(8, 1);
  if (nv <= 16) KIV_AT(16, 1);
  if (nv <= 32) KIV_AT(32, 1);
  if (nv <= 64) KIV_AT(32, 2);
#undef KIV_AT
  return KIV_ERR_UNSUPPORTED;
}

// ---------------------------------------------------------------------------
// Prefill-shaped attention (more than 16 query rows per KV head, e.g. a
// 4096-position chunk): flash-style, no split partials.  CTA = (batch row, KV
// head, 64 of its G*Q query rows); 4 warps own 16 rows each and run over all
// keys [selected cold ; hot] in tiles of 64: K and V rows gathered by
// cp.async into a 2-stage ring (padded rows), S = Q K^T and O += P V on
// m16n8k16 MMAs with the query fragments held in registers, online softmax in
// registers (P rounded to the store dtype for the second MMA, the running sum
// kept in fp32).  Hot rows past the last causally visible one of the tile are
// not loaded.  Masking and soft-capping as attend_mma_kernel: soft-cap on the
// scaled score, then the causal rule / additive mask on hot columns only.
constexpr int AP_THREADS = 128;
constexpr int AP_ROWS = 64;
constexpr int AP_KEYS = 64;

__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <typename T, int D>
__global__ void __launch_bounds__(AP_THREADS)
attend_prefill_kernel(AttnArgs<T> a, T *out, float *partial_out) {
  extern __shared__ __align__(128) uint8_t ap_smem[];
  using Op = MmaOp<T>;
  constexpr int PITCH = D * 2 + 16;            // bytes per staged row (conflict-free ldmatrix)
  constexpr int NC = D / 8;                    // 16-byte chunks per row
  constexpr int KD = D / 16;                   // k-steps of S = Q K^T
  constexpr int NO = D / 8;                    // 8-column output tiles
  const kiv_store &st = a.st;
  const kiv_query &q = a.q;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t4 = lane & 3;
  const int H = st.num_kv_heads, S = st.page_size;
  const int Hq = q.num_query_heads, G = Hq / H, Q = q.query_len;
  const int rows_kv = G * Q;
  const int nrt = (rows_kv + AP_ROWS - 1) / AP_ROWS;
  const int rt = blockIdx.x % nrt;
  const int bhi = blockIdx.x / nrt;
  const int b = bhi / H, kvh = bhi % H;
  const int r0 = rt * AP_ROWS;
  uint8_t *qs = ap_smem;                       // [64][PITCH]
  uint8_t *ks = qs + AP_ROWS * PITCH;          // [2][64][PITCH]
  uint8_t *vs = ks + 2 * AP_KEYS * PITCH;      // [2][64][PITCH]

  // ---- prologue: the query tile and the hot window were written before the step
  {
    const T *qb = reinterpret_cast<const T *>(q.q);
    for (int e = threadIdx.x; e < AP_ROWS * NC; e += AP_THREADS) {
      const int rr = e / NC, c = e % NC, r = r0 + rr;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (r < rows_kv) {
        const int h = kvh * G + r / Q, tq = r % Q;
        v = ld16(qb + b * q.stride_b + h * q.stride_h + tq * q.stride_t + c * 8);
      }
      *reinterpret_cast<uint4 *>(qs + rr * PITCH + c * 16) = v;
    }
  }
  const int64_t hot_len = st_ld(st.state, KIV_ST_HOT_LEN);
  const int64_t hot_start = st_ld(st.state, KIV_ST_HOT_START);
  const int64_t hot_lo = hot_len * a.hot_slice / a.hot_slices;
  const int64_t hot_hi = hot_len * (a.hot_slice + 1) / a.hot_slices;
  // ---- the selection (previous kernel) is needed from here on
  griddep_wait();
  const int64_t ncold = a.w.selcnt[b];
  int64_t hot_use = hot_hi - hot_lo;
  if (a.mask.causal && a.mask.add == nullptr) {
    const int rlast = min(rows_kv, r0 + AP_ROWS) - 1;
    const int tq_max = (r0 / Q != rlast / Q) ? Q - 1 : rlast % Q;
    hot_use = std::max<int64_t>(0, std::min<int64_t>(hot_use, hot_len - Q + tq_max + 1 - hot_lo));
  }
  const int64_t nkeys = ncold + hot_use;
  const int ntile = (int)((nkeys + AP_KEYS - 1) / AP_KEYS);
  const T *cold_k = reinterpret_cast<const T *>(st.cold_k);
  const T *cold_v = reinterpret_cast<const T *>(st.cold_v);
  const T *hot_k = reinterpret_cast<const T *>(st.hot_k);
  const T *hot_v = reinterpret_cast<const T *>(st.hot_v);
  const int32_t *selb = a.sel + (int64_t)b * a.sel_stride;
  const int64_t bhk = (int64_t)b * H + kvh;
  auto issue = [&](int t) {
    const int stage = t & 1;
    const int64_t k0 = (int64_t)t * AP_KEYS;
    for (int e = threadIdx.x; e < AP_KEYS * NC; e += AP_THREADS) {
      const int kr = e / NC, c = e % NC;
      const int64_t k = k0 + kr;
      uint8_t *dk = ks + ((size_t)stage * AP_KEYS + kr) * PITCH + c * 16;
      uint8_t *dv = vs + ((size_t)stage * AP_KEYS + kr) * PITCH + c * 16;
      if (k < nkeys) {
        int64_t off;
        const T *bk, *bv;
        if (k < ncold) {
          const int64_t tok = selb[k], p = tok / S;
          off = (bhk * st.cold_capacity + page_slot(st, a.w, p / st.shard_count) * S + tok % S) * D;
          bk = cold_k;
          bv = cold_v;
        } else {
          const int64_t slot = (hot_start + hot_lo + (k - ncold)) % st.hot_capacity;
          off = (bhk * st.hot_capacity + slot) * D;
          bk = hot_k;
          bv = hot_v;
        }
        cp_async16(dk, bk + off + c * 8);
        cp_async16(dv, bv + off + c * 8);
      } else {
        // past the last key: zero rows (P is 0 there, V must not be NaN)
        *reinterpret_cast<uint4 *>(dk) = make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4 *>(dv) = make_uint4(0, 0, 0, 0);
      }
    }
    cp_async_commit();
  };
  if (ntile > 0) issue(0);
  if (ntile > 1) issue(1);
  __syncthreads();   // query tile staged
  uint32_t qf[KD][4];
#pragma unroll
  for (int kk = 0; kk < KD; ++kk)
    ldsm_x4(qf[kk], qs + (warp * 16 + (lane & 15)) * PITCH + (kk * 16 + 8 * (lane >> 4)) * 2);
  float o[NO][4];
#pragma unroll
  for (int i = 0; i < NO; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
  // the two query rows of this thread: (head, position) and causal limits
  int rrow[2], hrow[2], tqrow[2];
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    rrow[hh] = r0 + warp * 16 + g + 8 * hh;
    hrow[hh] = kvh * G + rrow[hh] / Q;
    tqrow[hh] = rrow[hh] % Q;
  }
  // tiles whose every (row, key) of this warp is visible skip the per-element
  // masking: all 16 rows exist, and (causal) the tile's last hot row is visible
  // to the warp's earliest position
  const bool rows_full = r0 + warp * 16 + 15 < rows_kv;
  int tq_min = min(tqrow[0], tqrow[1]);
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) tq_min = min(tq_min, __shfl_xor_sync(KIV_FULL_MASK, tq_min, o));

  for (int t = 0; t < ntile; ++t) {
    if (t + 1 < ntile) cp_async_wait<1>();
    else cp_async_wait<0>();
    __syncthreads();
    const int stage = t & 1;
    const uint8_t *kst = ks + (size_t)stage * AP_KEYS * PITCH;
    const uint8_t *vst = vs + (size_t)stage * AP_KEYS * PITCH;
    // ---- S = Q K^T: 16 rows x 64 keys per warp
    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < KD; ++kk) {
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t kb[4];
        ldsm_x4(kb, kst + (np * 16 + (lane >> 4) * 8 + (lane & 7)) * PITCH + (kk * 16 + ((lane >> 3) & 1) * 8) * 2);
        Op::mma(s[2 * np], qf[kk], kb[0], kb[1]);
        Op::mma(s[2 * np + 1], qf[kk], kb[2], kb[3]);
      }
    }
    // ---- scale, soft-cap, mask; online softmax per row
    const int64_t k0 = (int64_t)t * AP_KEYS;
    float mx[2] = {-INFINITY, -INFINITY};
    const int64_t k_last = k0 + AP_KEYS - 1;
    const bool fast = rows_full && a.mask.add == nullptr && k_last < nkeys &&
                      (!a.mask.causal || k_last < ncold || hot_lo + (k_last - ncold) <= hot_len - Q + tq_min);
    if (fast) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          float sc = s[j][i] * q.scaling;
          if (q.softcap > 0.f) sc = q.softcap * tanhf(sc / q.softcap);
          s[j][i] = sc;
          mx[i >> 1] = fmaxf(mx[i >> 1], sc);
        }
      }
    } else
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int hh = i >> 1;
        const int64_t k = k0 + j * 8 + 2 * t4 + (i & 1);
        float sc = -INFINITY;
        if (k < nkeys && rrow[hh] < rows_kv) {
          sc = s[j][i] * q.scaling;
          if (q.softcap > 0.f) sc = q.softcap * tanhf(sc / q.softcap);
          if (k >= ncold) {
            const int64_t jh = hot_lo + (k - ncold);
            if (a.mask.causal && jh > hot_len - Q + tqrow[hh]) sc = -INFINITY;
            if (a.mask.add != nullptr)
              sc += a.mask.add[b * a.mask.stride_b + hrow[hh] * a.mask.stride_h + tqrow[hh] * a.mask.stride_t + jh];
          }
        }
        s[j][i] = sc;
        mx[hh] = fmaxf(mx[hh], sc);
      }
    }
    float alpha[2];
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      mx[hh] = fmaxf(mx[hh], __shfl_xor_sync(KIV_FULL_MASK, mx[hh], 1));
      mx[hh] = fmaxf(mx[hh], __shfl_xor_sync(KIV_FULL_MASK, mx[hh], 2));
      const float mn = fmaxf(mrow[hh], mx[hh]);
      alpha[hh] = mn == -INFINITY ? 1.f : __expf(mrow[hh] - mn);   // mrow == -inf: 0
      mrow[hh] = mn;
    }
    float lsum[2] = {0.f, 0.f};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int hh = i >> 1;
        const float p = (s[j][i] == -INFINITY) ? 0.f : __expf(s[j][i] - mrow[hh]);
        s[j][i] = p;
        lsum[hh] += p;
      }
    }
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) lrow[hh] = lrow[hh] * alpha[hh] + lsum[hh];
#pragma unroll
    for (int i = 0; i < NO; ++i) {
      o[i][0] *= alpha[0];
      o[i][1] *= alpha[0];
      o[i][2] *= alpha[1];
      o[i][3] *= alpha[1];
    }
    // ---- O += P V (P from the S accumulators, rounded to the store dtype)
#pragma unroll
    for (int kc = 0; kc < 4; ++kc) {
      uint32_t pa[4];
      pa[0] = Op::pack2(s[2 * kc][0], s[2 * kc][1]);
      pa[1] = Op::pack2(s[2 * kc][2], s[2 * kc][3]);
      pa[2] = Op::pack2(s[2 * kc + 1][0], s[2 * kc + 1][1]);
      pa[3] = Op::pack2(s[2 * kc + 1][2], s[2 * kc + 1][3]);
      const uint8_t *vrow = vst + (kc * 16 + (lane & 15)) * PITCH + 8 * (lane >> 4) * 2;
#pragma unroll
      for (int nt = 0; nt < NO; nt += 2) {
        uint32_t vb[4];
        ldsm_x4_t(vb, vrow + nt * 16);
        Op::mma(o[nt], pa, vb[0], vb[1]);
        Op::mma(o[nt + 1], pa, vb[2], vb[3]);
      }
    }
    __syncthreads();   // stage consumed
    if (t + 2 < ntile) issue(t + 2);
  }
  // ---- rows: final output [B, Q, Hq, D] or the (out, max, sum) partial
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    float l = lrow[hh];
    l += __shfl_xor_sync(KIV_FULL_MASK, l, 1);
    l += __shfl_xor_sync(KIV_FULL_MASK, l, 2);
    if (rrow[hh] >= rows_kv) continue;
    if (out) {
      const float inv = l > 0.f ? 1.f / l : 0.f;
      T *dst = out + (((int64_t)b * Q + tqrow[hh]) * Hq + hrow[hh]) * D + 2 * t4;
#pragma unroll
      for (int nt = 0; nt < NO; ++nt)
        *reinterpret_cast<uint32_t *>(dst + nt * 8) = Op::pack2(o[nt][2 * hh] * inv, o[nt][2 * hh + 1] * inv);
    } else {
      const int Dp = partial_stride(D);
      float *dst = partial_out + (((int64_t)b * Hq + hrow[hh]) * Q + tqrow[hh]) * Dp;
#pragma unroll
      for (int nt = 0; nt < NO; ++nt)
        *reinterpret_cast<float2 *>(dst + nt * 8 + 2 * t4) = make_float2(o[nt][2 * hh], o[nt][2 * hh + 1]);
      if (t4 == 0) {
        dst[D] = mrow[hh];
        dst[D + 1] = l;
      }
    }
  }
}

template <typename T>
static bool attend_prefill_eligible(const kiv_store *st, const kiv_query *q) {
  const int64_t rows_kv = (int64_t)(q->num_query_heads / st->num_kv_heads) * q->query_len;
  const int D = st->head_dim;
  return sizeof(T) == 2 && rows_kv > AM_ROWS && (D == 64 || D == 96 || D == 128) &&
         getenv("KIV_DISABLE_MMA_ATTN") == nullptr;
}

template <typename T>
static kiv_status launch_ap(const AttnArgs<T> &a, T *out, float *partial_out, cudaStream_t s) {
  const int D = a.st.head_dim;
  const int64_t rows_kv = (int64_t)(a.q.num_query_heads / a.st.num_kv_heads) * a.q.query_len;
  const int64_t grid = (int64_t)a.st.batch * a.st.num_kv_heads * ceil_div(rows_kv, AP_ROWS);
  if (grid > 0x7fffffff) return KIV_ERR_ARG;
  const size_t smem = (size_t)(AP_ROWS + 4 * AP_KEYS) * (D * 2 + 16);
  cudaError_t e;
#define KIV_AP(DD)                                                                                       \
  do {                                                                                                   \
    cudaFuncSetAttribute(attend_prefill_kernel<T, DD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); \
    e = launch_pdl(attend_prefill_kernel<T, DD>, dim3((unsigned)grid), dim3(AP_THREADS), smem, s, 1, a, out, \
                   partial_out);                                                                         \
  } while (0)
  if (D == 64) KIV_AP(64);
  else if (D == 96) KIV_AP(96);
  else KIV_AP(128);
#undef KIV_AP
  return cuda_status(e, "attend_prefill");
}

template <typename T>
static kiv_status attend_t(const kiv_store *st, const kiv_query *q, const kiv_mask *m,
                           const Workspace &w, const int32_t *sel, int32_t sel_stride,
                           int32_t hot_slice, int32_t hot_slices, void *out, float *partial_out,
                           cudaStream_t s, const kiv_peer_rows *peers = nullptr) {
  // host tier: the selected rows of host pages reach their staging pages first
  KIV_CHECK(launch_stage_selected(st, w, sel, sel_stride, s));
  const int64_t expected_hot = st->hot_hint > 0 ? st->hot_hint : st->hot_capacity;
  AttnArgs<T> a = {};
  if (peers) {
    if (!attend_mma_eligible<T>(st, q)) {
      set_error("peer-row attention needs 16-bit rows, <= %d query rows per KV head, head_dim % 64 == 0",
                AM_ROWS);
      return KIV_ERR_UNSUPPORTED;
    }
    a.peers = 1;
    for (int r = 0; r < st->shard_count; ++r) {
      a.peer_k[r] = peers->cold_k[r];
      a.peer_v[r] = peers->cold_v[r];
    }
  }
  a.st = *st;
  a.q = *q;
  if (m) a.mask = *m;
  else a.mask = kiv_mask{nullptr, 0, 0, 0, 0, 0};
  a.w = w;
  a.sel = sel;
  a.sel_stride = sel_stride;
  a.hot_slice = hot_slice;
  a.hot_slices = hot_slices;
  const int H = st->num_kv_heads;
  const int rows_kv = (q->num_query_heads / H) * q->query_len;
  const int64_t nchunks = ceil_div(rows_kv, rows_kv <= 4 ? 4 : 8);
  const int64_t base = (int64_t)st->batch * H * nchunks;
  // one tile of keys per split where the SMs allow it (at most about one CTA
  // per SM in total): each CTA then waits for a single round of row copies
  const int64_t keys_hint = std::max<int64_t>(1, (int64_t)q->top_p + expected_hot);
  a.n_split = (int)std::max<int64_t>(
      1, std::min<int64_t>({w.split_cap, ceil_div(keys_hint, ATT_TILE), ceil_div(sm_count(), base)}));
  kiv_status rc;
  if constexpr (sizeof(T) == 2) {
    if (attend_prefill_eligible<T>(st, q))
      return launch_ap<T>(a, partial_out ? nullptr : reinterpret_cast<T *>(out), partial_out, s);
    rc = attend_mma_eligible<T>(st, q) ? launch_am<T>(a, s) : dispatch_at<T>(a, s);
  } else {
    rc = dispatch_at<T>(a, s);
  }
  if (rc != KIV_OK) return rc;
  const int64_t rows = w.R;
  const int64_t rs = w.split_cap * partial_stride(st->head_dim);
  launch_combine<T>(w.part, rs, 1, a.n_split, st->head_dim, q->num_query_heads, q->query_len, rows,
                    partial_out ? nullptr : reinterpret_cast<T *>(out), partial_out, s);
  return cuda_status(cudaGetLastError(), "attend_combine");
}

kiv_status launch_attend_peers(const kiv_store *st, const kiv_query *q, const kiv_mask *m, const Workspace &w,
                               const int32_t *sel, int32_t sel_stride, const kiv_peer_rows *peers, void *out,
                               cudaStream_t s) {
  switch (st->dtype) {
    case KIV_DTYPE_BF16:
      return attend_t<__nv_bfloat16>(st, q, m, w, sel, sel_stride, 0, 1, out, nullptr, s, peers);
    case KIV_DTYPE_F16:
      return attend_t<__half>(st, q, m, w, sel, sel_stride, 0, 1, out, nullptr, s, peers);
  }
  set_error("peer-row attention needs a 16-bit store");
  return KIV_ERR_UNSUPPORTED;
}

kiv_status launch_attend(const kiv_store *st, const kiv_query *q, const kiv_mask *m,
                         const Workspace &w, const int32_t *sel, int32_t sel_stride,
                         int32_t hot_slice, int32_t hot_slices, void *out, float *partial_out,
                         cudaStream_t s) {
  switch (st->dtype) {
    case KIV_DTYPE_F32:
      return attend_t<float>(st, q, m, w, sel, sel_stride, hot_slice, hot_slices, out, partial_out, s);
    case KIV_DTYPE_BF16:
      return attend_t<__nv_bfloat16>(st, q, m, w, sel, sel_stride, hot_slice, hot_slices, out,
                                     partial_out, s);
    case KIV_DTYPE_F16:
      return attend_t<__half>(st, q, m, w, sel, sel_stride, hot_slice, hot_slices, out, partial_out, s);
  }
  return KIV_ERR_UNSUPPORTED;
}

kiv_status launch_attend_merge(const kiv_store *st, const kiv_query *q, const float *partials,
                               int32_t n, void *out, cudaStream_t s, const XArgs *x) {
  const int64_t rows = (int64_t)st->batch * q->num_query_heads * q->query_len;
  const int D = st->head_dim, Dp = partial_stride(D);
  if (x) {
    // partials: this rank's [R, Dp]; the ranks' partials meet in the arenas
    const int64_t nch = ceil_div(D, CB_COLS_X);
    const dim3 grid((unsigned)(rows * nch));
#define KIV_XC(TT)                                                                                         \
  launch_pdl(combine_kernel<TT, true, CB_COLS_X>, grid, dim3(CB_THREADS), 0, s, 1, (const float *)nullptr, (int64_t)Dp,      \
             rows, x->world, D, q->num_query_heads, q->query_len, (TT *)out, (float *)nullptr, *x, partials, rows, \
             st->state)
    switch (st->dtype) {
      case KIV_DTYPE_F32: KIV_XC(float); break;
      case KIV_DTYPE_BF16: KIV_XC(__nv_bfloat16); break;
      case KIV_DTYPE_F16: KIV_XC(__half); break;
      default: return KIV_ERR_UNSUPPORTED;
    }
#undef KIV_XC
    return cuda_status(cudaGetLastError(), "attend_exchange_merge");
  }
  // partials [n, R, Dp]: row r of partial i at (i*R + r)*Dp
  switch (st->dtype) {
    case KIV_DTYPE_F32:
      launch_combine<float>(partials, Dp, rows, n, D, q->num_query_heads, q->query_len, rows,
                            (float *)out, nullptr, s);
      break;
    case KIV_DTYPE_BF16:
      launch_combine<__nv_bfloat16>(partials, Dp, rows, n, D, q->num_query_heads, q->query_len, rows,
                                    (__nv_bfloat16 *)out, nullptr, s);
      break;
    case KIV_DTYPE_F16:
      launch_combine<__half>(partials, Dp, rows, n, D, q->num_query_heads, q->query_len, rows,
                             (__half *)out, nullptr, s);
      break;
    default:
      return KIV_ERR_UNSUPPORTED;
  }
  return cuda_status(cudaGetLastError(), "attend_merge");
}

// per-rank payload bytes of the three exchanges
void exchange_payloads(const kiv_store *st, const kiv_query *q, int64_t *cb, int64_t *fb, int64_t *ab,
                       int64_t *xb) {
  const int64_t R = (int64_t)st->batch * q->num_query_heads * q->query_len;
  // one flagged 64-bit word per 32-bit value
  *cb = R * q->top_pages * 16;
  *fb = (int64_t)st->batch * q->top_p * 16;
  *ab = R * partial_stride(st->head_dim) * 8;
  // candidate exchange: one word per candidate position of every batch row
  *xb = (int64_t)st->batch * workspace_layout(st, q, nullptr).c_cap * 8;
}

kiv_status launch_gather(const kiv_store *st, const int32_t *sel, int32_t sel_stride, int32_t P,
                         void *ok, void *ov, cudaStream_t s) {
  if (P <= 0) return KIV_OK;
  const int64_t total = (int64_t)st->batch * st->num_kv_heads * P * (st->head_dim * elem_bytes(st->dtype) / 16);
  const int64_t grid = std::max<int64_t>(1, std::min<int64_t>(ceil_div(total, 256), (int64_t)sm_count() * 8));
  switch (st->dtype) {
    case KIV_DTYPE_F32:
      launch_pdl(gather_kernel<float>, dim3((unsigned)grid), dim3(256), 0, s, 1, *st, sel, sel_stride, P,
                 (float *)ok, (float *)ov);
      break;
    case KIV_DTYPE_BF16:
      launch_pdl(gather_kernel<__nv_bfloat16>, dim3((unsigned)grid), dim3(256), 0, s, 1, *st, sel, sel_stride, P,
                                                                  (__nv_bfloat16 *)ok, (__nv_bfloat16 *)ov);
      break;
    case KIV_DTYPE_F16:
      launch_pdl(gather_kernel<__half>, dim3((unsigned)grid), dim3(256), 0, s, 1, *st, sel, sel_stride, P,
                 (__half *)ok, (__half *)ov);
      break;
    default:
      return KIV_ERR_UNSUPPORTED;
  }
  return cuda_status(cudaGetLastError(), "gather");
}

}  // namespace kiv
