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
#include "internal.h"

namespace kiv {

constexpr int AT_THREADS = 256;
constexpr int AT_STAGES = 2;
constexpr int CB_THREADS = 256;

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
  __syncthreads();
  // ---- the selection (previous kernel) is needed from here on
  griddep_wait();
  const int64_t ncold = a.w.selcnt[b];
  const int64_t nkeys = ncold + (hot_hi - hot_lo);
  int64_t kps = (nkeys + a.n_split - 1) / a.n_split;
  kps = (kps + 7) / 8 * 8;
  const int64_t k_lo = std::min<int64_t>(nkeys, split * kps);
  const int64_t k_hi = std::min<int64_t>(nkeys, k_lo + kps);
  const int ntile = (int)((k_hi - k_lo + ATT_TILE - 1) / ATT_TILE);

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

  auto key_rows = [&](int64_t k, const T *&pk, const T *&pv) {
    if (k < ncold) {
      const int64_t tok = selb[k];
      const int64_t p = tok / S;
      const int64_t slot = (p / st.shard_count) * S + tok % S;
      pk = cold_k + (bhk * st.cold_capacity + slot) * D;
      pv = cold_v + (bhk * st.cold_capacity + slot) * D;
    } else {
      const int64_t j = hot_lo + (k - ncold);
      const int64_t slot = (hot_start + j) % st.hot_capacity;
      pk = hot_k + (bhk * st.hot_capacity + slot) * D;
      pv = hot_v + (bhk * st.hot_capacity + slot) * D;
    }
  };
  // warp 0 issues one tile: lane i copies key row i (K and V)
  auto issue = [&](int t) {
    const int stage = t % AT_STAGES;
    const int64_t k0 = k_lo + (int64_t)t * ATT_TILE;
    const int n = (int)std::min<int64_t>(ATT_TILE, k_hi - k0);
    if (lane == 0) mbar_arrive_tx(&bars[stage], 2u * n * row_bytes);
    __syncwarp();
    if (lane < n) {
      const T *pk, *pv;
      key_rows(k0 + lane, pk, pv);
      bulk_g2s(kt + ((size_t)stage * ATT_TILE + lane) * D, pk, row_bytes, &bars[stage]);
      bulk_g2s(vt + ((size_t)stage * ATT_TILE + lane) * D, pv, row_bytes, &bars[stage]);
    }
  };
  if (warp == 0) {
    for (int t = 0; t < (ntile < AT_STAGES ? ntile : AT_STAGES); ++t) issue(t);
  }

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
            if (k >= ncold) {
              const int64_t j = hot_lo + (k - ncold);
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
  const int Dp = partial_stride(D);
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

// Merge n partials per row.  Partial i of row r is at
// part + r*row_stride + i*pstride*PSTRIDE(D): (out[D], max, sum, pad, pad).
// One CTA per row: threads over partials for the max and the sum, then warps
// over partials and lanes over float4 columns for the output, reduced across
// warps in shared memory.  final_out != nullptr: write out/sum in the store
// dtype at [B, Q, Hq, D]; otherwise write the merged (out, max, sum).
template <typename T>
__global__ void __launch_bounds__(CB_THREADS)
combine_kernel(const float *part, int64_t row_stride, int64_t pstride, int n, int D, int Hq, int Q,
               T *final_out, float *merged) {
  griddep_wait();
  extern __shared__ float cb_smem[];
  float *wgt = cb_smem;                       // [n] exp(m_i - M)
  float *red = cb_smem + ((n + 3) & ~3);      // [CB_THREADS/32][D]
  __shared__ float s_red[CB_THREADS / 32];
  __shared__ float s_M, s_L;
  const int64_t row = blockIdx.x;  // (b*Hq + h)*Q + t
  const float *p = part + row * row_stride;
  const int Dp = partial_stride(D);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  constexpr int NW = CB_THREADS / 32;
  float m = -INFINITY;
  for (int i = threadIdx.x; i < n; i += CB_THREADS) m = fmaxf(m, p[(int64_t)i * pstride * Dp + D]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(KIV_FULL_MASK, m, o));
  if (lane == 0) s_red[warp] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float M = -INFINITY;
    for (int w = 0; w < NW; ++w) M = fmaxf(M, s_red[w]);
    s_M = M;
  }
  __syncthreads();
  const float M = s_M;
  float l = 0.f;
  for (int i = threadIdx.x; i < n; i += CB_THREADS) {
    const float *pi = p + (int64_t)i * pstride * Dp;
    const float mi = pi[D];
    const float wi = (mi == -INFINITY) ? 0.f : __expf(mi - M);
    wgt[i] = wi;
    l += pi[D + 1] * wi;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(KIV_FULL_MASK, l, o);
  __syncthreads();
  if (lane == 0) s_red[warp] = l;
  __syncthreads();
  if (threadIdx.x == 0) {
    float L = 0.f;
    for (int w = 0; w < NW; ++w) L += s_red[w];
    s_L = L;
  }
  // weighted sum of the partial outputs: warp w takes partials w, w+NW, ...
  const int nd4 = D / 4;
  for (int c0 = 0; c0 < nd4; c0 += 32 * 2) {
    float4 acc[2] = {make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f)};
    for (int i = warp; i < n; i += NW) {
      const float wi = wgt[i];
      const float4 *pi = reinterpret_cast<const float4 *>(p + (int64_t)i * pstride * Dp);
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int c = c0 + lane + 32 * j;
        if (c < nd4 && wi != 0.f) {
          const float4 v = pi[c];
          acc[j].x = fmaf(wi, v.x, acc[j].x);
          acc[j].y = fmaf(wi, v.y, acc[j].y);
          acc[j].z = fmaf(wi, v.z, acc[j].z);
          acc[j].w = fmaf(wi, v.w, acc[j].w);
        }
      }
    }
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int c = c0 + lane + 32 * j;
      if (c < nd4) reinterpret_cast<float4 *>(red + warp * D)[c] = acc[j];
    }
  }
  __syncthreads();
  const float L = s_L;
  for (int d = threadIdx.x; d < D; d += CB_THREADS) {
    float acc = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) acc += red[w * D + d];
    if (final_out) {
      const int64_t t = row % Q, bh = row / Q;
      const int64_t h = bh % Hq, b = bh / Hq;
      final_out[((b * Q + t) * Hq + h) * D + d] = Elem<T>::from_f(L > 0.f ? acc / L : 0.f);
    } else {
      merged[row * Dp + d] = acc;
    }
  }
  if (!final_out && threadIdx.x == 0) {
    merged[row * Dp + D] = M;
    merged[row * Dp + D + 1] = L;
  }
}

template <typename T>
static void launch_combine(const float *part, int64_t row_stride, int64_t pstride, int n, int D, int Hq,
                           int Q, int64_t rows, T *final_out, float *merged, cudaStream_t s) {
  const size_t smem = (size_t)(((n + 3) & ~3) + (CB_THREADS / 32) * D) * sizeof(float);
  auto kern = combine_kernel<T>;
  if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  launch_pdl(kern, dim3((unsigned)rows), dim3(CB_THREADS), smem, s, 1, part, row_stride, pstride, n, D, Hq, Q,
             final_out, merged);
}

template <typename T>
__global__ void gather_kernel(kiv_store st, const int32_t *sel, int32_t stride, int32_t P, T *ok, T *ov) {
  griddep_wait();
  constexpr int V = Elem<T>::V;
  const int D = st.head_dim, H = st.num_kv_heads, S = st.page_size;
  const int nv = D / V;
  const int64_t cold_len = st_ld(st.state, KIV_ST_COLD_LEN);
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
    const int64_t slot = (p / st.shard_count) * S + tok % S;
    const int64_t src = (bh * st.cold_capacity + slot) * D + vi * V;
    const int64_t dst = (bh * P + i) * D + vi * V;
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

template <typename T>
static kiv_status attend_t(const kiv_store *st, const kiv_query *q, const kiv_mask *m,
                           const Workspace &w, const int32_t *sel, int32_t sel_stride,
                           int32_t hot_slice, int32_t hot_slices, void *out, float *partial_out,
                           cudaStream_t s) {
  const int64_t expected_hot = st->hot_hint > 0 ? st->hot_hint : st->hot_capacity;
  AttnArgs<T> a;
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
  kiv_status rc = dispatch_at<T>(a, s);
  if (rc != KIV_OK) return rc;
  const int64_t rows = w.R;
  const int64_t rs = w.split_cap * partial_stride(st->head_dim);
  launch_combine<T>(w.part, rs, 1, a.n_split, st->head_dim, q->num_query_heads, q->query_len, rows,
                    partial_out ? nullptr : reinterpret_cast<T *>(out), partial_out, s);
  return cuda_status(cudaGetLastError(), "attend_combine");
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
                               int32_t n, void *out, cudaStream_t s) {
  const int64_t rows = (int64_t)st->batch * q->num_query_heads * q->query_len;
  const int D = st->head_dim, Dp = partial_stride(D);
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
