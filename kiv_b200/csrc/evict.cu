// Kernel (a): append new rows to the hot ring and evict the oldest rows into
// the cold tier, writing each completed page's mean-K summary in the same pass.
//
// Reference behaviour restated (kiv/tiered_cache.py:107-142 update + :55-72
// _evict_layer, kiv/cold_store.py:142-184 evict_from_hot):
//   hot ++ new, then the oldest max(0, hot_len + n_new - keep) rows move to
//   the cold tier in token order; every page of page_size rows that fills gets
//   summary = mean over its rows of K.
// Here the cold tier is a preallocated token-slot array in HBM and the hot
// window is a ring, so nothing is re-concatenated: each evicted row is copied
// once (16-byte vectors) and the summary is an fp32 sum in token order divided
// by page_size, rounded to the store dtype.
#include "common.cuh"
#include "internal.h"

namespace kiv {

constexpr int EV_THREADS = 256;
constexpr int APPEND_ROWS = 16;   // new rows per append block

template <typename T>
__global__ void __launch_bounds__(EV_THREADS)
append_evict_kernel(kiv_store st, const T *__restrict__ k_new, const T *__restrict__ v_new,
                    int64_t sb, int64_t sh, int64_t stt, int32_t n_new, int64_t keep,
                    int64_t n_evict_max, int32_t pages_per_bh, int32_t app_per_bh) {
  griddep_wait();
  constexpr int V = Elem<T>::V;
  const int D = st.head_dim, S = st.page_size, H = st.num_kv_heads;
  const int nv = D / V;
  const int64_t cold_len = st_ld(st.state, KIV_ST_COLD_LEN);
  const int64_t hot_start = st_ld(st.state, KIV_ST_HOT_START);
  const int64_t hot_len = st_ld(st.state, KIV_ST_HOT_LEN);
  const int64_t hcap = st.hot_capacity;
  // direct mode: the new rows go straight to the cold tier, hot untouched
  const bool direct = keep == KIV_KEEP_DIRECT;
  int64_t n_ev = 0;
  if (direct) {
    n_ev = n_new;
  } else if (keep >= 0) {
    n_ev = hot_len + n_new - keep;
    n_ev = n_ev < 0 ? 0 : (n_ev > hot_len + n_new ? hot_len + n_new : n_ev);
  }
  // capacity guards (the host checks these too; never write out of bounds)
  const int64_t hot_after = direct ? hot_len : hot_len + n_new - n_ev;
  bool ok = direct || (hot_len + n_new <= hcap) || (hcap == 0 && hot_len == 0 && n_ev == n_new);
  ok = ok && (direct || hot_after <= (hcap > 0 ? hcap : 0));
  // the highest page this shard owns among those the evicted rows reach must
  // fit its local slots (with a host tier: its ring plus host pages)
  const bool tiered = st.host_capacity > 0;
  const int64_t ring = ring_pages(st);
  const int64_t last_page = (cold_len + n_ev + S - 1) / S - 1;  // global page of the last evicted row
  if (n_ev > 0 && last_page >= st.shard_rank &&
      ((last_page - st.shard_rank) / st.shard_count + 1) > (tiered ? summary_pages(st) : st.cold_capacity / S))
    ok = false;
  // replicated summaries: every global page the rows reach needs a summary row
  const bool repl = repl_summaries(st);
  if (repl && n_ev > 0 && last_page >= summary_pages(st)) ok = false;
  // the running sum of a page that spans calls: read from one slot, written to
  // the other (a call may read the first page's sum and write the last page's)
  const int64_t ps_in = repl ? st_ld(st.state, ST_PAGESUM_SLOT) & 1 : 0;
  // with a host tier one call may reach at most `ring` local pages (each ring
  // slot is spilled once, before this call overwrites it)
  if (tiered && pages_per_bh > ring) ok = false;
  // the grid covers ceil(n_evict_max / S) + 1 pages per (b, h)
  if (n_ev > n_evict_max) ok = false;

  const int nbh = st.batch * H;
  const int blk = blockIdx.x;
  if (ok && blk < nbh * pages_per_bh) {
    // ---------------- eviction role: one (b, h, page) per block -------------
    const int bh = blk / pages_per_bh;
    const int64_t p = cold_len / S + (blk % pages_per_bh);
    const int b = bh / H, h = bh % H;
    const int64_t lo = cold_len > p * S ? cold_len : p * S;
    const int64_t hi_all = cold_len + n_ev;
    const int64_t hi = hi_all < (p + 1) * S ? hi_all : (p + 1) * S;
    const bool owned = (p % st.shard_count) == st.shard_rank;
    if (repl && lo < hi) {
      // every shard: summary of a page completed here, or the running sum of
      // the page left incomplete -- fp32 adds of the page's rows in token
      // order from 0 (the sum carried in from earlier calls first), the same
      // operations as the summary over the cold slots below
      const int64_t nsl = (int64_t)st.batch * H * D;
      const float *sum_in = st.page_sums + ps_in * nsl + (int64_t)bh * D;
      float *sum_out = st.page_sums + (1 - ps_in) * nsl + (int64_t)bh * D;
      for (int c = threadIdx.x; c < D; c += EV_THREADS) {
        float acc = lo > p * S ? sum_in[c] : 0.f;
        for (int64_t g = lo; g < hi; ++g) {
          const int64_t j = g - cold_len;
          const T *src;
          if (!direct && j < hot_len) {
            src = reinterpret_cast<const T *>(st.hot_k) + ((int64_t)bh * hcap + (hot_start + j) % hcap) * D;
          } else {
            src = k_new + b * sb + h * sh + (direct ? j : j - hot_len) * stt;
          }
          acc += Elem<T>::to_f(src[c]);
        }
        if (hi == (p + 1) * S)
          reinterpret_cast<T *>(st.summaries)[((int64_t)bh * summary_pages(st) + p) * D + c] =
              Elem<T>::from_f(acc / (float)S);
        else
          sum_out[c] = acc;
      }
    }
    if (lo < hi && owned) {
      const int64_t lp = p / st.shard_count;
      const int64_t slot = tiered ? lp % ring : lp;
      T *ck = reinterpret_cast<T *>(st.cold_k) + ((int64_t)bh * st.cold_capacity + slot * S) * D;
      T *cv = reinterpret_cast<T *>(st.cold_v) + ((int64_t)bh * st.cold_capacity + slot * S) * D;
      if (tiered && lo == p * S && lp >= ring) {
        // this call starts page lp in ring slot lp % ring: its previous page
        // lp - ring moves to the host tier first
        T *hk = reinterpret_cast<T *>(st.host_k) + ((int64_t)bh * st.host_capacity + (lp - ring) * S) * D;
        T *hv = reinterpret_cast<T *>(st.host_v) + ((int64_t)bh * st.host_capacity + (lp - ring) * S) * D;
        for (int e = threadIdx.x; e < S * nv; e += EV_THREADS) {
          st16(hk + (int64_t)e * V, ld16(ck + (int64_t)e * V));
          st16(hv + (int64_t)e * V, ld16(cv + (int64_t)e * V));
        }
        __syncthreads();
      }
      const int rows = (int)(hi - lo);
      for (int e = threadIdx.x; e < rows * nv; e += EV_THREADS) {
        const int r = e / nv, vi = e % nv;
        const int64_t g = lo + r;
        const int64_t j = g - cold_len;  // logical row of (hot ++ new), or of new when direct
        const T *sk, *sv;
        if (!direct && j < hot_len) {
          const int64_t slot = (hot_start + j) % hcap;
          sk = reinterpret_cast<const T *>(st.hot_k) + ((int64_t)bh * hcap + slot) * D;
          sv = reinterpret_cast<const T *>(st.hot_v) + ((int64_t)bh * hcap + slot) * D;
        } else {
          const int64_t jn = direct ? j : j - hot_len;
          sk = k_new + b * sb + h * sh + jn * stt;
          sv = v_new + b * sb + h * sh + jn * stt;
        }
        const int64_t off = (g - p * S) * D + (int64_t)vi * V;
        st16(ck + off, ld16(sk + vi * V));
        st16(cv + off, ld16(sv + vi * V));
      }
      if (hi == (p + 1) * S && !repl) {
        // the page is complete: summary = (sum of its rows in token order) / S
        __syncthreads();
        T *sm = reinterpret_cast<T *>(st.summaries) + ((int64_t)bh * summary_pages(st) + lp) * D;
        for (int c = threadIdx.x; c < D; c += EV_THREADS) {
          float acc = 0.f;
          const T *col = ck + c;
#pragma unroll 8
          for (int t = 0; t < S; ++t) acc += Elem<T>::to_f(col[(int64_t)t * D]);
          sm[c] = Elem<T>::from_f(acc / (float)S);
        }
      }
    }
  } else if (ok && !direct && blk < nbh * (pages_per_bh + app_per_bh)) {
    // ---------------- append role: new rows that stay hot --------------------
    const int ab = blk - nbh * pages_per_bh;
    const int bh = ab / app_per_bh;
    const int b = bh / H, h = bh % H;
    const int64_t j0 = (int64_t)(ab % app_per_bh) * APPEND_ROWS;
    const int64_t first_kept = n_ev > hot_len ? n_ev - hot_len : 0;  // new rows before this were evicted
    for (int e = threadIdx.x; e < APPEND_ROWS * nv; e += EV_THREADS) {
      const int64_t jn = j0 + e / nv;
      const int vi = e % nv;
      if (jn >= n_new || jn < first_kept) continue;
      const int64_t slot = (hot_start + hot_len + jn) % hcap;
      T *dk = reinterpret_cast<T *>(st.hot_k) + ((int64_t)bh * hcap + slot) * D;
      T *dv = reinterpret_cast<T *>(st.hot_v) + ((int64_t)bh * hcap + slot) * D;
      st16(dk + vi * V, ld16(k_new + b * sb + h * sh + jn * stt + vi * V));
      st16(dv + vi * V, ld16(v_new + b * sb + h * sh + jn * stt + vi * V));
    }
  }

  // ---------------- the last block publishes the new state -------------------
  if (last_block(reinterpret_cast<unsigned long long *>(st.state + CTR_EVICT), gridDim.x)) {
    if (threadIdx.x == 0) {
      if (ok) {
        st.state[KIV_ST_COLD_LEN] = cold_len + n_ev;
        if (repl && n_ev > 0) st.state[ST_PAGESUM_SLOT] = 1 - ps_in;
        if (!direct) {
          st.state[KIV_ST_HOT_START] = hcap > 0 ? (hot_start + n_ev) % hcap : 0;
          st.state[KIV_ST_HOT_LEN] = hot_after;
        }
      } else {
        st.state[KIV_ST_ERROR] |= KIV_ERRBIT_EVICT_CAPACITY;  // nothing was written
      }
    }
  }
}

kiv_status launch_append_evict(const kiv_store *st, const void *k_new, const void *v_new,
                               int64_t sb, int64_t sh, int64_t stt, int32_t n_new, int64_t keep,
                               int64_t n_evict_max, cudaStream_t s) {
  const int nbh = st->batch * st->num_kv_heads;
  const int64_t ppb = n_evict_max > 0 ? ceil_div(n_evict_max, st->page_size) + 1 : 0;
  const int64_t apb = (n_new > 0 && keep != KIV_KEEP_DIRECT) ? ceil_div(n_new, APPEND_ROWS) : 0;
  const int64_t blocks = (int64_t)nbh * (ppb + apb);
  if (blocks == 0) return KIV_OK;
  if (blocks > 0x7fffffff) {
    set_error("append_evict: grid too large (%lld blocks)", (long long)blocks);
    return KIV_ERR_ARG;
  }
  switch (st->dtype) {
    case KIV_DTYPE_F32:
      launch_pdl(append_evict_kernel<float>, dim3((unsigned)blocks), dim3(EV_THREADS), 0, s, 1,
          *st, (const float *)k_new, (const float *)v_new, sb, sh, stt, n_new, keep, n_evict_max, (int)ppb, (int)apb);
      break;
    case KIV_DTYPE_BF16:
      launch_pdl(append_evict_kernel<__nv_bfloat16>, dim3((unsigned)blocks), dim3(EV_THREADS), 0, s, 1,
          *st, (const __nv_bfloat16 *)k_new, (const __nv_bfloat16 *)v_new, sb, sh, stt, n_new, keep,
          n_evict_max, (int)ppb, (int)apb);
      break;
    case KIV_DTYPE_F16:
      launch_pdl(append_evict_kernel<__half>, dim3((unsigned)blocks), dim3(EV_THREADS), 0, s, 1,
          *st, (const __half *)k_new, (const __half *)v_new, sb, sh, stt, n_new, keep, n_evict_max,
          (int)ppb, (int)apb);
      break;
    default:
      return KIV_ERR_UNSUPPORTED;
  }
  return cuda_status(cudaGetLastError(), "append_evict");
}

}  // namespace kiv
