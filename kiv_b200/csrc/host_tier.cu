// Host overflow tier: batched gathers of host-resident cold rows into the HBM
// staging pages, ahead of the kernels that read them.
//
// With a host tier the HBM cold slots hold the newest R local pages as a ring
// (local page lp at ring page lp % R; the eviction kernel moves a ring page to
// the host tier just before its slot is reused) and the pages older than that
// live in pinned, device-mapped host memory.  A local page is host-resident
// iff lp < n_started - R, n_started = local pages holding any row.
//
// stage_union_kernel (after the union is built, before fine scoring): the
// union is sorted, so its host-resident pages are a prefix of it; union entry
// u < stage_pages of a host page is copied (K rows of every (b, h)) into
// staging page R + u, and every union page records the HBM page it is read
// from in w.pslot (the partial page too).  stage_selected_kernel (after the
// token select, before the attention): the V rows of the selected tokens on
// host pages go to the same staging pages.  Both read host memory with 16-byte
// vector loads over the host link and write HBM; nothing else reads the host
// tier.
#include "common.cuh"
#include "internal.h"

namespace kiv {

constexpr int SG_THREADS = 256;
constexpr int SG_UNROLL = 4;     // 16-byte loads in flight per thread

// local pages of this shard that hold at least one cold row
__device__ __forceinline__ int64_t started_local_pages(const kiv_store &st) {
  const int64_t cold = st_ld(st.state, KIV_ST_COLD_LEN);
  const int64_t ng = (cold + st.page_size - 1) / st.page_size;
  return ng > st.shard_rank ? (ng - st.shard_rank + st.shard_count - 1) / st.shard_count : 0;
}

__global__ void __launch_bounds__(SG_THREADS) stage_union_kernel(kiv_store st, Workspace w) {
  griddep_wait();
  const int S = st.page_size, D = st.head_dim;
  const int eb = st.dtype == KIV_DTYPE_F32 ? 4 : 2;
  const int64_t R = ring_pages(st);
  const int64_t thr = started_local_pages(st) - R;     // local pages below this are on the host
  const int64_t U = st_ld(st.state, KIV_ST_UNION);
  const int64_t BH = (int64_t)st.batch * st.num_kv_heads;
  const int64_t chunks = (int64_t)S * D * eb / 16;    // 16-byte chunks of one page strip
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    // the partial (newest) page is always in the ring
    const int64_t n_started = started_local_pages(st);
    if (n_started > 0) w.pslot[n_started - 1] = (int32_t)((n_started - 1) % R);
  }
  for (int64_t it = blockIdx.x; it < U * BH; it += gridDim.x) {
    const int64_t u = it / BH, bh = it % BH;
    const int64_t lp = (int64_t)w.uni[u] / st.shard_count;
    if (lp >= thr) {
      if (bh == 0 && threadIdx.x == 0) w.pslot[lp] = (int32_t)(lp % R);
      continue;
    }
    if (u >= st.stage_pages) {
      if (bh == 0 && threadIdx.x == 0)
        atomicOr(reinterpret_cast<unsigned long long *>(st.state + KIV_ST_ERROR),
                 (unsigned long long)KIV_ERRBIT_STAGE_CAPACITY);
      continue;
    }
    if (bh == 0 && threadIdx.x == 0) w.pslot[lp] = (int32_t)(R + u);
    const uint4 *src = reinterpret_cast<const uint4 *>(static_cast<const char *>(st.host_k) +
                                                        ((bh * st.host_capacity + lp * S) * D) * eb);
    uint4 *dst = reinterpret_cast<uint4 *>(static_cast<char *>(st.cold_k) +
                                           ((bh * st.cold_capacity + (R + u) * S) * D) * eb);
    for (int64_t c0 = threadIdx.x; c0 < chunks; c0 += (int64_t)SG_THREADS * SG_UNROLL) {
      uint4 v[SG_UNROLL];
#pragma unroll
      for (int x = 0; x < SG_UNROLL; ++x) {
        const int64_t c = c0 + (int64_t)x * SG_THREADS;
        if (c < chunks) v[x] = src[c];
      }
#pragma unroll
      for (int x = 0; x < SG_UNROLL; ++x) {
        const int64_t c = c0 + (int64_t)x * SG_THREADS;
        if (c < chunks) dst[c] = v[x];
      }
    }
  }
}

// V rows of the selected tokens that live on host pages -> their staging pages
__global__ void __launch_bounds__(SG_THREADS)
stage_selected_kernel(kiv_store st, Workspace w, const int32_t *sel, int32_t sel_stride) {
  griddep_wait();
  const int S = st.page_size, D = st.head_dim;
  const int eb = st.dtype == KIV_DTYPE_F32 ? 4 : 2;
  const int64_t R = ring_pages(st);
  const int64_t thr = started_local_pages(st) - R;
  const int H = st.num_kv_heads;
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * SG_THREADS + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * SG_THREADS) >> 5;
  const int rc = D * eb / 16;                 // 16-byte chunks of a row
  const int64_t items = (int64_t)st.batch * sel_stride * H;
  for (int64_t it = warp; it < items; it += nwarps) {
    const int h = (int)(it % H);
    const int64_t bi = it / H;
    const int b = (int)(bi / sel_stride), i = (int)(bi % sel_stride);
    if (i >= w.selcnt[b]) continue;
    const int64_t tok = sel[(int64_t)b * sel_stride + i];
    const int64_t lp = (tok / S) / st.shard_count;
    if (lp >= thr) continue;
    const int64_t bh = (int64_t)b * H + h;
    const uint4 *src = reinterpret_cast<const uint4 *>(static_cast<const char *>(st.host_v) +
                                                        ((bh * st.host_capacity + lp * S + tok % S) * D) * eb);
    uint4 *dst = reinterpret_cast<uint4 *>(static_cast<char *>(st.cold_v) +
                                           ((bh * st.cold_capacity + (int64_t)w.pslot[lp] * S + tok % S) * D) * eb);
    for (int c = lane; c < rc; c += 32) dst[c] = src[c];
  }
}

kiv_status launch_stage_union(const kiv_store *st, const Workspace &w, cudaStream_t s) {
  if (st->host_capacity <= 0) return KIV_OK;
  const int64_t BH = (int64_t)st->batch * st->num_kv_heads;
  const int64_t grid = std::max<int64_t>(1, std::min<int64_t>(w.u_cap * BH, (int64_t)sm_count() * 8));
  return cuda_status(launch_pdl(stage_union_kernel, dim3((unsigned)grid), dim3(SG_THREADS), 0, s, 1, *st, w),
                     "stage_union");
}

kiv_status launch_stage_selected(const kiv_store *st, const Workspace &w, const int32_t *sel, int32_t sel_stride,
                                 cudaStream_t s) {
  if (st->host_capacity <= 0 || sel_stride <= 0) return KIV_OK;
  const int64_t items = (int64_t)st->batch * sel_stride * st->num_kv_heads;
  const int64_t grid = std::max<int64_t>(1, std::min<int64_t>(ceil_div(items, SG_THREADS / 32), (int64_t)sm_count() * 4));
  return cuda_status(launch_pdl(stage_selected_kernel, dim3((unsigned)grid), dim3(SG_THREADS), 0, s, 1, *st, w, sel,
                                sel_stride),
                     "stage_selected");
}

}  // namespace kiv
