// Host-side internals shared by the KIV translation units.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>
#include <stdlib.h>

#include <algorithm>
#include <utility>

#include "../../include/kiv_b200.h"

namespace kiv {

// kernel-private counters inside the device state block
enum : int {
  CTR_EVICT = 16,
  CTR_COARSE = 17,
  CTR_MERGE = 18,
  CTR_FINE = 19,
  CTR_SEL = 20,
  ST_PAGESUM_SLOT = 21,   // replicated summaries: which page_sums slot holds the carried sum
};

constexpr int ATT_TILE = 32;     // keys per attention tile
constexpr int ROW_CHUNK = 8;     // query rows per register chunk
constexpr int SEL_CLUSTER = 8;   // CTAs per cluster in the fine top-P select

// Scratch carved out of the caller's workspace for one store / query shape.
struct Workspace {
  float *scores;       // [R, np_cap]        coarse scores
  uint32_t *pbits;     // [np_cap / 32]      page marks of the union (one bit per local page; per
                       //                    global page with replicated summaries)
  int32_t *uni;        // [u_cap]            union pages (global ids, ascending)
  uint32_t *agg;       // [B, c_cap]         fine keys (monotone u32 of the max score)
  int32_t *selcnt;     // [B]                selected tokens of this shard per batch row
  uint32_t *fhist;     // [B, 2048]          histogram of fine keys >> 21 (select pass 0), self-clearing
  uint64_t *fstat;     // [B, 2]             largest fine key, sum of fine scores (double bits)
  uint32_t *chist;     // [R, 2048]          histogram of coarse keys >> 21 per query row, self-clearing
  uint64_t *cstat;     // [2]                largest coarse key, sum of coarse scores (double bits)
  float *part;         // [R, split_cap, D+2] attention split partials
  int32_t *pslot;      // [np_cap]            HBM page slot of each local page this step (host tier only)
  int64_t R, K, np_cap, u_cap, c_cap, split_cap;
  size_t bytes;
};

Workspace workspace_layout(const kiv_store *st, const kiv_query *q, void *base);

// ---- host overflow tier geometry (host_capacity > 0)
// ring pages of the HBM cold slots (the newest local pages), staging pages after them
__host__ __device__ inline int64_t ring_pages(const kiv_store &st) {
  return st.cold_capacity / st.page_size - (st.host_capacity > 0 ? st.stage_pages : 0);
}
// every shard keeps the summaries of all global pages (and scores them all)
__host__ __device__ inline bool repl_summaries(const kiv_store &st) {
  return st.shard_count > 1 && (st.flags & KIV_STORE_REPL_SUMMARIES) != 0;
}
// pages the summaries (and the page slot table) cover: local pages, or every
// global page the shards' slots can hold when summaries are replicated (the
// shards of one store hold local page counts that differ by at most one)
__host__ __device__ inline int64_t summary_pages(const kiv_store &st) {
  if (repl_summaries(st)) return (st.cold_capacity / st.page_size + 1) * st.shard_count;
  return st.host_capacity > 0 ? ring_pages(st) + st.host_capacity / st.page_size : st.cold_capacity / st.page_size;
}
// pages of this shard among the first np_global global pages (p % count == rank)
__host__ __device__ inline int64_t shard_local_pages(int64_t np_global, int rank, int count) {
  return np_global > rank ? (np_global - rank + count - 1) / count : 0;
}
// pages the coarse pass scores: all of them with replicated summaries, else this shard's
__host__ __device__ inline int64_t coarse_pages(const kiv_store &st, int64_t np_global) {
  return repl_summaries(st) ? np_global : shard_local_pages(np_global, st.shard_rank, st.shard_count);
}
// global page id of the i-th scored page
__host__ __device__ inline int64_t coarse_page_id(const kiv_store &st, int64_t i) {
  return repl_summaries(st) ? i : i * st.shard_count + st.shard_rank;
}
// HBM page slot to read local page lp from in this step: identity without a host
// tier; otherwise the slot the staging kernel recorded (ring slot, or a staging
// page for a host-resident page of the union)
__device__ __forceinline__ int64_t page_slot(const kiv_store &st, const Workspace &w, int64_t lp) {
  return st.host_capacity > 0 ? (int64_t)w.pslot[lp] : lp;
}
kiv_status launch_stage_union(const kiv_store *st, const Workspace &w, cudaStream_t s);
kiv_status launch_stage_selected(const kiv_store *st, const Workspace &w, const int32_t *sel, int32_t sel_stride,
                                 cudaStream_t s);

int sm_count();
void set_error(const char *fmt, ...);
kiv_status cuda_status(cudaError_t e, const char *where);

// launchers (one per kernel family); all stream-ordered, no host sync
kiv_status launch_append_evict(const kiv_store *st, const void *k_new, const void *v_new,
                               int64_t sb, int64_t sh, int64_t stt, int32_t n_new, int64_t keep,
                               int64_t n_evict_max, cudaStream_t s);
kiv_status launch_coarse(const kiv_store *st, const kiv_query *q, const Workspace &w,
                         float *row_scores, int32_t *row_pages, cudaStream_t s);
struct XArgs;   // peer exchange arguments (exchange.cuh)
kiv_status launch_coarse_merge(const kiv_store *st, const kiv_query *q, const Workspace &w,
                               const float *ls, const int32_t *lp, int32_t n, cudaStream_t s,
                               const XArgs *x = nullptr);
kiv_status launch_fine(const kiv_store *st, const kiv_query *q, const Workspace &w, int32_t *sel,
                       float *sel_scores, cudaStream_t s);
kiv_status launch_fine_score(const kiv_store *st, const kiv_query *q, const Workspace &w, cudaStream_t s);
kiv_status launch_union(const kiv_store *st, const Workspace &w, cudaStream_t s);
bool fine_tc_eligible(const kiv_store *st, const kiv_query *q);
kiv_status launch_fine_score_tc(const kiv_store *st, const kiv_query *q, const Workspace &w, cudaStream_t s);
bool prefill_shape(const kiv_store *st, const kiv_query *q);        // prefill-shaped scoring applies
bool prefill_tc_eligible(const kiv_store *st, const kiv_query *q);  // ... and the query suits TMA
kiv_status launch_prefill_coarse_scores(const kiv_store *st, const kiv_query *q, const Workspace &w, cudaStream_t s);
kiv_status launch_prefill_fine_scores(const kiv_store *st, const kiv_query *q, const Workspace &w, cudaStream_t s);
kiv_status launch_coarse_score_tc(const kiv_store *st, const kiv_query *q, const Workspace &w, cudaStream_t s);
// candidate exchange (page-sharded, replicated summaries): the scorer stores
// every key into every shard's arena, the select takes the global top-P
kiv_status launch_fine_score_tc_exchange(const kiv_store *st, const kiv_query *q, const Workspace &w,
                                         cudaStream_t s, const XArgs &x);
bool fine_exchange_eligible(const kiv_store *st, const kiv_query *q);
kiv_status launch_attend_peers(const kiv_store *st, const kiv_query *q, const kiv_mask *m, const Workspace &w,
                               const int32_t *sel, int32_t sel_stride, const kiv_peer_rows *peers, void *out,
                               cudaStream_t s);
kiv_status launch_fine_exchange_select(const kiv_store *st, const kiv_query *q, const Workspace &w, int32_t *sel,
                                       int32_t *sel_local, cudaStream_t s, const XArgs &x);
kiv_status launch_fine_topk(const kiv_store *st, const kiv_query *q, const Workspace &w, int32_t *sel,
                            float *sel_scores, cudaStream_t s);
kiv_status launch_fine_merge(const kiv_store *st, const kiv_query *q, const Workspace &w,
                             const float *ls, const int32_t *lt, int32_t n, int32_t *sel,
                             int32_t *sel_local, cudaStream_t s, const XArgs *x = nullptr);
kiv_status launch_gather(const kiv_store *st, const int32_t *sel, int32_t sel_stride, int32_t P,
                         void *ok, void *ov, cudaStream_t s);
kiv_status launch_attend(const kiv_store *st, const kiv_query *q, const kiv_mask *m,
                         const Workspace &w, const int32_t *sel, int32_t sel_stride,
                         int32_t hot_slice, int32_t hot_slices, void *out, float *partial_out,
                         cudaStream_t s);
kiv_status launch_attend_merge(const kiv_store *st, const kiv_query *q, const float *partials,
                               int32_t n, void *out, cudaStream_t s, const XArgs *x = nullptr);
// per-rank payload bytes of the three exchanges (coarse lists, fine lists, attention partial)
void exchange_payloads(const kiv_store *st, const kiv_query *q, int64_t *cb, int64_t *fb, int64_t *ab,
                       int64_t *xb);

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Programmatic dependent launch: a kernel may start (and run its prologue)
// while the previous kernel in the stream finishes; every kernel calls
// griddepcontrol.wait before reading the previous kernel's results and
// releases its dependents right after that wait.  KIV_DISABLE_PDL=1 turns it off.
inline bool pdl_enabled() {
  static const bool on = getenv("KIV_DISABLE_PDL") == nullptr;
  return on;
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              int cluster_x, Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  int n = 0;
  attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[n].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  ++n;
  if (cluster_x > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster_x;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

#define KIV_CHECK(x)                 \
  do {                               \
    const kiv_status _st = (x);      \
    if (_st != KIV_OK) return _st;   \
  } while (0)

// floats per attention partial row: out[D], max, sum, 16-byte aligned
__host__ __device__ inline int partial_stride(int D) { return (D + 2 + 3) & ~3; }

#ifdef __CUDACC__
// A coarse pass whose page marks were never consumed by a fine pass left them
// set: clear them (grid-stride) before this coarse pass marks its own.
__device__ __forceinline__ void clear_stale_marks(const kiv_store &st, const Workspace &w, int64_t np_local) {
  if (*reinterpret_cast<volatile const int64_t *>(st.state + KIV_ST_UNION_PENDING) == 0) return;
  const int64_t nw = (np_local + 31) / 32;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nw; i += (int64_t)gridDim.x * blockDim.x)
    w.pbits[i] = 0;
}
#endif
inline int64_t align_up(int64_t a, int64_t b) { return ceil_div(a, b) * b; }

inline int elem_bytes(int dtype) { return dtype == KIV_DTYPE_F32 ? 4 : 2; }

// number of attention splits per (b, kvh, row chunk) for this shape
// attention splits per query row: at most one tile of keys per split, and no
// more than the SMs spread over the CTAs of one split (prefill-shaped queries
// use no splits at all, but the bound keeps their workspace small too)
inline int64_t attn_split_cap(const kiv_store *st, const kiv_query *q) {
  const int64_t keys = (int64_t)q->top_p + st->hot_capacity;
  const int64_t rows_kv = (int64_t)(q->num_query_heads / st->num_kv_heads) * q->query_len;
  const int64_t base = (int64_t)st->batch * st->num_kv_heads * ceil_div(rows_kv, 16);
  return std::min<int64_t>(ceil_div(keys > 0 ? keys : 1, ATT_TILE), ceil_div(sm_count(), std::max<int64_t>(1, base)));
}

}  // namespace kiv
