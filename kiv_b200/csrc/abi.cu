// C ABI of libkiv_b200.so: argument validation, workspace layout, dispatch.
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>

#include <cuda.h>

#include "exchange.cuh"
#include "internal.h"

namespace kiv {

static thread_local char g_err[512] = {0};

void set_error(const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

kiv_status cuda_status(cudaError_t e, const char *where) {
  if (e == cudaSuccess) return KIV_OK;
  set_error("%s: %s", where, cudaGetErrorString(e));
  return KIV_ERR_CUDA;
}

int sm_count() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

static int64_t a256(int64_t x) { return align_up(x, 256); }

Workspace workspace_layout(const kiv_store *st, const kiv_query *q, void *base) {
  Workspace w = {};
  w.R = (int64_t)st->batch * q->num_query_heads * q->query_len;
  w.K = q->top_pages;
  w.np_cap = summary_pages(*st);
  w.u_cap = std::min<int64_t>(w.np_cap, w.R * w.K);
  w.c_cap = w.u_cap * st->page_size + st->page_size;
  w.split_cap = attn_split_cap(st, q);
  char *p = reinterpret_cast<char *>(base);
  int64_t off = 0;
  auto take = [&](int64_t bytes) {
    char *r = p ? p + off : nullptr;
    off += a256(bytes);
    return r;
  };
  w.scores = reinterpret_cast<float *>(take(w.R * w.np_cap * 4));
  w.pbits = reinterpret_cast<uint32_t *>(take(ceil_div(w.np_cap, 32) * 4));
  w.uni = reinterpret_cast<int32_t *>(take(w.u_cap * 4));
  w.agg = reinterpret_cast<uint32_t *>(take((int64_t)st->batch * w.c_cap * 4));
  w.selcnt = reinterpret_cast<int32_t *>(take((int64_t)st->batch * 4));
  w.fhist = reinterpret_cast<uint32_t *>(take((int64_t)st->batch * 2048 * 4));
  w.fstat = reinterpret_cast<uint64_t *>(take((int64_t)st->batch * 16));
  w.chist = reinterpret_cast<uint32_t *>(take(prefill_shape(st, q) ? 0 : w.R * 2048 * 4));
  w.cstat = reinterpret_cast<uint64_t *>(take(16));
  w.part = reinterpret_cast<float *>(take(w.R * w.split_cap * partial_stride(st->head_dim) * 4));
  w.pslot = reinterpret_cast<int32_t *>(take(st->host_capacity > 0 ? w.np_cap * 4 : 0));
  w.bytes = (size_t)off;
  return w;
}

static bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

static kiv_status check_store(const kiv_store *st) {
  if (!st) { set_error("store is NULL"); return KIV_ERR_ARG; }
  if (st->dtype < 0 || st->dtype > 2) { set_error("unknown dtype %d", st->dtype); return KIV_ERR_UNSUPPORTED; }
  const int eb = elem_bytes(st->dtype);
  if (st->batch < 1 || st->num_kv_heads < 1 || st->head_dim < 1 || st->page_size < 1) {
    set_error("bad store shape B=%d Hkv=%d D=%d S=%d", st->batch, st->num_kv_heads, st->head_dim,
              st->page_size);
    return KIV_ERR_ARG;
  }
  if ((st->head_dim * eb) % 16 != 0) {
    set_error("head_dim * element size must be a multiple of 16 bytes (D=%d)", st->head_dim);
    return KIV_ERR_UNSUPPORTED;
  }
  if (st->head_dim * eb > 1024) { set_error("head_dim %d too large", st->head_dim); return KIV_ERR_UNSUPPORTED; }
  if (st->page_size > 1024) { set_error("page_size %d > 1024", st->page_size); return KIV_ERR_UNSUPPORTED; }
  if (st->shard_count < 1 || st->shard_rank < 0 || st->shard_rank >= st->shard_count) {
    set_error("bad shard %d/%d", st->shard_rank, st->shard_count);
    return KIV_ERR_ARG;
  }
  if (st->cold_capacity < 0 || st->cold_capacity % st->page_size != 0) {
    set_error("cold_capacity %lld not a multiple of page_size", (long long)st->cold_capacity);
    return KIV_ERR_ARG;
  }
  if (!st->state) { set_error("state is NULL"); return KIV_ERR_ARG; }
  if (st->cold_capacity > 0 &&
      (!st->cold_k || !st->cold_v || !st->summaries || !aligned16(st->cold_k) || !aligned16(st->cold_v) ||
       !aligned16(st->summaries))) {
    set_error("cold buffers missing or not 16-byte aligned");
    return KIV_ERR_ARG;
  }
  if (st->hot_capacity > 0 && (!st->hot_k || !st->hot_v || !aligned16(st->hot_k) || !aligned16(st->hot_v))) {
    set_error("hot ring missing or not 16-byte aligned");
    return KIV_ERR_ARG;
  }
  if (st->host_capacity < 0 || st->host_capacity % st->page_size != 0) {
    set_error("host_capacity %lld not a multiple of page_size", (long long)st->host_capacity);
    return KIV_ERR_ARG;
  }
  if (st->flags & ~KIV_STORE_REPL_SUMMARIES) { set_error("unknown store flags 0x%x", st->flags); return KIV_ERR_ARG; }
  if (repl_summaries(*st)) {
    if (st->host_capacity > 0) {
      set_error("replicated summaries are not combined with a host tier");
      return KIV_ERR_UNSUPPORTED;
    }
    if (!st->page_sums || !aligned16(st->page_sums)) {
      set_error("replicated summaries need page_sums (fp32 [B, Hkv, D], 16-byte aligned)");
      return KIV_ERR_ARG;
    }
  }
  if (st->host_capacity > 0) {
    if (!st->host_k || !st->host_v || !aligned16(st->host_k) || !aligned16(st->host_v)) {
      set_error("host tier missing or not 16-byte aligned");
      return KIV_ERR_ARG;
    }
    if (st->stage_pages < 1 || ring_pages(*st) < 2) {
      set_error("host tier needs stage_pages >= 1 and at least 2 ring pages (cold_capacity %lld, stage %d)",
                (long long)st->cold_capacity, st->stage_pages);
      return KIV_ERR_ARG;
    }
  }
  return KIV_OK;
}

static kiv_status check_query(const kiv_store *st, const kiv_query *q) {
  if (!q || !q->q) { set_error("query is NULL"); return KIV_ERR_ARG; }
  const int eb = elem_bytes(st->dtype);
  if (q->num_query_heads < 1 || q->num_query_heads % st->num_kv_heads != 0 || q->query_len < 1) {
    set_error("bad query heads %d (kv heads %d) / length %d", q->num_query_heads, st->num_kv_heads,
              q->query_len);
    return KIV_ERR_ARG;
  }
  if (q->top_pages < 1 || q->top_p < 1) { set_error("top_pages/top_p must be >= 1"); return KIV_ERR_ARG; }
  if (!aligned16(q->q) || (q->stride_b * eb) % 16 || (q->stride_h * eb) % 16 || (q->stride_t * eb) % 16) {
    set_error("query rows must be 16-byte aligned");
    return KIV_ERR_ARG;
  }
  return KIV_OK;
}

static kiv_status check_ws(const kiv_store *st, const kiv_query *q, void *ws, size_t bytes, Workspace &w) {
  w = workspace_layout(st, q, ws);
  if (!ws || bytes < w.bytes || (reinterpret_cast<uintptr_t>(ws) & 255)) {
    set_error("workspace too small or misaligned (%zu < %zu)", bytes, w.bytes);
    return KIV_ERR_CAPACITY;
  }
  return KIV_OK;
}

}  // namespace kiv

using namespace kiv;

#define KIV_TRY(x)                      \
  do {                                  \
    kiv_status _rc = (x);               \
    if (_rc != KIV_OK) return _rc;      \
  } while (0)

extern "C" {

int32_t kiv_abi_version(void) { return 1; }

const char *kiv_status_string(kiv_status s) {
  switch (s) {
    case KIV_OK: return "ok";
    case KIV_ERR_ARG: return "invalid argument";
    case KIV_ERR_CAPACITY: return "capacity exceeded";
    case KIV_ERR_CUDA: return "CUDA error";
    case KIV_ERR_UNSUPPORTED: return "unsupported";
  }
  return "unknown status";
}

const char *kiv_last_error(void) { return g_err; }

size_t kiv_workspace_bytes(const kiv_store *st, const kiv_query *q) {
  if (check_store(st) != KIV_OK || !q) return 0;
  return workspace_layout(st, q, nullptr).bytes;
}

kiv_status kiv_workspace_layout(const kiv_store *st, const kiv_query *q, int64_t *out) {
  KIV_TRY(check_store(st));
  if (!q || !out) { set_error("bad layout arguments"); return KIV_ERR_ARG; }
  // offsets relative to a null base
  const Workspace w = workspace_layout(st, q, reinterpret_cast<void *>(0x100));
  const auto off = [](const void *p) { return (int64_t)(reinterpret_cast<uintptr_t>(p) - 0x100); };
  out[0] = off(w.scores);
  out[1] = off(w.pbits);
  out[2] = off(w.uni);
  out[3] = off(w.agg);
  out[4] = off(w.selcnt);
  out[5] = off(w.part);
  out[6] = w.R;
  out[7] = w.np_cap;
  out[8] = w.u_cap;
  out[9] = w.c_cap;
  return KIV_OK;
}

kiv_status kiv_state_reset(const kiv_store *st, void *stream) {
  if (!st || !st->state) { set_error("state is NULL"); return KIV_ERR_ARG; }
  return cuda_status(cudaMemsetAsync(st->state, 0, KIV_STATE_WORDS * sizeof(int64_t),
                                     (cudaStream_t)stream), "state_reset");
}

kiv_status kiv_append_evict(const kiv_store *st, const void *k_new, const void *v_new, int64_t stride_b,
                            int64_t stride_h, int64_t stride_t, int32_t n_new, int64_t keep,
                            int64_t n_evict_max, void *stream) {
  KIV_TRY(check_store(st));
  if (n_new < 0 || n_evict_max < 0) { set_error("negative row count"); return KIV_ERR_ARG; }
  if (n_new > 0) {
    const int eb = elem_bytes(st->dtype);
    if (!k_new || !v_new || !aligned16(k_new) || !aligned16(v_new) || (stride_b * eb) % 16 ||
        (stride_h * eb) % 16 || (stride_t * eb) % 16) {
      set_error("new rows missing or not 16-byte aligned");
      return KIV_ERR_ARG;
    }
  }
  return launch_append_evict(st, k_new, v_new, stride_b, stride_h, stride_t, n_new, keep, n_evict_max,
                             (cudaStream_t)stream);
}

kiv_status kiv_coarse_select(const kiv_store *st, const kiv_query *q, void *ws, size_t ws_bytes,
                             float *row_scores, int32_t *row_pages, void *stream) {
  KIV_TRY(check_store(st));
  KIV_TRY(check_query(st, q));
  Workspace w;
  KIV_TRY(check_ws(st, q, ws, ws_bytes, w));
  if (st->shard_count > 1 && !repl_summaries(*st) && (!row_scores || !row_pages)) {
    set_error("sharded coarse_select needs row_scores/row_pages (or replicated summaries)");
    return KIV_ERR_ARG;
  }
  return launch_coarse(st, q, w, row_scores, row_pages, (cudaStream_t)stream);
}

kiv_status kiv_coarse_merge(const kiv_store *st, const kiv_query *q, void *ws, size_t ws_bytes,
                            const float *lists_scores, const int32_t *lists_pages, int32_t n_lists,
                            void *stream) {
  KIV_TRY(check_store(st));
  KIV_TRY(check_query(st, q));
  Workspace w;
  KIV_TRY(check_ws(st, q, ws, ws_bytes, w));
  if (!lists_scores || !lists_pages || n_lists < 1) { set_error("bad merge lists"); return KIV_ERR_ARG; }
  return launch_coarse_merge(st, q, w, lists_scores, lists_pages, n_lists, (cudaStream_t)stream);
}

kiv_status kiv_fine_select(const kiv_store *st, const kiv_query *q, void *ws, size_t ws_bytes,
                           int32_t *sel, float *sel_scores, void *stream) {
  KIV_TRY(check_store(st));
  KIV_TRY(check_query(st, q));
  Workspace w;
  KIV_TRY(check_ws(st, q, ws, ws_bytes, w));
  if (!sel) { set_error("sel is NULL"); return KIV_ERR_ARG; }
  return launch_fine(st, q, w, sel, sel_scores, (cudaStream_t)stream);
}

kiv_status kiv_fine_score(const kiv_store *st, const kiv_query *q, void *ws, size_t ws_bytes, void *stream) {
  KIV_TRY(check_store(st));
  KIV_TRY(check_query(st, q));
  Workspace w;
  KIV_TRY(check_ws(st, q, ws, ws_bytes, w));
  return launch_fine_score(st, q, w, (cudaStream_t)stream);
}

kiv_status kiv_fine_topk(const kiv_store *st, const kiv_query *q, void *ws, size_t ws_bytes, int32_t *sel,
                         float *sel_scores, void *stream) {
  KIV_TRY(check_store(st));
  KIV_TRY(check_query(st, q));
  Workspace w;
  KIV_TRY(check_ws(st, q, ws, ws_bytes, w));
  if (!sel) { set_error("sel is NULL"); return KIV_ERR_ARG; }
  return launch_fine_topk(st, q, w, sel, sel_scores, (cudaStream_t)stream);
}

kiv_status kiv_fine_merge(const kiv_store *st, const kiv_query *q, void *ws, size_t ws_bytes,
                          const float *lists_scores, const int32_t *lists_tokens, int32_t n_lists,
                          int32_t *sel, int32_t *sel_local, void *stream) {
  KIV_TRY(check_store(st));
  KIV_TRY(check_query(st, q));
  Workspace w;
  KIV_TRY(check_ws(st, q, ws, ws_bytes, w));
  if (!lists_scores || !lists_tokens || n_lists < 1 || !sel || !sel_local) {
    set_error("bad fine merge arguments");
    return KIV_ERR_ARG;
  }
  return launch_fine_merge(st, q, w, lists_scores, lists_tokens, n_lists, sel, sel_local,
                           (cudaStream_t)stream);
}

kiv_status kiv_gather_rows(const kiv_store *st, const int32_t *sel, int32_t sel_stride, int32_t P,
                           void *out_k, void *out_v, void *stream) {
  KIV_TRY(check_store(st));
  if (P < 0 || (P > 0 && (!sel || !out_k || !out_v || sel_stride < P))) {
    set_error("bad gather arguments");
    return KIV_ERR_ARG;
  }
  if (P > 0 && (!aligned16(out_k) || !aligned16(out_v))) { set_error("gather outputs not aligned"); return KIV_ERR_ARG; }
  return launch_gather(st, sel, sel_stride, P, out_k, out_v, (cudaStream_t)stream);
}

kiv_status kiv_attend(const kiv_store *st, const kiv_query *q, const kiv_mask *mask, void *ws,
                      size_t ws_bytes, const int32_t *sel, int32_t sel_stride, int32_t hot_slice,
                      int32_t hot_slices, void *out, float *partial_out, void *stream) {
  KIV_TRY(check_store(st));
  KIV_TRY(check_query(st, q));
  Workspace w;
  KIV_TRY(check_ws(st, q, ws, ws_bytes, w));
  if (!sel || sel_stride < 0 || hot_slices < 1 || hot_slice < 0 || hot_slice >= hot_slices) {
    set_error("bad attend arguments");
    return KIV_ERR_ARG;
  }
  if (!out && !partial_out) { set_error("attend needs out or partial_out"); return KIV_ERR_ARG; }
  return launch_attend(st, q, mask, w, sel, sel_stride, hot_slice, hot_slices, out, partial_out,
                       (cudaStream_t)stream);
}

kiv_status kiv_attend_merge(const kiv_store *st, const kiv_query *q, const float *partials, int32_t n,
                            void *out, void *stream) {
  KIV_TRY(check_store(st));
  KIV_TRY(check_query(st, q));
  if (!partials || n < 1 || !out) { set_error("bad attend_merge arguments"); return KIV_ERR_ARG; }
  return launch_attend_merge(st, q, partials, n, out, (cudaStream_t)stream);
}

kiv_status kiv_retrieve_attend(const kiv_store *st, const kiv_query *q, const kiv_mask *mask, void *ws,
                               size_t ws_bytes, int32_t reuse, int32_t *sel, void *out, void *stream) {
  KIV_TRY(check_store(st));
  KIV_TRY(check_query(st, q));
  if (st->shard_count != 1) { set_error("retrieve_attend is the single-shard path"); return KIV_ERR_ARG; }
  Workspace w;
  KIV_TRY(check_ws(st, q, ws, ws_bytes, w));
  if (!sel || !out) { set_error("sel/out NULL"); return KIV_ERR_ARG; }
  cudaStream_t s = (cudaStream_t)stream;
  if (!reuse) KIV_TRY(launch_coarse(st, q, w, nullptr, nullptr, s));
  KIV_TRY(launch_fine(st, q, w, sel, nullptr, s));
  return launch_attend(st, q, mask, w, sel, q->top_p, 0, 1, out, nullptr, s);
}

// ---------------------------------------------------------------- exchange
size_t kiv_exchange_bytes(const kiv_store *st, const kiv_query *q, int32_t world) {
  if (check_store(st) != KIV_OK || check_query(st, q) != KIV_OK || world < 1 || world > KIV_MAX_PEERS) return 0;
  int64_t cb, fb, ab, xb;
  exchange_payloads(st, q, &cb, &fb, &ab, &xb);
  return (size_t)x_layout(cb, fb, ab, xb, world).total;
}

kiv_status kiv_peer_alloc(size_t bytes, void **dev_ptr, void *ipc_handle) {
  if (!dev_ptr || !ipc_handle || bytes == 0) { set_error("bad peer_alloc arguments"); return KIV_ERR_ARG; }
  static_assert(sizeof(cudaIpcMemHandle_t) <= KIV_IPC_HANDLE_BYTES, "IPC handle size");
  void *p = nullptr;
  KIV_TRY(cuda_status(cudaMalloc(&p, bytes), "peer_alloc: cudaMalloc"));
  kiv_status rc = cuda_status(cudaMemset(p, 0, bytes), "peer_alloc: cudaMemset");
  cudaIpcMemHandle_t h;
  if (rc == KIV_OK) rc = cuda_status(cudaIpcGetMemHandle(&h, p), "peer_alloc: cudaIpcGetMemHandle");
  if (rc != KIV_OK) {
    cudaFree(p);
    return rc;
  }
  memset(ipc_handle, 0, KIV_IPC_HANDLE_BYTES);
  memcpy(ipc_handle, &h, sizeof(h));
  *dev_ptr = p;
  return KIV_OK;
}

kiv_status kiv_peer_open(const void *ipc_handle, void **dev_ptr) {
  if (!dev_ptr || !ipc_handle) { set_error("bad peer_open arguments"); return KIV_ERR_ARG; }
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  return cuda_status(cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess), "peer_open");
}

kiv_status kiv_peer_close(void *dev_ptr) { return cuda_status(cudaIpcCloseMemHandle(dev_ptr), "peer_close"); }

kiv_status kiv_peer_export(const void *dev_ptr, void *ipc_handle, int64_t *offset) {
  if (!dev_ptr || !ipc_handle || !offset) { set_error("bad peer_export arguments"); return KIV_ERR_ARG; }
  // the allocation's base (driver entry point: the runtime has no range query)
  using RangeFn = CUresult (*)(CUdeviceptr *, size_t *, CUdeviceptr);
  static RangeFn range = nullptr;
  if (!range) {
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult qr;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &qr) != cudaSuccess ||
        qr != cudaDriverEntryPointSuccess || !fn) {
      set_error("cuMemGetAddressRange unavailable");
      return KIV_ERR_CUDA;
    }
    range = reinterpret_cast<RangeFn>(fn);
  }
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(dev_ptr)) != CUDA_SUCCESS) {
    set_error("peer_export: %p is not device memory", dev_ptr);
    return KIV_ERR_ARG;
  }
  cudaIpcMemHandle_t h;
  KIV_TRY(cuda_status(cudaIpcGetMemHandle(&h, reinterpret_cast<void *>(base)), "peer_export: cudaIpcGetMemHandle"));
  memset(ipc_handle, 0, KIV_IPC_HANDLE_BYTES);
  memcpy(ipc_handle, &h, sizeof(h));
  *offset = (int64_t)(reinterpret_cast<CUdeviceptr>(dev_ptr) - base);
  return KIV_OK;
}

kiv_status kiv_peer_free(void *dev_ptr) { return cuda_status(cudaFree(dev_ptr), "peer_free"); }

kiv_status kiv_host_alloc(size_t bytes, void **ptr) {
  if (!ptr || bytes == 0) { set_error("bad host_alloc arguments"); return KIV_ERR_ARG; }
  *ptr = nullptr;
  // pinned, mapped into every device's address space (UVA: same pointer)
  return cuda_status(cudaHostAlloc(ptr, bytes, cudaHostAllocMapped | cudaHostAllocPortable), "host_alloc");
}

kiv_status kiv_host_free(void *ptr) { return cuda_status(cudaFreeHost(ptr), "host_free"); }

static kiv_status check_exchange(const kiv_store *st, const kiv_query *q, const kiv_exchange *x, int t,
                                 int64_t ctas, kiv::XArgs &a) {
  if (!x || x->world != st->shard_count || x->rank != st->shard_rank || x->world < 1 ||
      x->world > KIV_MAX_PEERS) {
    set_error("exchange descriptor does not match the store's shard (rank/world)");
    return KIV_ERR_ARG;
  }
  int64_t cb, fb, ab, xb;
  exchange_payloads(st, q, &cb, &fb, &ab, &xb);
  const kiv::XLayout L = x_layout(cb, fb, ab, xb, x->world);
  if (x->arena_bytes < L.total) {
    set_error("exchange arena of %lld bytes, this shape needs %lld", (long long)x->arena_bytes,
              (long long)L.total);
    return KIV_ERR_CAPACITY;
  }
  // every CTA of a launch waits for every rank's CTAs: all must be resident
  if (ctas > sm_count()) {
    set_error("exchange merge of %lld CTAs exceeds the %d SMs", (long long)ctas, sm_count());
    return KIV_ERR_UNSUPPORTED;
  }
  a = kiv::XArgs{};
  a.world = x->world;
  a.rank = x->rank;
  for (int i = 0; i < x->world; ++i) {
    if (!x->arena[i] || (reinterpret_cast<uintptr_t>(x->arena[i]) & 255)) {
      set_error("exchange arena %d missing or misaligned", i);
      return KIV_ERR_ARG;
    }
    a.arena[i] = static_cast<char *>(x->arena[i]);
  }
  a.off = L.off[t];
  a.par_bytes = L.par[t];
  if (x->wait_cycles < 0) {
    set_error("negative exchange wait bound");
    return KIV_ERR_ARG;
  }
  a.budget = x->wait_cycles > 0 ? x->wait_cycles : kiv::X_DEFAULT_WAIT_CYCLES;
  return KIV_OK;
}

kiv_status kiv_coarse_exchange_merge(const kiv_store *st, const kiv_query *q, void *ws, size_t ws_bytes,
                                     const float *row_scores, const int32_t *row_pages, const kiv_exchange *x,
                                     void *stream) {
  KIV_TRY(check_store(st));
  KIV_TRY(check_query(st, q));
  Workspace w;
  KIV_TRY(check_ws(st, q, ws, ws_bytes, w));
  if (!row_scores || !row_pages) { set_error("bad merge lists"); return KIV_ERR_ARG; }
  kiv::XArgs a;
  KIV_TRY(check_exchange(st, q, x, kiv::X_COARSE, w.R, a));
  return launch_coarse_merge(st, q, w, row_scores, row_pages, x->world, (cudaStream_t)stream, &a);
}

kiv_status kiv_fine_exchange_merge(const kiv_store *st, const kiv_query *q, void *ws, size_t ws_bytes,
                                   const float *scores, const int32_t *tokens, const kiv_exchange *x,
                                   int32_t *sel, int32_t *sel_local, void *stream) {
  KIV_TRY(check_store(st));
  KIV_TRY(check_query(st, q));
  Workspace w;
  KIV_TRY(check_ws(st, q, ws, ws_bytes, w));
  if (!scores || !tokens || !sel_local) { set_error("bad fine merge arguments"); return KIV_ERR_ARG; }
  kiv::XArgs a;
  KIV_TRY(check_exchange(st, q, x, kiv::X_FINE, st->batch, a));
  return launch_fine_merge(st, q, w, scores, tokens, x->world, sel, sel_local, (cudaStream_t)stream, &a);
}

int32_t kiv_fine_exchange_supported(const kiv_store *st, const kiv_query *q) {
  if (check_store(st) != KIV_OK || check_query(st, q) != KIV_OK) return 0;
  return fine_exchange_eligible(st, q) ? 1 : 0;
}

kiv_status kiv_fine_exchange_select(const kiv_store *st, const kiv_query *q, void *ws, size_t ws_bytes,
                                    const kiv_exchange *x, int32_t *sel, int32_t *sel_local, void *stream) {
  KIV_TRY(check_store(st));
  KIV_TRY(check_query(st, q));
  Workspace w;
  KIV_TRY(check_ws(st, q, ws, ws_bytes, w));
  if (!sel) { set_error("sel is NULL"); return KIV_ERR_ARG; }
  if (!fine_exchange_eligible(st, q)) {
    set_error("candidate exchange needs a page-sharded store with replicated summaries, 16-bit rows, "
              "page_size 128 and a union of at most %d pages", 8192);
    return KIV_ERR_UNSUPPORTED;
  }
  kiv::XArgs a;
  KIV_TRY(check_exchange(st, q, x, kiv::X_CAND, (int64_t)st->batch * SEL_CLUSTER, a));
  cudaStream_t s = (cudaStream_t)stream;
  KIV_TRY(launch_fine_score_tc_exchange(st, q, w, s, a));
  return launch_fine_exchange_select(st, q, w, sel, sel_local, s, a);
}

kiv_status kiv_attend_peers(const kiv_store *st, const kiv_query *q, const kiv_mask *mask, void *ws,
                            size_t ws_bytes, const int32_t *sel, int32_t sel_stride, const kiv_peer_rows *peers,
                            void *out, void *stream) {
  KIV_TRY(check_store(st));
  KIV_TRY(check_query(st, q));
  Workspace w;
  KIV_TRY(check_ws(st, q, ws, ws_bytes, w));
  if (!sel || sel_stride < 0 || !out || !peers) { set_error("bad attend_peers arguments"); return KIV_ERR_ARG; }
  if (st->shard_count < 2 || st->host_capacity > 0) {
    set_error("attend_peers is the page-sharded path without a host tier");
    return KIV_ERR_ARG;
  }
  for (int r = 0; r < st->shard_count; ++r) {
    if (!peers->cold_k[r] || !peers->cold_v[r] || !aligned16(peers->cold_k[r]) || !aligned16(peers->cold_v[r])) {
      set_error("peer rows of shard %d missing or not 16-byte aligned", r);
      return KIV_ERR_ARG;
    }
  }
  if (peers->cold_k[st->shard_rank] != st->cold_k || peers->cold_v[st->shard_rank] != st->cold_v) {
    set_error("peer rows: this shard's entry must be the store's own cold rows");
    return KIV_ERR_ARG;
  }
  return launch_attend_peers(st, q, mask, w, sel, sel_stride, peers, out, (cudaStream_t)stream);
}

kiv_status kiv_attend_exchange_merge(const kiv_store *st, const kiv_query *q, const float *partial,
                                     const kiv_exchange *x, void *out, void *stream) {
  KIV_TRY(check_store(st));
  KIV_TRY(check_query(st, q));
  if (!partial || !out) { set_error("bad attend_merge arguments"); return KIV_ERR_ARG; }
  const int64_t rows = (int64_t)st->batch * q->num_query_heads * q->query_len;
  kiv::XArgs a;
  KIV_TRY(check_exchange(st, q, x, kiv::X_ATTN, rows * ceil_div(st->head_dim, 64), a));
  return launch_attend_merge(st, q, partial, x->world, out, (cudaStream_t)stream, &a);
}

kiv_status kiv_read_state(const kiv_store *st, int64_t *host_words, void *stream) {
  if (!st || !st->state || !host_words) { set_error("bad read_state arguments"); return KIV_ERR_ARG; }
  cudaStream_t s = (cudaStream_t)stream;
  KIV_TRY(cuda_status(cudaMemcpyAsync(host_words, st->state, KIV_STATE_WORDS * sizeof(int64_t),
                                      cudaMemcpyDeviceToHost, s), "read_state"));
  return cuda_status(cudaStreamSynchronize(s), "read_state sync");
}

}  // extern "C"
