// PyTorch operator registration of the C ABI: torch.ops.kiv.*
//
// Every operator is a thin adapter: it builds the POD descriptors of
// include/kiv_b200.h from tensors (data pointers, shapes, strides, dtype) and
// calls the `extern "C"` entry point on the current CUDA stream of the
// store's device.  The C ABI stays the boundary; this file only makes it
// visible to the dispatcher, so the operators show up in traces, run under
// torch.cuda.graph capture like any other CUDA op, and have Meta kernels
// (shape-only, no work) for tracing with fake tensors.
//
// A store is passed as two lists:
//   store = [cold_k, cold_v, summaries, hot_k, hot_v, state, host_k, host_v, page_sums]
//           (hot_*, host_* and page_sums may be empty tensors: no hot ring,
//           no host tier, no replicated summaries)
//   geom  = [page_size, shard_rank, shard_count, hot_hint, stage_pages, flags]
// and a query as (q [B, Hq, Q, D], scaling, top_pages, top_p, softcap).
// The operators that write return nothing and declare what they mutate in
// their schema.  Failures raise RuntimeError with the library's message.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include <cstdint>
#include <vector>

#include "../../include/kiv_b200.h"

namespace {

using at::Tensor;

void *ptr_or_null(const Tensor &t) { return t.defined() && t.numel() > 0 ? t.data_ptr() : nullptr; }

int32_t dtype_code(const Tensor &t) {
  switch (t.scalar_type()) {
    case at::kFloat: return KIV_DTYPE_F32;
    case at::kBFloat16: return KIV_DTYPE_BF16;
    case at::kHalf: return KIV_DTYPE_F16;
    default: TORCH_CHECK(false, "kiv: store dtype must be float32, bfloat16 or float16, got ", t.scalar_type());
  }
  return -1;
}

kiv_store make_store(at::TensorList s, at::IntArrayRef g) {
  TORCH_CHECK(s.size() == 9, "kiv: store list must hold 9 tensors (cold_k, cold_v, summaries, hot_k, hot_v, "
                             "state, host_k, host_v, page_sums), got ", s.size());
  TORCH_CHECK(g.size() == 6, "kiv: geom must hold 6 ints (page_size, shard_rank, shard_count, hot_hint, "
                             "stage_pages, flags), got ", g.size());
  const Tensor &ck = s[0], &hk = s[3], &st = s[5], &hok = s[6];
  TORCH_CHECK(ck.dim() == 4, "kiv: cold_k must be [B, Hkv, slots, D]");
  TORCH_CHECK(st.scalar_type() == at::kLong && st.numel() >= KIV_STATE_WORDS, "kiv: state must be int64[32]");
  kiv_store d = {};
  d.batch = (int32_t)ck.size(0);
  d.num_kv_heads = (int32_t)ck.size(1);
  d.head_dim = (int32_t)ck.size(3);
  d.page_size = (int32_t)g[0];
  d.dtype = dtype_code(ck);
  d.shard_rank = (int32_t)g[1];
  d.shard_count = (int32_t)g[2];
  d.hot_hint = (int32_t)g[3];
  d.cold_capacity = ck.size(2);
  d.hot_capacity = hk.defined() && hk.numel() > 0 ? hk.size(2) : 0;
  d.cold_k = ptr_or_null(s[0]);
  d.cold_v = ptr_or_null(s[1]);
  d.summaries = ptr_or_null(s[2]);
  d.hot_k = ptr_or_null(s[3]);
  d.hot_v = ptr_or_null(s[4]);
  d.state = static_cast<int64_t *>(st.data_ptr());
  d.host_capacity = hok.defined() && hok.numel() > 0 ? hok.size(2) : 0;
  d.host_k = ptr_or_null(s[6]);
  d.host_v = ptr_or_null(s[7]);
  d.stage_pages = (int32_t)g[4];
  d.flags = (int32_t)g[5];
  d.page_sums = static_cast<float *>(ptr_or_null(s[8]));
  return d;
}

kiv_query make_query(const Tensor &q, double scaling, int64_t top_pages, int64_t top_p, double softcap) {
  TORCH_CHECK(q.dim() == 4 && q.stride(3) == 1, "kiv: query must be [B, Hq, Q, D] with a contiguous last dim");
  kiv_query d = {};
  d.q = q.data_ptr();
  d.stride_b = q.stride(0);
  d.stride_h = q.stride(1);
  d.stride_t = q.stride(2);
  d.num_query_heads = (int32_t)q.size(1);
  d.query_len = (int32_t)q.size(2);
  d.scaling = (float)scaling;
  d.softcap = (float)softcap;
  d.top_pages = (int32_t)top_pages;
  d.top_p = (int32_t)top_p;
  return d;
}

kiv_mask make_mask(const c10::optional<Tensor> &add, bool causal) {
  kiv_mask m = {};
  m.causal = causal ? 1 : 0;
  if (add.has_value() && add->defined()) {
    const Tensor &a = *add;
    TORCH_CHECK(a.scalar_type() == at::kFloat && a.dim() == 4 && a.stride(3) == 1,
                "kiv: mask must be float32 [B, 1|Hq, Q, hot] with a contiguous last dim");
    m.add = a.data_ptr<float>();
    m.stride_b = a.size(0) == 1 ? 0 : a.stride(0);
    m.stride_h = a.size(1) == 1 ? 0 : a.stride(1);
    m.stride_t = a.stride(2);
  }
  return m;
}

kiv_exchange make_exchange(const kiv_store &st, at::IntArrayRef arenas, int64_t arena_bytes, int64_t wait_cycles) {
  TORCH_CHECK((int64_t)arenas.size() == st.shard_count && st.shard_count <= KIV_MAX_PEERS,
              "kiv: one arena address per rank expected");
  kiv_exchange x = {};
  x.world = st.shard_count;
  x.rank = st.shard_rank;
  for (size_t i = 0; i < arenas.size(); ++i) x.arena[i] = reinterpret_cast<void *>(arenas[i]);
  x.arena_bytes = arena_bytes;
  x.wait_cycles = wait_cycles;
  return x;
}

void check(kiv_status rc, const char *what) {
  TORCH_CHECK(rc == KIV_OK, "kiv.", what, ": ", kiv_status_string(rc), " (", rc, "): ", kiv_last_error());
}

void *stream_of(const Tensor &t) { return at::cuda::getCurrentCUDAStream(t.device().index()).stream(); }

// ------------------------------------------------------------- CUDA kernels
void state_reset(at::TensorList store, at::IntArrayRef geom) {
  const kiv_store st = make_store(store, geom);
  c10::cuda::CUDAGuard g(store[5].device());
  check(kiv_state_reset(&st, stream_of(store[5])), "state_reset");
}

void append_evict(at::TensorList store, at::IntArrayRef geom, const c10::optional<Tensor> &k_new,
                  const c10::optional<Tensor> &v_new, int64_t keep, int64_t n_evict_max) {
  const kiv_store st = make_store(store, geom);
  c10::cuda::CUDAGuard g(store[5].device());
  const void *kp = nullptr, *vp = nullptr;
  int64_t sb = 0, sh = 0, stt = 0;
  int32_t n_new = 0;
  if (k_new.has_value() && k_new->defined()) {
    const Tensor &k = *k_new, &v = *v_new;
    TORCH_CHECK(k.dim() == 4 && v.sizes() == k.sizes(), "kiv: new K/V rows must both be [B, Hkv, n, D]");
    // one set of strides serves both (a dimension of size 1 is never stepped)
    for (int d = 0; d < 4; ++d)
      TORCH_CHECK(k.size(d) == 1 || k.stride(d) == v.stride(d), "kiv: new K and V rows need the same strides");
    TORCH_CHECK(k.scalar_type() == store[0].scalar_type(), "kiv: new rows must have the store dtype");
    kp = k.data_ptr();
    vp = v.data_ptr();
    sb = k.stride(0);
    sh = k.stride(1);
    stt = k.stride(2);
    n_new = (int32_t)k.size(2);
  }
  check(kiv_append_evict(&st, kp, vp, sb, sh, stt, n_new, keep, n_evict_max, stream_of(store[5])), "append_evict");
}

void coarse_select(at::TensorList store, at::IntArrayRef geom, const Tensor &q, double scaling, int64_t top_pages,
                   int64_t top_p, double softcap, const Tensor &ws, const c10::optional<Tensor> &row_scores,
                   const c10::optional<Tensor> &row_pages) {
  const kiv_store st = make_store(store, geom);
  const kiv_query qd = make_query(q, scaling, top_pages, top_p, softcap);
  c10::cuda::CUDAGuard g(q.device());
  float *rs = row_scores.has_value() && row_scores->defined() ? row_scores->data_ptr<float>() : nullptr;
  int32_t *rp = row_pages.has_value() && row_pages->defined() ? row_pages->data_ptr<int32_t>() : nullptr;
  check(kiv_coarse_select(&st, &qd, ws.data_ptr(), (size_t)ws.nbytes(), rs, rp, stream_of(q)), "coarse_select");
}

void coarse_merge(at::TensorList store, at::IntArrayRef geom, const Tensor &q, double scaling, int64_t top_pages,
                  int64_t top_p, double softcap, const Tensor &ws, const Tensor &lists_scores,
                  const Tensor &lists_pages) {
  const kiv_store st = make_store(store, geom);
  const kiv_query qd = make_query(q, scaling, top_pages, top_p, softcap);
  c10::cuda::CUDAGuard g(q.device());
  check(kiv_coarse_merge(&st, &qd, ws.data_ptr(), (size_t)ws.nbytes(), lists_scores.data_ptr<float>(),
                         lists_pages.data_ptr<int32_t>(), (int32_t)lists_scores.size(0), stream_of(q)),
        "coarse_merge");
}

void fine_score(at::TensorList store, at::IntArrayRef geom, const Tensor &q, double scaling, int64_t top_pages,
                int64_t top_p, double softcap, const Tensor &ws) {
  const kiv_store st = make_store(store, geom);
  const kiv_query qd = make_query(q, scaling, top_pages, top_p, softcap);
  c10::cuda::CUDAGuard g(q.device());
  check(kiv_fine_score(&st, &qd, ws.data_ptr(), (size_t)ws.nbytes(), stream_of(q)), "fine_score");
}

void fine_topk(at::TensorList store, at::IntArrayRef geom, const Tensor &q, double scaling, int64_t top_pages,
               int64_t top_p, double softcap, const Tensor &ws, const Tensor &sel,
               const c10::optional<Tensor> &sel_scores) {
  const kiv_store st = make_store(store, geom);
  const kiv_query qd = make_query(q, scaling, top_pages, top_p, softcap);
  c10::cuda::CUDAGuard g(q.device());
  float *ss = sel_scores.has_value() && sel_scores->defined() ? sel_scores->data_ptr<float>() : nullptr;
  check(kiv_fine_topk(&st, &qd, ws.data_ptr(), (size_t)ws.nbytes(), sel.data_ptr<int32_t>(), ss, stream_of(q)),
        "fine_topk");
}

void fine_select(at::TensorList store, at::IntArrayRef geom, const Tensor &q, double scaling, int64_t top_pages,
                 int64_t top_p, double softcap, const Tensor &ws, const Tensor &sel,
                 const c10::optional<Tensor> &sel_scores) {
  const kiv_store st = make_store(store, geom);
  const kiv_query qd = make_query(q, scaling, top_pages, top_p, softcap);
  c10::cuda::CUDAGuard g(q.device());
  float *ss = sel_scores.has_value() && sel_scores->defined() ? sel_scores->data_ptr<float>() : nullptr;
  check(kiv_fine_select(&st, &qd, ws.data_ptr(), (size_t)ws.nbytes(), sel.data_ptr<int32_t>(), ss, stream_of(q)),
        "fine_select");
}

void fine_merge(at::TensorList store, at::IntArrayRef geom, const Tensor &q, double scaling, int64_t top_pages,
                int64_t top_p, double softcap, const Tensor &ws, const Tensor &lists_scores,
                const Tensor &lists_tokens, const Tensor &sel, const Tensor &sel_local) {
  const kiv_store st = make_store(store, geom);
  const kiv_query qd = make_query(q, scaling, top_pages, top_p, softcap);
  c10::cuda::CUDAGuard g(q.device());
  check(kiv_fine_merge(&st, &qd, ws.data_ptr(), (size_t)ws.nbytes(), lists_scores.data_ptr<float>(),
                       lists_tokens.data_ptr<int32_t>(), (int32_t)lists_scores.size(0), sel.data_ptr<int32_t>(),
                       sel_local.data_ptr<int32_t>(), stream_of(q)),
        "fine_merge");
}

void gather_rows(at::TensorList store, at::IntArrayRef geom, const Tensor &sel, int64_t P, const Tensor &out_k,
                 const Tensor &out_v) {
  const kiv_store st = make_store(store, geom);
  c10::cuda::CUDAGuard g(sel.device());
  check(kiv_gather_rows(&st, sel.data_ptr<int32_t>(), (int32_t)sel.size(1), (int32_t)P, ptr_or_null(out_k),
                        ptr_or_null(out_v), stream_of(sel)),
        "gather_rows");
}

void attend(at::TensorList store, at::IntArrayRef geom, const Tensor &q, double scaling, int64_t top_pages,
            int64_t top_p, double softcap, const Tensor &ws, const Tensor &sel, const c10::optional<Tensor> &mask_add,
            bool causal, int64_t hot_slice, int64_t hot_slices, const c10::optional<Tensor> &out,
            const c10::optional<Tensor> &partial_out) {
  const kiv_store st = make_store(store, geom);
  const kiv_query qd = make_query(q, scaling, top_pages, top_p, softcap);
  const kiv_mask md = make_mask(mask_add, causal);
  c10::cuda::CUDAGuard g(q.device());
  void *o = out.has_value() && out->defined() ? out->data_ptr() : nullptr;
  float *po = partial_out.has_value() && partial_out->defined() ? partial_out->data_ptr<float>() : nullptr;
  check(kiv_attend(&st, &qd, &md, ws.data_ptr(), (size_t)ws.nbytes(), sel.data_ptr<int32_t>(), (int32_t)sel.size(1),
                   (int32_t)hot_slice, (int32_t)hot_slices, o, po, stream_of(q)),
        "attend");
}

void attend_peers(at::TensorList store, at::IntArrayRef geom, const Tensor &q, double scaling, int64_t top_pages,
                  int64_t top_p, double softcap, const Tensor &ws, const Tensor &sel,
                  const c10::optional<Tensor> &mask_add, bool causal, at::IntArrayRef peer_k, at::IntArrayRef peer_v,
                  const Tensor &out) {
  const kiv_store st = make_store(store, geom);
  const kiv_query qd = make_query(q, scaling, top_pages, top_p, softcap);
  const kiv_mask md = make_mask(mask_add, causal);
  TORCH_CHECK(peer_k.size() == (size_t)st.shard_count && peer_v.size() == (size_t)st.shard_count &&
                  st.shard_count <= KIV_MAX_PEERS,
              "kiv: attend_peers needs one cold_k and cold_v address per shard");
  kiv_peer_rows pr = {};
  for (int r = 0; r < st.shard_count; ++r) {
    pr.cold_k[r] = reinterpret_cast<const void *>(static_cast<uintptr_t>(peer_k[r]));
    pr.cold_v[r] = reinterpret_cast<const void *>(static_cast<uintptr_t>(peer_v[r]));
  }
  c10::cuda::CUDAGuard g(q.device());
  check(kiv_attend_peers(&st, &qd, &md, ws.data_ptr(), (size_t)ws.nbytes(), sel.data_ptr<int32_t>(),
                         (int32_t)sel.size(1), &pr, out.data_ptr(), stream_of(q)),
        "attend_peers");
}

void attend_merge(at::TensorList store, at::IntArrayRef geom, const Tensor &q, double scaling, int64_t top_pages,
                  int64_t top_p, double softcap, const Tensor &partials, const Tensor &out) {
  const kiv_store st = make_store(store, geom);
  const kiv_query qd = make_query(q, scaling, top_pages, top_p, softcap);
  c10::cuda::CUDAGuard g(q.device());
  check(kiv_attend_merge(&st, &qd, partials.data_ptr<float>(), (int32_t)partials.size(0), out.data_ptr(),
                         stream_of(q)),
        "attend_merge");
}

void retrieve_attend(at::TensorList store, at::IntArrayRef geom, const Tensor &q, double scaling, int64_t top_pages,
                     int64_t top_p, double softcap, const Tensor &ws, int64_t reuse, const Tensor &sel,
                     const c10::optional<Tensor> &mask_add, bool causal, const Tensor &out) {
  const kiv_store st = make_store(store, geom);
  const kiv_query qd = make_query(q, scaling, top_pages, top_p, softcap);
  const kiv_mask md = make_mask(mask_add, causal);
  c10::cuda::CUDAGuard g(q.device());
  check(kiv_retrieve_attend(&st, &qd, &md, ws.data_ptr(), (size_t)ws.nbytes(), (int32_t)reuse,
                            sel.data_ptr<int32_t>(), out.data_ptr(), stream_of(q)),
        "retrieve_attend");
}

void coarse_exchange_merge(at::TensorList store, at::IntArrayRef geom, const Tensor &q, double scaling,
                           int64_t top_pages, int64_t top_p, double softcap, const Tensor &ws,
                           const Tensor &row_scores, const Tensor &row_pages, at::IntArrayRef arenas,
                           int64_t arena_bytes, int64_t wait_cycles) {
  const kiv_store st = make_store(store, geom);
  const kiv_query qd = make_query(q, scaling, top_pages, top_p, softcap);
  const kiv_exchange x = make_exchange(st, arenas, arena_bytes, wait_cycles);
  c10::cuda::CUDAGuard g(q.device());
  check(kiv_coarse_exchange_merge(&st, &qd, ws.data_ptr(), (size_t)ws.nbytes(), row_scores.data_ptr<float>(),
                                  row_pages.data_ptr<int32_t>(), &x, stream_of(q)),
        "coarse_exchange_merge");
}

void fine_exchange_merge(at::TensorList store, at::IntArrayRef geom, const Tensor &q, double scaling,
                         int64_t top_pages, int64_t top_p, double softcap, const Tensor &ws, const Tensor &scores,
                         const Tensor &tokens, at::IntArrayRef arenas, int64_t arena_bytes, int64_t wait_cycles,
                         const c10::optional<Tensor> &sel, const Tensor &sel_local) {
  const kiv_store st = make_store(store, geom);
  const kiv_query qd = make_query(q, scaling, top_pages, top_p, softcap);
  const kiv_exchange x = make_exchange(st, arenas, arena_bytes, wait_cycles);
  c10::cuda::CUDAGuard g(q.device());
  int32_t *s = sel.has_value() && sel->defined() ? sel->data_ptr<int32_t>() : nullptr;
  check(kiv_fine_exchange_merge(&st, &qd, ws.data_ptr(), (size_t)ws.nbytes(), scores.data_ptr<float>(),
                                tokens.data_ptr<int32_t>(), &x, s, sel_local.data_ptr<int32_t>(), stream_of(q)),
        "fine_exchange_merge");
}

void fine_exchange_select(at::TensorList store, at::IntArrayRef geom, const Tensor &q, double scaling,
                          int64_t top_pages, int64_t top_p, double softcap, const Tensor &ws, at::IntArrayRef arenas,
                          int64_t arena_bytes, int64_t wait_cycles, const Tensor &sel,
                          const c10::optional<Tensor> &sel_local) {
  const kiv_store st = make_store(store, geom);
  const kiv_query qd = make_query(q, scaling, top_pages, top_p, softcap);
  const kiv_exchange x = make_exchange(st, arenas, arena_bytes, wait_cycles);
  c10::cuda::CUDAGuard g(q.device());
  int32_t *sl = sel_local.has_value() && sel_local->defined() ? sel_local->data_ptr<int32_t>() : nullptr;
  check(kiv_fine_exchange_select(&st, &qd, ws.data_ptr(), (size_t)ws.nbytes(), &x, sel.data_ptr<int32_t>(), sl,
                                 stream_of(q)),
        "fine_exchange_select");
}

void attend_exchange_merge(at::TensorList store, at::IntArrayRef geom, const Tensor &q, double scaling,
                           int64_t top_pages, int64_t top_p, double softcap, const Tensor &partial,
                           at::IntArrayRef arenas, int64_t arena_bytes, int64_t wait_cycles, const Tensor &out) {
  const kiv_store st = make_store(store, geom);
  const kiv_query qd = make_query(q, scaling, top_pages, top_p, softcap);
  const kiv_exchange x = make_exchange(st, arenas, arena_bytes, wait_cycles);
  c10::cuda::CUDAGuard g(q.device());
  check(kiv_attend_exchange_merge(&st, &qd, partial.data_ptr<float>(), &x, out.data_ptr(), stream_of(q)),
        "attend_exchange_merge");
}

// ------------------------------------------------------------ shape queries
// Workspace size and sub-buffer offsets: pure arithmetic on shapes (the data
// pointers are stand-ins), so the same kernel serves real and fake tensors.
std::vector<int64_t> workspace_layout(at::TensorList store, at::IntArrayRef geom, const Tensor &q,
                                      int64_t top_pages, int64_t top_p) {
  TORCH_CHECK(store.size() == 9 && geom.size() == 6, "kiv: bad store descriptor lists");
  const Tensor &ck = store[0], &hk = store[3], &hok = store[6];
  TORCH_CHECK(ck.dim() == 4 && q.dim() == 4, "kiv: bad store or query rank");
  char *fake = reinterpret_cast<char *>(uintptr_t(1) << 20);
  kiv_store st = {};
  st.batch = (int32_t)ck.size(0);
  st.num_kv_heads = (int32_t)ck.size(1);
  st.head_dim = (int32_t)ck.size(3);
  st.page_size = (int32_t)geom[0];
  st.dtype = dtype_code(ck);
  st.shard_rank = (int32_t)geom[1];
  st.shard_count = (int32_t)geom[2];
  st.hot_hint = (int32_t)geom[3];
  st.cold_capacity = ck.size(2);
  st.hot_capacity = hk.numel() > 0 ? hk.size(2) : 0;
  st.cold_k = st.cold_v = st.summaries = fake;
  st.hot_k = st.hot_v = st.hot_capacity > 0 ? fake : nullptr;
  st.state = reinterpret_cast<int64_t *>(fake);
  st.host_capacity = hok.numel() > 0 ? hok.size(2) : 0;
  st.host_k = st.host_v = st.host_capacity > 0 ? fake : nullptr;
  st.stage_pages = (int32_t)geom[4];
  st.flags = (int32_t)geom[5];
  st.page_sums = store[8].numel() > 0 ? reinterpret_cast<float *>(fake) : nullptr;
  kiv_query qd = {};
  qd.q = fake;
  // strides of a contiguous query (only their 16-byte alignment is checked)
  qd.stride_t = q.size(3);
  qd.stride_h = q.size(2) * q.size(3);
  qd.stride_b = q.size(1) * qd.stride_h;
  qd.num_query_heads = (int32_t)q.size(1);
  qd.query_len = (int32_t)q.size(2);
  qd.scaling = 1.f;
  qd.top_pages = (int32_t)top_pages;
  qd.top_p = (int32_t)top_p;
  std::vector<int64_t> out(11, 0);
  check(kiv_workspace_layout(&st, &qd, out.data()), "workspace_layout");
  out[10] = (int64_t)kiv_workspace_bytes(&st, &qd);
  return out;
}

// ------------------------------------------------------------- Meta kernels
// Shape-only: the writes go to caller-provided tensors, so tracing with fake
// tensors has nothing to compute.
void state_reset_meta(at::TensorList, at::IntArrayRef) {}
void append_evict_meta(at::TensorList, at::IntArrayRef, const c10::optional<Tensor> &, const c10::optional<Tensor> &,
                       int64_t, int64_t) {}
void coarse_select_meta(at::TensorList, at::IntArrayRef, const Tensor &, double, int64_t, int64_t, double,
                        const Tensor &, const c10::optional<Tensor> &, const c10::optional<Tensor> &) {}
void coarse_merge_meta(at::TensorList, at::IntArrayRef, const Tensor &, double, int64_t, int64_t, double,
                       const Tensor &, const Tensor &, const Tensor &) {}
void fine_score_meta(at::TensorList, at::IntArrayRef, const Tensor &, double, int64_t, int64_t, double,
                     const Tensor &) {}
void fine_topk_meta(at::TensorList, at::IntArrayRef, const Tensor &, double, int64_t, int64_t, double,
                    const Tensor &, const Tensor &, const c10::optional<Tensor> &) {}
void fine_select_meta(at::TensorList, at::IntArrayRef, const Tensor &, double, int64_t, int64_t, double,
                      const Tensor &, const Tensor &, const c10::optional<Tensor> &) {}
void fine_merge_meta(at::TensorList, at::IntArrayRef, const Tensor &, double, int64_t, int64_t, double,
                     const Tensor &, const Tensor &, const Tensor &, const Tensor &, const Tensor &) {}
void gather_rows_meta(at::TensorList, at::IntArrayRef, const Tensor &, int64_t, const Tensor &, const Tensor &) {}
void attend_meta(at::TensorList, at::IntArrayRef, const Tensor &, double, int64_t, int64_t, double, const Tensor &,
                 const Tensor &, const c10::optional<Tensor> &, bool, int64_t, int64_t, const c10::optional<Tensor> &,
                 const c10::optional<Tensor> &) {}
void attend_merge_meta(at::TensorList, at::IntArrayRef, const Tensor &, double, int64_t, int64_t, double,
                       const Tensor &, const Tensor &) {}
void retrieve_attend_meta(at::TensorList, at::IntArrayRef, const Tensor &, double, int64_t, int64_t, double,
                          const Tensor &, int64_t, const Tensor &, const c10::optional<Tensor> &, bool,
                          const Tensor &) {}
void coarse_exchange_merge_meta(at::TensorList, at::IntArrayRef, const Tensor &, double, int64_t, int64_t, double,
                                const Tensor &, const Tensor &, const Tensor &, at::IntArrayRef, int64_t, int64_t) {}
void fine_exchange_merge_meta(at::TensorList, at::IntArrayRef, const Tensor &, double, int64_t, int64_t, double,
                              const Tensor &, const Tensor &, const Tensor &, at::IntArrayRef, int64_t, int64_t,
                              const c10::optional<Tensor> &, const Tensor &) {}
void fine_exchange_select_meta(at::TensorList, at::IntArrayRef, const Tensor &, double, int64_t, int64_t, double,
                               const Tensor &, at::IntArrayRef, int64_t, int64_t, const Tensor &,
                               const c10::optional<Tensor> &) {}
void attend_peers_meta(at::TensorList, at::IntArrayRef, const Tensor &, double, int64_t, int64_t, double,
                       const Tensor &, const Tensor &, const c10::optional<Tensor> &, bool, at::IntArrayRef,
                       at::IntArrayRef, const Tensor &) {}
void attend_exchange_merge_meta(at::TensorList, at::IntArrayRef, const Tensor &, double, int64_t, int64_t, double,
                                const Tensor &, at::IntArrayRef, int64_t, int64_t, const Tensor &) {}

}  // namespace

#define KIV_Q "Tensor q, float scaling, int top_pages, int top_p, float softcap"

TORCH_LIBRARY(kiv, m) {
  // Replaces: kiv/cold_store.py:142-184 (evict_from_hot), kiv/tiered_cache.py:55-72, :107-142
  m.def("state_reset(Tensor(a!)[] store, int[] geom) -> ()");
  m.def("append_evict(Tensor(a!)[] store, int[] geom, Tensor? k_new, Tensor? v_new, int keep, "
        "int n_evict_max) -> ()");
  m.def("workspace_layout(Tensor[] store, int[] geom, Tensor q, int top_pages, int top_p) -> int[]");
  // Replaces: kiv/cold_store.py:203-230 (coarse scoring, per-row top-k, union)
  m.def("coarse_select(Tensor(a!)[] store, int[] geom, " KIV_Q ", Tensor(b!) ws, Tensor(c!)? row_scores, "
        "Tensor(d!)? row_pages) -> ()");
  m.def("coarse_merge(Tensor(a!)[] store, int[] geom, " KIV_Q ", Tensor(b!) ws, Tensor lists_scores, "
        "Tensor lists_pages) -> ()");
  // Replaces: kiv/cold_store.py:227-262 (candidates), :301, :332-347 (fine scores, max, top-P)
  m.def("fine_score(Tensor(a!)[] store, int[] geom, " KIV_Q ", Tensor(b!) ws) -> ()");
  m.def("fine_topk(Tensor(a!)[] store, int[] geom, " KIV_Q ", Tensor(b!) ws, Tensor(c!) sel, "
        "Tensor(d!)? sel_scores) -> ()");
  m.def("fine_select(Tensor(a!)[] store, int[] geom, " KIV_Q ", Tensor(b!) ws, Tensor(c!) sel, "
        "Tensor(d!)? sel_scores) -> ()");
  m.def("fine_merge(Tensor(a!)[] store, int[] geom, " KIV_Q ", Tensor(b!) ws, Tensor lists_scores, "
        "Tensor lists_tokens, Tensor(c!) sel, Tensor(d!) sel_local) -> ()");
  // Replaces: kiv/cold_store.py:357-362 (gather of the selected K/V rows)
  m.def("gather_rows(Tensor[] store, int[] geom, Tensor sel, int P, Tensor(b!) out_k, Tensor(c!) out_v) -> ()");
  // Replaces: kiv/middleware.py:330-352 and kiv/mask_utils.py:8-38 (attention over [cold ; hot])
  m.def("attend(Tensor(a!)[] store, int[] geom, " KIV_Q ", Tensor(b!) ws, Tensor sel, Tensor? mask_add, "
        "bool causal, int hot_slice, int hot_slices, Tensor(c!)? out, Tensor(d!)? partial_out) -> ()");
  m.def("attend_merge(Tensor[] store, int[] geom, " KIV_Q ", Tensor partials, Tensor(b!) out) -> ()");
  // Replaces: kiv/cold_store.py:283-371 + kiv/middleware.py:308-354 (one call)
  m.def("retrieve_attend(Tensor(a!)[] store, int[] geom, " KIV_Q ", Tensor(b!) ws, int reuse, Tensor(c!) sel, "
        "Tensor? mask_add, bool causal, Tensor(d!) out) -> ()");
  // Sharded layer-step exchanges (no reference counterpart: it has no multi-GPU code)
  m.def("coarse_exchange_merge(Tensor(a!)[] store, int[] geom, " KIV_Q ", Tensor(b!) ws, Tensor row_scores, "
        "Tensor row_pages, int[] arenas, int arena_bytes, int wait_cycles) -> ()");
  m.def("fine_exchange_merge(Tensor(a!)[] store, int[] geom, " KIV_Q ", Tensor(b!) ws, Tensor scores, "
        "Tensor tokens, int[] arenas, int arena_bytes, int wait_cycles, Tensor(c!)? sel, Tensor(d!) sel_local) -> ()");
  m.def("attend_exchange_merge(Tensor(a!)[] store, int[] geom, " KIV_Q ", Tensor partial, int[] arenas, "
        "int arena_bytes, int wait_cycles, Tensor(b!) out) -> ()");
  // Replaces, for page-sharded stores: kiv/cold_store.py:283-371 steps 2-3 (fine pass over the whole union)
  m.def("fine_exchange_select(Tensor(a!)[] store, int[] geom, " KIV_Q ", Tensor(b!) ws, int[] arenas, "
        "int arena_bytes, int wait_cycles, Tensor(c!) sel, Tensor(d!)? sel_local) -> ()");
  // Replaces, for page-sharded stores: kiv/middleware.py:330-352, kiv/mask_utils.py:8-38 (rows read from
  // every shard's cold tier; peer addresses as int[])
  m.def("attend_peers(Tensor(a!)[] store, int[] geom, " KIV_Q ", Tensor(b!) ws, Tensor sel, Tensor? mask_add, "
        "bool causal, int[] peer_k, int[] peer_v, Tensor(c!) out) -> ()");
}

TORCH_LIBRARY_IMPL(kiv, CUDA, m) {
  m.impl("state_reset", &state_reset);
  m.impl("append_evict", &append_evict);
  m.impl("coarse_select", &coarse_select);
  m.impl("coarse_merge", &coarse_merge);
  m.impl("fine_score", &fine_score);
  m.impl("fine_topk", &fine_topk);
  m.impl("fine_select", &fine_select);
  m.impl("fine_merge", &fine_merge);
  m.impl("gather_rows", &gather_rows);
  m.impl("attend", &attend);
  m.impl("attend_merge", &attend_merge);
  m.impl("retrieve_attend", &retrieve_attend);
  m.impl("coarse_exchange_merge", &coarse_exchange_merge);
  m.impl("fine_exchange_merge", &fine_exchange_merge);
  m.impl("attend_exchange_merge", &attend_exchange_merge);
  m.impl("fine_exchange_select", &fine_exchange_select);
  m.impl("attend_peers", &attend_peers);
}

TORCH_LIBRARY_IMPL(kiv, Meta, m) {
  m.impl("state_reset", &state_reset_meta);
  m.impl("append_evict", &append_evict_meta);
  m.impl("coarse_select", &coarse_select_meta);
  m.impl("coarse_merge", &coarse_merge_meta);
  m.impl("fine_score", &fine_score_meta);
  m.impl("fine_topk", &fine_topk_meta);
  m.impl("fine_select", &fine_select_meta);
  m.impl("fine_merge", &fine_merge_meta);
  m.impl("gather_rows", &gather_rows_meta);
  m.impl("attend", &attend_meta);
  m.impl("attend_merge", &attend_merge_meta);
  m.impl("retrieve_attend", &retrieve_attend_meta);
  m.impl("coarse_exchange_merge", &coarse_exchange_merge_meta);
  m.impl("fine_exchange_merge", &fine_exchange_merge_meta);
  m.impl("attend_exchange_merge", &attend_exchange_merge_meta);
  m.impl("fine_exchange_select", &fine_exchange_select_meta);
  m.impl("attend_peers", &attend_peers_meta);
}

TORCH_LIBRARY_IMPL(kiv, CompositeExplicitAutograd, m) { m.impl("workspace_layout", &workspace_layout); }
