/*
 * kiv_b200.h -- C ABI of libkiv_b200.so, the sm_100a kernels behind KIV's
 * tiered-cache retrieval attention.
 *
 * The library replaces the tensor work of the reference's cold store
 * (kiv/cold_store.py) and of its HF attention wrapper (kiv/middleware.py).
 * Every entry point is `extern "C"`, takes plain pointers, sizes and POD
 * descriptors, launches its kernels on the caller's stream and returns a
 * status code; none synchronizes the host.  Memory is owned by the caller
 * (the Python host allocates it through PyTorch); the library allocates
 * nothing on any of these calls.
 *
 * Per-layer state that changes every decode step (cold length, hot-ring
 * start and length, the sizes of the last retrieval) lives in DEVICE memory
 * (`kiv_store.state`), so a decode step launches the same kernels with the
 * same arguments every time and can be captured in a CUDA graph and replayed.
 *
 * Layouts (all innermost-contiguous, element type = store dtype):
 *   cold_k, cold_v  [B, Hkv, cold_capacity, D]   token slots of this shard
 *   summaries       [B, Hkv, cold_capacity / S, D] mean-K of each finalized page
 *                   (shard_count * (cold_capacity / S + 1) pages with replicated summaries)
 *   hot_k, hot_v    [B, Hkv, hot_capacity, D]    ring: logical hot row j lives
 *                                                 at slot (hot_start + j) % hot_capacity
 * Sharding: global page p lives on shard p % shard_count at local page
 * p / shard_count; with shard_count == 1 local == global.
 *
 * Host overflow tier (host_capacity > 0): the HBM cold slots hold a ring of
 * the newest R = cold_capacity / S - stage_pages local pages (local page lp at
 * ring page lp % R) plus stage_pages staging pages after it; older pages live
 * in pinned, device-mapped host memory, page lp at rows [lp*S, lp*S + S) of
 *   host_k, host_v  [B, Hkv, host_capacity, D]
 * and the summaries cover all R + host_capacity / S local pages.  The
 * eviction kernel copies a ring page to the host tier just before the ring
 * slot is reused; a retrieval gathers the union's host pages (K) and its
 * selected host rows (V) into the staging pages before the kernels read them.
 */
#ifndef KIV_B200_H
#define KIV_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define KIV_API __attribute__((visibility("default")))
#else
#define KIV_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef int32_t kiv_status;
#define KIV_OK 0
#define KIV_ERR_ARG 1          /* invalid argument or shape */
#define KIV_ERR_CAPACITY 2     /* a buffer (store, ring, workspace) is too small */
#define KIV_ERR_CUDA 3         /* a CUDA runtime call failed; see kiv_last_error() */
#define KIV_ERR_UNSUPPORTED 4  /* dtype / head_dim / shape not compiled in */

#define KIV_DTYPE_F32 0
#define KIV_DTYPE_BF16 1
#define KIV_DTYPE_F16 2

/* Device-resident state words (int64 each) of one store. */
#define KIV_STATE_WORDS 32
#define KIV_ST_COLD_LEN 0   /* global tokens in the cold tier (finalized + partial) */
#define KIV_ST_HOT_START 1  /* ring slot of logical hot row 0 */
#define KIV_ST_HOT_LEN 2    /* live hot rows */
#define KIV_ST_UNION 3      /* pages in the last coarse union (this shard) */
#define KIV_ST_CAND 4       /* fine candidates of the last retrieval (this shard) */
#define KIV_ST_SEL 5        /* tokens selected by the last retrieval (per batch row) */
#define KIV_ST_SEL_LOCAL 6  /* of those, tokens owned by this shard */
#define KIV_ST_ERROR 7      /* sticky error bits set by kernels (KIV_ERRBIT_*) */
#define KIV_ST_COARSE_MAX 8  /* order-preserving key of the largest coarse score of the last pass */
#define KIV_ST_COARSE_SUM 9  /* double: sum of all coarse scores of the last pass */
#define KIV_ST_FINE_MAX 10   /* key of the largest fine (max over heads) score */
#define KIV_ST_FINE_SUM 11   /* double: sum of the fine scores of all candidates */
#define KIV_ST_UNION_PENDING 12  /* 1: the page marks hold a new union the fine pass must read */
/* words 16..31 are kernel-private counters */

/* Error bits a kernel sets in state[KIV_ST_ERROR] instead of writing out of bounds. */
#define KIV_ERRBIT_EVICT_CAPACITY 1   /* ring, cold store or grid too small: call skipped */
#define KIV_ERRBIT_UNION_CAPACITY 2   /* union larger than the workspace: truncated */
#define KIV_ERRBIT_CAND_CAPACITY 4    /* candidates larger than the workspace */
#define KIV_ERRBIT_WAIT_TIMEOUT 8     /* a bounded wait on a bulk copy gave up */
#define KIV_ERRBIT_STAGE_CAPACITY 16  /* more host pages in the union than staging pages */

typedef struct kiv_store {
  int32_t batch;
  int32_t num_kv_heads;
  int32_t head_dim;
  int32_t page_size;
  int32_t dtype;            /* KIV_DTYPE_* */
  int32_t shard_rank;
  int32_t shard_count;
  int32_t hot_hint;         /* expected live hot rows (sizes the attention grid); 0: hot_capacity */
  int64_t cold_capacity;    /* token slots of this shard (multiple of page_size) */
  int64_t hot_capacity;     /* ring slots; 0 when the store has no hot ring */
  void *cold_k, *cold_v, *summaries;
  void *hot_k, *hot_v;
  int64_t *state;           /* device, KIV_STATE_WORDS words */
  /* host overflow tier (all zero / NULL: none) */
  int64_t host_capacity;    /* token slots of the pinned host tier (multiple of page_size) */
  void *host_k, *host_v;    /* pinned, device-mapped host memory [B, Hkv, host_capacity, D] */
  int32_t stage_pages;      /* staging pages at the end of the HBM cold slots */
  int32_t flags;            /* KIV_STORE_* */
  /* replicated summaries (KIV_STORE_REPL_SUMMARIES): fp32 running sums of the
   * rows of the page being filled, [B, Hkv, D] */
  float *page_sums;
} kiv_store;

/* kiv_store.flags */
#define KIV_STORE_REPL_SUMMARIES 1
/* With shard_count > 1: every shard keeps the summary of EVERY global page
 * (summaries [B, Hkv, shard_count * (cold_capacity / S + 1), D], indexed by
 * global page), updated by each eviction from the rows it moves (all shards see them:
 * the hot window is replicated) and the running sums in page_sums.  The
 * coarse pass then scores every page on every shard and finds the exact
 * global per-row top pages locally: kiv_coarse_select marks this shard's
 * pages of the global union for the fine pass and no coarse exchange is
 * needed.  Not combined with a host tier. */

typedef struct kiv_query {
  const void *q;            /* [B, Hq, Q, D] store dtype, innermost contiguous */
  int64_t stride_b, stride_h, stride_t;  /* in elements */
  int32_t num_query_heads;
  int32_t query_len;
  float scaling;
  float softcap;            /* 0: no logit soft-capping */
  int32_t top_pages;
  int32_t top_p;
} kiv_query;

typedef struct kiv_mask {
  const float *add;         /* additive mask over hot keys [B, Hm, Q, hot_len] or NULL */
  int64_t stride_b, stride_h, stride_t;  /* elements; stride_h == 0 broadcasts over heads */
  int32_t causal;           /* 1: hot row j visible to query position i iff j <= hot_len - Q + i */
  int32_t reserved;
} kiv_mask;

/* Library identity and errors. */
KIV_API int32_t kiv_abi_version(void);
KIV_API const char *kiv_status_string(kiv_status s);
KIV_API const char *kiv_last_error(void);

/* Bytes of scratch one store needs for queries of this shape (256-byte aligned). */
KIV_API size_t kiv_workspace_bytes(const kiv_store *st, const kiv_query *q);

/* Byte offsets of the workspace sub-buffers, for inspection by the host:
 * out[0] scores (R x np_cap float, coarse scores of the last pass),
 * out[1] page marks (bitmap), out[2] union pages (int32, KIV_ST_UNION valid entries),
 * out[3] fine keys (B x c_cap uint32, order-preserving keys of the max
 * scores), out[4] per-row selected counts (int32 [B]), out[5] attention
 * partials; out[6..9] = R, np_cap, u_cap, c_cap. */
KIV_API kiv_status kiv_workspace_layout(const kiv_store *st, const kiv_query *q, int64_t *out);

/* Zero the device state of a store (stream-ordered). */
KIV_API kiv_status kiv_state_reset(const kiv_store *st, void *stream);

/*
 * Append n_new rows to the hot ring, then evict the oldest
 * max(0, hot_len + n_new - keep) rows of (hot ++ new) into the cold tier
 * (keep == -1: evict nothing; keep == KIV_KEEP_DIRECT: append the new rows
 * straight to the cold tier and leave the hot ring untouched).  Evicted rows
 * are written to their token slots
 * and every page they complete gets its mean-K summary (fp32 sum in token
 * order / page_size, rounded to the store dtype) in the same pass.  The
 * direct mode is the reference's ColdKVStore.evict_from_hot.
 * n_evict_max bounds the rows evicted by this call (sizes the grid).
 * Replaces: kiv/cold_store.py:142-184 (evict_from_hot),
 *           kiv/tiered_cache.py:55-72 (_evict_layer), :107-142 (update).
 */
#define KIV_KEEP_DIRECT (-2)
KIV_API kiv_status kiv_append_evict(const kiv_store *st, const void *k_new, const void *v_new,
                            int64_t stride_b, int64_t stride_h, int64_t stride_t,
                            int32_t n_new, int64_t keep, int64_t n_evict_max, void *stream);

/*
 * Coarse pass: score every finalized page summary of this shard against all
 * B*Hq*Q query rows (the G heads of a KV group read each summary once), take
 * the top min(top_pages, Np) pages per row (score desc, page id asc).
 * shard_count == 1: the union of all rows' pages (sorted) is left in the
 *   workspace for kiv_fine_select, and row_scores/row_pages may be NULL.
 * shard_count > 1: each row's local top list is written to row_scores /
 *   row_pages [R, top_pages] (R = B*Hq*Q; unused tail entries have page -1)
 *   for an all-gather, followed by kiv_coarse_merge -- or, with replicated
 *   summaries, the pages of the global union are marked directly (one bit per
 *   global page; row_scores / row_pages may be NULL; no merge follows).
 * Replaces: kiv/cold_store.py:203-230 (_repeat_kv + matmul, topk, unique).
 */
KIV_API kiv_status kiv_coarse_select(const kiv_store *st, const kiv_query *q, void *ws, size_t ws_bytes,
                             float *row_scores, int32_t *row_pages, void *stream);

/* Merge n_lists gathered per-row page lists into the global per-row top
 * lists and keep, sorted, the union pages this shard owns. */
KIV_API kiv_status kiv_coarse_merge(const kiv_store *st, const kiv_query *q, void *ws, size_t ws_bytes,
                            const float *lists_scores, const int32_t *lists_pages,
                            int32_t n_lists, void *stream);

/*
 * Fine pass: score every token of the union pages plus the partial page
 * (max over all Hq heads and Q positions) and select the top
 * P = min(top_p, cold_len, C) tokens per batch row (score desc, token asc).
 * shard_count == 1: writes the selected global token ids, ascending, to
 *   sel [B, top_p] (and their scores to sel_scores if not NULL).
 * shard_count > 1: writes this shard's local top list instead (score, token;
 *   unused tail entries -1) for an all-gather, followed by kiv_fine_merge.
 * Replaces: kiv/cold_store.py:227-262 (candidate ids), :301, :332-347.
 */
KIV_API kiv_status kiv_fine_select(const kiv_store *st, const kiv_query *q, void *ws, size_t ws_bytes,
                           int32_t *sel, float *sel_scores, void *stream);

/* The two halves of kiv_fine_select, callable separately (timing, pipelining):
 * scoring of every candidate token into the workspace, then the top-P select. */
KIV_API kiv_status kiv_fine_score(const kiv_store *st, const kiv_query *q, void *ws, size_t ws_bytes,
                                  void *stream);
KIV_API kiv_status kiv_fine_topk(const kiv_store *st, const kiv_query *q, void *ws, size_t ws_bytes,
                                 int32_t *sel, float *sel_scores, void *stream);

/* Merge n_lists gathered per-batch token lists [n_lists, B, top_p] into the
 * global top-P of each batch row: sel [B, top_p] gets all of them (ascending
 * ids), sel_local [B, top_p] the ones this shard owns (for kiv_attend). */
KIV_API kiv_status kiv_fine_merge(const kiv_store *st, const kiv_query *q, void *ws, size_t ws_bytes,
                          const float *lists_scores, const int32_t *lists_tokens,
                          int32_t n_lists, int32_t *sel, int32_t *sel_local, void *stream);

/*
 * Gather the K and V rows of the selected tokens: out_k/out_v [B, Hkv, P, D].
 * sel [B, sel_stride] global token ids; rows owned by other shards (and ids
 * < 0) are left untouched.
 * Replaces: kiv/cold_store.py:357-362.
 */
KIV_API kiv_status kiv_gather_rows(const kiv_store *st, const int32_t *sel, int32_t sel_stride,
                           int32_t P, void *out_k, void *out_v, void *stream);

/*
 * Attention over [selected cold ; hot] for all query rows, split-KV with
 * partial (max, sum, out) per split merged by log-sum-exp.  Cold keys are read
 * straight from the token slots named by sel (no gathered copy): the first
 * n_b entries of row b of sel, n_b being the count the preceding
 * kiv_fine_select / kiv_fine_merge left in the workspace.  Hot keys come from
 * the ring (the hot slice hot_slice of hot_slices, for sharded runs).
 * out: [B, Q, Hq, D] in the store dtype (the HF attention-interface layout),
 *   or NULL when partial_out is given.
 * partial_out: [B*Hq*Q, D + 4] fp32 (out[D], max, sum, 2 pad) of this shard,
 *   for an all-gather followed by kiv_attend_merge.
 * Replaces: kiv/middleware.py:330-352 (crop mask, cat cold/hot, extend mask,
 *   original attention) and kiv/mask_utils.py:8-38.
 */
KIV_API kiv_status kiv_attend(const kiv_store *st, const kiv_query *q, const kiv_mask *mask,
                      void *ws, size_t ws_bytes, const int32_t *sel, int32_t sel_stride,
                      int32_t hot_slice, int32_t hot_slices,
                      void *out, float *partial_out, void *stream);

/* Merge n gathered partials [n, R, D + 4] into out [B, Q, Hq, D]. */
KIV_API kiv_status kiv_attend_merge(const kiv_store *st, const kiv_query *q, const float *partials,
                            int32_t n, void *out, void *stream);

/*
 * One single-shard decode layer-step after the cache update:
 * coarse (or reuse when reuse != 0) + fine + attention, in one call.
 * Replaces: kiv/cold_store.py:283-371 + kiv/middleware.py:308-354.
 */
KIV_API kiv_status kiv_retrieve_attend(const kiv_store *st, const kiv_query *q, const kiv_mask *mask,
                               void *ws, size_t ws_bytes, int32_t reuse, int32_t *sel,
                               void *out, void *stream);

/*
 * kiv_retrieve_attend without a workspace argument: the scratch comes from a
 * fixed device array inside the library (KIV_NOALLOC_SCRATCH_BYTES per GPU,
 * held until the process exits), so the call allocates nothing.  For callers
 * that may not allocate device memory while they serve (engines that own all
 * memory through their own pool, plugin hosts without an allocator hook).
 * Shapes needing more scratch are rejected with KIV_ERR_CAPACITY.  All calls
 * on a device share the array, which keeps the last call's contents: every
 * call first clears, on its stream, the part that must start at zero, so a
 * call of another shape or a failed call before it does not matter.  Calls
 * that overlap on the GPU race on the array.  The first call on a device
 * looks up the array's address; make it before any stream capture.
 * No counterpart in the reference (it has no C interface).
 */
#define KIV_NOALLOC_SCRATCH_BYTES (32u << 20)
KIV_API kiv_status kiv_retrieve_attend_noalloc(const kiv_store *st, const kiv_query *q,
                                               const kiv_mask *mask, int32_t *sel, void *out,
                                               void *stream);

/*
 * Peer-memory exchange for sharded runs (one process per GPU of one box).
 * No counterpart in the reference (it has no multi-GPU code); replaces the
 * NCCL all-gathers of the sharded layer-step.
 *
 * Every rank allocates an exchange arena of kiv_exchange_bytes() with
 * kiv_peer_alloc (device memory, zeroed, exported as an IPC handle of
 * KIV_IPC_HANDLE_BYTES), the ranks swap the handles over any host channel,
 * and each rank maps the others' arenas with kiv_peer_open.  The
 * *_exchange_merge calls then store this rank's lists straight into every
 * rank's arena over NVLink as 64-bit words that carry the exchange's flag
 * next to each value (one single-copy atomic store per value), wait for
 * every rank's words to carry the flag (each wait bounded by wait_cycles; a
 * timeout sets KIV_ERRBIT_WAIT_TIMEOUT in the state) and merge, all in one
 * kernel.  Every rank must make the same sequence of these calls
 * with the same shapes.  An arena serves one (store shape, query shape);
 * stores of the same shape may share it when their calls are stream-ordered.
 */
#define KIV_MAX_PEERS 8
#define KIV_IPC_HANDLE_BYTES 64
typedef struct kiv_exchange {
  int32_t world;                  /* ranks (== kiv_store.shard_count), <= KIV_MAX_PEERS */
  int32_t rank;                   /* this rank (== kiv_store.shard_rank) */
  void *arena[KIV_MAX_PEERS];     /* every rank's arena as mapped in this process */
  int64_t arena_bytes;            /* size of every arena */
  int64_t wait_cycles;            /* bound of every wait on a peer, in SM clock cycles;
                                     0: 2^31 (about 1.1 s at 1965 MHz).  A wait that runs
                                     out sets KIV_ERRBIT_WAIT_TIMEOUT and the merge writes
                                     no output (the coarse merge marks no page, the fine
                                     merge selects nothing, the attention merge leaves
                                     `out` as it was) */
} kiv_exchange;

KIV_API size_t kiv_exchange_bytes(const kiv_store *st, const kiv_query *q, int32_t world);
KIV_API kiv_status kiv_peer_alloc(size_t bytes, void **dev_ptr, void *ipc_handle);
KIV_API kiv_status kiv_peer_open(const void *ipc_handle, void **dev_ptr);
KIV_API kiv_status kiv_peer_close(void *dev_ptr);
KIV_API kiv_status kiv_peer_free(void *dev_ptr);
/* IPC handle of the device allocation that contains dev_ptr (any cudaMalloc'd
 * buffer, e.g. a store's cold_k) and dev_ptr's byte offset in it: a peer maps
 * the handle with kiv_peer_open and adds the offset (one open per allocation
 * and process; kiv_peer_close unmaps it). */
KIV_API kiv_status kiv_peer_export(const void *dev_ptr, void *ipc_handle, int64_t *offset);

/* Every shard's cold rows as mapped in this process (index = shard rank; the
 * own entry is the store's cold_k / cold_v).  All shards' stores must have
 * the same cold_capacity. */
typedef struct kiv_peer_rows {
  const void *cold_k[KIV_MAX_PEERS];
  const void *cold_v[KIV_MAX_PEERS];
} kiv_peer_rows;

/* kiv_coarse_merge with the lists exchanged through the arenas: row_scores /
 * row_pages are this rank's lists from kiv_coarse_select. */
KIV_API kiv_status kiv_coarse_exchange_merge(const kiv_store *st, const kiv_query *q, void *ws, size_t ws_bytes,
                                             const float *row_scores, const int32_t *row_pages,
                                             const kiv_exchange *x, void *stream);
/* kiv_fine_merge with the lists exchanged through the arenas: scores /
 * tokens are this rank's lists from kiv_fine_select (or kiv_fine_topk).
 * sel may be NULL when only this shard's selection (sel_local) is needed. */
KIV_API kiv_status kiv_fine_exchange_merge(const kiv_store *st, const kiv_query *q, void *ws, size_t ws_bytes,
                                           const float *scores, const int32_t *tokens, const kiv_exchange *x,
                                           int32_t *sel, int32_t *sel_local, void *stream);
/*
 * Candidate exchange: the fine pass of a page-sharded store with replicated
 * summaries (KIV_STORE_REPL_SUMMARIES) in one scorer and one select, with no
 * list merge.  After kiv_coarse_select every shard holds the whole page union;
 * the scorer scores the union pages this shard owns and stores each key at its
 * global candidate position into every rank's arena, and every rank's select
 * takes the exact global top-P over all candidates (score descending, token id
 * ascending; the same order as kiv_fine_select on one GPU).  sel [B, top_p]
 * gets the global selection on every rank (ascending ids, tail -1).  With
 * sel_local, this shard's rows of it go there (ascending) for kiv_attend +
 * kiv_attend_exchange_merge; with sel_local NULL, kiv_attend_peers reads sel
 * itself.  (The workspace's per-row selected counts follow the list the
 * attention reads.)  A wait that runs out sets KIV_ERRBIT_WAIT_TIMEOUT and
 * selects nothing.
 * Every rank's store must have the same cold_capacity (the candidate
 * positions and the arena layout follow it).
 * kiv_fine_exchange_supported returns 1 when the store and query shapes can use
 * it (16-bit rows, page_size 128, head_dim a multiple of 64 up to 256, at most
 * 16 query rows per KV head, a union of at most 8192 pages, no host tier);
 * otherwise use kiv_fine_score + kiv_fine_topk + kiv_fine_exchange_merge.
 * Replaces, for sharded stores, the reference's fine pass
 * (kiv/cold_store.py:283-371 retrieve_top_kv, steps 2-3).
 */
KIV_API int32_t kiv_fine_exchange_supported(const kiv_store *st, const kiv_query *q);
KIV_API kiv_status kiv_fine_exchange_select(const kiv_store *st, const kiv_query *q, void *ws, size_t ws_bytes,
                                            const kiv_exchange *x, int32_t *sel, int32_t *sel_local,
                                            void *stream);
/* Attention of a page-sharded store over the global selection sel [B,
 * sel_stride] (from kiv_fine_exchange_select with sel_local NULL) and the
 * whole (replicated) hot window: every selected row is read from the cold
 * tier of the shard that owns its page, over NVLink for the other shards'
 * pages, so every rank computes the full output `out` ([B, Q, Hq, D]) with no
 * exchange of partials.  Same arithmetic as kiv_attend on one GPU.  16-bit
 * stores with at most 16 query rows per KV head, head_dim a multiple of 64
 * (<= 256), no host tier.  Replaces, for sharded stores: kiv/middleware.py:
 * 330-352 and kiv/mask_utils.py:8-38. */
KIV_API kiv_status kiv_attend_peers(const kiv_store *st, const kiv_query *q, const kiv_mask *mask, void *ws,
                                    size_t ws_bytes, const int32_t *sel, int32_t sel_stride,
                                    const kiv_peer_rows *peers, void *out, void *stream);
/* kiv_attend_merge with the partials exchanged through the arenas: partial is
 * this rank's [B*Hq*Q, D + 4] from kiv_attend. */
KIV_API kiv_status kiv_attend_exchange_merge(const kiv_store *st, const kiv_query *q, const float *partial,
                                             const kiv_exchange *x, void *out, void *stream);

/* Copy the store's device state words to host memory (synchronizes the stream). */
KIV_API kiv_status kiv_read_state(const kiv_store *st, int64_t *host_words, void *stream);

/* Host overflow tier: pinned host memory mapped into the device address space
 * (UVA), usable as kiv_store.host_k / host_v; freed with kiv_host_free.
 * No reference counterpart (the reference keeps its whole cold tier in host
 * memory, kiv/cold_store.py:92-109). */
KIV_API kiv_status kiv_host_alloc(size_t bytes, void **ptr);
KIV_API kiv_status kiv_host_free(void *ptr);

#ifdef __cplusplus
}
#endif

#endif /* KIV_B200_H */
