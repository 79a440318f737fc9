/*
 * rsllm_kv_cuda.h -- C ABI of the B200 (sm_100a) KV-cache path for rsLLM.
 *
 * This is the boundary a `rsllm-backend-cuda` crate binds with `extern "C"`
 * declarations: plain pointers, sizes and status codes, no C++ or torch types.
 * Every entry point states the rsLLM interface it replaces (path within the
 * rsLLM tree, file:line).
 *
 * Conventions (mirroring rsLLM's kernel conventions, crates/rsllm-backend-cpu/
 * src/lib.rs:43-60 and crates/rsllm-kvcache/src/lib.rs:28-70):
 *   - The caller owns every buffer.  Device pointers are CUDA device memory of
 *     the current device; nothing on a hot path allocates.
 *   - Calls are asynchronous on the given stream.  Errors the host can see
 *     before launch are returned at once; errors found per row on the device
 *     (bad page id, non-finite input) are OR-ed into a caller-provided device
 *     word as (1u << status) and the offending row is skipped -- never a trap.
 *     rkv_status_from_bits() maps such a word to one status.
 *   - A status maps 1:1 onto rsLLM's error variants (see rkv_status below).
 *   - Entry points are thread-safe; a stream must not be shared across threads
 *     without the caller's own ordering, as with any CUDA stream.
 */
#ifndef RSLLM_KV_CUDA_H
#define RSLLM_KV_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define RKV_API __attribute__((visibility("default")))
#else
#define RKV_API
#endif

/* Same type as cudaStream_t / CUstream; NULL is the legacy default stream. */
typedef struct CUstream_st* rkv_stream_t;

/* ---- status codes ------------------------------------------------------ */
typedef int32_t rkv_status;
#define RKV_OK 0
/* rsllm-kvcache Error::ShapeMismatch (crates/rsllm-kvcache/src/lib.rs:31-39)
 * and rsllm-backend-cpu Error::ShapeMismatch (crates/rsllm-backend-cpu/src/error.rs:12). */
#define RKV_ERR_SHAPE_MISMATCH 1
/* Error::IndexOutOfRange (crates/rsllm-kvcache/src/lib.rs:41-50). */
#define RKV_ERR_INDEX_OUT_OF_RANGE 2
/* Error::InvalidLayer (crates/rsllm-kvcache/src/lib.rs:52-59). */
#define RKV_ERR_INVALID_LAYER 3
/* Error::CompressedPoolFull (crates/rsllm-kvcache/src/lib.rs:61-69): the page
 * pool has no free page left. */
#define RKV_ERR_POOL_FULL 4
/* rsllm-backend-cpu Error::NonFiniteInput (crates/rsllm-backend-cpu/src/error.rs:33). */
#define RKV_ERR_NON_FINITE_INPUT 5
/* Null pointer, misaligned pointer or bad handle (Rust's types rule these out;
 * no rsLLM counterpart). */
#define RKV_ERR_INVALID_ARGUMENT 6
/* A CUDA runtime call failed; rkv_last_error() has the message. */
#define RKV_ERR_CUDA 7

/* ---- layout -------------------------------------------------------------
 * A row is one token of one layer: 512 MLA-latent lanes + 64 RoPE lanes
 * (rsLLM's fp8_kv_quantize_row_inplace(row, 576, 64), dsv4_quant.rs:316).
 * Stored form: 512 E4M3FN codes, 8 f32 power-of-two scales (one per 64 lanes),
 * 64 bf16 RoPE lanes.  A page holds 64 rows of one layer as a structure of
 * arrays: codes[64][512] u8 | scales[64][8] f32 | rope[64][64] bf16.
 * A slot is page * 64 + row-in-page. */
#define RKV_PAGE_TOKENS 64
#define RKV_LATENT_DIM 512
#define RKV_ROPE_DIM 64
#define RKV_ROW_DIM 576
#define RKV_BLOCK 64
#define RKV_PAGE_BYTES 43008

/* A pool: n_layers regions of n_pages pages, page p of layer l at
 * base + (l * n_pages + p) * RKV_PAGE_BYTES.  base must be 256-byte aligned. */
typedef struct rkv_pool_view {
  void* base;
  int64_t n_pages;  /* pages per layer; slots are < n_pages * 64 */
  int32_t n_layers;
  int32_t reserved; /* must be 0 */
} rkv_pool_view;

/* ---- utilities ----------------------------------------------------------- */

/* Library version, "major.minor.patch". */
RKV_API const char* rkv_version(void);

/* Message of the last failing call on this host thread ("" if none). */
RKV_API const char* rkv_last_error(void);

/* The data of the last failing call on this host thread, in the fields of
 * rsLLM's error variants (crates/rsllm-kvcache/src/lib.rs:28-70):
 *   SHAPE_MISMATCH     -> ShapeMismatch { what, expected, actual }
 *   INDEX_OUT_OF_RANGE -> IndexOutOfRange { what, idx, len }
 *   INVALID_LAYER      -> InvalidLayer { idx, max }
 *   POOL_FULL          -> CompressedPoolFull { cap } (cap in token rows)
 *   NON_FINITE_INPUT   -> NonFiniteInput(what)
 * A field that does not apply is -1 (what: "").  `row` is the first failing
 * row or entry for errors the device detects (set by the rkv_*_diagnose
 * calls below), else -1.  After a call that succeeded status is RKV_OK. */
typedef struct rkv_err_info {
  int32_t status;
  int32_t reserved;
  char what[48];
  int64_t idx;
  int64_t len;
  int64_t expected;
  int64_t actual;
  int64_t max;
  int64_t cap;
  int64_t row;
} rkv_err_info;
RKV_API rkv_status rkv_last_error_info(rkv_err_info* out);

/* Highest-priority status in a device status word (0 -> RKV_OK).  Priority:
 * INVALID_ARGUMENT, INVALID_LAYER, SHAPE_MISMATCH, INDEX_OUT_OF_RANGE,
 * POOL_FULL, NON_FINITE_INPUT. */
RKV_API rkv_status rkv_status_from_bits(uint32_t bits);

/* Bytes of one page and of a whole pool (n_layers * n_pages pages). */
RKV_API int64_t rkv_pool_bytes(int64_t n_pages, int32_t n_layers);

/* ---- quantize-on-append ---------------------------------------------------
 * Replaces fp8_kv_quantize_row_inplace (crates/rsllm-backend-cpu/src/ops/
 * dsv4_quant.rs:316-362) applied to each appended row, fused with the row
 * append of ThreeTierKvCache::append_layer / RawSwaRing::append
 * (crates/rsllm-kvcache/src/dsv4/three_tier.rs:187-202, swa.rs:73-94), into a
 * paged pool.
 *
 * rows:   bf16 [n_layers_in][n_tokens][576], 32-byte aligned.  Row t of layer
 *         layer0 + i is written to slot slot_mapping[t] of that layer.
 * slot_mapping: int32 [n_tokens], shared by the n_layers_in layers (one page
 *         table serves every layer); a negative slot skips the token.
 * Per row on the device: a slot >= n_pages * 64 sets INDEX_OUT_OF_RANGE, a
 * non-finite latent lane sets NON_FINITE_INPUT; such a row writes nothing.
 * Non-finite RoPE lanes are stored as they are (the reference never reads
 * them, dsv4_quant.rs:865-874).
 * Host errors: INVALID_LAYER if layer0 < 0 or layer0 + n_layers_in > n_layers;
 * INVALID_ARGUMENT for null / misaligned pointers.
 * d_status may be NULL (no per-row reporting). */
RKV_API rkv_status rkv_append_quant_bf16(const rkv_pool_view* pool, int32_t layer0, int32_t n_layers_in,
                                 const uint16_t* rows, int64_t n_tokens, const int32_t* slot_mapping,
                                 uint32_t* d_status, rkv_stream_t stream);

/* rkv_append_quant_bf16 with launch flags (same rsLLM items replaced, same
 * arguments, status rules and stored bytes).  The append is launched with
 * programmatic dependent launch, so it may start while the kernel issued just
 * before it on `stream` is still running; it waits for that kernel before any
 * write.  flags = 0 also waits before reading its inputs (what
 * rkv_append_quant_bf16 does).  RKV_APPEND_INPUTS_READY lets it read `rows`
 * and `slot_mapping` before that wait, overlapping the previous kernel's
 * drain: set it only when no kernel that can still be running when this call
 * starts writes them -- e.g. they came from host copies, from a kernel with a
 * stream synchronisation, event wait or memcpy after it, or are rows a decode
 * step prepared before the previous append.  Other flag bits:
 * INVALID_ARGUMENT. */
#define RKV_APPEND_INPUTS_READY 1u
RKV_API rkv_status rkv_append_quant_bf16_ex(const rkv_pool_view* pool, int32_t layer0, int32_t n_layers_in,
                                            const uint16_t* rows, int64_t n_tokens, const int32_t* slot_mapping,
                                            uint32_t flags, uint32_t* d_status, rkv_stream_t stream);

/* Measurement reference, not a replacement of any rsLLM item: moves exactly
 * the bytes rkv_append_quant_bf16_ex(..., RKV_APPEND_INPUTS_READY, ...) moves
 * -- every row read, 672 B written to its slot's code, scale and RoPE
 * regions -- with the same grid, the same reads before the wait on the
 * previous kernel and the same programmatic dependent launch, but without the
 * codec: it stores bytes of the input row, so the pool rows it writes are NOT
 * valid FP8 rows.  A benchmark times it beside the append to show the
 * append's distance from a plain copy of its own traffic.  Same host errors
 * as the append; no device status. */
RKV_API rkv_status rkv_copy_floor_bf16(const rkv_pool_view* pool, int32_t layer0, int32_t n_layers_in,
                                       const uint16_t* rows, int64_t n_tokens, const int32_t* slot_mapping,
                                       rkv_stream_t stream);

/* The same append for f32 rows, rsLLM's own row type: the arguments, status
 * rules and stored form of rkv_append_quant_bf16, with rows f32
 * [n_layers_in][n_tokens][576] (32-byte aligned).  The block exponent is
 * ceil(log2f(max(amax, 1e-4) / 448)) with the host's log2f, as the reference
 * evaluates it (dsv4_quant.rs:346-355), through the threshold table below; the
 * RoPE lanes are stored rounded to bf16 (nearest even).  Gathered rows equal
 * the reference's f32 round trip rounded to bf16. */
RKV_API rkv_status rkv_append_quant_f32(const rkv_pool_view* pool, int32_t layer0, int32_t n_layers_in,
                                        const float* rows, int64_t n_tokens, const int32_t* slot_mapping,
                                        uint32_t* d_status, rkv_stream_t stream);

/* The table rkv_append_quant_f32 decides the exponent with (no reference
 * counterpart; exposed for testing): for y = RN(max(amax, 1e-4) / 448) with
 * biased exponent b and mantissa m, the exponent is (b - 127) + (m >= out[b]).
 * out[b] is the smallest mantissa at which the host's log2f(y) exceeds b - 127
 * (0x800000 where none does).  Built once per process from log2f. */
RKV_API void rkv_scale_threshold_table(uint32_t out[256]);

/* ---- paged gather + dequant -----------------------------------------------
 * Replaces the chronological row reads RawSwaRing::rows / ::row
 * (crates/rsllm-kvcache/src/dsv4/swa.rs:131-149) and CompressedKvPool::rows
 * (compressed.rs:203-205) over a page table, with the E4M3 decode of
 * dsv4_quant.rs:359 ((sign * e4m3fn_value) * scale), rounded to bf16.
 *
 * page_table: int32 [n_seq][pt_stride], physical page of each 64-token page.
 * cu_seqlens: int32 [n_seq + 1], exclusive prefix sum of sequence lengths;
 *             row t of sequence s goes to out[cu_seqlens[s] + t].
 * max_seq_len: an upper bound of every sequence length (sizes the grid).
 * out:        bf16 [cu_seqlens[n_seq]][576], 32-byte aligned.
 * A page id outside [0, n_pages) sets INDEX_OUT_OF_RANGE and zero-fills the
 * rows it covers. */
RKV_API rkv_status rkv_gather_dequant_bf16(const rkv_pool_view* pool, int32_t layer, const int32_t* page_table,
                                   int64_t pt_stride, const int32_t* cu_seqlens, int32_t n_seq,
                                   int32_t max_seq_len, uint16_t* out, uint32_t* d_status,
                                   rkv_stream_t stream);

/* ---- indexer top-k selection -----------------------------------------------
 * Replaces the selection half of IndexerPool::select_top_k
 * (crates/rsllm-kvcache/src/dsv4/indexer.rs:218-236).  For query q the
 * candidates are keys [0, n_visible[q]) of row q of scores (f32 [n_q][ld]);
 * causal masking is expressed by n_visible.  effective_k = min(k, n_visible[q])
 * indices are written to out_idx[q][0..effective_k) in the reference's order:
 * descending score, ties to the lowest index; NaN and -inf never win, and when
 * fewer than effective_k candidates beat -inf the rest of the effective_k
 * entries are 0 (the reference's repeated index-0 pick).  Entries
 * [effective_k, k) are -1.
 * Limits: 1 <= k <= 4096, n_visible[q] <= ld, n_keys_max >= every n_visible.
 * scores need 4-byte alignment (16-byte alignment and ld % 4 == 0 take the
 * vectorised path). */
RKV_API rkv_status rkv_topk_select_f32(const float* scores, int64_t ld, int32_t n_q, const int32_t* n_visible,
                               int32_t n_keys_max, int32_t k, int32_t* out_idx, rkv_stream_t stream);

/* ---- sparse gather + dequant ----------------------------------------------
 * Replaces the top-k restricted row read of ThreeTierAttention::run_layer
 * (crates/rsllm-models/src/dsv4/attention.rs:549-560: only rows in the
 * selected set are read), over a page table, decoded as in the gather above.
 *
 * idx:          int32 [n_q][k] token positions (e.g. rkv_topk_select_f32
 *               output); a negative entry writes a zero row.
 * seq_of_query: int32 [n_q], the sequence (page-table row) of each query.
 * seq_lens:     int32 [n_seq], to bound-check positions (INDEX_OUT_OF_RANGE,
 *               zero row).
 * out:          bf16 [n_q][k][576], 32-byte aligned. */
RKV_API rkv_status rkv_sparse_gather_dequant_bf16(const rkv_pool_view* pool, int32_t layer,
                                          const int32_t* page_table, int64_t pt_stride,
                                          const int32_t* seq_of_query, const int32_t* seq_lens,
                                          const int32_t* idx, int32_t n_q, int32_t k, uint16_t* out,
                                          uint32_t* d_status, rkv_stream_t stream);

/* ---- data of device-detected errors -----------------------------------------
 * The kernels above report a bad slot, page id or position, or a non-finite
 * row, as a bit of the status word and skip the row.  After seeing such a
 * bit a caller passes the same inputs to the matching call below: it re-runs
 * the kernel's checks on the host over copies of them (synchronous on
 * `stream`; for the error path), in the kernel's row order, and returns the
 * first failure's status, filling `out` (may be NULL) and the thread's last
 * error (rkv_last_error_info) with rsLLM's fields (IndexOutOfRange { what,
 * idx, len }, crates/rsllm-kvcache/src/lib.rs:28-70; NonFiniteInput(what),
 * crates/rsllm-backend-cpu/src/error.rs:33) and `row`, the failing row's
 * index.  RKV_OK (out->status 0) when every row passes.
 *   append:        row = layer_in * n_tokens + token; a slot >= n_pages * 64
 *                  -> what "slot_mapping", idx = slot, len = n_pages * 64; a
 *                  non-finite latent lane -> NON_FINITE_INPUT, what "rows",
 *                  idx = the lane.
 *   gather:        row = the first output row of the bad page; what
 *                  "page_table", idx = page id, len = n_pages.
 *   sparse gather: row = q * k + j; what "seq_of_query" (idx outside
 *                  [0, n_seq)), "idx" (position >= seq_lens, len = seq_len)
 *                  or "page_table" (idx = page id, len = n_pages). */
RKV_API rkv_status rkv_append_diagnose_bf16(const rkv_pool_view* pool, int32_t layer0, int32_t n_layers_in,
                                            const uint16_t* rows, int64_t n_tokens, const int32_t* slot_mapping,
                                            rkv_err_info* out, rkv_stream_t stream);
RKV_API rkv_status rkv_gather_diagnose(const rkv_pool_view* pool, const int32_t* page_table, int64_t pt_stride,
                                       const int32_t* cu_seqlens, int32_t n_seq, rkv_err_info* out,
                                       rkv_stream_t stream);
RKV_API rkv_status rkv_sparse_gather_diagnose(const rkv_pool_view* pool, const int32_t* page_table,
                                              int64_t pt_stride, const int32_t* seq_of_query,
                                              const int32_t* seq_lens, int32_t n_seq, const int32_t* idx,
                                              int32_t n_q, int32_t k, rkv_err_info* out, rkv_stream_t stream);

/* ---- page moves: copy-on-write and compaction -------------------------------
 * No rsLLM implementation exists; the planned design is refcounted shared
 * prefix blocks with a free list (docs/03-HLD.md:363-369) and radix-tree
 * prefix reuse with LRU eviction (docs/03-HLD.md:371-376).
 *
 * rkv_copy_pages: for every layer, page dst[i] <- page src[i], i < n.  The
 * src and dst sets must be disjoint (copy-on-write targets are fresh pages;
 * compaction moves live pages into holes).  Ids outside [0, n_pages) set
 * INDEX_OUT_OF_RANGE and skip that pair. */
RKV_API rkv_status rkv_copy_pages(const rkv_pool_view* pool, const int32_t* src, const int32_t* dst, int64_t n,
                          uint32_t* d_status, rkv_stream_t stream);

/* rkv_remap_pages: page_table[i] <- remap[page_table[i]] for every entry
 * i < n_entries that is >= 0; remap is int32 [n_pages] (identity for pages
 * that did not move).  An entry >= n_pages sets INDEX_OUT_OF_RANGE and is
 * left unchanged. */
RKV_API rkv_status rkv_remap_pages(int32_t* page_table, int64_t n_entries, const int32_t* remap, int64_t n_pages,
                           uint32_t* d_status, rkv_stream_t stream);

/* ---- paged pool: allocator, page tables, radix prefix store ------------------
 * The host side of rsLLM's planned paged KV cache and radix-tree prefix cache
 * (docs/03-HLD.md:363-376; crates/rsllm-kvcache/src/lib.rs:9-13 lists them as
 * future layouts).  Rules, all deterministic:
 *   - a new page is the lowest-numbered free page;
 *   - sequences share prefix pages by refcount (fork, prefix match); writing
 *     into a partially filled last page that is shared first copies it to a
 *     fresh page (copy-on-write, enqueued on the caller's stream);
 *   - eviction drops released sequences and radix leaves in increasing
 *     (last use, sequences before nodes, id) order until enough pages are
 *     free;
 *   - compaction moves the highest live page into the lowest hole until all
 *     live pages sit below the live-page count, on the device, and rewrites
 *     every host page table (and, optionally, a device table).
 * A pool is single-owner: calls on one pool must not overlap, and its device
 * work must go to one stream (or be ordered by the caller).  Pool calls are
 * not capturable in CUDA graphs (they upload page lists from host memory).
 * Errors: an unknown sequence or a length past a sequence's end is
 * INDEX_OUT_OF_RANGE; not enough free pages is POOL_FULL and changes nothing. */
typedef struct rkv_pool rkv_pool;

/* rkv_pool_desc.device for a plan-only pool: no device memory; the page moves
 * it decides (copy-on-write copies, compaction moves) are handed to the
 * caller by rkv_pool_take_moves instead of being enqueued. */
#define RKV_PLAN_ONLY (-1)

typedef struct rkv_pool_desc {
  int64_t n_pages;   /* pages per layer */
  int32_t n_layers;
  int32_t device;    /* CUDA device ordinal, or RKV_PLAN_ONLY */
  void* storage;     /* optional caller-owned device memory of rkv_pool_bytes() bytes, 256-byte
                        aligned; NULL: the pool allocates it at creation */
} rkv_pool_desc;

typedef struct rkv_pool_stats {
  int64_t free_pages, live_pages, sequences, prefix_nodes, tick, high_water;
} rkv_pool_stats;

/* Create / destroy (allocation happens here only, never on a hot path). */
RKV_API rkv_status rkv_pool_create(const rkv_pool_desc* desc, rkv_pool** out);
RKV_API void rkv_pool_destroy(rkv_pool* pool);
RKV_API rkv_status rkv_pool_get_view(const rkv_pool* pool, rkv_pool_view* out);
RKV_API rkv_status rkv_pool_get_stats(const rkv_pool* pool, rkv_pool_stats* out);
/* Refcount of every page (int32 [n_pages]); 0 = free. */
RKV_API rkv_status rkv_page_refcount(const rkv_pool* pool, int32_t* out, int64_t cap);

/* Sequences (rsLLM's per-session block table, HLD 8.1). */
RKV_API rkv_status rkv_seq_create(rkv_pool* pool, int64_t* seq);
/* New sequence sharing the first n_tokens of parent (its pages refcounted). */
RKV_API rkv_status rkv_seq_fork(rkv_pool* pool, int64_t parent, int64_t n_tokens, int64_t* child);
/* Reserves n_tokens[i] more positions at the end of each seqs[i] (distinct
 * sequences): copy-on-write of a shared partial last page, new pages for the
 * rest; writes the slots of the new positions, sequence after sequence, to
 * slots (may be NULL).  All-or-nothing: POOL_FULL changes nothing.  The
 * copy-on-write copies are enqueued on stream before the call returns; write
 * the new rows on the same stream after it (rkv_append_quant_bf16). */
RKV_API rkv_status rkv_seq_reserve(rkv_pool* pool, int64_t n_seqs, const int64_t* seqs, const int64_t* n_tokens,
                                   int32_t* slots, rkv_stream_t stream);
/* Marks a finished sequence evictable (it keeps its pages until evicted). */
RKV_API rkv_status rkv_seq_release(rkv_pool* pool, int64_t seq);
/* Records a use for LRU. */
RKV_API rkv_status rkv_seq_touch(rkv_pool* pool, int64_t seq);
/* Drops a sequence now (ThreeTierKvCache::clear analogue, three_tier.rs:229). */
RKV_API rkv_status rkv_seq_free(rkv_pool* pool, int64_t seq);
RKV_API rkv_status rkv_seq_info(const rkv_pool* pool, int64_t seq, int64_t* len, int64_t* n_pages);
/* The sequence's page table (int32, one entry per 64 tokens). */
RKV_API rkv_status rkv_seq_page_table(const rkv_pool* pool, int64_t seq, int32_t* out, int64_t cap);

/* Radix prefix store (HLD 8.2).  Insert the first n tokens of seq (their
 * pages are refcounted by the tree); match returns the longest stored prefix
 * of tokens as a new sequence of that length sharing its pages. */
RKV_API rkv_status rkv_prefix_insert(rkv_pool* pool, const int32_t* tokens, int64_t n, int64_t seq);
RKV_API rkv_status rkv_prefix_match(rkv_pool* pool, const int32_t* tokens, int64_t n, int64_t* matched,
                                    int64_t* seq_out);

/* LRU eviction until target_pages pages were freed (or nothing is evictable). */
RKV_API rkv_status rkv_pool_evict(rkv_pool* pool, int64_t target_pages, int64_t* freed);
/* Compaction: page moves enqueued on stream (rkv_copy_pages); if d_tables is
 * given, its n_entries page ids are remapped on the device after the moves. */
RKV_API rkv_status rkv_pool_compact(rkv_pool* pool, int32_t* d_tables, int64_t n_entries, int64_t* moved,
                                    rkv_stream_t stream);
/* old page -> new page of the last compaction (identity before any). */
RKV_API rkv_status rkv_pool_last_remap(const rkv_pool* pool, int32_t* out, int64_t cap);
/* Plan-only pools: returns and clears the page moves decided so far, in order
 * (dst[i] <- src[i]; apply them in order).  *n = count; 0 for device pools.
 * With src == dst == NULL it only reports the count. */
RKV_API rkv_status rkv_pool_take_moves(rkv_pool* pool, int32_t* src, int32_t* dst, int64_t cap, int64_t* n);
/* Reads and clears the status bits of the pool's own device work (syncs). */
RKV_API rkv_status rkv_pool_device_status(rkv_pool* pool, uint32_t* bits);

/* ---- KVC on-disk format ---------------------------------------------------
 * Prefix persistence after rsLLM's plan (docs/03-HLD.md:242-282; rsLLM has
 * no implementation yet): the first n_tokens tokens of a pooled sequence,
 * every layer, in file <dir>/<SHA1 of the token ids as little-endian u32>.kvc.
 * Layout: a 48-byte header ("KVC", version 1, quant_bits 8, reason,
 * token_count, ctx_size, created_at, payload_bytes, 4 zero bytes), the
 * rendered text (u32 length + bytes), the engine payload ("DSV4" magic,
 * version 1, vocab_size, n_layers, head_dim 576, page_tokens 64, n_pages,
 * token ids, then every page of every layer as stored; rows past n_tokens are
 * zero).  All integers little-endian. */
#define RKV_KVC_HEADER_BYTES 48
#define RKV_KVC_COLD 0
#define RKV_KVC_CONTINUED 1
#define RKV_KVC_EVICT 2
#define RKV_KVC_SHUTDOWN 3
typedef struct rkv_kvc_header {
  uint32_t version, quant_bits, reason, reserved;
  uint64_t token_count, ctx_size, created_at, payload_bytes;
} rkv_kvc_header;
/* out: the 40 hex digits of SHA1(token ids) followed by ".kvc" and a NUL. */
RKV_API rkv_status rkv_kvc_name(const int32_t* token_ids, int64_t n_tokens, char out[46]);
RKV_API rkv_status rkv_kvc_read_header(const char* path, rkv_kvc_header* out);
/* Writes the file (through <name>.part, renamed when complete) and returns
 * its path in path_out (may be NULL).  Synchronises stream.  Errors:
 * SHAPE_MISMATCH if the sequence holds fewer than n_tokens tokens;
 * INVALID_ARGUMENT for IO failures or a plan-only pool. */
RKV_API rkv_status rkv_kvc_save(rkv_pool* pool, int64_t seq, const int32_t* token_ids, int64_t n_tokens,
                                uint32_t reason, uint32_t vocab_size, const char* text, int64_t text_len,
                                const char* dir, char* path_out, int64_t path_cap, rkv_stream_t stream);
/* Creates a sequence holding the file's tokens (POOL_FULL if the pool has no
 * room), uploads its pages, optionally registers it in the radix prefix store
 * (rkv_prefix_insert), and returns it in seq_out; token_ids_out (capacity
 * cap, may be NULL) receives the token ids and n_tokens_out their count.
 * SHAPE_MISMATCH if the file's layer count or row layout differs from the
 * pool's. */
RKV_API rkv_status rkv_kvc_load(rkv_pool* pool, const char* path, int32_t* token_ids_out, int64_t cap,
                                int64_t* n_tokens_out, int64_t* seq_out, int32_t insert_prefix, rkv_stream_t stream);

/* ---- page moves without allocation -----------------------------------------
 * No counterpart in rsLLM: an addition of this library for callers that cannot
 * allocate device memory -- an engine that reserves all of its device memory
 * at start-up and hands it out through its own allocator, or the owner of a
 * plan-only pool (RKV_PLAN_ONLY) moving its pages with memory it already has.
 * rkv_pool_compact stages its move lists in memory the pool allocated; this
 * entry point allocates nothing (no cudaMalloc, cudaFree or allocating library
 * call).  It stages the moves in a fixed array inside the library -- a 2 MB
 * __device__ array that every GPU which loads the library holds until the
 * process exits -- then copies page src[i] to dst[i] in every layer and, if
 * d_tables is given, rewrites its n_entries page ids (an id equal to src[i]
 * becomes dst[i]).
 * src: host int32 [n_moves], strictly ascending; dst: host int32 [n_moves],
 * no destination also a source and no page the destination of two moves
 * (the moves of one compaction, e.g. from rkv_pool_last_remap or
 * rkv_pool_take_moves, sorted by source); a list that breaks either rule is
 * INVALID_ARGUMENT and nothing is queued.  The call reads src and dst on the
 * host and queues their copy to the device on `stream`: pageable arrays may
 * be reused when the call returns, but pinned (page-locked) arrays are read
 * by that copy later, so keep them unchanged until the stream has passed the
 * call.  At most RKV_STATIC_MAX_MOVES moves per call: more is
 * SHAPE_MISMATCH.
 * The first call on a device looks up the array's device address with that
 * device current (once per device); make that first call before any stream
 * capture.  Every call shares the array and leaves its contents behind; calls
 * whose device work overlaps (other streams, other threads) race on it, so
 * order them on one stream. */
#define RKV_STATIC_MAX_MOVES 262144
RKV_API rkv_status rkv_apply_page_moves_static(const rkv_pool_view* pool, const int32_t* src, const int32_t* dst,
                                               int64_t n_moves, int32_t* d_tables, int64_t n_entries,
                                               uint32_t* d_status, rkv_stream_t stream);

/* ---- MLA decode attention over the FP8 pages -------------------------------
 * Replaces the per-token attention read of rsLLM's mixed sweep
 * (crates/rsllm-models/src/dsv4/attention.rs:493-663) -- logits over the
 * cached rows, softmax with the per-head sink as a value-less virtual key,
 * weighted sum of the rows -- for one query position per entry of q, reading
 * the FP8 pages directly (no bf16 copy of the rows is written).
 *
 * q:            bf16 [n_q][64 heads][576], 16-byte aligned; query qi belongs to
 *               sequence seq_of_query[qi] (int32 [n_q]).
 * keys:         idx == NULL: every row [0, seq_lens[seq]) of the sequence
 *               (page_table [n_seq][pt_stride], one entry per 64 rows);
 *               idx != NULL: the rows whose positions appear in idx [n_q][k]
 *               (the sparse mask of attention.rs:548-556): entries outside
 *               [0, seq_len) are ignored and a repeated 0 counts once (the
 *               top-k selection's fill value, indexer.rs:222-235).
 * logit:        (q_h . row) * softmax_scale over the 576 stored lanes (latent
 *               dequantised exactly, RoPE lanes as stored).
 * sinks:        f32 [64] or NULL (no sink).
 * out:          f32 [n_q][64][512] = softmax-weighted sum of the 512 latent
 *               lanes, 16-byte aligned; a head with no key and no sink, or a
 *               zero denominator, gives zeros (attention.rs:618-641).
 * n_splits:     dense only: the rows of a sequence are cut into n_splits page
 *               ranges processed in parallel and merged through workspace
 *               (rkv_mla_decode_workspace_bytes(n_q, n_splits) bytes, 16-byte
 *               aligned; may be NULL when n_splits == 1).  One CTA runs per
 *               (query, split) on each SM: choose n_splits so that
 *               n_q * n_splits ends in a nearly full wave of the GPU's SMs,
 *               as few as that allows (each split writes and the merge
 *               reads 64 x 512 f32 partials); 9 for 64 queries on 148 SMs.
 * Device status: a page id outside the pool sets INDEX_OUT_OF_RANGE (that
 * row is skipped); RKV_ERR_CUDA means a device-side wait timed out.
 * Numerics: P = exp2(...) is rounded to bf16 before the tensor-core product
 * (relative 2^-9 per weight), logits and sums are f32. */
RKV_API int64_t rkv_mla_decode_workspace_bytes(int32_t n_q, int32_t n_splits);
RKV_API rkv_status rkv_mla_decode_fp8(const rkv_pool_view* pool, int32_t layer, const int32_t* page_table,
                                      int64_t pt_stride, const int32_t* seq_lens, const int32_t* seq_of_query,
                                      const uint16_t* q, int32_t n_q, const int32_t* idx, int32_t k,
                                      const float* sinks, float softmax_scale, int32_t n_splits, void* workspace,
                                      float* out, uint32_t* d_status, rkv_stream_t stream);

/* ---- page staging --------------------------------------------------------
 * Contiguous copies of a page list (no rsLLM counterpart; the building block
 * of host offload and of the KVC file format below).  pages: device int32
 * [n]; the buffer is device memory of n_layers * n * RKV_PAGE_BYTES bytes laid
 * out [layer][i][page bytes], 16-byte aligned.  pack: buffer <- pages of
 * layers [layer0, layer0 + n_layers); unpack: pages <- buffer.  A page id
 * outside the pool sets INDEX_OUT_OF_RANGE and that page is skipped. */
RKV_API rkv_status rkv_pack_pages(const rkv_pool_view* pool, int32_t layer0, int32_t n_layers, const int32_t* pages,
                                  int64_t n, void* dst, uint32_t* d_status, rkv_stream_t stream);
RKV_API rkv_status rkv_unpack_pages(const rkv_pool_view* pool, int32_t layer0, int32_t n_layers,
                                    const int32_t* pages, int64_t n, const void* src, uint32_t* d_status,
                                    rkv_stream_t stream);

/* ---- compressor emission: aggregate, RMSNorm, RoPE, quantize-on-append -----
 * Replaces the per-token pool step of rsLLM's compressor
 * (crates/rsllm-models/src/dsv4/compressor.rs:264-357 after the two
 * projections: APE bias, CompressedKvPool::accumulate_wide and maybe_emit
 * (crates/rsllm-kvcache/src/dsv4/compressed.rs:310-417), the per-dimension
 * softmax aggregate (:481-554), RMSNorm with an f64 sum of squares, the YaRN
 * RoPE of the 64 tail lanes at position pos + 1 - ratio
 * (crates/rsllm-backend-cpu/src/ops/rope.rs:128-172 with
 * compress_rope_params, compressor.rs:372-397) and
 * fp8_kv_quantize_row_inplace(row, 576, 64)) for a batch of tokens, writing
 * each emitted row into the pool in the stored format.
 *
 * Rows are 576 lanes (512 latent + 64 RoPE); coff = 2 for ratio 4 (two lanes
 * per token: p = columns [0, 576), c = [576, 1152)) and 1 otherwise;
 * width = coff * 576.  A token at position pos writes its row into the state
 * of its sequence; when (pos + 1) % ratio == 0 it emits compressed row
 * k = (pos + 1) / ratio - 1 from the window's c lanes (positions
 * pos + 1 - ratio .. pos) and, for coff 2, the p lanes of the window before it
 * (positions before 0 read as kv 0, score -inf: a fresh state).  This equals
 * rsLLM's streaming state machine whenever its window counter equals
 * pos % ratio (streaming decode, or after finish_prefill_state).
 *
 * states:        device f32, n_states * rkv_compress_state_bytes(ratio) bytes:
 *                per state the last coff * ratio rows of kv, then of score
 *                (as given, without APE: the APE row is added when a row is
 *                read, so every call on these states must pass the same ape),
 *                [2][coff*ratio][width], row = pos % (coff*ratio).  Written by
 *                this call for the last coff * ratio tokens of each state; no
 *                initialisation is needed.
 * kv, score:     device f32 [n_tok][width] (the compressor projections),
 *                16-byte aligned.  The tokens of one state must appear in
 *                consecutive entries at consecutive positions, in order, and
 *                continue the positions of the previous call for that state.
 * pos, state_of_token, emit_slot: device int32 [n_tok]; emit_slot is the pool
 *                slot (page * 64 + row) of the row a token emits, -1 to drop it.
 * ape:           device f32 [ratio][width] (read at pos % ratio), or NULL.
 * norm:          device f32 [576] RMSNorm weight.
 * rope_table:    device f32 [rope_rows][32][2] from rkv_compress_rope_table.
 * Device status: an out-of-range state, position or RoPE row, or an emit slot
 * outside the pool sets INDEX_OUT_OF_RANGE (that token is skipped); an
 * emitted row with a non-finite latent lane sets NON_FINITE_INPUT and is not
 * written (rsLLM returns that error from the quantizer, remapped to
 * ShapeMismatch by compressor.rs:351-356).
 * Numerics: every f32 and f64 operation is rsLLM's, in its order and rounding
 * (no contraction), and exp is glibc's expf, so emitted rows are bit-exact. */
RKV_API int64_t rkv_compress_state_bytes(int32_t ratio);
/* Host: cos/sin * mscale of the 32 RoPE pairs of compressed rows k = 0 ..
 * n_rows - 1 (position k * ratio), out f32 [n_rows][32][2] (host memory),
 * computed with the host's libm exactly as rope.rs:128-172 does. */
RKV_API rkv_status rkv_compress_rope_table(int32_t ratio, int64_t n_rows, float* out);
/* Builds the expf correction table of this process and uploads it to the
 * current device (done by the first rkv_compress_append otherwise; call it
 * before capturing a CUDA graph). */
RKV_API rkv_status rkv_compress_prepare(void);
/* Test hook, no rsLLM counterpart: one thread waits, with the compressor
 * kernel's bounded wait, on a barrier nothing arrives on; after the limit
 * (1 s) it sets RKV_ERR_CUDA in the device status word and the kernel
 * returns.  Shows that a stalled wait ends in a status, not a hang. */
RKV_API rkv_status rkv_compress_wait_probe(uint32_t* d_status, rkv_stream_t stream);
RKV_API rkv_status rkv_compress_append(const rkv_pool_view* pool, int32_t layer, int32_t ratio, float* states,
                                       int64_t n_states, const float* kv, const float* score, int64_t n_tok,
                                       const int32_t* pos, const int32_t* state_of_token, const int32_t* emit_slot,
                                       const float* ape, const float* norm, const float* rope_table,
                                       int64_t rope_rows, uint32_t* d_status, rkv_stream_t stream);
/* The indexer pool's compressor step.  rsLLM runs compressor_decode_one a
 * second time per token on its indexer pool (crates/rsllm-models/src/dsv4/
 * attention.rs:405-429, head_dim 128): the same APE bias, window state,
 * per-dimension softmax aggregate, RMSNorm (f64 sum of squares) and RoPE of
 * the last 64 lanes as rkv_compress_append, on 128-lane rows (width =
 * coff * 128), then a Hadamard + FP4 QAT of the row (compressor.rs:343-348)
 * that this library does not restate.  Emitted rows are written as f32 to
 * out_rows[emit_row[t]] (f32 [n_out_rows][128], e.g. the packed indexer rows
 * rkv_indexer_scores_f32 reads; < 0 drops the row).  states:
 * rkv_indexer_compress_state_bytes(ratio) bytes per state, same rules as
 * rkv_compress_append; ape [ratio][width] or NULL; norm [128]; rope_table as
 * for rkv_compress_append (the rotation does not depend on the row width).
 * Device status: an out-of-range state, position, RoPE row or emit row sets
 * INDEX_OUT_OF_RANGE and skips the token.  Bit-exact with rsLLM's f32/f64
 * arithmetic up to the QAT step. */
RKV_API int64_t rkv_indexer_compress_state_bytes(int32_t ratio);
RKV_API rkv_status rkv_indexer_compress_append(int32_t ratio, float* states, int64_t n_states, const float* kv,
                                               const float* score, int64_t n_tok, const int32_t* pos,
                                               const int32_t* state_of_token, const int32_t* emit_row,
                                               const float* ape, const float* norm, const float* rope_table,
                                               int64_t rope_rows, float* out_rows, int64_t n_out_rows,
                                               uint32_t* d_status, rkv_stream_t stream);
/* rkv_compress_append with launch flags (same rsLLM items, arguments, status
 * rules and pool bytes).  The emission kernel is launched with programmatic
 * dependent launch and may start while the kernel issued just before it on
 * `stream` is still running.
 *   RKV_COMPRESS_INPUTS_READY: pos, state_of_token, emit_slot, ape, norm and
 *     rope_table are not written by any kernel that can still be running when
 *     this call starts (e.g. static per-step metadata and weight tables); the
 *     kernel reads them, resolves each window's rows and stages the APE table
 *     before waiting for that kernel.  kv, score and the states are still read
 *     only after the wait.
 *   RKV_COMPRESS_ONE_TOKEN_PER_STATE: no state has more than one token in the
 *     call (a decode step): the emission kernel writes every ring row and the
 *     second launch (deferred ring writes) is skipped.  A call that breaks
 *     this sets INVALID_ARGUMENT in the device status word (the affected ring
 *     rows are then not written).
 * Other flag bits: INVALID_ARGUMENT. */
#define RKV_COMPRESS_INPUTS_READY 1u
#define RKV_COMPRESS_ONE_TOKEN_PER_STATE 2u
RKV_API rkv_status rkv_compress_append_ex(const rkv_pool_view* pool, int32_t layer, int32_t ratio, float* states,
                                          int64_t n_states, const float* kv, const float* score, int64_t n_tok,
                                          const int32_t* pos, const int32_t* state_of_token,
                                          const int32_t* emit_slot, const float* ape, const float* norm,
                                          const float* rope_table, int64_t rope_rows, uint32_t flags,
                                          uint32_t* d_status, rkv_stream_t stream);
/* expf as the compressor kernel evaluates it, on the host (host != 0, x and
 * out host memory) or on the current device (x, out device memory): a
 * double-precision exp rounded to f32, corrected from a table wherever the
 * host's expf rounds differently.  Domain: x <= 0, -inf and NaN (the
 * aggregate's x = score - max); x > 0 is outside it.  Exposed to check it
 * against expf. */
RKV_API rkv_status rkv_compress_expf(const float* x, float* out, int64_t n, int32_t host, rkv_stream_t stream);
/* Number of table entries (x whose expf differs from the rounded double). */
RKV_API int64_t rkv_compress_expf_table_size(void);

/* ---- indexer scoring + top-k ----------------------------------------------------
 * Replaces the scoring half of IndexerPool::select_top_k
 * (crates/rsllm-kvcache/src/dsv4/indexer.rs:198-216): for query q and each
 * visible compressed indexer row c of its sequence,
 *   score[c] = sum over heads h (in order) of relu(dot(row_c, q_h)) * w_h,
 *   dot = sum over the 128 lanes (in order) of row_c[i] * q_h[i],
 * with f32 products and sums rounded one at a time (no contraction), as rsLLM
 * computes them -- so scores and the selection are bit-exact.
 *
 * rows:       device f32 [*][128]: the indexer rows of sequence s start at row
 *             row_start[s] (int64 [n_seq]) and number seq_rows[s] (int32).
 * q:          device f32 [n_q][64][128] (the rotated, QAT'd indexer queries).
 * w:          device f32 [n_q][64] (per-head weights, already scaled by
 *             1/sqrt(64 * 128) as attention.rs does).
 * seq_of_query, n_visible: device int32 [n_q]: query q scores rows
 *             [0, n_visible[q]) of its sequence (n_visible <= seq_rows).
 * scores:     device f32 [n_q][ld], 16-byte aligned, ld % 4 == 0 and
 *             ld >= max_visible >= every n_visible; entries past n_visible
 *             are left untouched.
 * rows, q: 16-byte aligned.  A query whose sequence or n_visible is out of
 * range sets INDEX_OUT_OF_RANGE and scores nothing. */
RKV_API rkv_status rkv_indexer_scores_f32(const float* rows, const int64_t* row_start, const int32_t* seq_rows,
                                          int64_t n_seq, const float* q, const float* w,
                                          const int32_t* seq_of_query, const int32_t* n_visible, int32_t n_q,
                                          int32_t max_visible, float* scores, int64_t ld, uint32_t* d_status,
                                          rkv_stream_t stream);
/* The whole IndexerPool::select_top_k (indexer.rs:169-236) for a batch of
 * queries: rkv_indexer_scores_f32 into the caller's scores workspace, then
 * rkv_topk_select_f32 (effective_k = min(k, n_visible), the reference's order
 * and fill rules) into out_idx [n_q][k]. */
RKV_API rkv_status rkv_indexer_topk_f32(const float* rows, const int64_t* row_start, const int32_t* seq_rows,
                                        int64_t n_seq, const float* q, const float* w, const int32_t* seq_of_query,
                                        const int32_t* n_visible, int32_t n_q, int32_t max_visible, int32_t k,
                                        float* scores, int64_t ld, int32_t* out_idx, uint32_t* d_status,
                                        rkv_stream_t stream);

/* ---- codec pin ---------------------------------------------------------------
 * out[i] = E4M3 code the append kernel stores for the f32 lane value whose
 * bit pattern is first_bits + i (already divided by its block scale), i < n:
 * the device side of e4m3fn_dequant (dsv4_quant.rs:128-163) with the code byte
 * sign(x < 0) | index.  Used to check the device codec exhaustively. */
RKV_API rkv_status rkv_e4m3fn_code_range(uint32_t first_bits, int64_t n, uint8_t* out, rkv_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* RSLLM_KV_CUDA_H */
