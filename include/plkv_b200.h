/*
 * plkv_b200.h -- C ABI of the B200 (sm_100a) paged latent-cache decode library
 * (libplkv_b200.so).
 *
 * Drop-in boundary for the hot path of tatavishnurao/LatentPagedAttention-rs:
 * the FP32 -> FP16 latent-row write through a block table, the direct
 * latent-space decode (scores, active-length mask, stable softmax, latent
 * context, W_v / W_uv projection), the W_o output projection and the FP16
 * full-KV paged GQA baseline.  The reference has no FFI of its own; each entry
 * point cites the reference function (Python oracle and Rust CPU reference)
 * whose argument meaning and error behaviour it keeps.
 *
 * Conventions
 *   - Every pointer is a device pointer to caller-owned memory unless the name
 *     ends in `_host`.  The library allocates no device memory.
 *   - Every launch is stream-ordered on `stream` (a cudaStream_t); no call
 *     synchronises.  Calls are thread-safe.
 *   - Return values are plkv_status codes.  Host-detectable argument errors
 *     return before anything is launched.  Data-dependent errors found on the
 *     device (a non-finite row, a table entry outside the pool) never trap:
 *     the row / block is skipped and a PLKV_FLAG_* bit is OR-ed into the
 *     caller's int32 `err_flags` word (may be NULL), which the caller reads
 *     after the stream work completes.
 *   - FP16 cache data is passed as uint16_t bit patterns (IEEE binary16).
 *   - Offsets into pools are 64-bit; block ids and lengths are int32.
 */
#ifndef PLKV_B200_H
#define PLKV_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* plkv_stream_t; /* same type as cudaStream_t */

/* Status codes.  1-5 mirror PlkvError (crates/plkv-core/src/lib.rs:12-18). */
enum plkv_status {
    PLKV_OK = 0,
    PLKV_ERR_ZERO_VALUE = 1,           /* PlkvError::ZeroValue            lib.rs:13 */
    PLKV_ERR_ARITHMETIC_OVERFLOW = 2,  /* PlkvError::ArithmeticOverflow   lib.rs:14 */
    PLKV_ERR_INVALID_PAGED_LOOKUP = 3, /* PlkvError::InvalidPagedLookup   lib.rs:15 */
    PLKV_ERR_TOKEN_OUT_OF_RANGE = 4,   /* PlkvError::TokenOutOfRange      lib.rs:16 */
    PLKV_ERR_TOKEN_NOT_ALLOCATED = 5,  /* PlkvError::TokenNotAllocated    lib.rs:17 */
    PLKV_ERR_NON_FINITE = 6,           /* "FP16 storage input must be finite" lib.rs:307-311 */
    PLKV_ERR_FP16_OVERFLOW = 7,        /* "FP16 storage conversion overflowed" lib.rs:313-316 */
    PLKV_ERR_INVALID_ARGUMENT = 8,     /* null pointer / unsupported shape */
    PLKV_ERR_WORKSPACE = 9,            /* workspace too small */
    PLKV_ERR_CUDA = 10,                /* a CUDA runtime call failed */
    PLKV_ERR_UNSUPPORTED = 11,         /* mode / shape not built for this device */
};

/* Device-side error flags (OR-ed into *err_flags). */
#define PLKV_FLAG_NON_FINITE_INPUT 0x1 /* row rejected: NaN/Inf input          lib.rs:307-311 */
#define PLKV_FLAG_FP16_OVERFLOW 0x2    /* row rejected: |x| rounds to inf      lib.rs:313-316 */
#define PLKV_FLAG_BAD_BLOCK 0x4        /* table entry outside [0, num_physical) lib.rs:178-182 */
#define PLKV_FLAG_BAD_POSITION 0x8     /* position not covered by the table    lib.rs:171-176 */
#define PLKV_FLAG_BAD_LENGTH 0x10      /* seq_len outside [0, max_blocks*bs]   lib.rs:1106-1111 */
#define PLKV_FLAG_TIMEOUT 0x20         /* a tensor-core pipeline wait gave up (results invalid) */

/* Decode arithmetic. */
#define PLKV_MODE_EXACT_F32 0 /* FP32 CUDA cores: parity mode, 1e-5 relative */
#define PLKV_MODE_TC_F16 1    /* tcgen05 FP16 operands, FP32 TMEM accumulation (~2e-3) */

const char* plkv_status_string(int status);
int plkv_version(void);

/* ------------------------------------------------------------------ storage */

/* FP32 -> FP16 storage bits, round to nearest even.
 * Replaces quantize_f32_to_f16_storage (crates/plkv-core/src/lib.rs:302-319)
 * and fp16_storage_bits (python_ref/latent_paged_attention/cache_ref.py:17-19).
 * Non-finite inputs set PLKV_FLAG_NON_FINITE_INPUT, overflow sets
 * PLKV_FLAG_FP16_OVERFLOW (the output element is still written). */
int plkv_quantize_f16(const float* in, uint16_t* out, int64_t n, int32_t* err_flags,
                      plkv_stream_t stream);

/* Writes one FP32 latent row per request into the FP16 latent cache
 * cache[num_physical, block_size, latent_dim] at the slot of `positions[i]`
 * through the block table of sequence `seq_ids[i]` (seq_ids NULL: i).
 * Replaces paged_latent_write_fp16_storage (lib.rs:889-939) and
 * paged_latent_write_fp16_storage_ref (cache_ref.py:103-114), batched and in
 * place.  A row with any non-finite / overflowing element is not written at
 * all (the reference rejects the whole write).
 * If `seq_lens_inout` is not NULL, positions are taken from it (positions may
 * be NULL) and each successful write increments it: an append. */
int plkv_latent_append_f16(const float* rows, const int32_t* block_tables, int64_t max_blocks,
                           const int32_t* seq_ids, const int32_t* positions,
                           int32_t* seq_lens_inout, int64_t n_rows, uint16_t* cache,
                           int64_t num_physical, int32_t block_size, int32_t latent_dim,
                           int32_t* err_flags, plkv_stream_t stream);

/* Slot-mapped form of the append: slot = physical_block * block_size + offset
 * (negative slots are padding and are skipped).  Same per-row rules. */
int plkv_latent_append_slots_f16(const float* rows, const int64_t* slots, int64_t n_rows,
                                 uint16_t* cache, int64_t num_slots, int32_t latent_dim,
                                 int32_t* err_flags, plkv_stream_t stream);

/* Materialised K / V from latent rows (replaces reconstruct_latent_kv_f32,
 * lib.rs:517-580; reconstruct_latent_kv, latent_kv_reconstruction.rs:4-28;
 * latent_kv_reconstruction_ref, attention_ref.py:227-274):
 *   K[row, kv, d] = sum_{l < latent_dim} latent[row, l] * w_k[kv, l, d]
 *   V[row, kv, d] = sum_{l < value_dim}  latent[row, l] * w_v[kv, l, d]
 * FP32 accumulation.  latent: [num_slots, latent_dim] FP32 or FP16
 * (latent_is_f16); rows: the slots listed in slots[n_rows] (NULL: slots
 * 0 .. n_rows-1; negative slots are skipped); w_k / w_v head-major
 * [kv_heads, latent_dim | value_dim, head_dim] FP32.  K / V are written at the
 * same slot in the head-major paged layout [num_slots / block_size, kv_heads,
 * block_size, head_dim], FP32 or FP16 (out_is_f16); block_size 1 gives the
 * reference's token-major [row, kv_heads, head_dim].  Non-finite inputs or
 * results raise PLKV_FLAG_NON_FINITE_INPUT, FP16 overflow
 * PLKV_FLAG_FP16_OVERFLOW, slots >= num_slots PLKV_FLAG_BAD_POSITION. */
int plkv_reconstruct_kv(const void* latent, int32_t latent_is_f16, int64_t num_slots,
                        int32_t latent_dim, int32_t value_dim, const int64_t* slots,
                        int64_t n_rows, const float* w_k, const float* w_v, int32_t kv_heads,
                        int32_t head_dim, int32_t block_size, void* k_out, void* v_out,
                        int32_t out_is_f16, int32_t* err_flags, plkv_stream_t stream);

/* ---- Split-K result exchange through peer memory (one node, NVLink) ----
 * Replaces the all-gather + plkv_lse_merge of the split-K shards with two
 * kernels over buffers that every rank maps (cudaIpc).  Rank r allocates
 * plkv_peer_buffer_bytes(rows, width) with plkv_peer_alloc, the ranks swap the
 * 64-byte handles (any host channel), and each rank opens the others' with
 * plkv_peer_open; bufs is then a DEVICE array of the W base pointers (own one
 * at index rank) and ctrl a zeroed DEVICE array of 4 uint64 of this rank.
 * Per step: plkv_peer_publish(ctx[rows, width], lse[rows]) after the rank's
 * combine, then plkv_peer_merge(out[rows, width], lse_out[rows] or NULL),
 * which waits (bounded, 1 s: PLKV_FLAG_TIMEOUT, rows 0 and lse -inf, no peer
 * memory read) for every rank's publish of the step and merges them with the
 * LSE rule.  Every rank issues the same sequence of steps with the same rows
 * and width; world <= 32.  Each buffer records its slot capacity at
 * allocation: a step whose rows x width exceeds a buffer is refused on the
 * device with PLKV_FLAG_BAD_POSITION (publish writes nothing, and the merges
 * of that step then time out).  The launch grid may change between steps.
 * Close and free the buffers only after every rank's last merge completed (a
 * host barrier).  plkv_peer_init_buffer prepares caller-allocated device
 * memory of `bytes` the same way (header zeroed, capacity recorded; it
 * synchronises `stream`), for ranks that live in one process. */
typedef struct plkv_ipc_handle {
    char bytes[64];
} plkv_ipc_handle;
size_t plkv_peer_buffer_bytes(int64_t rows, int32_t width);
int plkv_peer_alloc(size_t bytes, void** ptr, plkv_ipc_handle* handle);
int plkv_peer_init_buffer(void* buf, size_t bytes, plkv_stream_t stream);
int plkv_peer_open(const plkv_ipc_handle* handle, void** ptr);
int plkv_peer_close(void* ptr);
int plkv_peer_free(void* ptr);
int plkv_peer_publish(const float* ctx, const float* lse, int64_t rows, int32_t width,
                      void* const* bufs, int32_t world, int32_t rank, uint64_t* ctrl,
                      int32_t* err_flags, plkv_stream_t stream);
int plkv_peer_merge(int64_t rows, int32_t width, void* const* bufs, int32_t world, int32_t rank,
                    uint64_t* ctrl, float* out, float* lse_out, int32_t* err_flags,
                    plkv_stream_t stream);

/* Device-side allocation of new token positions (replaces the bump allocator
 * PagedBlockTable.allocate_token_positions, block_table.py:26-38, and
 * BlockTable::allocate_tokens, lib.rs:1346-1364, for a batch on the GPU).
 * Sequence b gets counts[b] new tokens (counts NULL: one each) at positions
 * seq_lens[b], seq_lens[b]+1, ...; a logical block whose table entry is < 0
 * takes the next physical block of the shared counter *next_block (blocks
 * are handed out in sequence order, then logical order).  Writes the slot
 * (physical * block_size + offset) of every new token to slots[sum(counts)]
 * in sequence order, stores the new blocks in block_tables, advances
 * seq_lens and *next_block.  Blocks past num_physical or past max_blocks are
 * not handed out: their tokens get slot -1 (the slot append skips them) and
 * PLKV_FLAG_BAD_BLOCK / PLKV_FLAG_BAD_POSITION is raised.  Slots past
 * max_slots (the capacity of slots) are not written (PLKV_FLAG_BAD_POSITION).
 * One CTA; stream ordered, no host synchronisation (capturable in a CUDA
 * graph). */
int plkv_allocate_slots(int32_t* block_tables, int64_t max_blocks, int32_t* seq_lens,
                        const int32_t* counts, int32_t batch, int32_t block_size,
                        int32_t* next_block, int64_t num_physical, int64_t* slots,
                        int64_t max_slots, int32_t* err_flags, plkv_stream_t stream);

/* Writes one K row and one V row ([kv_heads, head_dim] FP32 each) per request
 * into FP16 head-major caches [num_physical, kv_heads, block_size, head_dim]
 * (the layout of lib.rs:1232).  Replaces paged_kv_write_f32 (lib.rs:190-247)
 * and paged_kv_write_ref (cache_ref.py:43-73) for the FP16 full-KV baseline. */
int plkv_kv_append_f16(const float* k_rows, const float* v_rows, const int32_t* block_tables,
                       int64_t max_blocks, const int32_t* seq_ids, const int32_t* positions,
                       int32_t* seq_lens_inout, int64_t n_rows, uint16_t* k_cache,
                       uint16_t* v_cache, int64_t num_physical, int32_t kv_heads,
                       int32_t block_size, int32_t head_dim, int32_t* err_flags,
                       plkv_stream_t stream);

/* ---------------------------------------------------------------- planning */

/* One unit of split-K work: tokens [block_begin*bs, min(block_end*bs, len))
 * of sequence `seq`. */
typedef struct plkv_work_item {
    int32_t seq;
    int32_t block_begin;
    int32_t block_end;
    int32_t reserved;
} plkv_work_item;

/* Host-side split planner (no CUDA calls).  Cuts every sequence's blocks into
 * contiguous items of near-equal size so that about `target_items` items
 * cover the batch, none shorter than `min_blocks` blocks.  Items are ordered
 * by sequence; seq_item_begin_host[b]..[b+1] are sequence b's items.  A
 * sequence of length 0 gets one empty item.  Returns PLKV_ERR_WORKSPACE if
 * `max_items` is too small (n_items_host then holds the count needed). */
int plkv_plan_splits(const int32_t* seq_lens_host, int32_t batch, int32_t block_size,
                     int32_t target_items, int32_t min_blocks, plkv_work_item* items_host,
                     int32_t max_items, int32_t* seq_item_begin_host, int32_t* n_items_host);

/* Host-side balanced planner for the persistent tensor-core decode: the
 * blocks of all sequences, in sequence order, are cut into at most
 * `n_workers` contiguous ranges; every (worker, sequence) overlap becomes one
 * item.  A worker's cost is its blocks plus max(1, ceil(256 / block_size))
 * per item (an item reloads the query, refills the pipeline and writes its
 * partial context), and the ranges minimise the largest cost.  Worker w
 * processes items worker_item_begin_host[w] .. [w+1] in order (trailing
 * workers may get none); items are ordered by sequence as for
 * plkv_plan_splits (seq_item_begin_host has batch + 1 entries) and a
 * sequence of length 0 still gets one empty item.  Same return codes. */
int plkv_plan_workers(const int32_t* seq_lens_host, int32_t batch, int32_t block_size,
                      int32_t n_workers, plkv_work_item* items_host, int32_t max_items,
                      int32_t* seq_item_begin_host, int32_t* worker_item_begin_host,
                      int32_t* n_items_host);

/* ------------------------------------------------------------------ decode */

/* Query projection q_lat[b, h, :] = W_k[kv(h)] q[b, h, :] with W_k head-major
 * [kv_heads, latent_dim, head_dim], kv(h) = h / (q_heads / kv_heads).
 * Replaces the `projected` loop of lib.rs:1026-1032 / attention_ref.py:513. */
int plkv_project_query(const float* q, const float* w_k, float* q_lat, int32_t batch,
                       int32_t q_heads, int32_t kv_heads, int32_t head_dim, int32_t latent_dim,
                       plkv_stream_t stream);

/* Arguments of the direct paged latent decode. */
typedef struct plkv_latent_decode_args {
    const float* q_lat;           /* [batch, q_heads, latent_dim] projected / absorbed query */
    const uint16_t* cache;        /* [num_physical, block_size, latent_dim] FP16 */
    int64_t num_physical;
    int32_t block_size;
    int32_t latent_dim;           /* row width used by the scores (e.g. 576) */
    int32_t value_dim;            /* leading columns used by the context (e.g. 512) */
    int32_t batch;
    int32_t q_heads;
    float scale;                  /* 1/sqrt(head_dim) in the reference (lib.rs:1023) */
    const int32_t* block_tables;  /* [batch, max_blocks] physical block ids */
    int64_t max_blocks;
    const int32_t* seq_lens;      /* [batch] active lengths */
    const plkv_work_item* items;  /* [n_items] from a planner, on the device */
    const int32_t* seq_item_begin;/* [batch + 1] on the device */
    int32_t n_items;
    const int32_t* worker_item_begin; /* [n_workers + 1] from plkv_plan_workers, or NULL */
    int32_t n_workers;            /* tensor-core mode: persistent CTA pairs (0: one per item) */
    int32_t allow_empty;          /* 1: a sequence of length 0 yields ctx 0, lse -inf */
    const float* w_v;             /* [proj_heads, value_dim, head_dim] or NULL (latent ctx out) */
    int32_t proj_heads;
    int32_t head_dim;
    float* ctx;                   /* [batch, q_heads, head_dim] (value_dim if w_v == NULL) */
    float* lse;                   /* optional [batch, q_heads]: max + log(sum) of the scores */
    float* scores;                /* optional [batch, q_heads, max_seq_len]; masked = -FLT_MAX */
    float* probs;                 /* optional [batch, q_heads, max_seq_len]; masked = 0 */
    int32_t max_seq_len;
    int32_t mode;                 /* PLKV_MODE_* */
    void* workspace;              /* device memory, 256-byte aligned */
    size_t workspace_bytes;
    int32_t* err_flags;           /* optional */
} plkv_latent_decode_args;

/* Workspace bytes the decode needs for `n_items` items (either mode; it
 * includes the FP16 copy of the query used by the tensor-core mode). */
size_t plkv_latent_decode_workspace_size(int32_t n_items, int32_t batch, int32_t q_heads,
                                         int32_t latent_dim, int32_t value_dim);

/* Direct paged latent decode: split-K partial pass over the work items
 * (scores, active-length mask, online softmax, latent context), then the
 * log-sum-exp combine fused with the W_v / W_uv projection.
 * Replaces direct_paged_latent_gqa_decode_fp16_storage_runtime_f32_accum
 * (lib.rs:1090-1145, core at 941-1088) and
 * direct_paged_latent_gqa_fp16_storage_runtime_intermediates_ref
 * (attention_ref.py:617-648), batched with a table and a length per sequence.
 * Inactive positions come out as score -3.4028234663852886e38 and
 * probability 0 (lib.rs:1130-1140, attention_ref.py:604-609). */
int plkv_latent_decode(const plkv_latent_decode_args* args, plkv_stream_t stream);

/* The two halves of plkv_latent_decode, for callers that schedule them. */
int plkv_latent_decode_partial(const plkv_latent_decode_args* args, plkv_stream_t stream);
int plkv_latent_decode_combine(const plkv_latent_decode_args* args, plkv_stream_t stream);

/* Size of the library's fixed scratch array used by plkv_latent_decode_noalloc. */
#define PLKV_NOALLOC_SCRATCH_BYTES (32u * 1024u * 1024u)

/* plkv_latent_decode for callers that cannot allocate device memory (a plugin
 * host that owns every device byte and passes only inputs and outputs, or a
 * binding with no CUDA allocator).  No counterpart in the reference.
 * args->workspace / workspace_bytes are ignored: the split-K scratch is a
 * file-scope device array of PLKV_NOALLOC_SCRATCH_BYTES that every GPU loading
 * the library holds until exit.  Returns PLKV_ERR_WORKSPACE, launching
 * nothing, when plkv_latent_decode_workspace_size(n_items, batch, q_heads,
 * latent_dim, value_dim) exceeds that size (plan fewer work items).  Calls no cudaMalloc
 * or cudaFree.  The first call on a device looks up the array's device address
 * (cudaGetSymbolAddress) with that device current; make that first call
 * before any stream capture.  All calls share the array, so calls that overlap
 * on the GPU race; it keeps the last call's contents, none of which a later
 * call reads before writing. */
int plkv_latent_decode_noalloc(const plkv_latent_decode_args* args, plkv_stream_t stream);

/* ---- Head-sharded split-K merge through peer memory (one node, NVLink) ----
 * No counterpart in the reference (its decode is single-device).  Under
 * split-K each rank decodes its range of every sequence's blocks with
 * plkv_latent_decode_partial; instead of the combine, plkv_shard_publish
 * merges the rank's work items per (sequence, head) into a normalised latent
 * context and log-sum-exp, stores them into this rank's own buffer and
 * releases this rank's flag in every rank's buffer.  Rank r owns heads
 * [r H/W, (r+1) H/W).  plkv_shard_merge then waits (bounded, 1 s:
 * PLKV_FLAG_TIMEOUT, rows 0 and lse -inf) for every rank's publish of the
 * step, reads the owned heads' rows from every rank's buffer (peer loads),
 * merges the W sources with the LSE rule and applies W_v / W_uv of the owned
 * heads: out[batch, H/W, head_dim] and
 * lse_out[batch, H/W] (may be NULL) hold the merged result of this rank's
 * heads; w_v NULL writes the latent context (width value_dim).  Buffers of
 * plkv_shard_buffer_bytes(batch, q_heads, value_dim) bytes come from
 * plkv_peer_alloc / plkv_peer_open (or plkv_peer_init_buffer) and are used as
 * described for the peer exchange above: bufs a DEVICE array of the W base
 * pointers, ctrl a zeroed DEVICE array of 4 uint64 of this rank, every rank
 * issuing the same steps with the same shapes; q_heads % world == 0; world
 * <= 32.  publish reads args->workspace (the partial pass's
 * results), seq_item_begin, batch, q_heads, latent_dim, value_dim, n_items
 * and err_flags. */
size_t plkv_shard_buffer_bytes(int32_t batch, int32_t q_heads, int32_t value_dim);
int plkv_shard_publish(const plkv_latent_decode_args* args, void* const* bufs, int32_t world,
                       int32_t rank, uint64_t* ctrl, plkv_stream_t stream);
int plkv_shard_merge(void* const* bufs, int32_t world, int32_t rank, uint64_t* ctrl,
                     int32_t batch, int32_t q_heads, int32_t value_dim, const float* w_v,
                     int32_t head_dim, float* out, float* lse_out, int32_t* err_flags,
                     plkv_stream_t stream);

/* Log-sum-exp merge of per-shard results (split-K across GPUs):
 * ctx_shards [n_shards, rows, width] are normalised partial contexts and
 * lse_shards [n_shards, rows] their log-sum-exp (-inf = empty shard).
 * out[rows, width] = sum_s exp(lse_s - M) ctx_s / sum_s exp(lse_s - M). */
int plkv_lse_merge(const float* ctx_shards, const float* lse_shards, int32_t n_shards,
                   int64_t rows, int32_t width, float* out, float* lse_out,
                   plkv_stream_t stream);

/* W_o output projection out[batch, out_dim] = x[batch, in_dim] W_o[in_dim, out_dim]
 * (FP32; extension -- the reference stops at the per-head context).
 * The workspace holds k_splits * batch * out_dim floats. */
size_t plkv_out_proj_workspace_size(int32_t batch, int32_t out_dim, int32_t k_splits);
int plkv_out_proj(const float* x, const float* w_o, float* out, int32_t batch, int32_t in_dim,
                  int32_t out_dim, int32_t k_splits, void* workspace, size_t workspace_bytes,
                  plkv_stream_t stream);

/* W_o output projection on the tensor cores: the same product with tcgen05
 * kind::tf32 MMAs on the FP32 W_o as stored (both operands rounded to TF32,
 * FP32 accumulation; about 1e-3 normwise relative error, against the FP32
 * plkv_out_proj's 1e-6).  Extension, no counterpart in the reference.
 * in_dim % 32 == 0, out_dim % 32 == 0, 1 <= k_splits <= in_dim / 32; x, w_o and
 * the workspace 256-byte aligned; the workspace holds
 * plkv_out_proj_tc_workspace_size(batch, out_dim, k_splits) bytes.  A wait
 * that runs out of time raises PLKV_FLAG_TIMEOUT in *err_flags (may be NULL). */
size_t plkv_out_proj_tc_workspace_size(int32_t batch, int32_t out_dim, int32_t k_splits);
int plkv_out_proj_tc(const float* x, const float* w_o, float* out, int32_t batch, int32_t in_dim,
                     int32_t out_dim, int32_t k_splits, void* workspace, size_t workspace_bytes,
                     int32_t* err_flags, plkv_stream_t stream);

/* ------------------------------------------------------ full-KV baseline */

typedef struct plkv_fullkv_decode_args {
    const float* q;               /* [batch, q_heads, head_dim] */
    const uint16_t* k_cache;      /* [num_physical, kv_heads, block_size, head_dim] FP16 */
    const uint16_t* v_cache;
    int64_t num_physical;
    int32_t kv_heads;
    int32_t block_size;
    int32_t head_dim;
    int32_t batch;
    int32_t q_heads;
    float scale;
    const int32_t* block_tables;
    int64_t max_blocks;
    const int32_t* seq_lens;
    const plkv_work_item* items;
    const int32_t* seq_item_begin;
    int32_t n_items;
    int32_t allow_empty;
    float* ctx;                   /* [batch, q_heads, head_dim] */
    float* lse;
    float* scores;
    float* probs;
    int32_t max_seq_len;
    void* workspace;              /* device memory, 256-byte aligned */
    size_t workspace_bytes;
    int32_t* err_flags;
} plkv_fullkv_decode_args;

size_t plkv_fullkv_decode_workspace_size(int32_t n_items, int32_t batch, int32_t q_heads,
                                         int32_t head_dim);

/* FP16 full-KV paged GQA decode.  Replaces
 * paged_full_kv_gqa_decode_fp16_storage_runtime_f32_accum (lib.rs:1147-1269)
 * and paged_gqa_decode_attention_intermediates_ref (attention_ref.py:172-224)
 * on FP16 storage, batched with a table and a length per sequence.  The K and
 * V caches must be 16-byte aligned (PLKV_ERR_UNSUPPORTED otherwise).
 * head_dim 128 with up to 16 query heads per KV head and no intermediates
 * (scores / probs NULL) runs on the tensor cores with FP32-accurate
 * arithmetic (the FP32 query and probabilities split into two FP16 parts);
 * other shapes (head_dim <= 256, a multiple of 8, up to 8 query heads per KV
 * head) and calls that want intermediates run on the CUDA cores. */
int plkv_fullkv_decode(const plkv_fullkv_decode_args* args, plkv_stream_t stream);

/* ------------------------------------------------------------ diagnostics */

/* Self-test of the bounded waits of the tensor-core decode on this device
 * (no counterpart in the reference).  Two CTAs wait on a barrier that nothing
 * completes: CTA 0 gives up after its 1 s limit, ORs PLKV_FLAG_TIMEOUT into
 * *err_flags and sets *ctl (the launch's abort word, device memory, caller
 * initialised); CTA 1 starts 0.5 s later and gives up as soon as it sees *ctl
 * set.  elapsed_ns[2] (device) receives each wait's duration.  With *ctl = 1
 * on entry both waits end within microseconds and nothing is reported.  No
 * fault or trap is involved; the call returns after about 1 s. */
int plkv_selftest_bounded_wait(int32_t* ctl, int64_t* elapsed_ns, int32_t* err_flags,
                               plkv_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* PLKV_B200_H */
