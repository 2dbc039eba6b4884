// plkv_capi.cu -- extern "C" entry points of libplkv_b200.so.
//
// Host-side validation mirrors the checks of the reference functions each
// entry point replaces (crates/plkv-core/src/lib.rs: require_positive 45-50,
// GQA mapping 962-969, active length 1106-1111); the status codes are the
// PlkvError variants of lib.rs:12-18 (include/plkv_b200.h).
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "plkv_common.cuh"

namespace plkv {
void launch_quantize(const float*, uint16_t*, int64_t, int32_t*, cudaStream_t);
void launch_latent_append(const float*, const int32_t*, int64_t, const int32_t*, const int32_t*,
                          int32_t*, int64_t, uint16_t*, int64_t, int, int, int32_t*, cudaStream_t);
void launch_latent_append_slots(const float*, const int64_t*, int64_t, uint16_t*, int64_t, int,
                                int32_t*, cudaStream_t);
void launch_kv_append(const float*, const float*, const int32_t*, int64_t, const int32_t*,
                      const int32_t*, int32_t*, int64_t, uint16_t*, uint16_t*, int64_t, int, int,
                      int, int32_t*, cudaStream_t);
cudaError_t launch_latent_partial_exact(const plkv_latent_decode_args&, DecodeWorkspace,
                                        cudaStream_t);
cudaError_t launch_latent_partial_tc(const plkv_latent_decode_args&, DecodeWorkspace,
                                     cudaStream_t);
bool tc_supported(const plkv_latent_decode_args&);
bool latent_gqa_tc_supported(const plkv_latent_decode_args&);
cudaError_t launch_latent_partial_gqa_tc(const plkv_latent_decode_args&, DecodeWorkspace,
                                         cudaStream_t);
bool fullkv_tc_supported(const plkv_fullkv_decode_args&);
cudaError_t launch_fullkv_partial_tc(const plkv_fullkv_decode_args&, DecodeWorkspace,
                                     cudaStream_t);
cudaError_t launch_fullkv_partial_exact(const plkv_fullkv_decode_args&, DecodeWorkspace,
                                        cudaStream_t);
cudaError_t launch_project_query(const float*, const float*, float*, int, int, int, int, int,
                                 cudaStream_t);
cudaError_t launch_combine(DecodeWorkspace, const int32_t*, int, int, int, const float*, int, int,
                           float*, float*, cudaStream_t);
cudaError_t launch_finalize(DecodeWorkspace, const int32_t*, int, int, int64_t, float*, float*,
                            int, cudaStream_t);
cudaError_t launch_lse_merge(const float*, const float*, int, int64_t, int, float*, float*,
                             cudaStream_t);
cudaError_t launch_out_proj(const float*, const float*, float*, int, int, int, int, float*,
                            cudaStream_t);
cudaError_t launch_out_proj_tf32(const float*, const float*, float*, int, int, int, int, float*,
                                 int32_t*, int32_t*, cudaStream_t);
}  // namespace plkv

using namespace plkv;

#define PLKV_CUDA_CHECK(expr)                          \
    do {                                               \
        if ((expr) != cudaSuccess) return PLKV_ERR_CUDA; \
    } while (0)

static int cuda_status() { return cudaGetLastError() == cudaSuccess ? PLKV_OK : PLKV_ERR_CUDA; }

extern "C" {

const char* plkv_status_string(int status) {
    switch (status) {
        case PLKV_OK: return "ok";
        case PLKV_ERR_ZERO_VALUE: return "a dimension that must be > 0 is zero";
        case PLKV_ERR_ARITHMETIC_OVERFLOW: return "paged lookup size arithmetic overflowed";
        case PLKV_ERR_INVALID_PAGED_LOOKUP: return "invalid paged lookup";
        case PLKV_ERR_TOKEN_OUT_OF_RANGE: return "token position is out of range";
        case PLKV_ERR_TOKEN_NOT_ALLOCATED: return "token position is not allocated";
        case PLKV_ERR_NON_FINITE: return "FP16 storage input must be finite";
        case PLKV_ERR_FP16_OVERFLOW: return "FP16 storage conversion overflowed";
        case PLKV_ERR_INVALID_ARGUMENT: return "invalid argument";
        case PLKV_ERR_WORKSPACE: return "workspace too small";
        case PLKV_ERR_CUDA: return "CUDA runtime error";
        case PLKV_ERR_UNSUPPORTED: return "unsupported shape or mode";
        default: return "unknown status";
    }
}

int plkv_version(void) { return 100; }

int plkv_quantize_f16(const float* in, uint16_t* out, int64_t n, int32_t* err_flags,
                      plkv_stream_t stream) {
    if (n < 0) return PLKV_ERR_INVALID_ARGUMENT;
    if (n == 0) return PLKV_OK;
    if (!in || !out) return PLKV_ERR_INVALID_ARGUMENT;
    launch_quantize(in, out, n, err_flags, (cudaStream_t)stream);
    return cuda_status();
}

int plkv_latent_append_f16(const float* rows, const int32_t* block_tables, int64_t max_blocks,
                           const int32_t* seq_ids, const int32_t* positions,
                           int32_t* seq_lens_inout, int64_t n_rows, uint16_t* cache,
                           int64_t num_physical, int32_t block_size, int32_t latent_dim,
                           int32_t* err_flags, plkv_stream_t stream) {
    if (block_size <= 0 || latent_dim <= 0 || num_physical <= 0 || max_blocks <= 0)
        return PLKV_ERR_ZERO_VALUE;
    if (n_rows < 0) return PLKV_ERR_INVALID_ARGUMENT;
    if (n_rows == 0) return PLKV_OK;
    if (!rows || !block_tables || !cache || (!positions && !seq_lens_inout))
        return PLKV_ERR_INVALID_ARGUMENT;
    if (n_rows > 0x7fffffff) return PLKV_ERR_ARITHMETIC_OVERFLOW;
    launch_latent_append(rows, block_tables, max_blocks, seq_ids, positions, seq_lens_inout, n_rows,
                         cache, num_physical, block_size, latent_dim, err_flags,
                         (cudaStream_t)stream);
    return cuda_status();
}

int plkv_latent_append_slots_f16(const float* rows, const int64_t* slots, int64_t n_rows,
                                 uint16_t* cache, int64_t num_slots, int32_t latent_dim,
                                 int32_t* err_flags, plkv_stream_t stream) {
    if (latent_dim <= 0 || num_slots <= 0) return PLKV_ERR_ZERO_VALUE;
    if (n_rows < 0) return PLKV_ERR_INVALID_ARGUMENT;
    if (n_rows == 0) return PLKV_OK;
    if (!rows || !slots || !cache) return PLKV_ERR_INVALID_ARGUMENT;
    if (n_rows > 0x7fffffff) return PLKV_ERR_ARITHMETIC_OVERFLOW;
    launch_latent_append_slots(rows, slots, n_rows, cache, num_slots, latent_dim, err_flags,
                               (cudaStream_t)stream);
    return cuda_status();
}

int plkv_kv_append_f16(const float* k_rows, const float* v_rows, const int32_t* block_tables,
                       int64_t max_blocks, const int32_t* seq_ids, const int32_t* positions,
                       int32_t* seq_lens_inout, int64_t n_rows, uint16_t* k_cache,
                       uint16_t* v_cache, int64_t num_physical, int32_t kv_heads,
                       int32_t block_size, int32_t head_dim, int32_t* err_flags,
                       plkv_stream_t stream) {
    if (kv_heads <= 0 || block_size <= 0 || head_dim <= 0 || num_physical <= 0 || max_blocks <= 0)
        return PLKV_ERR_ZERO_VALUE;
    if (n_rows < 0) return PLKV_ERR_INVALID_ARGUMENT;
    if (n_rows == 0) return PLKV_OK;
    if (!k_rows || !v_rows || !block_tables || !k_cache || !v_cache ||
        (!positions && !seq_lens_inout))
        return PLKV_ERR_INVALID_ARGUMENT;
    launch_kv_append(k_rows, v_rows, block_tables, max_blocks, seq_ids, positions, seq_lens_inout,
                     n_rows, k_cache, v_cache, num_physical, kv_heads, block_size, head_dim,
                     err_flags, (cudaStream_t)stream);
    return cuda_status();
}

int plkv_plan_splits(const int32_t* seq_lens_host, int32_t batch, int32_t block_size,
                     int32_t target_items, int32_t min_blocks, plkv_work_item* items_host,
                     int32_t max_items, int32_t* seq_item_begin_host, int32_t* n_items_host) {
    if (batch <= 0 || block_size <= 0) return PLKV_ERR_ZERO_VALUE;
    if (!seq_lens_host || !n_items_host) return PLKV_ERR_INVALID_ARGUMENT;
    if (target_items < batch) target_items = batch;
    if (min_blocks < 1) min_blocks = 1;
    int64_t total_blocks = 0;
    for (int b = 0; b < batch; ++b) {
        if (seq_lens_host[b] < 0) return PLKV_ERR_INVALID_ARGUMENT;
        total_blocks += (seq_lens_host[b] + block_size - 1) / block_size;
    }
    int64_t per_item = (total_blocks + target_items - 1) / target_items;
    if (per_item < min_blocks) per_item = min_blocks;
    // Pass 1: count.
    int64_t n = 0;
    for (int b = 0; b < batch; ++b) {
        int64_t nb = (seq_lens_host[b] + block_size - 1) / block_size;
        n += nb == 0 ? 1 : (nb + per_item - 1) / per_item;
    }
    *n_items_host = (int32_t)n;
    if (n > max_items || !items_host || !seq_item_begin_host) return PLKV_ERR_WORKSPACE;
    // Pass 2: split each sequence's blocks evenly across its items.
    int32_t k = 0;
    for (int b = 0; b < batch; ++b) {
        seq_item_begin_host[b] = k;
        int64_t nb = (seq_lens_host[b] + block_size - 1) / block_size;
        int64_t parts = nb == 0 ? 1 : (nb + per_item - 1) / per_item;
        for (int64_t i = 0; i < parts; ++i) {
            plkv_work_item it;
            it.seq = b;
            it.block_begin = (int32_t)(nb * i / parts);
            it.block_end = (int32_t)(nb * (i + 1) / parts);
            it.reserved = 0;
            items_host[k++] = it;
        }
    }
    seq_item_begin_host[batch] = k;
    return PLKV_OK;
}

int plkv_plan_workers(const int32_t* seq_lens_host, int32_t batch, int32_t block_size,
                      int32_t n_workers, plkv_work_item* items_host, int32_t max_items,
                      int32_t* seq_item_begin_host, int32_t* worker_item_begin_host,
                      int32_t* n_items_host) {
    if (batch <= 0 || block_size <= 0 || n_workers <= 0) return PLKV_ERR_ZERO_VALUE;
    if (!seq_lens_host || !n_items_host) return PLKV_ERR_INVALID_ARGUMENT;
    std::vector<int64_t> nb(batch);
    int64_t total = 0;
    for (int b = 0; b < batch; ++b) {
        if (seq_lens_host[b] < 0) return PLKV_ERR_INVALID_ARGUMENT;
        nb[b] = (seq_lens_host[b] + block_size - 1) / block_size;
        total += nb[b];
    }
    // Cost of a worker = its blocks + kItemCost per item: every item reloads
    // the query, refills the pipeline and writes its partial context (about
    // four 64-token tiles of time on B200).  Sequences are walked in order and
    // each worker is filled up to a makespan T; the smallest T that needs at
    // most n_workers workers is found by bisection (the fill is monotone in T).
    const int64_t item_cost = std::max<int64_t>(1, (256 + block_size - 1) / block_size);
    std::vector<plkv_work_item> items;
    std::vector<int32_t> item_worker;
    std::vector<int32_t> seq_begin(batch + 1, 0);
    auto fill = [&](int64_t T, bool emit) -> int64_t {  // workers used, or n_workers + 1
        int64_t w = 0, used = 0;
        for (int b = 0; b < batch; ++b) {
            if (emit) seq_begin[b] = (int32_t)items.size();
            if (nb[b] == 0) {  // an empty sequence still gets one (empty) item
                if (used > 0 && used + item_cost > T) {
                    ++w;
                    used = 0;
                }
                if (w >= n_workers) return n_workers + 1;
                used += item_cost;
                if (emit) {
                    items.push_back({b, 0, 0, 0});
                    item_worker.push_back((int32_t)w);
                }
                continue;
            }
            int64_t pos = 0;
            while (pos < nb[b]) {
                if (used > 0 && used + item_cost >= T) {
                    ++w;
                    used = 0;
                }
                if (w >= n_workers) return n_workers + 1;
                const int64_t take = std::min(nb[b] - pos, std::max<int64_t>(1, T - used - item_cost));
                if (emit) {
                    items.push_back({b, (int32_t)pos, (int32_t)(pos + take), 0});
                    item_worker.push_back((int32_t)w);
                }
                used += item_cost + take;
                pos += take;
            }
        }
        if (emit) seq_begin[batch] = (int32_t)items.size();
        return w + 1;
    };
    int64_t lo = item_cost + 1, hi = total + item_cost * (int64_t)batch + 1;
    while (lo < hi) {
        const int64_t mid = lo + (hi - lo) / 2;
        if (fill(mid, false) <= n_workers)
            hi = mid;
        else
            lo = mid + 1;
    }
    fill(lo, true);
    *n_items_host = (int32_t)items.size();
    if ((int64_t)items.size() > max_items || !items_host || !seq_item_begin_host ||
        !worker_item_begin_host)
        return PLKV_ERR_WORKSPACE;
    std::copy(items.begin(), items.end(), items_host);
    std::copy(seq_begin.begin(), seq_begin.end(), seq_item_begin_host);
    // Items are in worker order already (workers take consecutive ranges).
    int32_t k = 0;
    for (int32_t ww = 0; ww <= n_workers; ++ww) {
        while (k < (int32_t)items.size() && item_worker[k] < ww) ++k;
        worker_item_begin_host[ww] = k;
    }
    worker_item_begin_host[n_workers] = (int32_t)items.size();
    return PLKV_OK;
}

int plkv_project_query(const float* q, const float* w_k, float* q_lat, int32_t batch,
                       int32_t q_heads, int32_t kv_heads, int32_t head_dim, int32_t latent_dim,
                       plkv_stream_t stream) {
    if (batch <= 0 || q_heads <= 0 || kv_heads <= 0 || head_dim <= 0 || latent_dim <= 0)
        return PLKV_ERR_ZERO_VALUE;
    if (q_heads % kv_heads) return PLKV_ERR_INVALID_PAGED_LOOKUP;  // "invalid GQA mapping"
    if (!q || !w_k || !q_lat) return PLKV_ERR_INVALID_ARGUMENT;
    if (head_dim > 256) return PLKV_ERR_UNSUPPORTED;
    return launch_project_query(q, w_k, q_lat, batch, q_heads, kv_heads, head_dim, latent_dim,
                                (cudaStream_t)stream) == cudaSuccess
               ? PLKV_OK
               : PLKV_ERR_CUDA;
}

size_t plkv_latent_decode_workspace_size(int32_t n_items, int32_t batch, int32_t q_heads,
                                         int32_t latent_dim, int32_t value_dim) {
    if (n_items <= 0 || batch <= 0 || q_heads <= 0 || latent_dim <= 0 || value_dim <= 0) return 0;
    return decode_workspace_bytes(n_items, batch, q_heads, latent_dim, value_dim);
}

static int validate_latent(const plkv_latent_decode_args* a) {
    if (!a) return PLKV_ERR_INVALID_ARGUMENT;
    if (a->batch <= 0 || a->q_heads <= 0 || a->latent_dim <= 0 || a->value_dim <= 0 ||
        a->block_size <= 0 || a->num_physical <= 0 || a->max_blocks <= 0 || a->n_items <= 0)
        return PLKV_ERR_ZERO_VALUE;
    if (!a->q_lat || !a->cache || !a->block_tables || !a->seq_lens || !a->items ||
        !a->seq_item_begin || !a->ctx || !a->workspace)
        return PLKV_ERR_INVALID_ARGUMENT;
    if (a->value_dim > a->latent_dim) return PLKV_ERR_INVALID_ARGUMENT;
    if (a->w_v) {
        if (a->proj_heads <= 0 || a->head_dim <= 0) return PLKV_ERR_ZERO_VALUE;
        if (a->q_heads % a->proj_heads) return PLKV_ERR_INVALID_PAGED_LOOKUP;
    }
    if ((a->scores || a->probs) && a->max_seq_len <= 0) return PLKV_ERR_ZERO_VALUE;
    if (a->probs && !a->scores) return PLKV_ERR_INVALID_ARGUMENT;
    if (a->latent_dim % 8 || a->value_dim % 4 || a->value_dim > 640) return PLKV_ERR_UNSUPPORTED;
    if (a->n_items > 65535) return PLKV_ERR_UNSUPPORTED;  // grid y of the partial pass
    if ((int64_t)a->max_blocks * a->block_size > 0x7fffffffLL) return PLKV_ERR_ARITHMETIC_OVERFLOW;
    if (a->workspace_bytes <
        decode_workspace_bytes(a->n_items, a->batch, a->q_heads, a->latent_dim, a->value_dim))
        return PLKV_ERR_WORKSPACE;
    if (reinterpret_cast<uintptr_t>(a->workspace) & 255) return PLKV_ERR_INVALID_ARGUMENT;
    if (a->n_workers < 0 || (a->n_workers > 0 && !a->worker_item_begin))
        return PLKV_ERR_INVALID_ARGUMENT;
    if (a->mode != PLKV_MODE_EXACT_F32 && a->mode != PLKV_MODE_TC_F16) return PLKV_ERR_UNSUPPORTED;
    return PLKV_OK;
}

int plkv_latent_decode_partial(const plkv_latent_decode_args* a, plkv_stream_t stream) {
    int st = validate_latent(a);
    if (st != PLKV_OK) return st;
    DecodeWorkspace ws = carve_workspace(a->workspace, a->n_items, a->batch, a->q_heads,
                                         a->latent_dim, a->value_dim);
    cudaError_t e;
    if (a->mode == PLKV_MODE_TC_F16) {
        if (!tc_supported(*a)) return PLKV_ERR_UNSUPPORTED;
        e = launch_latent_partial_tc(*a, ws, (cudaStream_t)stream);
    } else if (latent_gqa_tc_supported(*a)) {
        // exact mode, GQA-latent shapes without intermediates: tensor cores
        // with the query and probabilities split into FP16 hi + lo
        e = launch_latent_partial_gqa_tc(*a, ws, (cudaStream_t)stream);
    } else {
        e = launch_latent_partial_exact(*a, ws, (cudaStream_t)stream);
    }
    return e == cudaSuccess ? PLKV_OK : PLKV_ERR_CUDA;
}

int plkv_latent_decode_combine(const plkv_latent_decode_args* a, plkv_stream_t stream) {
    int st = validate_latent(a);
    if (st != PLKV_OK) return st;
    DecodeWorkspace ws = carve_workspace(a->workspace, a->n_items, a->batch, a->q_heads,
                                         a->latent_dim, a->value_dim);
    cudaStream_t s = (cudaStream_t)stream;
    PLKV_CUDA_CHECK(launch_combine(ws, a->seq_item_begin, a->batch, a->q_heads, a->value_dim,
                                   a->w_v, a->proj_heads, a->head_dim, a->ctx, a->lse, s));
    if (a->scores)
        PLKV_CUDA_CHECK(launch_finalize(ws, a->seq_lens, a->batch, a->q_heads,
                                        a->max_blocks * (int64_t)a->block_size, a->scores,
                                        a->probs, a->max_seq_len, s));
    return PLKV_OK;
}

int plkv_latent_decode(const plkv_latent_decode_args* a, plkv_stream_t stream) {
    int st = plkv_latent_decode_partial(a, stream);
    if (st != PLKV_OK) return st;
    return plkv_latent_decode_combine(a, stream);
}

int plkv_lse_merge(const float* ctx_shards, const float* lse_shards, int32_t n_shards,
                   int64_t rows, int32_t width, float* out, float* lse_out,
                   plkv_stream_t stream) {
    if (n_shards <= 0 || rows <= 0 || width <= 0) return PLKV_ERR_ZERO_VALUE;
    if (!ctx_shards || !lse_shards || !out) return PLKV_ERR_INVALID_ARGUMENT;
    return launch_lse_merge(ctx_shards, lse_shards, n_shards, rows, width, out, lse_out,
                            (cudaStream_t)stream) == cudaSuccess
               ? PLKV_OK
               : PLKV_ERR_CUDA;
}

size_t plkv_out_proj_workspace_size(int32_t batch, int32_t out_dim, int32_t k_splits) {
    if (batch <= 0 || out_dim <= 0 || k_splits <= 0) return 0;
    return size_t(k_splits) * batch * out_dim * 4;
}

int plkv_out_proj(const float* x, const float* w_o, float* out, int32_t batch, int32_t in_dim,
                  int32_t out_dim, int32_t k_splits, void* workspace, size_t workspace_bytes,
                  plkv_stream_t stream) {
    if (batch <= 0 || in_dim <= 0 || out_dim <= 0 || k_splits <= 0) return PLKV_ERR_ZERO_VALUE;
    if (!x || !w_o || !out || !workspace) return PLKV_ERR_INVALID_ARGUMENT;
    if (batch > 64) return PLKV_ERR_UNSUPPORTED;
    if (workspace_bytes < plkv_out_proj_workspace_size(batch, out_dim, k_splits))
        return PLKV_ERR_WORKSPACE;
    return launch_out_proj(x, w_o, out, batch, in_dim, out_dim, k_splits,
                           static_cast<float*>(workspace), (cudaStream_t)stream) == cudaSuccess
               ? PLKV_OK
               : PLKV_ERR_CUDA;
}

size_t plkv_out_proj_tc_workspace_size(int32_t batch, int32_t out_dim, int32_t k_splits) {
    if (batch <= 0 || out_dim <= 0 || k_splits <= 0) return 0;
    return 256 + size_t(k_splits) * batch * out_dim * 4;
}

int plkv_out_proj_tc(const float* x, const float* w_o, float* out, int32_t batch, int32_t in_dim,
                     int32_t out_dim, int32_t k_splits, void* workspace, size_t workspace_bytes,
                     int32_t* err_flags, plkv_stream_t stream) {
    if (batch <= 0 || in_dim <= 0 || out_dim <= 0 || k_splits <= 0) return PLKV_ERR_ZERO_VALUE;
    if (!x || !w_o || !out || !workspace) return PLKV_ERR_INVALID_ARGUMENT;
    if (in_dim % 32 || out_dim % 32 || k_splits > in_dim / 32 || batch > 65535 * 128)
        return PLKV_ERR_UNSUPPORTED;
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w_o) |
         reinterpret_cast<uintptr_t>(workspace)) & 255)
        return PLKV_ERR_INVALID_ARGUMENT;
    if (workspace_bytes < plkv_out_proj_tc_workspace_size(batch, out_dim, k_splits))
        return PLKV_ERR_WORKSPACE;
    int32_t* ctl = static_cast<int32_t*>(workspace);
    float* partial = reinterpret_cast<float*>(static_cast<char*>(workspace) + 256);
    return launch_out_proj_tf32(x, w_o, out, batch, in_dim, out_dim, k_splits, partial, ctl,
                                err_flags, (cudaStream_t)stream) == cudaSuccess
               ? PLKV_OK
               : PLKV_ERR_CUDA;
}

size_t plkv_fullkv_decode_workspace_size(int32_t n_items, int32_t batch, int32_t q_heads,
                                         int32_t head_dim) {
    if (n_items <= 0 || batch <= 0 || q_heads <= 0 || head_dim <= 0) return 0;
    return decode_workspace_bytes(n_items, batch, q_heads, 0, head_dim);
}

int plkv_fullkv_decode(const plkv_fullkv_decode_args* a, plkv_stream_t stream) {
    if (!a) return PLKV_ERR_INVALID_ARGUMENT;
    if (a->batch <= 0 || a->q_heads <= 0 || a->kv_heads <= 0 || a->head_dim <= 0 ||
        a->block_size <= 0 || a->num_physical <= 0 || a->max_blocks <= 0 || a->n_items <= 0)
        return PLKV_ERR_ZERO_VALUE;
    if (a->q_heads % a->kv_heads) return PLKV_ERR_INVALID_PAGED_LOOKUP;  // lib.rs:1177-1186
    if (!a->q || !a->k_cache || !a->v_cache || !a->block_tables || !a->seq_lens || !a->items ||
        !a->seq_item_begin || !a->ctx || !a->workspace)
        return PLKV_ERR_INVALID_ARGUMENT;
    if ((a->scores || a->probs) && a->max_seq_len <= 0) return PLKV_ERR_ZERO_VALUE;
    if (a->probs && !a->scores) return PLKV_ERR_INVALID_ARGUMENT;
    // the CUDA-core pass takes up to 8 query heads per KV head, the
    // tensor-core pass (head_dim 128, no intermediates) up to 16
    if (a->head_dim % 8 || a->head_dim > 256 ||
        (a->q_heads / a->kv_heads > 8 && !fullkv_tc_supported(*a)))
        return PLKV_ERR_UNSUPPORTED;
    if ((reinterpret_cast<uintptr_t>(a->k_cache) | reinterpret_cast<uintptr_t>(a->v_cache)) & 15)
        return PLKV_ERR_UNSUPPORTED;  // rows are copied in 16-byte pieces
    if ((int64_t)a->max_blocks * a->block_size > 0x7fffffffLL) return PLKV_ERR_ARITHMETIC_OVERFLOW;
    if (a->workspace_bytes <
        decode_workspace_bytes(a->n_items, a->batch, a->q_heads, 0, a->head_dim))
        return PLKV_ERR_WORKSPACE;
    if (reinterpret_cast<uintptr_t>(a->workspace) & 255) return PLKV_ERR_INVALID_ARGUMENT;
    DecodeWorkspace ws = carve_workspace(a->workspace, a->n_items, a->batch, a->q_heads, 0,
                                         a->head_dim);
    cudaStream_t s = (cudaStream_t)stream;
    // head_dim 128 and <= 16 query heads per KV head without intermediates run
    // on the tensor cores (FP32-accurate: Q and P split into FP16 hi + lo)
    if (fullkv_tc_supported(*a))
        PLKV_CUDA_CHECK(launch_fullkv_partial_tc(*a, ws, s));
    else
        PLKV_CUDA_CHECK(launch_fullkv_partial_exact(*a, ws, s));
    PLKV_CUDA_CHECK(launch_combine(ws, a->seq_item_begin, a->batch, a->q_heads, a->head_dim,
                                   nullptr, a->q_heads, a->head_dim, a->ctx, a->lse, s));
    if (a->scores)
        PLKV_CUDA_CHECK(launch_finalize(ws, a->seq_lens, a->batch, a->q_heads,
                                        a->max_blocks * (int64_t)a->block_size, a->scores,
                                        a->probs, a->max_seq_len, s));
    return PLKV_OK;
}

}  // extern "C"
