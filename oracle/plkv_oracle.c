/*
 * plkv_oracle.c -- CPU oracle for the paged latent-cache decode path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker, never the product:
 * only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load
 * the shared library built from it.  The CUDA library never links it.
 *
 * It is a C restatement of the Rust CPU reference of
 * tatavishnurao/LatentPagedAttention-rs (crates/plkv-core/src/lib.rs), which
 * cannot be built here (no Rust toolchain).  Each function keeps the
 * reference's loop order and FP32 accumulation ("faithful" mode) so that it
 * reproduces the reference's rounding; an FP64-accumulating mode of the same
 * loops gives the truth that kernel tolerances are measured against.
 *
 *   plkv_or_f32_to_f16_bits      half 2.7.1 `f16::from_f32` (round to nearest
 *                                even), used by quantize_f32_to_f16_storage
 *                                lib.rs:302-319 and numpy astype(float16) in
 *                                python_ref/.../cache_ref.py:6-19
 *   plkv_or_quantize_f16         lib.rs:302-319
 *   plkv_or_resolve_location     lib.rs:164-188, cache_ref.py:22-40
 *   plkv_or_latent_write_f16     lib.rs:889-939
 *   plkv_or_kv_write_f16         lib.rs:190-247 with FP16 head-major storage
 *                                (layout of lib.rs:1232)
 *   plkv_or_project_query        lib.rs:1026-1032
 *   plkv_or_latent_decode_seq    lib.rs:941-1145 (direct paged latent decode,
 *                                FP16 storage, runtime active length)
 *   plkv_or_fullkv_decode_seq    lib.rs:1147-1269
 *   plkv_or_latent_decode_batch  per-sequence tables / lengths over a batch,
 *                                OpenMP over (sequence, head); extension
 *   plkv_or_fullkv_decode_batch  same for the full-KV baseline
 *   plkv_or_out_proj             W_o output projection (extension; plain
 *                                matrix product)
 *   plkv_or_reconstruct_kv       lib.rs:517-580 (reconstruct_latent_kv_f32):
 *                                materialised K / V from latent rows
 *
 * Status codes are the PLKV_* values of include/plkv_b200.h.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

enum {
    OR_OK = 0,
    OR_ZERO_VALUE = 1,
    OR_ARITHMETIC_OVERFLOW = 2,
    OR_INVALID_PAGED_LOOKUP = 3,
    OR_TOKEN_OUT_OF_RANGE = 4,
    OR_TOKEN_NOT_ALLOCATED = 5,
    OR_NON_FINITE = 6,
    OR_FP16_OVERFLOW = 7,
    OR_INVALID_ARGUMENT = 8,
};

/* ---------------------------------------------------------------- FP16 */

/* IEEE binary32 -> binary16, round to nearest, ties to even.  Overflow gives
 * +-inf, NaN stays NaN (quiet).  Written from the IEEE 754 definition. */
uint16_t plkv_or_f32_to_f16_bits(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t exp = (x >> 23) & 0xffu;
    uint32_t man = x & 0x7fffffu;
    if (exp == 0xffu) {
        return (uint16_t)(sign | 0x7c00u | (man ? (0x200u | (man >> 13)) : 0u));
    }
    int e = (int)exp - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        uint32_t m = man | 0x800000u;
        int shift = 14 - e;
        uint32_t h = m >> shift;
        uint32_t rem = m & ((1u << shift) - 1u);
        uint32_t halfway = 1u << (shift - 1);
        if (rem > halfway || (rem == halfway && (h & 1u))) h++;
        return (uint16_t)(sign | h);
    }
    uint32_t h = sign | ((uint32_t)e << 10) | (man >> 13);
    uint32_t rem = man & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
    return (uint16_t)h;
}

float plkv_or_f16_bits_to_f32(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t exp = ((uint32_t)h >> 10) & 0x1fu;
    uint32_t man = (uint32_t)h & 0x3ffu;
    if (exp == 0) {
        float v = (float)man * 5.9604644775390625e-8f; /* 2^-24, exact */
        return sign ? -v : v;
    }
    uint32_t x;
    if (exp == 31) x = sign | 0x7f800000u | (man << 13);
    else x = sign | ((exp - 15u + 127u) << 23) | (man << 13);
    float f;
    memcpy(&f, &x, 4);
    return f;
}

static int f16_is_finite(uint16_t h) { return (h & 0x7c00u) != 0x7c00u; }

/* lib.rs:302-319: reject non-finite input, reject overflow to inf. */
int plkv_or_quantize_f16(const float* in, int64_t n, uint16_t* out) {
    for (int64_t i = 0; i < n; ++i) {
        if (!isfinite(in[i])) return OR_NON_FINITE;
        uint16_t h = plkv_or_f32_to_f16_bits(in[i]);
        if (!f16_is_finite(h)) return OR_FP16_OVERFLOW;
        out[i] = h;
    }
    return OR_OK;
}

/* ------------------------------------------------------------ addressing */

/* lib.rs:164-188 (block table of physical ids, token position, block size).
 * out[0] = logical block, out[1] = physical block, out[2] = offset. */
int plkv_or_resolve_location(const int64_t* table, int64_t ntable, int64_t pos,
                             int64_t block_size, int64_t num_physical, int64_t out[3]) {
    if (block_size <= 0 || num_physical <= 0) return OR_ZERO_VALUE;
    if (pos < 0) return OR_INVALID_ARGUMENT;
    int64_t logical = pos / block_size;
    if (logical >= ntable) return OR_INVALID_PAGED_LOOKUP;
    int64_t phys = table[logical];
    if (phys < 0 || phys >= num_physical) return OR_INVALID_PAGED_LOOKUP;
    out[0] = logical;
    out[1] = phys;
    out[2] = pos % block_size;
    return OR_OK;
}

/* lib.rs:889-939: quantize the new row, require a finite cache, write one
 * row of [P, block_size, latent_dim] FP16 storage in place. */
int plkv_or_latent_write_f16(uint16_t* cache, int64_t num_physical, int64_t block_size,
                             int64_t latent_dim, const int64_t* table, int64_t ntable,
                             int64_t pos, const float* new_row) {
    if (block_size <= 0 || latent_dim <= 0 || num_physical <= 0) return OR_ZERO_VALUE;
    uint16_t* row = (uint16_t*)malloc((size_t)latent_dim * sizeof(uint16_t));
    if (!row) return OR_INVALID_ARGUMENT;
    int st = plkv_or_quantize_f16(new_row, latent_dim, row);
    if (st != OR_OK) { free(row); return st; }
    int64_t n = num_physical * block_size * latent_dim;
    for (int64_t i = 0; i < n; ++i) {
        if (!f16_is_finite(cache[i])) { free(row); return OR_NON_FINITE; }
    }
    int64_t loc[3];
    st = plkv_or_resolve_location(table, ntable, pos, block_size, num_physical, loc);
    if (st != OR_OK) { free(row); return st; }
    memcpy(cache + (loc[1] * block_size + loc[2]) * latent_dim, row,
           (size_t)latent_dim * sizeof(uint16_t));
    free(row);
    return OR_OK;
}

/* lib.rs:190-247 restated for FP16 storage in the head-major layout
 * [P, kv_heads, block_size, head_dim] of lib.rs:1232.  new_k / new_v are
 * [kv_heads, head_dim] FP32 rows. */
int plkv_or_kv_write_f16(uint16_t* k_cache, uint16_t* v_cache, int64_t num_physical,
                         int64_t kv_heads, int64_t block_size, int64_t head_dim,
                         const int64_t* table, int64_t ntable, int64_t pos,
                         const float* new_k, const float* new_v) {
    if (kv_heads <= 0 || head_dim <= 0) return OR_ZERO_VALUE;
    int64_t width = kv_heads * head_dim;
    uint16_t* kq = (uint16_t*)malloc((size_t)width * 2 * sizeof(uint16_t));
    if (!kq) return OR_INVALID_ARGUMENT;
    uint16_t* vq = kq + width;
    int st = plkv_or_quantize_f16(new_k, width, kq);
    if (st == OR_OK) st = plkv_or_quantize_f16(new_v, width, vq);
    int64_t loc[3];
    if (st == OR_OK) st = plkv_or_resolve_location(table, ntable, pos, block_size, num_physical, loc);
    if (st == OR_OK) {
        for (int64_t g = 0; g < kv_heads; ++g) {
            int64_t base = ((loc[1] * kv_heads + g) * block_size + loc[2]) * head_dim;
            memcpy(k_cache + base, kq + g * head_dim, (size_t)head_dim * 2);
            memcpy(v_cache + base, vq + g * head_dim, (size_t)head_dim * 2);
        }
    }
    free(kq);
    return st;
}

/* lib.rs:1026-1032: projected[l] = sum_d q[h, d] * W_k[(l * kv + kv_head) * D + d]
 * for every query head; W_k is the canonical [latent, kv_heads, head_dim]. */
int plkv_or_project_query(const float* q, const float* w_k, int64_t q_heads, int64_t kv_heads,
                          int64_t head_dim, int64_t latent_dim, float* q_lat) {
    if (q_heads <= 0 || kv_heads <= 0 || head_dim <= 0 || latent_dim <= 0) return OR_ZERO_VALUE;
    if (q_heads % kv_heads) return OR_INVALID_PAGED_LOOKUP;
    int64_t group = q_heads / kv_heads;
    for (int64_t h = 0; h < q_heads; ++h) {
        int64_t kv = h / group;
        for (int64_t l = 0; l < latent_dim; ++l) {
            float acc = 0.0f;
            for (int64_t d = 0; d < head_dim; ++d)
                acc += q[h * head_dim + d] * w_k[(l * kv_heads + kv) * head_dim + d];
            q_lat[h * latent_dim + l] = acc;
        }
    }
    return OR_OK;
}

/* ---------------------------------------------------------- decode core */

/* One (sequence, query head) of the direct paged latent decode, lib.rs:1033-1071:
 *   score[t] = (sum_l f32(L[t, l]) * q_lat[l]) * scale            t < active
 *   p = exp(score - max) / sum
 *   c_lat[l] = sum_t p[t] * f32(L[t, l])                           l < value_dim
 *   ctx[d]   = sum_l c_lat[l] * W_v[(l * proj_heads + ph) * D + d]
 * TYPE is float (faithful) or double (truth). */
#define OR_DEFINE_LATENT_HEAD(NAME, TYPE)                                                  \
    static void NAME(const float* q_lat, const uint16_t* cache, int64_t block_size,        \
                     int64_t latent_dim, int64_t value_dim, const int32_t* table,          \
                     int64_t active, float scale, const float* w_v, int64_t proj_heads,    \
                     int64_t ph, int64_t head_dim, TYPE* s, float* scores_row,             \
                     float* probs_row, float* ctx_lat_row, float* ctx_row, TYPE* clat) {   \
        for (int64_t t = 0; t < active; ++t) {                                             \
            const uint16_t* row =                                                          \
                cache + ((int64_t)table[t / block_size] * block_size + t % block_size) *  \
                            latent_dim;                                                    \
            TYPE acc = 0;                                                                  \
            for (int64_t l = 0; l < latent_dim; ++l)                                       \
                acc += (TYPE)plkv_or_f16_bits_to_f32(row[l]) * (TYPE)q_lat[l];             \
            s[t] = acc * (TYPE)scale;                                                      \
        }                                                                                  \
        TYPE mx = -INFINITY;                                                               \
        for (int64_t t = 0; t < active; ++t) mx = s[t] > mx ? s[t] : mx;                   \
        TYPE den = 0;                                                                      \
        if (scores_row)                                                                    \
            for (int64_t t = 0; t < active; ++t) scores_row[t] = (float)s[t];              \
        for (int64_t t = 0; t < active; ++t) {                                             \
            TYPE e = (sizeof(TYPE) == 4) ? (TYPE)expf((float)(s[t] - mx)) : (TYPE)exp((double)(s[t] - mx)); \
            s[t] = e;                                                                      \
            den += e;                                                                      \
        }                                                                                  \
        for (int64_t t = 0; t < active; ++t) s[t] /= den;                                  \
        if (probs_row)                                                                     \
            for (int64_t t = 0; t < active; ++t) probs_row[t] = (float)s[t];               \
        for (int64_t l = 0; l < value_dim; ++l) clat[l] = 0;                               \
        for (int64_t t = 0; t < active; ++t) {                                             \
            const uint16_t* row =                                                          \
                cache + ((int64_t)table[t / block_size] * block_size + t % block_size) *  \
                            latent_dim;                                                    \
            for (int64_t l = 0; l < value_dim; ++l)                                        \
                clat[l] += s[t] * (TYPE)plkv_or_f16_bits_to_f32(row[l]);                   \
        }                                                                                  \
        if (ctx_lat_row)                                                                   \
            for (int64_t l = 0; l < value_dim; ++l) ctx_lat_row[l] = (float)clat[l];       \
        if (ctx_row && w_v) {                                                              \
            for (int64_t d = 0; d < head_dim; ++d) {                                       \
                TYPE acc = 0;                                                              \
                for (int64_t l = 0; l < value_dim; ++l)                                    \
                    acc += clat[l] * (TYPE)w_v[(l * proj_heads + ph) * head_dim + d];      \
                ctx_row[d] = (float)acc;                                                   \
            }                                                                              \
        }                                                                                  \
    }

OR_DEFINE_LATENT_HEAD(latent_head_f32, float)
OR_DEFINE_LATENT_HEAD(latent_head_f64, double)

static int validate_table(const int32_t* table, int64_t ntable, int64_t active,
                          int64_t block_size, int64_t num_physical) {
    if (ntable * block_size < active) return OR_INVALID_PAGED_LOOKUP;
    int64_t used = (active + block_size - 1) / block_size;
    for (int64_t i = 0; i < used; ++i)
        if (table[i] < 0 || table[i] >= num_physical) return OR_INVALID_PAGED_LOOKUP;
    return OR_OK;
}

/* Direct paged latent decode for one sequence, lib.rs:941-1145.
 *   q_lat    [q_heads, latent_dim]      projected (absorbed) query
 *   cache    [num_physical, block_size, latent_dim] FP16 bits
 *   table    [ntable] int32 physical block ids
 *   w_v      canonical [value_dim, proj_heads, head_dim] or NULL
 *   scores / probs [q_heads, max_len] or NULL: active part as computed,
 *   inactive scores = -FLT_MAX and probs = 0 (lib.rs:1130-1140)
 *   ctx_lat  [q_heads, value_dim] or NULL;  ctx [q_heads, head_dim] or NULL
 *   head_begin/head_end restrict the heads computed (others untouched). */
int plkv_or_latent_decode_seq(const float* q_lat, const uint16_t* cache, int64_t num_physical,
                              int64_t block_size, int64_t latent_dim, int64_t value_dim,
                              const int32_t* table, int64_t ntable, int64_t active,
                              int64_t max_len, int64_t q_heads, float scale, const float* w_v,
                              int64_t proj_heads, int64_t head_dim, float* scores, float* probs,
                              float* ctx_lat, float* ctx, int64_t head_begin, int64_t head_end,
                              int acc64) {
    if (q_heads <= 0 || latent_dim <= 0 || block_size <= 0 || num_physical <= 0 || active <= 0)
        return OR_ZERO_VALUE;
    if (active > max_len) return OR_INVALID_PAGED_LOOKUP;
    if (value_dim <= 0 || value_dim > latent_dim) return OR_INVALID_ARGUMENT;
    if (w_v && (proj_heads <= 0 || q_heads % proj_heads || head_dim <= 0)) return OR_INVALID_PAGED_LOOKUP;
    int st = validate_table(table, ntable, active, block_size, num_physical);
    if (st != OR_OK) return st;
    if (head_begin < 0) head_begin = 0;
    if (head_end <= 0 || head_end > q_heads) head_end = q_heads;
    int64_t group = w_v ? q_heads / proj_heads : 1;
    double* s = (double*)malloc((size_t)active * sizeof(double));
    double* clat = (double*)malloc((size_t)value_dim * sizeof(double));
    if (!s || !clat) { free(s); free(clat); return OR_INVALID_ARGUMENT; }
    for (int64_t h = head_begin; h < head_end; ++h) {
        float* srow = scores ? scores + h * max_len : NULL;
        float* prow = probs ? probs + h * max_len : NULL;
        if (acc64)
            latent_head_f64(q_lat + h * latent_dim, cache, block_size, latent_dim, value_dim, table,
                            active, scale, w_v, proj_heads, h / group, head_dim, s, srow, prow,
                            ctx_lat ? ctx_lat + h * value_dim : NULL,
                            ctx ? ctx + h * head_dim : NULL, clat);
        else
            latent_head_f32(q_lat + h * latent_dim, cache, block_size, latent_dim, value_dim, table,
                            active, scale, w_v, proj_heads, h / group, head_dim, (float*)s, srow,
                            prow, ctx_lat ? ctx_lat + h * value_dim : NULL,
                            ctx ? ctx + h * head_dim : NULL, (float*)clat);
        for (int64_t t = active; t < max_len; ++t) {
            if (srow) srow[t] = -3.4028234663852886e38f;
            if (prow) prow[t] = 0.0f;
        }
    }
    free(s);
    free(clat);
    return OR_OK;
}

/* One (sequence, query head) of the FP16 full-KV paged GQA baseline,
 * lib.rs:1222-1263.  K/V are head-major [P, kv_heads, block_size, head_dim]. */
#define OR_DEFINE_FULLKV_HEAD(NAME, TYPE)                                                  \
    static void NAME(const float* qh, const uint16_t* k, const uint16_t* v,                \
                     int64_t kv_heads, int64_t kv, int64_t block_size, int64_t head_dim,   \
                     const int32_t* table, int64_t active, float scale, TYPE* s,           \
                     float* scores_row, float* probs_row, float* ctx_row, TYPE* acc_ctx) { \
        for (int64_t t = 0; t < active; ++t) {                                             \
            int64_t base = (((int64_t)table[t / block_size] * kv_heads + kv) * block_size +\
                            t % block_size) * head_dim;                                    \
            TYPE dot = 0;                                                                  \
            for (int64_t d = 0; d < head_dim; ++d)                                         \
                dot += (TYPE)qh[d] * (TYPE)plkv_or_f16_bits_to_f32(k[base + d]);           \
            s[t] = dot * (TYPE)scale;                                                      \
        }                                                                                  \
        TYPE mx = -INFINITY;                                                               \
        for (int64_t t = 0; t < active; ++t) mx = s[t] > mx ? s[t] : mx;                   \
        if (scores_row)                                                                    \
            for (int64_t t = 0; t < active; ++t) scores_row[t] = (float)s[t];              \
        TYPE den = 0;                                                                      \
        for (int64_t t = 0; t < active; ++t) {                                             \
            TYPE e = (sizeof(TYPE) == 4) ? (TYPE)expf((float)(s[t] - mx)) : (TYPE)exp((double)(s[t] - mx)); \
            s[t] = e;                                                                      \
            den += e;                                                                      \
        }                                                                                  \
        for (int64_t t = 0; t < active; ++t) s[t] /= den;                                  \
        if (probs_row)                                                                     \
            for (int64_t t = 0; t < active; ++t) probs_row[t] = (float)s[t];               \
        for (int64_t d = 0; d < head_dim; ++d) acc_ctx[d] = 0;                             \
        for (int64_t t = 0; t < active; ++t) {                                             \
            int64_t base = (((int64_t)table[t / block_size] * kv_heads + kv) * block_size +\
                            t % block_size) * head_dim;                                    \
            for (int64_t d = 0; d < head_dim; ++d)                                         \
                acc_ctx[d] += s[t] * (TYPE)plkv_or_f16_bits_to_f32(v[base + d]);           \
        }                                                                                  \
        for (int64_t d = 0; d < head_dim; ++d) ctx_row[d] = (float)acc_ctx[d];             \
    }

OR_DEFINE_FULLKV_HEAD(fullkv_head_f32, float)
OR_DEFINE_FULLKV_HEAD(fullkv_head_f64, double)

/* FP16 full-KV paged GQA decode for one sequence, lib.rs:1147-1269. */
int plkv_or_fullkv_decode_seq(const float* q, const uint16_t* k, const uint16_t* v,
                              int64_t num_physical, int64_t kv_heads, int64_t block_size,
                              int64_t head_dim, const int32_t* table, int64_t ntable,
                              int64_t active, int64_t max_len, int64_t q_heads, float scale,
                              float* scores, float* probs, float* ctx, int64_t head_begin,
                              int64_t head_end, int acc64) {
    if (q_heads <= 0 || kv_heads <= 0 || head_dim <= 0 || block_size <= 0 || num_physical <= 0 ||
        active <= 0 || max_len <= 0)
        return OR_ZERO_VALUE;
    if (active > max_len) return OR_INVALID_PAGED_LOOKUP;
    if (q_heads % kv_heads) return OR_INVALID_PAGED_LOOKUP;
    int st = validate_table(table, ntable, active, block_size, num_physical);
    if (st != OR_OK) return st;
    if (head_begin < 0) head_begin = 0;
    if (head_end <= 0 || head_end > q_heads) head_end = q_heads;
    int64_t group = q_heads / kv_heads;
    double* s = (double*)malloc((size_t)active * sizeof(double));
    double* acc = (double*)malloc((size_t)head_dim * sizeof(double));
    if (!s || !acc) { free(s); free(acc); return OR_INVALID_ARGUMENT; }
    for (int64_t h = head_begin; h < head_end; ++h) {
        float* srow = scores ? scores + h * max_len : NULL;
        float* prow = probs ? probs + h * max_len : NULL;
        if (acc64)
            fullkv_head_f64(q + h * head_dim, k, v, kv_heads, h / group, block_size, head_dim, table,
                            active, scale, s, srow, prow, ctx + h * head_dim, acc);
        else
            fullkv_head_f32(q + h * head_dim, k, v, kv_heads, h / group, block_size, head_dim, table,
                            active, scale, (float*)s, srow, prow, ctx + h * head_dim, (float*)acc);
        for (int64_t t = active; t < max_len; ++t) {
            if (srow) srow[t] = -3.4028234663852886e38f;
            if (prow) prow[t] = 0.0f;
        }
    }
    free(s);
    free(acc);
    return OR_OK;
}

/* ------------------------------------------------------------ batches */

/* Batched direct paged latent decode with a table and an active length per
 * sequence (extension of lib.rs:1090-1145, which shares one table).
 *   q_lat  [batch, q_heads, latent_dim];  tables [batch, max_blocks] int32;
 *   lens [batch];  w_v canonical [value_dim, proj_heads, head_dim];
 *   ctx [batch, q_heads, head_dim].  Work is split over (sequence, head)
 *   pairs across `threads` OpenMP threads (0 = all). */
int plkv_or_latent_decode_batch(const float* q_lat, const uint16_t* cache, int64_t num_physical,
                                int64_t block_size, int64_t latent_dim, int64_t value_dim,
                                const int32_t* tables, int64_t max_blocks, const int32_t* lens,
                                int64_t batch, int64_t q_heads, float scale, const float* w_v,
                                int64_t proj_heads, int64_t head_dim, float* ctx, int acc64,
                                int threads) {
    if (batch <= 0) return OR_ZERO_VALUE;
    int64_t pairs = batch * q_heads;
    int status = OR_OK;
#ifdef _OPENMP
    if (threads <= 0) threads = omp_get_max_threads();
#pragma omp parallel for schedule(dynamic, 1) num_threads(threads)
#endif
    for (int64_t i = 0; i < pairs; ++i) {
        int64_t b = i / q_heads, h = i % q_heads;
        int st = plkv_or_latent_decode_seq(q_lat + b * q_heads * latent_dim, cache, num_physical,
                                           block_size, latent_dim, value_dim, tables + b * max_blocks,
                                           max_blocks, lens[b], lens[b], q_heads, scale, w_v,
                                           proj_heads, head_dim, NULL, NULL, NULL,
                                           ctx + b * q_heads * head_dim, h, h + 1, acc64);
        if (st != OR_OK) {
#ifdef _OPENMP
#pragma omp atomic write
#endif
            status = st;
        }
    }
    return status;
}

/* Batched FP16 full-KV paged GQA decode (extension of lib.rs:1147-1269). */
int plkv_or_fullkv_decode_batch(const float* q, const uint16_t* k, const uint16_t* v,
                                int64_t num_physical, int64_t kv_heads, int64_t block_size,
                                int64_t head_dim, const int32_t* tables, int64_t max_blocks,
                                const int32_t* lens, int64_t batch, int64_t q_heads, float scale,
                                float* ctx, int acc64, int threads) {
    if (batch <= 0) return OR_ZERO_VALUE;
    int64_t pairs = batch * q_heads;
    int status = OR_OK;
#ifdef _OPENMP
    if (threads <= 0) threads = omp_get_max_threads();
#pragma omp parallel for schedule(dynamic, 1) num_threads(threads)
#endif
    for (int64_t i = 0; i < pairs; ++i) {
        int64_t b = i / q_heads, h = i % q_heads;
        int st = plkv_or_fullkv_decode_seq(q + b * q_heads * head_dim, k, v, num_physical, kv_heads,
                                           block_size, head_dim, tables + b * max_blocks, max_blocks,
                                           lens[b], lens[b], q_heads, scale, NULL, NULL,
                                           ctx + b * q_heads * head_dim, h, h + 1, acc64);
        if (st != OR_OK) {
#ifdef _OPENMP
#pragma omp atomic write
#endif
            status = st;
        }
    }
    return status;
}

/* out[b, n] = sum_k x[b, k] * w[k, n] for the W_o output projection
 * (x = [batch, in_dim] concatenated head contexts, w = [in_dim, out_dim]). */
int plkv_or_out_proj(const float* x, const float* w, int64_t batch, int64_t in_dim,
                     int64_t out_dim, float* out, int acc64, int threads) {
    if (batch <= 0 || in_dim <= 0 || out_dim <= 0) return OR_ZERO_VALUE;
#ifdef _OPENMP
    if (threads <= 0) threads = omp_get_max_threads();
#pragma omp parallel for schedule(static) num_threads(threads)
#endif
    for (int64_t b = 0; b < batch; ++b) {
        if (acc64) {
            double* acc = (double*)calloc((size_t)out_dim, sizeof(double));
            for (int64_t kk = 0; kk < in_dim; ++kk) {
                double xv = x[b * in_dim + kk];
                const float* wr = w + kk * out_dim;
                for (int64_t n = 0; n < out_dim; ++n) acc[n] += xv * (double)wr[n];
            }
            for (int64_t n = 0; n < out_dim; ++n) out[b * out_dim + n] = (float)acc[n];
            free(acc);
        } else {
            float* acc = (float*)calloc((size_t)out_dim, sizeof(float));
            for (int64_t kk = 0; kk < in_dim; ++kk) {
                float xv = x[b * in_dim + kk];
                const float* wr = w + kk * out_dim;
                for (int64_t n = 0; n < out_dim; ++n) acc[n] += xv * wr[n];
            }
            memcpy(out + b * out_dim, acc, (size_t)out_dim * sizeof(float));
            free(acc);
        }
    }
    return OR_OK;
}

/* lib.rs:517-580: K[t, n] = sum_l latent[t, l] * w_k[l, n] over l < latent_dim
 * and V[t, n] = sum_l latent[t, l] * w_v[l, n] over l < value_dim (the
 * reference uses value_dim = latent_dim), n < width = kv_heads * head_dim,
 * token-major outputs.  The reference's loop order and FP32 accumulation
 * (product rounded, then the sum); acc64 accumulates in FP64 instead.
 * Rejects non-finite inputs and non-finite results like the reference. */
int plkv_or_reconstruct_kv(const float* latent, int64_t seq_len, int64_t latent_dim,
                           int64_t value_dim, const float* w_k, const float* w_v, int64_t width,
                           float* k_out, float* v_out, int acc64) {
    if (seq_len <= 0 || latent_dim <= 0 || value_dim <= 0 || width <= 0) return OR_ZERO_VALUE;
    if (value_dim > latent_dim) return OR_INVALID_ARGUMENT;
    for (int64_t i = 0; i < seq_len * latent_dim; ++i)
        if (!isfinite(latent[i])) return OR_NON_FINITE;
    for (int64_t i = 0; i < latent_dim * width; ++i)
        if (!isfinite(w_k[i])) return OR_NON_FINITE;
    for (int64_t i = 0; i < value_dim * width; ++i)
        if (!isfinite(w_v[i])) return OR_NON_FINITE;
    for (int64_t t = 0; t < seq_len; ++t) {
        const float* row = latent + t * latent_dim;
        for (int64_t n = 0; n < width; ++n) {
            float k_sum, v_sum;
            if (acc64) {
                double k = 0.0, v = 0.0;
                for (int64_t l = 0; l < latent_dim; ++l) k += (double)row[l] * w_k[l * width + n];
                for (int64_t l = 0; l < value_dim; ++l) v += (double)row[l] * w_v[l * width + n];
                k_sum = (float)k;
                v_sum = (float)v;
            } else {
                k_sum = 0.0f;
                v_sum = 0.0f;
                for (int64_t l = 0; l < latent_dim; ++l) {
                    float p = row[l] * w_k[l * width + n];
                    k_sum += p;
                    if (l < value_dim) {
                        float q = row[l] * w_v[l * width + n];
                        v_sum += q;
                    }
                }
            }
            if (!isfinite(k_sum) || !isfinite(v_sum)) return OR_NON_FINITE;
            k_out[t * width + n] = k_sum;
            v_out[t * width + n] = v_sum;
        }
    }
    return OR_OK;
}

int plkv_or_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
