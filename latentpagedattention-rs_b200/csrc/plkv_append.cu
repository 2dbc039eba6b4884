// plkv_append.cu -- FP32 -> FP16 storage conversion and slot-mapped cache
// appends (latent rows and the full-KV baseline's K/V rows).
//
// Reference semantics kept:
//   quantize_f32_to_f16_storage  crates/plkv-core/src/lib.rs:302-319
//   resolve_paged_token_location lib.rs:164-188, cache_ref.py:22-40
//   paged_latent_write_fp16_storage lib.rs:889-939 (whole row or nothing)
//   paged_kv_write_f32           lib.rs:190-247 (K and V rows together)
#include "plkv_common.cuh"

namespace plkv {

__global__ void quantize_f16_kernel(const float* __restrict__ in, uint16_t* __restrict__ out,
                                    int64_t n, int32_t* flags) {
    int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    int64_t stride = (int64_t)gridDim.x * blockDim.x;
    int bad = 0;
    for (; i < n; i += stride) {
        float x = in[i];
        uint16_t h = f32_to_f16_bits(x);
        if (!isfinite(x)) bad |= PLKV_FLAG_NON_FINITE_INPUT;
        else if ((h & 0x7c00u) == 0x7c00u) bad |= PLKV_FLAG_FP16_OVERFLOW;
        out[i] = h;
    }
    if (bad) set_flag(flags, bad);
}

// Resolves (sequence, position) to the element offset of the row's first
// value in a [P, kv_heads, bs, width] pool (kv_heads = 1 for the latent
// cache).  Returns -1 and raises a flag when the table does not cover it.
__device__ __forceinline__ int64_t resolve_row(const int32_t* tables, int64_t max_blocks, int seq,
                                               int pos, int bs, int64_t num_physical,
                                               int32_t* flags, int64_t* phys_out) {
    if (pos < 0 || (int64_t)(pos / bs) >= max_blocks) {
        set_flag(flags, PLKV_FLAG_BAD_POSITION);
        return -1;
    }
    int32_t phys = tables[(int64_t)seq * max_blocks + pos / bs];
    if (phys < 0 || phys >= num_physical) {
        set_flag(flags, PLKV_FLAG_BAD_BLOCK);
        return -1;
    }
    *phys_out = phys;
    return pos % bs;
}

// One CTA per request row.  Pass 1 checks that the whole row converts to
// finite FP16; pass 2 writes it.  A rejected row leaves the cache untouched.
__global__ void latent_append_kernel(const float* __restrict__ rows,
                                     const int32_t* __restrict__ tables, int64_t max_blocks,
                                     const int32_t* __restrict__ seq_ids,
                                     const int32_t* __restrict__ positions, int32_t* seq_lens,
                                     uint16_t* __restrict__ cache, int64_t num_physical, int bs,
                                     int L, int32_t* flags) {
    const int64_t i = blockIdx.x;
    const int seq = seq_ids ? seq_ids[i] : (int)i;
    const float* src = rows + i * L;
    int bad = 0;
    for (int c = threadIdx.x; c < L; c += blockDim.x) {
        float x = src[c];
        if (!isfinite(x)) bad |= PLKV_FLAG_NON_FINITE_INPUT;
        else if ((f32_to_f16_bits(x) & 0x7c00u) == 0x7c00u) bad |= PLKV_FLAG_FP16_OVERFLOW;
    }
    __shared__ int s_bad;
    __shared__ long long s_dst;
    __shared__ int s_pos;
    if (threadIdx.x == 0) s_bad = 0;
    __syncthreads();
    if (bad) atomicOr(&s_bad, bad);
    if (threadIdx.x == 0) {
        int pos = seq_lens ? seq_lens[seq] : positions[i];
        int64_t phys = 0;
        int64_t off = resolve_row(tables, max_blocks, seq, pos, bs, num_physical, flags, &phys);
        s_dst = off < 0 ? -1 : (phys * bs + off) * (int64_t)L;
        s_pos = pos;
    }
    __syncthreads();
    if (s_bad) {
        if (threadIdx.x == 0) set_flag(flags, s_bad);
        return;
    }
    if (s_dst < 0) return;
    uint16_t* dst = cache + s_dst;
    for (int c = threadIdx.x; c < L; c += blockDim.x) dst[c] = f32_to_f16_bits(src[c]);
    if (seq_lens && threadIdx.x == 0) seq_lens[seq] = s_pos + 1;
}

__global__ void latent_append_slots_kernel(const float* __restrict__ rows,
                                           const int64_t* __restrict__ slots,
                                           uint16_t* __restrict__ cache, int64_t num_slots, int L,
                                           int32_t* flags) {
    const int64_t i = blockIdx.x;
    const int64_t slot = slots[i];
    if (slot < 0) return;  // padding
    if (slot >= num_slots) {
        if (threadIdx.x == 0) set_flag(flags, PLKV_FLAG_BAD_BLOCK);
        return;
    }
    const float* src = rows + i * L;
    int bad = 0;
    for (int c = threadIdx.x; c < L; c += blockDim.x) {
        float x = src[c];
        if (!isfinite(x)) bad |= PLKV_FLAG_NON_FINITE_INPUT;
        else if ((f32_to_f16_bits(x) & 0x7c00u) == 0x7c00u) bad |= PLKV_FLAG_FP16_OVERFLOW;
    }
    bad = __syncthreads_or(bad) ? 1 : 0;
    if (bad) {
        // Recompute the exact bits for the flag word on thread 0 only.
        if (threadIdx.x == 0) {
            int b2 = 0;
            for (int c = 0; c < L; ++c) {
                float x = src[c];
                if (!isfinite(x)) b2 |= PLKV_FLAG_NON_FINITE_INPUT;
                else if ((f32_to_f16_bits(x) & 0x7c00u) == 0x7c00u) b2 |= PLKV_FLAG_FP16_OVERFLOW;
            }
            set_flag(flags, b2);
        }
        return;
    }
    uint16_t* dst = cache + slot * (int64_t)L;
    for (int c = threadIdx.x; c < L; c += blockDim.x) dst[c] = f32_to_f16_bits(src[c]);
}

// K/V rows [n, kv_heads, head_dim]; pool [P, kv_heads, bs, head_dim].
__global__ void kv_append_kernel(const float* __restrict__ k_rows, const float* __restrict__ v_rows,
                                 const int32_t* __restrict__ tables, int64_t max_blocks,
                                 const int32_t* __restrict__ seq_ids,
                                 const int32_t* __restrict__ positions, int32_t* seq_lens,
                                 uint16_t* __restrict__ k_cache, uint16_t* __restrict__ v_cache,
                                 int64_t num_physical, int KV, int bs, int D, int32_t* flags) {
    const int64_t i = blockIdx.x;
    const int seq = seq_ids ? seq_ids[i] : (int)i;
    const int W = KV * D;
    const float* ks = k_rows + i * W;
    const float* vs = v_rows + i * W;
    int bad = 0;
    for (int c = threadIdx.x; c < W; c += blockDim.x) {
        float a = ks[c], b = vs[c];
        if (!isfinite(a) || !isfinite(b)) bad |= PLKV_FLAG_NON_FINITE_INPUT;
        else if ((f32_to_f16_bits(a) & 0x7c00u) == 0x7c00u ||
                 (f32_to_f16_bits(b) & 0x7c00u) == 0x7c00u)
            bad |= PLKV_FLAG_FP16_OVERFLOW;
    }
    __shared__ int s_bad;
    __shared__ long long s_phys;
    __shared__ int s_off, s_pos;
    if (threadIdx.x == 0) s_bad = 0;
    __syncthreads();
    if (bad) atomicOr(&s_bad, bad);
    if (threadIdx.x == 0) {
        int pos = seq_lens ? seq_lens[seq] : positions[i];
        int64_t phys = 0;
        int64_t off = resolve_row(tables, max_blocks, seq, pos, bs, num_physical, flags, &phys);
        s_phys = off < 0 ? -1 : phys;
        s_off = (int)off;
        s_pos = pos;
    }
    __syncthreads();
    if (s_bad) {
        if (threadIdx.x == 0) set_flag(flags, s_bad);
        return;
    }
    if (s_phys < 0) return;
    for (int c = threadIdx.x; c < W; c += blockDim.x) {
        int g = c / D, d = c - g * D;
        int64_t dst = ((s_phys * KV + g) * bs + s_off) * (int64_t)D + d;
        k_cache[dst] = f32_to_f16_bits(ks[c]);
        v_cache[dst] = f32_to_f16_bits(vs[c]);
    }
    if (seq_lens && threadIdx.x == 0) seq_lens[seq] = s_pos + 1;
}

void launch_quantize(const float* in, uint16_t* out, int64_t n, int32_t* flags,
                     cudaStream_t st) {
    int64_t blocks = (n + 255) / 256;
    if (blocks > 148 * 16) blocks = 148 * 16;
    if (blocks < 1) blocks = 1;
    quantize_f16_kernel<<<(unsigned)blocks, 256, 0, st>>>(in, out, n, flags);
}

void launch_latent_append(const float* rows, const int32_t* tables, int64_t max_blocks,
                          const int32_t* seq_ids, const int32_t* positions, int32_t* seq_lens,
                          int64_t n, uint16_t* cache, int64_t num_physical, int bs, int L,
                          int32_t* flags, cudaStream_t st) {
    latent_append_kernel<<<(unsigned)n, 128, 0, st>>>(rows, tables, max_blocks, seq_ids, positions,
                                                      seq_lens, cache, num_physical, bs, L, flags);
}

void launch_latent_append_slots(const float* rows, const int64_t* slots, int64_t n,
                                uint16_t* cache, int64_t num_slots, int L, int32_t* flags,
                                cudaStream_t st) {
    latent_append_slots_kernel<<<(unsigned)n, 128, 0, st>>>(rows, slots, cache, num_slots, L, flags);
}

void launch_kv_append(const float* k_rows, const float* v_rows, const int32_t* tables,
                      int64_t max_blocks, const int32_t* seq_ids, const int32_t* positions,
                      int32_t* seq_lens, int64_t n, uint16_t* k_cache, uint16_t* v_cache,
                      int64_t num_physical, int KV, int bs, int D, int32_t* flags,
                      cudaStream_t st) {
    kv_append_kernel<<<(unsigned)n, 256, 0, st>>>(k_rows, v_rows, tables, max_blocks, seq_ids,
                                                  positions, seq_lens, k_cache, v_cache,
                                                  num_physical, KV, bs, D, flags);
}

}  // namespace plkv
