// plkv_common.cuh -- shared device helpers of libplkv_b200.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "plkv_b200.h"

namespace plkv {

constexpr float kMaskedScore = -3.4028234663852886e38f;  // lib.rs:1130, attention_ref.py:605
constexpr int kHeadGroup = 32;   // query heads per CTA in the exact decode
constexpr int kTileTokens = 32;  // tokens per smem tile in the exact decode

__device__ __forceinline__ void set_flag(int32_t* flags, int32_t bit) {
    if (flags) atomicOr(flags, bit);
}

// FP16 bits of an FP32 value, round to nearest even (cvt.rn.f16.f32).
__device__ __forceinline__ uint16_t f32_to_f16_bits(float x) {
    return __half_as_ushort(__float2half_rn(x));
}

__device__ __forceinline__ float f16_bits_to_f32(uint16_t h) {
    return __half2float(__ushort_as_half(h));
}

// Converts the 8 halves of a 16-byte word to FP32.
__device__ __forceinline__ void unpack8(const uint4& v, float* out) {
    const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float2 f = __half22float2(h[i]);
        out[2 * i] = f.x;
        out[2 * i + 1] = f.y;
    }
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__host__ __device__ inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// Workspace of one decode call: per-launch control words, per-item partial
// softmax state and context, per-row (sequence, head) final max / sum used to
// emit probabilities, and the FP16 pre-scaled query the tensor-core pass
// loads by TMA.
struct DecodeWorkspace {
    int32_t* ctl;     // [64] control words of one launch; ctl[0] = abort (zeroed per launch)
    float* part_m;    // [n_items, q_heads]   running max of the item's scores
    float* part_l;    // [n_items, q_heads]   sum of exp(score - part_m)
    float* part_ctx;  // [n_items, q_heads, width] unnormalised context
    float* row_m;     // [batch, q_heads]
    float* row_l;     // [batch, q_heads]
    float* row_ctx;   // [batch, q_heads, width] merged, normalised context (projection input)
    uint16_t* q16;    // [batch, q_heads, latent] FP16 (latent = 0: absent)
};

constexpr size_t kCtlBytes = 256;

__host__ __device__ inline size_t decode_workspace_bytes(int n_items, int batch, int q_heads,
                                                         int latent, int width) {
    size_t nh = size_t(n_items) * q_heads;
    return kCtlBytes + align256(nh * 4) * 2 + align256(nh * size_t(width) * 4) +
           align256(size_t(batch) * q_heads * 4) * 2 +
           align256(size_t(batch) * q_heads * size_t(width) * 4) +
           align256(size_t(batch) * q_heads * size_t(latent) * 2);
}

inline DecodeWorkspace carve_workspace(void* base, int n_items, int batch, int q_heads,
                                       int latent, int width) {
    char* p = static_cast<char*>(base);
    size_t nh = size_t(n_items) * q_heads;
    DecodeWorkspace w;
    w.ctl = reinterpret_cast<int32_t*>(p);
    p += kCtlBytes;
    w.part_m = reinterpret_cast<float*>(p);
    p += align256(nh * 4);
    w.part_l = reinterpret_cast<float*>(p);
    p += align256(nh * 4);
    w.part_ctx = reinterpret_cast<float*>(p);
    p += align256(nh * size_t(width) * 4);
    w.row_m = reinterpret_cast<float*>(p);
    p += align256(size_t(batch) * q_heads * 4);
    w.row_l = reinterpret_cast<float*>(p);
    p += align256(size_t(batch) * q_heads * 4);
    w.row_ctx = reinterpret_cast<float*>(p);
    p += align256(size_t(batch) * q_heads * size_t(width) * 4);
    w.q16 = latent > 0 ? reinterpret_cast<uint16_t*>(p) : nullptr;
    return w;
}

// Log-sum-exp merge of the split-K work items [ib, ie) of one (sequence,
// head) row h by one warp; every lane calls it with its own V consecutive
// columns [col, col + V) (V a multiple of 4: V / 4 16-byte loads per item,
// width and col multiples of V; V = 1 otherwise; a lane whose col is past
// `width` only takes part in the shuffles).  Computes M = max_i m_i,
// S = sum_i l_i exp(m_i - M) (per 32 items a tree sum over the lanes, then in
// order) and acc = sum_i ctx_i[col..] exp(m_i - M), items added in the order
// ib, ib + 1, ...  Lane j holds m, l and the weight of item i0 + j of each
// group of 32; the context loads of kItemBatch items are issued together and
// do not wait for the weights, so a row of up to 32 items costs one round
// trip per kItemBatch items (the first one shared with m and l).  An item
// whose weight is 0 (no tokens: m = -inf) is skipped, whatever its context
// row holds.
constexpr int kItemBatch = 8;

template <int V>
__device__ __forceinline__ void merge_row_warp(const DecodeWorkspace& ws, int ib, int ie, int Hq,
                                               int h, int width, int col, int lane,
                                               float (&acc)[V], float& M, float& S) {
    static_assert(V == 1 || V % 4 == 0, "V: 1 or whole 16-byte words");
#pragma unroll
    for (int k = 0; k < V; ++k) acc[k] = 0.f;
    S = 0.f;
    M = -INFINITY;
    const bool one_group = ie - ib <= 32;
    if (!one_group) {  // rows of many items: the max first
        for (int i = ib + lane; i < ie; i += 32) M = fmaxf(M, ws.part_m[(int64_t)i * Hq + h]);
        M = warp_max(M);
    }
    const int64_t istride = (int64_t)Hq * width;   // between items' context rows
    const bool col_in = col < width;
    for (int i0 = ib; i0 < ie; i0 += 32) {
        const int i = i0 + lane;
        const float m = i < ie ? ws.part_m[(int64_t)i * Hq + h] : -INFINITY;
        const float l = i < ie ? ws.part_l[(int64_t)i * Hq + h] : 0.f;
        const int n = min(32, ie - i0);
        const float* src0 = ws.part_ctx + ((int64_t)i0 * Hq + h) * width + col;
        float w = 0.f;
        bool have_w = false;
        for (int q0 = 0; q0 < n; q0 += kItemBatch) {
            float v[kItemBatch][V];
            const float* src = src0 + q0 * istride;
#pragma unroll
            for (int q = 0; q < kItemBatch; ++q, src += istride) {
                const bool in = q0 + q < n && col_in;
                if (V % 4 == 0) {
#pragma unroll
                    for (int k4 = 0; k4 < V / 4; ++k4) {
                        const float4 x = in ? reinterpret_cast<const float4*>(src)[k4]
                                            : make_float4(0.f, 0.f, 0.f, 0.f);
                        v[q][4 * k4] = x.x;
                        v[q][4 * k4 + 1] = x.y;
                        v[q][4 * k4 + 2] = x.z;
                        v[q][4 * k4 + 3] = x.w;
                    }
                } else {
                    v[q][0] = in ? src[0] : 0.f;
                }
            }
            if (!have_w) {  // weights of this group of 32, after its first loads are issued
                if (one_group) M = warp_max(m);
                w = (m == -INFINITY || M == -INFINITY) ? 0.f : expf(m - M);
                S += warp_sum(l * w);
                have_w = true;
            }
#pragma unroll
            for (int q = 0; q < kItemBatch; ++q) {
                const float wq = __shfl_sync(0xffffffffu, w, (q0 + q) & 31);
                if (q0 + q >= n || wq == 0.f) continue;
#pragma unroll
                for (int k = 0; k < V; ++k) acc[k] = fmaf(v[q][k], wq, acc[k]);
            }
        }
    }
}

// out[b, h, d] = sum_l rows[b, h, l] W[h / group, l, d] in a fixed order, for
// rows [B][Hr][width] and W [Hr / group][width][D] (lib.rs:1066-1071).  With
// rows_table the rows start rows_offset bytes into rows_table[rows_index] (a
// device-side pointer table).  D and width fit shared memory: width <= 5000.
cudaError_t launch_project_rows(const float* rows, void* const* rows_table, int rows_index,
                                size_t rows_offset, int B, int Hr, int width, const float* w,
                                int proj_heads, int D, float* out, cudaStream_t st);

// c[b, g G + j, :] = W[g] a[b, g G + j, :] for the G = Hq / heads rows of
// each head g, as a batched FP32 GEMM (plkv_rows_gemm.cu); W[g] is [K][N]
// row-major, or [N][K] when w_transposed.  Needs rows_gemm_supported.
bool rows_gemm_supported(const float* a, const float* w, const float* c, int K, int N);
cudaError_t launch_rows_gemm(const float* a, const float* w, bool w_transposed, float* c, int B,
                             int Hq, int heads, int K, int N, cudaStream_t st);

}  // namespace plkv
