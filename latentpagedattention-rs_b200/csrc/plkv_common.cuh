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
    uint16_t* q16;    // [batch, q_heads, latent] FP16 (latent = 0: absent)
};

constexpr size_t kCtlBytes = 256;

__host__ __device__ inline size_t decode_workspace_bytes(int n_items, int batch, int q_heads,
                                                         int latent, int width) {
    size_t nh = size_t(n_items) * q_heads;
    return kCtlBytes + align256(nh * 4) * 2 + align256(nh * size_t(width) * 4) +
           align256(size_t(batch) * q_heads * 4) * 2 +
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
    w.q16 = latent > 0 ? reinterpret_cast<uint16_t*>(p) : nullptr;
    return w;
}

}  // namespace plkv
