// plkv_reconstruct.cu -- materialised K / V from latent rows.
//
// Restates reconstruct_latent_kv_f32 (crates/plkv-core/src/lib.rs:517-580),
// the GPU kernel reconstruct_latent_kv
// (crates/plkv-kernels/src/cutile/latent_kv_reconstruction.rs:4-28) and
// latent_kv_reconstruction_ref (python_ref/.../attention_ref.py:227-274):
//
//   K[row, kv, d] = sum_{l < latent_dim} latent[row, l] * W_k[kv, l, d]
//   V[row, kv, d] = sum_{l < value_dim}  latent[row, l] * W_v[kv, l, d]
//
// with FP32 accumulation.  It is the "materialised" comparison point of the
// decode: rebuild full K / V from the latent pool, then run the full-KV decode
// on them, instead of attending in the latent space directly.
//
// Rows are pool slots (physical block * block_size + offset) of a latent pool
// [num_slots, latent_dim] in FP32 or FP16; the slot list selects which rows to
// rebuild (NULL: slots 0 .. n_rows-1).  K / V land at the same slot in the
// head-major paged layout [num_slots / bs, kv_heads, bs, head_dim] of the
// full-KV pool (bs = 1 gives the reference's token-major [row, kv, d]).
//
// Work split: one CTA computes a 128-row x 64-column tile of K or of V
// (grid.x = column tiles of K, then of V; grid.y strides over row tiles).
// The contraction runs in chunks of 32 latent columns staged in shared
// memory (latent chunk transposed, weight chunk row-major); each of the 256
// threads owns 8 rows x 4 columns.  This is FP32 CUDA-core arithmetic: the
// reference's formulation is FP32 end to end, and the point of this baseline
// is the cost of materialising, not a new numeric contract.
#include <algorithm>

#include "plkv_common.cuh"

namespace plkv {
namespace {

constexpr int kRecRows = 128;
constexpr int kRecCols = 64;
constexpr int kRecChunk = 32;

template <bool kInF16, bool kOutF16>
__global__ void __launch_bounds__(256)
reconstruct_kv_kernel(const void* __restrict__ latent, int64_t num_slots, int L, int Lv,
                      const int64_t* __restrict__ slots, int64_t n_rows,
                      const float* __restrict__ w_k, const float* __restrict__ w_v, int KV, int D,
                      int bs, void* __restrict__ k_out, void* __restrict__ v_out, int32_t* flags) {
    __shared__ float As[kRecChunk][kRecRows + 1];            // latent chunk, transposed
    __shared__ __align__(16) float Bs[kRecChunk][kRecCols];  // weight chunk
    __shared__ int64_t s_slot[kRecRows];
    const int width = KV * D;
    const int tiles_per_part = (width + kRecCols - 1) / kRecCols;
    const int part = blockIdx.x / tiles_per_part;  // 0: K, 1: V
    const int c0 = (blockIdx.x - part * tiles_per_part) * kRecCols;
    const int Lp = part ? Lv : L;
    const float* __restrict__ w = part ? w_v : w_k;
    void* out = part ? v_out : k_out;
    const int tid = threadIdx.x;
    const int tr = tid >> 4, tc = tid & 15;  // rows tr*8 .. +7, columns tc*4 .. +3

    for (int64_t r0 = (int64_t)blockIdx.y * kRecRows; r0 < n_rows;
         r0 += (int64_t)gridDim.y * kRecRows) {
        if (tid < kRecRows) {
            const int64_t r = r0 + tid;
            int64_t slot = -1;
            if (r < n_rows) {
                slot = slots ? slots[r] : r;
                if (slot >= num_slots) set_flag(flags, PLKV_FLAG_BAD_POSITION);
                if (slot < 0 || slot >= num_slots) slot = -1;  // negative: padding
            }
            s_slot[tid] = slot;
        }
        __syncthreads();
        float acc[8][4];
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;

        for (int l0 = 0; l0 < Lp; l0 += kRecChunk) {
            // Latent chunk: a warp reads 32 consecutive columns of one row.
            for (int i = tid; i < kRecRows * kRecChunk; i += 256) {
                const int r = i / kRecChunk, l = i - r * kRecChunk;
                const int64_t slot = s_slot[r];
                float x = 0.f;
                if (slot >= 0 && l0 + l < Lp) {
                    const int64_t idx = slot * (int64_t)L + l0 + l;
                    if constexpr (kInF16)
                        x = __half2float(reinterpret_cast<const __half*>(latent)[idx]);
                    else
                        x = reinterpret_cast<const float*>(latent)[idx];
                    if (!isfinite(x)) set_flag(flags, PLKV_FLAG_NON_FINITE_INPUT);
                }
                As[l][r] = x;
            }
            // Weight chunk: W[kv, l, d] of the tile's 64 columns.
            for (int i = tid; i < kRecChunk * kRecCols; i += 256) {
                const int l = i / kRecCols, c = i - l * kRecCols;
                const int col = c0 + c;
                float x = 0.f;
                if (col < width && l0 + l < Lp) {
                    const int kv = col / D, d = col - kv * D;
                    x = w[((int64_t)kv * Lp + l0 + l) * D + d];
                }
                Bs[l][c] = x;
            }
            __syncthreads();
#pragma unroll 8
            for (int l = 0; l < kRecChunk; ++l) {
                const float4 b = *reinterpret_cast<const float4*>(&Bs[l][tc * 4]);
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const float a = As[l][tr * 8 + i];
                    acc[i][0] = fmaf(a, b.x, acc[i][0]);
                    acc[i][1] = fmaf(a, b.y, acc[i][1]);
                    acc[i][2] = fmaf(a, b.z, acc[i][2]);
                    acc[i][3] = fmaf(a, b.w, acc[i][3]);
                }
            }
            __syncthreads();
        }

#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int64_t slot = s_slot[tr * 8 + i];
            if (slot < 0) continue;
            const int64_t blk = slot / bs, off = slot - blk * bs;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int col = c0 + tc * 4 + j;
                if (col >= width) continue;
                const int kv = col / D, d = col - kv * D;
                const float val = acc[i][j];
                if (!isfinite(val)) set_flag(flags, PLKV_FLAG_NON_FINITE_INPUT);
                const int64_t o = ((blk * KV + kv) * bs + off) * D + d;
                if constexpr (kOutF16) {
                    const __half h = __float2half_rn(val);
                    if (isfinite(val) && __hisinf(h)) set_flag(flags, PLKV_FLAG_FP16_OVERFLOW);
                    reinterpret_cast<__half*>(out)[o] = h;
                } else {
                    reinterpret_cast<float*>(out)[o] = val;
                }
            }
        }
        __syncthreads();  // s_slot is rewritten by the next row tile
    }
}

template <bool kInF16, bool kOutF16>
void launch(const void* latent, int64_t num_slots, int L, int Lv, const int64_t* slots,
            int64_t n_rows, const float* w_k, const float* w_v, int KV, int D, int bs,
            void* k_out, void* v_out, int32_t* flags, cudaStream_t st) {
    const int tiles_per_part = (KV * D + kRecCols - 1) / kRecCols;
    const int64_t row_tiles = (n_rows + kRecRows - 1) / kRecRows;
    dim3 grid(2 * tiles_per_part, (unsigned)std::min<int64_t>(row_tiles, 65535));
    reconstruct_kv_kernel<kInF16, kOutF16><<<grid, 256, 0, st>>>(
        latent, num_slots, L, Lv, slots, n_rows, w_k, w_v, KV, D, bs, k_out, v_out, flags);
}

}  // namespace
}  // namespace plkv

extern "C" int plkv_reconstruct_kv(const void* latent, int32_t latent_is_f16, int64_t num_slots,
                                   int32_t latent_dim, int32_t value_dim, const int64_t* slots,
                                   int64_t n_rows, const float* w_k, const float* w_v,
                                   int32_t kv_heads, int32_t head_dim, int32_t block_size,
                                   void* k_out, void* v_out, int32_t out_is_f16,
                                   int32_t* err_flags, plkv_stream_t stream) {
    if (num_slots <= 0 || latent_dim <= 0 || value_dim <= 0 || n_rows <= 0 || kv_heads <= 0 ||
        head_dim <= 0 || block_size <= 0)
        return PLKV_ERR_ZERO_VALUE;
    if (!latent || !w_k || !w_v || !k_out || !v_out || value_dim > latent_dim ||
        num_slots % block_size != 0 || (!slots && n_rows > num_slots))
        return PLKV_ERR_INVALID_ARGUMENT;
    if ((int64_t)kv_heads * head_dim > (1ll << 30) || num_slots > (1ll << 40))
        return PLKV_ERR_ARITHMETIC_OVERFLOW;
    const cudaStream_t st = (cudaStream_t)stream;
    const int L = latent_dim, Lv = value_dim, KV = kv_heads, D = head_dim, bs = block_size;
    if (latent_is_f16) {
        if (out_is_f16)
            plkv::launch<true, true>(latent, num_slots, L, Lv, slots, n_rows, w_k, w_v, KV, D, bs,
                                     k_out, v_out, err_flags, st);
        else
            plkv::launch<true, false>(latent, num_slots, L, Lv, slots, n_rows, w_k, w_v, KV, D,
                                      bs, k_out, v_out, err_flags, st);
    } else {
        if (out_is_f16)
            plkv::launch<false, true>(latent, num_slots, L, Lv, slots, n_rows, w_k, w_v, KV, D,
                                      bs, k_out, v_out, err_flags, st);
        else
            plkv::launch<false, false>(latent, num_slots, L, Lv, slots, n_rows, w_k, w_v, KV, D,
                                       bs, k_out, v_out, err_flags, st);
    }
    return cudaGetLastError() == cudaSuccess ? PLKV_OK : PLKV_ERR_CUDA;
}
