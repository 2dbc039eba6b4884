// plkv_combine.cu -- log-sum-exp combine of split-K partials fused with the
// value projection, probability finalisation, shard merge, and the W_o
// output projection.
//
//   latent context -> W_v / W_uv   lib.rs:1066-1071, attention_ref.py:530
//   masked intermediates            lib.rs:1130-1140, attention_ref.py:604-611
#include "plkv_common.cuh"

namespace plkv {

constexpr int kCombineRows = 8;   // (sequence, head) rows per CTA
constexpr int kMaxWidthPerLane = 20;  // width <= 640
constexpr int kLSlices = 8;       // latent-row slices of the projection
constexpr int kItemBatch = 4;     // split-K items whose loads are in flight together

// W is read by every step: its lines are kept in L2 (evict_last) while the
// partial pass streams the cache through L2 with evict_first.
__device__ __forceinline__ uint64_t l2_evict_last_policy() {
    uint64_t p;
    asm("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ float4 ldg_f4_keep(const float4* ptr, uint64_t pol) {
    float4 v;
    asm("ld.global.nc.L2::cache_hint.v4.f32 {%0, %1, %2, %3}, [%4], %5;"
        : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
        : "l"(ptr), "l"(pol));
    return v;
}

// grid = (proj_heads, ceil(batch * group / kCombineRows)), block = 256.
// Row r of the CTA is (b, h) with h = p * group + (gr % group), b = gr / group.
// Phase 1: warp per row merges the row's items in registers (lane owns
//   columns lane + 32k):  M = max_i m_i,  S = sum_i l_i exp(m_i - M),
//   c[col] = sum_i ctx_i[col] exp(m_i - M) / S.
// Phase 2: out[d] = sum_l c[l] * W[p, l, d] (lib.rs:1066-1071).  With
//   d % 4 == 0, D <= 128 and W 16-byte aligned the 256 threads are (latent
//   slice s) x (group of 4 columns): each thread sums its slice of l with
//   float4 weight loads, then the slices are added in a fixed order; otherwise
//   a column per thread.  W[p] (width x D floats) is prefetched into L2 when
//   the CTA starts, so that its loads overlap phase 1 instead of following it.
// Without a projection, c itself is written.
__global__ void __launch_bounds__(256)
combine_project_kernel(DecodeWorkspace ws, const int32_t* __restrict__ seq_item_begin, int B,
                       int Hq, int width, const float* __restrict__ w, int proj_heads, int D,
                       float* __restrict__ out, float* __restrict__ lse) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    float* cs = reinterpret_cast<float*>(smem_raw);           // [kCombineRows][width]
    float* red = cs + kCombineRows * width;                   // [kLSlices][kCombineRows][128]
    const int group = Hq / proj_heads;
    const int p = blockIdx.x;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int rows_total = B * group;
    const int r0 = blockIdx.y * kCombineRows;
    const int nrows = min(kCombineRows, rows_total - r0);
    const int ncol = (width + 31) / 32;
    const bool vec_w = w && (D & 3) == 0 && D <= 128 &&
                       (reinterpret_cast<uintptr_t>(w) & 15) == 0;
    if (vec_w && tid == 0) {
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;"
                     ::"l"(w + (int64_t)p * width * D), "r"((uint32_t)(width * D * 4)) : "memory");
    }

    for (int r = warp; r < kCombineRows; r += 8) {
        float acc[kMaxWidthPerLane];
#pragma unroll
        for (int k = 0; k < kMaxWidthPerLane; ++k) acc[k] = 0.f;
        float M = -INFINITY, S = 0.f;
        int b = 0, h = 0;
        if (r < nrows) {
            const int gr = r0 + r;
            b = gr / group;
            h = p * group + gr % group;
            const int ib = seq_item_begin[b], ie = seq_item_begin[b + 1];
            for (int i = ib + lane; i < ie; i += 32) M = fmaxf(M, ws.part_m[(int64_t)i * Hq + h]);
            M = warp_max(M);
            if (M != -INFINITY) {
                // kItemBatch items per round trip: all their loads are issued
                // before any is used, so the row costs one memory latency per
                // batch instead of one per item.  Items in the order i = ib..
                for (int i0 = ib; i0 < ie; i0 += kItemBatch) {
                    // The context loads do not wait for the item's max: an
                    // item without tokens is skipped below, whatever its row.
                    float wq[kItemBatch], lq[kItemBatch], v[kItemBatch][kMaxWidthPerLane];
#pragma unroll
                    for (int q = 0; q < kItemBatch; ++q) {
                        const int i = i0 + q;
                        wq[q] = i < ie ? ws.part_m[(int64_t)i * Hq + h] : -INFINITY;
                        lq[q] = i < ie ? ws.part_l[(int64_t)i * Hq + h] : 0.f;
                        const float* src = ws.part_ctx + ((int64_t)i * Hq + h) * width;
#pragma unroll
                        for (int k = 0; k < kMaxWidthPerLane; ++k) {
                            const int col = lane + 32 * k;
                            v[q][k] = (i < ie && k < ncol && col < width) ? src[col] : 0.f;
                        }
                    }
#pragma unroll
                    for (int q = 0; q < kItemBatch; ++q) {
                        if (wq[q] == -INFINITY) continue;
                        const float wi = expf(wq[q] - M);
                        S += lq[q] * wi;
#pragma unroll
                        for (int k = 0; k < kMaxWidthPerLane; ++k) acc[k] = fmaf(v[q][k], wi, acc[k]);
                    }
                }
            }
        }
        const float inv = (M != -INFINITY) ? 1.f / S : 0.f;
#pragma unroll
        for (int k = 0; k < kMaxWidthPerLane; ++k) {
            const int col = lane + 32 * k;
            if (k < ncol && col < width) cs[r * width + col] = acc[k] * inv;
        }
        if (r < nrows && lane == 0) {
            ws.row_m[(int64_t)b * Hq + h] = M;
            ws.row_l[(int64_t)b * Hq + h] = S;
            if (lse) lse[(int64_t)b * Hq + h] = (M == -INFINITY) ? -INFINITY : M + logf(S);
        }
    }
    __syncthreads();

    if (!w) {
        for (int i = tid; i < nrows * width; i += 256) {
            const int r = i / width, col = i - r * width;
            const int gr = r0 + r;
            const int b = gr / group, h = p * group + gr % group;
            out[((int64_t)b * Hq + h) * width + col] = cs[r * width + col];
        }
        return;
    }
    const float* wp = w + (int64_t)p * width * D;
    if (vec_w) {
        const uint64_t keep = l2_evict_last_policy();
        const int dg = tid & 31, slice = tid >> 5;
        const int l0 = (width * slice) / kLSlices, l1 = (width * (slice + 1)) / kLSlices;
        float acc[kCombineRows][4];
#pragma unroll
        for (int r = 0; r < kCombineRows; ++r)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[r][e] = 0.f;
        if (4 * dg < D) {
#pragma unroll 16
            for (int l = l0; l < l1; ++l) {
                const float4 wv = ldg_f4_keep(reinterpret_cast<const float4*>(wp + (int64_t)l * D) + dg, keep);
#pragma unroll
                for (int r = 0; r < kCombineRows; ++r) {
                    const float c = cs[r * width + l];
                    acc[r][0] = fmaf(c, wv.x, acc[r][0]);
                    acc[r][1] = fmaf(c, wv.y, acc[r][1]);
                    acc[r][2] = fmaf(c, wv.z, acc[r][2]);
                    acc[r][3] = fmaf(c, wv.w, acc[r][3]);
                }
            }
#pragma unroll
            for (int r = 0; r < kCombineRows; ++r)
                *reinterpret_cast<float4*>(red + (slice * kCombineRows + r) * 128 + 4 * dg) =
                    make_float4(acc[r][0], acc[r][1], acc[r][2], acc[r][3]);
        }
        __syncthreads();
        for (int i = tid; i < nrows * D; i += 256) {
            const int r = i / D, d = i - r * D;
            float v = 0.f;
#pragma unroll
            for (int sl = 0; sl < kLSlices; ++sl) v += red[(sl * kCombineRows + r) * 128 + d];
            const int gr = r0 + r;
            const int b = gr / group, h = p * group + gr % group;
            out[((int64_t)b * Hq + h) * D + d] = v;
        }
        return;
    }
    for (int d0 = 0; d0 < D; d0 += 256) {
        const int d = d0 + tid;
        if (d >= D) continue;
        float acc[kCombineRows];
#pragma unroll
        for (int r = 0; r < kCombineRows; ++r) acc[r] = 0.f;
        for (int l = 0; l < width; ++l) {
            const float wv = wp[(int64_t)l * D + d];
#pragma unroll
            for (int r = 0; r < kCombineRows; ++r) acc[r] = fmaf(cs[r * width + l], wv, acc[r]);
        }
        for (int r = 0; r < nrows; ++r) {
            const int gr = r0 + r;
            const int b = gr / group, h = p * group + gr % group;
            out[((int64_t)b * Hq + h) * D + d] = acc[r];
        }
    }
}

cudaError_t launch_combine(DecodeWorkspace ws, const int32_t* seq_item_begin, int B, int Hq,
                           int width, const float* w, int proj_heads, int D, float* out,
                           float* lse, cudaStream_t st) {
    if (!w) proj_heads = Hq;
    if (width > 32 * kMaxWidthPerLane) return cudaErrorInvalidValue;
    const int group = Hq / proj_heads;
    const size_t smem = size_t(kCombineRows) * width * 4 + size_t(kLSlices) * kCombineRows * 128 * 4;
    cudaError_t e = cudaFuncSetAttribute(combine_project_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    dim3 grid(proj_heads, (B * group + kCombineRows - 1) / kCombineRows);
    combine_project_kernel<<<grid, 256, smem, st>>>(ws, seq_item_begin, B, Hq, width, w,
                                                     proj_heads, D, out, lse);
    return cudaGetLastError();
}

// grid = batch * q_heads rows, block = 256: probabilities from the stored
// scores and the row's final (max, sum); inactive positions masked.
__global__ void finalize_probs_kernel(DecodeWorkspace ws, const int32_t* __restrict__ seq_lens,
                                      int Hq, int64_t cap, float* __restrict__ scores,
                                      float* __restrict__ probs, int max_seq_len) {
    const int64_t row = blockIdx.x;
    const int b = (int)(row / Hq);
    int len = seq_lens[b];
    if (len < 0) len = 0;
    if (len > cap) len = (int)cap;
    const float M = ws.row_m[row], S = ws.row_l[row];
    float* sr = scores + row * max_seq_len;
    float* pr = probs ? probs + row * max_seq_len : nullptr;
    for (int t = threadIdx.x; t < max_seq_len; t += blockDim.x) {
        if (t < len) {
            if (pr) pr[t] = expf(sr[t] - M) / S;
        } else {
            sr[t] = kMaskedScore;
            if (pr) pr[t] = 0.f;
        }
    }
}

cudaError_t launch_finalize(DecodeWorkspace ws, const int32_t* seq_lens, int B, int Hq,
                            int64_t cap, float* scores, float* probs, int max_seq_len,
                            cudaStream_t st) {
    finalize_probs_kernel<<<B * Hq, 256, 0, st>>>(ws, seq_lens, Hq, cap, scores, probs,
                                                  max_seq_len);
    return cudaGetLastError();
}

// grid = ceil(rows * width / 256): LSE merge of per-shard normalised contexts.
__global__ void lse_merge_kernel(const float* __restrict__ ctx, const float* __restrict__ lse,
                                 int S, int64_t rows, int width, float* __restrict__ out,
                                 float* __restrict__ lse_out) {
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= rows * width) return;
    const int64_t row = i / width;
    float M = -INFINITY;
    for (int s = 0; s < S; ++s) M = fmaxf(M, lse[s * rows + row]);
    float num = 0.f, den = 0.f;
    if (M != -INFINITY) {
        for (int s = 0; s < S; ++s) {
            const float ls = lse[s * rows + row];
            if (ls == -INFINITY) continue;
            const float wgt = expf(ls - M);
            num = fmaf(wgt, ctx[(int64_t)s * rows * width + i], num);
            den += wgt;
        }
    }
    out[i] = den > 0.f ? num / den : 0.f;
    if (lse_out && i % width == 0) lse_out[row] = den > 0.f ? M + logf(den) : -INFINITY;
}

cudaError_t launch_lse_merge(const float* ctx, const float* lse, int S, int64_t rows, int width,
                             float* out, float* lse_out, cudaStream_t st) {
    const int64_t n = rows * width;
    lse_merge_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(ctx, lse, S, rows, width, out,
                                                                   lse_out);
    return cudaGetLastError();
}

// ----------------------------------------------------------- W_o (FP32)

constexpr int kOutTileN = 128;
constexpr int kOutChunkK = 64;

// grid = (ceil(N / 128), k_splits), block = 256 (two k-halves x 128 columns).
// partial[s, b, n] = sum_{k in split s} x[b, k] * w[k, n].
template <int BMAX>
__global__ void __launch_bounds__(256)
out_proj_partial_kernel(const float* __restrict__ x, const float* __restrict__ w,
                        float* __restrict__ partial, int B, int K, int N, int k_per_split) {
    __shared__ __align__(16) float xs[BMAX][kOutChunkK];
    __shared__ float red[BMAX][kOutTileN];
    const int tid = threadIdx.x;
    const int col = tid & (kOutTileN - 1), half = tid >> 7;
    const int n = blockIdx.x * kOutTileN + col;
    const int k0 = blockIdx.y * k_per_split;
    const int k1 = min(K, k0 + k_per_split);
    float acc[BMAX];
#pragma unroll
    for (int r = 0; r < BMAX; ++r) acc[r] = 0.f;
    for (int kc = k0; kc < k1; kc += kOutChunkK) {
        const int kn = min(kOutChunkK, k1 - kc);
        __syncthreads();
        for (int i = tid; i < BMAX * kOutChunkK; i += 256) {
            const int r = i / kOutChunkK, kk = i - r * kOutChunkK;
            xs[r][kk] = (r < B && kk < kn) ? x[(int64_t)r * K + kc + kk] : 0.f;
        }
        __syncthreads();
        if (n < N) {
            for (int kk = half; kk < kn; kk += 2) {
                const float wv = w[(int64_t)(kc + kk) * N + n];
#pragma unroll
                for (int r = 0; r < BMAX; ++r) acc[r] = fmaf(xs[r][kk], wv, acc[r]);
            }
        }
    }
    __syncthreads();
    if (half == 1) {
#pragma unroll
        for (int r = 0; r < BMAX; ++r) red[r][col] = acc[r];
    }
    __syncthreads();
    if (half == 0 && n < N) {
        for (int r = 0; r < B && r < BMAX; ++r)
            partial[((int64_t)blockIdx.y * B + r) * N + n] = acc[r] + red[r][col];
    }
}

__global__ void out_proj_reduce_kernel(const float* __restrict__ partial, float* __restrict__ out,
                                       int S, int64_t BN) {
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= BN) return;
    float acc = 0.f;
    for (int s = 0; s < S; ++s) acc += partial[s * BN + i];
    out[i] = acc;
}

cudaError_t launch_out_proj(const float* x, const float* w, float* out, int B, int K, int N,
                            int k_splits, float* partial, cudaStream_t st) {
    const int kps = ((K + k_splits - 1) / k_splits + kOutChunkK - 1) / kOutChunkK * kOutChunkK;
    dim3 grid((N + kOutTileN - 1) / kOutTileN, k_splits);
    if (B <= 8)
        out_proj_partial_kernel<8><<<grid, 256, 0, st>>>(x, w, partial, B, K, N, kps);
    else if (B <= 16)
        out_proj_partial_kernel<16><<<grid, 256, 0, st>>>(x, w, partial, B, K, N, kps);
    else if (B <= 32)
        out_proj_partial_kernel<32><<<grid, 256, 0, st>>>(x, w, partial, B, K, N, kps);
    else
        out_proj_partial_kernel<64><<<grid, 256, 0, st>>>(x, w, partial, B, K, N, kps);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    const int64_t BN = int64_t(B) * N;
    out_proj_reduce_kernel<<<(unsigned)((BN + 255) / 256), 256, 0, st>>>(partial, out, k_splits,
                                                                         BN);
    return cudaGetLastError();
}

}  // namespace plkv
