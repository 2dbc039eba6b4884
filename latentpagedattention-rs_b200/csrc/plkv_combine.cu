// plkv_combine.cu -- log-sum-exp combine of split-K partials fused with the
// value projection, probability finalisation, shard merge, and the W_o
// output projection.
//
//   latent context -> W_v / W_uv   lib.rs:1066-1071, attention_ref.py:530
//   masked intermediates            lib.rs:1130-1140, attention_ref.py:604-611
#include "plkv_common.cuh"

namespace plkv {

constexpr int kCombineRows = 8;  // (sequence, head) rows per CTA

// grid = (proj_heads, ceil(batch * group / kCombineRows)), block = 256.
// Row r of the CTA is (b, h) with h = p * group + (gr % group), b = gr / group.
// Phase 1: warp per row merges the row's items:
//   M = max_i m_i,  S = sum_i l_i exp(m_i - M),
//   c[col] = sum_i ctx_i[col] exp(m_i - M) / S.
// Phase 2: out[d] = sum_l c[l] * W[p, l, d] in increasing l (lib.rs:1066-1071),
// or c itself when there is no projection.
__global__ void __launch_bounds__(256)
combine_project_kernel(DecodeWorkspace ws, const int32_t* __restrict__ seq_item_begin, int B,
                       int Hq, int width, const float* __restrict__ w, int proj_heads, int D,
                       float* __restrict__ out, float* __restrict__ lse) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    float* cs = reinterpret_cast<float*>(smem_raw);  // [kCombineRows][width]
    const int group = Hq / proj_heads;
    const int p = blockIdx.x;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int rows_total = B * group;
    const int r0 = blockIdx.y * kCombineRows;
    const int nrows = min(kCombineRows, rows_total - r0);

    for (int r = warp; r < kCombineRows; r += 8) {
        float* c = cs + r * width;
        if (r >= nrows) {
            for (int col = lane; col < width; col += 32) c[col] = 0.f;
            continue;
        }
        const int gr = r0 + r;
        const int b = gr / group, h = p * group + gr % group;
        const int ib = seq_item_begin[b], ie = seq_item_begin[b + 1];
        float M = -INFINITY;
        for (int i = ib + lane; i < ie; i += 32) M = fmaxf(M, ws.part_m[(int64_t)i * Hq + h]);
        M = warp_max(M);
        float S = 0.f;
        for (int i = ib + lane; i < ie; i += 32) {
            const float mi = ws.part_m[(int64_t)i * Hq + h];
            if (mi != -INFINITY) S += ws.part_l[(int64_t)i * Hq + h] * expf(mi - M);
        }
        S = warp_sum(S);
        for (int col = lane; col < width; col += 32) c[col] = 0.f;
        if (M != -INFINITY) {
            for (int i = ib; i < ie; ++i) {
                const float mi = ws.part_m[(int64_t)i * Hq + h];
                if (mi == -INFINITY) continue;
                const float wi = expf(mi - M);
                const float* src = ws.part_ctx + ((int64_t)i * Hq + h) * width;
                for (int col = lane; col < width; col += 32) c[col] = fmaf(src[col], wi, c[col]);
            }
            const float inv = 1.f / S;
            for (int col = lane; col < width; col += 32) c[col] *= inv;
        }
        if (lane == 0) {
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
    for (int d0 = 0; d0 < D; d0 += 256) {
        // Threads split as (row set) x (column d): tpr threads per row set.
        const int dcount = min(256, D - d0);
        const int sets = 256 / dcount;
        const int set = tid / dcount, d = d0 + tid % dcount;
        if (set >= sets) continue;
        float acc[kCombineRows];
#pragma unroll
        for (int r = 0; r < kCombineRows; ++r) acc[r] = 0.f;
        for (int l = 0; l < width; ++l) {
            const float wv = wp[(int64_t)l * D + d];
#pragma unroll
            for (int r = 0; r < kCombineRows; ++r)
                if (r % sets == set) acc[r] = fmaf(cs[r * width + l], wv, acc[r]);
        }
#pragma unroll
        for (int r = 0; r < kCombineRows; ++r) {
            if (r % sets != set || r >= nrows) continue;
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
    const int group = Hq / proj_heads;
    const size_t smem = size_t(kCombineRows) * width * 4;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(combine_project_kernel,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
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
