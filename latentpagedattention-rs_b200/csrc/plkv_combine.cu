// plkv_combine.cu -- log-sum-exp combine of split-K partials fused with the
// value projection, probability finalisation, shard merge, and the W_o
// output projection.
//
//   latent context -> W_v / W_uv   lib.rs:1066-1071, attention_ref.py:530
//   masked intermediates            lib.rs:1130-1140, attention_ref.py:604-611
#include "plkv_common.cuh"

namespace plkv {


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

// grid = ceil(B * Hq / (256 / TPR)), block = 256: the TPR / 32 warps of row
// x * (256 / TPR) + t / TPR merge the split-K items of row (b, h)
// (merge_row_warp), thread c = t % TPR for columns [Vc, Vc + V), [Vc + V TPR,
// ...) ... (V = 8 with 64 threads per row when width % 8 == 0, V = 4 with
// 128 when width % 4 == 0, else V = 1 with 128):
//   c[col] = sum_i ctx_i[col] exp(m_i - M) / S   (lib.rs:1066-1071 input).
// Writes dst[b, h, :] and, from thread 0 of the row, the row's M, S and lse.
// Registers capped so that a decode batch's grid is resident at once (V = 8:
// half the CTAs of V = 4, two per SM).
template <int V, int TPR>
__global__ void __launch_bounds__(256, V >= 8 ? 2 : 4)
merge_rows_kernel(DecodeWorkspace ws, const int32_t* __restrict__ seq_item_begin, int B, int Hq,
                  int width, float* __restrict__ dst, float* __restrict__ lse) {
    constexpr int kRows = 256 / TPR;
    const int64_t row = (int64_t)blockIdx.x * kRows + threadIdx.x / TPR;
    const int c = threadIdx.x % TPR, lane = threadIdx.x & 31;
    if (row >= (int64_t)B * Hq) return;  // whole warps: a row is TPR / 32 warps
    const int b = (int)(row / Hq), h = (int)(row % Hq);
    const int ib = seq_item_begin[b], ie = seq_item_begin[b + 1];
    float M = -INFINITY, S = 0.f;
    for (int base = 0; base < width; base += V * TPR) {   // the same passes in every lane
        const int col = base + V * c;
        float acc[V];
        merge_row_warp<V>(ws, ib, ie, Hq, h, width, col, lane, acc, M, S);
        const float inv = (M != -INFINITY) ? 1.f / S : 0.f;
        float* o = dst + row * width + col;
        if (V % 4 == 0) {
            if (col < width) {
#pragma unroll
                for (int k4 = 0; k4 < V / 4; ++k4)
                    reinterpret_cast<float4*>(o)[k4] =
                        make_float4(acc[4 * k4] * inv, acc[4 * k4 + 1] * inv,
                                    acc[4 * k4 + 2] * inv, acc[4 * k4 + 3] * inv);
            }
        } else if (col < width) {
            o[0] = acc[0] * inv;
        }
    }
    if (c == 0) {
        ws.row_m[row] = M;
        ws.row_l[row] = S;
        if (lse) lse[row] = (M == -INFINITY) ? -INFINITY : M + logf(S);
    }
}

// grid = (proj_heads, ceil(D / 32), ceil(B * group / 8)), block = 256.  The
// CTA projects 8 rows (b, h), h = p * group + (gr % group), b = gr / group, onto
// columns [32 y, 32 y + 32).  The rows are staged in shared memory as they
// lie (cs[8][width], 16-byte copies).  Vector path (D % 4 == 0, W 16-byte
// aligned): thread = (latent slice j of 32, 4 columns); slice j sums l = j,
// j + 32, ... for all 8 rows with float4 weight loads (8 rows of weights in
// flight per thread, each weight of the CTA loaded once), and the slices are
// added in a fixed order: two shuffles within the warp, then the 8 warps in
// order.  Otherwise thread (row, column) sums l in increasing order.
__global__ void __launch_bounds__(256)
project_rows_kernel(const float* __restrict__ rows, void* const* __restrict__ rows_table,
                    int rows_index, size_t rows_offset, int B, int Hr, int width,
                    const float* __restrict__ w, int proj_heads, int D, float* __restrict__ out) {
    extern __shared__ __align__(16) float smem_f[];
    if (rows_table)  // rows inside a buffer whose address only the device-side table holds
        rows = reinterpret_cast<const float*>(static_cast<const char*>(rows_table[rows_index]) +
                                              rows_offset);
    float* cs = smem_f;                       // [8][width]
    float* red = smem_f + (size_t)width * 8;  // [8 warps][8 rows][32]
    const int group = Hr / proj_heads;
    const int p = blockIdx.x, d0 = blockIdx.y * 32, r0 = blockIdx.z * 8;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nrows = min(8, B * group - r0);
    const float* wp = w + (int64_t)p * width * D;
    const bool vec = (D & 3) == 0 && (reinterpret_cast<uintptr_t>(w) & 15) == 0;
    const uint64_t keep = l2_evict_last_policy();
    const int lsub = lane >> 3, dq = lane & 7;
    const int slice = warp * 4 + lsub;
    const int dcol = d0 + 4 * dq;
    // The first 8 weight rows of this thread do not depend on the rows:
    // their loads are issued before the rows are staged, so that the two
    // latencies overlap.
    float4 wv[8];
    if (vec && dcol < D) {
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int l = slice + 32 * u;
            wv[u] = l < width ? ldg_f4_keep(reinterpret_cast<const float4*>(
                                                wp + (int64_t)l * D + dcol), keep)
                              : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
    if ((width & 3) == 0) {
        const int w4 = width >> 2;
        for (int r = 0; r < 8; ++r) {
            const int gr = r0 + r;
            const float4* src = reinterpret_cast<const float4*>(
                rows + ((int64_t)(gr / group) * Hr + p * group + gr % group) * width);
            for (int k = tid; k < w4; k += 256)
                reinterpret_cast<float4*>(cs + r * width)[k] =
                    r < nrows ? src[k] : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    } else {
        for (int idx = tid; idx < 8 * width; idx += 256) {
            const int r = idx / width, l = idx - r * width;
            float v = 0.f;
            if (r < nrows) {
                const int gr = r0 + r;
                v = rows[((int64_t)(gr / group) * Hr + p * group + gr % group) * width + l];
            }
            cs[idx] = v;
        }
    }
    __syncthreads();
    if (vec) {
        float acc[8][4];
#pragma unroll
        for (int r = 0; r < 8; ++r)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[r][e] = 0.f;
        if (dcol < D) {
            for (int l0 = slice; l0 < width; l0 += 32 * 8) {
                if (l0 != slice) {
#pragma unroll
                    for (int u = 0; u < 8; ++u) {
                        const int l = l0 + 32 * u;
                        wv[u] = l < width ? ldg_f4_keep(reinterpret_cast<const float4*>(
                                                            wp + (int64_t)l * D + dcol), keep)
                                          : make_float4(0.f, 0.f, 0.f, 0.f);
                    }
                }
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const int l = l0 + 32 * u;
                    if (l >= width) break;
#pragma unroll
                    for (int r = 0; r < 8; ++r) {
                        const float c = cs[r * width + l];
                        acc[r][0] = fmaf(c, wv[u].x, acc[r][0]);
                        acc[r][1] = fmaf(c, wv[u].y, acc[r][1]);
                        acc[r][2] = fmaf(c, wv[u].z, acc[r][2]);
                        acc[r][3] = fmaf(c, wv[u].w, acc[r][3]);
                    }
                }
            }
        }
#pragma unroll
        for (int r = 0; r < 8; ++r)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                acc[r][e] += __shfl_xor_sync(0xffffffffu, acc[r][e], 8);
                acc[r][e] += __shfl_xor_sync(0xffffffffu, acc[r][e], 16);
            }
        if (lsub == 0) {
#pragma unroll
            for (int r = 0; r < 8; ++r)
                *reinterpret_cast<float4*>(red + (warp * 8 + r) * 32 + 4 * dq) =
                    make_float4(acc[r][0], acc[r][1], acc[r][2], acc[r][3]);
        }
        __syncthreads();
        const int r = warp, d = d0 + lane;
        if (r < nrows && d < D) {
            float v = 0.f;
#pragma unroll
            for (int k = 0; k < 8; ++k) v += red[(k * 8 + r) * 32 + lane];
            const int gr = r0 + r;
            out[((int64_t)(gr / group) * Hr + p * group + gr % group) * D + d] = v;
        }
        return;
    }
    const int d = d0 + lane;
    if (d < D) {
        for (int r = warp; r < nrows; r += 8) {
            float v = 0.f;
            for (int l = 0; l < width; ++l) v = fmaf(cs[r * width + l], wp[(int64_t)l * D + d], v);
            const int gr = r0 + r;
            out[((int64_t)(gr / group) * Hr + p * group + gr % group) * D + d] = v;
        }
    }
}

cudaError_t launch_project_rows(const float* rows, void* const* rows_table, int rows_index,
                                size_t rows_offset, int B, int Hr, int width, const float* w,
                                int proj_heads, int D, float* out, cudaStream_t st) {
    const int group = Hr / proj_heads;
    // 32 or more rows per weight: a tiled GEMM reads each weight once per
    // 64-row tile, where the row-group kernel below re-reads it every 8 rows
    // (GQA write_attend, 8192 rows of width 256: 100 us per call).
    if (!rows_table && (int64_t)B * group >= 32 && rows_gemm_supported(rows, w, out, width, D))
        return launch_rows_gemm(rows, w, false, out, B, Hr, proj_heads, width, D, st);
    const size_t smem = (size_t)width * 8 * 4 + 8 * 8 * 32 * 4;
    cudaError_t e = cudaFuncSetAttribute(project_rows_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    dim3 grid(proj_heads, (D + 31) / 32, (B * group + 7) / 8);
    project_rows_kernel<<<grid, 256, smem, st>>>(rows, rows_table, rows_index, rows_offset, B, Hr,
                                                 width, w, proj_heads, D, out);
    return cudaGetLastError();
}

// Split-K combine: merge_rows (items -> normalised rows), then, with a
// projection, project_rows (rows -> out).
cudaError_t launch_combine(DecodeWorkspace ws, const int32_t* seq_item_begin, int B, int Hq,
                           int width, const float* w, int proj_heads, int D, float* out,
                           float* lse, cudaStream_t st) {
    if (!w) proj_heads = Hq;
    float* dst = w ? ws.row_ctx : out;
    const int64_t rows = (int64_t)B * Hq;
    if ((width & 7) == 0)
        merge_rows_kernel<8, 64><<<(unsigned)((rows + 3) / 4), 256, 0, st>>>(
            ws, seq_item_begin, B, Hq, width, dst, lse);
    else if ((width & 3) == 0)
        merge_rows_kernel<4, 128><<<(unsigned)((rows + 1) / 2), 256, 0, st>>>(
            ws, seq_item_begin, B, Hq, width, dst, lse);
    else
        merge_rows_kernel<1, 128><<<(unsigned)((rows + 1) / 2), 256, 0, st>>>(
            ws, seq_item_begin, B, Hq, width, dst, lse);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess || !w) return e;
    return launch_project_rows(ws.row_ctx, nullptr, 0, 0, B, Hq, width, w, proj_heads, D, out,
                               st);
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
