// plkv_rows_gemm.cu -- the per-KV-head projections of the GQA shapes as
// batched FP32 GEMMs on the CUDA cores (the exact mode's FP32 arithmetic).
//
// For KV head g the G = Hq / KV query heads of every sequence form M = B * G
// rows (b, j) of head h = g * G + j; row (b, j) of an [B, Hq, K] operand lies
// at ((b * Hq + h) * K).  Two projections have this shape:
//   query -> latent (lib.rs:1026-1032):  q_lat[b, h, :] = W_k[g] q[b, h, :],
//       A = q [B, Hq, D], B[k = d][n = l] = W_k[g, l, d]     (B transposed)
//   latent context -> value (lib.rs:1062-1071): out[b, h, :] = ctx[b, h, :] W_v[g],
//       A = ctx [B, Hq, L], B[k = l][n = d] = W_v[g, l, d]
// and the MLA value projection W_uv with G = 1 and one weight per head.
//
// grid = (ceil(M / 64), ceil(N / 64), heads), block = 256: a 64 x 64 output
// tile per CTA, K in chunks of 16 through shared memory (the next chunk held
// in registers while the current one is multiplied), 4 x 4 outputs per
// thread from two 16-byte shared-memory reads per k.  Every output is one
// FP32 accumulator summed in increasing k, so results do not depend on the
// launch shape.  Requires K and N multiples of 4 and 16-byte aligned
// operands (the callers fall back to their own kernels otherwise).
#include "plkv_common.cuh"

namespace plkv {
namespace {

constexpr int kBM = 64, kBN = 64, kBK = 16;

template <bool kBTrans>
__global__ void __launch_bounds__(256)
rows_gemm_kernel(const float* __restrict__ a, const float* __restrict__ w, float* __restrict__ c,
                 int B, int Hq, int G, int K, int N) {
    __shared__ __align__(16) float as[2][kBK][kBM];   // A tile, k-major
    __shared__ __align__(16) float bs[2][kBK][kBN];   // B tile, k-major
    const int g = blockIdx.z, m0 = blockIdx.x * kBM, n0 = blockIdx.y * kBN;
    const int M = B * G;
    const int tid = threadIdx.x, tm = tid >> 4, tn = tid & 15;
    const float* wg = w + (int64_t)g * K * N;

    // A loads: thread -> row ar, four consecutive k at ak4 (the same row for
    // every chunk, so its address is formed once).
    const int ar = tid >> 2, ak4 = (tid & 3) * 4;
    const float* arow = nullptr;
    {
        const int m = m0 + ar;
        if (m < M) {
            const int b = m / G, j = m - b * G;
            arow = a + ((int64_t)b * Hq + g * G + j) * K;
        }
    }
    // B loads: (not transposed) row k = tid / 16 of the chunk, four
    // consecutive n at 4 (tid % 16); (transposed) column n = tid / 4, four
    // consecutive k at 4 (tid % 4).
    const int bk = kBTrans ? (tid & 3) * 4 : tid >> 4;
    const int bn = kBTrans ? tid >> 2 : (tid & 15) * 4;

    auto load_a = [&](int k0) -> float4 {
        const int k = k0 + ak4;
        return (arow && k < K) ? *reinterpret_cast<const float4*>(arow + k)
                               : make_float4(0.f, 0.f, 0.f, 0.f);
    };
    auto load_b = [&](int k0) -> float4 {
        if (kBTrans) {
            const int n = n0 + bn, k = k0 + bk;
            return (n < N && k < K) ? *reinterpret_cast<const float4*>(wg + (int64_t)n * K + k)
                                    : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        const int k = k0 + bk, n = n0 + bn;
        return (k < K && n < N) ? *reinterpret_cast<const float4*>(wg + (int64_t)k * N + n)
                                : make_float4(0.f, 0.f, 0.f, 0.f);
    };
    auto store = [&](int buf, const float4& va, const float4& vb) {
        as[buf][ak4 + 0][ar] = va.x;
        as[buf][ak4 + 1][ar] = va.y;
        as[buf][ak4 + 2][ar] = va.z;
        as[buf][ak4 + 3][ar] = va.w;
        if (kBTrans) {
            bs[buf][bk + 0][bn] = vb.x;
            bs[buf][bk + 1][bn] = vb.y;
            bs[buf][bk + 2][bn] = vb.z;
            bs[buf][bk + 3][bn] = vb.w;
        } else {
            *reinterpret_cast<float4*>(&bs[buf][bk][bn]) = vb;
        }
    };

    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int k = 0; k < 4; ++k) acc[i][k] = 0.f;

    float4 va = load_a(0), vb = load_b(0);
    store(0, va, vb);
    __syncthreads();
    int buf = 0;
    for (int k0 = 0; k0 < K; k0 += kBK) {
        const bool more = k0 + kBK < K;
        if (more) {
            va = load_a(k0 + kBK);
            vb = load_b(k0 + kBK);
        }
#pragma unroll
        for (int kk = 0; kk < kBK; ++kk) {
            const float4 x = *reinterpret_cast<const float4*>(&as[buf][kk][4 * tm]);
            const float4 y = *reinterpret_cast<const float4*>(&bs[buf][kk][4 * tn]);
            const float xa[4] = {x.x, x.y, x.z, x.w}, ya[4] = {y.x, y.y, y.z, y.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int k = 0; k < 4; ++k) acc[i][k] = fmaf(xa[i], ya[k], acc[i][k]);
        }
        if (more) {
            store(buf ^ 1, va, vb);
            __syncthreads();
            buf ^= 1;
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int m = m0 + 4 * tm + i;
        const int n = n0 + 4 * tn;
        if (m >= M || n >= N) continue;
        const int b = m / G, j = m - b * G;
        *reinterpret_cast<float4*>(c + ((int64_t)b * Hq + g * G + j) * N + n) =
            make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
    }
}

}  // namespace

bool rows_gemm_supported(const float* a, const float* w, const float* c, int K, int N) {
    const auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    return K > 0 && N > 0 && (K & 3) == 0 && (N & 3) == 0 && al(a) && al(w) && al(c);
}

cudaError_t launch_rows_gemm(const float* a, const float* w, bool w_transposed, float* c, int B,
                             int Hq, int heads, int K, int N, cudaStream_t st) {
    const int G = Hq / heads, M = B * G;
    if (M <= 0) return cudaSuccess;
    dim3 grid((M + kBM - 1) / kBM, (N + kBN - 1) / kBN, heads);
    if (w_transposed)
        rows_gemm_kernel<true><<<grid, 256, 0, st>>>(a, w, c, B, Hq, G, K, N);
    else
        rows_gemm_kernel<false><<<grid, 256, 0, st>>>(a, w, c, B, Hq, G, K, N);
    return cudaGetLastError();
}

}  // namespace plkv
