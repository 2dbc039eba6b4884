// plkv_outproj_tc.cu -- W_o output projection on the tensor cores:
// out[batch, out_dim] = x[batch, in_dim] W_o[in_dim, out_dim] with tcgen05
// kind::tf32 MMAs on the FP32 W_o as stored (the tensor copy rounds both
// operands to TF32, round to nearest), FP32 accumulation in tensor memory.
// (Extension: the reference stops at the per-head context.)
//
// The product reads W_o once; at the workloads' sizes (470 MB of W_o for 64
// rows) it is bound by HBM, not by the tensor pipe: a CTA owns 256 output
// columns x a contiguous range of in_dim (split-K) x 128 batch rows, streams
// W_o tiles of 32 rows x 256 columns (one TMA box, a 1 KiB run per row)
// through a four-stage ring and issues per stage four M = 128, N = 256, K = 8
// MMAs (x rows past the batch are zero-filled by the copy).  The partial sums
// of the K splits go to the workspace and are added in a fixed order by the
// reduction kernel of plkv_combine.cu.
//
// Operands in shared memory: x is K-major with the 128-byte swizzle (A: 128
// rows x 32 FP32 per stage); W_o is MN-major, for which 32-bit operands take
// the 128-byte swizzle of 32-byte atoms (B: 8 blocks of 32 columns x 32 rows,
// 32-byte chunks permuted across 4-row groups; LBO = 4 KiB between column
// blocks, SBO = 512 B between 4-row groups; descriptor layout type 1).  Warp 0
// loads, warp 1 allocates tensor memory and issues, warps 2..5 read the
// accumulator (each its TMEM lane quarter) and store the partial sums.  Every
// wait is bounded (1 s, PLKV_FLAG_TIMEOUT).
#include <cudaTypedefs.h>

#include <algorithm>

#include "plkv_sm100.cuh"

namespace plkv {
namespace wo {

constexpr int kN = 256;          // output columns per CTA
constexpr int kKc = 32;          // in_dim rows per stage
constexpr int kM = 128;          // batch rows per CTA
constexpr int kStages = 4;
constexpr uint32_t kWBytes = kKc * kN * 4;     // 32 KiB
constexpr uint32_t kXBytes = kM * kKc * 4;     // 16 KiB
constexpr uint32_t kStageBytes = kWBytes + kXBytes;
constexpr uint32_t kMiscOff = kStages * kStageBytes;
constexpr uint32_t kSmemBytes = kMiscOff + 1024;
constexpr uint32_t kTmemCols = 256;

enum : uint32_t { kBarFull = 0, kBarEmpty = 8 * kStages, kBarDone = 16 * kStages,
                  kTmemSlot = kBarDone + 8, kAbort = kTmemSlot + 4 };

// kind::tf32, D FP32, A K-major, B MN-major, M = 128, N = 256.
constexpr uint32_t kIdesc = (1u << 4) | (2u << 7) | (2u << 10) | (1u << 16) |
                            (static_cast<uint32_t>(kN >> 3) << 17) |
                            (static_cast<uint32_t>(kM >> 4) << 24);

// Shared-memory descriptor of an MN-major operand of 32-bit elements with the
// 128-byte swizzle of 32-byte atoms (layout type 1), version 1.
__device__ __forceinline__ uint64_t sdesc_mn_sw128_32b(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4) |
           (static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16) |
           (static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (1ull << 61);
}

__device__ __forceinline__ void tmem_alloc1(uint32_t dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(dst_smem), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tmem_relinquish1() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc1(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;"
                 ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void mma_commit1(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tma_2d(uint32_t dst, const CUtensorMap* map, int x, int y,
                                       uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
        : "memory");
}
__device__ __forceinline__ void tma_3d(uint32_t dst, const CUtensorMap* map, int x, int y, int z,
                                       uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4}], [%5];"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(bar)
        : "memory");
}

// grid = (ceil(N / 256), k_splits, ceil(B / 128)), block = 192.
__global__ void __launch_bounds__(192, 1)
out_proj_tf32_kernel(const __grid_constant__ CUtensorMap w_map,
                     const __grid_constant__ CUtensorMap x_map, float* __restrict__ partial,
                     int B, int N, int n_chunks, int32_t* ctl, int32_t* flags) {
    using namespace sm100;
    extern __shared__ __align__(1024) uint8_t smem[];
    const uint32_t sbase = smem_u32(smem);
    if (sbase & 1023u) {
        if (threadIdx.x == 0) set_flag(flags, PLKV_FLAG_TIMEOUT);
        return;
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * kN, split = blockIdx.y, m0 = blockIdx.z * kM;
    const int c_begin = (int)((int64_t)n_chunks * split / gridDim.y);
    const int c_end = (int)((int64_t)n_chunks * (split + 1) / gridDim.y);
    const uint32_t mb = sbase + kMiscOff;
    uint8_t* misc = smem + kMiscOff;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(misc + kAbort);
    const WaitCtx wc{flags, ctl, abort_flag};
    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(mb + kBarFull + 8 * s, 1);
            mbar_init(mb + kBarEmpty + 8 * s, 1);
        }
        mbar_init(mb + kBarDone, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc1(mb + kTmemSlot, kTmemCols);
        tmem_relinquish1();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tensormap(&w_map);
        prefetch_tensormap(&x_map);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(misc + kTmemSlot);
    const int nk = c_end - c_begin;

    if (warp == 0) {
        if (lane == 0) {
            for (int i = 0; i < nk; ++i) {
                const int s = i % kStages;
                if (i >= kStages && !mbar_wait(mb + kBarEmpty + 8 * s, ((i / kStages) - 1) & 1, wc))
                    break;
                const uint32_t dst = sbase + s * kStageBytes;
                mbar_arrive_expect_tx(mb + kBarFull + 8 * s, kStageBytes);
                const int k0 = (c_begin + i) * kKc;
                tma_3d(dst, &w_map, 0, k0, n0 / 32, mb + kBarFull + 8 * s);
                tma_2d(dst + kWBytes, &x_map, k0, m0, mb + kBarFull + 8 * s);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            bool ok = true;
            for (int i = 0; i < nk; ++i) {
                const int s = i % kStages;
                if (!(ok = mbar_wait(mb + kBarFull + 8 * s, (i / kStages) & 1, wc))) break;
                tc_fence_after();
                const uint32_t wst = sbase + s * kStageBytes;
                const uint32_t xst = wst + kWBytes;
#pragma unroll
                for (int kq = 0; kq < kKc / 8; ++kq) {
                    const uint64_t a = sdesc_sw128(xst + kq * 32, 16, 1024);
                    const uint64_t b = sdesc_mn_sw128_32b(wst + kq * 1024, kKc * 128, 512);
                    mma_tf32(tmem, a, b, kIdesc, (i > 0 || kq > 0) ? 1u : 0u);
                }
                mma_commit1(mb + kBarEmpty + 8 * s);
            }
            if (ok) mma_commit1(mb + kBarDone);
        }
        __syncwarp();
    } else {
        // Accumulator -> partial sums: warp w reads TMEM lanes of quarter w % 4.
        const int q = warp & 3;
        const bool ok = nk > 0 ? __all_sync(0xffffffffu, mbar_wait(mb + kBarDone, 0, wc)) : true;
        const int row = m0 + 32 * q + lane;
        float* dst = partial + ((int64_t)split * B + row) * N + n0;
        if (ok) tc_fence_after();
#pragma unroll 1
        for (int u = 0; u < kN / 32; ++u) {
            float v[32];
            if (ok && nk > 0) {
                tmem_ld32(tmem + (static_cast<uint32_t>(32 * q) << 16) + 32 * u, v);
                tmem_wait_ld();
            } else {
#pragma unroll
                for (int e = 0; e < 32; ++e) v[e] = 0.f;
            }
            if (row < B) {
                const int c0 = 32 * u;
                if (n0 + c0 + 32 <= N) {
#pragma unroll
                    for (int e = 0; e < 32; e += 4)
                        *reinterpret_cast<float4*>(dst + c0 + e) =
                            make_float4(v[e], v[e + 1], v[e + 2], v[e + 3]);
                } else {
                    for (int e = 0; e < 32; ++e)
                        if (n0 + c0 + e < N) dst[c0 + e] = v[e];
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc1(tmem, kTmemCols);
}

}  // namespace wo

namespace tc {
bool encode_map(CUtensorMap* map, CUtensorMapDataType type, const void* base, int rank,
                const cuuint64_t* dims, const cuuint64_t* strides, const cuuint32_t* box,
                CUtensorMapSwizzle swizzle);
}
__global__ void out_proj_reduce_kernel(const float* __restrict__ partial, float* __restrict__ out,
                                       int S, int64_t BN);

cudaError_t launch_out_proj_tf32(const float* x, const float* w, float* out, int B, int K, int N,
                                 int k_splits, float* partial, int32_t* ctl, int32_t* flags,
                                 cudaStream_t st) {
    CUtensorMap w_map, x_map;
    const cuuint64_t w_dims[3] = {32, (cuuint64_t)K, (cuuint64_t)((N + 31) / 32)};
    const cuuint64_t w_str[2] = {(cuuint64_t)N * 4, 128};
    const cuuint32_t w_box[3] = {32, wo::kKc, wo::kN / 32};
    const cuuint64_t x_dims[2] = {(cuuint64_t)K, (cuuint64_t)B};
    const cuuint64_t x_str[1] = {(cuuint64_t)K * 4};
    const cuuint32_t x_box[2] = {wo::kKc, wo::kM};
    if (!tc::encode_map(&w_map, CU_TENSOR_MAP_DATA_TYPE_TFLOAT32, w, 3, w_dims, w_str, w_box,
                        CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B) ||
        !tc::encode_map(&x_map, CU_TENSOR_MAP_DATA_TYPE_TFLOAT32, x, 2, x_dims, x_str, x_box,
                        CU_TENSOR_MAP_SWIZZLE_128B))
        return cudaErrorInvalidValue;
    cudaError_t e = cudaMemsetAsync(ctl, 0, 4, st);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(wo::out_proj_tf32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)wo::kSmemBytes);
    if (e != cudaSuccess) return e;
    dim3 grid((N + wo::kN - 1) / wo::kN, k_splits, (B + wo::kM - 1) / wo::kM);
    wo::out_proj_tf32_kernel<<<grid, 192, wo::kSmemBytes, st>>>(w_map, x_map, partial, B, N,
                                                                 K / wo::kKc, ctl, flags);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    const int64_t BN = int64_t(B) * N;
    out_proj_reduce_kernel<<<(unsigned)((BN + 255) / 256), 256, 0, st>>>(partial, out, k_splits,
                                                                         BN);
    return cudaGetLastError();
}

}  // namespace plkv
