// plkv_decode_tc.cu -- tensor-core (tcgen05) split-K partial pass of the
// direct paged latent decode for the absorbed-MLA shapes: 128 query heads
// sharing one latent row of 576 columns (512 value columns + 64 RoPE
// columns), FP16 operands, FP32 accumulation in tensor memory.
//
// Same contract as the exact partial pass (plkv_decode_exact.cu): every work
// item (sequence, block range) emits per head the running max m (natural-log
// units), the sum l of exp(score - m) and the unnormalised latent context
// sum_t exp(score_t - m) L_t[:512]; the shared combine pass merges items and
// applies W_uv.  Scores are (L . q_lat) * scale as in lib.rs:1033-1041.
//
// Work split: a cluster of two CTAs (a tcgen05 CTA pair) processes one item
// in tiles of 64 tokens.  CTA r owns query heads [64r, 64r+64).
//   S = Q . L^T  : cta_group::2 MMA, M = 128 heads, N = 64 tokens, K = 576.
//                  CTA r supplies its heads' Q and tokens [32r, 32r+32) of L;
//                  TMEM of CTA r receives its 64 heads x 64 tokens (32 cols).
//   O += P . V   : cta_group::2 MMA, M = 128 heads, N = 256 value columns
//                  (two instructions), K = 64 tokens.  CTA r supplies its
//                  heads' P and value columns {0,1,4,5} (r = 0) or {2,3,6,7}
//                  (r = 1) in 64-column blocks; TMEM of CTA r holds its 64
//                  heads x 512 columns in 256 columns.
// Because the two MMAs need different slices of the tile at identical
// shared-memory offsets in both CTAs, each CTA loads its own token half of
// all nine 64-column blocks ("K region") and both token halves of its four
// value blocks ("V region"): 17 TMA boxes of 32 rows x 64 columns per tile.
//
// Softmax runs in the log2 domain (the query is pre-scaled by
// scale * log2(e)).  The running max is updated lazily: probabilities are
// taken against a stale max until a tile's max exceeds it by more than 8
// (probabilities stay <= 2^8 in FP16); only then is the accumulated O
// rescaled in TMEM.  The two threads that share a head (token halves) agree on
// every decision through shared memory, and TMEM lane = head, so no
// exchange between the two CTAs is needed.
//
// Every barrier wait is bounded (1 s): on expiry the kernel records
// PLKV_FLAG_TIMEOUT, abandons the item, releases its tensor memory and exits.
#include <cudaTypedefs.h>

#include <mutex>

#include "plkv_sm100.cuh"

namespace plkv {
namespace tc {

constexpr int kHeads = 128;
constexpr int kHeadsPerCta = 64;
constexpr int kLatent = 576;
constexpr int kValue = 512;
constexpr int kTile = 64;
constexpr int kKBlocks = kLatent / 64;                  // 9
constexpr uint32_t kBox = 32 * 128;                      // 32 rows x 64 FP16 = 4 KiB
constexpr uint32_t kQBytes = kKBlocks * kHeadsPerCta * 128;  // 72 KiB
constexpr uint32_t kKRegion = kKBlocks * kBox;           // 36 KiB
constexpr uint32_t kVRegion = 2 * 4 * kBox;              // 32 KiB
constexpr uint32_t kStageBytes = kKRegion + kVRegion;    // 68 KiB
constexpr int kStages = 2;
constexpr uint32_t kPBytes = kHeadsPerCta * kTile * 2;   // 8 KiB
constexpr uint32_t kQOff = 0;
constexpr uint32_t kStageOff = kQOff + kQBytes;
constexpr uint32_t kPOff = kStageOff + kStages * kStageBytes;
constexpr uint32_t kMiscOff = kPOff + 2 * kPBytes;       // 229376
constexpr uint32_t kMiscBytes = 2048;
constexpr uint32_t kSmemBytes = kMiscOff + kMiscBytes;   // 231424
constexpr uint32_t kTxBytes = 2u * 17u * kBox;           // both CTAs, one tile
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemO = 64;                          // S buffers at 0 and 32
constexpr float kTau = 8.f;
constexpr float kLn2 = 0.6931471805599453f;

// Misc region offsets.
constexpr uint32_t kBarFull = 0, kBarKEmpty = 16, kBarSFull = 32, kBarPFull = 48, kBarODone = 64;
constexpr uint32_t kTmemSlot = 80, kAbort = 84, kRedMax = 128, kRedSum = 128 + 2 * 128 * 4;

static_assert(kSmemBytes <= 232448, "shared memory budget");
static_assert(kRedSum + 128 * 4 <= kMiscBytes, "misc region");

__device__ __forceinline__ void named_sync_softmax() {
    asm volatile("bar.sync 1, 128;" ::: "memory");
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(256, 1)
latent_partial_tc_kernel(const __grid_constant__ CUtensorMap tmap, const float* __restrict__ q_lat,
                         float qscale, int bs, const int32_t* __restrict__ tables,
                         int64_t max_blocks, int64_t num_physical,
                         const int32_t* __restrict__ seq_lens,
                         const plkv_work_item* __restrict__ items, DecodeWorkspace ws,
                         int32_t* flags) {
    using namespace sm100;
    extern __shared__ __align__(1024) uint8_t smem[];
    const uint32_t sbase = smem_u32(smem);
    if (sbase & 1023u) {  // identical in both CTAs: both leave before any cluster operation
        if (threadIdx.x == 0) set_flag(flags, PLKV_FLAG_TIMEOUT);
        return;
    }
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const int item = blockIdx.x >> 1;
    uint8_t* misc = smem + kMiscOff;
    const uint32_t mbase = sbase + kMiscOff;
    const uint32_t bar_full = mbase + kBarFull, bar_kempty = mbase + kBarKEmpty;
    const uint32_t bar_sfull = mbase + kBarSFull, bar_pfull = mbase + kBarPFull;
    const uint32_t bar_odone = mbase + kBarODone;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(misc + kAbort);
    float* red_max = reinterpret_cast<float*>(misc + kRedMax);
    float* red_sum = reinterpret_cast<float*>(misc + kRedSum);

    if (tid == 0) {
        for (int i = 0; i < 2; ++i) {
            mbar_init(bar_full + 8 * i, 1);
            mbar_init(bar_kempty + 8 * i, 1);
            mbar_init(bar_sfull + 8 * i, 1);
            mbar_init(bar_pfull + 8 * i, 8);  // 4 softmax warps x 2 CTAs
            mbar_init(bar_odone + 8 * i, 1);
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc_pair(sbase + kMiscOff + kTmemSlot, kTmemCols);
        tmem_relinquish_pair();
    }
    if (warp == 0 && lane == 0) prefetch_tensormap(&tmap);

    // Item geometry (same in every thread).
    const plkv_work_item it = items[item];
    const int b = it.seq;
    const int64_t cap = max_blocks * (int64_t)bs;
    int len = seq_lens[b];
    if (len < 0 || len > cap) {
        if (tid == 0 && leader) set_flag(flags, PLKV_FLAG_BAD_LENGTH);
        len = len < 0 ? 0 : (int)cap;
    }
    const int t_begin = it.block_begin * bs;
    const int t_end = max(t_begin, min(it.block_end * bs, len));
    const int n_tiles = (t_end - t_begin + kTile - 1) / kTile;

    // Q of this CTA's 64 heads, scaled into log2 units, FP16, 128-byte swizzle:
    // nine atoms of [64 heads x 64 columns].
    {
        const float* qsrc = q_lat + ((int64_t)b * kHeads + kHeadsPerCta * rank) * kLatent;
        for (int i = tid; i < kHeadsPerCta * (kLatent / 4); i += 256) {
            const int r = i / (kLatent / 4), col = (i - r * (kLatent / 4)) * 4;
            const float4 v = __ldg(reinterpret_cast<const float4*>(qsrc + (int64_t)r * kLatent + col));
            const __half2 h01 = __floats2half2_rn(v.x * qscale, v.y * qscale);
            const __half2 h23 = __floats2half2_rn(v.z * qscale, v.w * qscale);
            uint2 pk;
            pk.x = *reinterpret_cast<const uint32_t*>(&h01);
            pk.y = *reinterpret_cast<const uint32_t*>(&h23);
            *reinterpret_cast<uint2*>(smem + kQOff + (col >> 6) * (kHeadsPerCta * 128) +
                                      sw128_offset(r, col & 63)) = pk;
        }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    cluster_sync();
    tc_fence_after();
    const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(misc + kTmemSlot);

    if (warp == 0) {
        // ------------------------------------------------------ TMA producer
        const uint64_t pol = policy_evict_first();
        const uint32_t full_leader0 = mapa(bar_full, 0), full_leader1 = mapa(bar_full + 8, 0);
        for (int j = 0; j < n_tiles; ++j) {
            const int st = j & 1;
            int y = 0;
            if (lane < 2) {
                int hs = t_begin + kTile * j + 32 * lane;
                if (hs >= t_end) hs = t_begin + kTile * j;  // half beyond the end: reuse half 0
                const int lb = hs / bs;
                int32_t phys = tables[(int64_t)b * max_blocks + lb];
                if (phys < 0 || phys >= num_physical) {
                    set_flag(flags, PLKV_FLAG_BAD_BLOCK);
                    phys = 0;
                }
                y = phys * bs + (hs - lb * bs);
            }
            const int y0 = __shfl_sync(0xffffffffu, y, 0);
            const int y1 = __shfl_sync(0xffffffffu, y, 1);
            int ok = 1;
            if (lane == 0) {
                if (j >= 2) ok = mbar_wait(bar_kempty + 8 * st, ((j - 2) >> 1) & 1, flags, abort_flag);
                if (ok) {
                    if (leader) mbar_arrive_expect_tx(bar_full + 8 * st, kTxBytes);
                    const uint32_t stage = sbase + kStageOff + st * kStageBytes;
                    const uint32_t fb = st ? full_leader1 : full_leader0;
                    const int yown = rank ? y1 : y0;
                    for (int c = 0; c < kKBlocks; ++c)
                        tma_load_2d_pair(stage + c * kBox, &tmap, c * 64, yown, fb, pol);
                    for (int h = 0; h < 2; ++h)
                        for (int s = 0; s < 4; ++s) {
                            const int cb = (s >> 1) * 4 + (s & 1) + 2 * (int)rank;
                            tma_load_2d_pair(stage + kKRegion + h * 4 * kBox + s * kBox, &tmap,
                                             cb * 64, h ? y1 : y0, fb, pol);
                        }
                }
            }
            if (!__shfl_sync(0xffffffffu, ok, 0)) break;
        }
    } else if (warp == 1) {
        // ---------------------------------------------- MMA issue (leader)
        if (leader && lane == 0 && n_tiles > 0) {
            const uint32_t id_s = idesc_f16(128, 64, false, false);
            const uint32_t id_o = idesc_f16(128, 256, false, true);
            auto issue_s = [&](int j) -> bool {
                const int st = j & 1;
                if (!mbar_wait(bar_full + 8 * st, (j >> 1) & 1, flags, abort_flag)) return false;
                tc_fence_after();
                const uint32_t kreg = sbase + kStageOff + st * kStageBytes;
                const uint32_t d = tmem + 32 * st;
#pragma unroll 4
                for (int k = 0; k < kKBlocks * 4; ++k) {
                    const uint64_t a = sdesc_sw128(sbase + kQOff + (k >> 2) * (kHeadsPerCta * 128) +
                                                       (k & 3) * 32, 16, 1024);
                    const uint64_t bd = sdesc_sw128(kreg + (k >> 2) * kBox + (k & 3) * 32, 16, 1024);
                    mma_pair_f16(d, a, bd, id_s, k > 0 ? 1u : 0u);
                }
                mma_commit_pair(bar_sfull + 8 * st, 0x3);
                return true;
            };
            bool ok = issue_s(0);
            if (ok && n_tiles > 1) ok = issue_s(1);
            for (int j = 0; ok && j < n_tiles; ++j) {
                const int st = j & 1;
                if (!mbar_wait(bar_pfull + 8 * st, (j >> 1) & 1, flags, abort_flag)) break;
                tc_fence_after();
                const uint32_t vreg = sbase + kStageOff + st * kStageBytes + kKRegion;
                const uint32_t preg = sbase + kPOff + st * kPBytes;
#pragma unroll
                for (int i = 0; i < 2; ++i)
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const uint64_t a = sdesc_sw128(preg + k * 32, 16, 1024);
                        const uint64_t bd = sdesc_sw128(
                            vreg + (k >> 1) * 4 * kBox + (k & 1) * 2048 + i * 2 * kBox, kBox, 1024);
                        mma_pair_f16(tmem + kTmemO + 128 * i, a, bd, id_o,
                                     (j > 0 || k > 0) ? 1u : 0u);
                    }
                mma_commit_pair(bar_odone + 8 * st, 0x3);
                mma_commit_pair(bar_kempty + 8 * st, 0x3);
                if (j + 2 < n_tiles) ok = issue_s(j + 2);
            }
        }
        __syncwarp();
    } else if (warp >= 4) {
        // ------------------------------------------- softmax and epilogue
        const int t = tid - 128;            // TMEM lane
        const int hl = t & 63, th = t >> 6; // head within the CTA, token / column half
        const uint32_t lane_base = static_cast<uint32_t>((warp - 4) * 32) << 16;
        float m_use = -INFINITY, l = 0.f;
        bool ok = true;
        // Every softmax warp runs all n_tiles iterations and reaches every
        // named barrier; after a failed wait it only skips the work.
        for (int j = 0; j < n_tiles; ++j) {
            const int st = j & 1;
            const int vc = min(kTile, t_end - (t_begin + kTile * j));
            if (ok)
                ok = __all_sync(0xffffffffu,
                                mbar_wait(bar_sfull + 8 * st, (j >> 1) & 1, flags, abort_flag));
            float s[32];
            if (ok) {
                tc_fence_after();
                tmem_ld32(tmem + lane_base + 32 * st, s);
                tmem_wait_ld();
            } else {
#pragma unroll
                for (int i = 0; i < 32; ++i) s[i] = -INFINITY;
            }
            float mx = -INFINITY;
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                if (th * 32 + i >= vc) s[i] = -INFINITY;
                mx = fmaxf(mx, s[i]);
            }
            red_max[st * 128 + t] = mx;
            named_sync_softmax();
            const float mt = fmaxf(mx, red_max[st * 128 + (t ^ 64)]);
            const float m_new = fmaxf(m_use, mt);
            const bool resc = m_new > m_use + kTau;
            float alpha = 1.f;
            if (resc) {
                alpha = (m_use == -INFINITY) ? 0.f : exp2f(m_use - m_new);
                m_use = m_new;
                l *= alpha;
            }
            uint32_t packed[16];
            float psum = 0.f;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const float p0 = (m_use == -INFINITY) ? 0.f : exp2f(s[2 * i] - m_use);
                const float p1 = (m_use == -INFINITY) ? 0.f : exp2f(s[2 * i + 1] - m_use);
                psum += p0 + p1;
                const __half2 h = __floats2half2_rn(p0, p1);
                packed[i] = *reinterpret_cast<const uint32_t*>(&h);
            }
            l += psum;
            if (ok && j >= 2)  // P buffer `st` is free once O of tile j-2 completed
                ok = __all_sync(0xffffffffu, mbar_wait(bar_odone + 8 * st, ((j - 2) >> 1) & 1,
                                                       flags, abort_flag));
            if (ok && __any_sync(0xffffffffu, resc && j > 0)) {
                const int jp = j - 1;  // rescale O accumulated through tile j-1
                ok = __all_sync(0xffffffffu, mbar_wait(bar_odone + 8 * (jp & 1), (jp >> 1) & 1,
                                                       flags, abort_flag));
                if (ok) {
                    tc_fence_after();
#pragma unroll 1
                    for (int u = 0; u < 8; ++u) {
                        float o[32];
                        tmem_ld32(tmem + lane_base + kTmemO + 32 * u, o);
                        tmem_wait_ld();
#pragma unroll
                        for (int e = 0; e < 32; ++e) o[e] *= alpha;
                        tmem_st32(tmem + lane_base + kTmemO + 32 * u, o);
                    }
                    tmem_wait_st();
                }
            }
            if (!ok) continue;
            uint8_t* prow = smem + kPOff + st * kPBytes + (hl >> 3) * 1024 + (hl & 7) * 128;
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const uint32_t chunk = static_cast<uint32_t>((th * 4 + u) ^ (hl & 7));
                *reinterpret_cast<uint4*>(prow + chunk * 16) =
                    make_uint4(packed[4 * u], packed[4 * u + 1], packed[4 * u + 2], packed[4 * u + 3]);
            }
            if (vc < kTile) {
                // Rows past the end of the item: zero their value rows so that
                // p = 0 times whatever the pool holds there stays 0.
                uint8_t* vreg = smem + kStageOff + st * kStageBytes + kKRegion;
                const int rows = kTile - vc;
                for (int idx = t; idx < rows * 4 * 8; idx += 128) {
                    const int tok = vc + idx / 32, rem = idx % 32, s4 = rem >> 3, c16 = rem & 7;
                    const int h = tok >> 5, rr = tok & 31;
                    *reinterpret_cast<uint4*>(vreg + h * 4 * kBox + s4 * kBox + (rr >> 3) * 1024 +
                                              (rr & 7) * 128 + c16 * 16) = make_uint4(0, 0, 0, 0);
                }
            }
            fence_proxy_async_smem();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(mapa(bar_pfull + 8 * st, 0));
        }
        if (ok && n_tiles > 0) {
            const int jl = n_tiles - 1;
            ok = __all_sync(0xffffffffu,
                            mbar_wait(bar_odone + 8 * (jl & 1), (jl >> 1) & 1, flags, abort_flag));
        }
        red_sum[t] = l;
        named_sync_softmax();
        const float l_tot = l + red_sum[t ^ 64];
        const int64_t row = (int64_t)item * kHeads + kHeadsPerCta * rank + hl;
        if (th == 0) {
            ws.part_m[row] = (ok && m_use != -INFINITY) ? m_use * kLn2 : -INFINITY;
            ws.part_l[row] = ok ? l_tot : 0.f;
        }
        float* dst = ws.part_ctx + row * kValue;
        const bool have = ok && n_tiles > 0;
        if (have) tc_fence_after();
#pragma unroll 1
        for (int u = 0; u < 8; ++u) {
            float o[32];
            if (have) {
                tmem_ld32(tmem + lane_base + kTmemO + 32 * u, o);
                tmem_wait_ld();
            } else {
#pragma unroll
                for (int e = 0; e < 32; ++e) o[e] = 0.f;
            }
            const int col = (u >> 2) * 256 + th * 128 + (u & 3) * 32;
#pragma unroll
            for (int e = 0; e < 32; e += 4)
                *reinterpret_cast<float4*>(dst + col + e) = make_float4(o[e], o[e + 1], o[e + 2], o[e + 3]);
        }
    }

    // Teardown: every role is done with shared and tensor memory.
    tc_fence_before();
    __syncthreads();
    cluster_sync();
    tc_fence_after();
    if (warp == 1) tmem_dealloc_pair(tmem, kTmemCols);
}

// Flag word used when the caller passes none: a wait that gives up must be
// visible to the other CTA of the pair so that its waits end at once too.
__device__ int32_t g_tc_flags;

static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
static std::once_flag g_encode_once;

static bool load_encode() {
    std::call_once(g_encode_once, [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    });
    return g_encode != nullptr;
}

}  // namespace tc

bool tc_supported(const plkv_latent_decode_args& a) {
    return a.q_heads == tc::kHeads && a.latent_dim == tc::kLatent && a.value_dim == tc::kValue &&
           a.block_size % 32 == 0 && !a.scores && !a.probs &&
           a.num_physical * (int64_t)a.block_size < (1ll << 31) &&
           (reinterpret_cast<uintptr_t>(a.cache) & 15) == 0 &&
           (reinterpret_cast<uintptr_t>(a.q_lat) & 15) == 0;
}

cudaError_t launch_latent_partial_tc(const plkv_latent_decode_args& a, DecodeWorkspace ws,
                                     cudaStream_t st) {
    if (!tc::load_encode()) return cudaErrorNotSupported;
    CUtensorMap map;
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(a.latent_dim),
                          static_cast<cuuint64_t>(a.num_physical) * a.block_size};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(a.latent_dim) * 2};
    cuuint32_t box[2] = {64, 32};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = tc::g_encode(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                              const_cast<uint16_t*>(a.cache), dims, strides, box, estr,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(tc::latent_partial_tc_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)tc::kSmemBytes);
    if (e != cudaSuccess) return e;
    int32_t* flags = a.err_flags;
    if (!flags) {
        e = cudaGetSymbolAddress(reinterpret_cast<void**>(&flags), tc::g_tc_flags);
        if (e != cudaSuccess) return e;
    }
    tc::latent_partial_tc_kernel<<<2 * a.n_items, 256, tc::kSmemBytes, st>>>(
        map, a.q_lat, a.scale * 1.4426950408889634f, a.block_size, a.block_tables, a.max_blocks,
        a.num_physical, a.seq_lens, a.items, ws, flags);
    return cudaGetLastError();
}

}  // namespace plkv
