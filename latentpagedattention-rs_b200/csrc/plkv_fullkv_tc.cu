// plkv_fullkv_tc.cu -- tensor-core (tcgen05) split-K partial pass of the FP16
// full-KV paged GQA decode (the baseline of lib.rs:1147-1269,
// attention_ref.py:172-224) for head_dim 128 and up to 16 query heads per KV
// head.
//
// Same contract as fullkv_partial_exact_kernel (plkv_decode_exact.cu): every
// (work item, KV head g) emits per query head h = g G + i the running max m
// (natural-log units), the sum l of exp(score - m) and the unnormalised
// context sum_t exp(score_t - m) V_t; the shared combine merges the items.
//
// The G query heads of one KV head are too few rows for a tcgen05 tile, so the
// tokens are the rows:
//   S^T = K . Q^T   M = 128 tokens, N = 16 (the G heads, padded), K = 128 dims
//   O^T = V^T . P^T M = 128 dims,   N = 16,                        K = 128 tokens
// both cta_group::1 kind::f16 with FP32 accumulators in tensor memory (S^T
// double-buffered, O^T resident for the item).  K and V are FP16 as stored,
// so only Q and P need care to keep FP32 accuracy: each is split into an FP16
// high part and an FP16 low part (x = hi + lo + O(2^-22 x)) and multiplied
// twice; FP16 x FP16 products are exact in FP32, so scores and context carry
// FP32 accumulation error only (~1e-7 relative; the exact-mode bar is 1e-5).
//
// Data movement: one TMA box per 16 tokens of a block and operand.  A block of
// KV head g is 16 rows x 256 contiguous bytes of the head-major pool (more
// for larger blocks), so the pool is viewed as a 4-D tensor (64 columns, 8
// rows, 2 column halves, 8-row groups): a box of 2 groups lands as
// [group][half][8 rows][128 B] with the 128-byte swizzle, and the 8 chunks of
// a 128-token tile laid side by side put the 8-row groups of each 64-column
// half at a uniform 2 KiB stride -- the SW128 K-major operand layout of K
// (column block h at h x 1 KiB, SBO 2 KiB) and, read as the MN-major A
// operand of O^T, of V (LBO 1 KiB between the halves, SBO 2 KiB).  16 boxes of
// 4 KiB per tile, three 64 KiB stages in flight, issued by one thread (16-byte
// copies from the SM's load-store path reached only ~18 GB/s per SM: too few
// requests in flight).  Chunks past the item's end, or of a table entry outside
// the pool, are read at an out-of-bounds group index and arrive as zeros; the
// rows past the end inside the item's last chunk are zeroed by the softmax
// warps before they release P (0 x garbage must stay 0 in the context MMA).
//
// Softmax: TMEM lane = token; per head a warp-shuffle max over the lanes and
// the four warps through shared memory; log2 domain with a lazily updated
// running max (threshold 8: probabilities stay <= 2^8), O^T rescaled in TMEM
// only when a head's max moved by more than that.
//
// Warps: 0-3 softmax and epilogue, 4 tensor-memory allocation and (lane 0)
// MMA issue, 5 loads.  Every wait is bounded (1 s): on expiry the kernel
// records PLKV_FLAG_TIMEOUT, abandons its work and frees tensor memory.
#include <cudaTypedefs.h>
#include <cuda_fp16.h>

#include "plkv_sm100.cuh"
#include "plkv_tc1.cuh"

namespace plkv {
namespace tc {
bool encode_map(CUtensorMap* map, CUtensorMapDataType type, const void* base, int rank,
                const cuuint64_t* dims, const cuuint64_t* strides, const cuuint32_t* box,
                CUtensorMapSwizzle swizzle);
}
namespace fkv {
using namespace tc1;

constexpr int kTok = 128;        // tokens per tile
constexpr int kD = 128;          // head_dim
constexpr int kN = 16;           // query heads of a KV head, padded
constexpr int kStages = 3;
constexpr uint32_t kHalf = kTok * 128;             // 64 columns x 128 rows: 16 KiB
constexpr uint32_t kTileBytes = 2 * kHalf;          // K or V tile: 32 KiB
constexpr uint32_t kStageBytes = 2 * kTileBytes;    // K + V: 64 KiB
constexpr uint32_t kOpBlock = kN * 128;             // 64 columns x 16 rows: 2 KiB
constexpr uint32_t kOpBytes = 2 * kOpBlock;         // a 16 x 128 FP16 operand: 4 KiB
constexpr uint32_t kKVOff = 0;
constexpr uint32_t kQOff = kKVOff + kStages * kStageBytes;  // Q hi, Q lo
constexpr uint32_t kPOff = kQOff + 2 * kOpBytes;            // [2 buffers][hi, lo]
constexpr uint32_t kMiscOff = kPOff + 4 * kOpBytes;
constexpr uint32_t kMiscBytes = 1024;
constexpr uint32_t kSmemBytes = kMiscOff + kMiscBytes;      // 222208
constexpr uint32_t kTmemCols = 64;
constexpr uint32_t kColS = 0;    // S^T buffers at columns 0 and 16
constexpr uint32_t kColO = 32;   // O^T
constexpr int kThreads = 192;
constexpr int kChunks = kTok / 16;                 // 16-token TMA boxes per tile and operand
constexpr uint32_t kChunkBytes = 16 * 256;         // one box: 2 groups x 2 halves x 8 rows x 128 B
constexpr float kTau = 8.f;
constexpr float kLn2 = 0.6931471805599453f;

enum : uint32_t {
    kBarKVFull = 0,                          // [kStages] TMA: the tile's K and V landed
    kBarKVEmpty = kBarKVFull + 8 * kStages,  // [kStages] MMA commit: S and O of the tile done
    kBarSFull = kBarKVEmpty + 8 * kStages,   // [2] MMA commit: S^T of the tile in TMEM
    kBarPFull = kBarSFull + 16,              // [2] softmax: P of the tile written
    kBarODone = kBarPFull + 16,              // [2] MMA commit: O^T through the tile done
    kTmemSlot = kBarODone + 16,
    kAbort = kTmemSlot + 4,
    kRedMax = 256,                           // [4 warps][16] float
    kRedSum = kRedMax + 256,                 // [4 warps][16] float
    kVote = kRedSum + 256,                   // [4 warps] int: some score above the running max
};
static_assert(kAbort + 4 <= kRedMax, "barriers");
static_assert(kVote + 16 <= kMiscBytes, "misc region");
static_assert(kSmemBytes <= 232448, "shared memory budget");

// Byte offset of element (row, k) of a 16-row FP16 operand stored K-major in
// 128-byte-swizzled 64-column blocks (Q^T's and P^T's rows are the heads).
__device__ __forceinline__ uint32_t op_offset(int row, int k) {
    return (uint32_t)(k >> 6) * kOpBlock + (uint32_t)(row >> 3) * 1024u +
           (uint32_t)(row & 7) * 128u + ((((uint32_t)(k & 63) >> 3) ^ (uint32_t)(row & 7)) << 4) +
           (uint32_t)(k & 7) * 2u;
}

// grid = (n_items, KV heads), block = 224, one CTA per SM (222 KiB).
__global__ void __launch_bounds__(kThreads, 1)
fullkv_partial_tc_kernel(const __grid_constant__ CUtensorMap k_map,
                         const __grid_constant__ CUtensorMap v_map, int64_t n_groups,
                         const float* __restrict__ q, int64_t num_physical, int KV,
                         int bs, int Hq, float scale_log2, const int32_t* __restrict__ tables,
                         int64_t max_blocks, const int32_t* __restrict__ seq_lens,
                         const plkv_work_item* __restrict__ items, DecodeWorkspace ws,
                         int32_t* flags) {
    using namespace sm100;
    extern __shared__ __align__(1024) uint8_t smem[];
    const uint32_t sbase = smem_u32(smem);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (sbase & 1023u) {  // the swizzled operands need 1 KiB alignment
        if (tid == 0) set_flag(flags, PLKV_FLAG_TIMEOUT);
        return;
    }
    const plkv_work_item it = items[blockIdx.x];
    const int b = it.seq, g = blockIdx.y;
    const int G = Hq / KV;
    int len = seq_lens[b];
    const int64_t cap = max_blocks * (int64_t)bs;
    if (len < 0 || len > cap) {
        if (tid == 0 && g == 0) set_flag(flags, PLKV_FLAG_BAD_LENGTH);
        len = len < 0 ? 0 : (int)cap;
    }
    const int t_begin = it.block_begin * bs;
    const int t_end = max(t_begin, min(it.block_end * bs, len));
    const int n_tiles = (t_end - t_begin + kTok - 1) / kTok;

    uint8_t* misc = smem + kMiscOff;
    const uint32_t mb = sbase + kMiscOff;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(misc + kAbort);
    const WaitCtx wc{flags, ws.ctl, abort_flag};

    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(mb + kBarKVFull + 8 * s, 1);
            mbar_init(mb + kBarKVEmpty + 8 * s, 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(mb + kBarSFull + 8 * i, 1);
            mbar_init(mb + kBarPFull + 8 * i, 1);
            mbar_init(mb + kBarODone + 8 * i, 1);
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    // Q^T as high and low FP16 parts (rows >= G zero), both P buffers zero.
    {
        // all of this thread's query loads in flight together
        constexpr int kPer = (kN * kD + kThreads - 1) / kThreads;
        float qv[kPer];
#pragma unroll
        for (int u = 0; u < kPer; ++u) {
            const int i = tid + u * kThreads, h = i / kD, d = i - h * kD;
            qv[u] = (i < kN * kD && h < G) ? q[((int64_t)b * Hq + g * G + h) * kD + d] : 0.f;
        }
#pragma unroll
        for (int u = 0; u < kPer; ++u) {
            const int i = tid + u * kThreads, h = i / kD, d = i - h * kD;
            if (i < kN * kD) {
                const __half hi = __float2half_rn(qv[u]);
                const __half lo = __float2half_rn(qv[u] - __half2float(hi));
                const uint32_t off = op_offset(h, d);
                *reinterpret_cast<__half*>(smem + kQOff + off) = hi;
                *reinterpret_cast<__half*>(smem + kQOff + kOpBytes + off) = lo;
            }
        }
    }
    for (int i = tid; i < (int)(4 * kOpBytes / 16); i += kThreads)
        reinterpret_cast<uint4*>(smem + kPOff)[i] = make_uint4(0, 0, 0, 0);
    fence_proxy_async_smem();
    if (warp == 4) {
        tmem_alloc(mb + kTmemSlot, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(misc + kTmemSlot);

    if (warp == 5) {
        // -------------------------------------------------------------- loads
        // Lane c < 8 resolves chunk c of a tile (its 8-row group index, or an
        // out-of-bounds index past the item or for a table entry outside the
        // pool) before the wait for the stage; lane 0 then issues the 16 boxes.
        const uint64_t pol = policy_evict_first();
        auto group_of = [&](int j) -> int {
            const int t = t_begin + j * kTok + 16 * lane;
            int grp = (int)n_groups;   // out of bounds: zeros
            if (lane < kChunks && t < t_end) {
                const int32_t phys = tables[(int64_t)b * max_blocks + t / bs];
                if (phys >= 0 && phys < num_physical)
                    grp = (int)((((int64_t)phys * KV + g) * bs + (t % bs)) >> 3);
                else if (g == 0)
                    set_flag(flags, PLKV_FLAG_BAD_BLOCK);
            }
            return grp;
        };
        bool ok = true;
        for (int j = 0; ok && j < n_tiles; ++j) {
            const int grp = group_of(j);
            const int st = j % kStages;
            if (j >= kStages)
                ok = __all_sync(0xffffffffu, mbar_wait(mb + kBarKVEmpty + 8 * st,
                                                       ((j / kStages) - 1) & 1, wc));
            if (!ok) break;
            int grps[kChunks];
#pragma unroll
            for (int c = 0; c < kChunks; ++c) grps[c] = __shfl_sync(0xffffffffu, grp, c);
            if (lane == 0) {
                const uint32_t bar = mb + kBarKVFull + 8 * st;
                const uint32_t kdst = sbase + kKVOff + (uint32_t)st * kStageBytes;
                mbar_arrive_expect_tx(bar, kStageBytes);
#pragma unroll
                for (int c = 0; c < kChunks; ++c) {
                    tma_chunk(kdst + c * kChunkBytes, &k_map, grps[c], bar, pol);
                    tma_chunk(kdst + kTileBytes + c * kChunkBytes, &v_map, grps[c], bar, pol);
                }
            }
            __syncwarp();
        }
    } else if (warp == 4) {
        // --------------------------------------------------------- MMA issue
        if (lane == 0 && n_tiles > 0) {
            const uint32_t id_s = idesc_f16(128, kN, false, false);
            const uint32_t id_o = idesc_f16(128, kN, true, false);
            // S of tile j (its K landed; S buffer j & 1 read by the softmax
            // of tile j - 2)
            auto issue_s = [&](int j) {
                const int st = j % kStages, sb = j & 1;
                tc_fence_after();
                const uint32_t kt = sbase + kKVOff + (uint32_t)st * kStageBytes;
#pragma unroll
                for (int kk = 0; kk < kD / 16; ++kk) {
                    const uint32_t koff = (uint32_t)(kk >> 2) * 1024u + (uint32_t)(kk & 3) * 32u;
                    const uint32_t qoff = (uint32_t)(kk >> 2) * kOpBlock + (uint32_t)(kk & 3) * 32u;
                    const uint64_t a = sdesc_sw128(kt + koff, 16, 2048);
                    mma_f16(tmem + kColS + 16 * sb, a, sdesc_sw128(sbase + kQOff + qoff, 16, 1024),
                            id_s, kk > 0 ? 1u : 0u);
                    mma_f16(tmem + kColS + 16 * sb, a,
                            sdesc_sw128(sbase + kQOff + kOpBytes + qoff, 16, 1024), id_s, 1u);
                }
                mma_commit(mb + kBarSFull + 8 * sb);
            };
            // O of tile j (its P written)
            auto issue_o = [&](int j) {
                const int st = j % kStages, pb = j & 1;
                tc_fence_after();
                const uint32_t vt = sbase + kKVOff + (uint32_t)st * kStageBytes + kTileBytes;
                const uint32_t pbase = sbase + kPOff + (uint32_t)pb * 2u * kOpBytes;
#pragma unroll
                for (int kt = 0; kt < kTok / 16; ++kt) {
                    // V^T: MN-major, the two 64-dim halves 1 KiB apart, 8-token
                    // groups 2 KiB apart, 16 tokens = one box
                    const uint64_t a = sdesc_sw128(vt + (uint32_t)kt * kChunkBytes, 1024, 2048);
                    const uint32_t poff = (uint32_t)(kt >> 2) * kOpBlock + (uint32_t)(kt & 3) * 32u;
                    mma_f16(tmem + kColO, a, sdesc_sw128(pbase + poff, 16, 1024), id_o,
                            (j > 0 || kt > 0) ? 1u : 0u);
                    mma_f16(tmem + kColO, a, sdesc_sw128(pbase + kOpBytes + poff, 16, 1024), id_o,
                            1u);
                }
                mma_commit(mb + kBarODone + 8 * pb);
                mma_commit(mb + kBarKVEmpty + 8 * st);
            };
            // Non-blocking: the S of the next tile as soon as its K and V
            // landed and its S buffer is free, the O of a tile as soon as its
            // P is written, whichever comes first; waits polled with
            // test_wait, bounded as in mbar_wait.
            int sj = 0, oj = 0;
            uint64_t idle_since = 0, next_check = 0;
            while (oj < n_tiles) {
                bool did = false;
                if (sj < n_tiles &&
                    mbar_test_wait(mb + kBarKVFull + 8 * (sj % kStages), (sj / kStages) & 1) &&
                    (sj < 2 || mbar_test_wait(mb + kBarPFull + 8 * (sj & 1), ((sj - 2) >> 1) & 1))) {
                    issue_s(sj);
                    ++sj;
                    did = true;
                }
                if (oj < sj && mbar_test_wait(mb + kBarPFull + 8 * (oj & 1), (oj >> 1) & 1)) {
                    issue_o(oj);
                    ++oj;
                    did = true;
                }
                if (did) {
                    idle_since = 0;
                } else if (*abort_flag) {
                    break;
                } else {
                    const uint64_t now = globaltimer();
                    if (idle_since == 0) {
                        idle_since = now;
                        next_check = now + kFlagPollNs;
                    } else if (now >= next_check) {
                        next_check = now + kFlagPollNs;
                        if (*wc.abort) {
                            *abort_flag = 1;
                            break;
                        }
                        if (now - idle_since > kWaitLimitNs) {
                            wait_give_up(wc);
                            break;
                        }
                    }
                }
            }
        }
        __syncwarp();
    } else {
        // ------------------------------------------------ softmax and epilogue
        const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
        float* red_max = reinterpret_cast<float*>(misc + kRedMax);
        float* red_sum = reinterpret_cast<float*>(misc + kRedSum);
        // m_use: the running max per head (identical in every thread); l_t:
        // this thread's share of the row sums (its token's probabilities),
        // reduced over the CTA once, in the epilogue.
        float m_use[kN], l_t[kN];
#pragma unroll
        for (int h = 0; h < kN; ++h) {
            m_use[h] = -INFINITY;
            l_t[h] = 0.f;
        }
        int* vote = reinterpret_cast<int*>(misc + kVote);
        // This thread's token of tile j: inside the item and of a block inside
        // the pool (boxes of any other arrived as zeros); looked up a tile
        // ahead, so that the table load never stalls the softmax.
        auto token_ok = [&](int j) -> bool {
            const int t = t_begin + j * kTok + tid;
            if (j >= n_tiles || t >= t_end) return false;
            const int32_t phys = tables[(int64_t)b * max_blocks + t / bs];
            return phys >= 0 && phys < num_physical;
        };
        bool tok_next = token_ok(0);
        bool ok = true;
        // Every softmax thread runs every iteration and reaches every named
        // barrier; after a failed wait it only skips the work.
        for (int j = 0; j < n_tiles; ++j) {
            const int sb = j & 1;
            const bool tok_ok = tok_next;
            tok_next = token_ok(j + 1);
            if (ok)
                ok = __all_sync(0xffffffffu, mbar_wait(mb + kBarSFull + 8 * sb, (j >> 1) & 1, wc));
            float s[kN];
            if (ok) {
                tc_fence_after();
                tmem_ld16(tmem + lane_base + kColS + 16 * sb, s);
                tmem_wait_ld();
            }
            const bool valid = ok && tok_ok;
            // Lazy running max: the tile's exact max per head is needed only
            // when some score exceeds the running max by more than kTau
            // (rare after the first tiles); a CTA-wide vote decides.
            bool above = false;
#pragma unroll
            for (int h = 0; h < kN; ++h) {
                s[h] = (valid && h < G) ? s[h] * scale_log2 : -INFINITY;
                above |= s[h] > m_use[h] + kTau;
            }
            above = __any_sync(0xffffffffu, above);
            if (lane == 0) vote[warp] = above ? 1 : 0;
            named_sync_softmax();
            const bool resc = (vote[0] | vote[1] | vote[2] | vote[3]) != 0;
            float alpha[kN];
#pragma unroll
            for (int h = 0; h < kN; ++h) alpha[h] = 1.f;
            if (resc) {
#pragma unroll
                for (int h = 0; h < kN; ++h) {
                    if (h < G) {
                        const float mx = warp_max(s[h]);
                        if (lane == 0) red_max[warp * kN + h] = mx;
                    }
                }
                named_sync_softmax();
#pragma unroll
                for (int h = 0; h < kN; ++h) {
                    if (h < G) {
                        const float mt = fmaxf(fmaxf(red_max[h], red_max[kN + h]),
                                               fmaxf(red_max[2 * kN + h], red_max[3 * kN + h]));
                        const float m_new = fmaxf(m_use[h], mt);
                        if (m_new > m_use[h]) {
                            alpha[h] = (m_use[h] == -INFINITY) ? 0.f : fast_exp2(m_use[h] - m_new);
                            m_use[h] = m_new;
                            l_t[h] *= alpha[h];
                        }
                    }
                }
                // the votes and maxima are read; the next tile may write them
                named_sync_softmax();
            }
            float p[kN];
#pragma unroll
            for (int h = 0; h < kN; ++h) {
                p[h] = (h < G && s[h] != -INFINITY) ? fast_exp2(s[h] - m_use[h]) : 0.f;
                l_t[h] += p[h];
            }
            if (ok && resc && j > 0) {
                // O^T through tile j - 1 must be complete before it is rescaled
                ok = __all_sync(0xffffffffu, mbar_wait(mb + kBarODone + 8 * ((j - 1) & 1),
                                                       ((j - 1) >> 1) & 1, wc));
                if (ok) {
                    tc_fence_after();
                    float o[kN];
                    tmem_ld16(tmem + lane_base + kColO, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int h = 0; h < kN; ++h) o[h] *= alpha[h];
                    tmem_st16(tmem + lane_base + kColO, o);
                    tmem_wait_st();
                }
            }
            // P buffer sb was last read by O of tile j - 2
            if (ok && j >= 2)
                ok = __all_sync(0xffffffffu, mbar_wait(mb + kBarODone + 8 * sb,
                                                       ((j - 2) >> 1) & 1, wc));
            if (ok) {
                uint8_t* pb = smem + kPOff + (uint32_t)sb * 2u * kOpBytes;
#pragma unroll
                for (int h = 0; h < kN; ++h) {
                    if (h < G) {
                        const __half hi = __float2half_rn(p[h]);
                        const __half lo = __float2half_rn(p[h] - __half2float(hi));
                        const uint32_t off = op_offset(h, tid);
                        *reinterpret_cast<__half*>(pb + off) = hi;
                        *reinterpret_cast<__half*>(pb + kOpBytes + off) = lo;
                    }
                }
            }
            // Last tile of the item: the rows past its end inside the last
            // loaded box hold whatever the pool holds there; zero their V
            // rows once the tile landed (p = 0 there, and 0 x garbage must
            // stay 0).  Boxes wholly past the end arrived as zeros.
            const int nt = min(kTok, t_end - (t_begin + j * kTok));
            if (ok && (nt & 15) != 0) {
                const int st = j % kStages;
                ok = __all_sync(0xffffffffu, mbar_wait(mb + kBarKVFull + 8 * st,
                                                       (j / kStages) & 1, wc));
                if (ok) {
                    uint8_t* vt = smem + kKVOff + (uint32_t)st * kStageBytes + kTileBytes;
                    const int rows = 16 - (nt & 15);
                    for (int i = tid; i < rows * 16; i += 128) {
                        const int r = nt + (i >> 4), h = (i >> 3) & 1, c16 = i & 7;
                        *reinterpret_cast<uint4*>(vt + (r >> 4) * kChunkBytes +
                                                  ((r >> 3) & 1) * 2048 + h * 1024 +
                                                  (r & 7) * 128 + c16 * 16) =
                            make_uint4(0, 0, 0, 0);
                    }
                }
            }
            fence_proxy_async_smem();
            tc_fence_before();
            named_sync_softmax();
            if (ok && tid == 0) mbar_arrive_local(mb + kBarPFull + 8 * sb);
        }
        // Epilogue: this item's (m, l, context) for the G heads.
        if (ok && n_tiles > 0)
            ok = __all_sync(0xffffffffu, mbar_wait(mb + kBarODone + 8 * ((n_tiles - 1) & 1),
                                                   ((n_tiles - 1) >> 1) & 1, wc));
#pragma unroll
        for (int h = 0; h < kN; ++h) {
            if (h < G) {
                const float lw = warp_sum(l_t[h]);
                if (lane == 0) red_sum[warp * kN + h] = lw;
            }
        }
        named_sync_softmax();
        float o[kN];
        const bool have = ok && n_tiles > 0;
        if (have) {
            tc_fence_after();
            tmem_ld16(tmem + lane_base + kColO, o);
            tmem_wait_ld();
        }
        const int64_t row0 = (int64_t)blockIdx.x * Hq + (int64_t)g * G;
#pragma unroll
        for (int h = 0; h < kN; ++h) {
            if (h < G) {
                ws.part_ctx[(row0 + h) * kD + tid] = have ? o[h] : 0.f;   // tid = dimension
                if (tid == h) {
                    const float l = red_sum[h] + red_sum[kN + h] + red_sum[2 * kN + h] +
                                    red_sum[3 * kN + h];
                    ws.part_m[row0 + h] = (have && m_use[h] != -INFINITY) ? m_use[h] * kLn2
                                                                          : -INFINITY;
                    ws.part_l[row0 + h] = have ? l : 0.f;
                }
            }
        }
    }

    // Teardown: every role is done with shared and tensor memory.
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 4) tmem_dealloc(tmem, kTmemCols);
}

}  // namespace fkv

bool fullkv_tc_supported(const plkv_fullkv_decode_args& a) {
    return a.head_dim == fkv::kD && a.q_heads % a.kv_heads == 0 &&
           a.q_heads / a.kv_heads <= fkv::kN && !a.scores && !a.probs && a.block_size % 16 == 0 &&
           a.num_physical * a.kv_heads * (int64_t)a.block_size / 8 < (1ll << 31);
}

cudaError_t launch_fullkv_partial_tc(const plkv_fullkv_decode_args& a, DecodeWorkspace ws,
                                     cudaStream_t st) {
    // 4-D view of a head-major pool [P, KV, bs, 128] FP16: (64 columns, 8 rows,
    // 2 column halves, 8-row groups), a box = 16 rows of one block
    const cuuint64_t n_groups = (cuuint64_t)a.num_physical * a.kv_heads * a.block_size / 8;
    const cuuint64_t dims[4] = {64, 8, 2, n_groups};
    const cuuint64_t strides[3] = {256, 128, 2048};
    const cuuint32_t box[4] = {64, 8, 2, 2};
    CUtensorMap k_map, v_map;
    if (!tc::encode_map(&k_map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a.k_cache, 4, dims, strides, box,
                        CU_TENSOR_MAP_SWIZZLE_128B) ||
        !tc::encode_map(&v_map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a.v_cache, 4, dims, strides, box,
                        CU_TENSOR_MAP_SWIZZLE_128B))
        return cudaErrorInvalidValue;
    cudaError_t e = cudaMemsetAsync(ws.ctl, 0, kCtlBytes, st);  // the launch's abort word
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(fkv::fullkv_partial_tc_kernel,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)fkv::kSmemBytes);
    if (e != cudaSuccess) return e;
    dim3 grid(a.n_items, a.kv_heads);
    fkv::fullkv_partial_tc_kernel<<<grid, fkv::kThreads, fkv::kSmemBytes, st>>>(
        k_map, v_map, (int64_t)n_groups, a.q, a.num_physical, a.kv_heads, a.block_size, a.q_heads,
        a.scale * 1.4426950408889634f, a.block_tables, a.max_blocks, a.seq_lens, a.items, ws,
        a.err_flags);
    return cudaGetLastError();
}

}  // namespace plkv
