// plkv_latent_gqa_tc.cu -- tensor-core (tcgen05) split-K partial pass of the
// exact-mode direct paged latent decode for the GQA-latent shapes (latent and
// value width 128 or 256, up to 32 query heads), FP32-accurate.
//
// Same contract as latent_partial_exact_kernel (plkv_decode_exact.cu): every
// work item emits per query head the running max m (natural-log units), the
// sum l of exp(score - m) and the unnormalised latent context
// sum_t exp(score_t - m) L_t[:Lv]; the shared combine merges the items and
// applies W_v (lib.rs:1033-1071, attention_ref.py:617-648).
//
// Every query head of a sequence attends the same latent row, so a CTA takes
// all heads of one work item and the tokens are the rows:
//   S^T = L . Q^T    M = 128 tokens, N = 64, K = latent width
//   O^T = Lv^T . P^T M = 128 value dimensions (one or two blocks), N = 64,
//                    K = 128 tokens
// cta_group::1 kind::f16, FP32 accumulators in tensor memory.  The latent
// rows are FP16 as stored; the FP32 query and probabilities are split into an
// FP16 high and low part (x = hi + lo to 2^-22 relative), and the two parts
// are stacked as the 64 columns of N (32 heads each), so one MMA forms both
// products and the softmax (scores) and the epilogue (context) add the two
// halves: FP32 accumulation error only (the exact-mode bar is 1e-5).
//
// Loads: the pool [P, bs, L] is viewed as a 4-D tensor (64 columns, 8 rows,
// L / 64 column blocks, 8-row groups); one TMA box is 16 tokens of a block,
// landing as [group][column block][8 rows][128 B] with the 128-byte swizzle,
// so a 128-token tile is the SW128 K-major operand of S^T (column block c at
// c x 1 KiB, SBO = one group) and, read as the MN-major A operand, of O^T
// (LBO 1 KiB between the two column blocks of a 128-dimension block).
// Boxes past the item's end, or of a table entry outside the pool, are read
// at an out-of-bounds group and arrive as zeros; rows past the end inside
// the last box are zeroed by the softmax warps before they release P.
//
// Softmax: TMEM lane = token, log2 domain, a lazily updated running max per
// head decided by a CTA-wide vote (the exact tile max only when a score
// passes the running max by more than 8), row sums kept per thread until
// the epilogue; O^T rescaled in tensor memory when the max moves.
//
// Warps: 0-7 softmax and epilogue (two per TMEM lane quarter, 16 heads
// each), 8 tensor-memory allocation and (lane 0) S^T issue, 9 loads, 10 and
// 11 (lane 0) O^T issue, one 128-dimension block each.  Every wait is bounded (1 s): on expiry the kernel
// records PLKV_FLAG_TIMEOUT, abandons its work and frees tensor memory.
#include <cuda_fp16.h>

#include "plkv_tc1.cuh"

namespace plkv {
namespace tc {
bool encode_map(CUtensorMap* map, CUtensorMapDataType type, const void* base, int rank,
                const cuuint64_t* dims, const cuuint64_t* strides, const cuuint32_t* box,
                CUtensorMapSwizzle swizzle);
}
namespace lgq {
using namespace tc1;

constexpr int kTok = 128;          // tokens per tile
constexpr int kHeads = 32;         // query heads, padded
constexpr int kN = 2 * kHeads;     // hi and lo parts stacked
constexpr int kSmWarps = 16;                 // softmax and epilogue warps
constexpr int kSmThreads = 32 * kSmWarps;
constexpr int kThreads = kSmThreads + 128;   // + allocation / S issue, loads, two O issuers
constexpr int kHalf = kHeads / (kSmWarps / 4);   // heads per softmax thread
static_assert(kHalf == 8 || kHalf == 16, "TMEM access width");

// kHalf consecutive TMEM columns of the warp's 32 lanes.
__device__ __forceinline__ void tmem_ld_heads(uint32_t taddr, float* v) {
    if constexpr (kHalf == 16) tmem_ld16(taddr, v); else tmem_ld8(taddr, v);
}
__device__ __forceinline__ void tmem_st_heads(uint32_t taddr, const float* v) {
    if constexpr (kHalf == 16) tmem_st16(taddr, v); else tmem_st8(taddr, v);
}
constexpr float kTau = 8.f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr uint32_t kOpBlock = kN * 128;   // 64 rows x 64 FP16 columns: 8 KiB

template <int L>
struct Cfg {
    static constexpr int kCB = L / 64;                          // 64-column blocks of a row
    static constexpr uint32_t kGroupBytes = kCB * 1024u;        // 8 rows, every column block
    static constexpr uint32_t kBoxBytes = 2 * kGroupBytes;      // 16 tokens
    static constexpr uint32_t kTileBytes = 16 * kGroupBytes;    // 128 tokens
    static constexpr int kStages = L == 256 ? 2 : 4;
    static constexpr uint32_t kQBytes = kCB * kOpBlock;         // Q^T hi / lo: [kCB][64][128 B]
    static constexpr uint32_t kPBytes = 2 * kOpBlock;           // P^T hi / lo, 128 tokens
    static constexpr uint32_t kQOff = kStages * kTileBytes;
    static constexpr uint32_t kPOff = kQOff + kQBytes;
    static constexpr uint32_t kMiscOff = kPOff + 2 * kPBytes;
    static constexpr uint32_t kMiscBytes = 2048;
    static constexpr uint32_t kSmemBytes = kMiscOff + kMiscBytes;
    static constexpr int kMB = L / 128;                         // 128-dimension blocks of O^T
    static constexpr uint32_t kColS = 0;                        // S^T buffers at 0, 64
    static constexpr uint32_t kColO = 128;                      // O^T block m at 128 + 64 m
    static constexpr uint32_t kTmemCols = 256;
    static_assert(kColO + 64 * kMB <= kTmemCols, "tensor memory");
    static_assert(kSmemBytes <= 232448, "shared memory budget");
};

enum : uint32_t {
    kBarKVFull = 0,          // [4] TMA: the tile landed
    kBarKVEmpty = 32,        // [4] MMA commit: S and O of the tile done
    kBarSFull = 64,          // [2] MMA commit: S^T of the tile in TMEM
    kBarPFull = 80,          // [2] softmax: P of the tile written
    kBarODone = 96,          // [2] MMA commit: O^T through the tile done
    kTmemSlot = 112,
    kAbort = 116,
    kVote = 128,             // [8 softmax warps] int
    kMUse = 256,             // [32] float: running max per head (log2 units)
    kAlpha = 384,            // [32] float: rescale factor of the tile per head
    kRedMax = 512,           // [4 lane quarters][32] float
    kRedSum = 1024,          // [4 lane quarters][32] float
};

__device__ __forceinline__ void named_sync_sm() {
    asm volatile("bar.sync 1, %0;" ::"n"(kSmThreads) : "memory");
}

// Byte offset of element (row, k) of a 64-row FP16 operand stored K-major in
// 128-byte-swizzled 64-column blocks (rows: the 32 heads' high parts, then
// their low parts).
__device__ __forceinline__ uint32_t op_offset(int row, int k) {
    return (uint32_t)(k >> 6) * kOpBlock + (uint32_t)(row >> 3) * 1024u +
           (uint32_t)(row & 7) * 128u + ((((uint32_t)(k & 63) >> 3) ^ (uint32_t)(row & 7)) << 4) +
           (uint32_t)(k & 7) * 2u;
}

// grid = n_items, block = 192, one CTA per SM.
template <int L>
__global__ void __launch_bounds__(kThreads, 1)
latent_gqa_tc_kernel(const __grid_constant__ CUtensorMap map, int64_t n_groups,
                     const float* __restrict__ q_lat, int64_t num_physical, int bs, int Hq,
                     float scale_log2, const int32_t* __restrict__ tables, int64_t max_blocks,
                     const int32_t* __restrict__ seq_lens,
                     const plkv_work_item* __restrict__ items, DecodeWorkspace ws,
                     int32_t* flags) {
    using namespace sm100;
    using C = Cfg<L>;
    extern __shared__ __align__(1024) uint8_t smem[];
    const uint32_t sbase = smem_u32(smem);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (sbase & 1023u) {  // the swizzled operands need 1 KiB alignment
        if (tid == 0) set_flag(flags, PLKV_FLAG_TIMEOUT);
        return;
    }
    const plkv_work_item it = items[blockIdx.x];
    const int b = it.seq;
    int len = seq_lens[b];
    const int64_t cap = max_blocks * (int64_t)bs;
    if (len < 0 || len > cap) {
        if (tid == 0) set_flag(flags, PLKV_FLAG_BAD_LENGTH);
        len = len < 0 ? 0 : (int)cap;
    }
    const int t_begin = it.block_begin * bs;
    const int t_end = max(t_begin, min(it.block_end * bs, len));
    const int n_tiles = (t_end - t_begin + kTok - 1) / kTok;

    uint8_t* misc = smem + C::kMiscOff;
    const uint32_t mb = sbase + C::kMiscOff;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(misc + kAbort);
    const WaitCtx wc{flags, ws.ctl, abort_flag};

    if (tid == 0) {
        for (int s = 0; s < C::kStages; ++s) {
            mbar_init(mb + kBarKVFull + 8 * s, 1);
            mbar_init(mb + kBarKVEmpty + 8 * s, C::kMB);   // one commit per O issuer
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(mb + kBarSFull + 8 * i, 1);
            mbar_init(mb + kBarPFull + 8 * i, 1);
            mbar_init(mb + kBarODone + 8 * i, C::kMB);
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    // The loader starts on the first tiles as soon as the barriers exist;
    // the other warps stage Q^T, clear P and allocate tensor memory in the
    // meantime and meet at a named barrier without it.
    __syncthreads();
    constexpr int kLoadWarp = kSmWarps + 1;
    uint32_t tmem = 0;
    if (warp != kLoadWarp) {
        if (tid < kSmThreads) {
            // Q^T: head h's high part in row h, its low part in row 32 + h
            // (rows of heads >= Hq zero); both P buffers zero (rows of heads
            // >= Hq stay so).
            constexpr int kBatch = 16;
            for (int i0 = tid; i0 < kHeads * L; i0 += kBatch * kSmThreads) {
                float qv[kBatch];
#pragma unroll
                for (int u = 0; u < kBatch; ++u) {
                    const int i = i0 + u * kSmThreads, h = i / L, d = i - h * L;
                    qv[u] = (i < kHeads * L && h < Hq) ? q_lat[((int64_t)b * Hq + h) * L + d]
                                                       : 0.f;
                }
#pragma unroll
                for (int u = 0; u < kBatch; ++u) {
                    const int i = i0 + u * kSmThreads, h = i / L, d = i - h * L;
                    if (i < kHeads * L) {
                        const __half hi = __float2half_rn(qv[u]);
                        const __half lo = __float2half_rn(qv[u] - __half2float(hi));
                        *reinterpret_cast<__half*>(smem + C::kQOff + op_offset(h, d)) = hi;
                        *reinterpret_cast<__half*>(smem + C::kQOff + op_offset(kHeads + h, d)) =
                            lo;
                    }
                }
            }
            for (int i = tid; i < (int)(2 * C::kPBytes / 16); i += kSmThreads)
                reinterpret_cast<uint4*>(smem + C::kPOff)[i] = make_uint4(0, 0, 0, 0);
            fence_proxy_async_smem();
        }
        if (warp == kSmWarps) {
            tmem_alloc(mb + kTmemSlot, C::kTmemCols);
            tmem_relinquish();
        }
        tc_fence_before();
        asm volatile("bar.sync 2, %0;" ::"n"(kThreads - 32) : "memory");
        tc_fence_after();
        tmem = *reinterpret_cast<volatile uint32_t*>(misc + kTmemSlot);
    }

    if (warp == kLoadWarp) {
        // -------------------------------------------------------------- loads
        // Lane c < 8 resolves box c of a tile (its 8-row group index, or an
        // out-of-bounds index past the item or for a table entry outside the
        // pool) before the wait for the stage; lane 0 then issues the 8 boxes.
        const uint64_t pol = policy_evict_first();
        auto group_of = [&](int j) -> int {
            const int t = t_begin + j * kTok + 16 * lane;
            int grp = (int)n_groups;   // out of bounds: zeros
            if (lane < 8 && t < t_end) {
                const int32_t phys = tables[(int64_t)b * max_blocks + t / bs];
                if (phys >= 0 && phys < num_physical)
                    grp = (int)(((int64_t)phys * bs + (t % bs)) >> 3);
                else
                    set_flag(flags, PLKV_FLAG_BAD_BLOCK);
            }
            return grp;
        };
        bool ok = true;
        for (int j = 0; ok && j < n_tiles; ++j) {
            const int grp = group_of(j);
            const int st = j % C::kStages;
            if (j >= C::kStages)
                ok = __all_sync(0xffffffffu, mbar_wait(mb + kBarKVEmpty + 8 * st,
                                                       ((j / C::kStages) - 1) & 1, wc));
            if (!ok) break;
            int grps[8];
#pragma unroll
            for (int c = 0; c < 8; ++c) grps[c] = __shfl_sync(0xffffffffu, grp, c);
            if (lane == 0) {
                const uint32_t bar = mb + kBarKVFull + 8 * st;
                const uint32_t dst = sbase + (uint32_t)st * C::kTileBytes;
                mbar_arrive_expect_tx(bar, C::kTileBytes);
#pragma unroll
                for (int c = 0; c < 8; ++c) tma_chunk(dst + c * C::kBoxBytes, &map, grps[c], bar, pol);
            }
            __syncwarp();
        }
    } else if (warp == kSmWarps || warp >= kSmWarps + 2) {
        // --------------------------------------------------------- MMA issue
        // Warp 8 issues S^T, warp 10 + m block m of O^T: one thread issues a
        // tcgen05.mma every ~60 cycles, so S of a tile never waits behind
        // the O instructions of the tile before it in one program order.
        const int role = warp == kSmWarps ? -1 : warp - (kSmWarps + 2);   // -1: S^T, else O^T block
        if (lane == 0 && n_tiles > 0 && role < C::kMB) {
            const uint32_t id_s = idesc_f16(128, kN, false, false);
            const uint32_t id_o = idesc_f16(128, kN, true, false);
            // S^T of tile j (its rows landed; S buffer j & 1 read by the
            // softmax of tile j - 2): both parts of Q at once (N = 64)
            auto issue_s = [&](int j) {
                const int st = j % C::kStages, sb = j & 1;
                tc_fence_after();
                const uint32_t tile = sbase + (uint32_t)st * C::kTileBytes;
#pragma unroll
                for (int kk = 0; kk < L / 16; ++kk) {
                    const uint32_t cb = (uint32_t)(kk >> 2), ko = (uint32_t)(kk & 3) * 32u;
                    mma_f16(tmem + C::kColS + 64 * sb,
                            sdesc_sw128(tile + cb * 1024u + ko, 16, C::kGroupBytes),
                            sdesc_sw128(sbase + C::kQOff + cb * kOpBlock + ko, 16, 1024), id_s,
                            kk > 0 ? 1u : 0u);
                }
                mma_commit(mb + kBarSFull + 8 * sb);
            };
            // O^T block `role` of tile j (its P written): both parts of P at once
            auto issue_o = [&](int j) {
                const int st = j % C::kStages, pb = j & 1;
                tc_fence_after();
                const uint32_t tile = sbase + (uint32_t)st * C::kTileBytes;
                const uint32_t pbase = sbase + C::kPOff + (uint32_t)pb * C::kPBytes;
#pragma unroll
                for (int kt = 0; kt < kTok / 16; ++kt) {
                    const uint64_t bdesc = sdesc_sw128(
                        pbase + (uint32_t)(kt >> 2) * kOpBlock + (uint32_t)(kt & 3) * 32u, 16, 1024);
                    // Lv^T block `role`: MN-major, its two 64-dimension
                    // column blocks 1 KiB apart, 8-token groups one group apart
                    mma_f16(tmem + C::kColO + 64 * role,
                            sdesc_sw128(tile + (uint32_t)(2 * role) * 1024u +
                                            (uint32_t)kt * 2u * C::kGroupBytes,
                                        1024, C::kGroupBytes),
                            bdesc, id_o, (j > 0 || kt > 0) ? 1u : 0u);
                }
                mma_commit(mb + kBarODone + 8 * pb);
                mma_commit(mb + kBarKVEmpty + 8 * st);
            };
            // Non-blocking: S as soon as its tile landed and its buffer is
            // free, O as soon as its P is written (which follows S of the
            // tile); bounded as in mbar_wait.
            int sj = 0, oj = 0;
            uint64_t idle_since = 0, next_check = 0;
            while (role < 0 ? sj < n_tiles : oj < n_tiles) {
                bool did = false;
                if (role < 0) {
                    if (mbar_test_wait(mb + kBarKVFull + 8 * (sj % C::kStages),
                                       (sj / C::kStages) & 1) &&
                        (sj < 2 ||
                         mbar_test_wait(mb + kBarPFull + 8 * (sj & 1), ((sj - 2) >> 1) & 1))) {
                        issue_s(sj);
                        ++sj;
                        did = true;
                    }
                } else if (mbar_test_wait(mb + kBarPFull + 8 * (oj & 1), (oj >> 1) & 1)) {
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
        // Eight warps: warp w reads TMEM lanes 32 (w & 3) .. + 31 (tokens of
        // the tile; value dimensions in the epilogue) and handles heads
        // [16 (w >> 2), + 16), so two warps share each SM sub-partition and
        // each issues half of a tile's softmax instructions.
        const int q4 = warp & 3, h0 = kHalf * (warp >> 2);
        const int t = tid & (kTok - 1);   // token row of the tile
        const uint32_t lane_base = static_cast<uint32_t>(q4 * 32) << 16;
        float* red_max = reinterpret_cast<float*>(misc + kRedMax);
        float* red_sum = reinterpret_cast<float*>(misc + kRedSum);
        int* vote = reinterpret_cast<int*>(misc + kVote);
        // m_use (shared memory): the running max per head, the same for
        // every thread; l_t: this thread's share of the row sums of its
        // heads (its token's probabilities), reduced in the epilogue.
        float* m_use = reinterpret_cast<float*>(misc + kMUse);
        float* alpha = reinterpret_cast<float*>(misc + kAlpha);
        float l_t[kHalf];
#pragma unroll
        for (int h = 0; h < kHalf; ++h) l_t[h] = 0.f;
        if (tid < kHeads) m_use[tid] = -INFINITY;
        named_sync_sm();
        // This thread's token of tile j: inside the item and of a block inside
        // the pool; looked up a tile ahead.
        auto token_ok = [&](int j) -> bool {
            const int tt = t_begin + j * kTok + t;
            if (j >= n_tiles || tt >= t_end) return false;
            const int32_t phys = tables[(int64_t)b * max_blocks + tt / bs];
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
            float s[kHalf];   // scores, then probabilities
            if (ok) {
                float lo[kHalf];
                tc_fence_after();
                tmem_ld_heads(tmem + lane_base + C::kColS + 64 * sb + h0, s);
                tmem_ld_heads(tmem + lane_base + C::kColS + 64 * sb + kHeads + h0, lo);
                tmem_wait_ld();
#pragma unroll
                for (int h = 0; h < kHalf; ++h) s[h] += lo[h];   // Q_hi . L + Q_lo . L
            }
            const bool valid = ok && tok_ok;
            bool above = false;
#pragma unroll
            for (int h = 0; h < kHalf; ++h) {
                s[h] = (valid && h0 + h < Hq) ? s[h] * scale_log2 : -INFINITY;
                above |= s[h] > m_use[h0 + h] + kTau;
            }
            above = __any_sync(0xffffffffu, above);
            if (lane == 0) vote[warp] = above ? 1 : 0;
            named_sync_sm();
            int any = 0;
#pragma unroll
            for (int w = 0; w < kSmWarps; ++w) any |= vote[w];
            const bool resc = any != 0;
            if (resc) {
#pragma unroll
                for (int h = 0; h < kHalf; ++h) {
                    if (h0 + h < Hq) {
                        const float mx = warp_max(s[h]);
                        if (lane == 0) red_max[q4 * kHeads + h0 + h] = mx;
                    }
                }
                named_sync_sm();
                if (tid < kHeads) {   // warp 0: the new max and factor of head tid
                    const int h = tid;
                    const float mt = fmaxf(fmaxf(red_max[h], red_max[kHeads + h]),
                                           fmaxf(red_max[2 * kHeads + h], red_max[3 * kHeads + h]));
                    const float m_old = m_use[h], m_new = fmaxf(m_old, mt);
                    float a = 1.f;
                    if (m_new > m_old) a = (m_old == -INFINITY) ? 0.f : fast_exp2(m_old - m_new);
                    m_use[h] = m_new;
                    alpha[h] = a;
                }
                named_sync_sm();
#pragma unroll
                for (int h = 0; h < kHalf; ++h) l_t[h] *= alpha[h0 + h];
            }
#pragma unroll
            for (int h = 0; h < kHalf; ++h) {
                s[h] = (h0 + h < Hq && s[h] != -INFINITY) ? fast_exp2(s[h] - m_use[h0 + h]) : 0.f;
                l_t[h] += s[h];
            }
            if (ok && resc && j > 0) {
                // O^T through tile j - 1 must be complete before it is rescaled
                ok = __all_sync(0xffffffffu, mbar_wait(mb + kBarODone + 8 * ((j - 1) & 1),
                                                       ((j - 1) >> 1) & 1, wc));
                if (ok) {
                    tc_fence_after();
#pragma unroll 1
                    for (int c = 0; c < 2 * C::kMB; ++c) {   // hi or lo part of block c / 2
                        float o[kHalf];
                        const uint32_t col = C::kColO + 64 * (c >> 1) + kHeads * (c & 1) + h0;
                        tmem_ld_heads(tmem + lane_base + col, o);
                        tmem_wait_ld();
#pragma unroll
                        for (int h = 0; h < kHalf; ++h) o[h] *= alpha[h0 + h];
                        tmem_st_heads(tmem + lane_base + col, o);
                    }
                    tmem_wait_st();
                }
            }
            const float* p = s;
            // P buffer sb was last read by O of tile j - 2
            if (ok && j >= 2)
                ok = __all_sync(0xffffffffu, mbar_wait(mb + kBarODone + 8 * sb,
                                                       ((j - 2) >> 1) & 1, wc));
            if (ok) {
                uint8_t* pb = smem + C::kPOff + (uint32_t)sb * C::kPBytes;
#pragma unroll
                for (int h = 0; h < kHalf; ++h) {
                    if (h0 + h < Hq) {
                        const __half hi = __float2half_rn(p[h]);
                        const __half lo = __float2half_rn(p[h] - __half2float(hi));
                        *reinterpret_cast<__half*>(pb + op_offset(h0 + h, t)) = hi;
                        *reinterpret_cast<__half*>(pb + op_offset(kHeads + h0 + h, t)) = lo;
                    }
                }
            }
            // Last tile of the item: rows past its end inside the last loaded
            // box hold whatever the pool holds there; zero them once the tile
            // landed (p = 0 there, and 0 x garbage must stay 0).
            const int nt = min(kTok, t_end - (t_begin + j * kTok));
            if (ok && (nt & 15) != 0) {
                const int st = j % C::kStages;
                ok = __all_sync(0xffffffffu, mbar_wait(mb + kBarKVFull + 8 * st,
                                                       (j / C::kStages) & 1, wc));
                if (ok) {
                    uint8_t* tile = smem + (uint32_t)st * C::kTileBytes;
                    const int rows = 16 - (nt & 15);
                    for (int i = tid; i < rows * C::kCB * 8; i += kSmThreads) {
                        const int r = nt + i / (C::kCB * 8), rem = i % (C::kCB * 8);
                        const int cb = rem >> 3, c16 = rem & 7;
                        *reinterpret_cast<uint4*>(tile + (uint32_t)(r >> 3) * C::kGroupBytes +
                                                  cb * 1024 + (r & 7) * 128 + c16 * 16) =
                            make_uint4(0, 0, 0, 0);
                    }
                }
            }
            fence_proxy_async_smem();
            tc_fence_before();
            named_sync_sm();
            if (ok && tid == 0) mbar_arrive_local(mb + kBarPFull + 8 * sb);
        }
        // Epilogue: this item's (m, l, context) for the Hq heads.
        if (ok && n_tiles > 0)
            ok = __all_sync(0xffffffffu, mbar_wait(mb + kBarODone + 8 * ((n_tiles - 1) & 1),
                                                   ((n_tiles - 1) >> 1) & 1, wc));
#pragma unroll
        for (int h = 0; h < kHalf; ++h) {
            if (h0 + h < Hq) {
                const float lw = warp_sum(l_t[h]);
                if (lane == 0) red_sum[q4 * kHeads + h0 + h] = lw;
            }
        }
        named_sync_sm();
        const bool have = ok && n_tiles > 0;
        if (have) tc_fence_after();
        const int64_t row0 = (int64_t)blockIdx.x * Hq;
#pragma unroll 1
        for (int m = 0; m < C::kMB; ++m) {
            float o[kHalf], lo[kHalf];
            if (have) {
                tmem_ld_heads(tmem + lane_base + C::kColO + 64 * m + h0, o);
                tmem_ld_heads(tmem + lane_base + C::kColO + 64 * m + kHeads + h0, lo);
                tmem_wait_ld();
            }
#pragma unroll
            for (int h = 0; h < kHalf; ++h)
                if (h0 + h < Hq)   // thread = value dimension 128 m + t
                    ws.part_ctx[(row0 + h0 + h) * L + 128 * m + t] = have ? o[h] + lo[h] : 0.f;
        }
        if (tid < Hq) {
            const float mh = m_use[tid];
            const float l = red_sum[tid] + red_sum[kHeads + tid] + red_sum[2 * kHeads + tid] +
                            red_sum[3 * kHeads + tid];
            ws.part_m[row0 + tid] = (have && mh != -INFINITY) ? mh * kLn2 : -INFINITY;
            ws.part_l[row0 + tid] = have ? l : 0.f;
        }
    }

    // Teardown: every role is done with shared and tensor memory.
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == kSmWarps) tmem_dealloc(tmem, C::kTmemCols);
}

template <int L>
cudaError_t launch(const plkv_latent_decode_args& a, DecodeWorkspace ws, cudaStream_t st) {
    using C = Cfg<L>;
    // 4-D view of the pool [P, bs, L] FP16: (64 columns, 8 rows, L / 64 column
    // blocks, 8-row groups); a box = 16 rows of one block
    const cuuint64_t n_groups = (cuuint64_t)a.num_physical * a.block_size / 8;
    const cuuint64_t dims[4] = {64, 8, (cuuint64_t)C::kCB, n_groups};
    const cuuint64_t strides[3] = {(cuuint64_t)L * 2, 128, (cuuint64_t)L * 16};
    const cuuint32_t box[4] = {64, 8, (cuuint32_t)C::kCB, 2};
    CUtensorMap map;
    if (!tc::encode_map(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a.cache, 4, dims, strides, box,
                        CU_TENSOR_MAP_SWIZZLE_128B))
        return cudaErrorInvalidValue;
    cudaError_t e = cudaMemsetAsync(ws.ctl, 0, kCtlBytes, st);  // the launch's abort word
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(latent_gqa_tc_kernel<L>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)C::kSmemBytes);
    if (e != cudaSuccess) return e;
    latent_gqa_tc_kernel<L><<<a.n_items, kThreads, C::kSmemBytes, st>>>(
        map, (int64_t)n_groups, a.q_lat, a.num_physical, a.block_size, a.q_heads,
        a.scale * 1.4426950408889634f, a.block_tables, a.max_blocks, a.seq_lens, a.items, ws,
        a.err_flags);
    return cudaGetLastError();
}

}  // namespace lgq

bool latent_gqa_tc_supported(const plkv_latent_decode_args& a) {
    return (a.latent_dim == 128 || a.latent_dim == 256) && a.value_dim == a.latent_dim &&
           a.q_heads <= lgq::kHeads && a.block_size % 16 == 0 && !a.scores && !a.probs &&
           a.num_physical * (int64_t)a.block_size / 8 < (1ll << 31) &&
           (reinterpret_cast<uintptr_t>(a.cache) & 15) == 0;
}

cudaError_t launch_latent_partial_gqa_tc(const plkv_latent_decode_args& a, DecodeWorkspace ws,
                                         cudaStream_t st) {
    return a.latent_dim == 256 ? lgq::launch<256>(a, ws, st) : lgq::launch<128>(a, ws, st);
}

}  // namespace plkv
