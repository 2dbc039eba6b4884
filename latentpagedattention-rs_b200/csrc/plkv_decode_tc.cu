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
// Work split.  A cluster of two CTAs (a tcgen05 CTA pair) is persistent: it
// processes the items of one worker of plkv_plan_workers (or one item) in
// tiles of 64 tokens.  CTA r owns query heads [64r, 64r+64).
//   S = Q . L^T  : cta_group::2 MMA, M = 128 heads, N = 64 tokens, K = 576
//                  (four partials of K = 144, see below).
//                  CTA r supplies its heads' Q and tokens [32r, 32r+32) of L;
//                  its TMEM receives its 64 heads x 64 tokens (32 columns).
//   O += P . V   : cta_group::2 MMA, M = 128 heads, N = 256 value columns
//                  (two instructions), K = 64 tokens.  CTA r supplies its
//                  heads' P and value columns {0,1,4,5} (r = 0) or {2,3,6,7}
//                  (r = 1) in 64-column blocks; its TMEM holds its 64 heads x
//                  512 columns in 256 columns.
// The two MMAs need different slices of a tile at identical shared-memory
// offsets in both CTAs, so each CTA loads its own token half of all nine
// 64-column blocks into the K ring (consumed by S, released when S is done)
// and both token halves of its four value blocks into the V ring (consumed by
// O): per tile and CTA one 3-D TMA copy of 36 KiB (K) and two 4-D copies of
// 16 KiB (V).  Small 2-D boxes (32 rows x 64 columns, 17 per tile) cost TMA
// issue time: from L2, nine such boxes per 36 KiB stream at 59 GB/s per SM
// and one 3-D box at 104 GB/s (measured on B200).  Decoupling the rings lets
// the next tiles' K loads start as soon as S completes.
//
// The query is converted once per call (q_prep kernel) to FP16 pre-scaled by
// scale * log2(e) and loaded per item by TMA.  Softmax runs in the log2
// domain with a lazily updated running max: probabilities are taken against a
// stale max until a tile's max exceeds it by more than 8 (probabilities stay
// <= 2^8 in FP16); only then is the accumulated O rescaled in TMEM.  TMEM lane
// = head, and the two threads sharing a head (token halves) agree through
// shared memory, so the CTAs never exchange softmax state.
//
// MMA issue is split over six threads of the leader CTA.  One thread issues
// a tcgen05.mma every ~60 cycles however small the MMA is, and at N = 64 the
// tensor pipe finishes one in less; measured on B200, 36 pair MMAs take 1.52
// us from one issuing warp, 0.83 us from two and 0.49 us from four.  So S is
// cut along K into four 9-step partials, each accumulated by its own issuer
// in its own TMEM columns and added by the softmax threads.  Two more threads
// issue the two 256-column halves of O, so that a tile's S never waits
// behind the O instructions of the previous tile in an issuer's program
// order (303 against 310 us per long-context pass on the same B200).
// Barriers completed by MMA commits count one arrival per issuer that
// commits to them.
//
// Warp roles per CTA: 0 = Q and K loads, 1 = TMEM allocation and (leader
// CTA) S issue, 2 = V loads, 3, 8, 9 = (leader CTA) S issue, 4..7 = softmax
// and epilogue, 10, 11 = (leader CTA) O issue.  Every barrier wait is bounded
// (1 s): on expiry the kernel records PLKV_FLAG_TIMEOUT, abandons its work,
// releases tensor memory and exits.
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
constexpr int kKBlocks = kLatent / 64;                       // 9
constexpr uint32_t kBox = 32 * 128;                           // 32 rows x 64 FP16
constexpr uint32_t kQAtom = kHeadsPerCta * 128;               // 64 rows x 64 FP16
constexpr uint32_t kQBytes = kKBlocks * kQAtom;               // 72 KiB
constexpr uint32_t kKStage = kKBlocks * kBox;                 // 36 KiB
constexpr uint32_t kVStage = 2 * 4 * kBox;                    // 32 KiB
constexpr int kStages = 2;
constexpr uint32_t kPBytes = kHeadsPerCta * kTile * 2;        // 8 KiB
constexpr uint32_t kQOff = 0;
constexpr uint32_t kKOff = kQOff + kQBytes;
constexpr uint32_t kVOff = kKOff + kStages * kKStage;
constexpr uint32_t kPOff = kVOff + kStages * kVStage;
constexpr uint32_t kMiscOff = kPOff + 2 * kPBytes;            // 229376
constexpr uint32_t kMiscBytes = 2048;
constexpr uint32_t kSmemBytes = kMiscOff + kMiscBytes;        // 231424
constexpr uint32_t kQTx = 2u * kQBytes;                       // both CTAs
constexpr uint32_t kKTx = 2u * kKStage;                       // both CTAs
constexpr uint32_t kVTx = kVStage;                            // own CTA
constexpr uint32_t kTmemCols = 512;
constexpr int kSBufs = 2;                                     // S accumulators in TMEM
constexpr uint32_t kTmemO = 0;                                // O at 0..255
constexpr int kIssuers = 4;                                   // S-issuing threads (warps 1, 3, 8, 9)
constexpr int kThreads = 384;                                 // warps 10, 11 issue O
constexpr int kKPer = 36 / kIssuers;                          // S k-steps per issuer
// S partial p of buffer sb at 256 + 32 (kSBufs p + sb)
__host__ __device__ constexpr uint32_t s_col(int p, int sb) { return 256u + 32u * (kSBufs * p + sb); }
constexpr float kTau = 8.f;
constexpr float kLn2 = 0.6931471805599453f;

// Misc region: barriers (8 bytes each), then small shared arrays.
enum : uint32_t {
    kBarQFull = 0,     // leader: Q of the item landed in both CTAs
    kBarQFree = 8,     // both: every MMA of the item completed (Q may be reloaded)
    kBarKFull = 16,    // [2] leader: K tile landed in both CTAs
    kBarKEmpty = 32,   // [2] both: S of the tile completed
    kBarVFull = 48,    // [2] own: V tile landed in this CTA
    kBarVEmpty = 64,   // [2] both: O of the tile completed (V reusable)
    kBarPFull = 80,    // [2] leader: P written (and V checked) in both CTAs
    kBarODone = 96,    // [2] both: O of the tile completed (P buffer reusable)
    kBarOFree = 112,   // leader: epilogue of the item read O in both CTAs
    kBarSFull = 120,   // [kSBufs] both: S of the tile in TMEM
    kTmemSlot = 152,
    kAbort = 156,
    kRedMax = 256,     // [2][128] float
    kRedSum = 256 + 1024,
};
static_assert(kSmemBytes <= 232448, "shared memory budget");
static_assert(kRedSum + 128 * 4 <= kMiscBytes, "misc region");

__device__ __forceinline__ void named_sync_softmax() {
    asm volatile("bar.sync 1, 128;" ::: "memory");
}

__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Rows [y, y + box rows) x all nine 64-column blocks in one instruction: the
// 3-D view (64 columns, rows, 9 column blocks at 128 B) of a row-major FP16
// matrix of 576 columns lands block after block, each block 128 B per row,
// which is the K-major SWIZZLE_128B operand layout of the MMAs.  Completes on
// a barrier of the leader CTA (cta_group::2); no multicast.
__device__ __forceinline__ void tma_load_3d_pair(uint32_t dst, const CUtensorMap* map, int y,
                                                 uint32_t cluster_bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        ".L2::cache_hint [%0], [%1, {%2, %3, %4}], [%5], %6;"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(0), "r"(y), "r"(0), "r"(cluster_bar),
          "l"(policy)
        : "memory");
}
// The four value column blocks [z0, z0 + 4) of 32 rows in one instruction:
// 3-D view (64 columns, rows, 8 blocks at 128 B), one 512-byte run per row;
// completes on a barrier of this CTA.
__device__ __forceinline__ void tma_load_v_own(uint32_t dst, const CUtensorMap* map, int y, int z0,
                                               uint32_t bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
        ".L2::cache_hint [%0], [%1, {%2, %3, %4}], [%5], %6;"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(0), "r"(y), "r"(z0), "r"(bar),
          "l"(policy)
        : "memory");
}

struct ItemGeom {
    int seq, t_begin, t_end, n_tiles;
};

__device__ __forceinline__ ItemGeom item_geom(const plkv_work_item* items, int idx,
                                              const int32_t* seq_lens, int bs, int64_t cap,
                                              int32_t* flags, bool report) {
    const plkv_work_item it = items[idx];
    ItemGeom g;
    g.seq = it.seq;
    int len = seq_lens[it.seq];
    if (len < 0 || len > cap) {
        if (report) set_flag(flags, PLKV_FLAG_BAD_LENGTH);
        len = len < 0 ? 0 : (int)cap;
    }
    g.t_begin = it.block_begin * bs;
    g.t_end = max(g.t_begin, min(it.block_end * bs, len));
    g.n_tiles = (g.t_end - g.t_begin + kTile - 1) / kTile;
    return g;
}

// Pool row of the first token of half-tile `h` of tile `j` (a half past the
// end reuses half 0 so that every load reads valid pool rows).
__device__ __forceinline__ int half_row(const ItemGeom& g, int j, int h,
                                        const int32_t* __restrict__ tables, int64_t max_blocks,
                                        int64_t num_physical, int bs, int32_t* flags) {
    int hs = g.t_begin + kTile * j + 32 * h;
    if (hs >= g.t_end) hs = g.t_begin + kTile * j;
    const int lb = hs / bs;
    int32_t phys = tables[(int64_t)g.seq * max_blocks + lb];
    if (phys < 0 || phys >= num_physical) {
        set_flag(flags, PLKV_FLAG_BAD_BLOCK);
        phys = 0;
    }
    return phys * bs + (hs - lb * bs);
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
latent_partial_tc_kernel(const __grid_constant__ CUtensorMap k_map,
                         const __grid_constant__ CUtensorMap v_map,
                         const __grid_constant__ CUtensorMap q_map,
                         int bs,
                         const int32_t* __restrict__ tables, int64_t max_blocks,
                         int64_t num_physical, const int32_t* __restrict__ seq_lens,
                         const plkv_work_item* __restrict__ items,
                         const int32_t* __restrict__ worker_item_begin, DecodeWorkspace ws,
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
    const int worker = blockIdx.x >> 1;
    const int i_begin = worker_item_begin ? worker_item_begin[worker] : worker;
    const int i_end = worker_item_begin ? worker_item_begin[worker + 1] : worker + 1;
    const int64_t cap = max_blocks * (int64_t)bs;

    uint8_t* misc = smem + kMiscOff;
    const uint32_t mb = sbase + kMiscOff;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(misc + kAbort);
    const WaitCtx wc{flags, ws.ctl, abort_flag};
    float* red_max = reinterpret_cast<float*>(misc + kRedMax);
    float* red_sum = reinterpret_cast<float*>(misc + kRedSum);

    if (tid == 0) {
        mbar_init(mb + kBarQFull, 1);
        mbar_init(mb + kBarQFree, kIssuers);
        mbar_init(mb + kBarOFree, 2);
        for (int i = 0; i < 2; ++i) {
            mbar_init(mb + kBarKFull + 8 * i, 1);
            mbar_init(mb + kBarKEmpty + 8 * i, kIssuers);
            mbar_init(mb + kBarVFull + 8 * i, 1);
            mbar_init(mb + kBarVEmpty + 8 * i, 2);
            mbar_init(mb + kBarPFull + 8 * i, 2);
            mbar_init(mb + kBarODone + 8 * i, 2);
        }
        for (int i = 0; i < kSBufs; ++i) mbar_init(mb + kBarSFull + 8 * i, kIssuers);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc_pair(mb + kTmemSlot, kTmemCols);
        tmem_relinquish_pair();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tensormap(&k_map);
        prefetch_tensormap(&v_map);
        prefetch_tensormap(&q_map);
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();
    tc_fence_after();
    const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(misc + kTmemSlot);

    if (warp == 0) {
        // ---------------------------------------------------- Q and K loads
        if (lane == 0) {
            // K rows are read a second time, from L2, by the V loads of the
            // same tile (the other CTA's token half, and this CTA's value
            // columns), so they enter L2 with the normal eviction priority;
            // the V loads, their last use, mark them evict-first.  K loads
            // marked evict-first lost part of those rows before the V loads
            // came: 352 -> 322 us per partial pass when this changed.
            const uint64_t pol = policy_evict_normal();
            const uint32_t kfull0 = mapa(mb + kBarKFull, 0), kfull1 = mapa(mb + kBarKFull + 8, 0);
            const uint32_t qfull = mapa(mb + kBarQFull, 0);
            int gt = 0;  // tile counter over the worker's items
            bool ok = true;
            for (int ii = i_begin; ok && ii < i_end; ++ii) {
                const ItemGeom g = item_geom(items, ii, seq_lens, bs, cap, flags, false);
                const int ni = ii - i_begin;
                auto load_q = [&]() -> bool {
                    if (ni >= 1 &&
                        !mbar_wait(mb + kBarQFree, (ni - 1) & 1, wc))
                        return false;
                    if (leader) mbar_arrive_expect_tx(mb + kBarQFull, kQTx);
                    const int y = g.seq * kHeads + kHeadsPerCta * (int)rank;
                    tma_load_3d_pair(sbase + kQOff, &q_map, y, qfull, pol);
                    return true;
                };
                // The first K tiles of an item only need free K stages; Q waits
                // for every MMA of the previous item, so load it after them.
                const int pre = min(2, g.n_tiles);
                for (int j = 0; ok && j < g.n_tiles; ++j) {
                    // Block-table lookups first: their latency then overlaps
                    // the wait for a free stage instead of following it.
                    const int y = half_row(g, j, (int)rank, tables, max_blocks, num_physical, bs, flags);
                    if (j == pre && !(ok = load_q())) break;
                    const int gj = gt + j, st = gj & 1;
                    if (gj >= 2 && !(ok = mbar_wait(mb + kBarKEmpty + 8 * st, ((gj - 2) >> 1) & 1,
                                                    wc)))
                        break;
                    if (leader) mbar_arrive_expect_tx(mb + kBarKFull + 8 * st, kKTx);
                    const uint32_t dst = sbase + kKOff + st * kKStage;
                    const uint32_t fb = st ? kfull1 : kfull0;
                    tma_load_3d_pair(dst, &k_map, y, fb, pol);
                }
                if (ok && pre == g.n_tiles) ok = load_q();
                gt += g.n_tiles;
            }
        }
        __syncwarp();
    } else if (warp == 2) {
        // --------------------------------------------------------- V loads
        if (lane == 0) {
            const uint64_t pol = policy_evict_first();
            int gt = 0;
            bool ok = true;
            for (int ii = i_begin; ok && ii < i_end; ++ii) {
                const ItemGeom g = item_geom(items, ii, seq_lens, bs, cap, flags, false);
                for (int j = 0; j < g.n_tiles; ++j) {
                    const int gj = gt + j, st = gj & 1;
                    const int y0 = half_row(g, j, 0, tables, max_blocks, num_physical, bs, flags);
                    const int y1 = half_row(g, j, 1, tables, max_blocks, num_physical, bs, flags);
                    if (gj >= 2 && !(ok = mbar_wait(mb + kBarVEmpty + 8 * st, ((gj - 2) >> 1) & 1,
                                                    wc)))
                        break;
                    mbar_arrive_expect_tx(mb + kBarVFull + 8 * st, kVTx);
                    const uint32_t dst = sbase + kVOff + st * kVStage;
                    for (int h = 0; h < 2; ++h)
                        tma_load_v_own(dst + h * 4 * kBox, &v_map, h ? y1 : y0, 4 * (int)rank,
                                        mb + kBarVFull + 8 * st, pol);
                }
                gt += g.n_tiles;
            }
        }
        __syncwarp();
    } else if (warp == 1 || warp == 3 || warp >= 8) {
        // ---------------------------------------------- MMA issue (leader)
        // Each issuer schedules its MMAs without blocking: its S partial of
        // tile g as soon as K tile g landed and S buffer g % kSBufs is free
        // (P of its previous tile was written, so the softmax read it); an O
        // issuer its O half of tile g as soon as P(g) is ready.
        // S work thus stays queued on the tensor pipe while the softmax of
        // earlier tiles runs.  S never crosses into the next item before that
        // item's Q is loaded, which waits until every issuer's S of the
        // current item completed (barrier QFree).  The barriers are polled
        // with test_wait, which never suspends: a try_wait on a barrier that
        // is not ready may put the thread to sleep while another one, which
        // is, waits to be noticed (about 0.3 us per tile, measured).
        if (leader && lane == 0) {
            const int part = warp == 1 ? 0 : warp == 3 ? 1 : warp == 8 ? 2 : warp == 9 ? 3 : warp - 10;
            const bool has_o = warp >= 10;  // warps 10 and 11 issue O half `part`, no S
            const uint32_t id_s = idesc_f16(128, 64, false, false);
            const uint32_t id_o = idesc_f16(128, 256, false, true);
            const int n_items_w = i_end - i_begin;
            int si = 0, sj = 0, sg = 0;  // S cursor: item, tile in item, global tile
            int oi = 0, oj = 0, og = 0;  // O cursor
            bool s_q = false;            // Q of item si waited for
            ItemGeom gs = n_items_w > 0 ? item_geom(items, i_begin, seq_lens, bs, cap, flags, false)
                                        : ItemGeom{0, 0, 0, 0};
            ItemGeom go = gs;
            uint64_t idle_since = 0, next_check = 0;
            while (has_o ? oi < n_items_w : si < n_items_w) {
                bool did = false;
                if (!has_o && si < n_items_w) {
                    if (!s_q && mbar_test_wait(mb + kBarQFull, si & 1)) {
                        s_q = true;
                        tc_fence_after();
                    }
                    if (s_q) {
                        if (sj >= gs.n_tiles) {
                            mma_commit_pair(mb + kBarQFree, 0x3);  // every S of item si issued
                            if (++si < n_items_w)
                                gs = item_geom(items, i_begin + si, seq_lens, bs, cap, flags, false);
                            sj = 0;
                            s_q = false;
                            did = true;
                        } else if ((sg < kSBufs ||
                                    mbar_test_wait(mb + kBarPFull + 8 * ((sg - kSBufs) & 1),
                                                  ((sg - kSBufs) >> 1) & 1)) &&
                                   mbar_test_wait(mb + kBarKFull + 8 * (sg & 1), (sg >> 1) & 1)) {
                            tc_fence_after();
                            const int st = sg & 1, sb = sg % kSBufs;
                            const uint32_t kreg = sbase + kKOff + st * kKStage;
                            const int k0 = kKPer * part;
                            const uint32_t dcol = s_col(part, sb);
#pragma unroll
                            for (int k = k0; k < k0 + kKPer; ++k) {
                                const uint64_t a = sdesc_sw128(
                                    sbase + kQOff + (k >> 2) * kQAtom + (k & 3) * 32, 16, 1024);
                                const uint64_t b =
                                    sdesc_sw128(kreg + (k >> 2) * kBox + (k & 3) * 32, 16, 1024);
                                mma_pair_f16(tmem + dcol, a, b, id_s, k > k0 ? 1u : 0u);
                            }
                            mma_commit_pair(mb + kBarSFull + 8 * sb, 0x3);
                            mma_commit_pair(mb + kBarKEmpty + 8 * st, 0x3);
                            ++sj;
                            ++sg;
                            did = true;
                        }
                    }
                }
                if (!has_o) {
                } else if (oj >= go.n_tiles) {
                    if (++oi < n_items_w)
                        go = item_geom(items, i_begin + oi, seq_lens, bs, cap, flags, false);
                    oj = 0;
                    did = true;
                } else if (mbar_test_wait(mb + kBarPFull + 8 * (og & 1), (og >> 1) & 1) &&
                           (oj > 0 || oi == 0 || mbar_test_wait(mb + kBarOFree, (oi - 1) & 1))) {
                    tc_fence_after();
                    const int st = og & 1;
                    const uint32_t vreg = sbase + kVOff + st * kVStage;
                    const uint32_t preg = sbase + kPOff + st * kPBytes;
                    {
                        const int i = part;
#pragma unroll
                        for (int k = 0; k < 4; ++k) {
                            const uint64_t a = sdesc_sw128(preg + k * 32, 16, 1024);
                            const uint64_t b = sdesc_sw128(
                                vreg + (k >> 1) * 4 * kBox + (k & 1) * 2048 + i * 2 * kBox, kBox,
                                1024);
                            mma_pair_f16(tmem + kTmemO + 128 * i, a, b, id_o,
                                         (oj > 0 || k > 0) ? 1u : 0u);
                        }
                    }
                    mma_commit_pair(mb + kBarODone + 8 * st, 0x3);
                    mma_commit_pair(mb + kBarVEmpty + 8 * st, 0x3);
                    ++oj;
                    ++og;
                    did = true;
                }
                // Idle: the abort flag (shared memory) is checked on every
                // pass, the global flag word and the time limit only every
                // kFlagPollNs, so that polling stays a shared-memory loop.
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
    } else if (warp >= 4) {
        // ------------------------------------------- softmax and epilogue
        const int t = tid - 128;            // TMEM lane
        const int hl = t & 63, th = t >> 6; // head within the CTA, token / column half
        const uint32_t lane_base = static_cast<uint32_t>((warp - 4) * 32) << 16;
        const uint32_t pfull_leader0 = mapa(mb + kBarPFull, 0);
        const uint32_t pfull_leader1 = mapa(mb + kBarPFull + 8, 0);
        const uint32_t ofree_leader = mapa(mb + kBarOFree, 0);
        bool ok = true;
        int gt = 0;
        // Every softmax thread runs every iteration and reaches every named
        // barrier; after a failed wait it only skips the work.
        for (int ii = i_begin; ii < i_end; ++ii) {
            const ItemGeom g = item_geom(items, ii, seq_lens, bs, cap, flags, t == 0 && leader);
            float m_use = -INFINITY, l = 0.f;
            for (int j = 0; j < g.n_tiles; ++j) {
                const int gj = gt + j, st = gj & 1;
                const int vc = min(kTile, g.t_end - (g.t_begin + kTile * j));
                const int sb = gj % kSBufs;
                if (ok)
                    ok = __all_sync(0xffffffffu, mbar_wait(mb + kBarSFull + 8 * sb,
                                                           (gj / kSBufs) & 1, wc));
                float s[32];
                if (ok) {
                    tc_fence_after();
                    float s1[32];
                    tmem_ld32(tmem + lane_base + s_col(0, sb), s);
                    tmem_ld32(tmem + lane_base + s_col(1, sb), s1);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; ++i) s[i] += s1[i];
                    tmem_ld32(tmem + lane_base + s_col(2, sb), s1);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; ++i) s[i] += s1[i];
                    tmem_ld32(tmem + lane_base + s_col(3, sb), s1);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; ++i) s[i] += s1[i];
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
                    alpha = (m_use == -INFINITY) ? 0.f : fast_exp2(m_use - m_new);
                    m_use = m_new;
                    l *= alpha;
                }
                const float mneg = (m_use == -INFINITY) ? 0.f : -m_use;
                uint32_t packed[16];
                float psum = 0.f;
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const float p0 = fast_exp2(s[2 * i] + mneg);
                    const float p1 = fast_exp2(s[2 * i + 1] + mneg);
                    psum += p0 + p1;
                    const __half2 h = __floats2half2_rn(p0, p1);
                    packed[i] = *reinterpret_cast<const uint32_t*>(&h);
                }
                l += psum;
                if (ok && gj >= 2)  // P buffer `st` is free once O of tile gj-2 completed
                    ok = __all_sync(0xffffffffu, mbar_wait(mb + kBarODone + 8 * st,
                                                           ((gj - 2) >> 1) & 1, wc));
                if (ok && __any_sync(0xffffffffu, resc && j > 0)) {
                    const int jp = gj - 1;  // rescale O accumulated through tile gj-1
                    ok = __all_sync(0xffffffffu, mbar_wait(mb + kBarODone + 8 * (jp & 1),
                                                           (jp >> 1) & 1, wc));
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
                if (ok) {
                    uint8_t* prow = smem + kPOff + st * kPBytes + (hl >> 3) * 1024 + (hl & 7) * 128;
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const uint32_t chunk = static_cast<uint32_t>((th * 4 + u) ^ (hl & 7));
                        *reinterpret_cast<uint4*>(prow + chunk * 16) = make_uint4(
                            packed[4 * u], packed[4 * u + 1], packed[4 * u + 2], packed[4 * u + 3]);
                    }
                    // The V tile of this CTA must have landed before O reads it
                    // (and before rows past the end are cleared).
                    ok = __all_sync(0xffffffffu, mbar_wait(mb + kBarVFull + 8 * st, (gj >> 1) & 1,
                                                           wc));
                }
                if (ok && vc < kTile) {
                    // Rows past the end of the item: zero their value rows so
                    // that p = 0 times whatever the pool holds there stays 0.
                    uint8_t* vreg = smem + kVOff + st * kVStage;
                    const int rows = kTile - vc;
                    for (int idx = t; idx < rows * 32; idx += 128) {
                        const int tok = vc + idx / 32, rem = idx % 32, s4 = rem >> 3, c16 = rem & 7;
                        const int h = tok >> 5, rr = tok & 31;
                        *reinterpret_cast<uint4*>(vreg + h * 4 * kBox + s4 * kBox + (rr >> 3) * 1024 +
                                                  (rr & 7) * 128 + c16 * 16) = make_uint4(0, 0, 0, 0);
                    }
                }
                fence_proxy_async_smem();
                tc_fence_before();
                named_sync_softmax();
                if (ok && t == 0) mbar_arrive_cluster(st ? pfull_leader1 : pfull_leader0);
            }
            // Epilogue of the item: partial (m, l, context) of this CTA's heads.
            if (ok && g.n_tiles > 0) {
                const int jl = gt + g.n_tiles - 1;
                ok = __all_sync(0xffffffffu, mbar_wait(mb + kBarODone + 8 * (jl & 1), (jl >> 1) & 1,
                                                       wc));
            }
            red_sum[t] = l;
            named_sync_softmax();
            const float l_tot = l + red_sum[t ^ 64];
            const int64_t row = (int64_t)ii * kHeads + kHeadsPerCta * rank + hl;
            if (th == 0) {
                ws.part_m[row] = (ok && m_use != -INFINITY) ? m_use * kLn2 : -INFINITY;
                ws.part_l[row] = ok ? l_tot : 0.f;
            }
            // Context rows, staged through the two P buffers (idle: every O
            // MMA of the item completed) so that the global stores are whole
            // 128-byte lines: thread t holds 32 columns of one head, and a
            // warp stores four heads' 128-byte segments per instruction.
            // Storing straight from the TMEM lanes (one head per thread, a
            // 2 KiB stride between threads) took 5.3 us per item.
            const bool have = ok && g.n_tiles > 0;
            if (have) tc_fence_after();
            uint8_t* stage = smem + kPOff;  // [128 threads][8 chunks of 16 B], chunk c at c ^ (t & 7)
            float* ctx_base = ws.part_ctx + ((int64_t)ii * kHeads + kHeadsPerCta * rank) * kValue;
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
                named_sync_softmax();  // the previous iteration's reads of the stage are done
#pragma unroll
                for (int c = 0; c < 8; ++c)
                    *reinterpret_cast<float4*>(stage + t * 128 + ((c ^ (t & 7)) << 4)) =
                        make_float4(o[4 * c], o[4 * c + 1], o[4 * c + 2], o[4 * c + 3]);
                named_sync_softmax();
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    const int idx = t + 128 * k, r = idx >> 3, c = idx & 7;
                    const float4 v =
                        *reinterpret_cast<const float4*>(stage + r * 128 + ((c ^ (r & 7)) << 4));
                    const int col = (r >> 6) * 256 + (u >> 2) * 128 + (u & 3) * 32 + 4 * c;
                    *reinterpret_cast<float4*>(ctx_base + (int64_t)(r & 63) * kValue + col) = v;
                }
            }
            tc_fence_before();
            named_sync_softmax();
            if (ok && t == 0) mbar_arrive_cluster(ofree_leader);
            gt += g.n_tiles;
        }
    }

    // Teardown: every role is done with shared and tensor memory.
    tc_fence_before();
    __syncthreads();
    cluster_sync();
    tc_fence_after();
    if (warp == 1) tmem_dealloc_pair(tmem, kTmemCols);
}

// q16[b, h, l] = FP16(q_lat[b, h, l] * qscale), the TMA source of Q; also
// clears the launch's control words (the partial pass follows in stream order).
__global__ void q_prep_kernel(const float4* __restrict__ q, uint2* __restrict__ q16, float qscale,
                              int64_t n4, int32_t* __restrict__ ctl) {
    if (blockIdx.x == 0 && threadIdx.x < kCtlBytes / 4) ctl[threadIdx.x] = 0;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4;
         i += (int64_t)gridDim.x * blockDim.x) {
        const float4 v = q[i];
        const __half2 a = __floats2half2_rn(v.x * qscale, v.y * qscale);
        const __half2 b = __floats2half2_rn(v.z * qscale, v.w * qscale);
        q16[i] = make_uint2(*reinterpret_cast<const uint32_t*>(&a),
                            *reinterpret_cast<const uint32_t*>(&b));
    }
}

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

static bool encode_f16(CUtensorMap* map, const void* base, int rank, const cuuint64_t* dims,
                       const cuuint64_t* strides, const cuuint32_t* box) {
    cuuint32_t estr[4] = {1, 1, 1, 1};
    return g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, rank, const_cast<void*>(base),
                    dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool encode_map(CUtensorMap* map, CUtensorMapDataType type, const void* base, int rank,
                const cuuint64_t* dims, const cuuint64_t* strides, const cuuint32_t* box,
                CUtensorMapSwizzle swizzle) {
    if (!load_encode()) return false;
    cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    return g_encode(map, type, rank, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace tc

bool tc_supported(const plkv_latent_decode_args& a) {
    return a.q_heads == tc::kHeads && a.latent_dim == tc::kLatent && a.value_dim == tc::kValue &&
           a.block_size % 32 == 0 && !a.scores && !a.probs &&
           a.num_physical * (int64_t)a.block_size < (1ll << 31) &&
           (int64_t)a.batch * tc::kHeads < (1ll << 31) &&
           (reinterpret_cast<uintptr_t>(a.cache) & 15) == 0 &&
           (reinterpret_cast<uintptr_t>(a.q_lat) & 15) == 0;
}

cudaError_t launch_latent_partial_tc(const plkv_latent_decode_args& a, DecodeWorkspace ws,
                                     cudaStream_t st) {
    if (!tc::load_encode() || !ws.q16) return cudaErrorNotSupported;
    CUtensorMap k_map, v_map, q_map;
    const cuuint64_t rows = static_cast<uint64_t>(a.num_physical) * a.block_size;
    const cuuint64_t row_bytes = tc::kLatent * 2;
    const cuuint64_t k_dims[3] = {64, rows, tc::kKBlocks}, k_str[2] = {row_bytes, 128};
    const cuuint32_t k_box[3] = {64, 32, tc::kKBlocks};
    const cuuint64_t v_dims[3] = {64, rows, 8}, v_str[2] = {row_bytes, 128};
    const cuuint32_t v_box[3] = {64, 32, 4};
    const cuuint64_t q_dims[3] = {64, static_cast<uint64_t>(a.batch) * tc::kHeads, tc::kKBlocks};
    const cuuint32_t q_box[3] = {64, tc::kHeadsPerCta, tc::kKBlocks};
    if (!tc::encode_f16(&k_map, a.cache, 3, k_dims, k_str, k_box) ||
        !tc::encode_f16(&v_map, a.cache, 3, v_dims, v_str, v_box) ||
        !tc::encode_f16(&q_map, ws.q16, 3, q_dims, k_str, q_box))
        return cudaErrorInvalidValue;
    const int64_t n4 = (int64_t)a.batch * tc::kHeads * tc::kLatent / 4;
    int blocks = (int)std::min<int64_t>((n4 + 255) / 256, 148 * 8);
    tc::q_prep_kernel<<<blocks, 256, 0, st>>>(reinterpret_cast<const float4*>(a.q_lat),
                                              reinterpret_cast<uint2*>(ws.q16),
                                              a.scale * 1.4426950408889634f, n4, ws.ctl);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(tc::latent_partial_tc_kernel,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tc::kSmemBytes);
    if (e != cudaSuccess) return e;
    int32_t* flags = a.err_flags;
    const int workers = (a.worker_item_begin && a.n_workers > 0) ? a.n_workers : a.n_items;
    tc::latent_partial_tc_kernel<<<2 * workers, tc::kThreads, tc::kSmemBytes, st>>>(
        k_map, v_map, q_map, a.block_size, a.block_tables, a.max_blocks, a.num_physical,
        a.seq_lens,
        a.items, (a.worker_item_begin && a.n_workers > 0) ? a.worker_item_begin : nullptr, ws,
        flags);
    return cudaGetLastError();
}

}  // namespace plkv
