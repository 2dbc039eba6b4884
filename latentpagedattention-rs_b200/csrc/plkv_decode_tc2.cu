// plkv_decode_tc2.cu -- tensor-core (tcgen05) split-K partial pass of the
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
// walks the items of one worker of plkv_plan_workers in tiles of 128 tokens,
// one 64-row block ("page") per CTA.  CTA r owns query heads [64r, 64r+64).
//   S = Q . L^T : cta_group::2 MMA, M = 128 heads, N = 128 tokens (CTA r
//                 supplies its heads' Q and its page), K = 576 (36 steps).
//   O += P . V  : cta_group::2 MMA, M = 128 heads, N = 256 value columns
//                 (two halves), K = 16 tokens; CTA r supplies its heads' P and
//                 the value blocks {4i+2r, 4i+2r+1} of half i for all tokens.
//
// Why this shape (measured on B200, one CTA pair per SM):
//   * TMA streams randomly placed pages at 2.26 TB/s when every box row is
//     one 128-byte column block, 6.2 TB/s with three column blocks (384 B)
//     per row and 7.1 TB/s with whole 1152-byte rows.  A K stage is
//     therefore 64 rows x 3 column blocks (24 KiB, one 3-D box): the rows of
//     one column block must be contiguous for the MMA, which limits a box to
//     one page, so the pair's N is 2 x 64 tokens.
//   * One thread issues a tcgen05.mma every ~72 cycles whatever its size; an
//     N = 128 pair MMA is 32 cycles of tensor work.  Two issuing threads in
//     different warps overlap (about 40 cycles per MMA together), so S is
//     split between them by column block (even blocks to issuer 0, odd to
//     issuer 1) into two TMEM partials the softmax adds, and each issuer also
//     issues one half of O.  Every K stage is consumed by both issuers at
//     once and released as soon as its 12 MMAs complete, so the K ring (one
//     tile, 72 KiB) keeps up to two stages of HBM reads in flight per CTA.
//   * V rows are read a second time, from L2 (the K loads give the rows
//     normal L2 priority, the V loads evict-first), in 32-row stages of the
//     CTA's four value blocks (a 4-D box of two 256-byte runs per row).
//
// The query is converted once per call (q_prep kernel) to FP16 pre-scaled by
// scale * log2(e) and loaded per item by TMA.  Softmax runs in the log2
// domain with a lazily updated running max: probabilities are taken against a
// stale max until a tile's max exceeds it by more than 8 (probabilities stay
// <= 2^8 in FP16); only then is the accumulated O rescaled in TMEM.  TMEM lane
// = head; a head's 128 tokens are spread over four softmax threads (two lanes,
// two column halves) that agree through shared memory.
//
// Rows past an item's end: K columns of such tokens are masked in the
// softmax; the last V stage of an item, when the item does not end on a
// 16-token step, is loaded into this CTA alone and the softmax warps zero its
// rows past the end before O reads them (p = 0 times a non-finite pool value
// would not be 0).  Pages wholly past the end are not loaded.
//
// Warp roles per CTA: 0 = Q and K loads, 1 = TMEM allocation and (leader)
// MMA issuer 0, 2 = V loads, 3 = (leader) MMA issuer 1, 4..11 = softmax and
// epilogue.  Every barrier wait is bounded (1 s): on expiry the kernel
// records PLKV_FLAG_TIMEOUT, abandons its work, releases tensor memory and
// exits.
#include <cudaTypedefs.h>

#include <cstdlib>
#include <mutex>

#include "plkv_sm100.cuh"

namespace plkv {
namespace tc2 {

constexpr int kHeads = 128;
constexpr int kHeadsPerCta = 64;
constexpr int kLatent = 576;
constexpr int kValue = 512;
constexpr int kTile = 128;                                    // tokens per tile (pair)
constexpr int kPage = 64;                                     // tokens per CTA per tile
constexpr int kCb = kLatent / 64;                             // 9 column blocks
constexpr int kCbPerStage = 3;
constexpr int kKStagesPerTile = kCb / kCbPerStage;            // 3
constexpr uint32_t kAtom = 64 * 128;                          // 64 rows x 64 FP16 (8 KiB)
constexpr uint32_t kQBytes = kCb * kAtom;                     // 72 KiB
constexpr uint32_t kKStage = kCbPerStage * kAtom;             // 24 KiB
#ifndef PLKV_TC2_NK
#define PLKV_TC2_NK 3
#endif
#ifndef PLKV_TC2_NV
#define PLKV_TC2_NV 3
#endif
constexpr int kNK = PLKV_TC2_NK;                              // K ring stages (24 KiB)
constexpr int kVRows = 32;
constexpr uint32_t kVBox = kVRows * 128;                      // 4 KiB: 32 rows x 64 FP16
constexpr uint32_t kVStage = 4 * kVBox;                       // 16 KiB
constexpr int kNV = PLKV_TC2_NV;                              // V ring stages (16 KiB)
constexpr uint32_t kPBytes = 2 * kAtom;                       // 16 KiB: 64 heads x 128 tokens
constexpr uint32_t kQOff = 0;
constexpr uint32_t kKOff = kQOff + kQBytes;
constexpr uint32_t kVOff = kKOff + kNK * kKStage;
constexpr uint32_t kPOff = kVOff + kNV * kVStage;
constexpr uint32_t kMiscOff = kPOff + 2 * kPBytes;
constexpr uint32_t kMiscBytes = 2048;
constexpr uint32_t kSmemBytes = kMiscOff + kMiscBytes;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemO = 0;                                // O half i at 128 i
__host__ __device__ constexpr uint32_t s_col(int p, int b) { return 256u + 64u * (2 * p + b); }
constexpr float kTau = 8.f;
constexpr float kLn2 = 0.6931471805599453f;

enum : uint32_t {
    kBarQFull = 0,              // leader: Q of the item landed in both CTAs
    kBarQFree = 8,              // both: every S MMA of the item completed
    kBarOFree = 16,             // leader: epilogue of the item read O in both CTAs
    kBarVTail = 24,             // own: this CTA's tail V stage landed
    kBarVReady = 32,            // leader: tail V rows zeroed in both CTAs
    kBarKFull = 40,             // [kNK] leader
    kBarKEmpty = kBarKFull + 8 * kNK,     // [kNK] both
    kBarVFull = kBarKEmpty + 8 * kNK,     // [kNV] leader
    kBarVEmpty = kBarVFull + 8 * kNV,     // [kNV] both
    kBarSFull = kBarVEmpty + 8 * kNV,     // [2] both: S partials of the tile in TMEM
    kBarSFree = kBarSFull + 16,           // [2] leader: both CTAs read S
    kBarPFull = kBarSFree + 16,           // [2] leader: P written in both CTAs
    kBarODone = kBarPFull + 16,           // [2] both: O of the tile completed
    kTmemSlot = kBarODone + 16,
    kAbort = kTmemSlot + 4,
    kRedMax = 512,              // [4][64] float: tile max (softmax) / row sum (epilogue)
    kRedSum = kRedMax,
};
static_assert(kAbort + 4 <= kRedMax, "barriers");
static_assert(kRedMax + 1024 <= kMiscBytes, "misc region");
static_assert(kSmemBytes <= 232448, "shared memory budget");

__device__ __forceinline__ void named_sync_softmax() {
    asm volatile("bar.sync 1, 256;" ::: "memory");
}

__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Rows [y, y + 64) x column blocks [z, z + 3) of the latent pool in one
// instruction (3-D view: 64 columns, rows, 9 column blocks at 128 B); lands
// as three 64-row K-major SWIZZLE_128B atoms.  Completes on a barrier of the
// leader CTA (cta_group::2); no multicast.
__device__ __forceinline__ void tma_k_pair(uint32_t dst, const CUtensorMap* map, int y, int z,
                                           uint32_t cluster_bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        ".L2::cache_hint [%0], [%1, {%2, %3, %4}], [%5], %6;"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(0), "r"(y), "r"(z),
          "r"(cluster_bar), "l"(policy)
        : "memory");
}
// The four value blocks [z0, z0 + 4) of 32 rows (3-D view: 64 columns, rows,
// 8 blocks at 128 B: one 512-byte run per row).  Pair form: completes on the
// leader's barrier; own form: on a barrier of this CTA.
__device__ __forceinline__ void tma_v_pair(uint32_t dst, const CUtensorMap* map, int y, int z0,
                                           uint32_t cluster_bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        ".L2::cache_hint [%0], [%1, {%2, %3, %4}], [%5], %6;"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(0), "r"(y), "r"(z0),
          "r"(cluster_bar), "l"(policy)
        : "memory");
}
__device__ __forceinline__ void tma_v_own(uint32_t dst, const CUtensorMap* map, int y, int z0,
                                          uint32_t bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
        ".L2::cache_hint [%0], [%1, {%2, %3, %4}], [%5], %6;"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(0), "r"(y), "r"(z0), "r"(bar),
          "l"(policy)
        : "memory");
}
// Q rows [y, y + 64) x all nine column blocks (3-D), pair form.
__device__ __forceinline__ void tma_q_pair(uint32_t dst, const CUtensorMap* map, int y,
                                           uint32_t cluster_bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        ".L2::cache_hint [%0], [%1, {%2, %3, %4}], [%5], %6;"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(0), "r"(y), "r"(0),
          "r"(cluster_bar), "l"(policy)
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

// Valid tokens of tile j of an item.
__device__ __forceinline__ int tile_valid(const ItemGeom& g, int j) {
    return min(kTile, g.t_end - (g.t_begin + kTile * j));
}

// Pool row of token `tok` of sequence `seq` (block-table lookup).
__device__ __forceinline__ int pool_row(int seq, int tok, const int32_t* __restrict__ tables,
                                        int64_t max_blocks, int64_t num_physical, int bs,
                                        int32_t* flags) {
    const int lb = tok / bs;
    int32_t phys = tables[(int64_t)seq * max_blocks + lb];
    if (phys < 0 || phys >= num_physical) {
        set_flag(flags, PLKV_FLAG_BAD_BLOCK);
        phys = 0;
    }
    return phys * bs + (tok - lb * bs);
}

// Tail V stage of the item's last tile (the stage holding token vc - 1 when
// vc is not a multiple of 16), or -1.
__device__ __forceinline__ int tail_stage(const ItemGeom& g, int j) {
    if (j != g.n_tiles - 1) return -1;
    const int vc = tile_valid(g, j);
    return (vc % 16) ? (vc - 1) / kVRows : -1;
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(384, 1)
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
        mbar_init(mb + kBarQFree, 2);
        mbar_init(mb + kBarOFree, 2);
        mbar_init(mb + kBarVTail, 1);
        mbar_init(mb + kBarVReady, 2);
        for (int i = 0; i < kNK; ++i) {
            mbar_init(mb + kBarKFull + 8 * i, 1);
            mbar_init(mb + kBarKEmpty + 8 * i, 2);
        }
        for (int i = 0; i < kNV; ++i) {
            mbar_init(mb + kBarVFull + 8 * i, 1);
            mbar_init(mb + kBarVEmpty + 8 * i, 2);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(mb + kBarSFull + 8 * i, 2);
            mbar_init(mb + kBarSFree + 8 * i, 2);
            mbar_init(mb + kBarPFull + 8 * i, 2);
            mbar_init(mb + kBarODone + 8 * i, 2);
        }
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
            // K rows are read again, from L2, by the V loads of both CTAs:
            // normal priority here, evict-first on the V loads (their last use).
            const uint64_t pol = policy_evict_normal();
            const uint32_t qfull = mapa(mb + kBarQFull, 0);
            int ks = 0;  // K stage counter over the worker's items
            int nq = 0;  // Q loads so far (items with tokens)
            bool ok = true;
            for (int ii = i_begin; ok && ii < i_end; ++ii) {
                const ItemGeom g = item_geom(items, ii, seq_lens, bs, cap, flags, false);
                if (g.n_tiles == 0) continue;
                auto load_q = [&]() -> bool {
                    if (nq >= 1 && !mbar_wait(mb + kBarQFree, (nq - 1) & 1, wc)) return false;
                    ++nq;
                    if (leader) mbar_arrive_expect_tx(mb + kBarQFull, 2u * kQBytes);
                    tma_q_pair(sbase + kQOff, &q_map, g.seq * kHeads + kHeadsPerCta * (int)rank,
                               qfull, pol);
                    return true;
                };
                // The first K stages of an item only need free slots; Q waits
                // for every S MMA of the previous item, so it follows them.
                const int pre = min(kNK, kKStagesPerTile * g.n_tiles);
                int sidx = 0;  // stage index within the item
                // This CTA's page row of tile j, looked up one tile ahead so
                // that the table read overlaps the waits for free stages.
                auto page_row = [&](int j) -> int {
                    return (j < g.n_tiles && kPage * (int)rank < tile_valid(g, j))
                               ? pool_row(g.seq, g.t_begin + kTile * j + kPage * (int)rank, tables,
                                          max_blocks, num_physical, bs, flags)
                               : 0;
                };
                int y_next = page_row(0);
                for (int j = 0; ok && j < g.n_tiles; ++j) {
                    const int vc = tile_valid(g, j);
                    const bool mine = kPage * (int)rank < vc;      // this CTA's page exists
                    const bool both = kPage < vc;
                    const int y = y_next;
                    y_next = page_row(j + 1);
                    for (int c = 0; c < kKStagesPerTile; ++c, ++sidx) {
                        if (sidx == pre && !(ok = load_q())) break;
                        const int st = ks % kNK;
                        if (ks >= kNK &&
                            !(ok = mbar_wait(mb + kBarKEmpty + 8 * st, ((ks / kNK) - 1) & 1, wc)))
                            break;
                        if (leader)
                            mbar_arrive_expect_tx(mb + kBarKFull + 8 * st,
                                                  (both ? 2u : 1u) * kKStage);
                        if (mine)
                            tma_k_pair(sbase + kKOff + st * kKStage, &k_map, y, kCbPerStage * c,
                                       mapa(mb + kBarKFull + 8 * st, 0), pol);
                        ++ks;
                    }
                }
                if (ok && pre == kKStagesPerTile * g.n_tiles) ok = load_q();
            }
        }
        __syncwarp();
    } else if (warp == 2) {
        // --------------------------------------------------------- V loads
        if (lane == 0) {
            const uint64_t pol = policy_evict_first();
            int vs = 0;  // V stage counter (stages past an item's end are skipped)
            bool ok = true;
            for (int ii = i_begin; ok && ii < i_end; ++ii) {
                const ItemGeom g = item_geom(items, ii, seq_lens, bs, cap, flags, false);
                // Rows of the tile's two pages, looked up one tile ahead.
                auto page_rows = [&](int j, int* r) {
                    for (int h = 0; h < 2; ++h)
                        r[h] = (j < g.n_tiles && kPage * h < tile_valid(g, j))
                                   ? pool_row(g.seq, g.t_begin + kTile * j + kPage * h, tables,
                                              max_blocks, num_physical, bs, flags)
                                   : 0;
                };
                int nxt[2];
                page_rows(0, nxt);
                for (int j = 0; ok && j < g.n_tiles; ++j) {
                    const int vc = tile_valid(g, j);
                    const int tail = tail_stage(g, j);
                    const int pr0 = nxt[0], pr1 = nxt[1];
                    page_rows(j + 1, nxt);
                    for (int v = 0; v * kVRows < vc; ++v) {
                        const int st = vs % kNV;
                        if (vs >= kNV &&
                            !(ok = mbar_wait(mb + kBarVEmpty + 8 * st, ((vs / kNV) - 1) & 1, wc)))
                            break;
                        const int y = (v < 2 ? pr0 : pr1) + kVRows * (v & 1);
                        const uint32_t dst = sbase + kVOff + st * kVStage;
                        if (v != tail) {
                            if (leader) mbar_arrive_expect_tx(mb + kBarVFull + 8 * st, 2u * kVStage);
                            tma_v_pair(dst, &v_map, y, 4 * (int)rank,
                                       mapa(mb + kBarVFull + 8 * st, 0), pol);
                        } else {
                            // Landed in this CTA alone: the softmax warps zero
                            // its rows past the end, then report to the leader.
                            mbar_arrive_expect_tx(mb + kBarVTail, kVStage);
                            tma_v_own(dst, &v_map, y, 4 * (int)rank, mb + kBarVTail, pol);
                            if (leader) mbar_arrive_local(mb + kBarVFull + 8 * st);
                        }
                        ++vs;
                    }
                }
            }
        }
        __syncwarp();
    } else if (warp == 1 || warp == 3) {
        // ---------------------------------------------- MMA issue (leader)
        // Issuer p: the S partial over column blocks cb = p, p + 2, ... of
        // every tile (p = 0: blocks 0, 2, 4, 6, 8; p = 1: 1, 3, 5, 7), and O
        // half p.  Each issuer schedules without blocking: the next K stage of
        // S as soon as it landed (its tile's S buffer free, its item's Q
        // loaded), and the next V stage of O as soon as it landed and the
        // tile's P is ready, so that S of later tiles stays queued on the
        // tensor pipe while the softmax of earlier ones runs.  Barriers are
        // polled with test_wait, which never suspends the thread.
        if (leader && lane == 0) {
            const int p = warp == 1 ? 0 : 1;
            const uint32_t id_s = idesc_f16(128, kTile, false, false);
            const uint32_t id_o = idesc_f16(128, 256, false, true);
            // S cursor
            int si = i_begin, sj = 0, sc = 0, sg = 0, ks = 0, nq = 0;
            bool s_q = false, s_free = false;
            ItemGeom gs = si < i_end ? item_geom(items, si, seq_lens, bs, cap, flags, false)
                                     : ItemGeom{0, 0, 0, 0};
            // O cursor
            int oi = i_begin, oj = 0, ov = 0, og = 0, vs = 0, tails = 0;
            bool o_p = false;
            ItemGeom go = gs;
            uint64_t idle_since = 0, next_check = 0;
            while (si < i_end || oi < i_end) {
                bool did = false;
                if (si < i_end) {
                    if (sj >= gs.n_tiles) {  // next item (its Q, if it has tokens)
                        if (++si < i_end) gs = item_geom(items, si, seq_lens, bs, cap, flags, false);
                        sj = 0;
                        s_q = false;
                        did = true;
                    } else {
                        if (!s_q && mbar_test_wait(mb + kBarQFull, nq & 1)) s_q = true;
                        if (s_q && !s_free &&
                            (sg < 2 || mbar_test_wait(mb + kBarSFree + 8 * (sg & 1),
                                                      ((sg - 2) >> 1) & 1)))
                            s_free = true;
                        const int st = ks % kNK;
                        if (s_q && s_free && mbar_test_wait(mb + kBarKFull + 8 * st, (ks / kNK) & 1)) {
                            tc_fence_after();
                            const int sb = sg & 1;
                            const uint32_t kreg = sbase + kKOff + st * kKStage;
                            for (int cc = 0; cc < kCbPerStage; ++cc) {
                                const int cb = kCbPerStage * sc + cc;
                                if ((cb & 1) != p) continue;
#pragma unroll
                                for (int kq = 0; kq < 4; ++kq) {
                                    const uint64_t a =
                                        sdesc_sw128(sbase + kQOff + cb * kAtom + kq * 32, 16, 1024);
                                    const uint64_t b =
                                        sdesc_sw128(kreg + cc * kAtom + kq * 32, 16, 1024);
                                    mma_pair_f16(tmem + s_col(p, sb), a, b, id_s,
                                                 (cb == p && kq == 0) ? 0u : 1u);
                                }
                            }
                            mma_commit_pair(mb + kBarKEmpty + 8 * st, 0x3);
                            ++ks;
                            if (++sc == kKStagesPerTile) {
                                mma_commit_pair(mb + kBarSFull + 8 * sb, 0x3);
                                if (sj == gs.n_tiles - 1) {
                                    mma_commit_pair(mb + kBarQFree, 0x3);
                                    ++nq;
                                }
                                sc = 0;
                                ++sj;
                                ++sg;
                                s_free = false;
                            }
                            did = true;
                        }
                    }
                }
                if (oi < i_end && (oi < si || (oi == si && oj < sj))) {
                    // O of tile og (item oi, tile oj) once its S was issued
                    if (oj >= go.n_tiles) {
                        if (++oi < i_end) go = item_geom(items, oi, seq_lens, bs, cap, flags, false);
                        oj = 0;
                        did = true;
                    } else {
                        const int pb = og & 1;
                        if (!o_p && mbar_test_wait(mb + kBarPFull + 8 * pb, (og >> 1) & 1) &&
                            (oj > 0 || oi == i_begin ||
                             mbar_test_wait(mb + kBarOFree, (oi - i_begin - 1) & 1)))
                            o_p = true;
                        const int vc = tile_valid(go, oj);
                        const int tail = tail_stage(go, oj);
                        const int st = vs % kNV;
                        if (o_p && mbar_test_wait(mb + kBarVFull + 8 * st, (vs / kNV) & 1) &&
                            (ov != tail || mbar_test_wait(mb + kBarVReady, tails & 1))) {
                            tc_fence_after();
                            const int ksteps = (vc + 15) / 16;
                            const uint32_t preg = sbase + kPOff + pb * kPBytes;
                            const uint32_t vreg = sbase + kVOff + st * kVStage + p * 2 * kVBox;
                            for (int kk = 2 * ov; kk < min(2 * ov + 2, ksteps); ++kk) {
                                const uint64_t a = sdesc_sw128(
                                    preg + (kk >> 2) * kAtom + (kk & 3) * 32, 16, 1024);
                                const uint64_t b = sdesc_sw128(vreg + (kk & 1) * 2048, kVBox, 1024);
                                mma_pair_f16(tmem + kTmemO + 128 * p, a, b, id_o,
                                             (oj > 0 || kk > 0) ? 1u : 0u);
                            }
                            mma_commit_pair(mb + kBarVEmpty + 8 * st, 0x3);
                            if (ov == tail) ++tails;
                            ++vs;
                            if (++ov * kVRows >= vc) {
                                mma_commit_pair(mb + kBarODone + 8 * pb, 0x3);
                                ov = 0;
                                ++oj;
                                ++og;
                                o_p = false;
                            }
                            did = true;
                        }
                    }
                }
                // Idle: the abort flag (shared memory) is checked on every
                // pass, the launch's abort word and the time limit only every
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
        const int ts = tid - 128;                 // 0..255
        const int wq = (warp - 4) & 3;            // TMEM lane quadrant
        const int ch = (warp - 4) >> 2;           // column half (S: 32-column half; O: half)
        const int t = 32 * wq + lane;             // TMEM lane
        const int hl = t & 63, th = t >> 6;       // head in the CTA, token / value half
        const int red = th * 2 + ch;              // the head's four threads
        const uint32_t lane_base = static_cast<uint32_t>(32 * wq) << 16;
        const uint32_t sfree_leader0 = mapa(mb + kBarSFree, 0), sfree_leader1 = mapa(mb + kBarSFree + 8, 0);
        const uint32_t pfull_leader0 = mapa(mb + kBarPFull, 0), pfull_leader1 = mapa(mb + kBarPFull + 8, 0);
        const uint32_t ofree_leader = mapa(mb + kBarOFree, 0);
        const uint32_t vready_leader = mapa(mb + kBarVReady, 0);
        bool ok = true;
        int g = 0, vs = 0, tails = 0;
        // Every softmax thread runs every iteration and reaches every named
        // barrier; after a failed wait it only skips the work.
        for (int ii = i_begin; ii < i_end; ++ii) {
            const ItemGeom gi = item_geom(items, ii, seq_lens, bs, cap, flags, ts == 0 && leader);
            float m_use = -INFINITY, l = 0.f;
            for (int j = 0; j < gi.n_tiles; ++j, ++g) {
                const int b = g & 1;
                const int vc = tile_valid(gi, j);
                if (ok)
                    ok = __all_sync(0xffffffffu, mbar_wait(mb + kBarSFull + 8 * b, (g >> 1) & 1, wc));
                float s[32];
                if (ok) {
                    tc_fence_after();
                    float s1[32];
                    tmem_ld32(tmem + lane_base + s_col(0, b) + 32 * ch, s);
                    tmem_ld32(tmem + lane_base + s_col(1, b) + 32 * ch, s1);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; ++i) s[i] += s1[i];
                } else {
#pragma unroll
                    for (int i = 0; i < 32; ++i) s[i] = -INFINITY;
                }
                // S buffer b may be rewritten once both CTAs read it.
                tc_fence_before();
                float mx = -INFINITY;
                const int tok0 = kPage * th + 32 * ch;
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    if (tok0 + i >= vc) s[i] = -INFINITY;
                    mx = fmaxf(mx, s[i]);
                }
                // One buffer suffices: the next tile's writes follow the
                // named barrier before P is published, after every read below.
                red_max[red * 64 + hl] = mx;
                named_sync_softmax();
                if (ok && ts == 0) mbar_arrive_cluster(b ? sfree_leader1 : sfree_leader0);
                float mt = red_max[hl];
#pragma unroll
                for (int k = 1; k < 4; ++k) mt = fmaxf(mt, red_max[k * 64 + hl]);
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
                    const __half2 h2 = __floats2half2_rn(p0, p1);
                    packed[i] = *reinterpret_cast<const uint32_t*>(&h2);
                }
                l += psum;
                if (ok && g >= 2)  // P buffer b is free once O of tile g - 2 completed
                    ok = __all_sync(0xffffffffu,
                                    mbar_wait(mb + kBarODone + 8 * b, ((g - 2) >> 1) & 1, wc));
                if (ok && __any_sync(0xffffffffu, resc && j > 0)) {
                    const int gp = g - 1;  // rescale O accumulated through tile g - 1
                    ok = __all_sync(0xffffffffu, mbar_wait(mb + kBarODone + 8 * (gp & 1),
                                                           (gp >> 1) & 1, wc));
                    if (ok) {
                        tc_fence_after();
#pragma unroll 1
                        for (int u = 0; u < 4; ++u) {
                            float o[32];
                            tmem_ld32(tmem + lane_base + kTmemO + 128 * ch + 32 * u, o);
                            tmem_wait_ld();
#pragma unroll
                            for (int e = 0; e < 32; ++e) o[e] *= alpha;
                            tmem_st32(tmem + lane_base + kTmemO + 128 * ch + 32 * u, o);
                        }
                        tmem_wait_st();
                    }
                }
                if (ok) {
                    // P[head][token], token block th, 128-byte row hl, chunks
                    // 4 ch .. 4 ch + 3 (SWIZZLE_128B: chunk c at c ^ (hl & 7)).
                    uint8_t* prow = smem + kPOff + b * kPBytes + th * kAtom + (hl >> 3) * 1024 +
                                    (hl & 7) * 128;
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const uint32_t chunk = static_cast<uint32_t>((4 * ch + u) ^ (hl & 7));
                        *reinterpret_cast<uint4*>(prow + chunk * 16) = make_uint4(
                            packed[4 * u], packed[4 * u + 1], packed[4 * u + 2], packed[4 * u + 3]);
                    }
                }
                fence_proxy_async_smem();
                tc_fence_before();
                named_sync_softmax();
                if (ok && ts == 0) mbar_arrive_cluster(b ? pfull_leader1 : pfull_leader0);
                // V stages of this tile (the producer's and issuers' count).
                const int tail = tail_stage(gi, j);
                const int nvs = (vc + kVRows - 1) / kVRows;
                if (tail >= 0) {
                    // Zero the tail stage's rows past the end in this CTA,
                    // once it landed, then report to the leader.
                    if (ok)
                        ok = __all_sync(0xffffffffu, mbar_wait(mb + kBarVTail, tails & 1, wc));
                    if (ok) {
                        uint8_t* vreg = smem + kVOff + ((vs + tail) % kNV) * kVStage;
                        const int r0 = vc - kVRows * tail;
                        const int r1 = min(kVRows, (vc + 15) / 16 * 16 - kVRows * tail);
                        for (int idx = ts; idx < (r1 - r0) * 32; idx += 256) {
                            const int rr = r0 + idx / 32, rem = idx % 32, blk = rem >> 3,
                                      c16 = rem & 7;
                            *reinterpret_cast<uint4*>(vreg + blk * kVBox + (rr >> 3) * 1024 +
                                                      (rr & 7) * 128 + c16 * 16) =
                                make_uint4(0, 0, 0, 0);
                        }
                    }
                    fence_proxy_async_smem();
                    named_sync_softmax();
                    if (ok && ts == 0) mbar_arrive_cluster(vready_leader);
                    ++tails;
                }
                vs += nvs;
            }
            // Epilogue of the item: partial (m, l, context) of this CTA's heads.
            if (ok && gi.n_tiles > 0) {
                const int gl = g - 1;
                ok = __all_sync(0xffffffffu, mbar_wait(mb + kBarODone + 8 * (gl & 1),
                                                       (gl >> 1) & 1, wc));
            }
            red_sum[red * 64 + hl] = l;
            named_sync_softmax();
            const float l_tot = red_sum[hl] + red_sum[64 + hl] + red_sum[128 + hl] +
                                red_sum[192 + hl];
            const int64_t row0 = (int64_t)ii * kHeads + kHeadsPerCta * rank;
            if (red == 0) {
                ws.part_m[row0 + hl] = (ok && m_use != -INFINITY) ? m_use * kLn2 : -INFINITY;
                ws.part_l[row0 + hl] = ok ? l_tot : 0.f;
            }
            // Context rows, staged through the two P buffers (idle: every O
            // MMA of the item completed) so that the global stores are whole
            // 128-byte lines.  Thread (t, ch) holds value columns
            // 256 ch + 128 th + 32 u .. + 32 of head hl.
            const bool have = ok && gi.n_tiles > 0;
            if (have) tc_fence_after();
            uint8_t* stage = smem + kPOff;  // [256 threads][8 chunks of 16 B], chunk c at c ^ (ts & 7)
            float* ctx_base = ws.part_ctx + row0 * kValue;
#pragma unroll 1
            for (int u = 0; u < 4; ++u) {
                float o[32];
                if (have) {
                    tmem_ld32(tmem + lane_base + kTmemO + 128 * ch + 32 * u, o);
                    tmem_wait_ld();
                } else {
#pragma unroll
                    for (int e = 0; e < 32; ++e) o[e] = 0.f;
                }
                named_sync_softmax();  // the previous round's reads of the stage are done
#pragma unroll
                for (int c = 0; c < 8; ++c)
                    *reinterpret_cast<float4*>(stage + ts * 128 + ((c ^ (ts & 7)) << 4)) =
                        make_float4(o[4 * c], o[4 * c + 1], o[4 * c + 2], o[4 * c + 3]);
                named_sync_softmax();
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    const int idx = ts + 256 * k, r = idx >> 3, c = idx & 7;
                    const float4 v =
                        *reinterpret_cast<const float4*>(stage + r * 128 + ((c ^ (r & 7)) << 4));
                    // thread r of the softmax group: lane t_r, column half ch_r
                    const int wr = r >> 5, t_r = 32 * (wr & 3) + (r & 31), ch_r = wr >> 2;
                    const int col = 256 * (t_r >> 6) + 128 * ch_r + 32 * u + 4 * c;
                    *reinterpret_cast<float4*>(ctx_base + (int64_t)(t_r & 63) * kValue + col) = v;
                }
            }
            tc_fence_before();
            named_sync_softmax();
            if (ok && ts == 0) mbar_arrive_cluster(ofree_leader);
        }
    }

    // Teardown: every role is done with shared and tensor memory.
    tc_fence_before();
    __syncthreads();
    cluster_sync();
    tc_fence_after();
    if (warp == 1) tmem_dealloc_pair(tmem, kTmemCols);
}

}  // namespace tc2

namespace tc {
__global__ void q_prep_kernel(const float4* __restrict__ q, uint2* __restrict__ q16, float qscale,
                              int64_t n4, int32_t* __restrict__ ctl);
bool encode_f16_map(CUtensorMap* map, const void* base, int rank, const cuuint64_t* dims,
                    const cuuint64_t* strides, const cuuint32_t* box);
}  // namespace tc

bool tc2_supported(const plkv_latent_decode_args& a) {
    return a.q_heads == tc2::kHeads && a.latent_dim == tc2::kLatent &&
           a.value_dim == tc2::kValue && a.block_size % 64 == 0 && !a.scores && !a.probs &&
           a.num_physical * (int64_t)a.block_size < (1ll << 31) &&
           (int64_t)a.batch * tc2::kHeads < (1ll << 31) &&
           (reinterpret_cast<uintptr_t>(a.cache) & 15) == 0 &&
           (reinterpret_cast<uintptr_t>(a.q_lat) & 15) == 0;
}

cudaError_t launch_latent_partial_tc2(const plkv_latent_decode_args& a, DecodeWorkspace ws,
                                      cudaStream_t st) {
    if (!ws.q16) return cudaErrorNotSupported;
    CUtensorMap k_map, v_map, q_map;
    const cuuint64_t rows = static_cast<uint64_t>(a.num_physical) * a.block_size;
    const cuuint64_t row_bytes = tc2::kLatent * 2;
    const cuuint64_t k_dims[3] = {64, rows, tc2::kCb}, k_str[2] = {row_bytes, 128};
    const cuuint32_t k_box[3] = {64, tc2::kPage, tc2::kCbPerStage};
    const cuuint64_t v_dims[3] = {64, rows, 8}, v_str[2] = {row_bytes, 128};
    const cuuint32_t v_box[3] = {64, tc2::kVRows, 4};
    const cuuint64_t q_dims[3] = {64, static_cast<uint64_t>(a.batch) * tc2::kHeads, tc2::kCb};
    const cuuint32_t q_box[3] = {64, tc2::kHeadsPerCta, tc2::kCb};
    if (!tc::encode_f16_map(&k_map, a.cache, 3, k_dims, k_str, k_box) ||
        !tc::encode_f16_map(&v_map, a.cache, 3, v_dims, v_str, v_box) ||
        !tc::encode_f16_map(&q_map, ws.q16, 3, q_dims, k_str, q_box))
        return cudaErrorInvalidValue;
    const int64_t n4 = (int64_t)a.batch * tc2::kHeads * tc2::kLatent / 4;
    int blocks = (int)std::min<int64_t>((n4 + 255) / 256, 148 * 8);
    tc::q_prep_kernel<<<blocks, 256, 0, st>>>(reinterpret_cast<const float4*>(a.q_lat),
                                              reinterpret_cast<uint2*>(ws.q16),
                                              a.scale * 1.4426950408889634f, n4, ws.ctl);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(tc2::latent_partial_tc_kernel,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tc2::kSmemBytes);
    if (e != cudaSuccess) return e;
    const int workers = (a.worker_item_begin && a.n_workers > 0) ? a.n_workers : a.n_items;
    tc2::latent_partial_tc_kernel<<<2 * workers, 384, tc2::kSmemBytes, st>>>(
        k_map, v_map, q_map, a.block_size, a.block_tables, a.max_blocks, a.num_physical,
        a.seq_lens, a.items,
        (a.worker_item_begin && a.n_workers > 0) ? a.worker_item_begin : nullptr, ws,
        a.err_flags);
    return cudaGetLastError();
}

}  // namespace plkv
