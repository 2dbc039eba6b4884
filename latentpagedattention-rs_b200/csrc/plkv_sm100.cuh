// plkv_sm100.cuh -- thin inline-PTX wrappers for sm_100a: mbarriers with
// bounded waits, cluster addressing, TMA tile loads, tcgen05 (TMEM
// allocation, MMA, commit, loads/stores, fences) and UMMA descriptors.
#pragma once

#include <cuda.h>
#include <stdint.h>

#include "plkv_common.cuh"

namespace plkv {
namespace sm100 {

constexpr uint64_t kWaitLimitNs = 1000000000ull;  // 1 s per wait, then give up
constexpr uint64_t kFlagPollNs = 20000ull;        // global flag word read every 20 us of waiting

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

__device__ __forceinline__ uint32_t cluster_id_x() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
    return r;
}

__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;"
                 ::: "memory");
}

// Address of the same shared-memory offset in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}

// ----------------------------------------------------------------- mbarrier

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;"
                 ::"r"(bar), "r"(bytes) : "memory");
}

// Arrive on a barrier given by its shared::cluster address (any CTA).
//
// The release is CTA-scoped.  A cluster-scoped release is a fence that waits
// for every earlier memory operation of the thread to reach cluster-wide
// visibility (about 1 us per arrive), and the data these arrives publish needs
// none of it: it is this CTA's own shared memory (P tiles) or tensor memory
// (the O accumulator that was read), complete once the writers passed a
// fence.proxy.async / tcgen05.fence and a CTA barrier, and read afterwards
// only by tensor-core operations that the peer issues after observing the
// barrier phase.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cluster.b64 _, [%0];"
                 ::"r"(cluster_bar) : "memory");
}

// Plain arrive (no transaction bytes) on a barrier of this CTA.
__device__ __forceinline__ void mbar_arrive_local(uint32_t bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Non-blocking probe of the same phase: unlike try_wait, test_wait never
// suspends the thread, so a scheduler polling several barriers in turn does
// not sleep on one while another is already complete.
__device__ __forceinline__ bool mbar_test_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Where a bounded wait reports and learns of failures.  `report` is the
// caller's error word (may be NULL): a wait that gives up ORs
// PLKV_FLAG_TIMEOUT into it.  `abort` is a control word of this launch in
// global memory, zeroed by the launch's first kernel: a wait that gives up
// sets it, and every other waiting CTA of the launch (the peer of a CTA pair
// included) sees it and gives up too.  The caller's word is never read, so an
// old error bit left in it does not end later launches.  `local` is this
// CTA's own flag in shared memory.
struct WaitCtx {
    int32_t* report;
    volatile int32_t* abort;
    volatile int* local;
};

__device__ __forceinline__ void wait_give_up(const WaitCtx& w) {
    set_flag(w.report, PLKV_FLAG_TIMEOUT);
    *w.abort = 1;
    __threadfence();
    *w.local = 1;
}

// Waits for the phase with the given parity to complete.  Gives up after
// kWaitLimitNs (or soon after another wait of this launch gave up) and
// returns false; the caller then abandons its work.  The launch's abort word
// is an L2 round trip, so it is read only every kFlagPollNs of waiting:
// reading it between every two polls would stretch each poll to that round
// trip and delay the waiter by as much.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, const WaitCtx& w) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    uint64_t next_check = t0 + kFlagPollNs;
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*w.local) return false;
        const uint64_t now = globaltimer();
        if (now < next_check) continue;
        next_check = now + kFlagPollNs;
        if (*w.abort) {
            *w.local = 1;
            return false;
        }
        if (now - t0 > kWaitLimitNs) {
            wait_give_up(w);
            return false;
        }
    }
}

// -------------------------------------------------------------------- TMA

// 2-D tile load into this CTA's shared memory; completion is signalled on
// `cluster_bar` (a shared::cluster address, possibly in the peer CTA of the
// pair).  No multicast.
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, int x, int y,
                                                 uint32_t cluster_bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        ".L2::cache_hint [%0], [%1, {%2, %3}], [%4], %5;"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(cluster_bar),
          "l"(policy)
        : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_normal() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
    return p;
}

__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// Bulk prefetch of a contiguous global range into L2 (16-byte aligned, size a
// multiple of 16); no shared memory is used.
__device__ __forceinline__ void prefetch_l2(const void* ptr, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;"
                 ::"l"(reinterpret_cast<uint64_t>(ptr)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Called by a whole warp: lane s < n waits until flags[s] >= e (system-scope
// acquire loads, so the writes released before each flag are visible to the
// warp and, after a CTA barrier, to the CTA).  All flags are polled together;
// the wait gives up after kWaitLimitNs.  Returns (warp-uniformly) whether
// every flag arrived.
__device__ __forceinline__ bool wait_flags_warp(const uint64_t* flags, int n, uint64_t e) {
    const int lane = threadIdx.x & 31;
    bool done = lane >= n, gave_up = false;
    const uint64_t t0 = globaltimer();
    while (!__all_sync(0xffffffffu, done || gave_up)) {
        if (!done && !gave_up) {
            uint64_t v;
            asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(flags + lane) : "memory");
            done = v >= e;
            if (!done && globaltimer() - t0 > kWaitLimitNs) gave_up = true;
        }
    }
    return !__any_sync(0xffffffffu, gave_up);
}

// ---------------------------------------------------------------- tcgen05

__device__ __forceinline__ void tmem_alloc_pair(uint32_t dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(dst_smem), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;"
                 ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem], FP16 inputs, FP32 accumulation, issued for
// the CTA pair by one thread of the leader CTA.
__device__ __forceinline__ void mma_pair_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                             uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive (once) on the barrier at the same offset in every CTA of `mask`
// when all previously issued tcgen05 operations of this thread complete.
__device__ __forceinline__ void mma_commit_pair(uint32_t bar, uint16_t mask) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
        " [%0], %1;" ::"r"(bar), "h"(mask) : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_wait_st() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp gets lane
// (warp's quarter * 32 + i), columns [col, col + 32).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
          "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
          "=r"(r[31])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float* v) {
    uint32_t r[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(v[i]);
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
        ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]),
          "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]),
          "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]),
          "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]),
          "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}

// ------------------------------------------------------------ descriptors

// Shared-memory matrix descriptor, 128-byte swizzle (layout type 2),
// version 1; lbo / sbo in bytes.
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4) |
           (static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16) |
           (static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}

// Instruction descriptor of kind::f16 with FP16 A and B, FP32 D.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N, bool a_mn_major, bool b_mn_major) {
    return (1u << 4) | (static_cast<uint32_t>(a_mn_major) << 15) |
           (static_cast<uint32_t>(b_mn_major) << 16) | (static_cast<uint32_t>(N >> 3) << 17) |
           (static_cast<uint32_t>(M >> 4) << 24);
}

// Byte offset of element (row, col) inside a 128-byte-swizzled tile of
// 16-bit elements with 64 columns per 128-byte row (8-row, 1024-byte atoms).
__device__ __forceinline__ uint32_t sw128_offset(uint32_t row, uint32_t col) {
    return (row >> 3) * 1024u + (row & 7u) * 128u + ((((col >> 3) ^ (row & 7u)) & 7u) << 4) +
           (col & 7u) * 2u;
}

}  // namespace sm100
}  // namespace plkv
