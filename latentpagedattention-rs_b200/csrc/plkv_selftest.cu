// plkv_selftest.cu -- exercises the bounded-wait machinery that the
// tensor-core decode relies on (plkv_sm100.cuh: mbar_wait, WaitCtx), on a
// barrier that nothing ever completes.  No GPU fault is involved: every wait
// gives up on its own time limit and the kernel returns normally.
//
// Two CTAs of one launch, one waiting thread each, both on a barrier of their
// own shared memory with no arrival.  CTA 0 starts waiting at once and gives
// up after kWaitLimitNs: it ORs PLKV_FLAG_TIMEOUT into the caller's word and
// sets the launch's abort word.  CTA 1 starts waiting kLateStartNs later; it
// would give up on its own limit at kLateStartNs + kWaitLimitNs, but learns of
// CTA 0's failure through the abort word (read every kFlagPollNs) and ends
// about kWaitLimitNs - kLateStartNs after it began.  With the abort word
// already set by the caller, both waits end after the first poll interval and
// nothing is reported (a wait that learns of another's failure does not report
// one of its own).
#include "plkv_sm100.cuh"

namespace plkv {
namespace {

constexpr uint64_t kLateStartNs = 500000000ull;

__global__ void __launch_bounds__(32, 1)
bounded_wait_selftest_kernel(int32_t* ctl, int64_t* elapsed_ns, int32_t* flags) {
    using namespace sm100;
    __shared__ __align__(8) uint64_t bar;
    __shared__ int local;
    if (threadIdx.x != 0) return;
    const uint32_t b = smem_u32(&bar);
    mbar_init(b, 1);
    local = 0;
    fence_mbar_init();
    if (blockIdx.x == 1) {
        const uint64_t t = globaltimer();
        while (globaltimer() - t < kLateStartNs) {
        }
    }
    const WaitCtx wc{flags, ctl, &local};
    const uint64_t t0 = globaltimer();
    const bool ok = mbar_wait(b, 0, wc);
    elapsed_ns[blockIdx.x] = ok ? -1 : (int64_t)(globaltimer() - t0);
}

}  // namespace
}  // namespace plkv

extern "C" int plkv_selftest_bounded_wait(int32_t* ctl, int64_t* elapsed_ns, int32_t* err_flags,
                                          plkv_stream_t stream) {
    if (!ctl || !elapsed_ns) return PLKV_ERR_INVALID_ARGUMENT;
    plkv::bounded_wait_selftest_kernel<<<2, 32, 0, (cudaStream_t)stream>>>(ctl, elapsed_ns,
                                                                          err_flags);
    return cudaGetLastError() == cudaSuccess ? PLKV_OK : PLKV_ERR_CUDA;
}
