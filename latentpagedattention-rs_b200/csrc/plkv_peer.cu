// plkv_peer.cu -- exchange of split-K shard results between the GPUs of one
// node through peer memory (NVLink / NVSwitch), without a collective library.
//
// Under split-K every rank decodes its range of every sequence's blocks and
// combines it into a normalised context and a log-sum-exp per (sequence,
// head) row.  The merged context is the LSE-weighted sum of the ranks' rows
// (the rule of plkv_lse_merge).  Instead of an all-gather followed by a merge
// kernel, each rank publishes its rows in a buffer of its own that every peer
// has mapped (cudaIpc), and each rank's merge kernel reads the W ranks' rows
// straight from their memory.
//
// Buffer of rank r (allocated by r, mapped by every peer):
//   [0, 256)            flags: uint64 epoch published by rank s at index s
//   [256, 264)          capacity of one slot in bytes, written at allocation
//   [512, ...)          two slots (epoch parity) of rows x (width + 1) floats,
//                       each padded to a multiple of 256 bytes: the rows'
//                       contexts, then their log-sum-exps
// Control words of rank r (local only): epoch of the last merge, and a
// counter of finished CTAs of the running kernel (the last CTA resets it, so
// the grid may differ from step to step).  A step whose rows x width does not
// fit a buffer's slots is refused on the device (PLKV_FLAG_BAD_POSITION):
// publish then writes nothing and does not advance its flag, so the peers'
// merges of that step end with PLKV_FLAG_TIMEOUT.
//
// Step e (= last epoch + 1), stream-ordered on every rank:
//   publish: copy this rank's (ctx, lse) into its own slot e & 1; the last CTA
//            to finish stores e into flag[r] of every rank's buffer
//            (system-scope release, after a system-scope fence);
//   merge:   every CTA waits until flag[s] >= e for all s (acquire, bounded:
//            after kWaitLimitNs it records PLKV_FLAG_TIMEOUT and goes on),
//            merges its rows from the W slots e & 1, and the last CTA to
//            finish records e as the last epoch.
// A slot of parity p is rewritten by its owner two steps later, at which
// point every rank has finished the merge that read it: the owner's merge of
// the step in between waited for every rank's publish of that step, which
// each rank issues only after its own previous merge.
#include <algorithm>
#include <cstring>

#include "plkv_common.cuh"
#include "plkv_sm100.cuh"

namespace plkv {
namespace {

constexpr int kFlagBytes = 512;
constexpr int kCapOffset = 256;  // uint64 slot capacity in bytes
constexpr int kMaxPeers = 32;    // one lane per rank in the merge

__device__ __forceinline__ void st_release_sys(uint64_t* p, uint64_t v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Bytes of one slot, padded to 256 so that both slots start 16-byte aligned
// (the publish copy stores float4).
__host__ __device__ __forceinline__ int64_t slot_bytes(int64_t rows, int width) {
    return (rows * (width + 1) * (int64_t)sizeof(float) + 255) / 256 * 256;
}

__device__ __forceinline__ float* slot(void* buf, int parity, int64_t rows, int width) {
    return reinterpret_cast<float*>(static_cast<uint8_t*>(buf) + kFlagBytes +
                                    parity * slot_bytes(rows, width));
}

__device__ __forceinline__ bool fits(const void* buf, int64_t rows, int width) {
    const uint64_t cap = *reinterpret_cast<const volatile uint64_t*>(
        static_cast<const uint8_t*>(buf) + kCapOffset);
    return (uint64_t)slot_bytes(rows, width) <= cap;
}

// grid-stride copy of (ctx, lse) into the own slot; the last CTA publishes.
__global__ void __launch_bounds__(256)
publish_kernel(const float* __restrict__ ctx, const float* __restrict__ lse, int64_t rows,
               int width, void* const* __restrict__ bufs, int world, int rank,
               uint64_t* __restrict__ ctrl, int32_t* flags) {
    if (!fits(bufs[rank], rows, width)) {
        if (blockIdx.x == 0 && threadIdx.x == 0) set_flag(flags, PLKV_FLAG_BAD_POSITION);
        return;
    }
    const uint64_t e = ctrl[0] + 1;
    float* dst = slot(bufs[rank], (int)(e & 1), rows, width);
    const int64_t n_ctx = rows * width;
    const int64_t n4 = n_ctx / 4;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += stride)
        reinterpret_cast<float4*>(dst)[i] = reinterpret_cast<const float4*>(ctx)[i];
    for (int64_t i = 4 * n4 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n_ctx;
         i += stride)
        dst[i] = ctx[i];
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < rows; i += stride)
        dst[n_ctx + i] = lse[i];
    // Device scope here: the last CTA observes every CTA's writes through the
    // counter below, and its system-scope release of the flags (cumulative)
    // then publishes them to the peers.
    __threadfence();
    __syncthreads();
    __shared__ bool last;
    if (threadIdx.x == 0) {
        const unsigned long long done =
            atomicAdd(reinterpret_cast<unsigned long long*>(ctrl + 1), 1ull);
        last = done + 1 == gridDim.x;
        if (last) ctrl[1] = 0;  // the next step's kernel follows in stream order
    }
    __syncthreads();
    if (last && threadIdx.x < world) {
        __threadfence_system();
        uint64_t* pflags = static_cast<uint64_t*>(bufs[threadIdx.x]);
        st_release_sys(pflags + rank, e);
    }
}

// one warp per row: waits for every rank's rows of this step, then merges
// them (lane s holds rank s's weight exp(lse_s - max)).  If a wait gives up
// (PLKV_FLAG_TIMEOUT) or a buffer is too small for the step
// (PLKV_FLAG_BAD_POSITION), no peer memory is read: the rows come out as 0
// with log-sum-exp -inf.
__global__ void __launch_bounds__(256)
merge_kernel(int64_t rows, int width, void* const* __restrict__ bufs, int world, int rank,
             uint64_t* __restrict__ ctrl, float* __restrict__ out, float* __restrict__ lse_out,
             int32_t* flags) {
    const uint64_t e = ctrl[0] + 1;
    const int parity = (int)(e & 1);
    __shared__ int ok_s;
    if (threadIdx.x < 32) {
        const bool fit = threadIdx.x >= world || fits(bufs[threadIdx.x], rows, width);
        const bool all_fit = __all_sync(0xffffffffu, fit);
        if (!all_fit && blockIdx.x == 0 && threadIdx.x == 0) set_flag(flags, PLKV_FLAG_BAD_POSITION);
        // every rank's flag polled at once (bounded)
        const bool arrived = sm100::wait_flags_warp(static_cast<const uint64_t*>(bufs[rank]),
                                                    all_fit ? world : 0, e);
        if (threadIdx.x == 0) {
            if (!arrived) set_flag(flags, PLKV_FLAG_TIMEOUT);
            ok_s = all_fit && arrived;
        }
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * 8 + warp;
    if (row < rows && !ok_s) {
        for (int c = lane; c < width; c += 32) out[row * width + c] = 0.f;
        if (lse_out && lane == 0) lse_out[row] = -INFINITY;
    } else if (row < rows) {
        const float* src_lane = lane < world ? slot(bufs[lane], parity, rows, width) : nullptr;
        const float l = src_lane ? src_lane[rows * width + row] : -INFINITY;
        float M = l;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
        const float w = (l == -INFINITY) ? 0.f : __expf(l - M);
        float den = w;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) den += __shfl_xor_sync(0xffffffffu, den, o);
        const float inv = den > 0.f ? 1.f / den : 0.f;
        // Every lane runs the same iterations (the shuffles name the whole
        // warp); only the loads and stores are guarded by the width.  The
        // sources' values of a column are all loaded before any is used, so
        // the remote reads of one row are in flight together.
        float wsrc[kMaxPeers];
#pragma unroll
        for (int s = 0; s < kMaxPeers; ++s) wsrc[s] = __shfl_sync(0xffffffffu, w, s);
        for (int c0 = 0; c0 < width; c0 += 32) {
            const int c = c0 + lane;
            float v[kMaxPeers];
#pragma unroll
            for (int s = 0; s < kMaxPeers; ++s)
                v[s] = (s < world && wsrc[s] != 0.f && c < width)
                           ? slot(bufs[s], parity, rows, width)[row * width + c]
                           : 0.f;
            float acc = 0.f;
#pragma unroll
            for (int s = 0; s < kMaxPeers; ++s) acc = fmaf(wsrc[s], v[s], acc);
            if (c < width) out[row * width + c] = acc * inv;
        }
        if (lse_out && lane == 0) lse_out[row] = den > 0.f ? M + logf(den) : -INFINITY;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned long long done =
            atomicAdd(reinterpret_cast<unsigned long long*>(ctrl + 2), 1ull);
        if (done + 1 == gridDim.x) {
            ctrl[2] = 0;
            __threadfence();
            ctrl[0] = e;
        }
    }
}

}  // namespace
}  // namespace plkv

extern "C" {

size_t plkv_peer_buffer_bytes(int64_t rows, int32_t width) {
    if (rows <= 0 || width <= 0) return 0;
    return plkv::kFlagBytes + 2 * (size_t)plkv::slot_bytes(rows, width);
}

int plkv_peer_alloc(size_t bytes, void** ptr, plkv_ipc_handle* handle) {
    if (!ptr || !handle || bytes == 0) return PLKV_ERR_INVALID_ARGUMENT;
    void* p = nullptr;
    if (cudaMalloc(&p, bytes) != cudaSuccess) return PLKV_ERR_CUDA;
    cudaIpcMemHandle_t h;
    const uint64_t cap = bytes > (size_t)plkv::kFlagBytes ? (bytes - plkv::kFlagBytes) / 2 : 0;
    if (cudaMemset(p, 0, bytes) != cudaSuccess ||
        cudaMemcpy(static_cast<uint8_t*>(p) + plkv::kCapOffset, &cap, sizeof(cap),
                   cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
        cudaFree(p);
        return PLKV_ERR_CUDA;
    }
    static_assert(sizeof(h) <= sizeof(handle->bytes), "IPC handle size");
    memcpy(handle->bytes, &h, sizeof(h));
    *ptr = p;
    return PLKV_OK;
}

int plkv_peer_open(const plkv_ipc_handle* handle, void** ptr) {
    if (!ptr || !handle) return PLKV_ERR_INVALID_ARGUMENT;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle->bytes, sizeof(h));
    return cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess
               ? PLKV_OK
               : PLKV_ERR_CUDA;
}

int plkv_peer_close(void* ptr) {
    return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? PLKV_OK : PLKV_ERR_CUDA;
}

int plkv_peer_free(void* ptr) { return cudaFree(ptr) == cudaSuccess ? PLKV_OK : PLKV_ERR_CUDA; }

int plkv_peer_init_buffer(void* buf, size_t bytes, plkv_stream_t stream) {
    if (!buf || bytes < (size_t)plkv::kFlagBytes + 512) return PLKV_ERR_INVALID_ARGUMENT;
    const uint64_t cap = (bytes - plkv::kFlagBytes) / 2;
    if (cudaMemsetAsync(buf, 0, plkv::kFlagBytes, (cudaStream_t)stream) != cudaSuccess ||
        cudaMemcpyAsync(static_cast<uint8_t*>(buf) + plkv::kCapOffset, &cap, sizeof(cap),
                        cudaMemcpyHostToDevice, (cudaStream_t)stream) != cudaSuccess ||
        cudaStreamSynchronize((cudaStream_t)stream) != cudaSuccess)
        return PLKV_ERR_CUDA;
    return PLKV_OK;
}

int plkv_peer_publish(const float* ctx, const float* lse, int64_t rows, int32_t width,
                      void* const* bufs, int32_t world, int32_t rank, uint64_t* ctrl,
                      int32_t* err_flags, plkv_stream_t stream) {
    if (rows <= 0 || width <= 0 || world <= 0) return PLKV_ERR_ZERO_VALUE;
    if (!ctx || !lse || !bufs || !ctrl || rank < 0 || rank >= world ||
        world > plkv::kMaxPeers || (reinterpret_cast<uintptr_t>(ctx) & 15))
        return PLKV_ERR_INVALID_ARGUMENT;
    const int64_t work = rows * width / 4 + rows;
    const int grid = (int)std::min<int64_t>((work + 255) / 256, 32);
    plkv::publish_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(ctx, lse, rows, width, bufs,
                                                                  world, rank, ctrl, err_flags);
    return cudaGetLastError() == cudaSuccess ? PLKV_OK : PLKV_ERR_CUDA;
}

int plkv_peer_merge(int64_t rows, int32_t width, void* const* bufs, int32_t world, int32_t rank,
                    uint64_t* ctrl, float* out, float* lse_out, int32_t* err_flags,
                    plkv_stream_t stream) {
    if (rows <= 0 || width <= 0 || world <= 0) return PLKV_ERR_ZERO_VALUE;
    if (!bufs || !ctrl || !out || rank < 0 || rank >= world || world > plkv::kMaxPeers)
        return PLKV_ERR_INVALID_ARGUMENT;
    const int grid = (int)((rows + 7) / 8);
    plkv::merge_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(rows, width, bufs, world, rank,
                                                                ctrl, out, lse_out, err_flags);
    return cudaGetLastError() == cudaSuccess ? PLKV_OK : PLKV_ERR_CUDA;
}

}  // extern "C"
