// plkv_shard.cu -- head-sharded merge of split-K results across the GPUs of
// one node, over peer memory (NVLink / NVSwitch).
//
// Under split-K every rank decodes its range of every sequence's blocks.  The
// exchange below gives rank r the merged result of the query heads it owns,
// [r * H/W, (r + 1) * H/W), and only those: each rank reads W_uv for H/W heads
// instead of all H, and the rows crossing NVLink are the heads' latent
// contexts (the projection is applied after the merge, by the owner).
//
//   publish (every rank): per (sequence b, head h), merge this rank's work
//       items with the LSE rule into a normalised latent context c[Lv] and
//       its log-sum-exp, and store them into the buffer of h's owner, at the
//       row of (source rank, b, h).  Every CTA then fences at system scope
//       (its peer stores have landed) and the last one stores the step's
//       epoch into flag[rank] of every rank's buffer.
//   merge (every rank): wait (bounded) until every rank's flag reached the
//       epoch, merge the W sources of each owned (b, h) with the LSE rule and
//       multiply by W_uv[h] (lib.rs:1066-1071), or write the latent context
//       when no projection is given.
//
// Buffer of rank r: [0, 256) uint64 flags, [256, 264) slot capacity in
// bytes, [512, ...) two slots (epoch parity), each [W][B][H/W][Lv + 1]
// floats padded to 256 bytes.  A slot is rewritten two steps later, after
// every rank's merge of the step in between waited for this rank's publish,
// which it issues only after its own previous merge.
#include <algorithm>

#include "plkv_common.cuh"
#include "plkv_sm100.cuh"

namespace plkv {
namespace {

constexpr int kFlagBytes = 512;
constexpr int kCapOffset = 256;
constexpr int kMaxRanks = 32;
constexpr int kRowsPerCta = 8;
constexpr int kMaxLvPerLane = 20;   // Lv <= 640

__host__ __device__ __forceinline__ int64_t shard_slot_bytes(int B, int H, int Lv) {
    return ((int64_t)B * H * (Lv + 1) * 4 + 255) / 256 * 256;
}

__device__ __forceinline__ float* shard_slot(void* buf, int parity, int B, int H, int Lv) {
    return reinterpret_cast<float*>(static_cast<uint8_t*>(buf) + kFlagBytes +
                                    parity * shard_slot_bytes(B, H, Lv));
}

__device__ __forceinline__ bool shard_fits(const void* buf, int B, int H, int Lv) {
    const uint64_t cap = *reinterpret_cast<const volatile uint64_t*>(
        static_cast<const uint8_t*>(buf) + kCapOffset);
    return (uint64_t)shard_slot_bytes(B, H, Lv) <= cap;
}

__device__ __forceinline__ void st_release_sys(uint64_t* p, uint64_t v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t* p) {
    uint64_t v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// grid = ceil(B * H / 8), block = 256: warp per (b, h) row, lane owns latent
// columns lane + 32 k.
__global__ void __launch_bounds__(256)
shard_publish_kernel(DecodeWorkspace ws, const int32_t* __restrict__ seq_item_begin, int B, int H,
                     int Lv, void* const* __restrict__ bufs, int world, int rank,
                     uint64_t* __restrict__ ctrl, int32_t* flags) {
    __shared__ int ok_s;
    if (threadIdx.x == 0) {
        int ok = 1;
        for (int s = 0; s < world; ++s) ok &= shard_fits(bufs[s], B, H, Lv) ? 1 : 0;
        if (!ok && blockIdx.x == 0) set_flag(flags, PLKV_FLAG_BAD_POSITION);
        ok_s = ok;
    }
    __syncthreads();
    if (!ok_s) return;
    const uint64_t e = ctrl[0] + 1;
    const int parity = (int)(e & 1);
    const int hpr = H / world;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * kRowsPerCta + warp;
    const int ncol = (Lv + 31) / 32;
    if (row < (int64_t)B * H) {
        const int b = (int)(row / H), h = (int)(row % H);
        const int ib = seq_item_begin[b], ie = seq_item_begin[b + 1];
        float M = -INFINITY;
        for (int i = ib + lane; i < ie; i += 32) M = fmaxf(M, ws.part_m[(int64_t)i * H + h]);
        M = warp_max(M);
        float acc[kMaxLvPerLane];
#pragma unroll
        for (int k = 0; k < kMaxLvPerLane; ++k) acc[k] = 0.f;
        float S = 0.f;
        if (M != -INFINITY) {
            for (int i = ib; i < ie; ++i) {
                const float mi = ws.part_m[(int64_t)i * H + h];
                if (mi == -INFINITY) continue;
                const float wi = expf(mi - M);
                S += ws.part_l[(int64_t)i * H + h] * wi;
                const float* src = ws.part_ctx + ((int64_t)i * H + h) * Lv;
#pragma unroll
                for (int k = 0; k < kMaxLvPerLane; ++k) {
                    const int col = lane + 32 * k;
                    if (k < ncol && col < Lv) acc[k] = fmaf(src[col], wi, acc[k]);
                }
            }
        }
        const float inv = (M != -INFINITY && S > 0.f) ? 1.f / S : 0.f;
        const int owner = h / hpr, hl = h % hpr;
        float* dst = shard_slot(bufs[owner], parity, B, H, Lv) +
                     (((int64_t)rank * B + b) * hpr + hl) * (Lv + 1);
#pragma unroll
        for (int k = 0; k < kMaxLvPerLane; ++k) {
            const int col = lane + 32 * k;
            if (k < ncol && col < Lv) dst[col] = acc[k] * inv;
        }
        if (lane == 0) dst[Lv] = (M == -INFINITY || S <= 0.f) ? -INFINITY : M + logf(S);
    }
    // System scope: this CTA's stores into the peers' memory have landed
    // before it is counted; the last CTA then releases the flags.
    __threadfence_system();
    __syncthreads();
    __shared__ bool last;
    if (threadIdx.x == 0) {
        const unsigned long long done =
            atomicAdd(reinterpret_cast<unsigned long long*>(ctrl + 1), 1ull);
        last = done + 1 == gridDim.x;
        if (last) ctrl[1] = 0;
    }
    __syncthreads();
    if (last && threadIdx.x < world) {
        __threadfence_system();
        st_release_sys(static_cast<uint64_t*>(bufs[threadIdx.x]) + rank, e);
    }
}

// grid = (H / W, ceil(D / 32), ceil(B / 8)), block = 256.  Phase 1: warp per
// owned (b, h) row merges the W sources (lane s holds source s's weight).
// Phase 2: thread (row, d) computes out[b, h, d] = sum_l c[l] W[h, l, d] in
// increasing l.  Without W the latent context itself is written (D = Lv).
__global__ void __launch_bounds__(256)
shard_merge_kernel(void* const* __restrict__ bufs, int world, int rank,
                   uint64_t* __restrict__ ctrl, int B, int H, int Lv,
                   const float* __restrict__ w, int D, float* __restrict__ out,
                   float* __restrict__ lse_out, int32_t* flags) {
    extern __shared__ __align__(16) float cs[];   // [8][Lv]
    const uint64_t e = ctrl[0] + 1;
    const int parity = (int)(e & 1);
    const int hpr = H / world;
    const int hl = blockIdx.x;
    const int h = rank * hpr + hl;
    const int d0 = blockIdx.y * 32;
    const int b0 = blockIdx.z * kRowsPerCta;
    __shared__ int ok_s;
    if (threadIdx.x == 0) {
        int ok = shard_fits(bufs[rank], B, H, Lv) ? 1 : 0;
        if (!ok && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0)
            set_flag(flags, PLKV_FLAG_BAD_POSITION);
        const uint64_t* f = static_cast<const uint64_t*>(bufs[rank]);
        const uint64_t t0 = sm100::globaltimer();
        for (int s = 0; s < world && ok; ++s) {
            while (ld_acquire_sys(f + s) < e) {
                if (sm100::globaltimer() - t0 > sm100::kWaitLimitNs) {
                    set_flag(flags, PLKV_FLAG_TIMEOUT);
                    ok = 0;
                    break;
                }
            }
        }
        ok_s = ok;
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int b = b0 + warp;
    if (b < B) {
        float* c = cs + warp * Lv;
        if (!ok_s) {
            for (int col = lane; col < Lv; col += 32) c[col] = 0.f;
            if (lse_out && lane == 0 && blockIdx.y == 0) lse_out[(int64_t)b * hpr + hl] = -INFINITY;
        } else {
            const float* base = shard_slot(bufs[rank], parity, B, H, Lv);
            const float l = lane < world
                                ? base[(((int64_t)lane * B + b) * hpr + hl) * (Lv + 1) + Lv]
                                : -INFINITY;
            const float M = warp_max(l);
            const float wgt = (l == -INFINITY) ? 0.f : __expf(l - M);
            const float den = warp_sum(wgt);
            const float inv = den > 0.f ? 1.f / den : 0.f;
            float wsrc[kMaxRanks];
#pragma unroll
            for (int s = 0; s < kMaxRanks; ++s) wsrc[s] = __shfl_sync(0xffffffffu, wgt, s);
            for (int col = lane; col < Lv; col += 32) {
                float acc = 0.f;
#pragma unroll
                for (int s = 0; s < kMaxRanks; ++s)
                    if (s < world && wsrc[s] != 0.f)
                        acc = fmaf(wsrc[s], base[(((int64_t)s * B + b) * hpr + hl) * (Lv + 1) + col],
                                   acc);
                c[col] = acc * inv;
            }
            if (lse_out && lane == 0 && blockIdx.y == 0)
                lse_out[(int64_t)b * hpr + hl] = den > 0.f ? M + logf(den) : -INFINITY;
        }
    }
    __syncthreads();
    const int nrows = min(kRowsPerCta, B - b0);
    const int r = threadIdx.x >> 5, d = d0 + (threadIdx.x & 31);
    if (r < nrows) {
        const int width = w ? D : Lv;
        if (d < width) {
            float v;
            if (w) {
                const float* wp = w + (int64_t)h * Lv * D + d;
                const float* c = cs + r * Lv;
                v = 0.f;
#pragma unroll 8
                for (int l = 0; l < Lv; ++l) v = fmaf(c[l], wp[(int64_t)l * D], v);
            } else {
                v = cs[r * Lv + d];
            }
            out[((int64_t)(b0 + r) * hpr + hl) * width + d] = v;
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned long long done =
            atomicAdd(reinterpret_cast<unsigned long long*>(ctrl + 2), 1ull);
        if (done + 1 == gridDim.x * gridDim.y * gridDim.z) {
            ctrl[2] = 0;
            __threadfence();
            ctrl[0] = e;
        }
    }
}

}  // namespace
}  // namespace plkv

extern "C" {

size_t plkv_shard_buffer_bytes(int32_t batch, int32_t q_heads, int32_t value_dim) {
    if (batch <= 0 || q_heads <= 0 || value_dim <= 0) return 0;
    return plkv::kFlagBytes + 2 * (size_t)plkv::shard_slot_bytes(batch, q_heads, value_dim);
}

int plkv_shard_publish(const plkv_latent_decode_args* a, void* const* bufs, int32_t world,
                       int32_t rank, uint64_t* ctrl, plkv_stream_t stream) {
    if (!a || !bufs || !ctrl) return PLKV_ERR_INVALID_ARGUMENT;
    if (a->batch <= 0 || a->q_heads <= 0 || a->latent_dim <= 0 || a->value_dim <= 0 ||
        a->n_items <= 0 || world <= 0)
        return PLKV_ERR_ZERO_VALUE;
    if (rank < 0 || rank >= world || world > plkv::kMaxRanks || a->q_heads % world ||
        !a->workspace || !a->seq_item_begin)
        return PLKV_ERR_INVALID_ARGUMENT;
    if (a->value_dim > 32 * plkv::kMaxLvPerLane) return PLKV_ERR_UNSUPPORTED;
    if (a->workspace_bytes < plkv::decode_workspace_bytes(a->n_items, a->batch, a->q_heads,
                                                          a->latent_dim, a->value_dim))
        return PLKV_ERR_WORKSPACE;
    plkv::DecodeWorkspace ws = plkv::carve_workspace(a->workspace, a->n_items, a->batch,
                                                     a->q_heads, a->latent_dim, a->value_dim);
    const int64_t rows = (int64_t)a->batch * a->q_heads;
    const int grid = (int)((rows + plkv::kRowsPerCta - 1) / plkv::kRowsPerCta);
    plkv::shard_publish_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(
        ws, a->seq_item_begin, a->batch, a->q_heads, a->value_dim, bufs, world, rank, ctrl,
        a->err_flags);
    return cudaGetLastError() == cudaSuccess ? PLKV_OK : PLKV_ERR_CUDA;
}

int plkv_shard_merge(void* const* bufs, int32_t world, int32_t rank, uint64_t* ctrl,
                     int32_t batch, int32_t q_heads, int32_t value_dim, const float* w_v,
                     int32_t head_dim, float* out, float* lse_out, int32_t* err_flags,
                     plkv_stream_t stream) {
    if (batch <= 0 || q_heads <= 0 || value_dim <= 0 || world <= 0 || (w_v && head_dim <= 0))
        return PLKV_ERR_ZERO_VALUE;
    if (!bufs || !ctrl || !out || rank < 0 || rank >= world || world > plkv::kMaxRanks ||
        q_heads % world)
        return PLKV_ERR_INVALID_ARGUMENT;
    const int width = w_v ? head_dim : value_dim;
    const size_t smem = (size_t)plkv::kRowsPerCta * value_dim * 4;
    if (smem > 48 * 1024) return PLKV_ERR_UNSUPPORTED;
    dim3 grid(q_heads / world, (width + 31) / 32, (batch + plkv::kRowsPerCta - 1) / plkv::kRowsPerCta);
    plkv::shard_merge_kernel<<<grid, 256, smem, (cudaStream_t)stream>>>(
        bufs, world, rank, ctrl, batch, q_heads, value_dim, w_v, head_dim, out, lse_out,
        err_flags);
    return cudaGetLastError() == cudaSuccess ? PLKV_OK : PLKV_ERR_CUDA;
}

}  // extern "C"
