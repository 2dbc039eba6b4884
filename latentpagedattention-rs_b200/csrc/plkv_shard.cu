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
//       its log-sum-exp, and store them into this rank's own slot at row
//       (b, h).  Every CTA fences at device scope before it is counted; the
//       last one then stores the step's epoch into flag[rank] of every
//       rank's buffer with a system-scope release, which (cumulatively)
//       publishes every CTA's rows.
//   merge (every rank): wait (bounded) until every rank's flag reached the
//       epoch, read the rows of the owned heads from every rank's slot over
//       NVLink, merge the W sources of each owned (b, h) with the LSE rule
//       and multiply by W_uv[h] (lib.rs:1066-1071), or write the latent
//       context when no projection is given.
// The rows thus cross NVLink once, as loads of their owner; no store reaches
// another GPU's memory except the flags.
//
// Buffer of rank r: [0, 256) uint64 flags, [256, 264) slot capacity in
// bytes, [512, ...) two slots (epoch parity), each [B][H] rows of
// slot_row(Lv) floats (Lv context floats, the lse at Lv; rows a multiple of
// 4 floats, 16-byte aligned) padded to 256 bytes, then [B][H][Lv] floats of
// local scratch (the merged rows of the owned heads before the projection;
// only the owner touches it).  A slot is rewritten two steps later, after
// every rank's merge of the step in between (which reads it) waited for this
// rank's publish of that step, which it issues only after its own previous
// merge.
#include <algorithm>

#include "plkv_common.cuh"
#include "plkv_sm100.cuh"

namespace plkv {
namespace {

constexpr int kFlagBytes = 512;
constexpr int kCapOffset = 256;
constexpr int kMaxRanks = 32;

__host__ __device__ __forceinline__ int slot_row(int Lv) { return (Lv + 1 + 3) & ~3; }

__host__ __device__ __forceinline__ int64_t shard_slot_bytes(int B, int H, int Lv) {
    return ((int64_t)B * H * slot_row(Lv) * 4 + 255) / 256 * 256;
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

// grid = ceil(B * H / (256 / TPR)), block = 256: the TPR / 32 warps of row
// x * (256 / TPR) + t / TPR merge the row's items (merge_row_warp), thread c =
// t % TPR for columns [Vc, Vc + V), ... (V = 8 with 64 threads per row when
// Lv % 8 == 0, V = 4 with 128 when Lv % 4 == 0, else V = 1 with 128), and
// store them, normalised, into this rank's slot; thread 0 of the row stores
// the lse.  Registers capped so that the grid is resident at once (V = 8:
// half the CTAs of V = 4, two per SM).
template <int V, int TPR>
__global__ void __launch_bounds__(256, V >= 8 ? 2 : 4)
shard_publish_kernel(DecodeWorkspace ws, const int32_t* __restrict__ seq_item_begin, int B, int H,
                     int Lv, void* const* __restrict__ bufs, int world, int rank,
                     uint64_t* __restrict__ ctrl, int32_t* flags) {
    __shared__ int ok_s;
    if (threadIdx.x < 32) {  // lane s checks rank s's buffer
        const bool fit = threadIdx.x >= world || shard_fits(bufs[threadIdx.x], B, H, Lv);
        const bool ok = __all_sync(0xffffffffu, fit);
        if (threadIdx.x == 0) {
            if (!ok && blockIdx.x == 0) set_flag(flags, PLKV_FLAG_BAD_POSITION);
            ok_s = ok;
        }
    }
    __syncthreads();
    if (!ok_s) return;
    const uint64_t e = ctrl[0] + 1;
    const int parity = (int)(e & 1);
    const int64_t row = (int64_t)blockIdx.x * (256 / TPR) + threadIdx.x / TPR;
    const int c = threadIdx.x % TPR, lane = threadIdx.x & 31;
    if (row < (int64_t)B * H) {   // whole warps: a row is TPR / 32 warps
        const int b = (int)(row / H), h = (int)(row % H);
        const int ib = seq_item_begin[b], ie = seq_item_begin[b + 1];
        float M = -INFINITY, S = 0.f;
        float* dst = shard_slot(bufs[rank], parity, B, H, Lv) + row * slot_row(Lv);
        for (int base = 0; base < Lv; base += V * TPR) {   // the same passes in every lane
            const int col = base + V * c;
            float acc[V];
            merge_row_warp<V>(ws, ib, ie, H, h, Lv, col, lane, acc, M, S);
            const float inv = (M != -INFINITY && S > 0.f) ? 1.f / S : 0.f;
            if (V % 4 == 0) {  // slot rows are 16-byte aligned
                if (col < Lv) {
#pragma unroll
                    for (int k4 = 0; k4 < V / 4; ++k4)
                        reinterpret_cast<float4*>(dst + col)[k4] =
                            make_float4(acc[4 * k4] * inv, acc[4 * k4 + 1] * inv,
                                        acc[4 * k4 + 2] * inv, acc[4 * k4 + 3] * inv);
                }
            } else if (col < Lv) {
                dst[col] = acc[0] * inv;
            }
        }
        if (c == 0) dst[Lv] = (M == -INFINITY || S <= 0.f) ? -INFINITY : M + logf(S);
    }
    // The CTA's rows are ordered before its count (the barrier, then one
    // cumulative device-scope fence by the counting thread); the last CTA's
    // system-scope release of the flags then publishes every CTA's rows.
    __syncthreads();
    __shared__ bool last;
    if (threadIdx.x == 0) {
        __threadfence();
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

// grid = ceil(B * H/W / 2), block = 256: thread (owned row (b, hl) = 2 x + t /
// 128, column group c) waits (bounded; warp 0 polls every rank's flag at
// once) until every rank's flag reached the epoch, reads its columns of the
// row from the W ranks' slots (peer loads, all sources' in flight together),
// merges them with the LSE rule (source s weighted exp(lse_s - max_s lse_s))
// and writes the row to
// `dst` ([B][H/W][Lv]: the output when there is no projection, else the
// scratch rows of this rank's buffer, dst_offset bytes into dst_table[rank]);
// column group 0 writes the lse.  The last CTA
// advances the epoch.
__global__ void __launch_bounds__(256)
shard_merge_rows_kernel(void* const* __restrict__ bufs, int world, int rank,
                        uint64_t* __restrict__ ctrl, int B, int H, int Lv,
                        float* __restrict__ dst, float* __restrict__ lse_out, int32_t* flags,
                        void* const* __restrict__ dst_table, size_t dst_offset) {
    if (dst_table)
        dst = reinterpret_cast<float*>(static_cast<char*>(dst_table[rank]) + dst_offset);
    const uint64_t e = ctrl[0] + 1;
    const int parity = (int)(e & 1);
    const int hpr = H / world;
    __shared__ int ok_s;
    if (threadIdx.x < 32) {
        const bool fits = shard_fits(bufs[rank], B, H, Lv);
        if (!fits && blockIdx.x == 0 && threadIdx.x == 0) set_flag(flags, PLKV_FLAG_BAD_POSITION);
        const bool arrived =
            sm100::wait_flags_warp(static_cast<const uint64_t*>(bufs[rank]), fits ? world : 0, e);
        if (threadIdx.x == 0) {
            if (!arrived) set_flag(flags, PLKV_FLAG_TIMEOUT);
            ok_s = fits && arrived;
        }
    }
    __syncthreads();
    const int64_t row = (int64_t)blockIdx.x * 2 + (threadIdx.x >> 7);
    const int c = threadIdx.x & 127;
    if (row < (int64_t)B * hpr) {
        const int b = (int)(row / hpr), hl = (int)(row % hpr);
        float* o = dst + row * Lv;
        if (!ok_s) {
            for (int col = c; col < Lv; col += 128) o[col] = 0.f;
            if (lse_out && c == 0) lse_out[row] = -INFINITY;
        } else {
            // lane s holds source s's lse and weight (world <= 32); the four
            // columns of a thread and up to 8 sources are loaded together
            const int lane = threadIdx.x & 31;
            // row (b, h) of source s: slot of rank s (peer memory)
            const int64_t roff = ((int64_t)b * H + (int64_t)rank * hpr + hl) * slot_row(Lv);
            const float* src_lane =
                lane < world ? shard_slot(bufs[lane], parity, B, H, Lv) + roff : nullptr;
            const float ls = src_lane ? src_lane[Lv] : -INFINITY;
            const float M = warp_max(ls);
            const float ws = (ls == -INFINITY) ? 0.f : __expf(ls - M);
            const float den = warp_sum(ws);
            const float inv = den > 0.f ? 1.f / den : 0.f;
            for (int c0 = 0; c0 < Lv; c0 += 4 * 128) {   // the same passes in every lane
                float acc[4] = {0.f, 0.f, 0.f, 0.f};
                for (int s0 = 0; s0 < world; s0 += 8) {
                    float v[8][4];
#pragma unroll
                    for (int q = 0; q < 8; ++q) {
                        const float* sp = reinterpret_cast<const float*>(__shfl_sync(
                            0xffffffffu, reinterpret_cast<uintptr_t>(src_lane), (s0 + q) & 31));
#pragma unroll
                        for (int k = 0; k < 4; ++k) {
                            const int col = c0 + c + 128 * k;
                            v[q][k] = (s0 + q < world && col < Lv) ? sp[col] : 0.f;
                        }
                    }
#pragma unroll
                    for (int q = 0; q < 8; ++q) {
                        const float wq = __shfl_sync(0xffffffffu, ws, (s0 + q) & 31);
                        if (s0 + q >= world || wq == 0.f) continue;
#pragma unroll
                        for (int k = 0; k < 4; ++k) acc[k] = fmaf(wq, v[q][k], acc[k]);
                    }
                }
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const int col = c0 + c + 128 * k;
                    if (col < Lv) o[col] = acc[k] * inv;
                }
            }
            if (lse_out && c == 0) lse_out[row] = den > 0.f ? M + logf(den) : -INFINITY;
        }
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

size_t plkv_shard_buffer_bytes(int32_t batch, int32_t q_heads, int32_t value_dim) {
    if (batch <= 0 || q_heads <= 0 || value_dim <= 0) return 0;
    return plkv::kFlagBytes + 2 * (size_t)plkv::shard_slot_bytes(batch, q_heads, value_dim) +
           plkv::align256((size_t)batch * q_heads * value_dim * 4);
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
    if (a->workspace_bytes < plkv::decode_workspace_bytes(a->n_items, a->batch, a->q_heads,
                                                          a->latent_dim, a->value_dim))
        return PLKV_ERR_WORKSPACE;
    plkv::DecodeWorkspace ws = plkv::carve_workspace(a->workspace, a->n_items, a->batch,
                                                     a->q_heads, a->latent_dim, a->value_dim);
    const int64_t rows = (int64_t)a->batch * a->q_heads;
    if ((a->value_dim & 7) == 0)
        plkv::shard_publish_kernel<8, 64><<<(unsigned)((rows + 3) / 4), 256, 0,
                                            (cudaStream_t)stream>>>(
            ws, a->seq_item_begin, a->batch, a->q_heads, a->value_dim, bufs, world, rank, ctrl,
            a->err_flags);
    else if ((a->value_dim & 3) == 0)
        plkv::shard_publish_kernel<4, 128><<<(unsigned)((rows + 1) / 2), 256, 0,
                                             (cudaStream_t)stream>>>(
            ws, a->seq_item_begin, a->batch, a->q_heads, a->value_dim, bufs, world, rank, ctrl,
            a->err_flags);
    else
        plkv::shard_publish_kernel<1, 128><<<(unsigned)((rows + 1) / 2), 256, 0,
                                             (cudaStream_t)stream>>>(
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
    const int hpr = q_heads / world;
    const unsigned grid = (unsigned)(((int64_t)batch * hpr + 1) / 2);
    // Without a projection the merged rows are the output; with one they go
    // to this rank's scratch rows (after the two slots of its buffer) and
    // the projection of the owned heads' W_uv follows.
    const size_t scratch_off =
        plkv::kFlagBytes + 2 * (size_t)plkv::shard_slot_bytes(batch, q_heads, value_dim);
    if (!w_v) {
        plkv::shard_merge_rows_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(
            bufs, world, rank, ctrl, batch, q_heads, value_dim, out, lse_out, err_flags, nullptr, 0);
        return cudaGetLastError() == cudaSuccess ? PLKV_OK : PLKV_ERR_CUDA;
    }
    plkv::shard_merge_rows_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(
        bufs, world, rank, ctrl, batch, q_heads, value_dim, nullptr, lse_out, err_flags, bufs,
        scratch_off);
    if (cudaGetLastError() != cudaSuccess) return PLKV_ERR_CUDA;
    const cudaError_t e = plkv::launch_project_rows(
        nullptr, bufs, rank, scratch_off, batch, hpr, value_dim,
        w_v + (size_t)rank * hpr * value_dim * head_dim, hpr, head_dim, out, (cudaStream_t)stream);
    return e == cudaSuccess ? PLKV_OK : PLKV_ERR_CUDA;
}

}  // extern "C"
