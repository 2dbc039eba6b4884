// plkv_decode_exact.cu -- FP32 CUDA-core ("exact" mode) decode kernels.
//
// Split-K partial pass of the direct paged latent decode (scores against the
// projected query, active-length mask, online softmax, latent context) and of
// the FP16 full-KV paged GQA baseline, plus the query projection.
//
// Arithmetic follows crates/plkv-core/src/lib.rs:1023-1071 (latent) and
// lib.rs:1222-1263 (full KV): scores are an FP32 dot product over the latent
// row in increasing column order, multiplied by `scale`; softmax uses expf of
// (score - running max); contexts accumulate p * row in FP32.  The online
// softmax keeps (max, sum, context) per work item; the combine pass merges
// items exactly as the reference's single pass would up to FP32 rounding.
#include "plkv_common.cuh"

namespace plkv {

// ---------------------------------------------------------------- latent

// grid = (ceil(q_heads / 32), n_items), block = 256 threads (8 warps); the
// head groups of one work item are adjacent in launch order so that they read
// the item's latent rows from L2 rather than each from HBM.
// Warp w owns heads 4w..4w+3 of the CTA's 32-head group in both phases:
//   scores : lane = token of the 32-token tile, 4 dot products per thread;
//   context: lane owns value columns 4*lane + 128*c (c < NCH), 4 heads.
// Shared memory: q tile [32][L+4], row tile [32][L+4] (FP32, converted once
// from FP16 when staged), probabilities [32 tokens][32 heads].
template <int NCH>
__global__ void __launch_bounds__(256, 1)
latent_partial_exact_kernel(const float* __restrict__ q_lat, const uint16_t* __restrict__ cache,
                            int64_t num_physical, int bs, int L, int Lv, int Hq, float scale,
                            const int32_t* __restrict__ tables, int64_t max_blocks,
                            const int32_t* __restrict__ seq_lens,
                            const plkv_work_item* __restrict__ items, DecodeWorkspace ws,
                            float* __restrict__ scores, int max_seq_len, int32_t* flags) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int LP = L + 4;
    float* qs = reinterpret_cast<float*>(smem_raw);
    float* lt = qs + kHeadGroup * LP;
    float* ps = lt + kTileTokens * LP;
    __shared__ const uint16_t* row_ptr[kTileTokens];

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const plkv_work_item it = items[blockIdx.y];
    const int b = it.seq;
    const int h0 = blockIdx.x * kHeadGroup;
    const int nh = min(kHeadGroup, Hq - h0);
    int len = seq_lens[b];
    const int64_t cap = max_blocks * (int64_t)bs;
    if (len < 0 || len > cap) {
        if (tid == 0 && blockIdx.x == 0) set_flag(flags, PLKV_FLAG_BAD_LENGTH);
        len = len < 0 ? 0 : (int)cap;
    }
    const int t_begin = it.block_begin * bs;
    const int t_end = min(it.block_end * bs, len);

    for (int i = tid; i < kHeadGroup * L; i += 256) {
        int h = i / L, k = i - h * L;
        qs[h * LP + k] = (h < nh) ? q_lat[((int64_t)b * Hq + h0 + h) * L + k] : 0.f;
    }

    float m_run[4], l_run[4], acc[4][NCH][4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        m_run[j] = -INFINITY;
        l_run[j] = 0.f;
#pragma unroll
        for (int c = 0; c < NCH; ++c)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[j][c][e] = 0.f;
    }

    const int cpr = L >> 3;  // 16-byte chunks per row
    for (int t0 = t_begin; t0 < t_end; t0 += kTileTokens) {
        const int nt = min(kTileTokens, t_end - t0);
        __syncthreads();  // previous tile consumed; q tile visible on the first pass
        if (tid < kTileTokens) {
            const uint16_t* rp = nullptr;
            if (tid < nt) {
                int t = t0 + tid;
                int lb = t / bs;
                int32_t phys = tables[(int64_t)b * max_blocks + lb];
                if (phys >= 0 && phys < num_physical)
                    rp = cache + ((int64_t)phys * bs + (t - lb * bs)) * (int64_t)L;
                else
                    set_flag(flags, PLKV_FLAG_BAD_BLOCK);
            }
            row_ptr[tid] = rp;
        }
        __syncthreads();
        for (int i = tid; i < kTileTokens * cpr; i += 256) {
            int r = i / cpr, c = i - r * cpr;
            float v[8];
            const uint16_t* rp = row_ptr[r];
            if (rp) {
                uint4 raw = __ldg(reinterpret_cast<const uint4*>(rp) + c);
                unpack8(raw, v);
            } else {
#pragma unroll
                for (int e = 0; e < 8; ++e) v[e] = 0.f;
            }
            float4* dst = reinterpret_cast<float4*>(lt + r * LP + c * 8);
            dst[0] = make_float4(v[0], v[1], v[2], v[3]);
            dst[1] = make_float4(v[4], v[5], v[6], v[7]);
        }
        __syncthreads();

        // Scores: sequential FMA over the latent columns (lib.rs:1033-1041).
        float s[4] = {0.f, 0.f, 0.f, 0.f};
        const float* xr = lt + lane * LP;
        const float* qw = qs + (4 * warp) * LP;
#pragma unroll 4
        for (int k = 0; k < L; k += 4) {
            float4 x = *reinterpret_cast<const float4*>(xr + k);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                float4 qv = *reinterpret_cast<const float4*>(qw + j * LP + k);
                s[j] = fmaf(x.x, qv.x, s[j]);
                s[j] = fmaf(x.y, qv.y, s[j]);
                s[j] = fmaf(x.z, qv.z, s[j]);
                s[j] = fmaf(x.w, qv.w, s[j]);
            }
        }
        const bool tok_ok = lane < nt && row_ptr[lane] != nullptr;
        float alpha[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int h = 4 * warp + j;
            const float sc = s[j] * scale;
            if (scores && lane < nt && h < nh && t0 + lane < max_seq_len)
                scores[((int64_t)b * Hq + h0 + h) * max_seq_len + t0 + lane] = sc;
            const float sv = tok_ok ? sc : -INFINITY;
            const float m_new = fmaxf(m_run[j], warp_max(sv));
            alpha[j] = (m_new == -INFINITY) ? 1.f : expf(m_run[j] - m_new);
            const float p = tok_ok ? expf(sv - m_new) : 0.f;
            l_run[j] = l_run[j] * alpha[j] + warp_sum(p);
            m_run[j] = m_new;
            ps[lane * kHeadGroup + 4 * warp + j] = p;
        }
        __syncwarp();

        // Context: acc = acc * alpha + sum_r p[r] * row[r] (lib.rs:1057-1065).
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int c = 0; c < NCH; ++c)
#pragma unroll
                for (int e = 0; e < 4; ++e) acc[j][c][e] *= alpha[j];
        for (int r = 0; r < nt; ++r) {
            const float4 pv = *reinterpret_cast<const float4*>(ps + r * kHeadGroup + 4 * warp);
            const float* xr2 = lt + r * LP + lane * 4;
#pragma unroll
            for (int c = 0; c < NCH; ++c) {
                if (lane * 4 + 128 * c < Lv) {
                    const float4 x = *reinterpret_cast<const float4*>(xr2 + 128 * c);
                    const float pj[4] = {pv.x, pv.y, pv.z, pv.w};
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        acc[j][c][0] = fmaf(pj[j], x.x, acc[j][c][0]);
                        acc[j][c][1] = fmaf(pj[j], x.y, acc[j][c][1]);
                        acc[j][c][2] = fmaf(pj[j], x.z, acc[j][c][2]);
                        acc[j][c][3] = fmaf(pj[j], x.w, acc[j][c][3]);
                    }
                }
            }
        }
    }

    const int64_t ib = blockIdx.y;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int h = 4 * warp + j;
        if (h >= nh) continue;
        const int64_t row = ib * Hq + h0 + h;
        if (lane == 0) {
            ws.part_m[row] = m_run[j];
            ws.part_l[row] = l_run[j];
        }
        float* dst = ws.part_ctx + row * Lv;
#pragma unroll
        for (int c = 0; c < NCH; ++c) {
            const int col = lane * 4 + 128 * c;
            if (col < Lv)
                *reinterpret_cast<float4*>(dst + col) =
                    make_float4(acc[j][c][0], acc[j][c][1], acc[j][c][2], acc[j][c][3]);
        }
    }
}

size_t latent_exact_smem_bytes(int L) {
    return size_t(kHeadGroup + kTileTokens) * (L + 4) * 4 + size_t(kTileTokens) * kHeadGroup * 4;
}

template <int NCH>
static cudaError_t launch_latent_exact_t(const plkv_latent_decode_args& a, DecodeWorkspace ws,
                                         cudaStream_t st) {
    const size_t smem = latent_exact_smem_bytes(a.latent_dim);
    cudaError_t e = cudaFuncSetAttribute(latent_partial_exact_kernel<NCH>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    dim3 grid((a.q_heads + kHeadGroup - 1) / kHeadGroup, a.n_items);
    latent_partial_exact_kernel<NCH><<<grid, 256, smem, st>>>(
        a.q_lat, a.cache, a.num_physical, a.block_size, a.latent_dim, a.value_dim, a.q_heads,
        a.scale, a.block_tables, a.max_blocks, a.seq_lens, a.items, ws, a.scores, a.max_seq_len,
        a.err_flags);
    return cudaGetLastError();
}

cudaError_t launch_latent_partial_exact(const plkv_latent_decode_args& a, DecodeWorkspace ws,
                                        cudaStream_t st) {
    const int nch = (a.value_dim + 127) / 128;
    switch (nch) {
        case 1: return launch_latent_exact_t<1>(a, ws, st);
        case 2: return launch_latent_exact_t<2>(a, ws, st);
        case 3: return launch_latent_exact_t<3>(a, ws, st);
        case 4: return launch_latent_exact_t<4>(a, ws, st);
        case 5: return launch_latent_exact_t<5>(a, ws, st);
        default: return cudaErrorInvalidValue;
    }
}

// --------------------------------------------------------------- full KV

constexpr int kKvStages = 5;    // 32-token K/V tiles in flight per CTA
constexpr int kKvPad = 8;       // FP16 padding per staged row (16 bytes)

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;"
                 ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst))),
                   "l"(gmem_src)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
    asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// grid = (n_items, kv_heads), block = 256, two CTAs per SM.  The item's K and
// V rows of KV head g stream through a ring of kKvStages 32-token tiles:
// every thread issues 16-byte asynchronous copies (cp.async) of its share of
// a tile's rows, kKvStages - 1 tiles ahead of the one being computed, so the
// HBM latency is covered by the tiles in flight instead of being paid per
// tile.  Rows land as FP16 with a 16-byte pad (a 272-byte row stride for
// D = 128), so that 32 lanes reading 16-byte chunks of 32 different rows, or
// of one row, hit distinct banks; they are converted to FP32 as they are read.
// Warp w < G owns query head kv*G + w: lane = token for the scores (FP32 sum
// over d in increasing order, lib.rs:1222-1230), warp-shuffle max / sum for
// the online softmax, then lane = 4 value columns (+128 c) for the context.
template <int NCH>
__global__ void __launch_bounds__(256, 2)
fullkv_partial_exact_kernel(const float* __restrict__ q, const uint16_t* __restrict__ k_cache,
                            const uint16_t* __restrict__ v_cache, int64_t num_physical, int KV,
                            int bs, int D, int Hq, float scale, const int32_t* __restrict__ tables,
                            int64_t max_blocks, const int32_t* __restrict__ seq_lens,
                            const plkv_work_item* __restrict__ items, DecodeWorkspace ws,
                            float* __restrict__ scores, int max_seq_len, int32_t* flags) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int DP = D + 4;                 // FP32 query row
    const int RS = D + kKvPad;            // FP16 staged row
    const int G = Hq / KV;
    float* qs = reinterpret_cast<float*>(smem_raw);                   // [8][DP]
    float* ps = qs + 8 * DP;                                          // [32][8]
    uint16_t* ring = reinterpret_cast<uint16_t*>(ps + kTileTokens * 8);  // [stages][2][32][RS]
    __shared__ int64_t row_off[kKvStages][kTileTokens];
    __shared__ int32_t ptab[kKvStages][kTileTokens];

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const plkv_work_item it = items[blockIdx.x];
    const int b = it.seq, g = blockIdx.y;
    int len = seq_lens[b];
    const int64_t cap = max_blocks * (int64_t)bs;
    if (len < 0 || len > cap) {
        if (tid == 0 && g == 0) set_flag(flags, PLKV_FLAG_BAD_LENGTH);
        len = len < 0 ? 0 : (int)cap;
    }
    const int t_begin = it.block_begin * bs;
    const int t_end = max(t_begin, min(it.block_end * bs, len));
    const int n_tiles = (t_end - t_begin + kTileTokens - 1) / kTileTokens;
    const bool active = warp < G;
    const int h = g * G + warp;
    const int cpr = D >> 3;               // 16-byte chunks per row

    for (int i = tid; i < 8 * D; i += 256) {
        int w = i / D, d = i - w * D;
        qs[w * DP + d] = (w < G) ? q[((int64_t)b * Hq + g * G + w) * D + d] : 0.f;
    }

    // Physical block of every token of tile j (-1: past the item or a table
    // entry outside the pool), kept in shared memory kKvStages tiles ahead
    // so that issuing a tile's copies never waits on a table read.
    auto table_of = [&](int j, int r) -> int32_t {
        const int t = t_begin + j * kTileTokens + r;
        if (j >= n_tiles || t >= t_end) return -1;
        const int32_t phys = tables[(int64_t)b * max_blocks + t / bs];
        if (phys < 0 || phys >= num_physical) {
            if (g == 0) set_flag(flags, PLKV_FLAG_BAD_BLOCK);
            return -1;
        }
        return phys;
    };

    // Issues the copies of tile j into ring slot j % kKvStages (nothing past
    // the item); thread t < 32 also records row t's offset for the compute
    // warps.
    auto issue = [&](int j) {
        if (j >= n_tiles) return;
        const int st = j % kKvStages;
        const int t0 = t_begin + j * kTileTokens;
        uint16_t* kdst = ring + (size_t)st * 2 * kTileTokens * RS;
        uint16_t* vdst = kdst + kTileTokens * RS;
        for (int i = tid; i < kTileTokens * cpr; i += 256) {
            const int r = i / cpr, c = i - r * cpr;
            const int32_t phys = ptab[st][r];
            const int t = t0 + r;
            const int64_t off =
                phys < 0 ? -1 : (((int64_t)phys * KV + g) * bs + (t - (t / bs) * bs)) * (int64_t)D;
            if (c == 0) row_off[st][r] = off;
            if (off >= 0) {
                cp_async16(kdst + r * RS + c * 8, k_cache + off + c * 8);
                cp_async16(vdst + r * RS + c * 8, v_cache + off + c * 8);
            }
        }
    };
    float m_run = -INFINITY, l_run = 0.f, acc[NCH][4];
#pragma unroll
    for (int c = 0; c < NCH; ++c)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[c][e] = 0.f;

    for (int i = tid; i < kKvStages * kTileTokens; i += 256)
        ptab[i / kTileTokens][i % kTileTokens] = table_of(i / kTileTokens, i % kTileTokens);
    __syncthreads();
#pragma unroll 1
    for (int j = 0; j < kKvStages - 1; ++j) {
        issue(j);
        cp_async_commit();
    }
    const bool loader = warp == 7;   // reads the table entries of tile j + kKvStages
#pragma unroll 1
    for (int j = 0; j < n_tiles; ++j) {
        issue(j + kKvStages - 1);
        cp_async_commit();
        cp_async_wait<kKvStages - 1>();   // this thread's copies of tile j landed
        __syncthreads();                   // everyone's did (and the query is staged)
        // ptab slot j % kKvStages was last read by issue(j); refill it with
        // tile j + kKvStages, whose copies are issued two iterations later.
        const int32_t nxt = loader ? table_of(j + kKvStages, lane) : -1;
        const int st = j % kKvStages;
        const int t0 = t_begin + j * kTileTokens;
        const int nt = min(kTileTokens, t_end - t0);
        const uint16_t* kt = ring + (size_t)st * 2 * kTileTokens * RS;
        const uint16_t* vt = kt + kTileTokens * RS;
        if (active) {
            const bool tok_ok = lane < nt && row_off[st][lane] >= 0;
            float s = 0.f;
            if (tok_ok) {
                const uint16_t* kr = kt + lane * RS;
                const float* qr = qs + warp * DP;
#pragma unroll 4
                for (int c = 0; c < cpr; ++c) {
                    float x[8];
                    unpack8(*reinterpret_cast<const uint4*>(kr + c * 8), x);
                    const float4 q0 = *reinterpret_cast<const float4*>(qr + c * 8);
                    const float4 q1 = *reinterpret_cast<const float4*>(qr + c * 8 + 4);
                    s = fmaf(q0.x, x[0], s);
                    s = fmaf(q0.y, x[1], s);
                    s = fmaf(q0.z, x[2], s);
                    s = fmaf(q0.w, x[3], s);
                    s = fmaf(q1.x, x[4], s);
                    s = fmaf(q1.y, x[5], s);
                    s = fmaf(q1.z, x[6], s);
                    s = fmaf(q1.w, x[7], s);
                }
            }
            const float sc = s * scale;
            if (scores && lane < nt && t0 + lane < max_seq_len)
                scores[((int64_t)b * Hq + h) * max_seq_len + t0 + lane] = sc;
            const float sv = tok_ok ? sc : -INFINITY;
            const float m_new = fmaxf(m_run, warp_max(sv));
            const float alpha = (m_new == -INFINITY) ? 1.f : expf(m_run - m_new);
            const float p = tok_ok ? expf(sv - m_new) : 0.f;
            l_run = l_run * alpha + warp_sum(p);
            m_run = m_new;
            ps[lane * 8 + warp] = p;
            __syncwarp();
#pragma unroll
            for (int c = 0; c < NCH; ++c)
#pragma unroll
                for (int e = 0; e < 4; ++e) acc[c][e] *= alpha;
            for (int r = 0; r < nt; ++r) {
                const float pr = ps[r * 8 + warp];
                if (pr == 0.f) continue;   // masked token: its row may be stale
                const uint16_t* vr = vt + r * RS + lane * 4;
#pragma unroll
                for (int c = 0; c < NCH; ++c) {
                    if (lane * 4 + 128 * c < D) {
                        const uint2 raw = *reinterpret_cast<const uint2*>(vr + 128 * c);
                        const float2 x01 = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
                        const float2 x23 = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
                        acc[c][0] = fmaf(pr, x01.x, acc[c][0]);
                        acc[c][1] = fmaf(pr, x01.y, acc[c][1]);
                        acc[c][2] = fmaf(pr, x23.x, acc[c][2]);
                        acc[c][3] = fmaf(pr, x23.y, acc[c][3]);
                    }
                }
            }
        }
        if (loader) ptab[j % kKvStages][lane] = nxt;
        __syncthreads();   // slot st is rewritten by the next iteration's issue
    }
    cp_async_wait<0>();
    if (!active) return;
    const int64_t row = (int64_t)blockIdx.x * Hq + h;
    if (lane == 0) {
        ws.part_m[row] = m_run;
        ws.part_l[row] = l_run;
    }
    float* dst = ws.part_ctx + row * D;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
        const int col = lane * 4 + 128 * c;
        if (col < D)
            *reinterpret_cast<float4*>(dst + col) =
                make_float4(acc[c][0], acc[c][1], acc[c][2], acc[c][3]);
    }
}

size_t fullkv_exact_smem_bytes(int D) {
    return size_t(8) * (D + 4) * 4 + size_t(kTileTokens) * 8 * 4 +
           size_t(kKvStages) * 2 * kTileTokens * (D + kKvPad) * 2;
}

template <int NCH>
static cudaError_t launch_fullkv_exact_t(const plkv_fullkv_decode_args& a, DecodeWorkspace ws,
                                         cudaStream_t st) {
    const size_t smem = fullkv_exact_smem_bytes(a.head_dim);
    cudaError_t e = cudaFuncSetAttribute(fullkv_partial_exact_kernel<NCH>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    dim3 grid(a.n_items, a.kv_heads);
    fullkv_partial_exact_kernel<NCH><<<grid, 256, smem, st>>>(
        a.q, a.k_cache, a.v_cache, a.num_physical, a.kv_heads, a.block_size, a.head_dim,
        a.q_heads, a.scale, a.block_tables, a.max_blocks, a.seq_lens, a.items, ws, a.scores,
        a.max_seq_len, a.err_flags);
    return cudaGetLastError();
}

cudaError_t launch_fullkv_partial_exact(const plkv_fullkv_decode_args& a, DecodeWorkspace ws,
                                        cudaStream_t st) {
    switch ((a.head_dim + 127) / 128) {
        case 1: return launch_fullkv_exact_t<1>(a, ws, st);
        case 2: return launch_fullkv_exact_t<2>(a, ws, st);
        default: return cudaErrorInvalidValue;
    }
}

// ------------------------------------------------------- query projection

// q_lat[b, g*G + j, l] = sum_d W_k[g, l, d] * q[b, g*G + j, d]: per KV head g
// a GEMM of the B*G query rows (b, j) by the L latent rows of W_k[g], K = D.
// grid = (ceil(B*G / 64), ceil(L / 32), KV), block = 256: a 64 x 32 output
// tile, D in chunks of 32 through shared memory; each thread owns 4 rows x 2
// columns and adds d in increasing order.  (One CTA per (b, g) with a warp
// per latent row re-read W_k[g] for every batch row and took 47 us for
// B = 64, 32 heads, L = 256.)
constexpr int kPqRows = 64, kPqCols = 32, kPqK = 32;

__global__ void __launch_bounds__(256)
project_query_kernel(const float* __restrict__ q, const float* __restrict__ w_k,
                     float* __restrict__ q_lat, int B, int Hq, int KV, int D, int L) {
    __shared__ float as[kPqRows][kPqK + 1];
    __shared__ float bs_[kPqCols][kPqK + 1];
    const int G = Hq / KV, M = B * G;
    const int g = blockIdx.z, m0 = blockIdx.x * kPqRows, l0 = blockIdx.y * kPqCols;
    const int tid = threadIdx.x, tm = tid >> 4, tn = tid & 15;
    float acc[4][2] = {{0.f, 0.f}, {0.f, 0.f}, {0.f, 0.f}, {0.f, 0.f}};
    for (int d0 = 0; d0 < D; d0 += kPqK) {
#pragma unroll
        for (int k = 0; k < kPqRows * kPqK / 256; ++k) {
            const int i = tid + 256 * k, r = i / kPqK, dd = i % kPqK;
            const int m = m0 + r, d = d0 + dd;
            float v = 0.f;
            if (m < M && d < D) {
                const int b = m / G, j = m - b * G;
                v = q[((int64_t)b * Hq + g * G + j) * D + d];
            }
            as[r][dd] = v;
        }
#pragma unroll
        for (int k = 0; k < kPqCols * kPqK / 256; ++k) {
            const int i = tid + 256 * k, c = i / kPqK, dd = i % kPqK;
            const int l = l0 + c, d = d0 + dd;
            bs_[c][dd] = (l < L && d < D) ? w_k[((int64_t)g * L + l) * D + d] : 0.f;
        }
        __syncthreads();
#pragma unroll 8
        for (int dd = 0; dd < kPqK; ++dd) {
            float a[4], w2[2];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = as[tm * 4 + i][dd];
#pragma unroll
            for (int k = 0; k < 2; ++k) w2[k] = bs_[tn * 2 + k][dd];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int k = 0; k < 2; ++k) acc[i][k] = fmaf(a[i], w2[k], acc[i][k]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int m = m0 + tm * 4 + i;
        if (m >= M) continue;
        const int b = m / G, j = m - b * G;
        float* dst = q_lat + ((int64_t)b * Hq + g * G + j) * L;
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const int l = l0 + tn * 2 + k;
            if (l < L) dst[l] = acc[i][k];
        }
    }
}

cudaError_t launch_project_query(const float* q, const float* w_k, float* q_lat, int B, int Hq,
                                 int KV, int D, int L, cudaStream_t st) {
    // The batched GEMM (4 x 4 outputs per thread, 16-byte operand loads)
    // where the shapes allow it: 1024 query rows per KV head x 256 latent
    // columns took 48 us per call in the 4 x 2 tiles below.
    if (rows_gemm_supported(q, w_k, q_lat, D, L))
        return launch_rows_gemm(q, w_k, true, q_lat, B, Hq, KV, D, L, st);
    const int M = B * (Hq / KV);
    dim3 grid((M + kPqRows - 1) / kPqRows, (L + kPqCols - 1) / kPqCols, KV);
    project_query_kernel<<<grid, 256, 0, st>>>(q, w_k, q_lat, B, Hq, KV, D, L);
    return cudaGetLastError();
}

}  // namespace plkv
