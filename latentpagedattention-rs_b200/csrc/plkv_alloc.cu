// plkv_alloc.cu -- device-side allocation of token positions in a paged pool.
//
// Restates the bump allocation of PagedBlockTable.allocate_token_positions
// (python_ref/latent_paged_attention/block_table.py:26-38) and
// BlockTable::allocate_tokens (crates/plkv-core/src/lib.rs:1346-1364) for a
// batch of sequences on the device, so a decode loop can advance its tables
// without host round trips:
//   for every new token position p = len, len+1, ...: the logical block p / bs
//   takes the next physical block of the pool's counter when it has none yet,
//   the token's slot is physical * bs + p % bs, and the length grows by one.
// The reference keeps one counter per table; here the sequences of a batch
// share the pool's counter, and blocks are handed out in sequence order (then
// logical-block order), so the result is deterministic: for one sequence and
// a counter starting at 0 it is exactly the reference's.  A table entry < 0
// means "no physical block yet" (the reference's list ends there).
#include "plkv_common.cuh"

namespace plkv {
namespace {

constexpr int kAllocThreads = 1024;

// Inclusive block-wide scan of two int32 values per thread.
__device__ __forceinline__ void scan2(int32_t* a, int32_t* b) {
    const int t = threadIdx.x;
    for (int off = 1; off < kAllocThreads; off <<= 1) {
        const int32_t va = t >= off ? a[t - off] : 0;
        const int32_t vb = t >= off ? b[t - off] : 0;
        __syncthreads();
        a[t] += va;
        b[t] += vb;
        __syncthreads();
    }
}

// One CTA walks the batch in chunks of kAllocThreads sequences, carrying the
// blocks handed out and the slots written so far across chunks.
__global__ void __launch_bounds__(kAllocThreads)
allocate_slots_kernel(int32_t* __restrict__ tables, int64_t max_blocks,
                      int32_t* __restrict__ seq_lens, const int32_t* __restrict__ counts,
                      int32_t batch, int32_t bs, int32_t* __restrict__ next_block,
                      int64_t num_physical, int64_t* __restrict__ slots, int64_t max_slots,
                      int32_t* flags) {
    __shared__ int32_t s_blocks[kAllocThreads], s_slots[kAllocThreads];
    __shared__ int64_t carry_blocks, carry_slots, base_block;
    const int t = threadIdx.x;
    if (t == 0) {
        carry_blocks = 0;
        carry_slots = 0;
        base_block = *next_block;
    }
    __syncthreads();
    for (int c0 = 0; c0 < batch; c0 += kAllocThreads) {
        const int b = c0 + t;
        int32_t len = 0, cnt = 0, need = 0;
        if (b < batch) {
            len = seq_lens[b];
            cnt = counts ? counts[b] : 1;
            if (len < 0 || cnt < 0 || (int64_t)len + cnt > INT32_MAX) {
                set_flag(flags, PLKV_FLAG_BAD_LENGTH);
                len = len < 0 ? 0 : len;
                cnt = 0;
            }
            if (cnt > 0) {
                const int64_t lb1 = ((int64_t)len + cnt - 1) / bs;
                for (int64_t lb = len / bs; lb <= lb1 && lb < max_blocks; ++lb)
                    if (tables[(int64_t)b * max_blocks + lb] < 0) ++need;
            }
        }
        s_blocks[t] = need;
        s_slots[t] = cnt;
        __syncthreads();
        scan2(s_blocks, s_slots);
        const int64_t first_block = base_block + carry_blocks + s_blocks[t] - need;
        const int64_t first_slot = carry_slots + s_slots[t] - cnt;
        if (b < batch && cnt > 0) {
            int32_t* row = tables + (int64_t)b * max_blocks;
            int64_t given = 0;
            const int64_t lb1 = ((int64_t)len + cnt - 1) / bs;
            for (int64_t lb = len / bs; lb <= lb1 && lb < max_blocks; ++lb) {
                if (row[lb] >= 0) continue;
                const int64_t id = first_block + given++;
                if (id < num_physical) row[lb] = static_cast<int32_t>(id);
                else set_flag(flags, PLKV_FLAG_BAD_BLOCK);  // pool exhausted
            }
            for (int32_t i = 0; i < cnt; ++i) {
                const int64_t pos = (int64_t)len + i, lb = pos / bs;
                const int32_t phys = lb < max_blocks ? row[lb] : -1;
                int64_t slot = -1;  // the append skips negative slots
                if (phys >= 0 && phys < num_physical) slot = (int64_t)phys * bs + (pos - lb * bs);
                else set_flag(flags, PLKV_FLAG_BAD_POSITION);
                if (first_slot + i < max_slots) slots[first_slot + i] = slot;
                else set_flag(flags, PLKV_FLAG_BAD_POSITION);  // slots buffer too small
            }
            seq_lens[b] = len + cnt;
        }
        __syncthreads();
        if (t == kAllocThreads - 1) {
            carry_blocks += s_blocks[t];
            carry_slots += s_slots[t];
        }
        __syncthreads();
    }
    if (t == 0) {
        const int64_t nb = base_block + carry_blocks;
        *next_block = static_cast<int32_t>(nb < INT32_MAX ? nb : INT32_MAX);
    }
}

}  // namespace
}  // namespace plkv

extern "C" int plkv_allocate_slots(int32_t* block_tables, int64_t max_blocks, int32_t* seq_lens,
                                   const int32_t* counts, int32_t batch, int32_t block_size,
                                   int32_t* next_block, int64_t num_physical, int64_t* slots,
                                   int64_t max_slots, int32_t* err_flags, plkv_stream_t stream) {
    if (batch <= 0 || block_size <= 0 || max_blocks <= 0 || num_physical <= 0 || max_slots <= 0)
        return PLKV_ERR_ZERO_VALUE;
    if (!block_tables || !seq_lens || !next_block || !slots) return PLKV_ERR_INVALID_ARGUMENT;
    if (num_physical > INT32_MAX) return PLKV_ERR_ARITHMETIC_OVERFLOW;  // int32 table entries
    plkv::allocate_slots_kernel<<<1, plkv::kAllocThreads, 0, (cudaStream_t)stream>>>(
        block_tables, max_blocks, seq_lens, counts, batch, block_size, next_block, num_physical,
        slots, max_slots, err_flags);
    return cudaGetLastError() == cudaSuccess ? PLKV_OK : PLKV_ERR_CUDA;
}
