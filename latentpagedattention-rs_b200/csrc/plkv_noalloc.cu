// plkv_noalloc.cu -- a decode entry point that needs no caller workspace.
//
// plkv_latent_decode needs a scratch workspace for its split-K partial
// results, which the caller allocates.  Some callers cannot allocate device
// memory at all: a plugin host that owns every device byte through its own
// pool and hands the library only input and output buffers, or a foreign-
// language binding with no CUDA allocator of its own.  For them this file
// keeps the scratch in a fixed array that is part of the library image, so
// the call itself never allocates.
//
// The array is file-scope device memory: every GPU that loads the library
// holds PLKV_NOALLOC_SCRATCH_BYTES of it until the process exits.  Every call
// shares it, so calls that overlap on the GPU (other streams, other host
// threads) race on it.  It keeps the last call's contents; nothing in it needs
// clearing because the partial pass writes every element the combine reads.
#include <mutex>

#include "plkv_common.cuh"

namespace {

__device__ __align__(256) unsigned char g_plkv_scratch[PLKV_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mutex;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of the scratch array on the current device.  The array's
// name is only a host-side stand-in for it, so the address is looked up once
// per device, with that device current, and cached.
int scratch_address(void** out) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return PLKV_ERR_CUDA;
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (!g_scratch_addr[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_plkv_scratch) != cudaSuccess || !p) return PLKV_ERR_CUDA;
        g_scratch_addr[dev] = p;
    }
    *out = g_scratch_addr[dev];
    return PLKV_OK;
}

}  // namespace

extern "C" int plkv_latent_decode_noalloc(const plkv_latent_decode_args* args,
                                          plkv_stream_t stream) {
    if (!args) return PLKV_ERR_INVALID_ARGUMENT;
    if (args->n_items <= 0 || args->batch <= 0 || args->q_heads <= 0 || args->latent_dim <= 0 ||
        args->value_dim <= 0)
        return PLKV_ERR_ZERO_VALUE;
    const size_t need =
        plkv::decode_workspace_bytes(args->n_items, args->batch, args->q_heads, args->latent_dim,
                                     args->value_dim);
    if (need > (size_t)PLKV_NOALLOC_SCRATCH_BYTES) return PLKV_ERR_WORKSPACE;
    void* scratch = nullptr;
    int st = scratch_address(&scratch);
    if (st != PLKV_OK) return st;
    plkv_latent_decode_args a = *args;
    a.workspace = scratch;
    a.workspace_bytes = (size_t)PLKV_NOALLOC_SCRATCH_BYTES;
    return plkv_latent_decode(&a, stream);
}
