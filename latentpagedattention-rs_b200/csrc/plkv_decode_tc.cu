// plkv_decode_tc.cu -- tcgen05 (tensor-core) split-K latent decode.
#include "plkv_common.cuh"

namespace plkv {

bool tc_supported(const plkv_latent_decode_args&) { return false; }

cudaError_t launch_latent_partial_tc(const plkv_latent_decode_args&, DecodeWorkspace,
                                     cudaStream_t) {
    return cudaErrorNotSupported;
}

}  // namespace plkv
