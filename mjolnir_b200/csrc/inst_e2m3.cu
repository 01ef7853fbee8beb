// The decode kernels (tensor-core and CUDA-core variants) for the e2m3 KV
// format: one translation unit per format, so the library compiles in parallel.
#include "decode_simt.cuh"
#include "decode_tc.cuh"

namespace mj {
template cudaError_t launch_tc_fmt<MJ_KV_E2M3>(const mj_decode_args&, int, bool, const CUtensorMap&, const CUtensorMap&,
                                               cudaStream_t, bool);
template cudaError_t launch_simt_fmt<MJ_KV_E2M3>(const mj_decode_args&, int, cudaStream_t);
}  // namespace mj
