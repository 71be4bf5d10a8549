// tcgen05 (UMMA + TMEM) paged chunked-prefill attention for sm_100a.
#include "common.cuh"
#include "launch.cuh"
#include "params.cuh"

namespace mi {

bool prefill_tc_supported(int dtype, int D, int G, int block_size) {
  (void)dtype;
  (void)D;
  (void)G;
  (void)block_size;
  return false;
}

cudaError_t launch_prefill_tc(const AttnParams &p, int dtype, int G, int32_t max_seqlen_q,
                              bool paged, cudaStream_t stream) {
  (void)p;
  (void)dtype;
  (void)G;
  (void)max_seqlen_q;
  (void)paged;
  (void)stream;
  return cudaErrorNotSupported;
}

}  // namespace mi
