// Tensor-core (tcgen05 / TMEM / TMA) block-sparse attention for sm_100a.
// Placeholder: no shapes are routed here yet.
#include "sbfa_common.cuh"

namespace sbfa {

bool tc_supports(int pass, int dtype, int64_t D) {
  (void)pass; (void)dtype; (void)D;
  return false;
}

int tc_tiles(int pass, int64_t* tm, int64_t* tn) {
  (void)pass;
  *tm = 128;
  *tn = 128;
  return SBFA_OK;
}

int tc_fwd(int, int, const void*, const void*, const void*, void*, float*, int, float,
           const MaskParams&, const int32_t*, const int32_t*, int*, cudaStream_t) {
  return fail(SBFA_ERR_UNSUPPORTED, "tensor-core forward not built");
}

int tc_bwd(int, int, const void*, const void*, const void*, const void*, const float*,
           const void*, void*, void*, void*, float*, int, float, const MaskParams&,
           const int32_t*, const int32_t*, const int32_t*, const int32_t*, int*, cudaStream_t) {
  return fail(SBFA_ERR_UNSUPPORTED, "tensor-core backward not built");
}

}  // namespace sbfa
