// Entry points of include/pa_b200.h whose kernels are not built yet.
#include "common.cuh"

using namespace pa;

extern "C" {
pa_status pa_comm_unique_id(uint8_t*) { return fail(PA_ERR_UNSUPPORTED, "ring not built yet"); }
pa_status pa_comm_init(pa_comm**, const uint8_t*, int32_t, int32_t) {
  return fail(PA_ERR_UNSUPPORTED, "ring not built yet");
}
pa_status pa_comm_destroy(pa_comm*) { return PA_OK; }
pa_status pa_ring_fwd(pa_comm*, const pa_sdpa_desc*, const void*, const void*, const void*, void*,
                      float*, void*) {
  return fail(PA_ERR_UNSUPPORTED, "ring not built yet");
}
pa_status pa_ring_bwd(pa_comm*, const pa_sdpa_desc*, const void*, const void*, const void*,
                      const void*, const void*, const float*, void*, void*, void*, void*) {
  return fail(PA_ERR_UNSUPPORTED, "ring not built yet");
}
}
