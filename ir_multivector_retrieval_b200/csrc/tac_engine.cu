// tac_engine.cu — general-dimension k-means engine (ragged problem batches).
#include "tac_engine.h"

namespace mvr {

int kmeans_general_device(Ctx* ctx, const float*, uint64_t, uint32_t, uint32_t, uint32_t, float,
                          uint64_t, float*, uint32_t*, float*, uint32_t*) {
  return fail(ctx, MVR_E_INVALID_ARGUMENT, "general-dimension k-means is not built yet");
}

}  // namespace mvr

extern "C" int mvr_tac_cluster_flat(mvr_ctx* h, const uint32_t*, uint64_t, const float*, uint64_t,
                                    uint32_t, const mvr_clustering_params*, float*, uint32_t*,
                                    uint32_t*, uint64_t, uint64_t*, float*) {
  if (!h) return MVR_E_INVALID_ARGUMENT;
  return mvr::fail(&h->impl, MVR_E_INVALID_ARGUMENT, "tac.clusterFlat device path is not built yet");
}
