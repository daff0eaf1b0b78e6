// placeholder: tensor-core forward (filled in below)
#include "capi_internal.h"
namespace ptof {
bool gdn_fwd_tc_supports(const ptof_gdn_params&) { return false; }
int launch_gdn_fwd_tc(Workspace*, const void*, const void*, const void*, const void*, const float*,
                      const float*, void*, float*, cudaStream_t) {
  return fail(PTOF_EUNSUPPORTED, "tensor-core forward not built");
}
}  // namespace ptof
