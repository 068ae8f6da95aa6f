// placeholder until the tcgen05 backward lands
#include "sfa_common.cuh"
#include "sfa_internal.h"
namespace sfa {
bool tc_bwd_supported(const SfaParams&, const char** why) { *why = "not built"; return false; }
cudaError_t launch_bwd_dq_tc(const SfaParams&, const float*, cudaStream_t) { return cudaErrorNotSupported; }
cudaError_t launch_bwd_dkdv_tc(const SfaParams&, const BwdLayout&, char*, const float*, cudaStream_t) { return cudaErrorNotSupported; }
}
