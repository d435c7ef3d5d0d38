// Tensor-core path of the scan (tcgen05 + TMA + TMEM). Placeholder until the
// chunked kernels land: reports the shape as unsupported.
#include "scan_common.cuh"
#include "scan_launch.h"

namespace subq {

bool tc_supported(const ScanParams&, int) { return false; }
size_t tc_fwd_workspace_bytes(const ScanParams&) { return 0; }
size_t tc_bwd_workspace_bytes(const ScanParams&) { return 0; }
cudaError_t launch_fwd_tc(const ScanParams&, int, cudaStream_t, int* launches) {
    *launches = 0;
    return cudaErrorNotSupported;
}
cudaError_t launch_bwd_tc(const ScanParams&, int, cudaStream_t, int* launches) {
    *launches = 0;
    return cudaErrorNotSupported;
}
cudaError_t tc_read_status(cudaStream_t, int* status) {
    *status = 0;
    return cudaSuccess;
}

}  // namespace subq
