// Host-side launchers of the scan kernels (internal to libsubq_b200).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>

#include "kernels.hpp"

namespace subq {

struct ScanParams;

// Exact float32 path (scan_simt.cu).
size_t exact_bwd_smem_bytes(int d, int e, int normalize, size_t acc_bytes);
cudaError_t launch_fwd_exact(const ScanParams& p, int dtype, cudaStream_t st);
cudaError_t launch_bwd_exact(const ScanParams& p, int dtype, cudaStream_t st);
cudaError_t launch_feature_map(void* x, int64_t n, int dtype, cudaStream_t st);
// dst[b, hk] = sum of src[b, hk * G .. hk * G + G) (grouped K/V gradients)
cudaError_t launch_group_sum(const void* src, void* dst, int dtype, int B, int Hkv, int G, int N, int e,
                             int64_t dsb, int64_t dsh, int64_t dsn, cudaStream_t st);

// Chunk-parallel float32 forward on the CUDA cores (scan_chunk.cu): the
// automatic path's choice for calls of at least kChunkMinTokens tokens that
// the tensor-core kernels do not take (float32, or d, e other than 64).
constexpr int kChunkMinTokens = 64;
bool chunk_fwd_usable(const ScanParams& p, int dtype);
size_t chunk_fwd_workspace_bytes(const ScanParams& p);
// Returns the number of kernel launches issued through *launches (2, or 4 in
// the chunk-parallel form for calls with few sequences).
cudaError_t launch_fwd_chunk(const ScanParams& p, int dtype, cudaStream_t st, int* launches);

// Per-head RMSNorm of the scan's output (head_norm.cu). Rows are the
// (b, n, h) of [B, H, N, D] views with element strides; D contiguous.
struct RmsParams {
    int B, H, N, D;
    float eps;
    const void* x; int64_t x_sb, x_sh, x_sn;     // input (the scan's output)
    void* y; int64_t y_sb, y_sh, y_sn;           // forward output
    const void* dy; int64_t dy_sb, dy_sh, dy_sn; // backward: upstream gradient
    void* dx; int64_t dx_sb, dx_sh, dx_sn;       // backward: input gradient
    const float* w;                              // [D] or null (weight 1)
    float* dw;                                   // backward: [D] or null
    float* part;                                 // backward: [rms_blocks][D] CTA partials of dw
    // bit t set: tensor t (x, y, dy, dx) is dense in (b, n, h) row order
    // (strides N*H*D, D, H*D), so row r starts at element r * D
    int dense;
};
constexpr int kRmsMaxBlocks = 148 * 8;
bool rms_supported_dim(int D);
int rms_blocks(const RmsParams& p);
cudaError_t launch_rms_fwd(const RmsParams& p, int dtype, cudaStream_t st);  // 1 launch
cudaError_t launch_rms_bwd(const RmsParams& p, int dtype, cudaStream_t st);  // 2 launches with dw, else 1

// Tensor-core path (scan_tc.cu).
bool tc_supported(const ScanParams& p, int dtype);
bool tc_bwd_supported(const ScanParams& p, int dtype);
size_t tc_fwd_workspace_bytes(const ScanParams& p);
size_t tc_bwd_workspace_bytes(const ScanParams& p);
size_t tc_segment_states_bytes(const ScanParams& p);
// Returns the number of kernel launches issued through *launches.
cudaError_t launch_fwd_tc(const ScanParams& p, int dtype, cudaStream_t st, int* launches);
cudaError_t launch_bwd_tc(const ScanParams& p, int dtype, cudaStream_t st, int* launches);
// One-pass backward from the forward's handover (scan_tc_bwd1.cu): no decay,
// segment_states and the forward's output given.
bool bwd1_usable(const ScanParams& p);
size_t bwd1_workspace_bytes(const ScanParams& p);
cudaError_t launch_bwd1(const ScanParams& p, int dtype, cudaStream_t st, int* launches);
// Device-side status word of the tensor-core kernels (bounded waits).
cudaError_t tc_read_status(cudaStream_t st, int* status);
// Diagnostic bounded wait that runs out (see subq_selftest_wait_timeout).
cudaError_t tc_selftest_wait_timeout(int polls, cudaStream_t st);

}  // namespace subq
