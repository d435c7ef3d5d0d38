// The C ABI (include/kernels.hpp): argument validation, workspace sizing,
// kernel-path selection and launch. No exception crosses this boundary.
#include <cuda_runtime.h>
#include <stdio.h>
#include <string.h>

#include <mutex>
#include <string>

#include "kernels.hpp"
#include "scan_common.cuh"
#include "scan_launch.h"

namespace {

thread_local std::string g_last_error;
thread_local int g_last_path = SUBQ_PATH_AUTO;
thread_local int g_last_launches = 0;

int fail(int code, const std::string& msg) {
    g_last_error = msg;
    return code;
}

int fail_cuda(cudaError_t err, const char* where) {
    return fail(SUBQ_ERR_CUDA, std::string(where) + ": " + cudaGetErrorString(err));
}

size_t elem_size(int dtype) { return dtype == SUBQ_FP64 ? 8 : dtype == SUBQ_FP32 ? 4 : 2; }

constexpr size_t kAlign = 256;
size_t align_up(size_t x) { return (x + kAlign - 1) / kAlign * kAlign; }

// Common checks of a scan description; fills the scalar part of ScanParams.
int check_desc(const subq_scan_desc& d, subq::ScanParams& p) {
    if (d.batch < 0 || d.heads < 0 || d.seq_len < 0)
        return fail(SUBQ_ERR_INVALID_ARGUMENT, "negative batch, heads or seq_len");
    if (d.head_dim <= 0 || d.value_dim <= 0)
        return fail(SUBQ_ERR_INVALID_ARGUMENT, "head_dim and value_dim must be positive");
    if (d.batch > 65535 || d.heads > 65535 || d.seq_len > (int64_t)1 << 30)
        return fail(SUBQ_ERR_INVALID_ARGUMENT, "batch/heads above 65535 or seq_len above 2^30");
    if (d.head_dim > 256 || d.value_dim > 256)
        return fail(SUBQ_ERR_UNSUPPORTED, "head_dim and value_dim above 256 are not supported");
    if (d.dtype != SUBQ_FP32 && d.dtype != SUBQ_FP16 && d.dtype != SUBQ_BF16 && d.dtype != SUBQ_FP64)
        return fail(SUBQ_ERR_INVALID_ARGUMENT, "unknown dtype");
    if (d.decay_mode < SUBQ_DECAY_NONE || d.decay_mode > SUBQ_DECAY_PER_TOKEN)
        return fail(SUBQ_ERR_INVALID_ARGUMENT, "unknown decay_mode");
    if ((d.decay_mode == SUBQ_DECAY_PER_HEAD || d.decay_mode == SUBQ_DECAY_PER_TOKEN) && !d.log_gamma)
        return fail(SUBQ_ERR_INVALID_ARGUMENT, "log_gamma pointer required by decay_mode");
    if (d.path < SUBQ_PATH_AUTO || d.path > SUBQ_PATH_CHUNKED)
        return fail(SUBQ_ERR_INVALID_ARGUMENT, "unknown kernel path");
    if (!(d.clamp_min >= 0.f))
        return fail(SUBQ_ERR_INVALID_ARGUMENT, "clamp_min must be >= 0");
    if (d.kv_heads < 0 || (d.kv_heads > 0 && d.heads % d.kv_heads != 0))
        return fail(SUBQ_ERR_INVALID_ARGUMENT, "kv_heads must be 0 or a divisor of heads");
    if (d.reverse != 0 && d.reverse != 1) return fail(SUBQ_ERR_INVALID_ARGUMENT, "reverse must be 0 or 1");
    memset(&p, 0, sizeof(p));
    p.B = (int)d.batch; p.H = (int)d.heads; p.N = (int)d.seq_len;
    p.d = (int)d.head_dim; p.e = (int)d.value_dim;
    p.normalize = d.normalize ? 1 : 0;
    p.scale = d.scale;
    p.clamp_min = d.clamp_min;
    p.decay_mode = d.decay_mode;
    p.lg_scalar = d.log_gamma_scalar;
    p.log_gamma = d.log_gamma;
    p.mask = d.mask;
    p.mask_sb = d.mask ? d.mask_stride_b : 0;
    p.flush = d.flush_subnormal ? 1 : 0;
    p.kvg = (d.kv_heads > 0 && d.heads > 0) ? (int)(d.heads / d.kv_heads) : 1;
    p.reverse = d.reverse;
    return SUBQ_OK;
}

// `empty`: the call touches no element (B, H or N is 0), so a null pointer is fine.
int check_tensor(const subq_tensor4& t, const char* name, int dtype, bool empty) {
    if (!t.data && !empty) return fail(SUBQ_ERR_INVALID_ARGUMENT, std::string(name) + " is null");
    if (reinterpret_cast<uintptr_t>(t.data) % elem_size(dtype) != 0)
        return fail(SUBQ_ERR_INVALID_ARGUMENT, std::string(name) + " is not aligned to its element size");
    if (t.stride_b < 0 || t.stride_h < 0 || t.stride_n < 0)
        return fail(SUBQ_ERR_INVALID_ARGUMENT, std::string(name) + " has a negative stride");
    return SUBQ_OK;
}

// Calls of at most this many tokens (streaming decode steps) run on the
// token-recurrent kernel under SUBQ_PATH_AUTO: a single-token step takes
// about 3.7 us there against about 13 us for one chunk of the tensor-core
// kernel (measured on B200 at B*H <= 48, CUDA-graph replay); the two meet
// near 16 tokens.
constexpr int kRecurrentMaxTokens = 16;

bool use_tc(const subq::ScanParams& p, int dtype, int path) {
    if (path == SUBQ_PATH_EXACT || path == SUBQ_PATH_CHUNKED || dtype == SUBQ_FP64) return false;
    if (path == SUBQ_PATH_AUTO && p.N <= kRecurrentMaxTokens) return false;
    return subq::tc_supported(p, dtype);
}

bool use_tc_bwd(const subq::ScanParams& p, int dtype, int path) {
    return use_tc(p, dtype, path) && subq::tc_bwd_supported(p, dtype);
}

// The automatic path takes the chunked forward while its workspace (about
// 0.8 KB per token-head at d = 64, 2.3 KB at d = 256) stays within this; larger
// calls run on the exact path, which needs none.
constexpr size_t kChunkMaxWorkspace = (size_t)4 << 30;

// The forward's kernel family when the tensor cores do not take the call.
int fwd_simt_path(const subq::ScanParams& p, int dtype, int path) {
    if (path == SUBQ_PATH_CHUNKED) return subq::chunk_fwd_usable(p, dtype) ? SUBQ_PATH_CHUNKED : -1;
    if (path == SUBQ_PATH_AUTO && p.N >= subq::kChunkMinTokens && subq::chunk_fwd_usable(p, dtype) &&
        subq::chunk_fwd_workspace_bytes(p) <= kChunkMaxWorkspace)
        return SUBQ_PATH_CHUNKED;
    return SUBQ_PATH_EXACT;
}

int fill_fwd(const subq_fwd_args* a, subq::ScanParams& p) {
    if (!a) return fail(SUBQ_ERR_INVALID_ARGUMENT, "null argument block");
    int rc = check_desc(a->desc, p);
    if (rc) return rc;
    const int dt = a->desc.dtype;
    const bool empty = p.B == 0 || p.H == 0 || p.N == 0;
    if ((rc = check_tensor(a->q, "q", dt, empty)) || (rc = check_tensor(a->k, "k", dt, empty)) ||
        (rc = check_tensor(a->v, "v", dt, empty)) || (rc = check_tensor(a->o, "o", dt, empty)))
        return rc;
    p.q = a->q.data; p.q_sb = a->q.stride_b; p.q_sh = a->q.stride_h; p.q_sn = a->q.stride_n;
    p.k = a->k.data; p.k_sb = a->k.stride_b; p.k_sh = a->k.stride_h; p.k_sn = a->k.stride_n;
    p.v = a->v.data; p.v_sb = a->v.stride_b; p.v_sh = a->v.stride_h; p.v_sn = a->v.stride_n;
    p.o = a->o.data; p.o_sb = a->o.stride_b; p.o_sh = a->o.stride_h; p.o_sn = a->o.stride_n;
    p.S_in = a->state_in; p.z_in = a->norm_in;
    p.S_out = a->state_out; p.z_out = a->norm_out;
    p.seg_out = a->segment_states;
    return SUBQ_OK;
}

int fill_bwd(const subq_bwd_args* a, subq::ScanParams& p) {
    if (!a) return fail(SUBQ_ERR_INVALID_ARGUMENT, "null argument block");
    int rc = check_desc(a->desc, p);
    if (rc) return rc;
    const int dt = a->desc.dtype;
    const bool empty = p.B == 0 || p.H == 0 || p.N == 0;
    if ((rc = check_tensor(a->q, "q", dt, empty)) || (rc = check_tensor(a->k, "k", dt, empty)) ||
        (rc = check_tensor(a->v, "v", dt, empty)) || (rc = check_tensor(a->dout, "dout", dt, empty)) ||
        (rc = check_tensor(a->dq, "dq", dt, empty)) || (rc = check_tensor(a->dk, "dk", dt, empty)) ||
        (rc = check_tensor(a->dv, "dv", dt, empty)))
        return rc;
    if (empty) return SUBQ_OK;
    const void* ins[] = {a->q.data, a->k.data, a->v.data, a->dout.data};
    const void* outs[] = {a->dq.data, a->dk.data, a->dv.data};
    for (const void* in : ins)
        for (const void* out : outs)
            if (in == out)
                return fail(SUBQ_ERR_ALIAS,
                            "subquadratic_attention_backward: gradient outputs must not alias inputs");
    if (a->dq.data == a->dk.data || a->dq.data == a->dv.data || a->dk.data == a->dv.data)
        return fail(SUBQ_ERR_ALIAS, "gradient outputs must be distinct buffers");
    p.q = a->q.data; p.q_sb = a->q.stride_b; p.q_sh = a->q.stride_h; p.q_sn = a->q.stride_n;
    p.k = a->k.data; p.k_sb = a->k.stride_b; p.k_sh = a->k.stride_h; p.k_sn = a->k.stride_n;
    p.v = a->v.data; p.v_sb = a->v.stride_b; p.v_sh = a->v.stride_h; p.v_sn = a->v.stride_n;
    p.g = a->dout.data; p.g_sb = a->dout.stride_b; p.g_sh = a->dout.stride_h; p.g_sn = a->dout.stride_n;
    p.o = a->dq.data; p.o_sb = a->dq.stride_b; p.o_sh = a->dq.stride_h; p.o_sn = a->dq.stride_n;
    p.dk = a->dk.data; p.dk_sb = a->dk.stride_b; p.dk_sh = a->dk.stride_h; p.dk_sn = a->dk.stride_n;
    p.dv = a->dv.data; p.dv_sb = a->dv.stride_b; p.dv_sh = a->dv.stride_h; p.dv_sn = a->dv.stride_n;
    p.S_in = a->state_in; p.z_in = a->norm_in;
    p.dlg = a->dlog_gamma;
    p.seg_in = a->segment_states;
    if (a->out.data) {
        if ((rc = check_tensor(a->out, "out", dt, false))) return rc;
        p.fo = a->out.data; p.fo_sb = a->out.stride_b; p.fo_sh = a->out.stride_h; p.fo_sn = a->out.stride_n;
    }
    return SUBQ_OK;
}

size_t exact_bwd_ws(const subq::ScanParams& p, int dtype) {
    return align_up(elem_size(dtype == SUBQ_FP64 ? SUBQ_FP64 : SUBQ_FP32) * 3 * (size_t)p.B * p.H * (size_t)p.N);
}

// Grouped K/V: the scan kernels write dk [B, H, N, d] and dv [B, H, N, e] per
// query head into contiguous buffers after the kernels' own workspace; group
// sums then write the caller's [B, kv_heads, N, *] gradients.
size_t gqa_dk_bytes(const subq::ScanParams& p, int dtype) {
    return align_up(elem_size(dtype) * (size_t)p.B * p.H * (size_t)p.N * (size_t)p.d);
}
size_t gqa_bytes(const subq::ScanParams& p, int dtype) {
    if (p.kvg <= 1) return 0;
    return gqa_dk_bytes(p, dtype) + align_up(elem_size(dtype) * (size_t)p.B * p.H * (size_t)p.N * (size_t)p.e);
}

size_t scan_bwd_ws(const subq::ScanParams& p, int dtype, bool tc) {
    if (!tc) return exact_bwd_ws(p, dtype);
    return subq::bwd1_usable(p) ? subq::bwd1_workspace_bytes(p) : subq::tc_bwd_workspace_bytes(p);
}

int check_workspace(void* ws, size_t have, size_t need) {
    if (need == 0) return SUBQ_OK;
    if (!ws) return fail(SUBQ_ERR_WORKSPACE, "workspace required: " + std::to_string(need) + " bytes");
    if (have < need)
        return fail(SUBQ_ERR_WORKSPACE, "workspace too small: need " + std::to_string(need) +
                                            " bytes, got " + std::to_string(have));
    if (reinterpret_cast<uintptr_t>(ws) % kAlign != 0)
        return fail(SUBQ_ERR_WORKSPACE, "workspace must be 256-byte aligned");
    return SUBQ_OK;
}

}  // namespace

extern "C" {

int subq_abi_version(void) { return SUBQ_ABI_VERSION; }

const char* subq_last_error(void) { return g_last_error.c_str(); }

int subq_last_path(void) { return g_last_path; }

int subq_device_status(void* stream, int* status) {
    if (!status) return fail(SUBQ_ERR_INVALID_ARGUMENT, "status is null");
    int v = 0;
    cudaError_t err = subq::tc_read_status(static_cast<cudaStream_t>(stream), &v);
    if (err != cudaSuccess) return fail_cuda(err, "subq_device_status");
    *status = v;
    return SUBQ_OK;
}

int subq_last_launches(void) { return g_last_launches; }

int subq_selftest_wait_timeout(int polls, void* stream) {
    if (polls < 1 || polls > (1 << 20)) return fail(SUBQ_ERR_INVALID_ARGUMENT, "polls must be in [1, 2^20]");
    cudaError_t err = subq::tc_selftest_wait_timeout(polls, static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return fail_cuda(err, "subq_selftest_wait_timeout launch");
    g_last_launches = 1;
    return SUBQ_OK;
}

size_t subq_fwd_workspace_bytes(const subq_fwd_args* a) {
    subq::ScanParams p;
    if (fill_fwd(a, p) != SUBQ_OK) return 0;
    if (use_tc(p, a->desc.dtype, a->desc.path)) return subq::tc_fwd_workspace_bytes(p);
    if (fwd_simt_path(p, a->desc.dtype, a->desc.path) == SUBQ_PATH_CHUNKED) return subq::chunk_fwd_workspace_bytes(p);
    return 0;
}

size_t subq_segment_states_bytes(const subq_fwd_args* a) {
    subq::ScanParams p;
    if (fill_fwd(a, p) != SUBQ_OK || p.B == 0 || p.H == 0) return 0;
    return use_tc(p, a->desc.dtype, a->desc.path) ? subq::tc_segment_states_bytes(p) : 0;
}

size_t subq_bwd_workspace_bytes(const subq_bwd_args* a) {
    subq::ScanParams p;
    if (fill_bwd(a, p) != SUBQ_OK) return 0;
    return scan_bwd_ws(p, a->desc.dtype, use_tc_bwd(p, a->desc.dtype, a->desc.path)) + gqa_bytes(p, a->desc.dtype);
}

int subq_fwd(const subq_fwd_args* a) {
    subq::ScanParams p;
    int rc = fill_fwd(a, p);
    if (rc) return rc;
    const bool tc = use_tc(p, a->desc.dtype, a->desc.path);
    if (a->desc.path == SUBQ_PATH_TENSORCORE && !tc)
        return fail(SUBQ_ERR_UNSUPPORTED, "tensor-core path needs bf16/fp16 with head_dim = value_dim = 64");
    const int simt = tc ? SUBQ_PATH_TENSORCORE : fwd_simt_path(p, a->desc.dtype, a->desc.path);
    if (simt < 0)
        return fail(SUBQ_ERR_UNSUPPORTED,
                    "chunked path needs fp32/fp16/bf16, head_dim <= 256, forward time and no decay fallback");
    const int used = tc ? SUBQ_PATH_TENSORCORE : simt;
    if (p.B == 0 || p.H == 0) {
        g_last_path = used;
        g_last_launches = 0;
        return SUBQ_OK;
    }
    cudaStream_t st = static_cast<cudaStream_t>(a->stream);
    cudaError_t err;
    int launches = 0;
    if (p.seg_out) {  // "not written" until the tensor-core kernel stamps its segment count
        err = cudaMemsetAsync(p.seg_out, 0, 256, st);
        if (err != cudaSuccess) return fail_cuda(err, "subq_fwd segment_states header");
        if (!tc) p.seg_out = nullptr;
    }
    if (tc) {
        const size_t need = subq::tc_fwd_workspace_bytes(p);
        if ((rc = check_workspace(a->workspace, a->workspace_bytes, need))) return rc;
        p.ws = static_cast<float*>(a->workspace);
        err = subq::launch_fwd_tc(p, a->desc.dtype, st, &launches);
    } else if (used == SUBQ_PATH_CHUNKED) {
        const size_t need = subq::chunk_fwd_workspace_bytes(p);
        if ((rc = check_workspace(a->workspace, a->workspace_bytes, need))) return rc;
        p.ws = static_cast<float*>(a->workspace);
        err = subq::launch_fwd_chunk(p, a->desc.dtype, st, &launches);
    } else {
        err = subq::launch_fwd_exact(p, a->desc.dtype, st);
        launches = 1;
    }
    if (err != cudaSuccess) return fail_cuda(err, "subq_fwd launch");
    g_last_path = used;
    g_last_launches = launches;
    return SUBQ_OK;
}

int subq_bwd(const subq_bwd_args* a) {
    subq::ScanParams p;
    int rc = fill_bwd(a, p);
    if (rc) return rc;
    const bool tc = use_tc_bwd(p, a->desc.dtype, a->desc.path);
    if (a->desc.path == SUBQ_PATH_TENSORCORE && !tc)
        return fail(SUBQ_ERR_UNSUPPORTED, "tensor-core path needs bf16/fp16 with head_dim = value_dim = 64");
    if (!tc && subq::exact_bwd_smem_bytes(p.d, p.e, p.normalize, a->desc.dtype == SUBQ_FP64 ? 8 : 4) > 220 * 1024)
        return fail(SUBQ_ERR_UNSUPPORTED, "backward state d x (e+1) does not fit in shared memory");
    if (p.B == 0 || p.H == 0 || p.N == 0) {
        g_last_path = tc ? SUBQ_PATH_TENSORCORE : SUBQ_PATH_EXACT;
        g_last_launches = 0;
        return SUBQ_OK;
    }
    cudaStream_t st = static_cast<cudaStream_t>(a->stream);
    cudaError_t err;
    int launches = 0;
    const size_t scan_need = scan_bwd_ws(p, a->desc.dtype, tc);
    const size_t need = scan_need + gqa_bytes(p, a->desc.dtype);
    if ((rc = check_workspace(a->workspace, a->workspace_bytes, need))) return rc;
    p.ws = static_cast<float*>(a->workspace);
    if (p.kvg > 1) {  // per-query-head dk, dv into the workspace; summed per group below
        char* base = static_cast<char*>(a->workspace) + scan_need;
        p.dk = base;
        p.dk_sn = p.d, p.dk_sh = (int64_t)p.N * p.d, p.dk_sb = p.dk_sh * p.H;
        p.dv = base + gqa_dk_bytes(p, a->desc.dtype);
        p.dv_sn = p.e, p.dv_sh = (int64_t)p.N * p.e, p.dv_sb = p.dv_sh * p.H;
    }
    if (tc && subq::bwd1_usable(p)) {  // one pass from the forward's handover
        err = subq::launch_bwd1(p, a->desc.dtype, st, &launches);
    } else if (tc) {
        err = subq::launch_bwd_tc(p, a->desc.dtype, st, &launches);
    } else {
        err = subq::launch_bwd_exact(p, a->desc.dtype, st);
        launches = 1;
    }
    if (err == cudaSuccess && p.kvg > 1) {
        const int Hkv = p.H / p.kvg;
        err = subq::launch_group_sum(p.dk, a->dk.data, a->desc.dtype, p.B, Hkv, p.kvg, p.N, p.d, a->dk.stride_b,
                                     a->dk.stride_h, a->dk.stride_n, st);
        if (err == cudaSuccess)
            err = subq::launch_group_sum(p.dv, a->dv.data, a->desc.dtype, p.B, Hkv, p.kvg, p.N, p.e, a->dv.stride_b,
                                         a->dv.stride_h, a->dv.stride_n, st);
        launches += 2;
    }
    if (err != cudaSuccess) return fail_cuda(err, "subq_bwd launch");
    g_last_path = tc ? SUBQ_PATH_TENSORCORE : SUBQ_PATH_EXACT;
    g_last_launches = launches;
    return SUBQ_OK;
}

int subq_feature_map(void* x, int64_t n, int32_t dtype, void* stream) {
    if (n < 0) return fail(SUBQ_ERR_INVALID_ARGUMENT, "negative element count");
    if (n > 0 && !x) return fail(SUBQ_ERR_INVALID_ARGUMENT, "x is null");
    if (dtype != SUBQ_FP32 && dtype != SUBQ_FP16 && dtype != SUBQ_BF16)
        return fail(SUBQ_ERR_INVALID_ARGUMENT, "subq_feature_map supports float32, float16 and bfloat16");
    cudaError_t err = subq::launch_feature_map(x, n, dtype, static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return fail_cuda(err, "subq_feature_map launch");
    g_last_launches = n > 0 ? 1 : 0;
    return SUBQ_OK;
}

// Checks of a per-head RMSNorm call; fills p. Rows must be 16-byte aligned
// (the kernels move 8 elements per thread).
static int fill_rms(const subq_rmsnorm_args* a, subq::RmsParams& p, bool bwd) {
    if (!a) return fail(SUBQ_ERR_INVALID_ARGUMENT, "null argument block");
    if (a->batch < 0 || a->heads < 0 || a->seq_len < 0 || a->head_dim <= 0)
        return fail(SUBQ_ERR_INVALID_ARGUMENT, "negative batch, heads or seq_len, or head_dim <= 0");
    if (a->batch > 65535 || a->heads > 65535 || a->seq_len > (int64_t)1 << 30)
        return fail(SUBQ_ERR_INVALID_ARGUMENT, "batch/heads above 65535 or seq_len above 2^30");
    if (a->dtype != SUBQ_FP32 && a->dtype != SUBQ_FP16 && a->dtype != SUBQ_BF16)
        return fail(SUBQ_ERR_INVALID_ARGUMENT, "head RMSNorm supports float32, float16 and bfloat16");
    if (!subq::rms_supported_dim((int)a->head_dim))
        return fail(SUBQ_ERR_UNSUPPORTED, "head RMSNorm needs head_dim 8, 16, 32, 64, 128 or 256");
    if (!(a->eps >= 0.f) || a->eps > 1e30f) return fail(SUBQ_ERR_INVALID_ARGUMENT, "eps must be >= 0 and finite");
    p = subq::RmsParams{};
    p.B = (int)a->batch; p.H = (int)a->heads; p.N = (int)a->seq_len; p.D = (int)a->head_dim;
    p.eps = a->eps;
    p.w = a->weight;
    const bool empty = p.B == 0 || p.H == 0 || p.N == 0;
    const size_t es = elem_size(a->dtype);
    auto rows_aligned = [&](const subq_tensor4& t, const char* name) {
        int rc = check_tensor(t, name, a->dtype, empty);
        if (rc) return rc;
        if (reinterpret_cast<uintptr_t>(t.data) % 16 != 0 || (t.stride_b * es) % 16 != 0 ||
            (t.stride_h * es) % 16 != 0 || (t.stride_n * es) % 16 != 0)
            return fail(SUBQ_ERR_INVALID_ARGUMENT, std::string(name) + ": rows must start on 16-byte boundaries");
        return (int)SUBQ_OK;
    };
    int rc = rows_aligned(a->x, "x");
    if (rc) return rc;
    p.x = a->x.data; p.x_sb = a->x.stride_b; p.x_sh = a->x.stride_h; p.x_sn = a->x.stride_n;
    if (!bwd) {
        if ((rc = rows_aligned(a->y, "y"))) return rc;
        p.y = a->y.data; p.y_sb = a->y.stride_b; p.y_sh = a->y.stride_h; p.y_sn = a->y.stride_n;
    } else {
        if ((rc = rows_aligned(a->dy, "dy")) || (rc = rows_aligned(a->dx, "dx"))) return rc;
        p.dy = a->dy.data; p.dy_sb = a->dy.stride_b; p.dy_sh = a->dy.stride_h; p.dy_sn = a->dy.stride_n;
        p.dx = a->dx.data; p.dx_sb = a->dx.stride_b; p.dx_sh = a->dx.stride_h; p.dx_sn = a->dx.stride_n;
        p.dw = a->dweight;
    }
    // dense (b, n, h) row order: row r at element r * D
    const int64_t D = p.D, H = p.H, N = p.N;
    auto dense = [&](const subq_tensor4& t) {
        return t.stride_h == D && t.stride_n == H * D && (t.stride_b == N * H * D || p.B == 1);
    };
    p.dense = (dense(a->x) ? 1 : 0) | (!bwd && dense(a->y) ? 2 : 0) | (bwd && dense(a->dy) ? 4 : 0) |
              (bwd && dense(a->dx) ? 8 : 0);
    return SUBQ_OK;
}

size_t subq_head_rmsnorm_bwd_workspace_bytes(const subq_rmsnorm_args* a) {
    subq::RmsParams p;
    if (fill_rms(a, p, true) != SUBQ_OK || !a->dweight) return 0;
    return align_up((size_t)subq::rms_blocks(p) * p.D * sizeof(float));
}

int subq_head_rmsnorm_fwd(const subq_rmsnorm_args* a) {
    subq::RmsParams p;
    int rc = fill_rms(a, p, false);
    if (rc) return rc;
    g_last_launches = 0;
    if (p.B == 0 || p.H == 0 || p.N == 0) return SUBQ_OK;
    cudaError_t err = subq::launch_rms_fwd(p, a->dtype, static_cast<cudaStream_t>(a->stream));
    if (err != cudaSuccess) return fail_cuda(err, "subq_head_rmsnorm_fwd launch");
    g_last_launches = 1;
    return SUBQ_OK;
}

int subq_head_rmsnorm_bwd(const subq_rmsnorm_args* a) {
    subq::RmsParams p;
    int rc = fill_rms(a, p, true);
    if (rc) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(a->stream);
    g_last_launches = 0;
    if (p.B == 0 || p.H == 0 || p.N == 0) {  // no rows: dweight is 0
        if (p.dw) {
            cudaError_t err = cudaMemsetAsync(p.dw, 0, sizeof(float) * p.D, st);
            if (err != cudaSuccess) return fail_cuda(err, "subq_head_rmsnorm_bwd dweight");
        }
        return SUBQ_OK;
    }
    if (p.dw) {
        const size_t need = (size_t)subq::rms_blocks(p) * p.D * sizeof(float);
        if ((rc = check_workspace(a->workspace, a->workspace_bytes, need))) return rc;
        p.part = static_cast<float*>(a->workspace);
    }
    cudaError_t err = subq::launch_rms_bwd(p, a->dtype, st);
    if (err != cudaSuccess) return fail_cuda(err, "subq_head_rmsnorm_bwd launch");
    g_last_launches = p.dw ? 2 : 1;
    return SUBQ_OK;
}

int subq_device_info(int device, char* arch, size_t arch_len, size_t* memory_bytes, int* bf16_supported) {
    cudaDeviceProp prop;
    cudaError_t err = cudaGetDeviceProperties(&prop, device);
    if (err != cudaSuccess) return fail_cuda(err, "cudaGetDeviceProperties");
    if (arch && arch_len) snprintf(arch, arch_len, "SM %d.%d", prop.major, prop.minor);
    if (memory_bytes) *memory_bytes = prop.totalGlobalMem;
    if (bf16_supported) *bf16_supported = prop.major >= 8 ? 1 : 0;
    return SUBQ_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free backward (subq_bwd_noalloc).
//
// Some callers cannot hand the library any device memory for scratch: a
// real-time audio callback must not block on, or fail in, an allocator in the
// middle of a frame, and a host that owns a fixed device budget (a pool sized
// up front) may not grow it per call. For them the backward runs with a
// scratch buffer that is part of this library's static device memory, placed
// when the module loads, so the call itself allocates nothing.
//
//  * Capacity: kNoAllocScratchBytes = 8 MiB against subq_bwd_workspace_bytes:
//    1,048,576 token-heads (B x H x N) on the recomputing tensor-core path (8
//    bytes each), about 699,000 with per-token decay (12 bytes each plus a
//    flag per sequence) and on the float32 exact path (12 bytes each), about
//    349,000 on the float64 exact path (24 bytes each); the one-pass backward
//    (given the forward's handover) takes a fixed 16.6 KB per SM whatever the
//    length; grouped K/V adds dK and dV per query head. A larger call is
//    rejected with SUBQ_ERR_WORKSPACE before anything is launched.
//  * Nothing in the scratch has to start at zero when the call begins: every
//    call writes each per-token entry it later reads (the clamped normaliser
//    and the quotient coefficient, the exact path's per-token values, or the
//    one-pass backward's adjoint sums) before reading it, and the decayed
//    path clears its per-sequence fallback flags itself (a memset on the
//    call's stream, not an allocation).
//  * One buffer per device: calls that overlap in time on one device (two
//    streams, or host threads without ordering between them) race on it, so
//    such callers must serialise their calls.
//  * The first call on a device looks the buffer's address up with
//    cudaGetSymbolAddress while that device is current; make that first call
//    before capturing any stream of the device, so the lookup is not part of
//    a capture.
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kNoAllocMaxDevices] = {};

// Address of this device's scratch; looked up once per device.
int noalloc_scratch(void** out) {
    int dev = -1;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return fail_cuda(err, "subq_bwd_noalloc: cudaGetDevice");
    if (dev < 0 || dev >= kNoAllocMaxDevices)
        return fail(SUBQ_ERR_UNSUPPORTED, "subq_bwd_noalloc: device index above 63");
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void* p = nullptr;
        err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (err != cudaSuccess) return fail_cuda(err, "subq_bwd_noalloc: cudaGetSymbolAddress");
        g_noalloc_ptr[dev] = p;
    }
    *out = g_noalloc_ptr[dev];
    return SUBQ_OK;
}

}  // namespace

extern "C" int subq_bwd_noalloc(const subq_bwd_args* args) {
    if (!args) return fail(SUBQ_ERR_INVALID_ARGUMENT, "args is null");
    const size_t need = subq_bwd_workspace_bytes(args);
    if (need > kNoAllocScratchBytes)
        return fail(SUBQ_ERR_WORKSPACE, "subq_bwd_noalloc: this call needs " + std::to_string(need) +
                                            " bytes of scratch, above the built-in " +
                                            std::to_string(kNoAllocScratchBytes) +
                                            " bytes (8 MiB); use subq_bwd with a caller workspace");
    void* scratch = nullptr;
    int rc = noalloc_scratch(&scratch);
    if (rc) return rc;
    subq_bwd_args a = *args;
    a.workspace = scratch;
    a.workspace_bytes = kNoAllocScratchBytes;
    return subq_bwd(&a);
}
