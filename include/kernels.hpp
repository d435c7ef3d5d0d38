/*
 * subq-b200 — C ABI of the causal ELU+1 linear-attention scan (sm_100a).
 *
 * This header is the drop-in boundary for the reference's kernel layer. Each
 * entry point replaces one reference interface (paths relative to the
 * reference tree):
 *
 *   subq_fwd            run_attention_forward(AttentionContext&)         include/attention.hpp:23-24
 *                       run_attention_forward_raw<T>(...) (declared only)  include/kernels.hpp:56-61
 *                       the torch chunked forward chunkwise_flash_linear_attention /
 *                       _single_direction_causal_scan                    python/subq_audio/autograd.py:292-438
 *   subq_bwd            subquadratic_attention_backward<T>,
 *                       run_attention_backward_raw<T>                    include/kernels.hpp:44-54
 *                       run_attention_backward_ex(...)                   include/attention.hpp:26-32
 *                       _single_direction_causal_backward                python/subq_audio/autograd.py:441-544
 *   subq_feature_map    run_feature_map(TensorDescriptor&)               include/attention.hpp:22
 *   subq_head_rmsnorm_fwd / _bwd
 *                       SubQLinearAttention's per-head nn.RMSNorm and the
 *                       transpose copy after it                          python/subq_audio/autograd.py:706-710,763-769
 *   subq_*_workspace_bytes, subq_last_error, subq_abi_version, subq_device_info:
 *                       no single counterpart; they carry the reference's
 *                       scratch allocation (attention_backward.cpp:305-361 allocated
 *                       per call) and its exception text (bindings.cpp:227-231) across
 *                       a C boundary.
 *
 * Conventions
 *   - Every call is stream-ordered on `stream` (a cudaStream_t, NULL = legacy
 *     default stream) and returns a subq_status; nothing throws across the ABI.
 *     subq_last_error() returns the message of the calling thread's last
 *     failing call.
 *   - The library allocates no device memory. Scratch comes from the caller
 *     as `workspace` (query its size with the *_workspace_bytes functions;
 *     256-byte alignment required).
 *   - Tensors are [B, H, N, D] views with element strides for b, h and n; the
 *     innermost dimension must be contiguous. q, k, v, o (and the gradients)
 *     share one dtype. State tensors are always float32.
 *   - Math (per (b,h) sequence, t = 0..N-1, m_t = mask, 1 if no mask):
 *       gamma_t = exp(log_gamma_t) (1 on masked tokens and with SUBQ_DECAY_NONE)
 *       S_t = gamma_t S_{t-1} + (m_t phi(k_t)) (m_t v_t)^T,   z_t = gamma_t z_{t-1} + m_t phi(k_t)
 *       normalize = 0:  o_t = m_t (scale phi(q_t))^T S_t
 *       normalize = 1:  o_t = m_t (scale phi(q_t))^T S_t / max((scale phi(q_t))^T z_t, clamp_min)
 *     with phi(x) = ELU(x) + 1. The reference's C++ engine is normalize = 0,
 *     scale = 1, scalar decay, flush_subnormal = 1; its torch path is
 *     normalize = 1, scale = 1/sqrt(D), clamp_min = 1e-5.
 */
#pragma once

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SUBQ_ABI_VERSION 5

typedef enum subq_status {
    SUBQ_OK = 0,
    SUBQ_ERR_INVALID_ARGUMENT = 1, /* shapes, strides, null pointers, alignment  */
    SUBQ_ERR_ALIAS = 2,            /* gradient outputs alias inputs (reference attention_backward.cpp:51-56) */
    SUBQ_ERR_UNSUPPORTED = 3,      /* a shape/dtype combination no kernel covers  */
    SUBQ_ERR_CUDA = 4,             /* a CUDA runtime error (message has the text) */
    SUBQ_ERR_TIMEOUT = 5,          /* a bounded device-side wait gave up          */
    SUBQ_ERR_WORKSPACE = 6,        /* workspace missing, too small or misaligned  */
    SUBQ_ERR_STATE = 7             /* device status: a backward's segment_states was not
                                      filled by the forward of the same call          */
} subq_status;

/* Same order as the reference's PrecisionMode (include/tensor.hpp:14-18);
 * SUBQ_FP64 (float64 storage and accumulation, exact path only) is an
 * addition for float64 gradient checks. */
typedef enum subq_dtype { SUBQ_FP32 = 0, SUBQ_FP16 = 1, SUBQ_BF16 = 2, SUBQ_FP64 = 3 } subq_dtype;

typedef enum subq_decay_mode {
    SUBQ_DECAY_NONE = 0,      /* gamma == 1                                     */
    SUBQ_DECAY_SCALAR = 1,    /* log_gamma_scalar for every token               */
    SUBQ_DECAY_PER_HEAD = 2,  /* log_gamma[h], float32 [H]                      */
    SUBQ_DECAY_PER_TOKEN = 3  /* log_gamma[(b*H + h)*N + t], float32 [B,H,N]   */
} subq_decay_mode;

/* Which kernel family a call may use. AUTO picks the tensor-core path when
 * the shape allows it (bf16/fp16, d = e = 64; with per-token decay bf16
 * only); otherwise the chunk-parallel float32 forward for calls of at least
 * 64 tokens (d <= 256, forward time, scalar gamma <= 1, at most 4 GiB of
 * workspace), and the exact
 * float32 path for the rest. Calls of at most 16 tokens (streaming decode
 * steps) take the exact, token-recurrent path, which is faster there. The
 * backward has no chunked variant: CHUNKED runs it on the exact path. */
typedef enum subq_kernel_path {
    SUBQ_PATH_AUTO = 0,
    SUBQ_PATH_EXACT = 1,       /* SIMT float32 sequential scan, any d, e <= 256          */
    SUBQ_PATH_TENSORCORE = 2,  /* tcgen05 chunked scan, bf16/fp16, d = e = 64            */
    SUBQ_PATH_CHUNKED = 3      /* SIMT float32 chunk-parallel forward, d <= 256, no reverse */
} subq_kernel_path;

typedef struct subq_tensor4 {
    void* data;
    int64_t stride_b, stride_h, stride_n; /* element strides; d is contiguous */
} subq_tensor4;

typedef struct subq_scan_desc {
    int64_t batch, heads, seq_len, head_dim, value_dim;
    int32_t dtype;           /* subq_dtype of q, k, v, o and of the gradients */
    int32_t normalize;       /* 0: engine form, 1: normalised form            */
    float scale;             /* multiplies phi(q)                             */
    float clamp_min;         /* lower clamp of the denominator                */
    int32_t decay_mode;      /* subq_decay_mode                               */
    float log_gamma_scalar;  /* SUBQ_DECAY_SCALAR                             */
    const float* log_gamma;  /* SUBQ_DECAY_PER_HEAD / SUBQ_DECAY_PER_TOKEN    */
    const uint8_t* mask;     /* [B, N] (row stride mask_stride_b), nonzero = live; NULL = all live */
    int64_t mask_stride_b;
    int32_t flush_subnormal; /* flush |S| < FLT_MIN to 0 after every update   */
    int32_t path;            /* subq_kernel_path                              */
    /* Grouped K/V (GQA, python/subq_audio/autograd.py:746-748): 0 or `heads`
     * = one K/V head per query head; else a divisor of `heads`, and query
     * head h reads K/V head h / (heads / kv_heads). k, v (and dk, dv) then
     * have kv_heads heads; the backward's dk, dv sum over each group, as the
     * reference's repeat_interleave does under autograd. The state S, z and
     * log gamma stay per query head. */
    int64_t kv_heads;
    /* 1: reverse time - token t sees itself and the later tokens, with the
     * decay of tokens t..tau-1 between key tau and query t: the second
     * direction of the bidirectional scan (python/subq_audio/autograd.py:
     * 407-433, which runs it on time-flipped copies). The caller combines the
     * two directions. The state runs from the end of the sequence. */
    int32_t reverse;
} subq_scan_desc;

typedef struct subq_fwd_args {
    subq_scan_desc desc;
    subq_tensor4 q, k, v, o;
    const float* state_in;  /* S [B,H,d,e] float32, NULL = zeros                 */
    const float* norm_in;   /* z [B,H,d] float32, NULL = zeros (normalize = 1)   */
    float* state_out;       /* final S, may equal state_in, NULL = not wanted    */
    float* norm_out;        /* final z, may equal norm_in, NULL = not wanted     */
    void* workspace;
    size_t workspace_bytes;
    void* stream;           /* cudaStream_t */
    /* Optional (NULL = not wanted): receives the state at the start of each
     * segment of each sequence as the tensor-core forward computes it,
     * subq_segment_states_bytes(args) bytes. Passing the same buffer to the
     * backward of the same call spares it recomputing those states (the
     * reference's backward recomputes them, autograd.py:207-222). */
    float* segment_states;
} subq_fwd_args;

typedef struct subq_bwd_args {
    subq_scan_desc desc;
    subq_tensor4 q, k, v, dout; /* inputs of the forward and the upstream gradient */
    subq_tensor4 dq, dk, dv;    /* outputs; must not alias q, k, v or dout          */
    const float* state_in;      /* the forward's initial S (NULL = zeros)           */
    const float* norm_in;       /* the forward's initial z (NULL = zeros)           */
    float* dlog_gamma;          /* [B,H,N] float32 d loss / d log(gamma_t), or NULL */
    void* workspace;
    size_t workspace_bytes;
    void* stream;
    /* Optional: the segment_states buffer the forward of the same inputs
     * filled. Alone, it is used when it matches this call's segment split and
     * ignored otherwise. */
    const float* segment_states;
    /* Optional (ABI 4): the forward's output o of the same call. Given with
     * segment_states on the tensor-core path without decay, the backward runs
     * in one pass from what that forward handed over (its per-chunk states and
     * normalisers) instead of recomputing them; the buffer must then come from
     * that very forward, else no gradient is written and subq_device_status
     * reports SUBQ_ERR_STATE. */
    subq_tensor4 out;
} subq_bwd_args;

/* Forward scan. Replaces run_attention_forward / the torch chunked forward. */
int subq_fwd(const subq_fwd_args* args);

/* Backward scan (recomputes the forward; saves nothing between calls).
 * Replaces subquadratic_attention_backward / _single_direction_causal_backward. */
int subq_bwd(const subq_bwd_args* args);

/* Bytes of `workspace` the call needs (0 is possible). */
size_t subq_fwd_workspace_bytes(const subq_fwd_args* args);
size_t subq_bwd_workspace_bytes(const subq_bwd_args* args);
/* Bytes of the forward's optional segment_states buffer (0: the call would
 * not fill one, e.g. on the exact path). */
size_t subq_segment_states_bytes(const subq_fwd_args* args);

/* In-place phi(x) = ELU(x) + 1 over n contiguous elements (run_feature_map). */
int subq_feature_map(void* x, int64_t n, int32_t dtype, void* stream);

/* Per-head RMSNorm of the scan's output, y = x * rsqrt(mean_D(x^2) + eps) * w
 * over each row of D values (one token of one head): SubQLinearAttention's
 * nn.RMSNorm(head_dim, eps=1e-5) and the [B, H, L, D] -> [B, L, H*D] copy
 * after it (reference python/subq_audio/autograd.py:706-710, 763-769); y is
 * written through its own strides, so giving it the [B, L, H, D] layout
 * replaces the copy. Math in float32 whatever the dtype (fp32, fp16 or bf16).
 * x, y, dy and dx are [B, H, N, D] views with element strides; D is 8, 16,
 * 32, 64, 128 or 256 (SUBQ_ERR_UNSUPPORTED otherwise); every row starts on a
 * 16-byte boundary (data and strides). The backward reads x and dy and writes
 *   dx = r (dy w - xh mean_D(dy w xh)),  xh = x r,  r = rsqrt(mean_D(x^2) + eps)
 * and, when `dweight` is given, dweight = sum over rows of dy xh (written,
 * not accumulated; bitwise reproducible), which needs `workspace` of
 * subq_head_rmsnorm_bwd_workspace_bytes. dx may be x or dy (in place). */
typedef struct subq_rmsnorm_args {
    int64_t batch, heads, seq_len, head_dim;
    int32_t dtype;
    float eps;
    subq_tensor4 x, y;      /* forward: input and output (the backward reads x) */
    subq_tensor4 dy, dx;    /* backward: upstream gradient and input gradient */
    const float* weight;    /* [D] float32, or NULL for a weight of 1 */
    float* dweight;         /* backward: [D] float32, or NULL */
    void* workspace;
    size_t workspace_bytes;
    void* stream;
} subq_rmsnorm_args;

int subq_head_rmsnorm_fwd(const subq_rmsnorm_args* args);
int subq_head_rmsnorm_bwd(const subq_rmsnorm_args* args);
size_t subq_head_rmsnorm_bwd_workspace_bytes(const subq_rmsnorm_args* args);

/* Backward scan with no allocation and no caller workspace (no counterpart in
 * the reference, whose backward allocates its scratch on every call). For
 * callers that may not supply or grow device memory per call, such as a
 * real-time audio callback or a host with a fixed device budget: the scratch
 * is a static 8 MiB device buffer of the library. A call fits when
 * subq_bwd_workspace_bytes(args) <= 8 MiB: the recomputing tensor-core path
 * takes 8 bytes per token-head (B x H x N; 1,048,576 token-heads), 12 with
 * per-token decay (plus 4 bytes per sequence) and on the float32 exact path
 * (699,050), 24 on the float64 exact path (349,525); the one-pass backward
 * (segment_states and out given) takes a fixed 16.6 KB per SM (about 2.5 MB on
 * a B200) whatever the length; grouped K/V adds dK and dV per query head.
 * Larger calls return SUBQ_ERR_WORKSPACE. `workspace` and `workspace_bytes` of
 * args are ignored. Nothing in the buffer needs to start at zero (what must,
 * the call clears itself). There is one buffer per device, so calls that
 * overlap in time on one device race: serialise them. The first call on a
 * device looks the buffer up with that device current; make it before
 * capturing any of the device's streams. Results equal subq_bwd's. */
int subq_bwd_noalloc(const subq_bwd_args* args);

/* Reads and clears (in one atomic step, ordered on `stream`) the device status
 * word of the current device, then synchronises `stream`: SUBQ_OK, or
 * SUBQ_ERR_TIMEOUT when a bounded device-side wait of a tensor-core kernel gave
 * up since the last query, or SUBQ_ERR_STATE when a backward was given the
 * segment_states of another call's forward (the outputs are then not valid).
 * Returns SUBQ_ERR_CUDA if the launch or the synchronisation fails. */
int subq_device_status(void* stream, int* status);

/* Diagnostic (no counterpart in the reference): launches one block whose
 * bounded device-side wait - the one every tensor-core kernel uses on its
 * pipeline barriers - waits on a barrier that nothing arrives at, with its
 * limit shortened to `polls` (1..2^20) polls. It gives up and records
 * SUBQ_ERR_TIMEOUT in the device status word, as a stalled kernel would, so
 * that a caller can test its handling of subq_device_status without a fault. */
int subq_selftest_wait_timeout(int polls, void* stream);

/* Kernel path the last successful subq_fwd / subq_bwd of this thread ran. */
int subq_last_path(void);

/* Number of device kernels the last successful call of this thread launched. */
int subq_last_launches(void);

/* Message of this thread's last failing call ("" if none). */
const char* subq_last_error(void);

int subq_abi_version(void);

/* Device description for get_device_info (reference python/bindings.cpp:37-65).
 * `arch` receives e.g. "SM 10.0" (NUL-terminated, at most arch_len bytes). */
int subq_device_info(int device, char* arch, size_t arch_len, size_t* memory_bytes,
                     int* bf16_supported);

#ifdef __cplusplus
} /* extern "C" */
#endif
