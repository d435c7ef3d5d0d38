// Host-side plumbing of the tensor-core path: shape support checks, TMA
// tensor maps, segment (cluster size) choice, cluster launches and the
// device status word. The kernels live in scan_tc_fwd.cu / scan_tc_bwd.cu.
#include "tc_common.cuh"

#include <algorithm>
#include <map>
#include <mutex>
#include <tuple>

namespace subq {

// First error code raised by a bounded device-side wait of the tensor-core
// kernels (SUBQ_ERR_TIMEOUT) or by a backward given another call's forward
// handover (SUBQ_ERR_STATE); read and cleared by subq_device_status.
__device__ int g_tc_status;
// Where the read-and-clear kernel leaves the value it took.
__device__ int g_tc_status_taken;

namespace tcs {

// Device address of the status word, looked up once per device (on the
// device's first tensor-core launch or status query) under a lock.
int* status_ptr() {
    static std::mutex mu;
    static int* ptrs[64] = {nullptr};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lock(mu);
    if (!ptrs[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_tc_status) != cudaSuccess) return nullptr;
        ptrs[dev] = static_cast<int*>(p);
    }
    return ptrs[dev];
}

namespace {
// Takes the status word and clears it in one atomic step (a timeout recorded
// by a kernel on another stream is not lost between a read and a clear).
__global__ void status_take_kernel() { g_tc_status_taken = atomicExch(&g_tc_status, 0); }

// Diagnostic: one bounded wait on a barrier that nothing arrives at, with the
// limit shortened to `polls`; it gives up and records SUBQ_ERR_TIMEOUT.
__global__ void wait_timeout_kernel(int polls) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        tc::mbar_init(&bar, 1);
        tc::fence_mbar_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        bool done = false;
        for (int i = 0; i < polls && !done; ++i) done = tc::mbar_test_wait(&bar, 0);
        if (!done) atomicCAS(&g_tc_status, 0, (int)SUBQ_ERR_TIMEOUT);
    }
}
}  // namespace

cudaError_t launch_fwd_v2(const ScanParams& p, int dtype, cudaStream_t st);
int fwd_segment_count(const ScanParams& p);
cudaError_t launch_bwd_v2(const ScanParams& p, int dtype, cudaStream_t st);

namespace {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(ptr);
    }
    return fn;
}

// TMA needs a 16-byte aligned base and strides that are multiples of 16 bytes.
bool strides_ok(int64_t sb, int64_t sh, int64_t sn, const void* ptr) {
    return (reinterpret_cast<uintptr_t>(ptr) % 16 == 0) && sn % 8 == 0 && sh % 8 == 0 && sb % 8 == 0 && sn >= kD &&
           sn * 2 < ((int64_t)1 << 40) && sh * 2 < ((int64_t)1 << 40) && sb * 2 < ((int64_t)1 << 40);
}

}  // namespace

// [B, H, N, 64] 16-bit tensor, box of 64 x 128 tokens, 128-byte swizzle.
bool make_map(CUtensorMap* m, const void* base, int dtype, int N, int H, int B, int64_t sn, int64_t sh, int64_t sb) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return false;
    if (H == 1) sh = sn * (int64_t)(N > 0 ? N : 1);
    if (B == 1) sb = sh * H;
    cuuint64_t dims[4] = {(cuuint64_t)kD, (cuuint64_t)N, (cuuint64_t)H, (cuuint64_t)B};
    cuuint64_t strides[3] = {(cuuint64_t)sn * 2, (cuuint64_t)sh * 2, (cuuint64_t)sb * 2};
    cuuint32_t box[4] = {(cuuint32_t)kD, (cuuint32_t)kC, 1, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = enc(m, dtype == SUBQ_FP16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4,
                     const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// Clusters of G CTAs of `kern` that the device holds at once (cached per
// device, kernel and G; a cluster must fit in one GPC, so this is below
// SMs / G when G does not divide a GPC's SM count).
static int max_active_clusters(const void* kern, int G, int threads, size_t smem) {
    static std::mutex mu;
    static std::map<std::tuple<int, const void*, int>, int> cache;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    const auto key = std::make_tuple(dev, kern, G);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
    int n = 0;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) == cudaSuccess) {
        cudaLaunchConfig_t cfg;
        memset(&cfg, 0, sizeof(cfg));
        cfg.gridDim = dim3(G, 1, 1);
        cfg.blockDim = dim3(threads, 1, 1);
        cfg.dynamicSmemBytes = smem;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = G;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) n = 0;
    }
    cudaGetLastError();  // a failed query leaves no sticky error behind
    cache[key] = n;
    return n;
}

// Segments (CTAs of one cluster) per sequence: the largest G <= 8 (and <= the
// chunk count) for which every sequence's cluster is resident at once, so the
// grid runs in one wave; G = 1 when even single CTAs need more than one wave.
int pick_segments(const ScanParams& p, const void* kern, int threads, size_t smem) {
    const int nC = (p.N + kC - 1) / kC;
    const int bh = p.B * p.H;
    for (int G = std::min(8, nC); G > 1; --G)
        if (bh <= max_active_clusters(kern, G, threads, smem)) return G;
    return 1;
}

cudaError_t launch_cluster(const void* kern, int G, int BH, int threads, size_t smem, cudaStream_t st, void** args) {
    cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (err != cudaSuccess) return err;
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3(G, BH, 1);
    cfg.blockDim = dim3(threads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = G;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelExC(&cfg, kern, args);
}

}  // namespace tcs

bool tc_supported(const ScanParams& p, int dtype) {
    using namespace tcs;
    if (dtype != SUBQ_BF16 && dtype != SUBQ_FP16) return false;
    if (p.d != kD || p.e != kD || p.N < 1) return false;
    if (p.flush) return false;
    if (p.reverse && !p.normalize) return false;  // reverse time: the normalised form (the module's)
    // per-token decay runs factorised through the chunk midpoint, which needs
    // bf16's exponent range (fp16 decayed scans take the exact path)
    if (p.decay_mode != SUBQ_DECAY_NONE && dtype != SUBQ_BF16) return false;
    if (!(p.scale > 0.f)) return false;  // phi'(q) is recovered from scale * phi(q)
    if (p.B * p.H > 65535) return false;
    return strides_ok(p.q_sb, p.q_sh, p.q_sn, p.q) && strides_ok(p.k_sb, p.k_sh, p.k_sn, p.k) &&
           strides_ok(p.v_sb, p.v_sh, p.v_sn, p.v) && strides_ok(p.o_sb, p.o_sh, p.o_sn, p.o) && encode_fn() != nullptr;
}

bool tc_bwd_supported(const ScanParams& p, int) {
    using namespace tcs;
    // d log(gamma) comes with the decayed kernels only (without decay it is not defined)
    if (p.dlg != nullptr && p.decay_mode == SUBQ_DECAY_NONE) return false;
    // (with grouped K/V the kernel writes dk, dv into contiguous workspace buffers)
    return strides_ok(p.g_sb, p.g_sh, p.g_sn, p.g) &&
           (p.kvg > 1 || (strides_ok(p.dk_sb, p.dk_sh, p.dk_sn, p.dk) && strides_ok(p.dv_sb, p.dv_sh, p.dv_sn, p.dv)));
}

static size_t align256(size_t x) { return (x + 255) / 256 * 256; }

// With decay: the per-sequence fallback flags.
size_t tc_fwd_workspace_bytes(const ScanParams& p) {
    return p.decay_mode == SUBQ_DECAY_NONE ? 0 : align256((size_t)p.B * p.H * sizeof(int));
}

// (Zc_t, c_t) per token, written by the backward's dQ pass and read by its dK/dV pass;
// with decay also s q~ . dQ~ per token (12 bytes per token, which also holds the
// exact kernel's three floats per token of a sequence it takes over), then the
// per-sequence fallback flags.
static size_t tc_bwd_token_bytes(const ScanParams& p) {
    const size_t per = p.decay_mode == SUBQ_DECAY_NONE ? sizeof(float2) : 3 * sizeof(float);
    return align256((size_t)p.B * p.H * (size_t)p.N * per);
}

size_t tc_bwd_workspace_bytes(const ScanParams& p) {
    const size_t flags = p.decay_mode == SUBQ_DECAY_NONE ? 0 : align256((size_t)p.B * p.H * sizeof(int));
    return tc_bwd_token_bytes(p) + flags;
}

// The forward -> backward handover (tc_common.cuh HandLayout): segment-start
// states, live-chunk plan and, without decay, the per-chunk state operands
// and per-token normalisers of the one-pass backward.
size_t tc_segment_states_bytes(const ScanParams& p) {
    const int G = tcs::fwd_segment_count(p);
    return tcs::HandLayout(p.B * p.H, p.N, G, p.decay_mode == SUBQ_DECAY_NONE).total;
}

cudaError_t launch_fwd_tc(const ScanParams& p, int dtype, cudaStream_t st, int* launches) {
    *launches = 1;
    if (p.decay_mode == SUBQ_DECAY_NONE) return tcs::launch_fwd_v2(p, dtype, st);
    // decayed: the tensor-core kernel flags the sequences whose decay leaves its
    // range; the exact kernel then recomputes exactly those
    ScanParams q = p;
    q.fallback = reinterpret_cast<int*>(p.ws);
    cudaError_t err = cudaMemsetAsync(q.fallback, 0, (size_t)p.B * p.H * sizeof(int), st);
    if (err == cudaSuccess) err = tcs::launch_fwd_v2(q, dtype, st);
    if (err == cudaSuccess) err = launch_fwd_exact(q, dtype, st);
    *launches = 2;
    return err;
}

cudaError_t launch_bwd_tc(const ScanParams& p, int dtype, cudaStream_t st, int* launches) {
    *launches = 1;
    if (p.decay_mode == SUBQ_DECAY_NONE) return tcs::launch_bwd_v2(p, dtype, st);
    ScanParams q = p;
    q.fallback = reinterpret_cast<int*>(reinterpret_cast<char*>(p.ws) + tc_bwd_token_bytes(p));
    cudaError_t err = cudaMemsetAsync(q.fallback, 0, (size_t)p.B * p.H * sizeof(int), st);
    if (err == cudaSuccess) err = tcs::launch_bwd_v2(q, dtype, st);
    if (err == cudaSuccess) err = launch_bwd_exact(q, dtype, st);
    *launches = 2;
    return err;
}

cudaError_t tc_read_status(cudaStream_t st, int* status) {
    int v = 0;
    tcs::status_take_kernel<<<1, 1, 0, st>>>();
    cudaError_t err = cudaGetLastError();
    if (err == cudaSuccess)
        err = cudaMemcpyFromSymbolAsync(&v, g_tc_status_taken, sizeof(int), 0, cudaMemcpyDeviceToHost, st);
    if (err == cudaSuccess) err = cudaStreamSynchronize(st);
    *status = v;
    return err;
}

cudaError_t tc_selftest_wait_timeout(int polls, cudaStream_t st) {
    tcs::wait_timeout_kernel<<<1, 32, 0, st>>>(polls);
    return cudaGetLastError();
}

}  // namespace subq
