// pybind11 module subq_audio._C: the reference's native Python surface
// (python/bindings.cpp:412-465) over the device-resident engine.
//
// Same class, method and argument names, defaults and error prefixes as the
// reference; forward/backward run on the GPU through the C ABI. Additions:
// `carry_state` / `normalize` keywords, reset_state(), and state accessors.
#include <cuda_runtime.h>
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <mutex>
#include <stdexcept>
#include <string>

#include "arena.hpp"
#include "engine.hpp"
#include "kernels.hpp"
#include "safetensors.hpp"

namespace py = pybind11;

namespace {

void check_cuda(cudaError_t err, const char* what) {
    if (err != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(err));
}

py::dict get_device_info() {
    py::dict info;
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) {
        cudaGetLastError();
        info["backend"] = "CPU";
        info["architecture"] = "Host";
        info["memory_size"] = 0;
        info["bfloat16_supported"] = false;
        return info;
    }
    int dev = 0;
    cudaGetDevice(&dev);
    char arch[32] = {0};
    size_t mem = 0;
    int bf16 = 0;
    subq_device_info(dev, arch, sizeof(arch), &mem, &bf16);
    info["backend"] = "CUDA";
    info["architecture"] = std::string(arch);
    info["memory_size"] = mem;
    info["bfloat16_supported"] = bf16 != 0;
    return info;
}

using F32Array = py::array_t<float, py::array::c_style | py::array::forcecast>;

class SubQEngineWrapper {
public:
    static int prepare_device(int device_id) {
        if (device_id >= 0) {
            cudaError_t err = cudaSetDevice(device_id);
            if (err != cudaSuccess)
                throw std::runtime_error("cudaSetDevice failed for device " + std::to_string(device_id) + ": " +
                                         cudaGetErrorString(err));
        }
        return device_id;
    }

    explicit SubQEngineWrapper(size_t vram_capacity, int device_id)
        : device_id_(prepare_device(device_id)), arena_(vram_capacity), engine_(arena_) {}

    int device_id() const { return device_id_; }

    void load(const std::string& filepath) {
        py::gil_scoped_release nogil;
        std::lock_guard<std::mutex> lock(mu_);
        try {
            set_device();
            SafetensorLoader loader(arena_);
            if (!loader.load(filepath)) throw std::runtime_error("Failed to load safetensors file: " + filepath);
            state_valid_ = false;  // the loader may have moved the arena head past the state
        } catch (const std::exception& e) {
            throw std::runtime_error(std::string("Loader Error: ") + e.what());
        }
    }

    py::array_t<float> forward(F32Array Q, F32Array K, F32Array V, float decay_factor, bool carry_state,
                               bool normalize) {
        py::buffer_info bq = Q.request(), bk = K.request(), bv = V.request();
        try {
            if (bq.ndim != 3 || bk.ndim != 3 || bv.ndim != 3)
                throw std::runtime_error("Number of dimensions must be 3 (batch, seq_len, d_model)");
            const size_t B = bq.shape[0], N = bq.shape[1], D = bq.shape[2];
            if ((size_t)bk.shape[0] != B || (size_t)bk.shape[1] != N || (size_t)bk.shape[2] != D ||
                (size_t)bv.shape[0] != B || (size_t)bv.shape[1] != N || (size_t)bv.shape[2] != D)
                throw std::runtime_error("Shape mismatch between Q, K, V tensors");
            py::array_t<float> out({B, N, D});
            float* host_out = out.mutable_data();
            const float* hq = static_cast<const float*>(bq.ptr);
            const float* hk = static_cast<const float*>(bk.ptr);
            const float* hv = static_cast<const float*>(bv.ptr);
            {
                py::gil_scoped_release nogil;
                std::lock_guard<std::mutex> lock(mu_);
                set_device();
                prepare_state(B, D, normalize, carry_state);
                const size_t saved = arena_.get_offset();
                const size_t avail = arena_.get_total_bytes() > saved ? arena_.get_total_bytes() - saved : 0;
                // four piece buffers, each rounded up to the arena's 256-byte alignment, and
                // the kernels' workspace: at most (64-token pieces + 1) x that of 64 tokens
                const size_t buf_tok = 4 * B * D * sizeof(float);
                const size_t ws64 = N >= 64 ? forward_workspace(B, 64, D, decay_factor, normalize) : 0;
                size_t max_chunk = 0;
                if (buf_tok && ws64 && avail > 5 * 255 + ws64)
                    max_chunk = (avail - 5 * 255 - ws64) / (buf_tok + (ws64 + 63) / 64);
                if (max_chunk < 64)  // too little room for it: pieces without (the exact path)
                    max_chunk = !buf_tok ? 1024 : avail > 4 * 255 ? (avail - 4 * 255) / buf_tok : 0;
                const size_t chunk = std::max<size_t>(1, std::min<size_t>(max_chunk, 16384));
                for (size_t t = 0; t < N; t += chunk) {
                    const size_t cur = std::min(chunk, N - t);
                    arena_.set_offset(saved);
                    const size_t bytes = B * cur * D * sizeof(float);
                    float* dq = reinterpret_cast<float*>(arena_.allocate(bytes));
                    float* dk = reinterpret_cast<float*>(arena_.allocate(bytes));
                    float* dv = reinterpret_cast<float*>(arena_.allocate(bytes));
                    float* dout = reinterpret_cast<float*>(arena_.allocate(bytes));
                    const size_t row = cur * D * sizeof(float), pitch = N * D * sizeof(float);
                    check_cuda(cudaMemcpy2D(dq, row, hq + t * D, pitch, row, B, cudaMemcpyHostToDevice), "H2D Q");
                    check_cuda(cudaMemcpy2D(dk, row, hk + t * D, pitch, row, B, cudaMemcpyHostToDevice), "H2D K");
                    check_cuda(cudaMemcpy2D(dv, row, hv + t * D, pitch, row, B, cudaMemcpyHostToDevice), "H2D V");
                    run_forward(dq, dk, dv, dout, B, cur, D, decay_factor, normalize);
                    check_cuda(cudaMemcpy2D(host_out + t * D, pitch, dout, row, row, B, cudaMemcpyDeviceToHost),
                               "D2H O");
                }
                arena_.set_offset(saved);
                check_cuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
                engine_.check_device();
            }
            return out;
        } catch (const std::exception& e) {
            throw std::runtime_error(std::string("Engine Forward Error: ") + e.what());
        }
    }

    void forward_raw(uintptr_t q_ptr, uintptr_t k_ptr, uintptr_t v_ptr, uintptr_t o_ptr, size_t batch,
                     size_t seq_len, size_t d_model, float decay_factor, bool carry_state, bool normalize) {
        py::gil_scoped_release nogil;
        std::lock_guard<std::mutex> lock(mu_);
        try {
            set_device();
            prepare_state(batch, d_model, normalize, carry_state);
            run_forward(reinterpret_cast<void*>(q_ptr), reinterpret_cast<void*>(k_ptr),
                        reinterpret_cast<void*>(v_ptr), reinterpret_cast<void*>(o_ptr), batch, seq_len, d_model,
                        decay_factor, normalize);
        } catch (const std::exception& e) {
            throw std::runtime_error(std::string("Engine Forward Raw Error: ") + e.what());
        }
    }

    py::tuple backward(F32Array dO, F32Array Q, F32Array K, F32Array V, float decay_factor) {
        py::buffer_info bo = dO.request(), bq = Q.request(), bk = K.request(), bv = V.request();
        try {
            if (bo.ndim != 3 || bq.ndim != 3 || bk.ndim != 3 || bv.ndim != 3)
                throw std::runtime_error("Number of dimensions must be 3 (batch, seq_len, d_model)");
            const size_t B = bq.shape[0], N = bq.shape[1], D = bq.shape[2];
            for (auto* b : {&bo, &bk, &bv})
                if ((size_t)b->shape[0] != B || (size_t)b->shape[1] != N || (size_t)b->shape[2] != D)
                    throw std::runtime_error("Shape mismatch between dO, Q, K, V tensors");
            py::array_t<float> gq({B, N, D}), gk({B, N, D}), gv({B, N, D});
            float* hgq = gq.mutable_data();
            float* hgk = gk.mutable_data();
            float* hgv = gv.mutable_data();
            float d_gamma = 0.f;
            {
                py::gil_scoped_release nogil;
                std::lock_guard<std::mutex> lock(mu_);
                set_device();
                const size_t saved = arena_.get_offset();
                const size_t bytes = B * N * D * sizeof(float);
                try {
                    void* d[7];
                    for (int i = 0; i < 7; ++i) d[i] = arena_.allocate(bytes);
                    check_cuda(cudaMemcpy(d[0], bo.ptr, bytes, cudaMemcpyHostToDevice), "H2D dO");
                    check_cuda(cudaMemcpy(d[1], bq.ptr, bytes, cudaMemcpyHostToDevice), "H2D Q");
                    check_cuda(cudaMemcpy(d[2], bk.ptr, bytes, cudaMemcpyHostToDevice), "H2D K");
                    check_cuda(cudaMemcpy(d[3], bv.ptr, bytes, cudaMemcpyHostToDevice), "H2D V");
                    d_gamma = engine_.backward_engine(d[0], d[1], d[2], d[3], d[4], d[5], d[6], B, N, D,
                                                      decay_factor, nullptr, nullptr);
                    check_cuda(cudaMemcpy(hgq, d[4], bytes, cudaMemcpyDeviceToHost), "D2H dQ");
                    check_cuda(cudaMemcpy(hgk, d[5], bytes, cudaMemcpyDeviceToHost), "D2H dK");
                    check_cuda(cudaMemcpy(hgv, d[6], bytes, cudaMemcpyDeviceToHost), "D2H dV");
                } catch (...) {
                    arena_.set_offset(saved);
                    throw;
                }
                arena_.set_offset(saved);
            }
            return py::make_tuple(gq, gk, gv, d_gamma);
        } catch (const std::exception& e) {
            throw std::runtime_error(std::string("Engine Backward Error: ") + e.what());
        }
    }

    float backward_raw(uintptr_t do_ptr, uintptr_t q_ptr, uintptr_t k_ptr, uintptr_t v_ptr, uintptr_t dq_ptr,
                       uintptr_t dk_ptr, uintptr_t dv_ptr, size_t batch, size_t seq_len, size_t d_model,
                       float decay_factor) {
        py::gil_scoped_release nogil;
        std::lock_guard<std::mutex> lock(mu_);
        try {
            set_device();
            return engine_.backward_engine(
                reinterpret_cast<const void*>(do_ptr), reinterpret_cast<const void*>(q_ptr),
                reinterpret_cast<const void*>(k_ptr), reinterpret_cast<const void*>(v_ptr),
                reinterpret_cast<void*>(dq_ptr), reinterpret_cast<void*>(dk_ptr), reinterpret_cast<void*>(dv_ptr),
                batch, seq_len, d_model, decay_factor, nullptr, nullptr);
        } catch (const std::exception& e) {
            throw std::runtime_error(std::string("Engine Backward Raw Error: ") + e.what());
        }
    }

    void reset_state() {
        py::gil_scoped_release nogil;
        std::lock_guard<std::mutex> lock(mu_);
        state_valid_ = false;
    }

    // Copy of the carried state S [B, D, D] (float32) for inspection.
    py::object state() {
        size_t B, D;
        {
            std::lock_guard<std::mutex> lock(mu_);
            if (!state_valid_) return py::none();
            B = state_B_;
            D = state_D_;
        }
        py::array_t<float> out({B, D, D});
        float* host = out.mutable_data();
        {
            py::gil_scoped_release nogil;
            std::lock_guard<std::mutex> lock(mu_);
            set_device();
            check_cuda(cudaMemcpy(host, S_, B * D * D * sizeof(float), cudaMemcpyDeviceToHost), "D2H state");
        }
        return std::move(out);
    }

private:
    void set_device() {
        if (device_id_ >= 0) check_cuda(cudaSetDevice(device_id_), "cudaSetDevice");
    }

    // The reference resets and zeroes S on every call (python/bindings.cpp:153-161);
    // with carry_state the state of the previous call (same shape) is kept.
    void prepare_state(size_t B, size_t D, bool normalize, bool carry) {
        if (carry && state_valid_ && state_B_ == B && state_D_ == D && state_norm_ == normalize) {
            arena_.set_offset(state_end_);
            return;
        }
        arena_.reset_head();
        S_ = reinterpret_cast<float*>(arena_.allocate(B * D * D * sizeof(float)));
        z_ = reinterpret_cast<float*>(arena_.allocate(B * D * sizeof(float)));
        check_cuda(cudaMemset(S_, 0, B * D * D * sizeof(float)), "cudaMemset state");
        check_cuda(cudaMemset(z_, 0, B * D * sizeof(float)), "cudaMemset state");
        state_end_ = arena_.get_offset();
        state_B_ = B;
        state_D_ = D;
        state_norm_ = normalize;
        state_valid_ = true;
    }

    void run_forward(void* q, void* k, void* v, void* o, size_t B, size_t N, size_t D, float decay_factor,
                     bool normalize) {
        if (!(decay_factor >= 0.f)) throw std::invalid_argument("decay_factor must be a number >= 0");
        engine_.forward(forward_args(q, k, v, o, B, N, D, decay_factor, normalize));
    }

    // Device workspace of a forward over N tokens (0 on the exact path).
    size_t forward_workspace(size_t B, size_t N, size_t D, float decay_factor, bool normalize) {
        void* any = reinterpret_cast<void*>(256);  // the query reads shapes, not data
        subq_fwd_args a = forward_args(any, any, any, any, B, N, D, decay_factor, normalize);
        return subq_fwd_workspace_bytes(&a);
    }

    subq_fwd_args forward_args(void* q, void* k, void* v, void* o, size_t B, size_t N, size_t D,
                               float decay_factor, bool normalize) {
        subq_fwd_args a{};
        a.desc.batch = (int64_t)B;
        a.desc.heads = 1;
        a.desc.seq_len = (int64_t)N;
        a.desc.head_dim = (int64_t)D;
        a.desc.value_dim = (int64_t)D;
        a.desc.dtype = SUBQ_FP32;
        a.desc.normalize = normalize ? 1 : 0;
        a.desc.scale = normalize ? 1.f / std::sqrt((float)D) : 1.f;
        a.desc.clamp_min = 1e-5f;
        a.desc.decay_mode = decay_factor == 1.f ? SUBQ_DECAY_NONE : SUBQ_DECAY_SCALAR;
        a.desc.log_gamma_scalar = std::log(decay_factor);
        a.desc.flush_subnormal = normalize ? 0 : 1;
        a.desc.path = SUBQ_PATH_AUTO;
        auto t3 = [&](void* p) {
            subq_tensor4 t;
            t.data = p;
            t.stride_b = (int64_t)(N * D);
            t.stride_h = 0;
            t.stride_n = (int64_t)D;
            return t;
        };
        a.q = t3(q);
        a.k = t3(k);
        a.v = t3(v);
        a.o = t3(o);
        a.state_in = S_;
        a.state_out = S_;
        if (normalize) {
            a.norm_in = z_;
            a.norm_out = z_;
        }
        return a;
    }

    int device_id_{0};
    std::mutex mu_;
    MemoryArena arena_;
    Engine engine_;
    float* S_ = nullptr;
    float* z_ = nullptr;
    size_t state_B_ = 0, state_D_ = 0, state_end_ = 0;
    bool state_norm_ = false, state_valid_ = false;
};

}  // namespace

PYBIND11_MODULE(_C, m) {
    m.doc() = "Sub-Quadratic Audio Transformer Engine native module (B200, sm_100a)";
    m.def("get_device_info", &get_device_info, "Get hardware info (backend, architecture, memory, bfloat16)");
    m.def("abi_version", []() { return subq_abi_version(); });

    py::class_<SubQEngineWrapper>(m, "SubQEngine")
        .def(py::init<size_t, int>(), py::arg("vram_capacity") = 1024 * 1024 * 32, py::arg("device_id") = 0)
        .def_property_readonly("device_id", &SubQEngineWrapper::device_id, "GPU device of this engine's arena")
        .def("load", &SubQEngineWrapper::load, py::arg("filepath"), "Load weights from a safetensors file")
        .def("forward", &SubQEngineWrapper::forward, py::arg("Q"), py::arg("K"), py::arg("V"),
             py::arg("decay_factor") = 0.99f, py::kw_only(), py::arg("carry_state") = false,
             py::arg("normalize") = false, "Forward causal linear-attention scan on NumPy arrays (runs on the GPU)")
        .def("forward_raw", &SubQEngineWrapper::forward_raw, py::arg("q_ptr"), py::arg("k_ptr"), py::arg("v_ptr"),
             py::arg("o_ptr"), py::arg("batch"), py::arg("seq_len"), py::arg("d_model"),
             py::arg("decay_factor") = 0.99f, py::kw_only(), py::arg("carry_state") = false,
             py::arg("normalize") = false, "Forward scan on float32 device pointers")
        .def("backward", &SubQEngineWrapper::backward, py::arg("dO"), py::arg("Q"), py::arg("K"), py::arg("V"),
             py::arg("decay_factor") = 0.99f, "Backward scan returning (dQ, dK, dV, d_decay)")
        .def("backward_raw", &SubQEngineWrapper::backward_raw, py::arg("do_ptr"), py::arg("q_ptr"),
             py::arg("k_ptr"), py::arg("v_ptr"), py::arg("dq_ptr"), py::arg("dk_ptr"), py::arg("dv_ptr"),
             py::arg("batch"), py::arg("seq_len"), py::arg("d_model"), py::arg("decay_factor") = 0.99f,
             "Backward scan on float32 device pointers returning d_decay")
        .def("reset_state", &SubQEngineWrapper::reset_state, "Forget the carried state")
        .def("state", &SubQEngineWrapper::state, "Copy of the carried state S [B, D, D] (or None)");
}
