// quantmatmul.cu — the QuantMatMul section of include/jv.h on caller-owned device buffers:
// re-tiling GGUF rows and the single-token product (reference
// src/Jevstral/Numerics/QuantMatMul.cs:127-176 and src/Jevstral/Numerics/WeightMatrix.cs).
#include <mutex>
#include <string>

#include "jv_internal.h"

using namespace jv;

namespace {

// jv_qmatvec's split-K partial buffer, one per device, grown on demand and kept.
struct PartialCache {
    std::mutex mu;
    float* buf[64] = {};
    size_t cap[64] = {};
    float* get(int dev, size_t n) {
        std::lock_guard<std::mutex> g(mu);
        if (dev < 0 || dev >= 64) throw Error(JV_ERR_ARG, "device index out of range");
        if (n > cap[dev]) {
            if (buf[dev]) cudaFree(buf[dev]);
            buf[dev] = nullptr;
            cap[dev] = 0;
            void* p = nullptr;
            cudaError_t e = cudaMalloc(&p, n * sizeof(float));
            if (e != cudaSuccess) {
                cudaGetLastError();
                throw Error(JV_ERR_OOM, std::string("cudaMalloc of the matvec partials: ") + cudaGetErrorString(e));
            }
            buf[dev] = (float*)p;
            cap[dev] = n;
        }
        return buf[dev];
    }
};
PartialCache g_partials;

int sm_count_of_current() {
    int dev = 0, sms = 148;
    JV_CUDA(cudaGetDevice(&dev));
    JV_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    return sms;
}

template <class F>
int api(F&& f) {
    try {
        f();
        return JV_OK;
    } catch (const Error& e) {
        return api_error(e.code, e.what());
    } catch (const std::exception& e) {
        return api_error(JV_ERR_ARG, e.what());
    }
}

}  // namespace

extern "C" {

int64_t jv_qweight_bytes(int32_t type, int32_t rows, int32_t cols) {
    try {
        return (int64_t)qweight_view(type, nullptr, rows, cols).bytes();
    } catch (const Error& e) {
        api_error(e.code, e.what());
        return -1;
    }
}

int jv_qweight_pack(int32_t type, const void* gguf_rows, int32_t rows, int32_t cols, void* tiled, void* stream) {
    return api([&] {
        QWeight w = qweight_view(type, tiled, rows, cols);
        if (!gguf_rows || !tiled) throw Error(JV_ERR_ARG, "NULL buffer");
        int64_t rb = (int64_t)cols / 32 * (type == T_Q8_0 ? 34 : type == T_Q4_0 ? 18 : 24);
        launch_repack((const uint8_t*)gguf_rows, type, rows, cols, rb, w.data, w.tiles, w.ksteps, 0, 0, 0,
                      (cudaStream_t)stream);
        JV_CUDA(cudaGetLastError());
    });
}

int jv_qmatvec(int32_t type, const void* tiled, int32_t rows, int32_t cols, const float* x, float* y, void* stream) {
    return api([&] {
        QWeight w = qweight_view(type, tiled, rows, cols);
        if (!tiled || !x || !y) throw Error(JV_ERR_ARG, "NULL buffer");
        int dev = 0;
        JV_CUDA(cudaGetDevice(&dev));
        int splits = gemv_splits_for(w, sm_count_of_current());
        float* part = g_partials.get(dev, (size_t)splits * rows);
        launch_gemv(w, x, part, splits, (cudaStream_t)stream);
        launch_gemv_reduce(part, splits, rows, y, EPI_STORE, (cudaStream_t)stream);
        JV_CUDA(cudaGetLastError());
    });
}

}  // extern "C"
