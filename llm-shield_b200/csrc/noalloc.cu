// noalloc.cu — jv_qmatvec_noalloc: the single-token quantized product of jv_qmatvec with its
// split-K partial sums kept in a fixed, statically sized device array instead of a buffer
// the library allocates.
//
// Who needs it: callers that must not allocate device memory on the call path — a host
// that pre-plans every byte of HBM (a serving process that has handed the rest of the
// GPU to its KV pool), or code that runs where an allocation would synchronize the device
// or fail (inside allocator callbacks, or under a memory cap set by another component).
// jv_qmatvec grows a cached cudaMalloc buffer on first use for each new size; this entry
// point never calls cudaMalloc, cudaFree or any allocating routine.
//
// Limits and sharing:
//  * The scratch array holds JV_QMATVEC_SCRATCH_FLOATS_MAX floats (1 MiB) per device. A call
//    needs splits × rows floats, where splits is the same split-K factor jv_qmatvec picks;
//    larger requests fail with JV_ERR_RANGE and a message giving both numbers.
//  * Every call on a device uses the same array. Each call overwrites, before reading, every
//    partial it sums, so nothing has to start at zero; but two calls whose kernels overlap in
//    time on one device (different streams, or different host threads) race on the array.
//    Serialize them (one stream, or events between streams).
//  * The first call on a device does a one-time set-up on that device: it looks up the
//    array's device address with cudaGetSymbolAddress while that device is current. Make the
//    first call on each device before any stream capture begins.
#include <mutex>
#include <string>

#include "jv_internal.h"

using namespace jv;

#define JV_QMATVEC_SCRATCH_FLOATS JV_QMATVEC_SCRATCH_FLOATS_MAX

static __device__ __align__(256) float g_qmatvec_scratch[JV_QMATVEC_SCRATCH_FLOATS];

namespace {

constexpr int kMaxDevices = 64;

struct ScratchAddress {
    std::mutex mu;
    float* ptr[kMaxDevices] = {};
    // The device address of g_qmatvec_scratch on `dev`, which must be the current device.
    float* get(int dev) {
        if (dev < 0 || dev >= kMaxDevices) throw Error(JV_ERR_ARG, "device index out of range");
        std::lock_guard<std::mutex> g(mu);
        if (!ptr[dev]) {
            void* p = nullptr;
            cudaError_t e = cudaGetSymbolAddress(&p, g_qmatvec_scratch);
            if (e != cudaSuccess || !p) {
                cudaGetLastError();
                throw Error(JV_ERR_DEVICE, std::string("cudaGetSymbolAddress of the matvec scratch: ") +
                                               cudaGetErrorString(e));
            }
            ptr[dev] = (float*)p;
        }
        return ptr[dev];
    }
};
ScratchAddress g_scratch;

}  // namespace

extern "C" int jv_qmatvec_noalloc(int32_t type, const void* tiled, int32_t rows, int32_t cols, const float* x,
                                  float* y, void* stream) {
    try {
        QWeight w = qweight_view(type, tiled, rows, cols);
        if (!tiled || !x || !y) throw Error(JV_ERR_ARG, "NULL buffer");
        int dev = 0, sms = 0;
        JV_CUDA(cudaGetDevice(&dev));
        JV_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
        int splits = gemv_splits_for(w, sms);
        int64_t need = (int64_t)splits * rows;
        if (need > JV_QMATVEC_SCRATCH_FLOATS)
            throw Error(JV_ERR_RANGE, "jv_qmatvec_noalloc: " + std::to_string(rows) + " rows x " +
                                          std::to_string(splits) + " k-splits need " + std::to_string(need) +
                                          " scratch floats; the fixed scratch holds " +
                                          std::to_string(JV_QMATVEC_SCRATCH_FLOATS));
        float* part = g_scratch.get(dev);
        launch_gemv(w, x, part, splits, (cudaStream_t)stream);
        launch_gemv_reduce(part, splits, rows, y, EPI_STORE, (cudaStream_t)stream);
        JV_CUDA(cudaGetLastError());
        return JV_OK;
    } catch (const Error& e) {
        return api_error(e.code, e.what());
    } catch (const std::exception& e) {
        return api_error(JV_ERR_ARG, e.what());
    }
}
