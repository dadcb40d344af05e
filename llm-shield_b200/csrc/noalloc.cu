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
//  * The address is remembered per CUDA context (the context current at the call), so a
//    device reset, after which the device gets a new context, is followed by a fresh look-up
//    on the next call instead of a stale address.
#include <cuda.h>

#include <mutex>
#include <string>
#include <utility>
#include <vector>

#include "jv_internal.h"

using namespace jv;

#define JV_QMATVEC_SCRATCH_FLOATS JV_QMATVEC_SCRATCH_FLOATS_MAX

static __device__ __align__(256) float g_qmatvec_scratch[JV_QMATVEC_SCRATCH_FLOATS];

namespace {

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);

// The CUDA context current on this thread, or nullptr before the runtime has set one up, read
// through the driver entry point the runtime hands out (no link against libcuda is needed).
CUcontext current_context() {
    static CtxGetCurrentFn fn = [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            f = nullptr;
        cudaGetLastError();
        return (CtxGetCurrentFn)f;
    }();
    if (!fn) throw Error(JV_ERR_DEVICE, "cuCtxGetCurrent is not available from the CUDA driver");
    CUcontext c = nullptr;
    if (fn(&c) != CUDA_SUCCESS) throw Error(JV_ERR_DEVICE, "cuCtxGetCurrent failed");
    return c;
}

struct ScratchAddress {
    std::mutex mu;
    std::vector<std::pair<CUcontext, float*>> known;
    // The device address of g_qmatvec_scratch in the current context. The first call in a
    // context looks it up (cudaGetSymbolAddress, which also sets up the current device's
    // context if nothing has yet) and remembers it for that context.
    float* get() {
        std::lock_guard<std::mutex> g(mu);
        if (CUcontext c = current_context())
            for (auto& k : known)
                if (k.first == c) return k.second;
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_qmatvec_scratch);
        if (e != cudaSuccess || !p) {
            cudaGetLastError();
            throw Error(JV_ERR_DEVICE, std::string("cudaGetSymbolAddress of the matvec scratch: ") +
                                           cudaGetErrorString(e));
        }
        CUcontext c = current_context();
        if (!c) throw Error(JV_ERR_DEVICE, "no CUDA context is current after the scratch look-up");
        known.emplace_back(c, (float*)p);
        return (float*)p;
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
        float* part = g_scratch.get();
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
