// Host-side helpers shared by the engine (error strings, driver entry points).
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>
#include <string>

#include "vdb_internal.h"
#include "vdb_ops.h"

namespace vdb {

namespace {
thread_local std::string g_last_error;
}

void set_error(const std::string& msg) { g_last_error = msg; }
const std::string& get_error() { return g_last_error; }

EncodeTiledFn encode_tiled_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    if (!fn) {
        // Report through the op error path; callers check the CUresult.
        static EncodeTiledFn missing = [](CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                          const cuuint64_t*, const cuuint64_t*,
                                          const cuuint32_t*, const cuuint32_t*,
                                          CUtensorMapInterleave, CUtensorMapSwizzle,
                                          CUtensorMapL2promotion,
                                          CUtensorMapFloatOOBfill) -> CUresult {
            return CUDA_ERROR_NOT_FOUND;
        };
        return missing;
    }
    return fn;
}

void keep_async_pool() {
    // Stream-ordered workspace (cudaMallocAsync) comes from the device's default
    // memory pool, which by default returns freed memory to the driver at every
    // synchronisation, so the next call pays a full allocation (about a millisecond
    // for the 100 MB an identify call uses). Keep it cached instead: once per device,
    // the pool's release threshold is raised to "never". It only affects this
    // process's pool and ends with it.
    static std::mutex mu;
    static bool done[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return;
    std::lock_guard<std::mutex> lk(mu);
    if (done[dev]) return;
    cudaMemPool_t pool = nullptr;
    if (cudaDeviceGetDefaultMemPool(&pool, dev) == cudaSuccess && pool) {
        uint64_t keep = UINT64_MAX;
        cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
    }
    done[dev] = true;
}

int num_sms() {
    int dev = 0;
    cudaGetDevice(&dev);
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n > 0 ? n : 1;
}

}  // namespace vdb

extern "C" const char* vdb_last_error(void) { return vdb::get_error().c_str(); }
