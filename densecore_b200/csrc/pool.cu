// pool.cu -- the library's own stream-ordered memory pool (one per device).
//
// Scratch whose size the C ABI's workspace arguments do not cover (the tensor-core backward's
// TF32 hi / lo copies of q, k, v and grad_out) comes from here. The pool keeps freed memory
// for reuse (release threshold = no limit), so a steady training loop allocates from the
// device once; the pool is private to the library and is not the device's current pool.
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>
#include <string>

#include "common.cuh"
#include "kernels.h"

namespace dc {

namespace {
constexpr int kPoolDevices = 64;
std::mutex g_pool_mu;
cudaMemPool_t g_pools[kPoolDevices];
}  // namespace

int pool_alloc(void **ptr, size_t bytes, cudaStream_t stream) {
    *ptr = nullptr;
    if (bytes == 0) return DC_OK;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "memory pool: current device");
    if (dev < 0 || dev >= kPoolDevices)
        return fail(DC_ERR_UNSUPPORTED, "memory pool: device ordinal " + std::to_string(dev) + " is above 63");
    cudaMemPool_t pool;
    {
        std::lock_guard<std::mutex> lock(g_pool_mu);
        if (!g_pools[dev]) {
            cudaMemPoolProps props{};
            props.allocType = cudaMemAllocationTypePinned;
            props.location.type = cudaMemLocationTypeDevice;
            props.location.id = dev;
            e = cudaMemPoolCreate(&pool, &props);
            if (e != cudaSuccess) return cuda_fail(e, "memory pool: create");
            uint64_t keep = UINT64_MAX;
            e = cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
            if (e != cudaSuccess) return cuda_fail(e, "memory pool: release threshold");
            g_pools[dev] = pool;
        }
        pool = g_pools[dev];
    }
    e = cudaMallocFromPoolAsync(ptr, bytes, pool, stream);
    if (e != cudaSuccess) {
        *ptr = nullptr;
        return cuda_fail(e, "memory pool: allocate");
    }
    return DC_OK;
}

void pool_free(void *ptr, cudaStream_t stream) {
    if (ptr) cudaFreeAsync(ptr, stream);
}

}  // namespace dc
