// selftest.cu -- the wait probe behind dc_debug_wait_probe.
//
// Every tensor-core kernel of the library waits on mbarriers through sm100::mbar_wait, whose
// wait is bounded: a phase that has not completed within the bound sets the CTA's abort flag,
// records DEV_WAIT_TIMEOUT in the library's device status word, and the CTA frees its tensor
// memory and returns. The probe kernel runs that same wait on a barrier nothing ever arrives
// at, with the bound shortened, while holding tensor memory, so that a test can show on a GPU
// that such a wait gives up, that the status word says so, and that the next call (which
// allocates all 512 TMEM columns of an SM) runs normally. Nothing faults, traps or spins
// without a bound: the probe's only wait is the bounded one.
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.h"
#include "sm100.cuh"
#include "trace.h"

namespace dc {
namespace {

using namespace sm100;

constexpr uint32_t kProbeTmemCols = 32;  // 16 probe CTAs fit the 512 columns of one SM

__global__ void __launch_bounds__(128) wait_probe_kernel(uint64_t timeout_ns, int *err) {
    __shared__ __align__(8) uint64_t bar_mem;
    __shared__ uint32_t tmem_slot;
    __shared__ int abort_flag;
    const uint32_t bar = smem_addr(&bar_mem);
    const int warp = threadIdx.x >> 5;
    if (threadIdx.x == 0) {
        mbar_init(bar, 1);  // one arrival would complete phase 0; none is ever made
        abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc(smem_addr(&tmem_slot), kProbeTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // Phase 0 of a freshly initialised barrier never completes here: every thread's wait
    // runs into the bound (or sees the abort flag another thread set when it did).
    mbar_wait(bar, 0, &abort_flag, err, timeout_ns);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) tmem_dealloc(tmem_slot, kProbeTmemCols);
}

}  // namespace
}  // namespace dc

using namespace dc;

extern "C" DC_API int dc_debug_wait_probe(uint64_t timeout_ns, int blocks, void *stream) {
    if (timeout_ns < 1000 || timeout_ns > sm100::WAIT_TIMEOUT_NS)
        return fail(DC_ERR_VALUE, "dc_debug_wait_probe: timeout_ns must be in [1000, 1000000000], got " +
                                      std::to_string(timeout_ns));
    if (blocks < 1 || blocks > 1024)
        return fail(DC_ERR_VALUE, "dc_debug_wait_probe: blocks must be in [1, 1024], got " + std::to_string(blocks));
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess || n == 0) return e != cudaSuccess ? cuda_fail(e, "no CUDA device") : fail(DC_ERR_CUDA, "no CUDA device");
    int *err = device_error_word();
    if (!err) return fail(DC_ERR_CUDA, "device error word is unavailable");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    KernelTrace tr("wait_probe", s);
    wait_probe_kernel<<<blocks, 128, 0, s>>>(timeout_ns, err);
    return check_launch("wait_probe");
}
