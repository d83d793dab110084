// trace.h -- RAII bracket that records CUDA events around one kernel launch when tracing
// is on (dc_kernel_timing). Construct it right before the launch, in the same scope.
#pragma once

#include <cuda_runtime.h>

namespace dc {

bool trace_enabled();

class KernelTrace {
   public:
    KernelTrace(const char *name, cudaStream_t stream);
    ~KernelTrace();
    KernelTrace(const KernelTrace &) = delete;
    KernelTrace &operator=(const KernelTrace &) = delete;

   private:
    const char *name_;
    cudaStream_t stream_;
    cudaEvent_t start_ = nullptr;
};

}  // namespace dc
