// streams.cu -- the library's own side streams and the event edges that fork and join them,
// and the device's SM count (the size of the persistent kernels' grids).
//
// Work that may run beside the caller's stream (the backward's dQ kernel, ring attention's
// NCCL transfers) goes to a side stream that belongs to the caller's stream: one per (device,
// caller stream, role), created on first use and kept for the life of the process. Calls on
// different caller streams -- other host threads, or a stream being captured into a CUDA graph
// -- therefore never share a side stream, so they pick up no false dependencies and an eager
// call cannot enqueue onto a stream that another thread is capturing. The map grows by one
// entry per distinct caller stream a process uses.
#include <cuda_runtime.h>

#include <map>
#include <mutex>
#include <tuple>

#include "common.cuh"
#include "kernels.h"

namespace dc {

namespace {
std::mutex g_mu;
std::map<std::tuple<int, cudaStream_t, int>, cudaStream_t> g_side;
}  // namespace

int side_stream(cudaStream_t caller, int role, cudaStream_t *out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "side stream: current device");
    std::lock_guard<std::mutex> lock(g_mu);
    auto key = std::make_tuple(dev, caller, role);
    auto it = g_side.find(key);
    if (it == g_side.end()) {
        // Ring transfers (role 1) run at the device's greatest priority: their few blocks then
        // take the next free SM ahead of the attention blocks queued beside them.
        int least = 0, greatest = 0;
        if (role == 1 && cudaDeviceGetStreamPriorityRange(&least, &greatest) != cudaSuccess) greatest = 0;
        cudaStream_t s = nullptr;
        e = cudaStreamCreateWithPriority(&s, cudaStreamNonBlocking, role == 1 ? greatest : 0);
        if (e != cudaSuccess) return cuda_fail(e, "side stream: create");
        it = g_side.emplace(key, s).first;
    }
    *out = it->second;
    return DC_OK;
}

int device_sm_count() {
    static int counts[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (!counts[dev]) {
        int n = 0;
        counts[dev] = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && n > 0 ? n : 148;
    }
    return counts[dev];
}

int stream_edge(cudaStream_t from, cudaStream_t to) {
    cudaEvent_t ev = nullptr;
    cudaError_t e = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventRecord(ev, from);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(to, ev, 0);
    if (ev) cudaEventDestroy(ev);  // released once the recorded work completes
    return e == cudaSuccess ? DC_OK : cuda_fail(e, "stream fork / join");
}

StreamJoin::~StreamJoin() {
    if (side_ && !joined_) {
        // An error path left the side stream forked: join it so that the caller's stream (and
        // a capture on it) sees no unjoined work. The call's own error is what it returns.
        const std::string saved = last_error();
        stream_edge(side_, caller_);
        set_error(saved);
    }
}

int StreamJoin::join() {
    if (!side_ || joined_) return DC_OK;
    joined_ = true;
    return stream_edge(side_, caller_);
}

}  // namespace dc
