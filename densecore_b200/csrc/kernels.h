// kernels.h -- host-side launchers of the SDPA kernels (internal to the library).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace dc {

struct MergeStrides {
    int64_t oas[4], las[3], ops[4], lps[3];
};

// CUDA-core kernels (attn_simt.cu): any head dim <= 256, any strides.
int simt_forward(const AttnProblem &p, cudaStream_t stream);
int bwd_delta(const AttnProblem &p, const AttnGrads &g, cudaStream_t stream);
int simt_backward(const AttnProblem &p, const AttnGrads &g, cudaStream_t stream);
int simt_probs(const AttnProblem &p, float *probs, const int64_t ps[4], int average,
               cudaStream_t stream);
int merge(float *oa, float *la, const float *op, const float *lp, int64_t B, int64_t H,
          int64_t L, int64_t Ev, const MergeStrides &st, cudaStream_t stream);

// Split-KV decode (decode.cu): q_len == 1, head dim 64 or 128, rows of 16-byte multiples.
bool decode_supported(const AttnProblem &p);
int decode_pick_splits(const AttnProblem &p);
size_t decode_workspace_bytes(int64_t B, int64_t H, int64_t Ev, int splits);
int decode_forward(const AttnProblem &p, int splits, void *workspace, cudaStream_t stream);

// tcgen05 tensor-core kernels (attn_tc.cu, attn_tc_bwd.cu). Forward: head dim 64 or 128,
// E == Ev, unit-stride rows on 16-byte boundaries. Backward: E == Ev == 64, any strides (its
// pre-pass copies the operands into contiguous TF32 hi / lo buffers); it also writes delta.
bool tc_forward_supported(const AttnProblem &p);
int tc_forward(const AttnProblem &p, int precision, cudaStream_t stream);
bool tc_backward_supported(const AttnProblem &p, const AttnGrads &g);
int tc_backward(const AttnProblem &p, const AttnGrads &g, int precision, cudaStream_t stream);
// The tensor-core kernels' device error word (sm100::DeviceError); -1 if it cannot be read.
int device_error(int reset);
// Device address of that word (passed to the kernels), or nullptr.
int *device_error_word();

// Dropout keep masks (rng.cu): n bernoulli(keep_prob) draws of DenseCore's generator stream
// from the device state st_in (624 words, left, next) as packed bits; the advanced state goes
// to st_out (which may equal st_in). rng_skip: the same advance on host memory, no device.
int keep_bits(const uint32_t *st_in, uint32_t *st_out, int64_t n, double keep_prob, uint32_t *bits,
              cudaStream_t stream);
int rng_skip(const uint32_t *st_in, uint64_t outputs, uint32_t *st_out);

// SM count of the current device (cached per device; 148 if it cannot be read).
int device_sm_count();

// Side streams (streams.cu): the library's stream for `role` (0 = the backward's dQ kernel,
// 1 = ring attention's transfers) beside caller stream `caller` on the current device, and an
// event edge that makes `to` wait for the work enqueued on `from` so far.
int side_stream(cudaStream_t caller, int role, cudaStream_t *out);
int stream_edge(cudaStream_t from, cudaStream_t to);

// A fork of `side` from `caller` that is joined back exactly once: by join(), or, on an error
// path that returns early, by the destructor (which keeps the call's error message).
class StreamJoin {
   public:
    StreamJoin(cudaStream_t caller, cudaStream_t side) : caller_(caller), side_(side) {}
    ~StreamJoin();
    int join();
    StreamJoin(const StreamJoin &) = delete;
    StreamJoin &operator=(const StreamJoin &) = delete;

   private:
    cudaStream_t caller_, side_;
    bool joined_ = false;
};

// The library's stream-ordered scratch pool (pool.cu): memory for `bytes` on `stream`'s
// order of the current device, and its release on the same stream.
int pool_alloc(void **ptr, size_t bytes, cudaStream_t stream);
void pool_free(void *ptr, cudaStream_t stream);

}  // namespace dc
