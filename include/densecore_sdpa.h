/*
 * densecore_sdpa.h -- C ABI of the B200 (sm_100a) scaled-dot-product-attention library.
 *
 * This is the drop-in boundary for DenseCore's flash-attention path. DenseCore reaches its
 * native kernels through two pyo3 functions in src/lib.rs; each entry point below replaces
 * one of them (or adds a device-only step the CPU path did not need) and keeps their
 * argument meaning and error behaviour:
 *
 *   dc_sdpa_fwd   <- _flash_attention           src/lib.rs:609-638 (-> torch_attention::forward)
 *   dc_sdpa_bwd   <- _flash_attention_backward  src/lib.rs:640-683 (-> torch_attention::backward)
 *   dc_sdpa_decode   q_len == 1 case of _flash_attention (torch_attention.rs:157, q_split -> 1)
 *   dc_sdpa_decode_noalloc  the same with a static scratch array (no reference counterpart)
 *   dc_attn_merge    logsumexp merge of partial results (ring attention; no CPU counterpart)
 *   dc_ring_sdpa_fwd  _flash_attention sharded by sequence over an NCCL communicator (ring
 *                    attention; the reference has no sequence parallelism)
 *   dc_attn_probs    softmax(scale*QK^T + mask) averaged over heads: the need_weights output of
 *                    multi_head_attention_forward (python/densecore/functional.py:456-461)
 *   dc_dropout_keep_bits  the bernoulli draw of _dropout_noise (functional.py:638-641,
 *                    src/torch_random.rs:242-254) as a device bit mask
 *   dc_sdpa_fwd_dropout / dc_sdpa_bwd_dropout / dc_attn_probs_dropout  SDPA and MHA with
 *                    dropout_p > 0 (functional.py:312-340, :450-451), fused
 *   dc_rng_skip      host-side skip-ahead of the generator state (no reference counterpart)
 *   dc_last_error    the message of the last failure on this thread (PyErr text in lib.rs)
 *
 * Conventions
 *  - Tensors are device pointers with sizes and strides in elements (dc_tensor_t). q is
 *    (B, H, L, E); k is (B, Hkv, S, E); v is (B, Hkv, S, Ev); H % Hkv == 0 (grouped-query).
 *    out is (B, H, L, Ev) and lse is (B, H, L), both float32, written by the library.
 *  - mask (nullable) is either float32 (added to the scaled scores) or bool/uint8 (1 = may
 *    attend, 0 = -inf), of 4 dims broadcastable to (B, H, L, S): a broadcast dim has size 1 or
 *    stride 0. This is the mask DenseCore's _flash_mask (functional.py:343-364) builds, without
 *    materialising it.
 *  - causal is top-left aligned: query row i attends keys j <= i (torch_attention.rs:176-180).
 *  - has_scale == 0 means scale = (float)(1/sqrt(E)) computed in double
 *    (torch_attention.rs:37-40).
 *  - A fully masked query row gives out = 0, lse = 0 and zero gradients, as
 *    torch_attention.rs:223-226 and :258-271 do.
 *  - precision: DC_PREC_3XTF32 (default; fp32-class accuracy on tcgen05 tensor cores),
 *    DC_PREC_TF32 (opt-in single-pass TF32) or DC_PREC_FP32 (CUDA-core fp32). Shapes the
 *    tensor-core kernels do not cover run the CUDA-core kernels whatever the precision.
 *  - Launches are asynchronous on `stream` (a cudaStream_t; NULL = legacy default stream).
 *    No call synchronises the host. There is no CPU fallback: with no usable device the call
 *    fails with DC_ERR_CUDA.
 *  - The library keeps per-device state for the life of the process (side streams, the device
 *    status word's and the no-alloc scratch's addresses, the dropout jump tables): calling
 *    cudaDeviceReset while the library is loaded and then using it again is not supported.
 *  - Return value: DC_OK, or an error code; dc_last_error() then holds the message.
 *    DC_ERR_VALUE corresponds to the reference's ValueError (shape errors, lib.rs:562-570,
 *    :601-605, :658-662); DC_ERR_RUNTIME / DC_ERR_CUDA to its RuntimeError (lib.rs:633, :677).
 */
#ifndef DENSECORE_SDPA_H
#define DENSECORE_SDPA_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define DC_API __attribute__((visibility("default")))
#else
#define DC_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define DC_SDPA_ABI_VERSION 1

enum dc_status {
    DC_OK = 0,
    DC_ERR_VALUE = 1,       /* bad shapes / arguments (the reference's ValueError) */
    DC_ERR_RUNTIME = 2,     /* kernel-side failure (the reference's RuntimeError) */
    DC_ERR_CUDA = 3,        /* CUDA runtime / driver error */
    DC_ERR_UNSUPPORTED = 4  /* valid request this build does not implement */
};

enum dc_dtype { DC_F32 = 0, DC_BOOL = 1 };

enum dc_precision { DC_PREC_3XTF32 = 0, DC_PREC_TF32 = 1, DC_PREC_FP32 = 2 };

/* A strided device tensor view. Unused trailing dims are ignored (ndim <= 4). */
typedef struct dc_tensor {
    void *data;
    int32_t dtype;      /* enum dc_dtype */
    int32_t ndim;
    int64_t sizes[4];
    int64_t strides[4]; /* in elements */
} dc_tensor_t;

/* Forward: out (B,H,L,Ev) and lse (B,H,L).  Replaces _flash_attention, src/lib.rs:609-638. */
DC_API int dc_sdpa_fwd(const dc_tensor_t *q, const dc_tensor_t *k, const dc_tensor_t *v,
                const dc_tensor_t *mask, int causal, int has_scale, double scale, int precision,
                dc_tensor_t *out, dc_tensor_t *lse, void *stream);

/* Bytes of device scratch dc_sdpa_bwd needs for these shapes (the per-row
 * sum(grad_out*out) of torch_attention.rs:327-330, plus alignment). */
DC_API size_t dc_sdpa_bwd_workspace_size(int64_t batch, int64_t heads, int64_t q_len);

/* Backward: grad_q (B,H,L,E), grad_k (B,Hkv,S,E), grad_v (B,Hkv,S,Ev), overwritten.
 * workspace may be NULL (then the library takes stream-ordered memory with
 * cudaMallocAsync); otherwise it must hold dc_sdpa_bwd_workspace_size() bytes.
 * Replaces _flash_attention_backward, src/lib.rs:640-683. */
DC_API int dc_sdpa_bwd(const dc_tensor_t *grad_out, const dc_tensor_t *q, const dc_tensor_t *k,
                const dc_tensor_t *v, const dc_tensor_t *out, const dc_tensor_t *lse,
                const dc_tensor_t *mask, int causal, int has_scale, double scale, int precision,
                dc_tensor_t *grad_q, dc_tensor_t *grad_k, dc_tensor_t *grad_v, void *workspace,
                size_t workspace_bytes, void *stream);

/* Bytes of scratch dc_sdpa_decode needs for num_splits partial results per (batch, head). */
DC_API size_t dc_sdpa_decode_workspace_size(int64_t batch, int64_t heads, int64_t head_dim_v,
                                     int num_splits);

/* The split count dc_sdpa_decode picks for num_splits <= 0 on the current device. */
DC_API int dc_sdpa_decode_default_splits(int64_t batch, int64_t heads, int64_t kv_len);

/* Decode (q_len == 1) by split-KV: num_splits CTAs stream disjoint key ranges of each
 * (batch, head) and a second pass merges them by logsumexp. num_splits <= 0 picks a split
 * count that fills the GPU. Same result contract as dc_sdpa_fwd with L == 1, non-causal
 * (a causal q_len == 1 row sees only key 0 and is served by dc_sdpa_fwd).
 * The q_len == 1 case of _flash_attention, src/lib.rs:609-638 / torch_attention.rs:157. */
DC_API int dc_sdpa_decode(const dc_tensor_t *q, const dc_tensor_t *k, const dc_tensor_t *v,
                   const dc_tensor_t *mask, int has_scale, double scale, int num_splits,
                   dc_tensor_t *out, dc_tensor_t *lse, void *workspace, size_t workspace_bytes,
                   void *stream);

/* Fixed size of the device scratch dc_sdpa_decode_noalloc holds per device: 8 MiB, enough for
 * the default split count (148 SMs) of up to 16131 (batch, head) rows at head dim 128 -- the
 * default split count falls to 1 at 3552 rows and more, so that at 16131 rows one split's
 * partials (130 floats per row) still fit. */
#define DC_DECODE_NOALLOC_SCRATCH_BYTES (8u << 20)

/* dc_sdpa_decode that allocates no device memory: the split partials go to a static device
 * array of DC_DECODE_NOALLOC_SCRATCH_BYTES in the library instead of a workspace. For callers
 * that cannot let the library allocate (device memory reserved up front for a KV cache; C
 * hosts with no allocator to hand a workspace from). No counterpart in the reference: its CPU
 * path allocates its scratch on the heap per call.
 *  - A request whose partials need more than DC_DECODE_NOALLOC_SCRATCH_BYTES
 *    (B*H*splits*(Ev+2)*4 bytes) fails with DC_ERR_VALUE before anything is launched.
 *  - There is one scratch array per device, shared by every call on that device: calls whose
 *    kernels overlap in time (different streams, or host threads without ordering between
 *    them) overwrite each other's partials. Order them, e.g. on one stream.
 *  - The first call on a device looks up the array's address (cudaGetSymbolAddress, which
 *    may load the module); make that first call before any stream capture begins.
 * Results are those of dc_sdpa_decode with the same num_splits. */
DC_API int dc_sdpa_decode_noalloc(const dc_tensor_t *q, const dc_tensor_t *k, const dc_tensor_t *v,
                                  const dc_tensor_t *mask, int has_scale, double scale,
                                  int num_splits, dc_tensor_t *out, dc_tensor_t *lse, void *stream);

/* In-place logsumexp merge of a partial attention result into an accumulator over the same
 * rows: lse = log(exp(lse_acc) + exp(lse_part)), out_acc = out_acc*exp(lse_acc - lse) +
 * out_part*exp(lse_part - lse). Rows with lse_part = -inf leave the accumulator unchanged; an
 * accumulator row with lse_acc = -inf takes the partial as it is. Tensors are (B,H,L,Ev) and (B,H,L)
 * strided views. Used by ring attention after each K/V block (no reference counterpart: the
 * reference has no sequence parallelism). */
DC_API int dc_attn_merge(dc_tensor_t *out_acc, dc_tensor_t *lse_acc, const dc_tensor_t *out_part,
                  const dc_tensor_t *lse_part, void *stream);

/* ---- Ring attention (sequence parallelism over an NCCL communicator) ----
 * NCCL's communicator type: ncclComm_t in nccl.h is `struct ncclComm *`. */
struct ncclComm;

/* Bytes of device workspace dc_ring_sdpa_fwd needs for local shards q (B, H, 2C, E) and
 * k, v (B, Hkv, 2C, E): two packed K/V blocks and one partial result. */
DC_API size_t dc_ring_sdpa_fwd_workspace_size(int64_t batch, int64_t heads, int64_t kv_heads,
                                              int64_t local_len, int64_t head_dim);

/* Ring attention forward over the P ranks of `comm` (rank and P are the communicator's own).
 * Each rank passes its zig-zag shard of one sequence: chunks r and 2P-1-r of 2P equal chunks,
 * back to back, as q (B, H, 2C, E) and contiguous k, v (B, Hkv, 2C, E); out (B, H, 2C, E) and
 * lse (B, H, 2C) receive what dc_sdpa_fwd over the whole sequence gives for those query rows
 * (top-left causal when causal != 0). K/V blocks go round the ring with ncclSend / ncclRecv on
 * a side stream of the library's, overlapped with each step's attention on `stream`; partial
 * results are merged by logsumexp (dc_attn_merge). Every rank must make the same call (same
 * shapes, causal flag and order of calls on `comm`). workspace: device memory of
 * dc_ring_sdpa_fwd_workspace_size() bytes, 256-byte aligned. No user mask (a row fully masked
 * inside one block would give the reference's out = 0, lse = 0 for that block, which a merge
 * cannot tell from a real contribution). If a call fails after its first transfer was issued,
 * the peers' matching transfers are left pending: abort the communicator (ncclCommAbort).
 * The reference has no sequence parallelism: this shards torch_attention.rs:146-284 by
 * sequence, and its result contract is that of dc_sdpa_fwd / _flash_attention (lib.rs:609-638). */
DC_API int dc_ring_sdpa_fwd(const dc_tensor_t *q, const dc_tensor_t *k, const dc_tensor_t *v,
                            int causal, int has_scale, double scale, int precision,
                            struct ncclComm *comm, dc_tensor_t *out, dc_tensor_t *lse,
                            void *workspace, size_t workspace_bytes, void *stream);

/* Head-averaged attention probabilities (B, L, S): mean over H of
 * exp(scale*q.k + mask - lse) with lse from dc_sdpa_fwd, zero where masked or causal-hidden.
 * The need_weights=True, average_attn_weights=True output of
 * multi_head_attention_forward (python/densecore/functional.py:456-461). With
 * average_heads == 0, probs is (B, H, L, S) instead. */
DC_API int dc_attn_probs(const dc_tensor_t *q, const dc_tensor_t *k, const dc_tensor_t *lse,
                  const dc_tensor_t *mask, int causal, int has_scale, double scale,
                  int average_heads, dc_tensor_t *probs, void *stream);

/* ---- Dropout (python/densecore/functional.py:229-244, :312-340, :450-451, :638-641) ----
 * DenseCore runs SDPA with dropout_p > 0 on its math path: the softmax weights are multiplied
 * by noise = bernoulli(1 - p) / float32(1 - p), drawn in row-major (B, H, L, S) order from the
 * CPU generator that manual_seed seeds (PyTorch's mt19937 as src/torch_random.rs ports it).
 * Here the generator's engine state lives in device memory as 626 uint32 words -- the 624
 * state words, then `left` and `next` (src/torch_random.rs:19-26) -- the keep mask is drawn
 * on the device, and the attention kernels apply it. */

/* n bernoulli(keep_prob) draws as packed bits -- element e is bit e % 32 of bits[e / 32],
 * ceil(n / 32) words, 4-byte aligned -- bit-identical to DenseCore's Generator::bernoulli
 * (src/torch_random.rs:242-254) continuing from the device state state_in: each draw takes
 * two 32-bit outputs, x = (random64 & (2^53 - 1)) * 2^-53, keep when x < keep_prob. The
 * state after the 2n outputs is written to state_out (which may equal state_in). A state
 * whose `left` is not in 1..624 sets dc_device_status() to 2 and writes nothing.
 * The first call in a process computes the generator's jump tables on the host (a fraction
 * of a second, on up to 16 host threads), and the first call on each device copies them there
 * with synchronous copies: make that call before any stream capture. */
DC_API int dc_dropout_keep_bits(const uint32_t *state_in, uint32_t *state_out, int64_t n,
                                double keep_prob, uint32_t *bits, void *stream);

/* Host memory only, no device: state_out = the engine state (626 words, as above) after
 * `outputs` 32-bit outputs from state_in, outputs <= 2^36. state_out may equal state_in.
 * No counterpart in the reference (it draws sequentially). */
DC_API int dc_rng_skip(const uint32_t *state_in, uint64_t outputs, uint32_t *state_out);

/* dc_sdpa_fwd with dropout on the attention weights: weight (b, h, i, j) is multiplied by
 * keep_scale when bit ((b*H + h)*L + i)*S + j of keep_bits is set and by 0 otherwise (the
 * mask of dc_dropout_keep_bits over B*H*L*S elements; keep_scale = float32(1) /
 * float32(1 - p), as _dropout_noise divides). lse is the logsumexp of the undropped scores.
 * Shapes that dc_sdpa_fwd gives the tensor-core kernels take them here too, with the keep
 * bits applied to the weights inside; every other shape (the q_len = 1 decode shapes
 * included) takes the CUDA-core fp32 kernel, whatever the precision.
 * Replaces the math path of scaled_dot_product_attention with dropout (functional.py:318-340). */
DC_API int dc_sdpa_fwd_dropout(const dc_tensor_t *q, const dc_tensor_t *k, const dc_tensor_t *v,
                               const dc_tensor_t *mask, int causal, int has_scale, double scale,
                               int precision, const uint32_t *keep_bits, float keep_scale,
                               dc_tensor_t *out, dc_tensor_t *lse, void *stream);

/* The backward of dc_sdpa_fwd_dropout (same keep_bits and keep_scale; out and lse from it):
 * dV = (P Z)^T dO, dS = P (Z (dO V^T) - rowsum(dO * out)) with Z the dropout factors. The
 * kernels are chosen as dc_sdpa_bwd chooses them (tensor cores unless DC_PREC_FP32 or an
 * unsupported shape). */
DC_API int dc_sdpa_bwd_dropout(const dc_tensor_t *grad_out, const dc_tensor_t *q,
                               const dc_tensor_t *k, const dc_tensor_t *v, const dc_tensor_t *out,
                               const dc_tensor_t *lse, const dc_tensor_t *mask, int causal,
                               int has_scale, double scale, int precision,
                               const uint32_t *keep_bits, float keep_scale, dc_tensor_t *grad_q,
                               dc_tensor_t *grad_k, dc_tensor_t *grad_v, void *workspace,
                               size_t workspace_bytes, void *stream);

/* dc_attn_probs with each probability times its dropout factor: the weights
 * multi_head_attention_forward returns when it trains with dropout (functional.py:450-461). */
DC_API int dc_attn_probs_dropout(const dc_tensor_t *q, const dc_tensor_t *k,
                                 const dc_tensor_t *lse, const dc_tensor_t *mask, int causal,
                                 int has_scale, double scale, const uint32_t *keep_bits,
                                 float keep_scale, int average_heads, dc_tensor_t *probs,
                                 void *stream);

/* Kernel tracing. While enabled, every kernel the library launches is bracketed by two
 * CUDA events on its launch stream. dc_kernel_timing_report() waits for the recorded events
 * and writes {"<kernel>": [launches, total_ms], ...} as JSON into buf (truncated to len);
 * reset != 0 then forgets the records. Returns the number of launches reported, or -1.
 * (DenseCore has no tracing of its own; it profiles with cProfile.) */
DC_API int dc_kernel_timing(int enable);
DC_API int dc_kernel_timing_report(char *buf, size_t len, int reset);

/* Device-side status of the library's kernels: 0; 1 when a tensor-core kernel gave up on a
 * wait that did not complete within its bound (1 s) -- that CTA then unwound without writing
 * its outputs; 2 when dc_dropout_keep_bits read a generator state whose `left` word is not in
 * 1..624 -- it then wrote neither mask nor state. Synchronises with the device. reset != 0
 * clears the status. -1 on a CUDA error. */
DC_API int dc_device_status(int reset);

/* Failure-detection hook for tests: launches `blocks` (1..1024) CTAs of a probe kernel that
 * takes 32 columns of tensor memory and then waits on an mbarrier that nothing arrives at,
 * through the same bounded wait the tensor-core kernels use, with the bound shortened to
 * timeout_ns (1000 ns .. 1 s). Each wait gives up after the bound, sets dc_device_status() to
 * 1, and its CTA frees its tensor memory and returns: the call ends, the device stays usable
 * and the next call runs normally. Nothing faults or hangs. No counterpart in the reference,
 * whose CPU kernels report failure through their Result slots (torch_attention.rs:163,
 * :274-276; raised as RuntimeError at lib.rs:633, :677). */
DC_API int dc_debug_wait_probe(uint64_t timeout_ns, int blocks, void *stream);

/* Message of the last failing call on this host thread ("" if none). */
DC_API const char *dc_last_error(void);

/* DC_SDPA_ABI_VERSION of the loaded library. */
DC_API int dc_abi_version(void);

/* Which kernel family dc_sdpa_fwd would pick for these shapes: 0 = CUDA-core (fp32 FMA),
 * 1 = tcgen05 tensor cores, 2 = split-KV decode; -1 on invalid shapes. For tests and the
 * benchmark's launch accounting. */
DC_API int dc_sdpa_fwd_path(const dc_tensor_t *q, const dc_tensor_t *k, const dc_tensor_t *v,
                     const dc_tensor_t *mask, int causal, int precision);

#ifdef __cplusplus
}
#endif

#endif /* DENSECORE_SDPA_H */
