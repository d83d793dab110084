// common.cuh -- shared definitions of the sm_100a SDPA library: the problem description
// every kernel receives, mask access, the per-thread error slot and launch helpers.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/densecore_sdpa.h"

namespace dc {

// One attention problem: q (B,H,L,E), k (B,Hkv,S,E), v (B,Hkv,S,Ev), out (B,H,L,Ev),
// lse (B,H,L). Strides are in elements; a mask stride of 0 broadcasts that dim.
struct AttnProblem {
    const float *q, *k, *v;
    float *out, *lse;
    int64_t B, H, Hkv, L, S, E, Ev;
    int64_t qs[4], ks[4], vs[4], os[4], ls[3];
    const void *mask;
    int mask_kind;  // 0 none, 1 float additive, 2 bool (nonzero = may attend)
    int64_t ms[4];
    int causal;
    float scale;
    int group;  // H / Hkv
    // Dropout on the attention weights (null = none): weight (b, h, i, j) is multiplied by
    // keep_scale when bit e % 32 of keep[e / 32] is set, e = ((b * H + h) * L + i) * S + j,
    // and by 0 otherwise.
    const uint32_t *keep;
    float keep_scale;
};

// Backward extras: grad_out (B,H,L,Ev), dq (B,H,L,E), dk (B,Hkv,S,E), dv (B,Hkv,S,Ev),
// delta (B*H*L, contiguous; sum(grad_out * out) per row).
struct AttnGrads {
    const float *dout;
    float *dq, *dk, *dv;
    float *delta;
    int64_t dos[4], dqs[4], dks[4], dvs[4];
};

enum MaskKind { MASK_NONE = 0, MASK_FLOAT = 1, MASK_BOOL = 2 };

__device__ __forceinline__ float mask_value(const AttnProblem &p, int64_t b, int64_t h,
                                            int64_t i, int64_t j) {
    int64_t off = b * p.ms[0] + h * p.ms[1] + i * p.ms[2] + j * p.ms[3];
    if (p.mask_kind == MASK_FLOAT) return static_cast<const float *>(p.mask)[off];
    return static_cast<const uint8_t *>(p.mask)[off] ? 0.0f : -INFINITY;
}

// N mask values of (b, h) starting at element (i, j) and stepping `step` elements (the key
// stride for a run along a row, the query stride for a run along a column), for the entries
// whose bit is set in `bits` (the others read as 0). Float masks give their value, bool masks 0
// or -inf. A run with unit step on a 16-byte (float) or 4-byte (bool) boundary loads four
// values at a time; a zero step loads one value.
template <int N>
__device__ __forceinline__ void mask_run(const AttnProblem &p, int64_t b, int64_t h, int64_t i, int64_t j,
                                         int64_t step, uint32_t bits, float (&out)[N]) {
    const int64_t off = b * p.ms[0] + h * p.ms[1] + i * p.ms[2] + j * p.ms[3];
    if (p.mask_kind == MASK_FLOAT) {
        const float *m = static_cast<const float *>(p.mask) + off;
        if (step == 0) {
            const float v = bits ? *m : 0.0f;
#pragma unroll
            for (int c = 0; c < N; c++) out[c] = v;
        } else if (step == 1 && (reinterpret_cast<uintptr_t>(m) & 15u) == 0) {
#pragma unroll
            for (int g = 0; g < N / 4; g++) {
                if (((bits >> (4 * g)) & 15u) == 15u) {
                    const float4 v = *reinterpret_cast<const float4 *>(m + 4 * g);
                    out[4 * g] = v.x;
                    out[4 * g + 1] = v.y;
                    out[4 * g + 2] = v.z;
                    out[4 * g + 3] = v.w;
                } else {
#pragma unroll
                    for (int e = 0; e < 4; e++) out[4 * g + e] = ((bits >> (4 * g + e)) & 1u) ? m[4 * g + e] : 0.0f;
                }
            }
        } else {
#pragma unroll
            for (int c = 0; c < N; c++) out[c] = ((bits >> c) & 1u) ? m[c * step] : 0.0f;
        }
    } else {
        const uint8_t *m = static_cast<const uint8_t *>(p.mask) + off;
        if (step == 0) {
            const float v = (bits && !*m) ? -INFINITY : 0.0f;
#pragma unroll
            for (int c = 0; c < N; c++) out[c] = v;
        } else if (step == 1 && (reinterpret_cast<uintptr_t>(m) & 3u) == 0) {
#pragma unroll
            for (int g = 0; g < N / 4; g++) {
                uint32_t w = 0x01010101u;
                if (((bits >> (4 * g)) & 15u) == 15u) {
                    w = *reinterpret_cast<const uint32_t *>(m + 4 * g);
                } else {
#pragma unroll
                    for (int e = 0; e < 4; e++)
                        if ((bits >> (4 * g + e)) & 1u) w = (w & ~(0xFFu << (8 * e))) | ((uint32_t)m[4 * g + e] << (8 * e));
                }
#pragma unroll
                for (int e = 0; e < 4; e++) out[4 * g + e] = ((w >> (8 * e)) & 0xFFu) ? 0.0f : -INFINITY;
            }
        } else {
#pragma unroll
            for (int c = 0; c < N; c++) out[c] = (((bits >> c) & 1u) && !m[c * step]) ? -INFINITY : 0.0f;
        }
    }
}

// The dropout factor of weight (b, h, i, j): keep_scale or 0 (1 without dropout).
__device__ __forceinline__ float keep_factor(const AttnProblem &p, int64_t b, int64_t h, int64_t i, int64_t j) {
    if (!p.keep) return 1.0f;
    const int64_t e = ((b * p.H + h) * p.L + i) * p.S + j;
    return (__ldg(p.keep + (e >> 5)) >> (e & 31)) & 1u ? p.keep_scale : 0.0f;
}

// Dropout keep bits of the weights (b, h, i, j0 + c), c = 0..31, as one word (bit c). Words
// past the end of the bit array read as 0; the caller's validity bits cover those columns.
__device__ __forceinline__ uint32_t keep_run32(const AttnProblem &p, int64_t b, int64_t h, int64_t i, int64_t j0) {
    const int64_t e = ((b * p.H + h) * p.L + i) * p.S + j0;
    const int64_t nw = (p.B * p.H * p.L * p.S + 31) >> 5;
    const int64_t w = e >> 5;
    const uint32_t lo = w < nw ? __ldg(p.keep + w) : 0u;
    const uint32_t hi = w + 1 < nw ? __ldg(p.keep + w + 1) : 0u;
    return __funnelshift_r(lo, hi, (uint32_t)(e & 31));
}

// Dropout keep bits down key columns, for a warp whose lane l owns key j0 + l: lane r holds
// w_r = keep_run32(row i0 + r, keys j0 .. j0 + 31) and gets back the word whose bit c is bit l
// of w_c, i.e. lane l's bits over rows i0 + c. The 32 x 32 bit block is transposed in five
// butterfly stages: at stage j, lanes l and l ^ j swap the j x j sub-blocks off the diagonal of
// each 2j x 2j block (a lane with bit j clear keeps the low j bits of every 2j-bit group and
// takes its partner's low bits shifted up; the other keeps the high bits and takes its
// partner's high bits shifted down). A warp reads one word pair per lane instead of one word
// per (row, lane). All 32 lanes must call it.
__device__ __forceinline__ uint32_t transpose_bits32(uint32_t w, int lane) {
    constexpr uint32_t masks[5] = {0x0000FFFFu, 0x00FF00FFu, 0x0F0F0F0Fu, 0x33333333u, 0x55555555u};
#pragma unroll
    for (int s = 0; s < 5; s++) {
        const int j = 16 >> s;
        const uint32_t m = masks[s];
        const uint32_t y = __shfl_xor_sync(0xffffffffu, w, j);
        w = (lane & j) ? ((w & ~m) | ((y >> j) & m)) : ((w & m) | ((y << j) & ~m));
    }
    return w;
}

// Whether key j is visible to query row i under top-left causal alignment.
__device__ __forceinline__ bool causal_visible(int causal, int64_t i, int64_t j) {
    return !causal || j <= i;
}

// Host side: the thread's last error message and a setter that returns the status.
void set_error(const std::string &msg);
std::string last_error();
int fail(int status, const std::string &msg);
int cuda_fail(cudaError_t err, const char *what);

// Checks the launch just issued on `stream`; returns DC_OK or DC_ERR_CUDA.
int check_launch(const char *what);

// Programmatic dependent launch: the kernel may become resident while the kernel before it on
// `stream` drains (and run its set-up: barriers, tensor memory, tensor-map prefetch); it must
// execute griddep_wait() before it reads anything that kernel wrote. The primary lets its
// dependents launch early with griddep_launch_dependents(); without that they launch as it
// completes. (The runtime tracks the dependency; nothing spins on a flag.)
template <typename... Params, typename... Args>
cudaError_t launch_dependent(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                             Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<Args &&>(args)...);
}

// Device side of the above (no-ops for a kernel launched without the attribute).
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

}  // namespace dc
