// decode.cu -- split-KV attention for q_len == 1 (the decode step).
//
// DenseCore runs this case through its ordinary flash forward with a q block of one row
// (src/torch_attention.rs:157, q_split(1) -> 1) and a 512-key kv block. On a GPU the case is
// bound by HBM: every (batch, head) streams its whole K and V once and does 2 flops per
// loaded float. The design here:
//   * grid = (splits, H, B): each CTA streams a contiguous key range of one (batch, head);
//   * a group of G = D/16 lanes owns one key at a time; each lane loads 16 floats of the K
//     row and of the V row with four 128-bit loads (a group reads whole 64-byte-aligned
//     row segments, so each warp-wide load instruction covers whole 128-byte lines);
//   * each group keeps its own online-softmax state (max, sum, 16 accumulators per lane);
//   * the CTA merges its groups in shared memory and writes one partial (acc, max, sum);
//   * a second kernel merges the splits of each row by logsumexp and applies the
//     reference's finalisation (max -inf -> 0, sum 0 -> 1, out = acc/sum, lse = max+log sum,
//     torch_attention.rs:258-271).
#include <cuda_runtime.h>
#include <math.h>

#include "common.cuh"
#include "kernels.h"
#include "trace.h"

namespace dc {
namespace {

constexpr int DEC_WARPS = 8;
constexpr int DEC_THREADS = DEC_WARPS * 32;
constexpr int VEC = 16;  // floats per lane per row

__device__ __forceinline__ float4 ld_stream(const float *p) {
    float4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
                 : "l"(p));
    return r;
}

template <int D>
__global__ void __launch_bounds__(DEC_THREADS) decode_split_kernel(AttnProblem p, int splits,
                                                                   float *part) {
    constexpr int G = D / VEC;                 // lanes per key
    constexpr int GROUPS_PER_WARP = 32 / G;
    constexpr int GROUPS = DEC_WARPS * GROUPS_PER_WARP;
    __shared__ float s_acc[GROUPS][D];
    __shared__ float s_m[GROUPS], s_l[GROUPS];

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int gl = lane % G;                          // lane within the group
    const int group = warp * GROUPS_PER_WARP + lane / G;
    const int64_t b = blockIdx.z, h = blockIdx.y, hk = h / p.group;
    const int split = blockIdx.x;
    const int64_t per = (p.S + splits - 1) / splits;
    const int64_t k_begin = split * per;
    const int64_t k_end = min(p.S, k_begin + per);

    float q[VEC];
    {
        const float *qr = p.q + b * p.qs[0] + h * p.qs[1] + gl * VEC;
#pragma unroll
        for (int c = 0; c < VEC / 4; c++) {
            float4 t = *reinterpret_cast<const float4 *>(qr + 4 * c);
            q[4 * c] = t.x * p.scale;
            q[4 * c + 1] = t.y * p.scale;
            q[4 * c + 2] = t.z * p.scale;
            q[4 * c + 3] = t.w * p.scale;
        }
    }
    const float *kb = p.k + b * p.ks[0] + hk * p.ks[1] + gl * VEC;
    const float *vb = p.v + b * p.vs[0] + hk * p.vs[1] + gl * VEC;

    float m = -INFINITY, l = 0.0f, acc[VEC];
#pragma unroll
    for (int x = 0; x < VEC; x++) acc[x] = 0.0f;

    constexpr int UNROLL = 2;
    // The trip count is uniform over the CTA so that every lane reaches the shuffles.
    for (int64_t base = k_begin; base < k_end; base += (int64_t)GROUPS * UNROLL) {
        const int64_t j0 = base + group;
        float4 kv[UNROLL][VEC / 4], vv[UNROLL][VEC / 4];
        bool ok[UNROLL];
#pragma unroll
        for (int u = 0; u < UNROLL; u++) {
            const int64_t j = j0 + (int64_t)u * GROUPS;
            ok[u] = j < k_end;
            if (ok[u]) {
#pragma unroll
                for (int c = 0; c < VEC / 4; c++) kv[u][c] = ld_stream(kb + j * p.ks[2] + 4 * c);
#pragma unroll
                for (int c = 0; c < VEC / 4; c++) vv[u][c] = ld_stream(vb + j * p.vs[2] + 4 * c);
            } else {
#pragma unroll
                for (int c = 0; c < VEC / 4; c++) kv[u][c] = vv[u][c] = make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
#pragma unroll
        for (int u = 0; u < UNROLL; u++) {
            float dot = 0.0f;
#pragma unroll
            for (int c = 0; c < VEC / 4; c++) {
                dot = fmaf(q[4 * c], kv[u][c].x, dot);
                dot = fmaf(q[4 * c + 1], kv[u][c].y, dot);
                dot = fmaf(q[4 * c + 2], kv[u][c].z, dot);
                dot = fmaf(q[4 * c + 3], kv[u][c].w, dot);
            }
#pragma unroll
            for (int o = G / 2; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
            if (!ok[u]) continue;
            const int64_t j = j0 + (int64_t)u * GROUPS;
            float s = dot;
            if (p.mask_kind) s += mask_value(p, b, h, 0, j);
            const float m_new = fmaxf(m, s);
            if (m_new == -INFINITY) continue;
            const float corr = expf(m - m_new), pr = expf(s - m_new);
            l = fmaf(l, corr, pr);
            m = m_new;
#pragma unroll
            for (int c = 0; c < VEC / 4; c++) {
                acc[4 * c] = fmaf(pr, vv[u][c].x, acc[4 * c] * corr);
                acc[4 * c + 1] = fmaf(pr, vv[u][c].y, acc[4 * c + 1] * corr);
                acc[4 * c + 2] = fmaf(pr, vv[u][c].z, acc[4 * c + 2] * corr);
                acc[4 * c + 3] = fmaf(pr, vv[u][c].w, acc[4 * c + 3] * corr);
            }
        }
    }
    // Merge the groups of this CTA.
#pragma unroll
    for (int x = 0; x < VEC; x++) s_acc[group][gl * VEC + x] = acc[x];
    if (gl == 0) {
        s_m[group] = m;
        s_l[group] = l;
    }
    __syncthreads();
    float *dst = part + ((b * p.H + h) * splits + split) * (D + 2);
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
        float mx = -INFINITY;
        for (int g = 0; g < GROUPS; g++) mx = fmaxf(mx, s_m[g]);
        float a = 0.0f, ll = 0.0f;
        if (mx != -INFINITY) {
            for (int g = 0; g < GROUPS; g++) {
                if (s_m[g] == -INFINITY) continue;
                const float w = expf(s_m[g] - mx);
                a = fmaf(s_acc[g][d], w, a);
                ll = fmaf(s_l[g], w, ll);
            }
        }
        dst[d] = a;
        if (d == 0) {
            dst[D] = mx;
            dst[D + 1] = ll;
        }
    }
}

// One warp per (batch, head) row: merge its splits and finalise.
template <int D>
__global__ void decode_combine_kernel(AttnProblem p, int splits, const float *part) {
    const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (row >= p.B * p.H) return;
    const int64_t b = row / p.H, h = row % p.H;
    const float *src = part + row * splits * (D + 2);
    float mx = -INFINITY;
    for (int s = 0; s < splits; s++) mx = fmaxf(mx, src[s * (D + 2) + D]);
    float ll = 0.0f;
    float acc[D / 32];
#pragma unroll
    for (int t = 0; t < D / 32; t++) acc[t] = 0.0f;
    if (mx != -INFINITY) {
        for (int s = 0; s < splits; s++) {
            const float ms = src[s * (D + 2) + D];
            if (ms == -INFINITY) continue;
            const float w = expf(ms - mx);
            ll = fmaf(src[s * (D + 2) + D + 1], w, ll);
#pragma unroll
            for (int t = 0; t < D / 32; t++) acc[t] = fmaf(src[s * (D + 2) + lane + 32 * t], w, acc[t]);
        }
    }
    const float m_fin = mx == -INFINITY ? 0.0f : mx;
    const float l_fin = ll == 0.0f ? 1.0f : ll;
    const float recip = 1.0f / l_fin;
    float *orow = p.out + b * p.os[0] + h * p.os[1];
#pragma unroll
    for (int t = 0; t < D / 32; t++) orow[(lane + 32 * t) * p.os[3]] = acc[t] * recip;
    if (lane == 0) p.lse[b * p.ls[0] + h * p.ls[1]] = m_fin + logf(l_fin);
}

bool aligned16(const void *ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

}  // namespace

bool decode_supported(const AttnProblem &p) {
    if (p.L != 1 || p.causal) return false;
    if (p.E != p.Ev || (p.E != 64 && p.E != 128)) return false;
    if (p.qs[3] != 1 || p.ks[3] != 1 || p.vs[3] != 1) return false;
    if (p.ks[2] % 4 || p.vs[2] % 4 || p.ks[1] % 4 || p.vs[1] % 4 || p.ks[0] % 4 || p.vs[0] % 4)
        return false;
    if (p.qs[0] % 4 || p.qs[1] % 4) return false;
    return aligned16(p.q) && aligned16(p.k) && aligned16(p.v);
}

int decode_pick_splits(const AttnProblem &p) {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess)
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int64_t rows = p.B * p.H;
    const int64_t target = (int64_t)sms * 8 * 3;  // ~3 waves of 8 resident CTAs per SM
    int64_t splits = (target + rows - 1) / (rows > 0 ? rows : 1);
    const int64_t max_splits = (p.S + 255) / 256;  // keep >= 256 keys per CTA
    if (splits > max_splits) splits = max_splits;
    if (splits < 1) splits = 1;
    if (splits > 1024) splits = 1024;
    return (int)splits;
}

size_t decode_workspace_bytes(int64_t B, int64_t H, int64_t Ev, int splits) {
    return (size_t)B * H * splits * (Ev + 2) * sizeof(float);
}

int decode_forward(const AttnProblem &p, int splits, void *workspace, cudaStream_t stream) {
    float *part = static_cast<float *>(workspace);
    dim3 grid((unsigned)splits, (unsigned)p.H, (unsigned)p.B);
    const int64_t rows = p.B * p.H;
    const unsigned cgrid = (unsigned)((rows + 7) / 8);
    {
        KernelTrace tr("decode_split", stream);
        if (p.E == 64)
            decode_split_kernel<64><<<grid, DEC_THREADS, 0, stream>>>(p, splits, part);
        else
            decode_split_kernel<128><<<grid, DEC_THREADS, 0, stream>>>(p, splits, part);
        int st = check_launch("decode_split");
        if (st) return st;
    }
    KernelTrace tr("decode_combine", stream);
    if (p.E == 64)
        decode_combine_kernel<64><<<cgrid, 256, 0, stream>>>(p, splits, part);
    else
        decode_combine_kernel<128><<<cgrid, 256, 0, stream>>>(p, splits, part);
    return check_launch("decode_combine");
}

}  // namespace dc
