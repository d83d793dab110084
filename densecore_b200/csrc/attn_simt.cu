// attn_simt.cu -- CUDA-core (fp32 FMA) kernels of the SDPA path.
//
// These serve every shape the tcgen05 tensor-core kernels do not cover (any head dim up to
// 256, Ev != E, any strides) and DC_PREC_FP32 requests. They compute in plain fp32 with
// the same online-softmax rules as DenseCore's CPU flash path (src/torch_attention.rs):
//   * scores s = scale * q.k (+ additive mask); causal is top-left (:176-180, :202-207);
//   * running max m and sum l per row; a block whose max is -inf contributes nothing
//     (:218-226); l = l*exp(m - m') + sum(exp(s - m')) (:227-236);
//   * finalise: m == -inf -> 0, l == 0 -> 1, out = acc * (1/l), lse = m + log(l) (:258-271);
//   * backward recomputes P = exp(s - lse) (:363-374), dV += P^T dO, dP = dO V^T,
//     dS = P (dP - delta) with delta = sum(dO * O) per row (:327-330, :411-416),
//     dQ += scale dS K, dK += scale dS^T Q (:417-446).
// With dropout (AttnProblem::keep) the weights that meet V are P * Z, Z = keep_scale or 0 per
// element, while the softmax normaliser and lse stay those of P -- DenseCore's math path
// multiplies the softmax output by the noise (python/densecore/functional.py:336-340). The
// backward then uses dV += (P Z)^T dO and dS = P (Z dP - delta).
#include <cuda_runtime.h>
#include <math.h>

#include "common.cuh"
#include "kernels.h"
#include "trace.h"

namespace dc {
namespace {

constexpr int WARP = 32;

__device__ __forceinline__ float warp_max(float x) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o));
    return x;
}
__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    return x;
}

// ------------------------------------------------------------------------ forward ----
// CTA: 4 warps x 4 query rows; keys in blocks of 32 (one per lane); the output
// accumulator of a row is spread over the lanes (d = lane + 32 t).
constexpr int FW_WARPS = 4, FW_RPW = 4, FW_BQ = FW_WARPS * FW_RPW, FW_BK = 32;

template <int MAXE>
__global__ void __launch_bounds__(FW_WARPS *WARP) fwd_simt_kernel(AttnProblem p) {
    constexpr int T = MAXE / WARP;
    extern __shared__ float smem[];
    const int E = (int)p.E, Ev = (int)p.Ev, KP = E + 1, VP = Ev;
    float *sq = smem;                 // [FW_BQ][E]
    float *sk = sq + FW_BQ * E;       // [FW_BK][E+1]
    float *sv = sk + FW_BK * KP;      // [FW_BK][Ev]
    const int warp = threadIdx.x / WARP, lane = threadIdx.x % WARP;
    const int64_t b = blockIdx.z, h = blockIdx.y, hk = h / p.group;
    const int64_t q0 = (int64_t)blockIdx.x * FW_BQ;
    const float *qb = p.q + b * p.qs[0] + h * p.qs[1];
    const float *kb = p.k + b * p.ks[0] + hk * p.ks[1];
    const float *vb = p.v + b * p.vs[0] + hk * p.vs[1];

    for (int idx = threadIdx.x; idx < FW_BQ * E; idx += blockDim.x) {
        int r = idx / E, d = idx % E;
        int64_t i = q0 + r;
        sq[idx] = i < p.L ? qb[i * p.qs[2] + d * p.qs[3]] : 0.0f;
    }
    float m[FW_RPW], l[FW_RPW], acc[FW_RPW][T];
#pragma unroll
    for (int r = 0; r < FW_RPW; r++) {
        m[r] = -INFINITY;
        l[r] = 0.0f;
#pragma unroll
        for (int t = 0; t < T; t++) acc[r][t] = 0.0f;
    }
    int64_t num_keys = p.S;
    if (p.causal) num_keys = min(p.S, q0 + FW_BQ);
    for (int64_t n = 0; n < num_keys; n += FW_BK) {
        __syncthreads();
        for (int idx = threadIdx.x; idx < FW_BK * E; idx += blockDim.x) {
            int j = idx / E, d = idx % E;
            int64_t kj = n + j;
            sk[j * KP + d] = kj < p.S ? kb[kj * p.ks[2] + d * p.ks[3]] : 0.0f;
        }
        for (int idx = threadIdx.x; idx < FW_BK * Ev; idx += blockDim.x) {
            int j = idx / Ev, d = idx % Ev;
            int64_t kj = n + j;
            sv[j * VP + d] = kj < p.S ? vb[kj * p.vs[2] + d * p.vs[3]] : 0.0f;
        }
        __syncthreads();
        const int64_t kj = n + lane;
#pragma unroll
        for (int r = 0; r < FW_RPW; r++) {
            const int rr = warp * FW_RPW + r;
            const int64_t i = q0 + rr;
            float s = -INFINITY, z = 1.0f;
            if (i < p.L && kj < p.S && causal_visible(p.causal, i, kj)) {
                const float *qr = sq + rr * E, *kr = sk + lane * KP;
                float dot = 0.0f;
                for (int d = 0; d < E; d++) dot = fmaf(qr[d], kr[d], dot);
                s = dot * p.scale;
                if (p.mask_kind) s += mask_value(p, b, h, i, kj);
                z = keep_factor(p, b, h, i, kj);
            }
            const float m_new = fmaxf(m[r], warp_max(s));
            if (m_new == -INFINITY) continue;  // the block adds nothing (warp-uniform)
            const float pj = expf(s - m_new);
            const float corr = expf(m[r] - m_new);
            l[r] = fmaf(l[r], corr, warp_sum(pj));
            m[r] = m_new;
            const float pz = pj * z;
#pragma unroll
            for (int t = 0; t < T; t++) acc[r][t] *= corr;
            for (int j = 0; j < FW_BK; j++) {
                const float pb = __shfl_sync(0xffffffffu, pz, j);
                if (pb == 0.0f) continue;
                const float *vr = sv + j * VP;
#pragma unroll
                for (int t = 0; t < T; t++) {
                    const int d = lane + t * WARP;
                    if (d < Ev) acc[r][t] = fmaf(pb, vr[d], acc[r][t]);
                }
            }
        }
    }
#pragma unroll
    for (int r = 0; r < FW_RPW; r++) {
        const int64_t i = q0 + warp * FW_RPW + r;
        if (i >= p.L) continue;
        float mm = m[r] == -INFINITY ? 0.0f : m[r];
        float ll = l[r] == 0.0f ? 1.0f : l[r];
        const float recip = 1.0f / ll;
        float *orow = p.out + b * p.os[0] + h * p.os[1] + i * p.os[2];
#pragma unroll
        for (int t = 0; t < T; t++) {
            const int d = lane + t * WARP;
            if (d < Ev) orow[d * p.os[3]] = acc[r][t] * recip;
        }
        if (lane == 0) p.lse[b * p.ls[0] + h * p.ls[1] + i * p.ls[2]] = mm + logf(ll);
    }
}

// ---------------------------------------------------------------- backward: delta ----
// delta[b,h,i] = sum_d dO[b,h,i,d] * O[b,h,i,d]; one warp per row.
__global__ void bwd_delta_kernel(AttnProblem p, AttnGrads g) {
    const int64_t row = (int64_t)blockIdx.x * (blockDim.x / WARP) + threadIdx.x / WARP;
    const int lane = threadIdx.x % WARP;
    const int64_t rows = p.B * p.H * p.L;
    if (row >= rows) return;
    const int64_t i = row % p.L, bh = row / p.L, h = bh % p.H, b = bh / p.H;
    const float *o = p.out + b * p.os[0] + h * p.os[1] + i * p.os[2];
    const float *d = g.dout + b * g.dos[0] + h * g.dos[1] + i * g.dos[2];
    float s = 0.0f;
    for (int64_t x = lane; x < p.Ev; x += WARP) s = fmaf(d[x * g.dos[3]], o[x * p.os[3]], s);
    s = warp_sum(s);
    if (lane == 0) g.delta[row] = s;
}

// -------------------------------------------------------------- backward: dK, dV ----
// CTA: 32 keys (one per lane), 8 warps; query rows in blocks of 8 (one per warp).
constexpr int BK_KEYS = 32, BK_WARPS = 8, BK_ROWS = 8;

template <int MAXE>
__global__ void __launch_bounds__(BK_WARPS *WARP) bwd_dkdv_simt_kernel(AttnProblem p, AttnGrads g) {
    constexpr int U = MAXE / 8;
    extern __shared__ float smem[];
    const int E = (int)p.E, Ev = (int)p.Ev, KP = E + 1, VP = Ev + 1;
    float *sk = smem;                     // [32][E+1]
    float *sv = sk + BK_KEYS * KP;        // [32][Ev+1]
    float *sq = sv + BK_KEYS * VP;        // [8][E]
    float *sdo = sq + BK_ROWS * E;        // [8][Ev]
    float *sP = sdo + BK_ROWS * Ev;       // [8][32]
    float *sDS = sP + BK_ROWS * BK_KEYS;  // [8][32]
    float *srow = sDS + BK_ROWS * BK_KEYS;  // [8][2]: lse, delta
    const int warp = threadIdx.x / WARP, lane = threadIdx.x % WARP;
    const int64_t b = blockIdx.z, hk = blockIdx.y, k0 = (int64_t)blockIdx.x * BK_KEYS;
    const float *kb = p.k + b * p.ks[0] + hk * p.ks[1];
    const float *vb = p.v + b * p.vs[0] + hk * p.vs[1];
    for (int idx = threadIdx.x; idx < BK_KEYS * E; idx += blockDim.x) {
        int j = idx / E, d = idx % E;
        sk[j * KP + d] = k0 + j < p.S ? kb[(k0 + j) * p.ks[2] + d * p.ks[3]] : 0.0f;
    }
    for (int idx = threadIdx.x; idx < BK_KEYS * Ev; idx += blockDim.x) {
        int j = idx / Ev, d = idx % Ev;
        sv[j * VP + d] = k0 + j < p.S ? vb[(k0 + j) * p.vs[2] + d * p.vs[3]] : 0.0f;
    }
    // This thread accumulates key jj = lane at dims d = warp + 8u.
    float dk[U], dv[U];
#pragma unroll
    for (int u = 0; u < U; u++) dk[u] = dv[u] = 0.0f;
    const int64_t kj = k0 + lane;
    for (int gi = 0; gi < p.group; gi++) {
        const int64_t h = hk * p.group + gi;
        const float *qb = p.q + b * p.qs[0] + h * p.qs[1];
        const float *db = g.dout + b * g.dos[0] + h * g.dos[1];
        const float *lb = p.lse + b * p.ls[0] + h * p.ls[1];
        const float *deb = g.delta + (b * p.H + h) * p.L;
        const int64_t row_start = p.causal ? min(k0, p.L) : 0;
        for (int64_t r0 = row_start; r0 < p.L; r0 += BK_ROWS) {
            __syncthreads();
            for (int idx = threadIdx.x; idx < BK_ROWS * E; idx += blockDim.x) {
                int r = idx / E, d = idx % E;
                sq[idx] = r0 + r < p.L ? qb[(r0 + r) * p.qs[2] + d * p.qs[3]] : 0.0f;
            }
            for (int idx = threadIdx.x; idx < BK_ROWS * Ev; idx += blockDim.x) {
                int r = idx / Ev, d = idx % Ev;
                sdo[idx] = r0 + r < p.L ? db[(r0 + r) * g.dos[2] + d * g.dos[3]] : 0.0f;
            }
            if (threadIdx.x < BK_ROWS) {
                int64_t i = r0 + threadIdx.x;
                srow[2 * threadIdx.x] = i < p.L ? lb[i * p.ls[2]] : 0.0f;
                srow[2 * threadIdx.x + 1] = i < p.L ? deb[i] : 0.0f;
            }
            __syncthreads();
            {
                const int64_t i = r0 + warp;
                float pr = 0.0f, ds = 0.0f;
                if (i < p.L && kj < p.S && causal_visible(p.causal, i, kj)) {
                    const float *qr = sq + warp * E, *kr = sk + lane * KP;
                    float dot = 0.0f;
                    for (int d = 0; d < E; d++) dot = fmaf(qr[d], kr[d], dot);
                    float s = dot * p.scale;
                    if (p.mask_kind) s += mask_value(p, b, h, i, kj);
                    pr = expf(s - srow[2 * warp]);
                    const float *dr = sdo + warp * Ev, *vr = sv + lane * VP;
                    float dp = 0.0f;
                    for (int d = 0; d < Ev; d++) dp = fmaf(dr[d], vr[d], dp);
                    const float z = keep_factor(p, b, h, i, kj);
                    ds = pr * (dp * z - srow[2 * warp + 1]);
                    pr *= z;
                }
                sP[warp * BK_KEYS + lane] = pr;
                sDS[warp * BK_KEYS + lane] = ds;
            }
            __syncthreads();
#pragma unroll
            for (int r = 0; r < BK_ROWS; r++) {
                const float pr = sP[r * BK_KEYS + lane], ds = sDS[r * BK_KEYS + lane];
#pragma unroll
                for (int u = 0; u < U; u++) {
                    const int d = warp + 8 * u;
                    if (d < Ev) dv[u] = fmaf(pr, sdo[r * Ev + d], dv[u]);
                    if (d < E) dk[u] = fmaf(ds, sq[r * E + d], dk[u]);
                }
            }
        }
    }
    if (kj < p.S) {
        float *dkr = g.dk + b * g.dks[0] + hk * g.dks[1] + kj * g.dks[2];
        float *dvr = g.dv + b * g.dvs[0] + hk * g.dvs[1] + kj * g.dvs[2];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int d = warp + 8 * u;
            if (d < E) dkr[d * g.dks[3]] = dk[u] * p.scale;
            if (d < Ev) dvr[d * g.dvs[3]] = dv[u];
        }
    }
}

// ------------------------------------------------------------------- backward: dQ ----
// CTA: 8 query rows (one per warp), keys in blocks of 32 (one per lane).
template <int MAXE>
__global__ void __launch_bounds__(BK_WARPS *WARP) bwd_dq_simt_kernel(AttnProblem p, AttnGrads g) {
    constexpr int T = MAXE / WARP;
    extern __shared__ float smem[];
    const int E = (int)p.E, Ev = (int)p.Ev, KP = E + 1, VP = Ev + 1;
    float *sk = smem;                      // [32][E+1]
    float *sv = sk + BK_KEYS * KP;         // [32][Ev+1]
    float *sq = sv + BK_KEYS * VP;         // [8][E]
    float *sdo = sq + BK_ROWS * E;         // [8][Ev]
    float *sDS = sdo + BK_ROWS * Ev;       // [8][32]
    const int warp = threadIdx.x / WARP, lane = threadIdx.x % WARP;
    const int64_t b = blockIdx.z, h = blockIdx.y, hk = h / p.group;
    const int64_t q0 = (int64_t)blockIdx.x * BK_ROWS, i = q0 + warp;
    const float *qb = p.q + b * p.qs[0] + h * p.qs[1];
    const float *db = g.dout + b * g.dos[0] + h * g.dos[1];
    const float *kb = p.k + b * p.ks[0] + hk * p.ks[1];
    const float *vb = p.v + b * p.vs[0] + hk * p.vs[1];
    for (int idx = threadIdx.x; idx < BK_ROWS * E; idx += blockDim.x) {
        int r = idx / E, d = idx % E;
        sq[idx] = q0 + r < p.L ? qb[(q0 + r) * p.qs[2] + d * p.qs[3]] : 0.0f;
    }
    for (int idx = threadIdx.x; idx < BK_ROWS * Ev; idx += blockDim.x) {
        int r = idx / Ev, d = idx % Ev;
        sdo[idx] = q0 + r < p.L ? db[(q0 + r) * g.dos[2] + d * g.dos[3]] : 0.0f;
    }
    float lse_i = 0.0f, delta_i = 0.0f;
    if (i < p.L) {
        lse_i = p.lse[b * p.ls[0] + h * p.ls[1] + i * p.ls[2]];
        delta_i = g.delta[(b * p.H + h) * p.L + i];
    }
    float dq[T];
#pragma unroll
    for (int t = 0; t < T; t++) dq[t] = 0.0f;
    int64_t num_keys = p.S;
    if (p.causal) num_keys = min(p.S, q0 + BK_ROWS);
    for (int64_t n = 0; n < num_keys; n += BK_KEYS) {
        __syncthreads();
        for (int idx = threadIdx.x; idx < BK_KEYS * E; idx += blockDim.x) {
            int j = idx / E, d = idx % E;
            sk[j * KP + d] = n + j < p.S ? kb[(n + j) * p.ks[2] + d * p.ks[3]] : 0.0f;
        }
        for (int idx = threadIdx.x; idx < BK_KEYS * Ev; idx += blockDim.x) {
            int j = idx / Ev, d = idx % Ev;
            sv[j * VP + d] = n + j < p.S ? vb[(n + j) * p.vs[2] + d * p.vs[3]] : 0.0f;
        }
        __syncthreads();
        const int64_t kj = n + lane;
        float ds = 0.0f;
        if (i < p.L && kj < p.S && causal_visible(p.causal, i, kj)) {
            const float *qr = sq + warp * E, *kr = sk + lane * KP;
            float dot = 0.0f;
            for (int d = 0; d < E; d++) dot = fmaf(qr[d], kr[d], dot);
            float s = dot * p.scale;
            if (p.mask_kind) s += mask_value(p, b, h, i, kj);
            const float pr = expf(s - lse_i);
            const float *dr = sdo + warp * Ev, *vr = sv + lane * VP;
            float dp = 0.0f;
            for (int d = 0; d < Ev; d++) dp = fmaf(dr[d], vr[d], dp);
            ds = pr * (dp * keep_factor(p, b, h, i, kj) - delta_i);
        }
        sDS[warp * BK_KEYS + lane] = ds;
        __syncwarp();
        for (int j = 0; j < BK_KEYS; j++) {
            const float dsj = sDS[warp * BK_KEYS + j];
            if (dsj == 0.0f) continue;
            const float *kr = sk + j * KP;
#pragma unroll
            for (int t = 0; t < T; t++) {
                const int d = lane + t * WARP;
                if (d < E) dq[t] = fmaf(dsj, kr[d], dq[t]);
            }
        }
    }
    if (i < p.L) {
        float *dqr = g.dq + b * g.dqs[0] + h * g.dqs[1] + i * g.dqs[2];
#pragma unroll
        for (int t = 0; t < T; t++) {
            const int d = lane + t * WARP;
            if (d < E) dqr[d * g.dqs[3]] = dq[t] * p.scale;
        }
    }
}

// ------------------------------------------------------------- probabilities ----
// probs[b, (h,) i, j] = exp(scale q.k + mask - lse) (times the dropout factor); averaged over
// heads when requested.
__global__ void probs_kernel(AttnProblem p, float *probs, int64_t ps0, int64_t ps1, int64_t ps2,
                             int64_t ps3, int average) {
    const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t i = blockIdx.y, b = blockIdx.z;
    if (j >= p.S) return;
    float avg = 0.0f;
    for (int64_t h = 0; h < p.H; h++) {
        const int64_t hk = h / p.group;
        float pr = 0.0f;
        if (causal_visible(p.causal, i, j)) {
            const float *qr = p.q + b * p.qs[0] + h * p.qs[1] + i * p.qs[2];
            const float *kr = p.k + b * p.ks[0] + hk * p.ks[1] + j * p.ks[2];
            float dot = 0.0f;
            for (int64_t d = 0; d < p.E; d++) dot = fmaf(qr[d * p.qs[3]], kr[d * p.ks[3]], dot);
            float s = dot * p.scale;
            if (p.mask_kind) s += mask_value(p, b, h, i, j);
            pr = expf(s - p.lse[b * p.ls[0] + h * p.ls[1] + i * p.ls[2]]) * keep_factor(p, b, h, i, j);
        }
        if (average)
            avg += pr;
        else
            probs[b * ps0 + h * ps1 + i * ps2 + j * ps3] = pr;
    }
    if (average) probs[b * ps0 + i * ps2 + j * ps3] = avg / (float)p.H;
}

// --------------------------------------------------------------------- merge ----
// Logsumexp merge of a partial result into the accumulator, one warp per row.
__global__ void merge_kernel(float *oa, float *la, const float *op, const float *lp, int64_t B,
                             int64_t H, int64_t L, int64_t Ev, MergeStrides st) {
    const int64_t row = (int64_t)blockIdx.x * (blockDim.x / WARP) + threadIdx.x / WARP;
    const int lane = threadIdx.x % WARP;
    if (row >= B * H * L) return;
    const int64_t i = row % L, bh = row / L, h = bh % H, b = bh / H;
    float *lacc = la + b * st.las[0] + h * st.las[1] + i * st.las[2];
    const float lpart = lp[b * st.lps[0] + h * st.lps[1] + i * st.lps[2]];
    const float lold = *lacc;
    if (lpart == -INFINITY) return;
    float *orow = oa + b * st.oas[0] + h * st.oas[1] + i * st.oas[2];
    const float *prow = op + b * st.ops[0] + h * st.ops[1] + i * st.ops[2];
    const float mx = fmaxf(lold, lpart);
    const float wa = lold == -INFINITY ? 0.0f : expf(lold - mx);
    const float wp = expf(lpart - mx);
    const float lnew = mx + logf(wa + wp);
    const float ca = lold == -INFINITY ? 0.0f : expf(lold - lnew);
    const float cp = expf(lpart - lnew);
    for (int64_t d = lane; d < Ev; d += WARP) {
        const float a = lold == -INFINITY ? 0.0f : orow[d * st.oas[3]];
        orow[d * st.oas[3]] = a * ca + prow[d * st.ops[3]] * cp;
    }
    __syncwarp();
    if (lane == 0) *lacc = lnew;
}

template <int MAXE>
size_t fwd_smem(const AttnProblem &p) {
    return sizeof(float) * (FW_BQ * p.E + FW_BK * (p.E + 1) + FW_BK * p.Ev);
}
size_t bwd_dkdv_smem(const AttnProblem &p) {
    return sizeof(float) * (BK_KEYS * (p.E + 1) + BK_KEYS * (p.Ev + 1) + BK_ROWS * p.E +
                            BK_ROWS * p.Ev + 2 * BK_ROWS * BK_KEYS + 2 * BK_ROWS);
}
size_t bwd_dq_smem(const AttnProblem &p) {
    return sizeof(float) * (BK_KEYS * (p.E + 1) + BK_KEYS * (p.Ev + 1) + BK_ROWS * p.E +
                            BK_ROWS * p.Ev + BK_ROWS * BK_KEYS);
}

template <typename K>
int launch_dyn(K kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
               const char *what, const AttnProblem &p) {
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
        if (e != cudaSuccess) return cuda_fail(e, what);
    }
    KernelTrace tr(what, stream);
    kernel<<<grid, block, smem, stream>>>(p);
    return check_launch(what);
}

template <typename K>
int launch_dyn2(K kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                const char *what, const AttnProblem &p, const AttnGrads &g) {
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
        if (e != cudaSuccess) return cuda_fail(e, what);
    }
    KernelTrace tr(what, stream);
    kernel<<<grid, block, smem, stream>>>(p, g);
    return check_launch(what);
}

int maxe_of(const AttnProblem &p) {
    int64_t e = p.E > p.Ev ? p.E : p.Ev;
    return e <= 64 ? 64 : e <= 128 ? 128 : e <= 256 ? 256 : 0;
}

}  // namespace

int simt_forward(const AttnProblem &p, cudaStream_t stream) {
    dim3 grid((unsigned)((p.L + FW_BQ - 1) / FW_BQ), (unsigned)p.H, (unsigned)p.B);
    dim3 block(FW_WARPS * WARP);
    switch (maxe_of(p)) {
        case 64: return launch_dyn(fwd_simt_kernel<64>, grid, block, fwd_smem<64>(p), stream, "fwd_simt", p);
        case 128: return launch_dyn(fwd_simt_kernel<128>, grid, block, fwd_smem<128>(p), stream, "fwd_simt", p);
        case 256: return launch_dyn(fwd_simt_kernel<256>, grid, block, fwd_smem<256>(p), stream, "fwd_simt", p);
    }
    return fail(DC_ERR_UNSUPPORTED, "head dim above 256 is not supported");
}

int simt_backward(const AttnProblem &p, const AttnGrads &g, cudaStream_t stream) {
    const int maxe = maxe_of(p);
    if (!maxe) return fail(DC_ERR_UNSUPPORTED, "head dim above 256 is not supported");
    dim3 block(BK_WARPS * WARP);
    dim3 gk((unsigned)((p.S + BK_KEYS - 1) / BK_KEYS), (unsigned)p.Hkv, (unsigned)p.B);
    dim3 gq((unsigned)((p.L + BK_ROWS - 1) / BK_ROWS), (unsigned)p.H, (unsigned)p.B);
    const bool run_kv = p.S > 0, run_q = p.L > 0;  // empty grids are not launched
    int st = DC_OK;
    switch (maxe) {
        case 64:
            if (run_kv) st = launch_dyn2(bwd_dkdv_simt_kernel<64>, gk, block, bwd_dkdv_smem(p), stream, "bwd_dkdv_simt", p, g);
            if (!st && run_q) st = launch_dyn2(bwd_dq_simt_kernel<64>, gq, block, bwd_dq_smem(p), stream, "bwd_dq_simt", p, g);
            break;
        case 128:
            if (run_kv) st = launch_dyn2(bwd_dkdv_simt_kernel<128>, gk, block, bwd_dkdv_smem(p), stream, "bwd_dkdv_simt", p, g);
            if (!st && run_q) st = launch_dyn2(bwd_dq_simt_kernel<128>, gq, block, bwd_dq_smem(p), stream, "bwd_dq_simt", p, g);
            break;
        default:
            if (run_kv) st = launch_dyn2(bwd_dkdv_simt_kernel<256>, gk, block, bwd_dkdv_smem(p), stream, "bwd_dkdv_simt", p, g);
            if (!st && run_q) st = launch_dyn2(bwd_dq_simt_kernel<256>, gq, block, bwd_dq_smem(p), stream, "bwd_dq_simt", p, g);
            break;
    }
    return st;
}

int bwd_delta(const AttnProblem &p, const AttnGrads &g, cudaStream_t stream) {
    const int64_t rows = p.B * p.H * p.L;
    const int per = 8;
    KernelTrace tr("bwd_delta", stream);
    bwd_delta_kernel<<<(unsigned)((rows + per - 1) / per), per * WARP, 0, stream>>>(p, g);
    return check_launch("bwd_delta");
}

int simt_probs(const AttnProblem &p, float *probs, const int64_t ps[4], int average,
               cudaStream_t stream) {
    dim3 grid((unsigned)((p.S + 127) / 128), (unsigned)p.L, (unsigned)p.B);
    KernelTrace tr("attn_probs", stream);
    probs_kernel<<<grid, 128, 0, stream>>>(p, probs, ps[0], ps[1], ps[2], ps[3], average);
    return check_launch("attn_probs");
}

int merge(float *oa, float *la, const float *op, const float *lp, int64_t B, int64_t H,
          int64_t L, int64_t Ev, const MergeStrides &st, cudaStream_t stream) {
    const int64_t rows = B * H * L;
    const int per = 8;
    KernelTrace tr("attn_merge", stream);
    merge_kernel<<<(unsigned)((rows + per - 1) / per), per * WARP, 0, stream>>>(oa, la, op, lp, B, H,
                                                                                  L, Ev, st);
    return check_launch("attn_merge");
}

}  // namespace dc
