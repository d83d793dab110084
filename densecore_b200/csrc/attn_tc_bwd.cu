// attn_tc_bwd.cu -- tcgen05 tensor-core attention backward for sm_100a (head dim 64).
//
// Replaces DenseCore's torch_attention::backward (src/torch_attention.rs:291-468), which per
// (q block, kv block) recomputes P = exp(scale*S + mask - lse) (:338-380) and accumulates
//   dV += P^T dO, dP = dO V^T, dS = P (dP - delta), dQ += scale dS K, dK += scale dS^T Q
// (:381-446), with delta = sum(dO * O) per row (:327-330, computed by bwd_delta_kernel).
//
// Two kernels, so every accumulator has one owner and no atomics are needed:
//
//   dkdv: a CTA owns 128 keys of one (batch, kv head). K and V are the A operands: tf32 hi in
//         TMEM, lo in shared memory. 32-row blocks of Q and dO stream through shared memory,
//         each in two layouts (128-byte swizzle for the K-major use, 32-byte-atom swizzle for
//         the MN-major use that tf32 requires). Per block i: S^T = K Q^T and dP^T = V dO^T
//         into one of two TMEM buffers; the softmax threads (one per key) turn them into P^T
//         and dS^T (tf32 hi / lo, in place); then dV_blk += P^T dO and dK_blk += dS^T Q.
//         Issue order S0, S1, G0, S2, G1, ... keeps the tensor core busy while the softmax
//         threads work. Fold threads add the block accumulators into fp32 registers every
//         FOLD blocks (the tensor core's accumulation is coarser than fp32 over long chains).
//   dq:   a CTA owns 128 query rows of one (batch, head). Q and dO are the A operands (hi in
//         TMEM, lo in shared memory); 32-key blocks of K (two layouts) and V stream through
//         shared memory. Per block: S = Q K^T and dP = dO V^T, dS in TMEM, dQ_blk += dS K;
//         the fold threads keep dQ in fp32 registers.
//
// Roles: warps 0-3 softmax (one TMEM lane each); fold warps (dq: 4-7 for dQ; dkdv: 4-7 for
// dV and 8-11 for dK, one lane each); converter warps (fp32 -> tf32 hi / lo; per-block lse and
// delta into shared memory; dq: four, which also load Q / dO into TMEM; dkdv: two, the
// softmax warps load K / V); one TMA producer warp; one MMA issuer warp (also the TMEM owner).
// No SM sub-partition holds more than four warps, so a thread may use 128 registers. Every
// wait is bounded; on a timeout the kernel records an error and unwinds.
#include <cuda.h>
#include <cuda_runtime.h>
#include <math.h>

#include "common.cuh"
#include "kernels.h"
#include "sm100.cuh"
#include "tma_host.h"
#include "trace.h"

namespace dc {
namespace {

using namespace sm100;

constexpr float LOG2E = 1.4426950408889634f;
constexpr int D = 64;        // head dim of these kernels
constexpr int CHUNKS = D / 32;
constexpr int TILE = 128;    // rows owned by a CTA (the MMA M)
constexpr int BLK = 32;      // streamed rows per step (the MMA N of S / dP, the K of the rest)
constexpr int FOLD = 2;      // blocks per tensor-core accumulation chain

constexpr uint32_t RES_BYTES = TILE * D * 4;      // one resident fp32 tile (32 KB)
constexpr uint32_t RES_CHUNK = TILE * 128;        // 16 KB per 32-column chunk
constexpr uint32_t BLK_BYTES = BLK * D * 4;       // one streamed fp32 tile (8 KB)
constexpr uint32_t BLK_CHUNK = BLK * 128;         // 4 KB per chunk

constexpr uint32_t IDESC_S = idesc_tf32(128, BLK, 0, 0);  // S / dP: N = 32, both K-major
constexpr uint32_t IDESC_G = idesc_tf32(128, D, 0, 1);    // gradients: N = 64, B MN-major

// k-step offsets in 16-byte units: K-major 128-byte swizzle (8 tf32 = 32 bytes per k-step,
// 4 k-steps per 128-byte chunk of `chunk` bytes) and MN-major 32-byte-atom swizzle (a k-step
// is 8 rows = 1024 bytes).
template <uint32_t CHUNK>
__device__ __forceinline__ constexpr uint32_t koff(int kk) {
    return (uint32_t)(((kk >> 2) * CHUNK + (kk & 3) * 32) >> 4);
}
__device__ __forceinline__ constexpr uint32_t mnoff(int kk) { return (uint32_t)(kk * 64); }

// S-type product over D (3 passes with SPLIT, cross terms first):
//   d = A_hi B_lo + A_lo B_hi + A_hi B_hi,
// A_hi in TMEM (columns a_hi + 8 kk), A_lo in shared memory (K-major, descriptor a_lo),
// B hi / lo K-major in shared memory (descriptor b_hi, lo BLK_BYTES further).
template <bool SPLIT>
__device__ __forceinline__ void mma_s(uint32_t d, uint32_t a_hi, uint64_t a_lo, uint64_t b_hi) {
    constexpr uint32_t BLO = BLK_BYTES >> 4;
    if (SPLIT) {
#pragma unroll
        for (int kk = 0; kk < D / 8; kk++) {
            mma_tf32_ts(d, a_hi + kk * 8, b_hi + (BLO + koff<BLK_CHUNK>(kk)), IDESC_S, kk > 0 ? 1u : 0u);
            mma_tf32_ss(d, a_lo + koff<RES_CHUNK>(kk), b_hi + koff<BLK_CHUNK>(kk), IDESC_S, 1u);
        }
    }
#pragma unroll
    for (int kk = 0; kk < D / 8; kk++)
        mma_tf32_ts(d, a_hi + kk * 8, b_hi + koff<BLK_CHUNK>(kk), IDESC_S, (SPLIT || kk > 0) ? 1u : 0u);
}

// Gradient-type product over BLK (3 passes with SPLIT): d (+)= A B with A hi / lo in TMEM and
// B hi / lo MN-major in shared memory (descriptor b_hi, lo BLK_BYTES further).
template <bool SPLIT>
__device__ __forceinline__ void mma_g(uint32_t d, uint32_t a_hi, uint32_t a_lo, uint64_t b_hi, bool accumulate) {
    constexpr uint32_t BLO = BLK_BYTES >> 4;
    if (SPLIT) {
#pragma unroll
        for (int kk = 0; kk < BLK / 8; kk++) {
            mma_tf32_ts(d, a_hi + kk * 8, b_hi + (BLO + mnoff(kk)), IDESC_G, (accumulate || kk > 0) ? 1u : 0u);
            mma_tf32_ts(d, a_lo + kk * 8, b_hi + mnoff(kk), IDESC_G, 1u);
        }
    }
#pragma unroll
    for (int kk = 0; kk < BLK / 8; kk++)
        mma_tf32_ts(d, a_hi + kk * 8, b_hi + mnoff(kk), IDESC_G, (accumulate || SPLIT || kk > 0) ? 1u : 0u);
}

// Row `row` of a raw 128-byte-swizzled TILE-row tile: tf32 hi into TMEM (col_hi, this lane)
// and, with SPLIT, lo into `lo` at the same swizzled position. A full warp calls it.
template <bool SPLIT>
__device__ __forceinline__ void row_split(const uint8_t *raw, uint8_t *lo, int row, uint32_t tlane,
                                          uint32_t col_hi) {
#pragma unroll
    for (int c = 0; c < CHUNKS; c++) {
        uint32_t hi[32];
#pragma unroll
        for (int g = 0; g < 8; g++) {
            const uint32_t off = c * RES_CHUNK + row * 128 + ((g ^ (row & 7)) * 16);
            const float4 x = *reinterpret_cast<const float4 *>(raw + off);
            const float v[4] = {x.x, x.y, x.z, x.w};
            float4 lv;
            float *lp = &lv.x;
#pragma unroll
            for (int e = 0; e < 4; e++) {
                hi[4 * g + e] = tf32_rna(v[e]);
                lp[e] = __uint_as_float(tf32_rna(v[e] - __uint_as_float(hi[4 * g + e])));
            }
            if (SPLIT) *reinterpret_cast<float4 *>(lo + off) = lv;
        }
        tmem_st32(tlane + col_hi + 32 * c, hi);
    }
}

// hi = tf32(x) in place and, with SPLIT, lo = tf32(x - hi) BLK_BYTES further, over a tile
// (NT threads).
template <bool SPLIT, int NT = 128>
__device__ __forceinline__ void split_tile(uint8_t *hi, int t) {
    for (uint32_t i = t; i < BLK_BYTES / 16; i += NT) {
        float4 *ph = reinterpret_cast<float4 *>(hi) + i;
        const float4 x = *ph;
        float4 hv;
        hv.x = __uint_as_float(tf32_rna(x.x));
        hv.y = __uint_as_float(tf32_rna(x.y));
        hv.z = __uint_as_float(tf32_rna(x.z));
        hv.w = __uint_as_float(tf32_rna(x.w));
        *ph = hv;
        if (SPLIT) {
            float4 lv;
            lv.x = __uint_as_float(tf32_rna(x.x - hv.x));
            lv.y = __uint_as_float(tf32_rna(x.y - hv.y));
            lv.z = __uint_as_float(tf32_rna(x.z - hv.z));
            lv.w = __uint_as_float(tf32_rna(x.w - hv.w));
            *(reinterpret_cast<float4 *>(hi + BLK_BYTES) + i) = lv;
        }
    }
}

struct TcBwdArgs {
    AttnProblem p;
    AttnGrads g;
    float scale_log2;
    int *err;
};

// ==================================================================== dK / dV ========
namespace kv {
constexpr int NST = 2;
// 16 warps (4 per SM sub-partition, so up to 128 registers per thread).
constexpr int THREADS = 512;
constexpr int W_DVF = 4, W_DKF = 8, W_CVT = 12, N_CVT = 64, W_PROD = 14, W_MMA = 15;
// stage: Q_K hi, lo | Q_MN hi, lo | dO_K hi, lo | dO_MN hi, lo (8 KB each) | lse2[32], delta[32]
constexpr uint32_t ST_QK = 0, ST_QMN = 2 * BLK_BYTES, ST_DOK = 4 * BLK_BYTES, ST_DOMN = 6 * BLK_BYTES,
                   ST_ROWS = 8 * BLK_BYTES;
constexpr uint32_t STAGE_BYTES = 8 * BLK_BYTES + 1024;  // 1024-byte aligned stages
constexpr uint32_t OFF_KLO = NST * STAGE_BYTES, OFF_VLO = OFF_KLO + RES_BYTES;
constexpr uint32_t OFF_BAR = OFF_VLO + RES_BYTES;
// G_DONE[b]: the gradient MMAs that read buffer b finished (guards its reuse); CHAIN_DONE:
// the last gradient MMAs of an accumulation chain finished (the fold may read); BLK_FREE: the
// fold has read the block accumulators (the next chain may overwrite them).
enum { KV_FULL, KV_READY, ST_FULL, ST_READY = ST_FULL + NST, ST_EMPTY = ST_READY + NST,
       S_FULL = ST_EMPTY + NST, P_FULL = S_FULL + 2, G_DONE = P_FULL + 2, CHAIN_DONE = G_DONE + 2, BLK_FREE,
       DRAIN, NBAR };
constexpr uint32_t OFF_MISC = OFF_BAR + NBAR * 8;
constexpr uint32_t SMEM = OFF_MISC + 16 + 1024;
// TMEM: K hi | V hi | 2 x (S^T / P^T hi, P^T lo, dP^T / dS^T hi, dS^T lo) | dV_blk | dK_blk
constexpr uint32_t C_KHI = 0, C_VHI = 64, C_DV = 384, C_DK = 448, TCOLS = 512;
__device__ __forceinline__ constexpr uint32_t c_s(int b) { return 128 + b * 128; }
__device__ __forceinline__ constexpr uint32_t c_plo(int b) { return 160 + b * 128; }
__device__ __forceinline__ constexpr uint32_t c_dp(int b) { return 192 + b * 128; }
__device__ __forceinline__ constexpr uint32_t c_dslo(int b) { return 224 + b * 128; }
static_assert(2 * RES_BYTES <= STAGE_BYTES, "the raw K / V tiles are staged in stage 0");
static_assert(SMEM <= 232448, "smem");
}  // namespace kv

template <bool SPLIT>
__global__ void __maxnreg__(128)
    attn_bwd_dkdv_tc_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                            const __grid_constant__ CUtensorMap tm_qk, const __grid_constant__ CUtensorMap tm_qmn,
                            const __grid_constant__ CUtensorMap tm_dok, const __grid_constant__ CUtensorMap tm_domn,
                            const TcBwdArgs a) {
    using namespace kv;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_addr(smem_raw);
    const uint32_t sb = (raw + 1023u) & ~1023u;
    uint8_t *sg = smem_raw + (sb - raw);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const AttnProblem &p = a.p;
    const int64_t hk = blockIdx.y, b = blockIdx.z, k0 = (int64_t)blockIdx.x * TILE;
    // Query blocks this CTA visits: for each query head of the group, rows [r_begin, L).
    const int64_t r_begin = p.causal ? min(k0, p.L) : 0;
    const int qb_first = (int)(r_begin / BLK);
    const int qb_per_head = (int)((p.L + BLK - 1) / BLK) - qb_first;
    const int nblk = qb_per_head * p.group;
    auto bar = [&](int i) { return sb + OFF_BAR + 8u * (uint32_t)i; };
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(sg + OFF_MISC);
    volatile int *abort = reinterpret_cast<volatile int *>(sg + OFF_MISC + 4);
    int *err = a.err;
    auto blk_coords = [&](int i, int64_t &h, int64_t &q0) {
        h = hk * p.group + i / qb_per_head;
        q0 = (int64_t)(qb_first + i % qb_per_head) * BLK;
    };

    if (threadIdx.x == 0) {
        mbar_init(bar(KV_FULL), 1);
        mbar_init(bar(KV_READY), 128);
        for (int s = 0; s < NST; s++) {
            mbar_init(bar(ST_FULL + s), 1);
            mbar_init(bar(ST_READY + s), N_CVT);
            mbar_init(bar(ST_EMPTY + s), 1);
        }
        for (int s = 0; s < 2; s++) {
            mbar_init(bar(S_FULL + s), 1);
            mbar_init(bar(P_FULL + s), 128);
        }
        mbar_init(bar(G_DONE), 1);
        mbar_init(bar(G_DONE + 1), 1);
        mbar_init(bar(CHAIN_DONE), 1);
        mbar_init(bar(BLK_FREE), 256);  // both fold groups
        mbar_init(bar(DRAIN), 1);
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == W_MMA) {
        tmem_alloc(smem_addr(tmem_slot), TCOLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == W_PROD) {
        // ---------------------------------------------------------------- producer ----
        if (lane == 0) {
            int issued = -1;
            // K and V of the CTA, raw, into stage 0 (K at 0, V at RES_BYTES).
            mbar_expect_tx(bar(KV_FULL), 2 * RES_BYTES);
            for (int c = 0; c < CHUNKS; c++) {
                tma_load_4d(&tm_k, sb + c * RES_CHUNK, bar(KV_FULL), 32 * c, (int)k0, (int)hk, (int)b);
                tma_load_4d(&tm_v, sb + RES_BYTES + c * RES_CHUNK, bar(KV_FULL), 32 * c, (int)k0, (int)hk, (int)b);
            }
            bool ok = mbar_wait(bar(KV_READY), 0, abort, err);
            for (int i = 0; ok && i < nblk; i++) {
                const int s = i % NST;
                if (i >= NST && !mbar_wait(bar(ST_EMPTY + s), ((i / NST) - 1) & 1, abort, err)) break;
                int64_t h, q0;
                blk_coords(i, h, q0);
                const uint32_t st = sb + s * STAGE_BYTES;
                mbar_expect_tx(bar(ST_FULL + s), 4 * BLK_BYTES);
                for (int c = 0; c < CHUNKS; c++) {
                    tma_load_4d(&tm_qk, st + ST_QK + c * BLK_CHUNK, bar(ST_FULL + s), 32 * c, (int)q0, (int)h, (int)b);
                    tma_load_4d(&tm_qmn, st + ST_QMN + c * BLK_CHUNK, bar(ST_FULL + s), 32 * c, (int)q0, (int)h, (int)b);
                    tma_load_4d(&tm_dok, st + ST_DOK + c * BLK_CHUNK, bar(ST_FULL + s), 32 * c, (int)q0, (int)h, (int)b);
                    tma_load_4d(&tm_domn, st + ST_DOMN + c * BLK_CHUNK, bar(ST_FULL + s), 32 * c, (int)q0, (int)h, (int)b);
                }
                issued = i;
            }
            if (*abort) {
                volatile int never = 0;
                mbar_wait(bar(KV_FULL), 0, &never, nullptr);
                for (int i = max(0, issued - NST + 1); i <= issued; i++)
                    mbar_wait(bar(ST_FULL + i % NST), (i / NST) & 1, &never, nullptr);
            }
        }
    } else if (warp == W_MMA) {
        // ------------------------------------------------------------------ MMA ------
        if (lane == 0) {
            const uint64_t klo = sdesc_sw128(sb + OFF_KLO, 16, 1024), vlo = sdesc_sw128(sb + OFF_VLO, 16, 1024);
            auto issue_g = [&](int i) -> bool {  // gradients of block i
                const int s = i % NST, bb = i & 1;
                const uint32_t st = sb + s * STAGE_BYTES;
                if (!mbar_wait(bar(P_FULL + bb), (i >> 1) & 1, abort, err)) return false;
                const bool first = (i % FOLD) == 0;
                if (first && i >= FOLD && !mbar_wait(bar(BLK_FREE), ((i / FOLD) - 1) & 1, abort, err)) return false;
                tc_fence_after();
                mma_g<SPLIT>(tmem + C_DV, tmem + c_s(bb), tmem + c_plo(bb), sdesc_mn_sw128_32b(st + ST_DOMN, BLK_CHUNK, 512),
                             !first);
                mma_g<SPLIT>(tmem + C_DK, tmem + c_dp(bb), tmem + c_dslo(bb),
                             sdesc_mn_sw128_32b(st + ST_QMN, BLK_CHUNK, 512), !first);
                tc_commit(bar(G_DONE + bb));
                if ((i % FOLD) == FOLD - 1 || i == nblk - 1) tc_commit(bar(CHAIN_DONE));
                tc_commit(bar(ST_EMPTY + s));
                return true;
            };
            bool ok = mbar_wait(bar(KV_READY), 0, abort, err);
            tc_fence_after();
            for (int i = 0; ok && i < nblk; i++) {
                const int s = i % NST, bb = i & 1;
                const uint32_t st = sb + s * STAGE_BYTES;
                if (!mbar_wait(bar(ST_READY + s), (i / NST) & 1, abort, err)) break;
                // Buffer bb holds P^T / dS^T of block i-2 until its gradient MMAs finish.
                if (i >= 2 && !mbar_wait(bar(G_DONE + bb), ((i - 2) >> 1) & 1, abort, err)) break;
                tc_fence_after();
                mma_s<SPLIT>(tmem + c_s(bb), tmem + C_KHI, klo, sdesc_sw128(st + ST_QK, 16, 1024));
                mma_s<SPLIT>(tmem + c_dp(bb), tmem + C_VHI, vlo, sdesc_sw128(st + ST_DOK, 16, 1024));
                tc_commit(bar(S_FULL + bb));
                if (i >= 1 && !issue_g(i - 1)) {
                    ok = false;
                    break;
                }
            }
            if (ok && nblk > 0) issue_g(nblk - 1);
            tc_commit(bar(DRAIN));
            volatile int never = 0;
            mbar_wait(bar(DRAIN), 0, &never, nullptr);
        }
    } else if (warp >= W_CVT) {
        // ------------------------------------------------------------- converters -----
        const int ct = threadIdx.x - 32 * W_CVT;
        if (mbar_wait(bar(KV_READY), 0, abort, err)) {  // stage 0 is free of the raw K / V
            for (int i = 0; i < nblk; i++) {
                const int s = i % NST;
                if (!mbar_wait(bar(ST_FULL + s), (i / NST) & 1, abort, err)) break;
                uint8_t *st = sg + s * STAGE_BYTES;
                split_tile<SPLIT, N_CVT>(st + ST_QK, ct);
                split_tile<SPLIT, N_CVT>(st + ST_QMN, ct);
                split_tile<SPLIT, N_CVT>(st + ST_DOK, ct);
                split_tile<SPLIT, N_CVT>(st + ST_DOMN, ct);
                if (ct < BLK) {  // this block's lse (in base 2) and delta, one row per thread
                    int64_t h, q0;
                    blk_coords(i, h, q0);
                    const int64_t q = q0 + ct;
                    float *rows = reinterpret_cast<float *>(st + ST_ROWS);
                    rows[ct] = q < p.L ? p.lse[b * p.ls[0] + h * p.ls[1] + q * p.ls[2]] * LOG2E : 0.0f;
                    rows[BLK + ct] = q < p.L ? a.g.delta[(b * p.H + h) * p.L + q] : 0.0f;
                }
                fence_proxy_async_smem();
                mbar_arrive(bar(ST_READY + s));
            }
        }
    } else if (warp >= W_DVF) {
        // ------------------------------------------ fold: fp32 dV (4-7) and dK (8-11) --
        const bool is_dk = warp >= W_DKF;
        const int row = threadIdx.x - 32 * (is_dk ? W_DKF : W_DVF);  // key row (lane quadrant warp & 3)
        const int64_t key = k0 + row;
        const uint32_t tl = tmem + ((uint32_t)((warp & 3) * 32) << 16);
        const uint32_t col = is_dk ? C_DK : C_DV;
        float acc[D];
#pragma unroll
        for (int x = 0; x < D; x++) acc[x] = 0.0f;
        bool ok = true;
        const int nchain = (nblk + FOLD - 1) / FOLD;
        for (int ch = 0; ch < nchain; ch++) {
            if (!mbar_wait(bar(CHAIN_DONE), ch & 1, abort, err)) {
                ok = false;
                break;
            }
            tc_fence_after();
#pragma unroll
            for (int c = 0; c < D / 16; c++) {
                uint32_t r[16];
                tmem_ld16(tl + col + 16 * c, r);
                tmem_wait_ld();
#pragma unroll
                for (int x = 0; x < 16; x++) acc[16 * c + x] += __uint_as_float(r[x]);
            }
            tc_fence_before();
            mbar_arrive(bar(BLK_FREE));
        }
        const bool aborted = __any_sync(0xffffffffu, *abort != 0);
        if (ok && !aborted && key < p.S) {
            if (is_dk) {
                float *dkr = a.g.dk + b * a.g.dks[0] + hk * a.g.dks[1] + key * a.g.dks[2];
#pragma unroll
                for (int c = 0; c < D; c++) dkr[c * a.g.dks[3]] = acc[c] * p.scale;
            } else {
                float *dvr = a.g.dv + b * a.g.dvs[0] + hk * a.g.dvs[1] + key * a.g.dvs[2];
#pragma unroll
                for (int c = 0; c < D; c++) dvr[c * a.g.dvs[3]] = acc[c];
            }
        }
    } else {
        // ---------------------------------------------------------- P^T and dS^T ------
        const int row = threadIdx.x;  // key row of this CTA
        const int64_t key = k0 + row;
        const bool key_ok = key < p.S;
        const uint32_t tl = tmem + ((uint32_t)(warp * 32) << 16);
        // First, this CTA's K and V rows into TMEM (hi) and shared memory (lo).
        if (!mbar_wait(bar(KV_FULL), 0, abort, err)) goto done;
        row_split<SPLIT>(sg, sg + OFF_KLO, row, tl, C_KHI);
        row_split<SPLIT>(sg + RES_BYTES, sg + OFF_VLO, row, tl, C_VHI);
        tmem_wait_st();
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(bar(KV_READY));
        for (int i = 0; i < nblk; i++) {
            const int s = i % NST, bb = i & 1;
            int64_t h, q0;
            blk_coords(i, h, q0);
            if (!mbar_wait(bar(S_FULL + bb), (i >> 1) & 1, abort, err)) break;
            if (!mbar_wait(bar(ST_READY + s), (i / NST) & 1, abort, err)) break;  // lse / delta visible
            tc_fence_after();
            const float4 *rows = reinterpret_cast<const float4 *>(sg + s * STAGE_BYTES + ST_ROWS);
            const bool edge = !key_ok || q0 + BLK > p.L || (p.causal && key > q0) || p.mask_kind != MASK_NONE;
#pragma unroll
            for (int hf = 0; hf < 2; hf++) {  // 16 query columns at a time
                uint32_t sr[16], dr[16], phi[16], plo[16];
                tmem_ld16(tl + c_s(bb) + 16 * hf, sr);
                tmem_ld16(tl + c_dp(bb) + 16 * hf, dr);
                const float *lse2 = reinterpret_cast<const float *>(rows) + 16 * hf;
                const float *del = reinterpret_cast<const float *>(rows) + BLK + 16 * hf;
                tmem_wait_ld();
#pragma unroll
                for (int c = 0; c < 16; c++) {
                    float x = __uint_as_float(sr[c]) * a.scale_log2;
                    bool valid = true;
                    if (edge) {
                        const int64_t q = q0 + 16 * hf + c;
                        valid = key_ok && q < p.L && !(p.causal && key > q);
                        if (valid && p.mask_kind != MASK_NONE) x += mask_value(p, b, h, q, key) * LOG2E;
                    }
                    const float pc = valid ? ex2_approx(x - lse2[c]) : 0.0f;
                    const float ds = pc * (__uint_as_float(dr[c]) - del[c]);
                    phi[c] = tf32_rna(pc);
                    sr[c] = tf32_rna(ds);
                    if (SPLIT) {
                        plo[c] = tf32_rna(pc - __uint_as_float(phi[c]));
                        dr[c] = tf32_rna(ds - __uint_as_float(sr[c]));
                    }
                }
                tmem_st16(tl + c_s(bb) + 16 * hf, phi);
                tmem_st16(tl + c_dp(bb) + 16 * hf, sr);
                if (SPLIT) {
                    tmem_st16(tl + c_plo(bb) + 16 * hf, plo);
                    tmem_st16(tl + c_dslo(bb) + 16 * hf, dr);
                }
            }
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(bar(P_FULL + bb));
        }
    done:;
    }

    tc_fence_before();
    __syncthreads();
    if (warp == W_MMA) {
        tc_fence_after();
        tmem_dealloc(tmem, kv::TCOLS);
    }
}

// ========================================================================= dQ ========
namespace qq {
constexpr int NST = 3;
constexpr int THREADS = 448;
constexpr int W_FOLD = 4, W_PROD = 8, W_MMA = 9, W_CVT = 10;
// stage: K_K hi, lo | K_MN hi, lo | V_K hi, lo  (8 KB each)
constexpr uint32_t ST_KK = 0, ST_KMN = 2 * BLK_BYTES, ST_VK = 4 * BLK_BYTES;
constexpr uint32_t STAGE_BYTES = 6 * BLK_BYTES;  // 48 KB
constexpr uint32_t OFF_QLO = NST * STAGE_BYTES, OFF_DOLO = OFF_QLO + RES_BYTES;
constexpr uint32_t OFF_BAR = OFF_DOLO + RES_BYTES;
enum { QD_FULL, QD_READY, ST_FULL, ST_READY = ST_FULL + NST, ST_EMPTY = ST_READY + NST, S_FULL = ST_EMPTY + NST,
       DS_FULL = S_FULL + 2, G_DONE = DS_FULL + 2, CHAIN_DONE = G_DONE + 2, BLK_FREE, DRAIN, NBAR };
constexpr uint32_t OFF_MISC = OFF_BAR + NBAR * 8;
constexpr uint32_t SMEM = OFF_MISC + 16 + 1024;
// TMEM: Q hi | dO hi | 2 x (S, dP / dS hi, dS lo) | dQ_blk
constexpr uint32_t C_QHI = 0, C_DOHI = 64, C_DQB = 320, TCOLS = 512;
__device__ __forceinline__ constexpr uint32_t c_s(int b) { return 128 + b * 96; }
__device__ __forceinline__ constexpr uint32_t c_dp(int b) { return 160 + b * 96; }
__device__ __forceinline__ constexpr uint32_t c_dslo(int b) { return 192 + b * 96; }
static_assert(2 * RES_BYTES <= 2 * STAGE_BYTES, "the raw Q / dO tiles are staged in stages 0-1");
static_assert(SMEM <= 232448, "smem");
}  // namespace qq

template <bool SPLIT>
__global__ void __maxnreg__(128)
    attn_bwd_dq_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_do,
                          const __grid_constant__ CUtensorMap tm_kk, const __grid_constant__ CUtensorMap tm_kmn,
                          const __grid_constant__ CUtensorMap tm_vk, const TcBwdArgs a) {
    using namespace qq;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_addr(smem_raw);
    const uint32_t sb = (raw + 1023u) & ~1023u;
    uint8_t *sg = smem_raw + (sb - raw);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const AttnProblem &p = a.p;
    const int64_t h = blockIdx.y, b = blockIdx.z, hk = h / p.group;
    const int64_t q0 = (int64_t)blockIdx.x * TILE;
    const int64_t kv_end = p.causal ? min(p.S, q0 + TILE) : p.S;
    const int nblk = (int)((kv_end + BLK - 1) / BLK);
    auto bar = [&](int i) { return sb + OFF_BAR + 8u * (uint32_t)i; };
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(sg + OFF_MISC);
    volatile int *abort = reinterpret_cast<volatile int *>(sg + OFF_MISC + 4);
    int *err = a.err;

    if (threadIdx.x == 0) {
        mbar_init(bar(QD_FULL), 1);
        mbar_init(bar(QD_READY), 128);
        for (int s = 0; s < NST; s++) {
            mbar_init(bar(ST_FULL + s), 1);
            mbar_init(bar(ST_READY + s), 128);
            mbar_init(bar(ST_EMPTY + s), 1);
        }
        for (int s = 0; s < 2; s++) {
            mbar_init(bar(S_FULL + s), 1);
            mbar_init(bar(DS_FULL + s), 128);
        }
        mbar_init(bar(G_DONE), 1);
        mbar_init(bar(G_DONE + 1), 1);
        mbar_init(bar(CHAIN_DONE), 1);
        mbar_init(bar(BLK_FREE), 128);
        mbar_init(bar(DRAIN), 1);
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == W_MMA) {
        tmem_alloc(smem_addr(tmem_slot), TCOLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == W_PROD) {
        if (lane == 0) {
            int issued = -1;
            mbar_expect_tx(bar(QD_FULL), 2 * RES_BYTES);
            for (int c = 0; c < CHUNKS; c++) {
                tma_load_4d(&tm_q, sb + c * RES_CHUNK, bar(QD_FULL), 32 * c, (int)q0, (int)h, (int)b);
                tma_load_4d(&tm_do, sb + RES_BYTES + c * RES_CHUNK, bar(QD_FULL), 32 * c, (int)q0, (int)h, (int)b);
            }
            bool ok = mbar_wait(bar(QD_READY), 0, abort, err);
            for (int j = 0; ok && j < nblk; j++) {
                const int s = j % NST;
                if (j >= NST && !mbar_wait(bar(ST_EMPTY + s), ((j / NST) - 1) & 1, abort, err)) break;
                const uint32_t st = sb + s * STAGE_BYTES;
                mbar_expect_tx(bar(ST_FULL + s), 3 * BLK_BYTES);
                for (int c = 0; c < CHUNKS; c++) {
                    tma_load_4d(&tm_kk, st + ST_KK + c * BLK_CHUNK, bar(ST_FULL + s), 32 * c, j * BLK, (int)hk, (int)b);
                    tma_load_4d(&tm_kmn, st + ST_KMN + c * BLK_CHUNK, bar(ST_FULL + s), 32 * c, j * BLK, (int)hk, (int)b);
                    tma_load_4d(&tm_vk, st + ST_VK + c * BLK_CHUNK, bar(ST_FULL + s), 32 * c, j * BLK, (int)hk, (int)b);
                }
                issued = j;
            }
            if (*abort) {
                volatile int never = 0;
                mbar_wait(bar(QD_FULL), 0, &never, nullptr);
                for (int j = max(0, issued - NST + 1); j <= issued; j++)
                    mbar_wait(bar(ST_FULL + j % NST), (j / NST) & 1, &never, nullptr);
            }
        }
    } else if (warp == W_MMA) {
        if (lane == 0) {
            const uint64_t qlo = sdesc_sw128(sb + OFF_QLO, 16, 1024), dolo = sdesc_sw128(sb + OFF_DOLO, 16, 1024);
            auto issue_g = [&](int j) -> bool {
                const int s = j % NST, bb = j & 1;
                const uint32_t st = sb + s * STAGE_BYTES;
                if (!mbar_wait(bar(DS_FULL + bb), (j >> 1) & 1, abort, err)) return false;
                const bool first = (j % FOLD) == 0;
                if (first && j >= FOLD && !mbar_wait(bar(BLK_FREE), ((j / FOLD) - 1) & 1, abort, err)) return false;
                tc_fence_after();
                mma_g<SPLIT>(tmem + C_DQB, tmem + c_dp(bb), tmem + c_dslo(bb),
                             sdesc_mn_sw128_32b(st + ST_KMN, BLK_CHUNK, 512), !first);
                tc_commit(bar(G_DONE + bb));
                if ((j % FOLD) == FOLD - 1 || j == nblk - 1) tc_commit(bar(CHAIN_DONE));
                tc_commit(bar(ST_EMPTY + s));
                return true;
            };
            bool ok = mbar_wait(bar(QD_READY), 0, abort, err);
            tc_fence_after();
            for (int j = 0; ok && j < nblk; j++) {
                const int s = j % NST, bb = j & 1;
                const uint32_t st = sb + s * STAGE_BYTES;
                if (!mbar_wait(bar(ST_READY + s), (j / NST) & 1, abort, err)) break;
                // Buffer bb holds dS of block j-2 until its gradient MMAs finish.
                if (j >= 2 && !mbar_wait(bar(G_DONE + bb), ((j - 2) >> 1) & 1, abort, err)) break;
                tc_fence_after();
                mma_s<SPLIT>(tmem + c_s(bb), tmem + C_QHI, qlo, sdesc_sw128(st + ST_KK, 16, 1024));
                mma_s<SPLIT>(tmem + c_dp(bb), tmem + C_DOHI, dolo, sdesc_sw128(st + ST_VK, 16, 1024));
                tc_commit(bar(S_FULL + bb));
                if (j >= 1 && !issue_g(j - 1)) {
                    ok = false;
                    break;
                }
            }
            if (ok && nblk > 0) issue_g(nblk - 1);
            tc_commit(bar(DRAIN));
            volatile int never = 0;
            mbar_wait(bar(DRAIN), 0, &never, nullptr);
        }
    } else if (warp >= W_CVT) {
        const int ct = threadIdx.x - 32 * W_CVT;
        const int quad = warp & 3;
        const int row = quad * 32 + lane;
        const uint32_t tl = tmem + ((uint32_t)(quad * 32) << 16);
        if (mbar_wait(bar(QD_FULL), 0, abort, err)) {
            row_split<SPLIT>(sg, sg + OFF_QLO, row, tl, C_QHI);
            row_split<SPLIT>(sg + RES_BYTES, sg + OFF_DOLO, row, tl, C_DOHI);
            tmem_wait_st();
            fence_proxy_async_smem();
            tc_fence_before();
            mbar_arrive(bar(QD_READY));
            for (int j = 0; j < nblk; j++) {
                const int s = j % NST;
                if (!mbar_wait(bar(ST_FULL + s), (j / NST) & 1, abort, err)) break;
                uint8_t *st = sg + s * STAGE_BYTES;
                split_tile<SPLIT>(st + ST_KK, ct);
                split_tile<SPLIT>(st + ST_KMN, ct);
                split_tile<SPLIT>(st + ST_VK, ct);
                fence_proxy_async_smem();
                mbar_arrive(bar(ST_READY + s));
            }
        }
    } else if (warp >= W_FOLD) {
        // ------------------------------------------------------------ fold: fp32 dQ ---
        const int row = threadIdx.x - 32 * W_FOLD;
        const int64_t q = q0 + row;
        const uint32_t tl = tmem + ((uint32_t)((warp & 3) * 32) << 16);
        float dq[D];
#pragma unroll
        for (int x = 0; x < D; x++) dq[x] = 0.0f;
        bool ok = true;
        const int nchain = (nblk + FOLD - 1) / FOLD;
        for (int ch = 0; ch < nchain; ch++) {
            if (!mbar_wait(bar(CHAIN_DONE), ch & 1, abort, err)) {
                ok = false;
                break;
            }
            tc_fence_after();
#pragma unroll
            for (int c = 0; c < D / 16; c++) {
                uint32_t r[16];
                tmem_ld16(tl + C_DQB + 16 * c, r);
                tmem_wait_ld();
#pragma unroll
                for (int x = 0; x < 16; x++) dq[16 * c + x] += __uint_as_float(r[x]);
            }
            tc_fence_before();
            mbar_arrive(bar(BLK_FREE));
        }
        const bool aborted = __any_sync(0xffffffffu, *abort != 0);
        if (ok && !aborted && q < p.L) {
            float *dqr = a.g.dq + b * a.g.dqs[0] + h * a.g.dqs[1] + q * a.g.dqs[2];
#pragma unroll
            for (int c = 0; c < D; c++) dqr[c * a.g.dqs[3]] = dq[c] * p.scale;
        }
    } else {
        // ---------------------------------------------------------------------- dS ----
        const int row = threadIdx.x;
        const int64_t q = q0 + row;
        const bool row_ok = q < p.L;
        const uint32_t tl = tmem + ((uint32_t)(warp * 32) << 16);
        const float lse2 = row_ok ? p.lse[b * p.ls[0] + h * p.ls[1] + q * p.ls[2]] * LOG2E : 0.0f;
        const float del = row_ok ? a.g.delta[(b * p.H + h) * p.L + q] : 0.0f;
        for (int j = 0; j < nblk; j++) {
            const int bb = j & 1;
            const int64_t kb0 = (int64_t)j * BLK;
            if (!mbar_wait(bar(S_FULL + bb), (j >> 1) & 1, abort, err)) break;
            tc_fence_after();
            const bool edge = !row_ok || kb0 + BLK > p.S || (p.causal && kb0 + BLK - 1 > q0) || p.mask_kind != MASK_NONE;
#pragma unroll
            for (int hf = 0; hf < 2; hf++) {  // 16 key columns at a time
                uint32_t sr[16], dr[16];
                tmem_ld16(tl + c_s(bb) + 16 * hf, sr);
                tmem_ld16(tl + c_dp(bb) + 16 * hf, dr);
                tmem_wait_ld();
#pragma unroll
                for (int c = 0; c < 16; c++) {
                    float x = __uint_as_float(sr[c]) * a.scale_log2;
                    bool valid = true;
                    if (edge) {
                        const int64_t key = kb0 + 16 * hf + c;
                        valid = row_ok && key < p.S && !(p.causal && key > q);
                        if (valid && p.mask_kind != MASK_NONE) x += mask_value(p, b, h, q, key) * LOG2E;
                    }
                    const float pc = valid ? ex2_approx(x - lse2) : 0.0f;
                    const float ds = pc * (__uint_as_float(dr[c]) - del);
                    sr[c] = tf32_rna(ds);
                    if (SPLIT) dr[c] = tf32_rna(ds - __uint_as_float(sr[c]));
                }
                tmem_st16(tl + c_dp(bb) + 16 * hf, sr);
                if (SPLIT) tmem_st16(tl + c_dslo(bb) + 16 * hf, dr);
            }
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(bar(DS_FULL + bb));
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == W_MMA) {
        tc_fence_after();
        tmem_dealloc(tmem, qq::TCOLS);
    }
}

}  // namespace

bool tc_backward_supported(const AttnProblem &p, const AttnGrads &g) {
    if (!tc_forward_supported(p) || p.E != D) return false;
    if (p.L >= (1ll << 31) - TILE) return false;
    // grad_out is read through TMA as well.
    if (g.dos[3] != 1 || !tma_stride_ok(p.L, g.dos[2]) || !tma_stride_ok(p.H, g.dos[1]) ||
        !tma_stride_ok(p.B, g.dos[0]))
        return false;
    return (reinterpret_cast<uintptr_t>(g.dout) & 15u) == 0;
}

int tc_backward(const AttnProblem &p, const AttnGrads &g, int precision, cudaStream_t stream) {
    TcBwdArgs a;
    a.p = p;
    a.g = g;
    a.scale_log2 = p.scale * LOG2E;
    a.err = device_error_word();
    if (!a.err) return fail(DC_ERR_CUDA, "device error word is unavailable");
    const bool split = precision != DC_PREC_TF32;
    const int64_t *dos = g.dos;  // grad_out shares q's shape but has its own strides
    int st = DC_OK;
    if (p.S > 0) {
        CUtensorMap tk, tv, tqk, tqmn, tdok, tdomn;
        st = make_tmap(&tk, p.k, D, p.S, p.Hkv, p.B, p.ks, TILE);
        if (!st) st = make_tmap(&tv, p.v, D, p.S, p.Hkv, p.B, p.vs, TILE);
        if (!st) st = make_tmap(&tqk, p.q, D, p.L, p.H, p.B, p.qs, BLK);
        if (!st) st = make_tmap(&tqmn, p.q, D, p.L, p.H, p.B, p.qs, BLK, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
        if (!st) st = make_tmap(&tdok, g.dout, D, p.L, p.H, p.B, dos, BLK);
        if (!st) st = make_tmap(&tdomn, g.dout, D, p.L, p.H, p.B, dos, BLK, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
        if (st) return st;
        auto kernel = split ? attn_bwd_dkdv_tc_kernel<true> : attn_bwd_dkdv_tc_kernel<false>;
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kv::SMEM);
        if (e != cudaSuccess) return cuda_fail(e, "attn_bwd_dkdv_tc smem attribute");
        dim3 grid((unsigned)((p.S + TILE - 1) / TILE), (unsigned)p.Hkv, (unsigned)p.B);
        KernelTrace tr("bwd_dkdv_tc", stream);
        kernel<<<grid, kv::THREADS, kv::SMEM, stream>>>(tk, tv, tqk, tqmn, tdok, tdomn, a);
        if ((st = check_launch("attn_bwd_dkdv_tc"))) return st;
    }
    if (p.L > 0) {
        CUtensorMap tq, tdo, tkk, tkmn, tvk;
        st = make_tmap(&tq, p.q, D, p.L, p.H, p.B, p.qs, TILE);
        if (!st) st = make_tmap(&tdo, g.dout, D, p.L, p.H, p.B, dos, TILE);
        if (!st) st = make_tmap(&tkk, p.k, D, p.S, p.Hkv, p.B, p.ks, BLK);
        if (!st) st = make_tmap(&tkmn, p.k, D, p.S, p.Hkv, p.B, p.ks, BLK, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
        if (!st) st = make_tmap(&tvk, p.v, D, p.S, p.Hkv, p.B, p.vs, BLK);
        if (st) return st;
        auto kernel = split ? attn_bwd_dq_tc_kernel<true> : attn_bwd_dq_tc_kernel<false>;
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)qq::SMEM);
        if (e != cudaSuccess) return cuda_fail(e, "attn_bwd_dq_tc smem attribute");
        dim3 grid((unsigned)((p.L + TILE - 1) / TILE), (unsigned)p.H, (unsigned)p.B);
        KernelTrace tr("bwd_dq_tc", stream);
        kernel<<<grid, qq::THREADS, qq::SMEM, stream>>>(tq, tdo, tkk, tkmn, tvk, a);
        if ((st = check_launch("attn_bwd_dq_tc"))) return st;
    }
    return DC_OK;
}

}  // namespace dc
