// attn_tc_bwd.cu -- tcgen05 tensor-core attention backward for sm_100a (head dim 64).
//
// Replaces DenseCore's torch_attention::backward (src/torch_attention.rs:291-468), which per
// (q block, kv block) recomputes P = exp(scale*S + mask - lse) (:338-380) and accumulates
//   dV += P^T dO, dP = dO V^T, dS = P (dP - delta), dQ += scale dS K, dK += scale dS^T Q
// (:381-446), with delta = sum(dO * O) per row (:327-330, computed by bwd_delta_kernel).
//
// Two kernels, so every accumulator has one owner and no atomics are needed:
//
//   dkdv: a CTA owns 128 keys of one (batch, kv head). K and V (tf32 hi and lo) sit in TMEM
//         as the A operands; 32-row blocks of Q and dO stream through shared memory, each
//         in two layouts (128-byte swizzle for the K-major use, 32-byte-atom swizzle for the
//         MN-major use that tf32 requires). Per block: S^T = K Q^T and dP^T = V dO^T into
//         TMEM, the softmax threads (one per key) form P^T and dS^T in TMEM, then
//         dV_blk += P^T dO and dK_blk += dS^T Q. The block accumulators are folded into fp32
//         shared-memory accumulators every FOLD blocks (the tensor core's accumulation is
//         coarser than fp32 over long chains).
//   dq:   a CTA owns 128 query rows of one (batch, head). Q and dO (hi, lo) sit in TMEM;
//         32-key blocks of K (two layouts) and V stream through shared memory. Per block:
//         S = Q K^T, dP = dO V^T, dS in TMEM, dQ_blk += dS K, folded in fp32 every FOLD.
//
// Roles in both: warps 0-3 one row (TMEM lane) per thread, warp 4 TMA producer, warp 5 MMA
// issuer and TMEM owner, warps 6-9 converters (fp32 -> tf32 hi/lo; resident tiles into TMEM).
// Every wait is bounded; on a timeout the kernel records an error and unwinds.
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
constexpr int THREADS = 320;

constexpr uint32_t RES_BYTES = TILE * D * 4;      // one resident fp32 tile (32 KB)
constexpr uint32_t RES_CHUNK = TILE * 128;        // 16 KB per 32-column chunk
constexpr uint32_t BLK_BYTES = BLK * D * 4;       // one streamed fp32 tile (8 KB)
constexpr uint32_t BLK_CHUNK = BLK * 128;         // 4 KB per chunk

constexpr uint32_t IDESC_S = idesc_tf32(128, BLK, 0, 0);  // S / dP: N = 32, both K-major
constexpr uint32_t IDESC_G = idesc_tf32(128, D, 0, 1);    // gradients: N = 64, B MN-major

// One resident row (TMEM lane `row`) from a raw 128-byte-swizzled tile of TILE rows into
// TMEM: hi at col_hi, lo at col_lo (lo only when split). Called by a full warp.
__device__ __forceinline__ void row_to_tmem(const uint8_t *raw, int row, uint32_t taddr_lane, uint32_t col_hi,
                                            uint32_t col_lo, int split) {
#pragma unroll
    for (int c = 0; c < CHUNKS; c++) {
        uint32_t hi[32], lo[32];
#pragma unroll
        for (int g = 0; g < 8; g++) {
            const float4 x = *reinterpret_cast<const float4 *>(raw + c * RES_CHUNK + row * 128 +
                                                               (((g ^ (row & 7)) & 7) * 16));
            const float v[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
            for (int e = 0; e < 4; e++) {
                if (split) {
                    hi[4 * g + e] = tf32_rna(v[e]);
                    lo[4 * g + e] = tf32_rna(v[e] - __uint_as_float(hi[4 * g + e]));
                } else {
                    hi[4 * g + e] = tf32_rna(v[e]);
                }
            }
        }
        tmem_st32(taddr_lane + col_hi + 32 * c, hi);
        if (split) tmem_st32(taddr_lane + col_lo + 32 * c, lo);
    }
}

// hi = tf32(x) in place and, when split, lo = tf32(x - hi) `lo_off` bytes further; elementwise
// over a tile. Single-pass TF32 rounds to nearest here rather than letting the tensor core
// drop the low mantissa bits (which would bias every operand toward zero).
__device__ __forceinline__ void split_tile(uint8_t *hi, uint32_t lo_off, uint32_t bytes, int t, int split) {
    for (uint32_t i = t; i < bytes / 16; i += 128) {
        float4 *ph = reinterpret_cast<float4 *>(hi) + i;
        const float4 x = *ph;
        float4 hv;
        hv.x = __uint_as_float(tf32_rna(x.x));
        hv.y = __uint_as_float(tf32_rna(x.y));
        hv.z = __uint_as_float(tf32_rna(x.z));
        hv.w = __uint_as_float(tf32_rna(x.w));
        *ph = hv;
        if (split) {
            float4 lv;
            lv.x = __uint_as_float(tf32_rna(x.x - hv.x));
            lv.y = __uint_as_float(tf32_rna(x.y - hv.y));
            lv.z = __uint_as_float(tf32_rna(x.z - hv.z));
            lv.w = __uint_as_float(tf32_rna(x.w - hv.w));
            *(reinterpret_cast<float4 *>(hi + lo_off) + i) = lv;
        }
    }
}

// D[tmem] (+)= A x B over the three tf32 passes (cross terms first): A in TMEM (hi, lo
// columns), B in shared memory: `bhi` is the descriptor of the hi tile, the lo tile sits
// BLK_BYTES further, and k-step kk starts OFF(kk) 16-byte units into the tile.
template <bool SPLIT, int KSTEPS, class Off>
__device__ __forceinline__ void mma3_ts(uint32_t d, uint32_t a_hi, uint32_t a_lo, uint64_t bhi, Off off,
                                        uint32_t idesc, bool accumulate) {
    constexpr uint32_t LO = BLK_BYTES >> 4;
    if (SPLIT) {
#pragma unroll
        for (int kk = 0; kk < KSTEPS; kk++) {
            mma_tf32_ts(d, a_hi + kk * 8, bhi + (LO + off(kk)), idesc, (accumulate || kk > 0) ? 1u : 0u);
            mma_tf32_ts(d, a_lo + kk * 8, bhi + off(kk), idesc, 1u);
        }
    }
#pragma unroll
    for (int kk = 0; kk < KSTEPS; kk++)
        mma_tf32_ts(d, a_hi + kk * 8, bhi + off(kk), idesc, (accumulate || SPLIT || kk > 0) ? 1u : 0u);
}
// k-step offsets (16-byte units): K-major 128-byte swizzle (8 tf32 = 32 bytes per k-step,
// 4 k-steps per 128-byte chunk) and MN-major 32-byte-atom swizzle (8 rows = 1024 bytes).
struct KOff {
    __device__ __forceinline__ uint32_t operator()(int kk) const {
        return (uint32_t)(((kk >> 2) * BLK_CHUNK + (kk & 3) * 32) >> 4);
    }
};
struct MnOff {
    __device__ __forceinline__ uint32_t operator()(int kk) const { return (uint32_t)(kk * 64); }
};

struct TcBwdArgs {
    AttnProblem p;
    AttnGrads g;
    float scale_log2;
    int *err;
};

// ==================================================================== dK / dV ========
namespace kv {
constexpr int NST = 2;
// stage: Q_K hi, lo | Q_MN hi, lo | dO_K hi, lo | dO_MN hi, lo  (8 KB each)
constexpr uint32_t ST_QK = 0, ST_QMN = 2 * BLK_BYTES, ST_DOK = 4 * BLK_BYTES, ST_DOMN = 6 * BLK_BYTES;
constexpr uint32_t STAGE_BYTES = 8 * BLK_BYTES;  // 64 KB
constexpr uint32_t OFF_STAGE = 0;
constexpr uint32_t OFF_ACC = NST * STAGE_BYTES;               // fp32 [2*D cols][TILE rows]
constexpr uint32_t OFF_BAR = OFF_ACC + 2 * D * TILE * 4;
enum { KV_FULL, KV_READY, ST_FULL, ST_READY = ST_FULL + NST, ST_EMPTY = ST_READY + NST,
       S_FULL = ST_EMPTY + NST, P_FULL, BLK_DONE, BLK_FREE, DRAIN, NBAR };
constexpr uint32_t OFF_MISC = OFF_BAR + NBAR * 8;
constexpr uint32_t SMEM = OFF_MISC + 16 + 1024;
// TMEM columns
constexpr uint32_t C_KHI = 0, C_KLO = 64, C_VHI = 128, C_VLO = 192, C_S = 256, C_PLO = 288, C_DP = 320,
                   C_DSLO = 352, C_DV = 384, C_DK = 448, TCOLS = 512;
static_assert(SMEM <= 232448, "smem");
}  // namespace kv

template <bool SPLIT>
__global__ void __launch_bounds__(THREADS, 1)
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
    float *acc = reinterpret_cast<float *>(sg + OFF_ACC);  // [c][row], c < D: dV, c >= D: dK

    if (threadIdx.x == 0) {
        mbar_init(bar(KV_FULL), 1);
        mbar_init(bar(KV_READY), 128);
        for (int s = 0; s < NST; s++) {
            mbar_init(bar(ST_FULL + s), 1);
            mbar_init(bar(ST_READY + s), 128);
            mbar_init(bar(ST_EMPTY + s), 1);
        }
        mbar_init(bar(S_FULL), 1);
        mbar_init(bar(P_FULL), 128);
        mbar_init(bar(BLK_DONE), 1);
        mbar_init(bar(BLK_FREE), 128);
        mbar_init(bar(DRAIN), 1);
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == 5) {
        tmem_alloc(smem_addr(tmem_slot), TCOLS);
        tmem_relinquish();
    }
    if (warp < 4)
        for (int i = threadIdx.x; i < 2 * D * TILE; i += 128) acc[i] = 0.0f;
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    auto blk_coords = [&](int i, int64_t &h, int64_t &q0) {
        h = hk * p.group + i / qb_per_head;
        q0 = (int64_t)(qb_first + i % qb_per_head) * BLK;
    };

    if (warp == 4) {
        // ---------------------------------------------------------------- producer ----
        if (lane == 0) {
            int issued = -1;
            // K and V of the CTA, raw, into stage 0 (K at 0, V at RES_BYTES).
            mbar_expect_tx(bar(KV_FULL), 2 * RES_BYTES);
            for (int c = 0; c < CHUNKS; c++) {
                tma_load_4d(&tm_k, sb + c * RES_CHUNK, bar(KV_FULL), 32 * c, (int)k0, (int)hk, (int)b);
                tma_load_4d(&tm_v, sb + RES_BYTES + c * RES_CHUNK, bar(KV_FULL), 32 * c, (int)k0, (int)hk, (int)b);
            }
            bool ok = mbar_wait(bar(KV_READY), 0, abort, a.err);
            for (int i = 0; ok && i < nblk; i++) {
                const int s = i % NST;
                if (i >= NST && !mbar_wait(bar(ST_EMPTY + s), ((i / NST) - 1) & 1, abort, a.err)) break;
                int64_t h, q0;
                blk_coords(i, h, q0);
                const uint32_t st = sb + OFF_STAGE + s * STAGE_BYTES;
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
    } else if (warp == 5) {
        // ------------------------------------------------------------------ MMA ------
        if (lane == 0) {
            bool ok = mbar_wait(bar(KV_READY), 0, abort, a.err);
            tc_fence_after();
            for (int i = 0; ok && i < nblk; i++) {
                const int s = i % NST;
                const uint32_t st = sb + OFF_STAGE + s * STAGE_BYTES;
                if (!mbar_wait(bar(ST_READY + s), (i / NST) & 1, abort, a.err)) break;
                // The S / dP columns hold the previous block's P^T and dS^T until its
                // gradient MMAs finish.
                if (i >= 1 && !mbar_wait(bar(BLK_DONE), (i - 1) & 1, abort, a.err)) break;
                tc_fence_after();
                mma3_ts<SPLIT, D / 8>(tmem + C_S, tmem + C_KHI, tmem + C_KLO, sdesc_sw128(st + ST_QK, 16, 1024), KOff(),
                                      IDESC_S, false);
                mma3_ts<SPLIT, D / 8>(tmem + C_DP, tmem + C_VHI, tmem + C_VLO, sdesc_sw128(st + ST_DOK, 16, 1024),
                                      KOff(), IDESC_S, false);
                tc_commit(bar(S_FULL));
                if (!mbar_wait(bar(P_FULL), i & 1, abort, a.err)) break;
                const bool first = (i % FOLD) == 0;
                if (first && i >= FOLD && !mbar_wait(bar(BLK_FREE), ((i / FOLD) - 1) & 1, abort, a.err)) break;
                tc_fence_after();
                mma3_ts<SPLIT, BLK / 8>(tmem + C_DV, tmem + C_S, tmem + C_PLO,
                                        sdesc_mn_sw128_32b(st + ST_DOMN, BLK_CHUNK, 512), MnOff(), IDESC_G, !first);
                mma3_ts<SPLIT, BLK / 8>(tmem + C_DK, tmem + C_DP, tmem + C_DSLO,
                                        sdesc_mn_sw128_32b(st + ST_QMN, BLK_CHUNK, 512), MnOff(), IDESC_G, !first);
                tc_commit(bar(BLK_DONE));
                tc_commit(bar(ST_EMPTY + s));
            }
            tc_commit(bar(DRAIN));
            volatile int never = 0;
            mbar_wait(bar(DRAIN), 0, &never, nullptr);
        }
    } else if (warp >= 6) {
        // ------------------------------------------------------------- converters -----
        const int ct = threadIdx.x - 192;
        const int quad = warp & 3;  // this warp's TMEM lane quadrant
        const int row = quad * 32 + lane;
        const uint32_t tl = tmem + ((uint32_t)(quad * 32) << 16);
        if (mbar_wait(bar(KV_FULL), 0, abort, a.err)) {
            row_to_tmem(sg, row, tl, C_KHI, C_KLO, SPLIT);
            row_to_tmem(sg + RES_BYTES, row, tl, C_VHI, C_VLO, SPLIT);
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(bar(KV_READY));
            for (int i = 0; i < nblk; i++) {
                const int s = i % NST;
                if (!mbar_wait(bar(ST_FULL + s), (i / NST) & 1, abort, a.err)) break;
                {
                    uint8_t *st = sg + OFF_STAGE + s * STAGE_BYTES;
                    split_tile(st + ST_QK, BLK_BYTES, BLK_BYTES, ct, SPLIT);
                    split_tile(st + ST_QMN, BLK_BYTES, BLK_BYTES, ct, SPLIT);
                    split_tile(st + ST_DOK, BLK_BYTES, BLK_BYTES, ct, SPLIT);
                    split_tile(st + ST_DOMN, BLK_BYTES, BLK_BYTES, ct, SPLIT);
                    fence_proxy_async_smem();
                }
                mbar_arrive(bar(ST_READY + s));
            }
        }
    } else {
        // ------------------------------------------------- P^T, dS^T and the folds ----
        const int row = threadIdx.x;  // key row of this CTA
        const int64_t key = k0 + row;
        const bool key_ok = key < p.S;
        const uint32_t tl = tmem + ((uint32_t)(warp * 32) << 16);
        bool ok = true;
        float lse_next = 0.0f, del_next = 0.0f;
        auto load_rows = [&](int i, float &lse_v, float &del_v) {
            int64_t h, q0;
            blk_coords(i, h, q0);
            const int64_t q = q0 + lane;
            lse_v = q < p.L ? p.lse[b * p.ls[0] + h * p.ls[1] + q * p.ls[2]] * LOG2E : 0.0f;
            del_v = q < p.L ? a.g.delta[(b * p.H + h) * p.L + q] : 0.0f;
        };
        if (nblk > 0) load_rows(0, lse_next, del_next);
        for (int i = 0; i < nblk; i++) {
            const float lse_v = lse_next, del_v = del_next;
            if (i + 1 < nblk) load_rows(i + 1, lse_next, del_next);
            int64_t h, q0;
            blk_coords(i, h, q0);
            if (!mbar_wait(bar(S_FULL), i & 1, abort, a.err)) {
                ok = false;
                break;
            }
            tc_fence_after();
            uint32_t sr[32], dr[32];
            tmem_ld32(tl + C_S, sr);
            tmem_ld32(tl + C_DP, dr);
            tmem_wait_ld();
            const bool edge = !key_ok || q0 + BLK > p.L || (p.causal && key > q0) || p.mask_kind != MASK_NONE;
            uint32_t phi[32], plo[32];
#pragma unroll
            for (int c = 0; c < BLK; c++) {
                const float lse_c = __shfl_sync(0xffffffffu, lse_v, c);
                const float del_c = __shfl_sync(0xffffffffu, del_v, c);
                float x = __uint_as_float(sr[c]) * a.scale_log2;
                bool valid = true;
                if (edge) {
                    const int64_t q = q0 + c;
                    valid = key_ok && q < p.L && !(p.causal && key > q);
                    if (valid && p.mask_kind != MASK_NONE) x += mask_value(p, b, h, q, key) * LOG2E;
                }
                const float pc = valid ? ex2_approx(x - lse_c) : 0.0f;
                const float ds = pc * (__uint_as_float(dr[c]) - del_c);
                if (SPLIT) {
                    phi[c] = tf32_rna(pc);
                    plo[c] = tf32_rna(pc - __uint_as_float(phi[c]));
                    sr[c] = tf32_rna(ds);
                    dr[c] = tf32_rna(ds - __uint_as_float(sr[c]));
                } else {
                    phi[c] = tf32_rna(pc);
                    sr[c] = tf32_rna(ds);
                }
            }
            tmem_st32(tl + C_S, phi);
            tmem_st32(tl + C_DP, sr);
            if (SPLIT) {
                tmem_st32(tl + C_PLO, plo);
                tmem_st32(tl + C_DSLO, dr);
            }
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(bar(P_FULL));
            if ((i % FOLD) == FOLD - 1 || i == nblk - 1) {
                // Fold this chain of block accumulators into the fp32 accumulators.
                if (!mbar_wait(bar(BLK_DONE), i & 1, abort, a.err)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
#pragma unroll
                for (int c = 0; c < 2 * CHUNKS; c++) {
                    uint32_t r[32];
                    tmem_ld32(tl + C_DV + 32 * c, r);
                    tmem_wait_ld();
#pragma unroll
                    for (int x = 0; x < 32; x++) acc[(32 * c + x) * TILE + row] += __uint_as_float(r[x]);
                }
                tc_fence_before();
                mbar_arrive(bar(BLK_FREE));
            }
        }
        const bool aborted = __any_sync(0xffffffffu, *abort != 0);
        if (ok && !aborted && key_ok) {
            float *dvr = a.g.dv + b * a.g.dvs[0] + hk * a.g.dvs[1] + key * a.g.dvs[2];
            float *dkr = a.g.dk + b * a.g.dks[0] + hk * a.g.dks[1] + key * a.g.dks[2];
            const float scale = p.scale;
            for (int c = 0; c < D; c++) {
                dvr[c * a.g.dvs[3]] = acc[c * TILE + row];
                dkr[c * a.g.dks[3]] = acc[(D + c) * TILE + row] * scale;
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 5) {
        tc_fence_after();
        tmem_dealloc(tmem, kv::TCOLS);
    }
}

// ========================================================================= dQ ========
namespace qq {
constexpr int NST = 4;
// stage: K_K hi, lo | K_MN hi, lo | V_K hi, lo  (8 KB each)
constexpr uint32_t ST_KK = 0, ST_KMN = 2 * BLK_BYTES, ST_VK = 4 * BLK_BYTES;
constexpr uint32_t STAGE_BYTES = 6 * BLK_BYTES;  // 48 KB
constexpr uint32_t OFF_BAR = NST * STAGE_BYTES;  // the resident Q / dO tiles land in stages 0-1 first
enum { QD_FULL, QD_READY, ST_FULL, ST_READY = ST_FULL + NST, ST_EMPTY = ST_READY + NST, S_FULL = ST_EMPTY + NST,
       DS_FULL, BLK_DONE, BLK_FREE, DRAIN, NBAR };
constexpr uint32_t OFF_MISC = OFF_BAR + NBAR * 8;
constexpr uint32_t SMEM = OFF_MISC + 16 + 1024;
constexpr uint32_t C_QHI = 0, C_QLO = 64, C_DOHI = 128, C_DOLO = 192, C_S = 256, C_DP = 288, C_DSLO = 320,
                   C_DQB = 352, C_DQ = 416, TCOLS = 512;
static_assert(2 * RES_BYTES <= 2 * STAGE_BYTES, "resident staging fits in stages 0-1");
static_assert(SMEM <= 232448, "smem");
}  // namespace qq

template <bool SPLIT>
__global__ void __launch_bounds__(THREADS, 1)
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

    if (threadIdx.x == 0) {
        mbar_init(bar(QD_FULL), 1);
        mbar_init(bar(QD_READY), 128);
        for (int s = 0; s < NST; s++) {
            mbar_init(bar(ST_FULL + s), 1);
            mbar_init(bar(ST_READY + s), 128);
            mbar_init(bar(ST_EMPTY + s), 1);
        }
        mbar_init(bar(S_FULL), 1);
        mbar_init(bar(DS_FULL), 128);
        mbar_init(bar(BLK_DONE), 1);
        mbar_init(bar(BLK_FREE), 128);
        mbar_init(bar(DRAIN), 1);
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == 5) {
        tmem_alloc(smem_addr(tmem_slot), TCOLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 4) {
        if (lane == 0) {
            int issued = -1;
            mbar_expect_tx(bar(QD_FULL), 2 * RES_BYTES);
            for (int c = 0; c < CHUNKS; c++) {
                tma_load_4d(&tm_q, sb + c * RES_CHUNK, bar(QD_FULL), 32 * c, (int)q0, (int)h, (int)b);
                tma_load_4d(&tm_do, sb + RES_BYTES + c * RES_CHUNK, bar(QD_FULL), 32 * c, (int)q0, (int)h, (int)b);
            }
            bool ok = mbar_wait(bar(QD_READY), 0, abort, a.err);
            for (int j = 0; ok && j < nblk; j++) {
                const int s = j % NST;
                if (j >= NST && !mbar_wait(bar(ST_EMPTY + s), ((j / NST) - 1) & 1, abort, a.err)) break;
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
    } else if (warp == 5) {
        if (lane == 0) {
            bool ok = mbar_wait(bar(QD_READY), 0, abort, a.err);
            tc_fence_after();
            for (int j = 0; ok && j < nblk; j++) {
                const int s = j % NST;
                const uint32_t st = sb + s * STAGE_BYTES;
                if (!mbar_wait(bar(ST_READY + s), (j / NST) & 1, abort, a.err)) break;
                if (j >= 1 && !mbar_wait(bar(BLK_DONE), (j - 1) & 1, abort, a.err)) break;
                tc_fence_after();
                mma3_ts<SPLIT, D / 8>(tmem + C_S, tmem + C_QHI, tmem + C_QLO, sdesc_sw128(st + ST_KK, 16, 1024), KOff(),
                                      IDESC_S, false);
                mma3_ts<SPLIT, D / 8>(tmem + C_DP, tmem + C_DOHI, tmem + C_DOLO, sdesc_sw128(st + ST_VK, 16, 1024),
                                      KOff(), IDESC_S, false);
                tc_commit(bar(S_FULL));
                if (!mbar_wait(bar(DS_FULL), j & 1, abort, a.err)) break;
                const bool first = (j % FOLD) == 0;
                if (first && j >= FOLD && !mbar_wait(bar(BLK_FREE), ((j / FOLD) - 1) & 1, abort, a.err)) break;
                tc_fence_after();
                mma3_ts<SPLIT, BLK / 8>(tmem + C_DQB, tmem + C_DP, tmem + C_DSLO,
                                        sdesc_mn_sw128_32b(st + ST_KMN, BLK_CHUNK, 512), MnOff(), IDESC_G, !first);
                tc_commit(bar(BLK_DONE));
                tc_commit(bar(ST_EMPTY + s));
            }
            tc_commit(bar(DRAIN));
            volatile int never = 0;
            mbar_wait(bar(DRAIN), 0, &never, nullptr);
        }
    } else if (warp >= 6) {
        const int ct = threadIdx.x - 192;
        const int quad = warp & 3;
        const int row = quad * 32 + lane;
        const uint32_t tl = tmem + ((uint32_t)(quad * 32) << 16);
        if (mbar_wait(bar(QD_FULL), 0, abort, a.err)) {
            row_to_tmem(sg, row, tl, C_QHI, C_QLO, SPLIT);
            row_to_tmem(sg + RES_BYTES, row, tl, C_DOHI, C_DOLO, SPLIT);
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(bar(QD_READY));
            for (int j = 0; j < nblk; j++) {
                const int s = j % NST;
                if (!mbar_wait(bar(ST_FULL + s), (j / NST) & 1, abort, a.err)) break;
                {
                    uint8_t *st = sg + s * STAGE_BYTES;
                    split_tile(st + ST_KK, BLK_BYTES, BLK_BYTES, ct, SPLIT);
                    split_tile(st + ST_KMN, BLK_BYTES, BLK_BYTES, ct, SPLIT);
                    split_tile(st + ST_VK, BLK_BYTES, BLK_BYTES, ct, SPLIT);
                    fence_proxy_async_smem();
                }
                mbar_arrive(bar(ST_READY + s));
            }
        }
    } else {
        const int row = threadIdx.x;
        const int64_t q = q0 + row;
        const bool row_ok = q < p.L;
        const uint32_t tl = tmem + ((uint32_t)(warp * 32) << 16);
        const float lse2 = row_ok ? p.lse[b * p.ls[0] + h * p.ls[1] + q * p.ls[2]] * LOG2E : 0.0f;
        const float del = row_ok ? a.g.delta[(b * p.H + h) * p.L + q] : 0.0f;
        bool ok = true;
        for (int j = 0; j < nblk; j++) {
            const int64_t kb0 = (int64_t)j * BLK;
            if (!mbar_wait(bar(S_FULL), j & 1, abort, a.err)) {
                ok = false;
                break;
            }
            tc_fence_after();
            uint32_t sr[32], dr[32];
            tmem_ld32(tl + C_S, sr);
            tmem_ld32(tl + C_DP, dr);
            tmem_wait_ld();
            const bool edge = !row_ok || kb0 + BLK > p.S || (p.causal && kb0 + BLK - 1 > q0) || p.mask_kind != MASK_NONE;
#pragma unroll
            for (int c = 0; c < BLK; c++) {
                float x = __uint_as_float(sr[c]) * a.scale_log2;
                bool valid = true;
                if (edge) {
                    const int64_t key = kb0 + c;
                    valid = row_ok && key < p.S && !(p.causal && key > q);
                    if (valid && p.mask_kind != MASK_NONE) x += mask_value(p, b, h, q, key) * LOG2E;
                }
                const float pc = valid ? ex2_approx(x - lse2) : 0.0f;
                const float ds = pc * (__uint_as_float(dr[c]) - del);
                if (SPLIT) {
                    sr[c] = tf32_rna(ds);
                    dr[c] = tf32_rna(ds - __uint_as_float(sr[c]));
                } else {
                    sr[c] = tf32_rna(ds);
                }
            }
            tmem_st32(tl + C_DP, sr);
            if (SPLIT) tmem_st32(tl + C_DSLO, dr);
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(bar(DS_FULL));
            if ((j % FOLD) == FOLD - 1 || j == nblk - 1) {
                if (!mbar_wait(bar(BLK_DONE), j & 1, abort, a.err)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const bool first_fold = j < FOLD;
#pragma unroll
                for (int c = 0; c < CHUNKS; c++) {
                    uint32_t r[32], o[32];
                    tmem_ld32(tl + C_DQB + 32 * c, r);
                    if (!first_fold) tmem_ld32(tl + C_DQ + 32 * c, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int x = 0; x < 32; x++)
                        o[x] = __float_as_uint(first_fold ? __uint_as_float(r[x])
                                                          : __uint_as_float(o[x]) + __uint_as_float(r[x]));
                    tmem_st32(tl + C_DQ + 32 * c, o);
                }
                tmem_wait_st();
                tc_fence_before();
                mbar_arrive(bar(BLK_FREE));
            }
        }
        const bool aborted = __any_sync(0xffffffffu, *abort != 0);
        const bool any = __all_sync(0xffffffffu, ok) && nblk > 0;
        if (!aborted) {
            tc_fence_after();
            float *dqr = a.g.dq + b * a.g.dqs[0] + h * a.g.dqs[1] + q * a.g.dqs[2];
#pragma unroll
            for (int c = 0; c < CHUNKS; c++) {
                uint32_t o[32];
                if (any) {
                    tmem_ld32(tl + C_DQ + 32 * c, o);
                    tmem_wait_ld();
                } else {
#pragma unroll
                    for (int x = 0; x < 32; x++) o[x] = 0u;
                }
                if (row_ok) {
#pragma unroll
                    for (int x = 0; x < 32; x++) dqr[(32 * c + x) * a.g.dqs[3]] = __uint_as_float(o[x]) * p.scale;
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 5) {
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
    // grad_out shares q's shape but has its own strides.
    const int64_t *dos = g.dos;
    CUtensorMap tk, tv, tqk, tqmn, tdok, tdomn;
    int st = make_tmap(&tk, p.k, D, p.S, p.Hkv, p.B, p.ks, TILE);
    if (!st) st = make_tmap(&tv, p.v, D, p.S, p.Hkv, p.B, p.vs, TILE);
    if (!st) st = make_tmap(&tqk, p.q, D, p.L, p.H, p.B, p.qs, BLK);
    if (!st) st = make_tmap(&tqmn, p.q, D, p.L, p.H, p.B, p.qs, BLK, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
    if (!st) st = make_tmap(&tdok, g.dout, D, p.L, p.H, p.B, dos, BLK);
    if (!st) st = make_tmap(&tdomn, g.dout, D, p.L, p.H, p.B, dos, BLK, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
    if (st) return st;
    if (p.S > 0) {
        auto kernel = split ? attn_bwd_dkdv_tc_kernel<true> : attn_bwd_dkdv_tc_kernel<false>;
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kv::SMEM);
        if (e != cudaSuccess) return cuda_fail(e, "attn_bwd_dkdv_tc smem attribute");
        dim3 grid((unsigned)((p.S + TILE - 1) / TILE), (unsigned)p.Hkv, (unsigned)p.B);
        KernelTrace tr("bwd_dkdv_tc", stream);
        kernel<<<grid, THREADS, kv::SMEM, stream>>>(tk, tv, tqk, tqmn, tdok, tdomn, a);
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
        kernel<<<grid, THREADS, qq::SMEM, stream>>>(tq, tdo, tkk, tkmn, tvk, a);
        if ((st = check_launch("attn_bwd_dq_tc"))) return st;
    }
    return DC_OK;
}

}  // namespace dc
