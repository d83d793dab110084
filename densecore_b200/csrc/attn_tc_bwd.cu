// attn_tc_bwd.cu -- tcgen05 tensor-core attention backward for sm_100a (head dims 64 and 128).
//
// Replaces DenseCore's torch_attention::backward (src/torch_attention.rs:291-468), which per
// (q block, kv block) recomputes P = exp(scale*S + mask - lse) (:338-380) and accumulates
//   dV += P^T dO, dP = dO V^T, dS = P (dP - delta), dQ += scale dS K, dK += scale dS^T Q
// (:381-446), with delta = sum(dO * O) per row (:327-330).
//
// Three launches (the last two run concurrently, on the caller's stream and a second one; for
// rows of at most 512 queries the dK / dV kernel is a programmatic dependent of the pre-pass,
// resident and set up before the pre-pass ends):
//
//   prep: one pass over q, grad_out, out, k and v (HBM-bound). Writes TF32 hi = tf32(x) and
//         lo = tf32(x - hi) copies of q, grad_out, k and v into contiguous scratch (3xTF32:
//         a*b ~ ah*bl + al*bh + ah*bh), delta per query row, and lse in base 2. The tensor-core
//         kernels then load ready operands with TMA and never convert on the critical path;
//         they also accept inputs of any strides.
//   dkdv: a CTA owns 128 keys of one (batch, kv head) -- at head dim 128, one 64-column half of
//         their dK and dV (two CTAs per tile, both recomputing S^T and dP^T). K and V are the A
//         operands: hi in TMEM, lo in shared memory. Blocks of 64 (head dim 64) or 32 (128)
//         query rows stream as four tiles, Q and dO each K-major (the S / dP MMAs) and MN-major
//         (the gradient MMAs, this CTA's 64 columns), one stage each, each freed by its reader.
//         Per block i: S^T = K Q^T and dP^T = V dO^T (one MMA warp), P^T while dP^T runs, dS^T
//         while dV runs, dV_blk = P^T dO and dK_blk = dS^T Q (a second MMA warp); eight softmax
//         warps (two per TMEM lane quadrant) then fold the block accumulators into fp32
//         registers (the tensor core's accumulation is coarser than fp32 over long chains):
//         the first four keep dV, the other four dK.
//   dq:   a CTA owns 128 query rows of one (batch, head) -- at head dim 128, one 64-column half
//         of their dQ. Q and dO are the A operands: hi and lo in TMEM at head dim 64, hi in TMEM
//         and lo in shared memory at 128. Blocks of 64 (64) or 32 (128) keys of K and V
//         (K-major) and of K (MN-major, this CTA's columns) stream through three rings, each
//         freed by its reader. Per block: S = Q K^T and dP = dO V^T, dS in TMEM, dQ_blk = dS K,
//         folded into fp32 registers (each softmax warp keeps 32 of the 64 columns). The S, dP
//         and dQ columns are single; the order in which the MMAs are issued keeps the tensor
//         core busy (see the kernel).
//
// Roles: warps 0-7 softmax + fold, warp 8 TMA producer, warp 9 MMA issuer (the whole warp,
// converged, with one elected lane issuing; it also owns TMEM), warp 10 a second TMA producer
// (the MN-major tiles), warp 11 the gradient MMAs (so that either issuer's barrier waits
// overlap the other's MMAs). Every wait is bounded; a timeout records an error and unwinds.
// The softmax loops stay branch-free per column (validity as a bit mask; a user mask in a
// separate pass) to keep the hot code small: twelve warps running different loops already
// crowd the instruction cache. Grids are 1-D: groups of GROUP_HEADS (batch, head[, half])
// units, and within a group the tiles with the most causal work first. The group keeps the
// streamed operands of its heads in L2; the order within it keeps the last wave short.
#include <cuda.h>
#include <cuda_runtime.h>
#include <math.h>

#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "sm100.cuh"
#include "tma_host.h"
#include "trace.h"

namespace dc {
namespace {

using namespace sm100;

constexpr float LOG2E = 1.4426950408889634f;
constexpr int D = 64;        // head dim of the helpers' defaults; the MN-major gradient tiles are 64 wide
constexpr int TILE = 128;    // rows owned by a CTA (the MMA M)
constexpr int BLK = 32;      // default streamed rows per block of the MMA helpers
constexpr int THREADS = 384; // 8 softmax / fold warps, 2 producers, 2 MMA issuers
constexpr int W_PROD = 8, W_MMA = 9, W_PROD2 = 10, W_GMMA = 11;
constexpr int GROUP_HEADS = 16;  // (batch, head) pairs whose tiles are handed out together
constexpr unsigned FULL = 0xffffffffu;

constexpr uint32_t RES_BYTES = TILE * D * 4;      // one resident fp32 tile (32 KB)
constexpr uint32_t RES_CHUNK = TILE * 128;        // 16 KB per 32-column chunk

constexpr uint32_t IDESC_G = idesc_tf32(128, D, 0, 1);    // gradients: N = 64, B MN-major

// k-step offsets in 16-byte units: K-major 128-byte swizzle (8 tf32 = 32 bytes per k-step,
// 4 k-steps per 128-byte chunk of `chunk` bytes) and MN-major 32-byte-atom swizzle (a k-step
// is 8 rows = 1024 bytes).
template <uint32_t CHUNK>
__device__ __forceinline__ constexpr uint32_t koff(int kk) {
    return (uint32_t)(((kk >> 2) * CHUNK + (kk & 3) * 32) >> 4);
}
__device__ __forceinline__ constexpr uint32_t mnoff(int kk) { return (uint32_t)(kk * 64); }

// S-type product over the head dim DD (3 passes with SPLIT, cross terms first):
//   d = A_hi B_lo + A_lo B_hi + A_hi B_hi,
// A_hi in TMEM (columns a_hi + 8 kk), A_lo in shared memory (K-major, TILE rows, descriptor
// a_lo), B hi / lo K-major NB-row tiles in shared memory (descriptor b_hi, lo NB * DD * 4 bytes
// further); N = NB.
template <bool SPLIT, int NB = BLK, int DD = D>
__device__ __forceinline__ void mma_s(uint32_t d, uint32_t a_hi, uint64_t a_lo, uint64_t b_hi) {
    constexpr uint32_t BLO = (uint32_t)(NB * DD * 4) >> 4, CH = NB * 128;
    constexpr uint32_t ID = idesc_tf32(128, NB, 0, 0);
    if (SPLIT) {
#pragma unroll
        for (int kk = 0; kk < DD / 8; kk++) {
            mma_tf32_ts_w(d, a_hi + kk * 8, b_hi + (BLO + koff<CH>(kk)), ID, kk > 0 ? 1u : 0u);
            mma_tf32_ss_w(d, a_lo + koff<RES_CHUNK>(kk), b_hi + koff<CH>(kk), ID, 1u);
        }
    }
#pragma unroll
    for (int kk = 0; kk < DD / 8; kk++)
        mma_tf32_ts_w(d, a_hi + kk * 8, b_hi + koff<CH>(kk), ID, (SPLIT || kk > 0) ? 1u : 0u);
}

// mma_s with A_lo in TMEM too (columns a_lo + 8 kk): every pass reads A from TMEM and only
// the streamed B tile from shared memory. An A operand in shared memory costs the tensor core
// 4 KB of shared-memory reads per k-step, more than the whole N = 32 product.
template <bool SPLIT, int NB = BLK, int DD = D>
__device__ __forceinline__ void mma_s_t(uint32_t d, uint32_t a_hi, uint32_t a_lo, uint64_t b_hi) {
    constexpr uint32_t BLO = (uint32_t)(NB * DD * 4) >> 4, CH = NB * 128;
    constexpr uint32_t ID = idesc_tf32(128, NB, 0, 0);
    if (SPLIT) {
#pragma unroll
        for (int kk = 0; kk < DD / 8; kk++) {
            mma_tf32_ts_w(d, a_hi + kk * 8, b_hi + (BLO + koff<CH>(kk)), ID, kk > 0 ? 1u : 0u);
            mma_tf32_ts_w(d, a_lo + kk * 8, b_hi + koff<CH>(kk), ID, 1u);
        }
    }
#pragma unroll
    for (int kk = 0; kk < DD / 8; kk++)
        mma_tf32_ts_w(d, a_hi + kk * 8, b_hi + koff<CH>(kk), ID, (SPLIT || kk > 0) ? 1u : 0u);
}

// Gradient-type product over NB rows (3 passes with SPLIT): d (+)= A B with A hi / lo in TMEM
// and B hi / lo MN-major in shared memory (descriptor b_hi, lo NB * D * 4 bytes further).
template <bool SPLIT, int NB = BLK>
__device__ __forceinline__ void mma_g(uint32_t d, uint32_t a_hi, uint32_t a_lo, uint64_t b_hi, bool accumulate) {
    constexpr uint32_t BLO = (uint32_t)(NB * D * 4) >> 4;
    if (SPLIT) {
#pragma unroll
        for (int kk = 0; kk < NB / 8; kk++) {
            mma_tf32_ts_w(d, a_hi + kk * 8, b_hi + (BLO + mnoff(kk)), IDESC_G, (accumulate || kk > 0) ? 1u : 0u);
            mma_tf32_ts_w(d, a_lo + kk * 8, b_hi + mnoff(kk), IDESC_G, 1u);
        }
    }
#pragma unroll
    for (int kk = 0; kk < NB / 8; kk++)
        mma_tf32_ts_w(d, a_hi + kk * 8, b_hi + mnoff(kk), IDESC_G, (accumulate || SPLIT || kk > 0) ? 1u : 0u);
}

// Row `row` of a 128-byte-swizzled TILE-row tile (DD columns) in shared memory into TMEM
// columns [col, col + DD) of this thread's lane. A full warp calls it.
template <int DD = D>
__device__ __forceinline__ void row_to_tmem(const uint8_t *tile, int row, uint32_t tlane, uint32_t col) {
#pragma unroll
    for (int c = 0; c < DD / 32; c++) {
        uint32_t v[32];
#pragma unroll
        for (int g = 0; g < 8; g++) {
            const uint4 x = *reinterpret_cast<const uint4 *>(tile + c * RES_CHUNK + row * 128 + ((g ^ (row & 7)) * 16));
            v[4 * g] = x.x;
            v[4 * g + 1] = x.y;
            v[4 * g + 2] = x.z;
            v[4 * g + 3] = x.w;
        }
        tmem_st32(tlane + col + 32 * c, v);
    }
}

// A bounded mbarrier wait whose outcome every lane of the warp shares, so that the
// warp-collective tcgen05.ld / st and shuffles after it run converged.
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, volatile int *abort, int *err) {
    return __all_sync(FULL, mbar_wait(bar, parity, abort, err));
}

// Bit c set for the columns c of [lo, hi) within 0..15.
__device__ __forceinline__ uint32_t col_bits(int64_t lo, int64_t hi) {
    lo = lo < 0 ? 0 : lo;
    hi = hi > 16 ? 16 : hi;
    return hi > lo ? ((0xFFFFu >> (16 - (int)(hi - lo))) << (int)lo) : 0u;
}

// Bit c set for the columns c of [lo, hi) within 0..31.
__device__ __forceinline__ uint32_t col_bits32(int64_t lo, int64_t hi) {
    lo = lo < 0 ? 0 : lo;
    hi = hi > 32 ? 32 : hi;
    return hi > lo ? ((0xFFFFFFFFu >> (32 - (int)(hi - lo))) << (int)lo) : 0u;
}

// Adds 16 TMEM columns of this lane into acc[0..15].
__device__ __forceinline__ void fold16(uint32_t taddr, float *acc) {
    uint32_t r[16];
    tmem_ld16(taddr, r);
    tmem_wait_ld();
#pragma unroll
    for (int x = 0; x < 16; x++) acc[x] += __uint_as_float(r[x]);
}

// Writes n (multiple of 4) floats of acc * mul to a row with element stride `inner`.
template <int N>
__device__ __forceinline__ void store_row(float *dst, int64_t inner, const float *acc, float mul) {
    if (inner == 1 && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0) {
#pragma unroll
        for (int c = 0; c < N; c += 4)
            *reinterpret_cast<float4 *>(dst + c) =
                make_float4(acc[c] * mul, acc[c + 1] * mul, acc[c + 2] * mul, acc[c + 3] * mul);
    } else {
#pragma unroll
        for (int c = 0; c < N; c++) dst[c * inner] = acc[c] * mul;
    }
}

// Tile `tile` and (batch, head) pair `bh` of CTA `idx` in the grouped order: idx runs over
// groups of GROUP_HEADS pairs, inside a group over tiles (outer) and pairs (inner). The grids
// are below 2^31 CTAs (tc_backward_supported), so the decode divides in 32 bits (every CTA
// runs it before its first load).
__device__ __forceinline__ void grouped_tile(uint32_t idx, uint32_t ntiles, uint32_t bh_n, int64_t &tile, int64_t &bh) {
    const uint32_t per_group = ntiles * GROUP_HEADS;
    const uint32_t g = idx / per_group, base = g * GROUP_HEADS;
    const uint32_t gsize = min((uint32_t)GROUP_HEADS, bh_n - base), r = idx - g * per_group;
    tile = r / gsize;
    bh = base + r % gsize;
}

struct TcBwdArgs {
    AttnProblem p;
    AttnGrads g;
    const float *lse2;  // (B*H, L) lse * log2(e), written by the pre-pass
    float scale_log2;
    int *err;
};

// ================================================================= pre-pass ==========
struct PrepArgs {
    AttnProblem p;
    AttnGrads g;
    // [S2][B][heads][rows][DD] contiguous: hi, then lo; with lo_only, [B][heads][rows][DD] of lo
    float *qhl, *dohl, *khl, *vhl;
    float *lse2;  // [B*H][L]
    int split;
    int vec;      // every input row is 16-byte aligned with unit inner stride
    // The kernels read the hi operand from the inputs themselves (the tensor core reads their
    // top 19 bits: x truncated to TF32); write only lo = x - trunc(x), exact in fp32.
    int lo_only;
    // Every row index (rows of q plus rows of k) is below 2^31: the (batch, head, row) decode
    // divides in 32 bits (its 64-bit divisions were a large share of this memory-bound
    // kernel's instructions).
    int rows32;
};

// Row r of a (B, heads, rows) stack as (batch, head, row).
__device__ __forceinline__ void row_bhl(int64_t r, int64_t rows, int64_t heads, int rows32, int64_t &b, int64_t &h,
                                        int64_t &l) {
    if (rows32) {
        const uint32_t r32 = (uint32_t)r, n = (uint32_t)rows, hh = (uint32_t)heads;
        const uint32_t bh = r32 / n, b32 = bh / hh;
        l = r32 - bh * n;
        b = b32;
        h = bh - b32 * hh;
    } else {
        const int64_t bh = r / rows;
        l = r - bh * rows;
        b = bh / heads;
        h = bh - b * heads;
    }
}

__device__ __forceinline__ float4 load4(const float *row, int64_t inner, int j, int vec) {
    if (vec) return *reinterpret_cast<const float4 *>(row + 4 * j);
    return make_float4(row[(4 * j) * inner], row[(4 * j + 1) * inner], row[(4 * j + 2) * inner],
                       row[(4 * j + 3) * inner]);
}

__device__ __forceinline__ void split_store(float *hl, int64_t at, int64_t lo_off, float4 x, int split, int lo_only) {
    if (lo_only) {
        *reinterpret_cast<uint4 *>(hl + at) =
            make_uint4(tf32_lo_trunc(x.x), tf32_lo_trunc(x.y), tf32_lo_trunc(x.z), tf32_lo_trunc(x.w));
        return;
    }
    float4 h;
    h.x = __uint_as_float(tf32_rna(x.x));
    h.y = __uint_as_float(tf32_rna(x.y));
    h.z = __uint_as_float(tf32_rna(x.z));
    h.w = __uint_as_float(tf32_rna(x.w));
    *reinterpret_cast<float4 *>(hl + at) = h;
    if (split) {
        float4 l;
        l.x = __uint_as_float(tf32_rna(x.x - h.x));
        l.y = __uint_as_float(tf32_rna(x.y - h.y));
        l.z = __uint_as_float(tf32_rna(x.z - h.z));
        l.w = __uint_as_float(tf32_rna(x.w - h.w));
        *reinterpret_cast<float4 *>(hl + lo_off + at) = l;
    }
}

// DD / 4 lanes per row of DD (a float4 each): rows of (q, grad_out, out) first, then rows of
// (k, v).
template <int DD>
__global__ void __launch_bounds__(256) bwd_prep_kernel(PrepArgs a) {
    constexpr int LPR = DD / 4, RPB = 256 / LPR;  // lanes per row, rows per block
    // The dK / dV kernel after this one may become resident now (when it is launched as a
    // dependent: short rows).
    griddep_launch_dependents();
    const AttnProblem &p = a.p;
    const int64_t rows_a = p.B * p.H * p.L, rows_b = p.B * p.Hkv * p.S;
    const int64_t r = (int64_t)blockIdx.x * RPB + threadIdx.x / LPR;
    const int j = threadIdx.x % LPR;
    const unsigned group_mask = LPR == 32 ? FULL : (0xFFFFu << (threadIdx.x & 16));
    if (r < rows_a) {
        int64_t b, h, l;
        row_bhl(r, p.L, p.H, a.rows32, b, h, l);
        const float4 q4 = load4(p.q + b * p.qs[0] + h * p.qs[1] + l * p.qs[2], p.qs[3], j, a.vec);
        const float4 d4 = load4(a.g.dout + b * a.g.dos[0] + h * a.g.dos[1] + l * a.g.dos[2], a.g.dos[3], j, a.vec);
        const float4 o4 = load4(p.out + b * p.os[0] + h * p.os[1] + l * p.os[2], p.os[3], j, a.vec);
        float s = fmaf(d4.w, o4.w, fmaf(d4.z, o4.z, fmaf(d4.y, o4.y, d4.x * o4.x)));
#pragma unroll
        for (int o = LPR / 2; o > 0; o >>= 1) s += __shfl_xor_sync(group_mask, s, o);
        split_store(a.qhl, r * DD + 4 * j, rows_a * DD, q4, a.split, a.lo_only);
        split_store(a.dohl, r * DD + 4 * j, rows_a * DD, d4, a.split, a.lo_only);
        if (j == 0) {
            a.g.delta[r] = s;
            a.lse2[r] = p.lse[b * p.ls[0] + h * p.ls[1] + l * p.ls[2]] * LOG2E;
        }
    } else if (r < rows_a + rows_b) {
        const int64_t rr = r - rows_a;
        int64_t b, hk, sidx;
        row_bhl(rr, p.S, p.Hkv, a.rows32, b, hk, sidx);
        const float4 k4 = load4(p.k + b * p.ks[0] + hk * p.ks[1] + sidx * p.ks[2], p.ks[3], j, a.vec);
        const float4 v4 = load4(p.v + b * p.vs[0] + hk * p.vs[1] + sidx * p.vs[2], p.vs[3], j, a.vec);
        split_store(a.khl, rr * DD + 4 * j, rows_b * DD, k4, a.split, a.lo_only);
        split_store(a.vhl, rr * DD + 4 * j, rows_b * DD, v4, a.split, a.lo_only);
    }
}

// ==================================================================== dK / dV ========
// Head dim DD = 64: a CTA computes all of dK and dV for its keys. DD = 128: two CTAs per key
// tile, each computing one 64-column half of dK and dV (both recompute S^T and dP^T over the
// whole head dim), so that tensor memory holds K hi and V hi (DD columns each), one S^T / dP^T
// block and the two half accumulators.
template <int DD>
struct KvCfg {
    static constexpr int NH = DD / 64;            // gradient column halves (CTAs per key tile)
    static constexpr int QB = DD == 64 ? 64 : 32; // query rows per streamed block (S / dP's N)
    static constexpr int CPT = QB / 2;            // query columns per softmax thread
    static constexpr uint32_t RESB = TILE * DD * 4;     // resident K or V tile (hi or lo)
    static constexpr uint32_t TK_BYTES = QB * DD * 4;   // K-major streamed tile (hi or lo)
    static constexpr uint32_t TK_CHUNK = QB * 128;
    static constexpr uint32_t TM_BYTES = QB * 64 * 4;   // MN-major half tile (hi or lo)
    static constexpr uint32_t TM_CHUNK = QB * 128;
    // Shared memory: K lo | V lo | Q_K | dO_K | dO_MN | Q_MN (hi + lo each), one stage per
    // streamed tile, each freed by its own reader. K hi and V hi wait for the softmax warps to
    // move them into TMEM: DD = 64 in the Q_MN and dO_MN stages (the gradient MMAs need those
    // tiles last, so the Q_K and dO_K tiles of the first S^T / dP^T load meanwhile), DD = 128
    // in the K lo / V lo areas (whose lo copies are loaded after).
    static constexpr uint32_t OFF_KLO = 0, OFF_VLO = RESB, OFF_QK = 2 * RESB, OFF_DOK = OFF_QK + 2 * TK_BYTES,
                              OFF_DOMN = OFF_DOK + 2 * TK_BYTES, OFF_QMN = OFF_DOMN + 2 * TM_BYTES,
                              OFF_BAR = OFF_QMN + 2 * TM_BYTES;
    static constexpr uint32_t OFF_KHI_STAGE = DD == 64 ? OFF_QMN : OFF_KLO;
    static constexpr uint32_t OFF_VHI_STAGE = DD == 64 ? OFF_DOMN : OFF_VLO;
    // Per block i: S^T (S_FULL) turned into P^T (P_READY); dP^T (DP_FULL) into dS^T (DS_READY);
    // dV (DV_DONE: P^T read, S^T_{i+1} may overwrite it) and dK (DK_DONE: dS^T read, dP^T_{i+1}
    // may overwrite it); DV_FREE / DK_FREE: the fold has read that accumulator. KVLO_FULL: the
    // resident lo copies (DD = 128 loads them once the hi tiles are in TMEM).
    enum { KV_FULL, KV_READY, KVLO_FULL, QK_FULL, QK_EMPTY, DOK_FULL, DOK_EMPTY, DOMN_FULL, DOMN_EMPTY, QMN_FULL,
           QMN_EMPTY, S_FULL, DP_FULL, P_READY, DS_READY, DV_DONE, DK_DONE, DV_FREE, DK_FREE, DRAIN, DRAIN_G,
           DK_ISSUED, NBAR };
    static constexpr uint32_t OFF_MISC = OFF_BAR + NBAR * 8;
    static constexpr uint32_t SMEM = OFF_MISC + 16 + 1024;
    // TMEM: K hi | V hi | S^T / P^T hi | P^T lo | dP^T / dS^T hi | dS^T lo | dV_blk | dK_blk
    static constexpr uint32_t C_KHI = 0, C_VHI = DD, C_S = 2 * DD, C_PLO = C_S + QB, C_DP = C_S + 2 * QB,
                              C_DSLO = C_S + 3 * QB, C_DV = C_S + 4 * QB, C_DK = C_DV + 64, TCOLS = 512;
    static_assert(C_DK + 64 <= TCOLS, "tensor memory budget");
    static_assert(RESB <= 2 * TM_BYTES || DD != 64, "K / V hi are staged in the Q_MN and dO_MN stages");
    static_assert(SMEM <= 232448, "smem");
};

// tm_k / tm_v: (DD, S, Hkv, S2*B) over the hi / lo copies (lo at batch B + b), box 128 rows;
// tm_q* / tm_do*: (DD, L, H, S2*B), box QB rows, K-major (128-byte swizzle) or MN-major
// (32-byte-atom swizzle; this CTA's 64-column half).
//
// MMA order per block i: S^T_i, dP^T_i (warp 9), dV_i, dK_i (warp 11). S^T_{i+1} waits for dV_i
// and runs after dK_i; dP^T_{i+1} waits for dK_i. The softmax warps compute P^T_i while dP^T_i
// runs and dS^T_i while dV_i runs.
template <int DD, bool SPLIT, bool MASKED, bool DROP>
__global__ void __maxnreg__(168)
    attn_bwd_dkdv_tc_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                            const __grid_constant__ CUtensorMap tm_qk, const __grid_constant__ CUtensorMap tm_qmn,
                            const __grid_constant__ CUtensorMap tm_dok, const __grid_constant__ CUtensorMap tm_domn,
                            const __grid_constant__ CUtensorMap tm_k_lo, const __grid_constant__ CUtensorMap tm_v_lo,
                            const __grid_constant__ CUtensorMap tm_qk_lo, const __grid_constant__ CUtensorMap tm_qmn_lo,
                            const __grid_constant__ CUtensorMap tm_dok_lo, const __grid_constant__ CUtensorMap tm_domn_lo,
                            const TcBwdArgs a) {
    using C = KvCfg<DD>;
    constexpr int QB = C::QB, CPT = C::CPT;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_addr(smem_raw);
    const uint32_t sb = (raw + 1023u) & ~1023u;
    uint8_t *sg = smem_raw + (sb - raw);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const AttnProblem &p = a.p;
    // Key tiles in ascending order: under causal masking tile 0 sees the most query rows.
    int64_t kt, bhd;
    grouped_tile(blockIdx.x, (uint32_t)((p.S + TILE - 1) / TILE), (uint32_t)(p.B * p.Hkv * C::NH), kt, bhd);
    const int dh = (int)(bhd % C::NH);  // gradient column half
    const uint32_t bh = (uint32_t)(bhd / C::NH);
    const int64_t hk = bh % (uint32_t)p.Hkv, b = bh / (uint32_t)p.Hkv, k0 = kt * TILE;
    // Query blocks this CTA visits: for each query head of the group, rows [r_begin, L).
    const int64_t r_begin = p.causal ? min(k0, p.L) : 0;
    const int qb_first = (int)(r_begin / QB);
    const int qb_per_head = (int)((p.L + QB - 1) / QB) - qb_first;
    const int nblk = qb_per_head * p.group;
    auto bar = [&](int i) { return sb + C::OFF_BAR + 8u * (uint32_t)i; };
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(sg + C::OFF_MISC);
    volatile int *abort = reinterpret_cast<volatile int *>(sg + C::OFF_MISC + 4);
    int *err = a.err;
    auto blk_coords = [&](int i, int64_t &h, int64_t &q0) {
        h = hk * p.group + i / qb_per_head;
        q0 = (int64_t)(qb_first + i % qb_per_head) * QB;
    };

    if (threadIdx.x == 0) {
        mbar_init(bar(C::KV_FULL), 1);
        mbar_init(bar(C::KV_READY), 256);
        mbar_init(bar(C::KVLO_FULL), 1);
        for (int i = C::QK_FULL; i <= C::QMN_EMPTY; i++) mbar_init(bar(i), 1);
        mbar_init(bar(C::S_FULL), 1);
        mbar_init(bar(C::DP_FULL), 1);
        mbar_init(bar(C::P_READY), 256);
        mbar_init(bar(C::DS_READY), 256);
        mbar_init(bar(C::DV_DONE), 1);
        mbar_init(bar(C::DK_DONE), 1);
        mbar_init(bar(C::DV_FREE), 128);
        mbar_init(bar(C::DK_FREE), 128);
        mbar_init(bar(C::DRAIN), 1);
        mbar_init(bar(C::DRAIN_G), 1);
        mbar_init(bar(C::DK_ISSUED), 1);
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == W_MMA) {
        tmem_alloc(smem_addr(tmem_slot), C::TCOLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // Launched as a dependent of the pre-pass: set-up above overlapped its last blocks; its
    // lo copies, lse and delta are read only after this.
    griddep_wait();

    // One streamed tile (hi and, with SPLIT, lo) of query block i into a stage: all DD columns
    // (K-major) or this CTA's 64-column half (MN-major).
    auto load_tile = [&](const CUtensorMap *tm, const CUtensorMap *tm_lo, uint32_t stage, uint32_t full, int i, bool mn) {
        int64_t h, q0;
        blk_coords(i, h, q0);
        const int nch = mn ? 2 : DD / 32;
        const uint32_t bytes = mn ? C::TM_BYTES : C::TK_BYTES, chunk = mn ? C::TM_CHUNK : C::TK_CHUNK;
        const int col0 = mn ? 64 * dh : 0;
        mbar_expect_tx(full, (SPLIT ? 2 : 1) * bytes);
        for (int c = 0; c < nch; c++) {
            tma_load_4d(tm, stage + c * chunk, full, col0 + 32 * c, (int)q0, (int)h, (int)b);
            if (SPLIT) tma_load_4d(tm_lo, stage + bytes + c * chunk, full, col0 + 32 * c, (int)q0, (int)h, (int)b);
        }
    };

    if (warp == W_PROD) {
        // ------------------------ producer: K / V (hi, then lo), then the Q_K and dO_K tiles ----
        if (lane == 0) {
            int qk_issued = -1, dok_issued = -1;
            const bool lo_later = DD != 64;  // DD = 128 stages the hi tiles in the lo areas
            mbar_expect_tx(bar(C::KV_FULL), ((SPLIT && !lo_later) ? 4 : 2) * C::RESB);
            for (int c = 0; c < DD / 32; c++) {
                tma_load_4d(&tm_k, sb + C::OFF_KHI_STAGE + c * RES_CHUNK, bar(C::KV_FULL), 32 * c, (int)k0, (int)hk, (int)b);
                tma_load_4d(&tm_v, sb + C::OFF_VHI_STAGE + c * RES_CHUNK, bar(C::KV_FULL), 32 * c, (int)k0, (int)hk, (int)b);
                if (SPLIT && !lo_later) {
                    tma_load_4d(&tm_k_lo, sb + C::OFF_KLO + c * RES_CHUNK, bar(C::KV_FULL), 32 * c, (int)k0, (int)hk, (int)b);
                    tma_load_4d(&tm_v_lo, sb + C::OFF_VLO + c * RES_CHUNK, bar(C::KV_FULL), 32 * c, (int)k0, (int)hk, (int)b);
                }
            }
            if (!SPLIT || !lo_later) mbar_arrive(bar(C::KVLO_FULL));
            // DD = 128 loads the lo copies where the hi tiles wait: after they left for TMEM.
            bool ok = !lo_later || mbar_wait(bar(C::KV_READY), 0, abort, err);
            if (ok && SPLIT && lo_later) {
                mbar_expect_tx(bar(C::KVLO_FULL), 2 * C::RESB);
                for (int c = 0; c < DD / 32; c++) {
                    tma_load_4d(&tm_k_lo, sb + C::OFF_KLO + c * RES_CHUNK, bar(C::KVLO_FULL), 32 * c, (int)k0, (int)hk, (int)b);
                    tma_load_4d(&tm_v_lo, sb + C::OFF_VLO + c * RES_CHUNK, bar(C::KVLO_FULL), 32 * c, (int)k0, (int)hk, (int)b);
                }
            }
            for (int i = 0; ok && i < nblk; i++) {
                if (i >= 1 && !mbar_wait(bar(C::QK_EMPTY), (i - 1) & 1, abort, err)) break;
                load_tile(&tm_qk, &tm_qk_lo, sb + C::OFF_QK, bar(C::QK_FULL), i, false);
                qk_issued = i;
                if (i >= 1 && !mbar_wait(bar(C::DOK_EMPTY), (i - 1) & 1, abort, err)) break;
                load_tile(&tm_dok, &tm_dok_lo, sb + C::OFF_DOK, bar(C::DOK_FULL), i, false);
                dok_issued = i;
            }
            if (*abort) {  // let the copies in flight land before the CTA exits
                volatile int never = 0;
                mbar_wait(bar(C::KV_FULL), 0, &never, nullptr);
                if (ok && SPLIT && lo_later) mbar_wait(bar(C::KVLO_FULL), 0, &never, nullptr);
                if (qk_issued >= 0) mbar_wait(bar(C::QK_FULL), qk_issued & 1, &never, nullptr);
                if (dok_issued >= 0) mbar_wait(bar(C::DOK_FULL), dok_issued & 1, &never, nullptr);
            }
        }
    } else if (warp == W_PROD2) {
        // ------------------------------------------ producer: the dO_MN and Q_MN tiles ----
        if (lane == 0) {
            int domn_issued = -1, qmn_issued = -1;
            // DD = 64: K hi and V hi wait in these stages until the softmax warps moved them.
            const bool staged = DD != 64 || mbar_wait(bar(C::KV_READY), 0, abort, err);
            for (int i = 0; staged && i < nblk; i++) {
                if (i >= 1 && !mbar_wait(bar(C::DOMN_EMPTY), (i - 1) & 1, abort, err)) break;
                load_tile(&tm_domn, &tm_domn_lo, sb + C::OFF_DOMN, bar(C::DOMN_FULL), i, true);
                domn_issued = i;
                if (i >= 1 && !mbar_wait(bar(C::QMN_EMPTY), (i - 1) & 1, abort, err)) break;
                load_tile(&tm_qmn, &tm_qmn_lo, sb + C::OFF_QMN, bar(C::QMN_FULL), i, true);
                qmn_issued = i;
                if (*abort) break;
            }
            if (*abort) {
                volatile int never = 0;
                if (domn_issued >= 0) mbar_wait(bar(C::DOMN_FULL), domn_issued & 1, &never, nullptr);
                if (qmn_issued >= 0) mbar_wait(bar(C::QMN_FULL), qmn_issued & 1, &never, nullptr);
            }
        }
    } else if (warp == W_MMA) {
        // ---------------------------------------------------- MMA: S^T and dP^T, one warp ----
        {
            const uint64_t klo = sdesc_sw128(sb + C::OFF_KLO, 16, 1024), vlo = sdesc_sw128(sb + C::OFF_VLO, 16, 1024);
            bool ok = warp_wait(bar(C::KV_READY), 0, abort, err) && warp_wait(bar(C::KVLO_FULL), 0, abort, err);
            tc_fence_after();
            for (int i = 0; ok && i < nblk; i++) {
                if (!warp_wait(bar(C::QK_FULL), i & 1, abort, err)) break;
                if (i >= 1 && !warp_wait(bar(C::DV_DONE), (i - 1) & 1, abort, err)) break;
                // dK_{i-1} goes to the tensor core ahead of S^T_i: the warps folding dK finish
                // with it while S^T_i runs, instead of after, on the way to P^T_i.
                if (i >= 1 && !warp_wait(bar(C::DK_ISSUED), (i - 1) & 1, abort, err)) break;
                tc_fence_after();
                mma_s<SPLIT, QB, DD>(tmem + C::C_S, tmem + C::C_KHI, klo, sdesc_sw128(sb + C::OFF_QK, 16, 1024));
                tc_commit_w(bar(C::S_FULL));
                tc_commit_w(bar(C::QK_EMPTY));
                if (!warp_wait(bar(C::DOK_FULL), i & 1, abort, err)) break;
                if (i >= 1 && !warp_wait(bar(C::DK_DONE), (i - 1) & 1, abort, err)) break;
                tc_fence_after();
                mma_s<SPLIT, QB, DD>(tmem + C::C_DP, tmem + C::C_VHI, vlo, sdesc_sw128(sb + C::OFF_DOK, 16, 1024));
                tc_commit_w(bar(C::DP_FULL));
                tc_commit_w(bar(C::DOK_EMPTY));
            }
            // Every MMA this warp issued completes before TMEM is released.
            tc_commit_w(bar(C::DRAIN));
            volatile int never = 0;
            warp_wait(bar(C::DRAIN), 0, &never, nullptr);
        }
    } else if (warp == W_GMMA) {
        // ------------------------------------------------ MMA: dV_blk and dK_blk, one warp ----
        {
            bool ok = true;
            for (int i = 0; ok && i < nblk; i++) {
                if (!warp_wait(bar(C::P_READY), i & 1, abort, err)) break;
                if (!warp_wait(bar(C::DOMN_FULL), i & 1, abort, err)) break;
                if (i >= 1 && !warp_wait(bar(C::DV_FREE), (i - 1) & 1, abort, err)) break;
                tc_fence_after();
                mma_g<SPLIT, QB>(tmem + C::C_DV, tmem + C::C_S, tmem + C::C_PLO,
                                 sdesc_mn_sw128_32b(sb + C::OFF_DOMN, C::TM_CHUNK, 512), false);
                tc_commit_w(bar(C::DV_DONE));
                tc_commit_w(bar(C::DOMN_EMPTY));
                if (!warp_wait(bar(C::DS_READY), i & 1, abort, err)) break;
                if (!warp_wait(bar(C::QMN_FULL), i & 1, abort, err)) break;
                if (i >= 1 && !warp_wait(bar(C::DK_FREE), (i - 1) & 1, abort, err)) break;
                tc_fence_after();
                mma_g<SPLIT, QB>(tmem + C::C_DK, tmem + C::C_DP, tmem + C::C_DSLO,
                                 sdesc_mn_sw128_32b(sb + C::OFF_QMN, C::TM_CHUNK, 512), false);
                tc_commit_w(bar(C::DK_DONE));
                if (lane == 0) mbar_arrive(bar(C::DK_ISSUED));
                tc_commit_w(bar(C::QMN_EMPTY));
            }
            tc_commit_w(bar(C::DRAIN_G));
            volatile int never = 0;
            warp_wait(bar(C::DRAIN_G), 0, &never, nullptr);
        }
    } else if (warp < W_PROD) {
        // ------------------------- P^T and dS^T, then the fp32 dV / dK folds, every block ----
        const int quad = warp & 3, half = warp >> 2;  // lane quadrant; query-column half / dV or dK
        const int row = quad * 32 + lane;             // key row of this CTA
        const int64_t key = k0 + row;
        const bool key_ok = key < p.S;
        const uint32_t tl = tmem + ((uint32_t)(quad * 32) << 16);
        const int cb = half * CPT;  // this thread's query columns of a block
        float acc[64];              // this CTA's 64 columns of dV (half 0) or dK (half 1)
#pragma unroll
        for (int x = 0; x < 64; x++) acc[x] = 0.0f;
        bool ok = warp_wait(bar(C::KV_FULL), 0, abort, err);
        if (ok) {  // K (half 0) or V (half 1) hi rows into TMEM
            row_to_tmem<DD>(sg + (half ? C::OFF_VHI_STAGE : C::OFF_KHI_STAGE), row, tl, half ? C::C_VHI : C::C_KHI);
            tmem_wait_st();
            fence_proxy_async_smem();
            tc_fence_before();
            mbar_arrive(bar(C::KV_READY));
        }
        // Adds block i's accumulator (dV for half 0, dK for half 1) into registers and frees it.
        // (Deferring it until after the next block's P^T was measured slower: the fold's TMEM
        // loads then sit on the path to dS^T.)
        auto fold = [&](int i) -> bool {
            if (!warp_wait(bar(half ? C::DK_DONE : C::DV_DONE), i & 1, abort, err)) return false;
            tc_fence_after();
            const uint32_t col = half ? C::C_DK : C::C_DV;
#pragma unroll
            for (int c = 0; c < 4; c++) fold16(tl + col + 16 * c, acc + 16 * c);
            tc_fence_before();
            mbar_arrive(bar(half ? C::DK_FREE : C::DV_FREE));
            return true;
        };
        // Lane c holds the lse (base 2) and the delta of this half's query column c of block i.
        auto colvals = [&](int i, float &lse2, float &del) {
            int64_t h, q0;
            blk_coords(i, h, q0);
            const int64_t q = q0 + cb + (lane % CPT);
            lse2 = del = 0.0f;
            if (q < p.L) {
                const int64_t idx = (b * p.H + h) * p.L + q;
                lse2 = a.lse2[idx];
                del = a.g.delta[idx];
            }
        };
        float cur_l = 0.0f, cur_d = 0.0f;
        if (ok && nblk > 0) colvals(0, cur_l, cur_d);
        for (int i = 0; ok && i < nblk; i++) {
            int64_t h, q0;
            blk_coords(i, h, q0);
            float nxt_l = 0.0f, nxt_d = 0.0f;
            if (i + 1 < nblk) colvals(i + 1, nxt_l, nxt_d);
            // Column c is query base + c: valid below L and, under causal masking, from `key` on.
            const int64_t base = q0 + cb;
            const bool edge = MASKED || !key_ok || q0 + QB > p.L || (p.causal && key > q0);
            uint32_t vbits = 0xFFFFFFFFu;
            if (edge) vbits = key_ok ? col_bits32(p.causal ? key - base : 0, p.L - base) : 0u;
            // The user mask down this key's column, loaded before the wait for S.
            float mk[MASKED ? CPT : 1];
            if constexpr (MASKED) mask_run<CPT>(p, b, h, base, key, p.ms[2], vbits, mk);
            // Dropout: the keep bits of (query base + c, this key). The weights that meet dO are
            // P * Z; dS = P (Z dP - delta), Z = keep_scale where kept, 0 where dropped. The
            // warp's lanes are 32 consecutive keys: one row read per lane, transposed by ballots.
            uint32_t zb = 0;
            if constexpr (DROP) {
                zb = transpose_bits32(lane < CPT ? keep_run32(p, b, h, base + lane, key - lane) : 0u, lane);
                if (!key_ok) zb = 0u;  // every lane took part in the ballots
            }
            if (!warp_wait(bar(C::S_FULL), i & 1, abort, err)) {
                ok = false;
                break;
            }
            tc_fence_after();
            float pv[CPT];  // P (undropped) of this key and the query columns
#pragma unroll
            for (int r0 = 0; r0 < CPT; r0 += 16) {
                uint32_t sr[16];
                tmem_ld16(tl + C::C_S + cb + r0, sr);
                tmem_wait_ld();
#pragma unroll
                for (int c = 0; c < 16; c++) {
                    const float lse2 = __shfl_sync(FULL, cur_l, r0 + c);
                    float x;
                    if (MASKED) x = fmaf(mk[MASKED ? r0 + c : 0], LOG2E, __uint_as_float(sr[c]) * a.scale_log2) - lse2;
                    else x = fmaf(__uint_as_float(sr[c]), a.scale_log2, -lse2);
                    pv[r0 + c] = ((vbits >> (r0 + c)) & 1u) ? ex2_approx(x) : 0.0f;
                }
            }
#pragma unroll
            for (int r0 = 0; r0 < CPT; r0 += 16) {
                uint32_t xh[16], xl[16];
#pragma unroll
                for (int c = 0; c < 16; c++) {
                    float pw = pv[r0 + c];
                    if constexpr (DROP) pw = ((zb >> (r0 + c)) & 1u) ? pw * p.keep_scale : 0.0f;
                    if (SPLIT) {
                        xh[c] = __float_as_uint(pw);
                        xl[c] = tf32_lo_trunc(pw);
                    } else {
                        xh[c] = tf32_rna(pw);
                    }
                }
                tmem_st16(tl + C::C_S + cb + r0, xh);
                if (SPLIT) tmem_st16(tl + C::C_PLO + cb + r0, xl);
            }
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(bar(C::P_READY));
            if (!warp_wait(bar(C::DP_FULL), i & 1, abort, err)) {
                ok = false;
                break;
            }
            tc_fence_after();
#pragma unroll
            for (int r0 = 0; r0 < CPT; r0 += 16) {
                uint32_t dr[16], xh[16], xl[16];
                tmem_ld16(tl + C::C_DP + cb + r0, dr);
                tmem_wait_ld();
#pragma unroll
                for (int c = 0; c < 16; c++) {
                    const float del = __shfl_sync(FULL, cur_d, r0 + c);
                    float dpv = __uint_as_float(dr[c]);
                    if constexpr (DROP) dpv = ((zb >> (r0 + c)) & 1u) ? dpv * p.keep_scale : 0.0f;
                    const float ds = pv[r0 + c] * (dpv - del);
                    if (SPLIT) {
                        xh[c] = __float_as_uint(ds);
                        xl[c] = tf32_lo_trunc(ds);
                    } else {
                        xh[c] = tf32_rna(ds);
                    }
                }
                tmem_st16(tl + C::C_DP + cb + r0, xh);
                if (SPLIT) tmem_st16(tl + C::C_DSLO + cb + r0, xl);
            }
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(bar(C::DS_READY));
            cur_l = nxt_l;
            cur_d = nxt_d;
            if (!fold(i)) {
                ok = false;
                break;
            }
        }
        const bool aborted = __any_sync(FULL, *abort != 0);
        if (ok && !aborted && key_ok) {
            if (half) {
                float *dkr = a.g.dk + b * a.g.dks[0] + hk * a.g.dks[1] + key * a.g.dks[2] + (int64_t)(64 * dh) * a.g.dks[3];
                store_row<64>(dkr, a.g.dks[3], acc, p.scale);
            } else {
                float *dvr = a.g.dv + b * a.g.dvs[0] + hk * a.g.dvs[1] + key * a.g.dvs[2] + (int64_t)(64 * dh) * a.g.dvs[3];
                store_row<64>(dvr, a.g.dvs[3], acc, 1.0f);
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == W_MMA) {
        tc_fence_after();
        tmem_dealloc(tmem, C::TCOLS);
    }
}

// ========================================================================= dQ ========
// Head dim DD = 64: a CTA computes all of dQ for its query rows, with Q and dO (hi and lo) in
// TMEM. DD = 128: two CTAs per query tile, each computing one 64-column half of dQ (both
// recompute S and dP over the whole head dim); Q hi and dO hi fill 256 TMEM columns, so their
// lo copies stay in shared memory and those passes read A from there.
template <int DD>
struct QqCfg {
    static constexpr int NH = DD / 64;             // dQ column halves (CTAs per query tile)
    static constexpr int NB = DD == 64 ? 64 : 32;  // keys per streamed block (S / dP's N)
    static constexpr int CPT = NB / 2;             // key columns per softmax thread
    static constexpr bool LO_TMEM = DD == 64;      // Q lo / dO lo in TMEM, else in shared memory
    static constexpr uint32_t RESB = TILE * DD * 4;                        // resident Q or dO tile
    static constexpr uint32_t TK_BYTES = NB * DD * 4, TK_CHUNK = NB * 128;  // K-major K / V tile
    static constexpr uint32_t TM_BYTES = NB * 64 * 4, TM_CHUNK = NB * 128;  // MN-major K half tile
    // Rings (a stage holds a tile's hi and lo copies), each freed by its own reader: K (K-major)
    // by the S MMAs, V (K-major) by the dP MMAs, K (MN-major) by the dQ MMAs.
    static constexpr int NST_K = DD == 64 ? 2 : 1, NST_G = 2;
    static constexpr uint32_t KSTAGE = 2 * TK_BYTES, GSTAGE = 2 * TM_BYTES;
    static constexpr uint32_t OFF_QLO = 0, OFF_DOLO = RESB, OFF_KK = LO_TMEM ? 0 : 2 * RESB,
                              OFF_VK = OFF_KK + NST_K * KSTAGE, OFF_KMN = OFF_VK + NST_K * KSTAGE,
                              OFF_BAR = OFF_KMN + NST_G * GSTAGE;
    // Where Q / dO wait until the softmax warps move them into TMEM: DD = 64, Q in the MN-major
    // ring and dO in the V ring (the K ring, which the first S MMA needs, fills meanwhile);
    // DD = 128, hi in the lo areas (the lo copies are loaded after).
    static constexpr uint32_t OFF_QHI_STAGE = LO_TMEM ? OFF_KMN : OFF_QLO,
                              OFF_DOHI_STAGE = LO_TMEM ? OFF_VK : OFF_DOLO,
                              OFF_QLO_STAGE = OFF_KMN + RESB, OFF_DOLO_STAGE = OFF_VK + RESB;
    // Per block j: S (S_FULL) read out by the softmax warps (S_READ: S_{j+1} may overwrite it);
    // dP (DP_FULL) turned into dS hi / lo (DS_READY); dQ_blk = dS K (DQ_DONE: dS read, dP_{j+1}
    // may overwrite it) folded into registers (DQ_FREE: the accumulator may restart).
    // QDLO_FULL: the lo copies of Q / dO in shared memory (DD = 128).
    enum { QD_FULL, QD_READY, QDLO_FULL, KK_FULL, KK_EMPTY = KK_FULL + NST_K, VK_FULL = KK_EMPTY + NST_K,
           VK_EMPTY = VK_FULL + NST_K, SG_FULL = VK_EMPTY + NST_K, SG_EMPTY = SG_FULL + NST_G,
           S_FULL = SG_EMPTY + NST_G, S_READ, DP_FULL, DS_READY, DQ_DONE, DQ_FREE, DRAIN, DRAIN_G, NBAR };
    static constexpr uint32_t OFF_MISC = OFF_BAR + NBAR * 8;
    static constexpr uint32_t SMEM = OFF_MISC + 16 + 1024;
    // TMEM: Q hi | [Q lo] | dO hi | [dO lo] | S | dP / dS hi | dS lo | dQ_blk
    static constexpr uint32_t C_QHI = 0, C_QLO = DD, C_DOHI = LO_TMEM ? 2 * DD : DD, C_DOLO = C_DOHI + DD,
                              C_S = LO_TMEM ? 4 * DD : 2 * DD, C_DP = C_S + NB, C_DSLO = C_S + 2 * NB,
                              C_DQB = C_S + 3 * NB, TCOLS = 512;
    static_assert(C_DQB + 64 <= TCOLS, "tensor memory budget");
    static_assert(!LO_TMEM || (2 * RESB <= NST_K * KSTAGE && 2 * RESB <= NST_G * GSTAGE),
                  "Q / dO tiles are staged in the MN-major and V rings");
    static_assert(SMEM <= 232448, "smem");
};

// tm_q / tm_do: (DD, L, H, S2*B), box 128 rows; tm_kk / tm_kmn / tm_vk: (DD, S, Hkv, S2*B),
// box NB rows (tm_kmn: this CTA's 64-column half).
//
// One MMA warp issues S_0, dP_0, then per block j: S_{j+1} (once the softmax warps have read
// S_j) and dP_{j+1} (once dQ_j has read dS_j); a second issues dQ_j once dS_j is in TMEM. The
// tensor core thus runs ... dQ_j, dP_{j+1}, S_{j+2}, dQ_{j+1} ... while the softmax warps
// compute dS_{j+1} under S_{j+2} and P_{j+2} under dQ_{j+1}.
template <int DD, bool SPLIT, bool MASKED, bool DROP>
__global__ void __maxnreg__(168)
    attn_bwd_dq_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_do,
                          const __grid_constant__ CUtensorMap tm_kk, const __grid_constant__ CUtensorMap tm_kmn,
                          const __grid_constant__ CUtensorMap tm_vk, const __grid_constant__ CUtensorMap tm_q_lo,
                          const __grid_constant__ CUtensorMap tm_do_lo, const __grid_constant__ CUtensorMap tm_kk_lo,
                          const __grid_constant__ CUtensorMap tm_kmn_lo, const __grid_constant__ CUtensorMap tm_vk_lo,
                          const TcBwdArgs a) {
    using C = QqCfg<DD>;
    constexpr int NB = C::NB, CPT = C::CPT, NST_K = C::NST_K, NST_G = C::NST_G;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_addr(smem_raw);
    const uint32_t sb = (raw + 1023u) & ~1023u;
    uint8_t *sg = smem_raw + (sb - raw);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const AttnProblem &p = a.p;
    // Query tiles in descending order: under causal masking the last tile sees the most keys.
    const int64_t ntiles = (p.L + TILE - 1) / TILE;
    int64_t qt, bhd;
    grouped_tile(blockIdx.x, (uint32_t)ntiles, (uint32_t)(p.B * p.H * C::NH), qt, bhd);
    qt = ntiles - 1 - qt;
    const int dh = (int)(bhd % C::NH);  // dQ column half
    const uint32_t bh = (uint32_t)(bhd / C::NH);
    const int64_t h = bh % (uint32_t)p.H, b = bh / (uint32_t)p.H, hk = (uint32_t)h / (uint32_t)p.group;
    const int64_t q0 = qt * TILE;
    const int64_t kv_end = p.causal ? min(p.S, q0 + TILE) : p.S;
    const int nblk = (int)((kv_end + NB - 1) / NB);
    auto bar = [&](int i) { return sb + C::OFF_BAR + 8u * (uint32_t)i; };
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(sg + C::OFF_MISC);
    volatile int *abort = reinterpret_cast<volatile int *>(sg + C::OFF_MISC + 4);
    int *err = a.err;

    if (threadIdx.x == 0) {
        mbar_init(bar(C::QD_FULL), 1);
        mbar_init(bar(C::QD_READY), 256);
        mbar_init(bar(C::QDLO_FULL), 1);
        for (int s = 0; s < NST_K; s++) {
            mbar_init(bar(C::KK_FULL + s), 1);
            mbar_init(bar(C::KK_EMPTY + s), 1);
            mbar_init(bar(C::VK_FULL + s), 1);
            mbar_init(bar(C::VK_EMPTY + s), 1);
        }
        for (int s = 0; s < NST_G; s++) {
            mbar_init(bar(C::SG_FULL + s), 1);
            mbar_init(bar(C::SG_EMPTY + s), 1);
        }
        mbar_init(bar(C::S_FULL), 1);
        mbar_init(bar(C::S_READ), 256);
        mbar_init(bar(C::DP_FULL), 1);
        mbar_init(bar(C::DS_READY), 256);
        mbar_init(bar(C::DQ_DONE), 1);
        mbar_init(bar(C::DQ_FREE), 256);
        mbar_init(bar(C::DRAIN), 1);
        mbar_init(bar(C::DRAIN_G), 1);
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == W_MMA) {
        tmem_alloc(smem_addr(tmem_slot), C::TCOLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == W_PROD) {
        // ------------------------------ producer: Q / dO (hi, lo), then the K and V rings ----
        if (lane == 0) {
            int k_issued = -1, v_issued = -1;
            const bool lo_now = SPLIT && C::LO_TMEM;
            mbar_expect_tx(bar(C::QD_FULL), (lo_now ? 4 : 2) * C::RESB);
            for (int c = 0; c < DD / 32; c++) {
                tma_load_4d(&tm_q, sb + C::OFF_QHI_STAGE + c * RES_CHUNK, bar(C::QD_FULL), 32 * c, (int)q0, (int)h, (int)b);
                tma_load_4d(&tm_do, sb + C::OFF_DOHI_STAGE + c * RES_CHUNK, bar(C::QD_FULL), 32 * c, (int)q0, (int)h, (int)b);
                if (lo_now) {
                    tma_load_4d(&tm_q_lo, sb + C::OFF_QLO_STAGE + c * RES_CHUNK, bar(C::QD_FULL), 32 * c, (int)q0, (int)h, (int)b);
                    tma_load_4d(&tm_do_lo, sb + C::OFF_DOLO_STAGE + c * RES_CHUNK, bar(C::QD_FULL), 32 * c, (int)q0, (int)h, (int)b);
                }
            }
            if (!(SPLIT && !C::LO_TMEM)) mbar_arrive(bar(C::QDLO_FULL));
            // DD = 64 stages dO in the V ring: the K ring fills at once and the first V load
            // waits below. DD = 128 loads the lo copies where the hi tiles wait, after they left.
            bool ok = C::LO_TMEM || mbar_wait(bar(C::QD_READY), 0, abort, err);
            const bool lo_later = ok && SPLIT && !C::LO_TMEM;
            if (lo_later) {
                mbar_expect_tx(bar(C::QDLO_FULL), 2 * C::RESB);
                for (int c = 0; c < DD / 32; c++) {
                    tma_load_4d(&tm_q_lo, sb + C::OFF_QLO + c * RES_CHUNK, bar(C::QDLO_FULL), 32 * c, (int)q0, (int)h, (int)b);
                    tma_load_4d(&tm_do_lo, sb + C::OFF_DOLO + c * RES_CHUNK, bar(C::QDLO_FULL), 32 * c, (int)q0, (int)h, (int)b);
                }
            }
            for (int j = 0; ok && j < nblk; j++) {
                const int st = j % NST_K;
                if (j >= NST_K && !mbar_wait(bar(C::KK_EMPTY + st), ((j / NST_K) - 1) & 1, abort, err)) break;
                mbar_expect_tx(bar(C::KK_FULL + st), (SPLIT ? 2 : 1) * C::TK_BYTES);
                for (int c = 0; c < DD / 32; c++) {
                    const uint32_t o = C::OFF_KK + st * C::KSTAGE + c * C::TK_CHUNK;
                    tma_load_4d(&tm_kk, sb + o, bar(C::KK_FULL + st), 32 * c, j * NB, (int)hk, (int)b);
                    if (SPLIT) tma_load_4d(&tm_kk_lo, sb + o + C::TK_BYTES, bar(C::KK_FULL + st), 32 * c, j * NB, (int)hk, (int)b);
                }
                k_issued = j;
                if (C::LO_TMEM && j == 0 && !(ok = mbar_wait(bar(C::QD_READY), 0, abort, err))) break;
                if (j >= NST_K && !mbar_wait(bar(C::VK_EMPTY + st), ((j / NST_K) - 1) & 1, abort, err)) break;
                mbar_expect_tx(bar(C::VK_FULL + st), (SPLIT ? 2 : 1) * C::TK_BYTES);
                for (int c = 0; c < DD / 32; c++) {
                    const uint32_t o = C::OFF_VK + st * C::KSTAGE + c * C::TK_CHUNK;
                    tma_load_4d(&tm_vk, sb + o, bar(C::VK_FULL + st), 32 * c, j * NB, (int)hk, (int)b);
                    if (SPLIT) tma_load_4d(&tm_vk_lo, sb + o + C::TK_BYTES, bar(C::VK_FULL + st), 32 * c, j * NB, (int)hk, (int)b);
                }
                v_issued = j;
            }
            if (*abort) {
                volatile int never = 0;
                mbar_wait(bar(C::QD_FULL), 0, &never, nullptr);
                if (lo_later) mbar_wait(bar(C::QDLO_FULL), 0, &never, nullptr);
                for (int j = max(0, k_issued - NST_K + 1); j <= k_issued; j++)
                    mbar_wait(bar(C::KK_FULL + j % NST_K), (j / NST_K) & 1, &never, nullptr);
                for (int j = max(0, v_issued - NST_K + 1); j <= v_issued; j++)
                    mbar_wait(bar(C::VK_FULL + j % NST_K), (j / NST_K) & 1, &never, nullptr);
            }
        }
    } else if (warp == W_PROD2) {
        // ------------------------------------------------ producer: the MN-major ring ----
        if (lane == 0) {
            int issued = -1;
            // DD = 64 stages Q in this ring: its first load waits until Q has left for TMEM.
            const bool staged = !C::LO_TMEM || mbar_wait(bar(C::QD_READY), 0, abort, err);
            for (int j = 0; staged && j < nblk; j++) {
                const int st = j % NST_G;
                if (j >= NST_G && !mbar_wait(bar(C::SG_EMPTY + st), ((j / NST_G) - 1) & 1, abort, err)) break;
                mbar_expect_tx(bar(C::SG_FULL + st), (SPLIT ? 2 : 1) * C::TM_BYTES);
                for (int c = 0; c < 2; c++) {
                    const uint32_t o = C::OFF_KMN + st * C::GSTAGE + c * C::TM_CHUNK;
                    const int col = 64 * dh + 32 * c;
                    tma_load_4d(&tm_kmn, sb + o, bar(C::SG_FULL + st), col, j * NB, (int)hk, (int)b);
                    if (SPLIT) tma_load_4d(&tm_kmn_lo, sb + o + C::TM_BYTES, bar(C::SG_FULL + st), col, j * NB, (int)hk, (int)b);
                }
                issued = j;
                if (*abort) break;
            }
            if (*abort) {
                volatile int never = 0;
                for (int j = max(0, issued - NST_G + 1); j <= issued; j++)
                    mbar_wait(bar(C::SG_FULL + j % NST_G), (j / NST_G) & 1, &never, nullptr);
            }
        }
    } else if (warp == W_MMA) {
        // ------------------------------------------------------ MMA: S and dP, one warp ----
        // A tensor-core MMA issue blocks once a few hundred cycles of work are queued, so any
        // wait of the issuing warp idles the tensor core: S / dP and dQ have a warp each, and
        // one warp's waits overlap the other's MMAs.
        {
            const uint64_t qlo = sdesc_sw128(sb + C::OFF_QLO, 16, 1024), dolo = sdesc_sw128(sb + C::OFF_DOLO, 16, 1024);
            auto s_mma = [&](int j) {
                const uint32_t st = C::OFF_KK + (j % NST_K) * C::KSTAGE;
                if constexpr (C::LO_TMEM)
                    mma_s_t<SPLIT, NB, DD>(tmem + C::C_S, tmem + C::C_QHI, tmem + C::C_QLO, sdesc_sw128(sb + st, 16, 1024));
                else
                    mma_s<SPLIT, NB, DD>(tmem + C::C_S, tmem + C::C_QHI, qlo, sdesc_sw128(sb + st, 16, 1024));
                tc_commit_w(bar(C::S_FULL));
                tc_commit_w(bar(C::KK_EMPTY + j % NST_K));
            };
            auto dp_mma = [&](int j) {
                const uint32_t st = C::OFF_VK + (j % NST_K) * C::KSTAGE;
                if constexpr (C::LO_TMEM)
                    mma_s_t<SPLIT, NB, DD>(tmem + C::C_DP, tmem + C::C_DOHI, tmem + C::C_DOLO, sdesc_sw128(sb + st, 16, 1024));
                else
                    mma_s<SPLIT, NB, DD>(tmem + C::C_DP, tmem + C::C_DOHI, dolo, sdesc_sw128(sb + st, 16, 1024));
                tc_commit_w(bar(C::DP_FULL));
                tc_commit_w(bar(C::VK_EMPTY + j % NST_K));
            };
            bool ok = warp_wait(bar(C::QD_READY), 0, abort, err) && warp_wait(bar(C::QDLO_FULL), 0, abort, err);
            tc_fence_after();
            if (ok && nblk > 0) {
                ok = warp_wait(bar(C::KK_FULL), 0, abort, err) && warp_wait(bar(C::VK_FULL), 0, abort, err);
                tc_fence_after();
                if (ok) {
                    s_mma(0);
                    dp_mma(0);
                }
            }
            for (int j = 0; ok && j + 1 < nblk; j++) {
                const int nx = j + 1;
                // S of block j+1 overwrites S_j once the softmax warps hold it in registers.
                if (!warp_wait(bar(C::S_READ), j & 1, abort, err)) break;
                if (!warp_wait(bar(C::KK_FULL + nx % NST_K), (nx / NST_K) & 1, abort, err)) break;
                tc_fence_after();
                s_mma(nx);
                // dP of block j+1 overwrites dS_j once dQ_j has read it.
                if (!warp_wait(bar(C::DQ_DONE), j & 1, abort, err)) break;
                if (!warp_wait(bar(C::VK_FULL + nx % NST_K), (nx / NST_K) & 1, abort, err)) break;
                tc_fence_after();
                dp_mma(nx);
            }
            // Every MMA this warp issued completes before TMEM is released.
            tc_commit_w(bar(C::DRAIN));
            volatile int never = 0;
            warp_wait(bar(C::DRAIN), 0, &never, nullptr);
        }
    } else if (warp == W_GMMA) {
        // ------------------------------------------------------------- MMA: dQ_blk = dS K ----
        {
            bool ok = true;
            for (int j = 0; ok && j < nblk; j++) {
                const int sgi = j % NST_G;
                if (!warp_wait(bar(C::DS_READY), j & 1, abort, err)) break;
                if (!warp_wait(bar(C::SG_FULL + sgi), (j / NST_G) & 1, abort, err)) break;
                if (j >= 1 && !warp_wait(bar(C::DQ_FREE), (j - 1) & 1, abort, err)) break;
                tc_fence_after();
                mma_g<SPLIT, NB>(tmem + C::C_DQB, tmem + C::C_DP, tmem + C::C_DSLO,
                                 sdesc_mn_sw128_32b(sb + C::OFF_KMN + sgi * C::GSTAGE, C::TM_CHUNK, 512), false);
                tc_commit_w(bar(C::DQ_DONE));
                tc_commit_w(bar(C::SG_EMPTY + sgi));
            }
            tc_commit_w(bar(C::DRAIN_G));
            volatile int never = 0;
            warp_wait(bar(C::DRAIN_G), 0, &never, nullptr);
        }
    } else if (warp < W_PROD) {
        // ----------------------------------------------------- dS, then the fp32 dQ fold --
        const int quad = warp & 3, half = warp >> 2;
        const int row = quad * 32 + lane;
        const int64_t q = q0 + row;
        const bool row_ok = q < p.L;
        const uint32_t tl = tmem + ((uint32_t)(quad * 32) << 16);
        const int cb = half * CPT;  // this thread's key columns of a block
        float acc[32];              // dQ columns [64 dh + 32 half, +32)
#pragma unroll
        for (int x = 0; x < 32; x++) acc[x] = 0.0f;
        bool ok = warp_wait(bar(C::QD_FULL), 0, abort, err);
        if (ok) {  // Q (half 0) or dO (half 1) rows into TMEM: hi, and lo when it lives there
            row_to_tmem<DD>(sg + (half ? C::OFF_DOHI_STAGE : C::OFF_QHI_STAGE), row, tl, half ? C::C_DOHI : C::C_QHI);
            if (SPLIT && C::LO_TMEM)
                row_to_tmem<DD>(sg + (half ? C::OFF_DOLO_STAGE : C::OFF_QLO_STAGE), row, tl, half ? C::C_DOLO : C::C_QLO);
            tmem_wait_st();
            fence_proxy_async_smem();
            tc_fence_before();
            mbar_arrive(bar(C::QD_READY));
        }
        const int64_t ridx = (b * p.H + h) * p.L + q;
        const float lse2 = row_ok ? a.lse2[ridx] : 0.0f;
        const float del = row_ok ? a.g.delta[ridx] : 0.0f;
        float pv[CPT];      // P of the block in flight, this thread's columns
        uint32_t zcur = 0;  // its dropout keep bits
        // Reads S_j, releases its columns, and leaves P_j in pv.
        auto load_p = [&](int j) -> bool {
            const int64_t base = (int64_t)j * NB + cb;
            // Column c is key base + c: valid below S and, under causal masking, up to q.
            const bool edge = MASKED || !row_ok || (int64_t)(j + 1) * NB > p.S || (p.causal && (int64_t)(j + 1) * NB - 1 > q0);
            uint32_t vbits = 0xFFFFFFFFu;
            if (edge) vbits = row_ok ? col_bits32(0, (p.causal ? min(p.S, q + 1) : p.S) - base) : 0u;
            // The user mask along this query's row, loaded before the wait for S.
            float mk[MASKED ? CPT : 1];
            if constexpr (MASKED) mask_run<CPT>(p, b, h, q, base, p.ms[3], vbits, mk);
            if constexpr (DROP) zcur = row_ok ? keep_run32(p, b, h, q, base) : 0u;
            if (!warp_wait(bar(C::S_FULL), j & 1, abort, err)) return false;
            tc_fence_after();
            uint32_t sr[CPT];
#pragma unroll
            for (int r0 = 0; r0 < CPT; r0 += 16) tmem_ld16(tl + C::C_S + cb + r0, *reinterpret_cast<uint32_t(*)[16]>(&sr[r0]));
            tmem_wait_ld();
            tc_fence_before();
            mbar_arrive(bar(C::S_READ));
#pragma unroll
            for (int c = 0; c < CPT; c++) {
                float x;
                if (MASKED) x = fmaf(mk[MASKED ? c : 0], LOG2E, __uint_as_float(sr[c]) * a.scale_log2) - lse2;
                else x = fmaf(__uint_as_float(sr[c]), a.scale_log2, -lse2);
                pv[c] = ((vbits >> c) & 1u) ? ex2_approx(x) : 0.0f;
            }
            return true;
        };
        if (ok && nblk > 0) ok = load_p(0);
        for (int j = 0; ok && j < nblk; j++) {
            if (!warp_wait(bar(C::DP_FULL), j & 1, abort, err)) {
                ok = false;
                break;
            }
            tc_fence_after();
#pragma unroll
            for (int r0 = 0; r0 < CPT; r0 += 16) {  // dS in 16-column pieces
                uint32_t dr[16], xh[16], xl[16];
                tmem_ld16(tl + C::C_DP + cb + r0, dr);
                tmem_wait_ld();
#pragma unroll
                for (int c = 0; c < 16; c++) {
                    // dS = P (Z dP - delta), Z = keep_scale where kept, 0 where dropped.
                    float dpv = __uint_as_float(dr[c]);
                    if constexpr (DROP) dpv = ((zcur >> (r0 + c)) & 1u) ? dpv * p.keep_scale : 0.0f;
                    const float ds = pv[r0 + c] * (dpv - del);
                    if (SPLIT) {
                        xh[c] = __float_as_uint(ds);
                        xl[c] = tf32_lo_trunc(ds);
                    } else {
                        xh[c] = tf32_rna(ds);
                    }
                }
                tmem_st16(tl + C::C_DP + cb + r0, xh);
                if (SPLIT) tmem_st16(tl + C::C_DSLO + cb + r0, xl);
            }
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(bar(C::DS_READY));
            // P of the next block while the tensor core runs dQ_j.
            if (j + 1 < nblk && !load_p(j + 1)) {
                ok = false;
                break;
            }
            if (!warp_wait(bar(C::DQ_DONE), j & 1, abort, err)) {
                ok = false;
                break;
            }
            tc_fence_after();
            fold16(tl + C::C_DQB + 32 * half, acc);
            fold16(tl + C::C_DQB + 32 * half + 16, acc + 16);
            tc_fence_before();
            mbar_arrive(bar(C::DQ_FREE));
        }
        const bool aborted = __any_sync(FULL, *abort != 0);
        if (ok && !aborted && row_ok) {
            float *dqr = a.g.dq + b * a.g.dqs[0] + h * a.g.dqs[1] + q * a.g.dqs[2] +
                         (int64_t)(64 * dh + 32 * half) * a.g.dqs[3];
            store_row<32>(dqr, a.g.dqs[3], acc, p.scale);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == W_MMA) {
        tc_fence_after();
        tmem_dealloc(tmem, C::TCOLS);
    }
}

bool rows_vec(const void *ptr, const int64_t *st) {
    return st[3] == 1 && st[0] % 4 == 0 && st[1] % 4 == 0 && st[2] % 4 == 0 &&
           (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0;
}

struct PoolScratch {
    void *ptr = nullptr;
    cudaStream_t stream = nullptr;
    ~PoolScratch() { pool_free(ptr, stream); }
};

// The dQ kernel does not depend on the dK / dV kernel: it runs on a side stream of the
// library's that belongs to the caller's stream (streams.cu), forked from the caller's stream
// after the pre-pass and joined back before the call returns -- on error paths too -- so that
// the two kernels share the GPU (the CTAs of one fill the SMs that the other's last, shorter
// tiles leave idle). The fork and join events are created per call.
constexpr int kSideRoleDq = 0;

}  // namespace

bool tc_backward_supported(const AttnProblem &p, const AttnGrads &g) {
    (void)g;
    if (p.E != p.Ev || (p.E != 64 && p.E != 128)) return false;
    if (p.L >= (1ll << 31) - TILE || p.S >= (1ll << 31) - TILE) return false;
    // 1-D grids of tiles x heads x batch (x column halves at head dim 128).
    const int64_t tiles = (max(p.L, p.S) + TILE - 1) / TILE;
    return 2 * p.B < (1ll << 31) && tiles * p.H * p.B * (p.E / 64) < (1ll << 31);
}

namespace {

// The instantiation of a backward kernel for (split, masked, dropout).
template <class F>
F pick_kernel(bool split, bool masked, bool drop, F ttt, F ttf, F tft, F tff, F ftt, F ftf, F fft, F fff) {
    if (split) return masked ? (drop ? ttt : ttf) : (drop ? tft : tff);
    return masked ? (drop ? ftt : ftf) : (drop ? fft : fff);
}

// Whether the tensor-core kernels can read a (B, heads, rows, DD) input's rows themselves
// through a TMA map: unit inner stride, 16-byte multiples for the other strides, 16-byte base.
bool tma_readable(const float *ptr, int64_t B, int64_t heads, int64_t rows, const int64_t *st) {
    return st[3] == 1 && tma_stride_ok(rows, st[2]) && tma_stride_ok(heads, st[1]) && tma_stride_ok(B, st[0]) &&
           (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0;
}

// The hi and lo TMA maps of one operand. Copy mode: hi and lo in the pre-pass's contiguous
// scratch (lo after hi). Raw mode: hi is the input itself (strides `ust`), lo the pre-pass's
// lo-only scratch.
struct HiLoMaps {
    CUtensorMap hi, lo;
};
int make_hilo(HiLoMaps &m, bool raw, const float *input, const int64_t *ust, const float *scratch, int64_t DD,
              int64_t rows, int64_t heads, int64_t B, int box, CUtensorMapSwizzle sw) {
    const int64_t cst[3] = {heads * rows * DD, rows * DD, DD};
    int st = raw ? make_tmap(&m.hi, input, DD, rows, heads, B, ust, box, sw)
                 : make_tmap(&m.hi, scratch, DD, rows, heads, B, cst, box, sw);
    if (st) return st;
    const float *lo = raw ? scratch : scratch + B * heads * rows * DD;
    return make_tmap(&m.lo, lo, DD, rows, heads, B, cst, box, sw);
}

template <int DD>
int tc_backward_dd(const AttnProblem &p, const AttnGrads &g, int precision, cudaStream_t stream) {
    using KC = KvCfg<DD>;
    using QC = QqCfg<DD>;
    const bool split = precision != DC_PREC_TF32;
    const int64_t rows_a = p.B * p.H * p.L, rows_b = p.B * p.Hkv * p.S;
    // Raw mode (3xTF32 with TMA-readable q, k, v and grad_out): the kernels read the hi
    // operands from the inputs and the pre-pass writes only the lo parts (half the scratch
    // and the pre-pass's writes). Otherwise the pre-pass copies hi (rounded) and lo.
    const bool raw = split && tma_readable(p.q, p.B, p.H, p.L, p.qs) && tma_readable(p.k, p.B, p.Hkv, p.S, p.ks) &&
                     tma_readable(p.v, p.B, p.Hkv, p.S, p.vs) && tma_readable(g.dout, p.B, p.H, p.L, g.dos);
    const int64_t NC = raw ? 1 : (split ? 2 : 1);  // copies per operand in the scratch
    const size_t bytes = sizeof(float) * (size_t)(NC * 2 * (rows_a + rows_b) * DD + rows_a);
    PoolScratch ws;
    ws.stream = stream;
    int st = pool_alloc(&ws.ptr, bytes, stream);
    if (st) return st;
    PrepArgs pa;
    pa.p = p;
    pa.g = g;
    pa.qhl = static_cast<float *>(ws.ptr);
    pa.dohl = pa.qhl + NC * rows_a * DD;
    pa.khl = pa.dohl + NC * rows_a * DD;
    pa.vhl = pa.khl + NC * rows_b * DD;
    pa.lse2 = pa.vhl + NC * rows_b * DD;
    pa.split = split ? 1 : 0;
    pa.lo_only = raw ? 1 : 0;
    pa.rows32 = rows_a + rows_b < (1ll << 31) ? 1 : 0;
    pa.vec = rows_vec(p.q, p.qs) && rows_vec(p.k, p.ks) && rows_vec(p.v, p.vs) && rows_vec(g.dout, g.dos) &&
             rows_vec(p.out, p.os);
    if (rows_a + rows_b > 0) {
        constexpr int rpb = 256 / (DD / 4);  // rows per block
        KernelTrace tr("bwd_prep", stream);
        bwd_prep_kernel<DD><<<(unsigned)((rows_a + rows_b + rpb - 1) / rpb), 256, 0, stream>>>(pa);
        if ((st = check_launch("bwd_prep"))) return st;
    }

    TcBwdArgs a;
    a.p = p;
    a.g = g;
    a.lse2 = pa.lse2;
    a.scale_log2 = p.scale * LOG2E;
    a.err = device_error_word();
    if (!a.err) return fail(DC_ERR_CUDA, "device error word is unavailable");
    const bool masked = p.mask_kind != MASK_NONE;
    const bool drop = p.keep != nullptr;
    constexpr CUtensorMapSwizzle KM = CU_TENSOR_MAP_SWIZZLE_128B, MN = CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B;
    auto q_maps = [&](HiLoMaps &m, int box, CUtensorMapSwizzle sw) {
        return make_hilo(m, raw, p.q, p.qs, pa.qhl, DD, p.L, p.H, p.B, box, sw);
    };
    auto do_maps = [&](HiLoMaps &m, int box, CUtensorMapSwizzle sw) {
        return make_hilo(m, raw, g.dout, g.dos, pa.dohl, DD, p.L, p.H, p.B, box, sw);
    };
    auto k_maps = [&](HiLoMaps &m, int box, CUtensorMapSwizzle sw) {
        return make_hilo(m, raw, p.k, p.ks, pa.khl, DD, p.S, p.Hkv, p.B, box, sw);
    };
    auto v_maps = [&](HiLoMaps &m, int box, CUtensorMapSwizzle sw) {
        return make_hilo(m, raw, p.v, p.vs, pa.vhl, DD, p.S, p.Hkv, p.B, box, sw);
    };
    // The two tensor-core kernels run concurrently; with tracing on, this record spans both
    // (from before the fork to after the join, on the caller's stream).
    KernelTrace pair("bwd_tc", stream);
    // Fork the dQ stream here, after the pre-pass and before the dK / dV launch.
    cudaStream_t side = nullptr;
    if (p.L > 0) {
        if ((st = side_stream(stream, kSideRoleDq, &side))) return st;
        if ((st = stream_edge(stream, side))) return st;
    }
    StreamJoin join(stream, side);  // joins side back into stream on every return below
    if (p.S > 0) {
        HiLoMaps tk, tv, tqk, tqmn, tdok, tdomn;
        st = k_maps(tk, TILE, KM);
        if (!st) st = v_maps(tv, TILE, KM);
        if (!st) st = q_maps(tqk, KC::QB, KM);
        if (!st) st = q_maps(tqmn, KC::QB, MN);
        if (!st) st = do_maps(tdok, KC::QB, KM);
        if (!st) st = do_maps(tdomn, KC::QB, MN);
        if (st) return st;
        auto kernel = pick_kernel(split, masked, drop, attn_bwd_dkdv_tc_kernel<DD, true, true, true>,
                                  attn_bwd_dkdv_tc_kernel<DD, true, true, false>,
                                  attn_bwd_dkdv_tc_kernel<DD, true, false, true>,
                                  attn_bwd_dkdv_tc_kernel<DD, true, false, false>,
                                  attn_bwd_dkdv_tc_kernel<DD, false, true, true>,
                                  attn_bwd_dkdv_tc_kernel<DD, false, true, false>,
                                  attn_bwd_dkdv_tc_kernel<DD, false, false, true>,
                                  attn_bwd_dkdv_tc_kernel<DD, false, false, false>);
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)KC::SMEM);
        if (e != cudaSuccess) return cuda_fail(e, "attn_bwd_dkdv_tc smem attribute");
        const unsigned grid = (unsigned)((p.S + TILE - 1) / TILE * p.Hkv * p.B * KC::NH);
        KernelTrace tr("bwd_dkdv_tc", stream);
        // Short rows (at most 512 queries): the CTAs are short and start-up bound, so the dK / dV
        // CTAs become resident while the pre-pass drains (a programmatic dependent launch).
        // Longer rows launch normally: there dK / dV taking every SM first delays the dQ kernel,
        // the pair's longer part.
        if (p.L <= 512) {
            e = launch_dependent(kernel, dim3(grid), dim3(THREADS), KC::SMEM, stream, tk.hi, tv.hi, tqk.hi, tqmn.hi,
                                 tdok.hi, tdomn.hi, tk.lo, tv.lo, tqk.lo, tqmn.lo, tdok.lo, tdomn.lo, a);
            if (e != cudaSuccess) return cuda_fail(e, "attn_bwd_dkdv_tc");
        } else {
            kernel<<<grid, THREADS, KC::SMEM, stream>>>(tk.hi, tv.hi, tqk.hi, tqmn.hi, tdok.hi, tdomn.hi, tk.lo, tv.lo,
                                                         tqk.lo, tqmn.lo, tdok.lo, tdomn.lo, a);
            if ((st = check_launch("attn_bwd_dkdv_tc"))) return st;
        }
    }
    if (p.L > 0) {
        HiLoMaps tq, tdo, tkk, tkmn, tvk;
        st = q_maps(tq, TILE, KM);
        if (!st) st = do_maps(tdo, TILE, KM);
        if (!st) st = k_maps(tkk, QC::NB, KM);
        if (!st) st = k_maps(tkmn, QC::NB, MN);
        if (!st) st = v_maps(tvk, QC::NB, KM);
        if (st) return st;
        auto kernel = pick_kernel(split, masked, drop, attn_bwd_dq_tc_kernel<DD, true, true, true>,
                                  attn_bwd_dq_tc_kernel<DD, true, true, false>,
                                  attn_bwd_dq_tc_kernel<DD, true, false, true>,
                                  attn_bwd_dq_tc_kernel<DD, true, false, false>,
                                  attn_bwd_dq_tc_kernel<DD, false, true, true>,
                                  attn_bwd_dq_tc_kernel<DD, false, true, false>,
                                  attn_bwd_dq_tc_kernel<DD, false, false, true>,
                                  attn_bwd_dq_tc_kernel<DD, false, false, false>);
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)QC::SMEM);
        if (e != cudaSuccess) return cuda_fail(e, "attn_bwd_dq_tc smem attribute");
        const unsigned grid = (unsigned)((p.L + TILE - 1) / TILE * p.H * p.B * QC::NH);
        {
            KernelTrace tr("bwd_dq_tc", side);
            kernel<<<grid, THREADS, QC::SMEM, side>>>(tq.hi, tdo.hi, tkk.hi, tkmn.hi, tvk.hi, tq.lo, tdo.lo, tkk.lo,
                                                      tkmn.lo, tvk.lo, a);
        }
        const int launched = check_launch("attn_bwd_dq_tc");
        if ((st = join.join())) return st;
        if (launched) return launched;
    }
    return DC_OK;
}

}  // namespace

int tc_backward(const AttnProblem &p, const AttnGrads &g, int precision, cudaStream_t stream) {
    return p.E == 64 ? tc_backward_dd<64>(p, g, precision, stream) : tc_backward_dd<128>(p, g, precision, stream);
}

}  // namespace dc
