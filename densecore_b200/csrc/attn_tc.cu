// attn_tc.cu -- tcgen05 tensor-core attention forward for sm_100a.
//
// Replaces DenseCore's torch_attention::forward (src/torch_attention.rs:146-284) for head dim
// 64 and 128 with a warp-specialised kernel; one CTA computes a 128-row query tile of one
// (batch, head):
//
//   warp 8      TMA producer: the Q tile once (staged in the V ring, so that the K ring fills
//               while the converters move Q into TMEM), then K and V tiles of BN keys into 3-stage
//               shared-memory rings (4-D tensor maps over the caller's strided (B, H, L, E)
//               views, zero fill past the sequence end). K uses the 128-byte swizzle (K-major
//               B operand); V uses the 32-byte-atom 128-byte swizzle, the only layout tf32
//               accepts for an MN-major operand.
//   warps 10-13 converters: Q goes into TMEM as tf32 hi / lo (the A operand of S = Q K^T, so
//               the S MMAs read only K from shared memory); each landed K / V tile x stays as
//               the hi operand (the tensor core reads x truncated to TF32) and its lo part
//               x - trunc(x) is written beside it (3xTF32: a*b ~ ah*bh + ah*bl + al*bh keeps
//               fp32-class accuracy on the TF32 tensor cores).
//   warps 9, 14 MMA issuers (whole warps, one elected lane issuing; descriptors precomputed): warp 9 issues
//               S_j = Q K_j^T into one of two TMEM buffers, warp 14 O_blk = P_j V_j with P read
//               from TMEM. With two issuers one warp's barrier waits overlap the other's
//               MMAs, and S_{j+1} runs on the tensor core while the softmax warps work on
//               block j.
//   warps 0-7   softmax, two threads per query row (TMEM lane), each owning half of the
//               block's columns and half of the output row (in registers). Online softmax in
//               base 2 with DenseCore's rules: a block whose running max is -inf adds nothing
//               (:218-226); the row max is shared between the pair through shared memory;
//               the running max moves only when it grows by more than 2^8 (sum and output
//               share the stale max, so the result is unchanged). P goes back to TMEM as tf32
//               hi / lo over the consumed S columns. Each block's P V lands in a fresh TMEM
//               accumulator (a few tensor-core accumulation steps, whose internal rounding is
//               coarser than fp32) that the pair folds into its registers in fp32. Finalisation
//               as the reference: max -inf -> 0, sum 0 -> 1, out = acc/sum, lse = max +
//               log(sum) (:258-271).
//
// Every mbarrier wait is bounded (sm100::mbar_wait); a wait that times out sets the device
// error word and the CTA unwinds, frees its TMEM and exits.
#include <cuda.h>
#include <cuda_runtime.h>
#include <math.h>

#include "common.cuh"
#include "kernels.h"
#include "sm100.cuh"
#include "tma_host.h"
#include "trace.h"

namespace dc {

__device__ int g_tc_error = 0;

namespace {

using namespace sm100;

constexpr float LOG2E = 1.4426950408889634f;
constexpr float LN2 = 0.6931471805599453f;

template <int D_, int BN_, int KST_, int VST_>
struct FwdCfg {
    static constexpr int D = D_, BN = BN_, KST = KST_, VST = VST_;
    static constexpr int BM = 128;
    static constexpr int CHUNKS = D / 32;   // 128-byte column chunks of a row
    static constexpr int HB = BN / 2;       // S columns per softmax thread
    static constexpr int HD = D / 2;        // output columns per softmax thread
    static constexpr uint32_t Q_CHUNK = BM * 128;
    static constexpr uint32_t KV_CHUNK = BN * 128;
    static constexpr uint32_t Q_BYTES = BM * D * 4;
    static constexpr uint32_t KV_BYTES = BN * D * 4;
    static constexpr uint32_t KV_STAGE = 2 * KV_BYTES;  // hi, lo
    static constexpr uint32_t OFF_K = 0;
    static constexpr uint32_t OFF_V = OFF_K + KST * KV_STAGE;
    static constexpr uint32_t OFF_XMAX = OFF_V + VST * KV_STAGE;     // float [2][2][BM]
    static constexpr uint32_t OFF_XSUM = OFF_XMAX + 2 * 2 * BM * 4;  // float [2][BM]
    static constexpr uint32_t OFF_BAR = OFF_XSUM + 2 * BM * 4;
    static constexpr int Q_FULL = 0, Q_READY = 1, K_FULL = 2, K_READY = K_FULL + KST,
                         K_EMPTY = K_READY + KST, V_FULL = K_EMPTY + KST, V_READY = V_FULL + VST,
                         V_EMPTY = V_READY + VST, S_FULL = V_EMPTY + VST, P_FULL = S_FULL + 2,
                         PV_DONE_B = P_FULL + 2, OB_FREE = PV_DONE_B + 2,
                         XCH = OB_FREE + 2, XSUM = XCH + 2, DRAIN = XSUM + 1, DRAIN_PV = DRAIN + 1,
                         NBAR = DRAIN_PV + 1;
    static constexpr uint32_t OFF_MISC = OFF_BAR + NBAR * 8;
    static constexpr uint32_t SMEM = OFF_MISC + 16 + 1024;  // + slack for 1024-byte alignment
    // TMEM: Q hi | Q lo | 2 x (S / P hi, P lo) | NOB x O_blk. Two O_blk buffers where they fit
    // (D = 64), so that P_{j+1} V_{j+1} need not wait for the fold of block j.
    static constexpr int NOB = (4 * D + 4 * BN <= 512) ? 2 : 1;
    static constexpr uint32_t COL_QHI = 0, COL_QLO = D, COL_OB = 2 * D + 4 * BN;
    static constexpr uint32_t COLS_USED = (2 + NOB) * D + 4 * BN;
    __host__ __device__ static constexpr uint32_t col_ob(int i) { return COL_OB + (uint32_t)((i % NOB) * D); }
    static constexpr uint32_t TMEM_COLS = COLS_USED <= 256 ? 256 : 512;
    static constexpr int SOFTMAX_THREADS = 256;
    static constexpr int W_PROD = 8, W_MMA = 9, W_CVT = 10, W_PV = 14;
    static constexpr int THREADS = 480;  // <= 4 warps per SM sub-partition: 128 registers
    static constexpr uint32_t IDESC_S = idesc_tf32(128, BN, 0, 0);
    static constexpr uint32_t IDESC_O = idesc_tf32(128, D, 0, 1);
    __host__ __device__ static constexpr uint32_t col_s(int b) { return 2 * D + b * 2 * BN; }
    __host__ __device__ static constexpr uint32_t col_plo(int b) { return 2 * D + b * 2 * BN + BN; }
    static_assert(SMEM <= 232448, "shared memory budget");
    static_assert(COLS_USED <= 512, "tensor memory budget");
    // The raw Q tile takes QS consecutive items of the V ring (Q_CHUNKS_PER_SLOT 128-byte
    // column chunks each).
    static constexpr int QS = (int)(Q_BYTES / KV_STAGE), Q_CHUNKS_PER_SLOT = (int)(KV_STAGE / Q_CHUNK);
    static_assert(QS * KV_STAGE == Q_BYTES && Q_CHUNKS_PER_SLOT * Q_CHUNK == KV_STAGE && QS < VST,
                  "the raw Q tile is staged in whole V-ring slots");
    static_assert(HB == 16 || HB == 32, "softmax half-block width");
};

struct TcFwdArgs {
    AttnProblem p;
    int num_q_tiles;
    int64_t num_tiles;    // num_q_tiles * H * B
    int64_t group_heads;  // (batch, head) pairs whose tiles are ordered together (their K / V fit in L2)
    float scale_log2;
    int *err;
};

// tcgen05.ld / st of 16 or 32 consecutive columns of this thread's lane.
template <int N>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, uint32_t (&r)[N]) {
    if constexpr (N == 32) tmem_ld32(taddr, r);
    else tmem_ld16(taddr, r);
}
template <int N>
__device__ __forceinline__ void tmem_st(uint32_t taddr, const uint32_t (&r)[N]) {
    if constexpr (N == 32) tmem_st32(taddr, r);
    else tmem_st16(taddr, r);
}

// 3xTF32 (SPLIT): the landed tile x stays in place as the hi operand (the tensor core reads
// x truncated to TF32) and lo = x - trunc(x), exact, goes `lo_off` bytes further. Single-pass
// TF32 rounds x to nearest in place instead of letting the tensor core drop the low mantissa
// bits (which would bias every operand toward zero).
template <bool SPLIT>
__device__ __forceinline__ void split_tile(uint8_t *hi, uint32_t lo_off, uint32_t bytes, int t) {
    for (uint32_t i = t; i < bytes / 16; i += 128) {
        float4 *ph = reinterpret_cast<float4 *>(hi) + i;
        const float4 x = *ph;
        if (SPLIT) {
            *(reinterpret_cast<uint4 *>(hi + lo_off) + i) =
                make_uint4(tf32_lo_trunc(x.x), tf32_lo_trunc(x.y), tf32_lo_trunc(x.z), tf32_lo_trunc(x.w));
        } else {
            float4 hv;
            hv.x = __uint_as_float(tf32_rna(x.x));
            hv.y = __uint_as_float(tf32_rna(x.y));
            hv.z = __uint_as_float(tf32_rna(x.z));
            hv.w = __uint_as_float(tf32_rna(x.w));
            *ph = hv;
        }
    }
}

// max over N values as a balanced tree (a dependency chain of log2 N instead of N).
template <int N>
__device__ __forceinline__ float max_tree(const float (&v)[N]) {
    float t[N / 2];
#pragma unroll
    for (int i = 0; i < N / 2; i++) t[i] = fmaxf(v[2 * i], v[2 * i + 1]);
#pragma unroll
    for (int w = N / 4; w >= 1; w /= 2)
#pragma unroll
        for (int i = 0; i < w; i++) t[i] = fmaxf(t[2 * i], t[2 * i + 1]);
    return t[0];
}

// Row `row` of a raw 128-byte-swizzled tile (rows of 128-byte chunks, chunk stride
// `chunk_bytes`) into TMEM: with SPLIT the raw values as hi at col_hi and the exact remainder of
// their TF32 truncation as lo at col_lo; without, the rounded TF32 values at col_hi.
template <int CHUNKS, bool SPLIT>
__device__ __forceinline__ void row_to_tmem(const uint8_t *raw, uint32_t chunk_bytes, int row, uint32_t tlane,
                                            uint32_t col_hi, uint32_t col_lo) {
#pragma unroll
    for (int c = 0; c < CHUNKS; c++) {
        uint32_t hi[32], lo[32];
#pragma unroll
        for (int g = 0; g < 8; g++) {
            const float4 x =
                *reinterpret_cast<const float4 *>(raw + c * chunk_bytes + row * 128 + ((g ^ (row & 7)) * 16));
            const float v[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
            for (int e = 0; e < 4; e++) {
                if (SPLIT) {
                    hi[4 * g + e] = __float_as_uint(v[e]);
                    lo[4 * g + e] = tf32_lo_trunc(v[e]);
                } else {
                    hi[4 * g + e] = tf32_rna(v[e]);
                }
            }
        }
        tmem_st32(tlane + col_hi + 32 * c, hi);
        if (SPLIT) tmem_st32(tlane + col_lo + 32 * c, lo);
    }
}

// One CTA per tile (long tiles: config 4). Grid (q-tiles, H, B), longest causal tiles first
// within a head, so that the tiles the hardware runs together share their head's K / V in L2.
// The same roles and pipelines as the persistent kernel below for a single tile: the raw Q tile
// waits in the V ring while the K ring fills, and the first V load waits until Q has left.
template <class C, bool SPLIT, bool MASKED, bool DROP>
__global__ void __maxnreg__(128)
    attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                       const __grid_constant__ CUtensorMap tmv, const TcFwdArgs a) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_addr(smem_raw);
    const uint32_t sb = (raw + 1023u) & ~1023u;
    uint8_t *sg = smem_raw + (sb - raw);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const AttnProblem &p = a.p;
    const int qt = a.num_q_tiles - 1 - (int)blockIdx.x;  // longest (causal) tiles first
    const int64_t h = blockIdx.y, b = blockIdx.z, hk = h / p.group;
    const int64_t q0 = (int64_t)qt * C::BM;
    const int64_t kv_end = p.causal ? min(p.S, q0 + C::BM) : p.S;
    const int nblk = (int)((kv_end + C::BN - 1) / C::BN);
    auto bar = [&](int i) { return sb + C::OFF_BAR + 8u * (uint32_t)i; };
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(sg + C::OFF_MISC);
    volatile int *abort = reinterpret_cast<volatile int *>(sg + C::OFF_MISC + 4);
    int *err = a.err;

    if (threadIdx.x == 0) {
        mbar_init(bar(C::Q_FULL), 1);
        mbar_init(bar(C::Q_READY), 128);
        for (int s = 0; s < C::KST; s++) {
            mbar_init(bar(C::K_FULL + s), 1);
            mbar_init(bar(C::K_READY + s), 128);
            mbar_init(bar(C::K_EMPTY + s), 1);
        }
        for (int s = 0; s < C::VST; s++) {
            mbar_init(bar(C::V_FULL + s), 1);
            mbar_init(bar(C::V_READY + s), 128);
            mbar_init(bar(C::V_EMPTY + s), 1);
        }
        for (int s = 0; s < 2; s++) {
            mbar_init(bar(C::S_FULL + s), 1);
            mbar_init(bar(C::P_FULL + s), C::SOFTMAX_THREADS);
        }
        mbar_init(bar(C::PV_DONE_B), 1);
        mbar_init(bar(C::PV_DONE_B + 1), 1);
        mbar_init(bar(C::OB_FREE), C::SOFTMAX_THREADS);
        mbar_init(bar(C::OB_FREE + 1), C::SOFTMAX_THREADS);
        mbar_init(bar(C::XCH), C::SOFTMAX_THREADS);
        mbar_init(bar(C::XCH + 1), C::SOFTMAX_THREADS);
        mbar_init(bar(C::XSUM), C::SOFTMAX_THREADS);
        mbar_init(bar(C::DRAIN), 1);
        mbar_init(bar(C::DRAIN_PV), 1);
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == C::W_MMA) {
        tmem_alloc(smem_addr(tmem_slot), C::TMEM_COLS);
        tmem_relinquish();
    }
    if (warp == C::W_PROD && lane == 0) {
        prefetch_tmap(&tmq);
        prefetch_tmap(&tmk);
        prefetch_tmap(&tmv);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == C::W_PROD) {
        // ------------------------------------------------------------ TMA producer ----
        if (lane == 0) {
            int k_issued = -1, v_issued = -1;
            // The raw Q tile lands in the V ring and the converters move it into TMEM; the K
            // ring fills meanwhile (S_0 needs Q and K_0), and the first V load waits until Q has
            // left the V ring.
            mbar_expect_tx(bar(C::Q_FULL), C::Q_BYTES);
            for (int c = 0; c < C::CHUNKS; c++)
                tma_load_4d(&tmq, sb + C::OFF_V + c * C::Q_CHUNK, bar(C::Q_FULL), 32 * c, (int)q0, (int)h, (int)b);
            bool ok = true;
            for (int j = 0; ok && j < nblk; j++) {
                const int ks = j % C::KST, vs = j % C::VST;
                if (j >= C::KST && !mbar_wait(bar(C::K_EMPTY + ks), ((j / C::KST) - 1) & 1, abort, err)) break;
                mbar_expect_tx(bar(C::K_FULL + ks), C::KV_BYTES);
                const uint32_t kd = sb + C::OFF_K + ks * C::KV_STAGE;
                for (int c = 0; c < C::CHUNKS; c++)
                    tma_load_4d(&tmk, kd + c * C::KV_CHUNK, bar(C::K_FULL + ks), 32 * c, j * C::BN, (int)hk, (int)b);
                k_issued = j;
                if (j == 0 && !(ok = mbar_wait(bar(C::Q_READY), 0, abort, err))) break;
                if (j >= C::VST && !mbar_wait(bar(C::V_EMPTY + vs), ((j / C::VST) - 1) & 1, abort, err)) break;
                mbar_expect_tx(bar(C::V_FULL + vs), C::KV_BYTES);
                const uint32_t vd = sb + C::OFF_V + vs * C::KV_STAGE;
                for (int c = 0; c < C::CHUNKS; c++)
                    tma_load_4d(&tmv, vd + c * C::KV_CHUNK, bar(C::V_FULL + vs), 32 * c, j * C::BN, (int)hk, (int)b);
                v_issued = j;
            }
            if (*abort) {
                // Let the copies already in flight land before the CTA's memory goes away.
                volatile int never = 0;
                mbar_wait(bar(C::Q_FULL), 0, &never, nullptr);
                for (int j = max(0, k_issued - C::KST + 1); j <= k_issued; j++)
                    mbar_wait(bar(C::K_FULL + j % C::KST), (j / C::KST) & 1, &never, nullptr);
                for (int j = max(0, v_issued - C::VST + 1); j <= v_issued; j++)
                    mbar_wait(bar(C::V_FULL + j % C::VST), (j / C::VST) & 1, &never, nullptr);
            }
        }
    } else if (warp == C::W_MMA) {
        // -------------------------------------------------------- MMA issuer: S = Q K^T ----
        // The whole warp runs the loop converged; one elected lane issues each MMA.
        {
            // Descriptor of K stage 0; stage and k-step offsets go into the address field.
            const uint64_t kdesc0 = sdesc_sw128(sb + C::OFF_K, 16, 1024);
            const uint32_t q_hi = tmem + C::COL_QHI, q_lo = tmem + C::COL_QLO;
            bool ok = mbar_wait_warp(bar(C::Q_READY), 0, abort, err);
            tc_fence_after();
            for (int j = 0; ok && j < nblk; j++) {
                const int bb = j & 1, ks = j % C::KST;
                // S buffer bb held P_{j-2}, read by PV_{j-2}.
                if (j >= 2 && !mbar_wait_warp(bar(C::PV_DONE_B + bb), ((j - 2) >> 1) & 1, abort, err)) break;
                if (!mbar_wait_warp(bar(C::K_READY + ks), (j / C::KST) & 1, abort, err)) break;
                tc_fence_after();
                const uint64_t kd = kdesc0 + ((ks * C::KV_STAGE) >> 4);
                const uint32_t d_s = tmem + C::col_s(bb);
                if (SPLIT) {  // Qhi Klo + Qlo Khi first, then Qhi Khi
#pragma unroll
                    for (int kk = 0; kk < C::D / 8; kk++) {
                        const uint32_t off = ((kk >> 2) * C::KV_CHUNK + (kk & 3) * 32) >> 4;
                        mma_tf32_ts_w(d_s, q_hi + kk * 8, kd + ((C::KV_BYTES >> 4) + off), C::IDESC_S, kk > 0 ? 1u : 0u);
                        mma_tf32_ts_w(d_s, q_lo + kk * 8, kd + off, C::IDESC_S, 1u);
                    }
                }
#pragma unroll
                for (int kk = 0; kk < C::D / 8; kk++) {
                    const uint32_t off = ((kk >> 2) * C::KV_CHUNK + (kk & 3) * 32) >> 4;
                    mma_tf32_ts_w(d_s, q_hi + kk * 8, kd + off, C::IDESC_S, (SPLIT || kk > 0) ? 1u : 0u);
                }
                tc_commit_w(bar(C::S_FULL + bb));
                tc_commit_w(bar(C::K_EMPTY + ks));
            }
            // Every MMA this warp issued completes before TMEM is released.
            tc_commit_w(bar(C::DRAIN));
            volatile int never = 0;
            mbar_wait_warp(bar(C::DRAIN), 0, &never, nullptr);
        }
    } else if (warp == C::W_PV) {
        // ----------------------------------------------------- MMA issuer: O_blk = P V ----
        {
            const uint64_t vdesc0 = sdesc_mn_sw128_32b(sb + C::OFF_V, C::KV_CHUNK, 512);
            for (int i = 0; i < nblk; i++) {
                const int bi = i & 1, vs = i % C::VST;
                if (!mbar_wait_warp(bar(C::P_FULL + bi), (i >> 1) & 1, abort, err)) break;
                if (!mbar_wait_warp(bar(C::V_READY + vs), (i / C::VST) & 1, abort, err)) break;
                // O_blk buffer i % NOB held block i - NOB until the softmax threads folded it.
                if (i >= C::NOB && !mbar_wait_warp(bar(C::OB_FREE + i % C::NOB), ((i / C::NOB) - 1) & 1, abort, err))
                    break;
                const uint32_t d_ob = tmem + C::col_ob(i);
                tc_fence_after();
                const uint64_t vd = vdesc0 + ((vs * C::KV_STAGE) >> 4);
                const uint32_t a_hi = tmem + C::col_s(bi), a_lo = tmem + C::col_plo(bi);
                if (SPLIT) {  // the small cross terms first, then the main products
#pragma unroll
                    for (int kk = 0; kk < C::BN / 8; kk++) {
                        mma_tf32_ts_w(d_ob, a_hi + kk * 8, vd + ((C::KV_BYTES + kk * 1024) >> 4), C::IDESC_O,
                                      kk > 0 ? 1u : 0u);
                        mma_tf32_ts_w(d_ob, a_lo + kk * 8, vd + ((kk * 1024) >> 4), C::IDESC_O, 1u);
                    }
                }
#pragma unroll
                for (int kk = 0; kk < C::BN / 8; kk++)
                    mma_tf32_ts_w(d_ob, a_hi + kk * 8, vd + ((kk * 1024) >> 4), C::IDESC_O, (SPLIT || kk > 0) ? 1u : 0u);
                tc_commit_w(bar(C::PV_DONE_B + bi));
                tc_commit_w(bar(C::V_EMPTY + vs));
            }
            tc_commit_w(bar(C::DRAIN_PV));
            volatile int never = 0;
            mbar_wait_warp(bar(C::DRAIN_PV), 0, &never, nullptr);
        }
    } else if (warp >= C::W_CVT && warp < C::W_PV) {
        // --------------------------------------------------------------- converters ----
        const int ct = threadIdx.x - 32 * C::W_CVT;
        const int quad = warp & 3;
        if (mbar_wait(bar(C::Q_FULL), 0, abort, err)) {
            row_to_tmem<C::CHUNKS, SPLIT>(sg + C::OFF_V, C::Q_CHUNK, quad * 32 + lane,
                                          tmem + ((uint32_t)(quad * 32) << 16), C::COL_QHI, C::COL_QLO);
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(bar(C::Q_READY));
            for (int j = 0; j < nblk; j++) {
                const int ks = j % C::KST, vs = j % C::VST;
                if (!mbar_wait(bar(C::K_FULL + ks), (j / C::KST) & 1, abort, err)) break;
                split_tile<SPLIT>(sg + C::OFF_K + ks * C::KV_STAGE, C::KV_BYTES, C::KV_BYTES, ct);
                fence_proxy_async_smem();
                mbar_arrive(bar(C::K_READY + ks));
                if (!mbar_wait(bar(C::V_FULL + vs), (j / C::VST) & 1, abort, err)) break;
                split_tile<SPLIT>(sg + C::OFF_V + vs * C::KV_STAGE, C::KV_BYTES, C::KV_BYTES, ct);
                fence_proxy_async_smem();
                mbar_arrive(bar(C::V_READY + vs));
            }
        }
    } else {
        // ------------------------------------------------------------------ softmax ----
        const int row = threadIdx.x & 127, half = threadIdx.x >> 7;
        const int64_t qrow = q0 + row;
        const bool row_ok = qrow < p.L;
        const uint32_t tl = tmem + ((uint32_t)((warp & 3) * 32) << 16);
        float *xmax = reinterpret_cast<float *>(sg + C::OFF_XMAX);  // [2][2][BM]
        float *xsum = reinterpret_cast<float *>(sg + C::OFF_XSUM);  // [2][BM]
        float m = -INFINITY, l = 0.0f;
        float o[C::HD];
#pragma unroll
        for (int x = 0; x < C::HD; x++) o[x] = 0.0f;
        bool ok = true;
        for (int j = 0; j < nblk; j++) {
            const int bb = j & 1;
            const int64_t k0 = (int64_t)j * C::BN + half * C::HB;
            // Rows past L (zero-filled by TMA) are computed but never stored. Column c is key
            // k0 + c: valid below S and, under causal masking, up to qrow (one bit per column
            // keeps the edge path as short as the fast one).
            const bool edge = MASKED || (k0 + C::HB > p.S) || (p.causal && k0 + C::HB - 1 > q0);
            uint32_t vbits = 0xFFFFFFFFu;
            if (edge) {
                const int64_t lim = (p.causal ? min(p.S, qrow + 1) : p.S) - k0;
                const int n = !row_ok || lim <= 0 ? 0 : (lim >= C::HB ? C::HB : (int)lim);
                vbits = n == 0 ? 0u : (0xFFFFFFFFu >> (32 - n));
            }
            // The user mask's values for these columns, loaded before the wait for S so that
            // the wait hides their latency.
            float mk[MASKED ? C::HB : 1];
            if constexpr (MASKED) mask_run<C::HB>(p, b, h, qrow, k0, p.ms[3], vbits, mk);
            // Dropout: this row's keep bits for these columns (the weights that meet V are
            // P * keep_scale where kept, 0 where dropped; the row sum and lse stay undropped).
            uint32_t kbits = 0;
            if constexpr (DROP) kbits = row_ok ? keep_run32(p, b, h, qrow, k0) : 0u;
            if (!mbar_wait(bar(C::S_FULL + bb), (j >> 1) & 1, abort, err)) {
                ok = false;
                break;
            }
            tc_fence_after();
            float s[C::HB];
            {
                uint32_t r[C::HB];
                tmem_ld<C::HB>(tl + C::col_s(bb) + half * C::HB, r);
                tmem_wait_ld();
#pragma unroll
                for (int x = 0; x < C::HB; x++) s[x] = __uint_as_float(r[x]);
            }
            // Interior blocks keep the raw scores and fold the scale into the exponent's FFMA
            // (the max commutes with a positive scale); edge blocks scale, mask and fill first.
            const bool raw = !edge && a.scale_log2 > 0.0f;
            const float smul = raw ? a.scale_log2 : 1.0f;
            if (!raw) {
#pragma unroll
                for (int c = 0; c < C::HB; c++) {
                    float x = s[c] * a.scale_log2;
                    if (MASKED) x += mk[MASKED ? c : 0] * LOG2E;
                    s[c] = ((vbits >> c) & 1u) ? x : -INFINITY;
                }
            }
            float bmax = max_tree<C::HB>(s) * smul;
            // The block's row max, shared with the partner thread (the other half) through
            // shared memory and an mbarrier (a bounded wait, unlike bar.sync).
            xmax[(bb * 2 + half) * C::BM + row] = bmax;
            mbar_arrive(bar(C::XCH + bb));
            if (!mbar_wait(bar(C::XCH + bb), (j >> 1) & 1, abort, err)) {
                ok = false;
                break;
            }
            bmax = fmaxf(bmax, xmax[(bb * 2 + (half ^ 1)) * C::BM + row]);
            const float m_new = fmaxf(m, bmax);
            const bool rescale = m_new > m + 8.0f;
            float corr = 1.0f;
            if (rescale) {
                corr = ex2_approx(m - m_new);
                m = m_new;
            }
            const bool dead = (m == -INFINITY);
            float part[4] = {0.0f, 0.0f, 0.0f, 0.0f};  // four partial row sums: shorter chains
#pragma unroll
            for (int r0 = 0; r0 < C::HB; r0 += 16) {  // P in 16-column pieces
                uint32_t phi[16], plo[16];
#pragma unroll
                for (int c = 0; c < 16; c++) {
                    const float pc = dead ? 0.0f : ex2_approx(fmaf(s[r0 + c], smul, -m));
                    part[c & 3] += pc;
                    float pw = pc;
                    if constexpr (DROP) pw = ((kbits >> (r0 + c)) & 1u) ? pc * p.keep_scale : 0.0f;
                    if (SPLIT) {
                        phi[c] = __float_as_uint(pw);
                        plo[c] = tf32_lo_trunc(pw);
                    } else {
                        phi[c] = tf32_rna(pw);
                    }
                }
                tmem_st16(tl + C::col_s(bb) + half * C::HB + r0, phi);
                if (SPLIT) tmem_st16(tl + C::col_plo(bb) + half * C::HB + r0, plo);
            }
            const float rs = (part[0] + part[1]) + (part[2] + part[3]);
            l = fmaf(l, corr, rs);
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(bar(C::P_FULL + bb));
            // Fold the previous block: o = (o + O_blk(j-1)) * corr (both relative to the
            // previous max; corr moves them to m).
            if (j >= 1) {
                // Per-buffer barrier: with two O_blk buffers PV_j may finish before this wait,
                // so a single barrier could be two phases ahead of it.
                if (!mbar_wait(bar(C::PV_DONE_B + ((j - 1) & 1)), ((j - 1) >> 1) & 1, abort, err)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const bool scaled = __any_sync(0xffffffffu, corr != 1.0f);
#pragma unroll
                for (int c = 0; c < C::HD / 16; c++) {
                    uint32_t r[16];
                    tmem_ld16(tl + C::col_ob(j - 1) + half * C::HD + 16 * c, r);
                    tmem_wait_ld();
                    if (scaled) {
#pragma unroll
                        for (int x = 0; x < 16; x++) o[16 * c + x] = (o[16 * c + x] + __uint_as_float(r[x])) * corr;
                    } else {
#pragma unroll
                        for (int x = 0; x < 16; x++) o[16 * c + x] += __uint_as_float(r[x]);
                    }
                }
                tc_fence_before();
                mbar_arrive(bar(C::OB_FREE + (j - 1) % C::NOB));
            }
        }
        if (ok && nblk > 0) {
            ok = mbar_wait(bar(C::PV_DONE_B + ((nblk - 1) & 1)), ((nblk - 1) >> 1) & 1, abort, err);
            tc_fence_after();
        }
        const bool read_o = __all_sync(0xffffffffu, ok) && nblk > 0;
        const bool aborted = __any_sync(0xffffffffu, *abort != 0);
        if (read_o) {
#pragma unroll
            for (int c = 0; c < C::HD / 32; c++) {
                uint32_t r[32];
                tmem_ld32(tl + C::col_ob(nblk - 1) + half * C::HD + 32 * c, r);
                tmem_wait_ld();
#pragma unroll
                for (int x = 0; x < 32; x++) o[32 * c + x] += __uint_as_float(r[x]);
            }
        }
        // The row sum: this half's part plus the partner's.
        xsum[half * C::BM + row] = l;
        mbar_arrive(bar(C::XSUM));
        const bool have_sum = mbar_wait(bar(C::XSUM), 0, abort, err);
        l += xsum[(half ^ 1) * C::BM + row];
        if (!aborted && have_sum && row_ok) {
            const float lfin = l == 0.0f ? 1.0f : l;
            const float mnat = m == -INFINITY ? 0.0f : m * LN2;
            const float inv = 1.0f / lfin;
            float *orow = p.out + b * p.os[0] + h * p.os[1] + qrow * p.os[2] + (int64_t)half * C::HD * p.os[3];
            if (p.os[3] == 1 && (reinterpret_cast<uintptr_t>(orow) & 15u) == 0) {
#pragma unroll
                for (int x = 0; x < C::HD; x += 4)
                    *reinterpret_cast<float4 *>(orow + x) =
                        make_float4(o[x] * inv, o[x + 1] * inv, o[x + 2] * inv, o[x + 3] * inv);
            } else {
#pragma unroll
                for (int x = 0; x < C::HD; x++) orow[x * p.os[3]] = o[x] * inv;
            }
            if (half == 0) p.lse[b * p.ls[0] + h * p.ls[1] + qrow * p.ls[2]] = mnat + logf(lfin);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == C::W_MMA) {
        tc_fence_after();
        tmem_dealloc(tmem, C::TMEM_COLS);
    }
}

// Tile t of the schedule: groups of group_heads (batch, head) pairs, and within a group the
// tiles with the most causal work first (q-tile major, pair minor). Tiles handed out together
// then share their heads' K / V in L2.
// The persistent kernel runs only when the tile count is below 2^31 (checked at launch), so
// the decode divides in 32 bits: the 64-bit divisions had sat on the softmax warps' path from
// one tile to the next.
__device__ __forceinline__ void fwd_tile(const TcFwdArgs &a, int64_t t, int64_t &q0, int64_t &h, int64_t &b) {
    const uint32_t nq = (uint32_t)a.num_q_tiles, g = (uint32_t)a.group_heads, hb = (uint32_t)(a.p.H * a.p.B),
                   H = (uint32_t)a.p.H, tt = (uint32_t)t;
    const uint32_t grp = tt / (g * nq), base = grp * g, gs = min(g, hb - base), r = tt - grp * g * nq;
    const uint32_t qt = nq - 1 - r / gs, bh = base + r % gs;
    h = bh % H;
    b = bh / H;
    q0 = (int64_t)qt * 128;
}

// Tile of round r of CTA c among G persistent CTAs: rounds alternate direction (a snake), which
// evens out the causal tiles' unequal lengths across CTAs. -1 when the tiles have run out.
__device__ __forceinline__ int64_t fwd_tile_of(int64_t r, int c, int G, int64_t T) {
    const int64_t t = r * G + ((r & 1) ? G - 1 - c : c);
    return t < T ? t : -1;
}

// Persistent (short tiles: configs 1-3): gridDim.x CTAs (at most one per SM) walk the tiles in
// fwd_tile_of order. Every
// role keeps running counters across tiles: K items (one per key block) in the K ring; V-ring
// items, which are each tile's Q (QS slots) followed by its V blocks, so that the barriers of a
// V-ring slot count Q and V uses alike; and blocks (the S / P buffers, the O blocks). The next
// tile's Q lands and its first K / V tiles load while the tensor core and the softmax warps
// still work on the current tile; the converters move Q into TMEM once the current tile's last
// S MMA has read the old Q, and the softmax warps' epilogue (last fold, normalisation, stores)
// overlaps the next tile's first S MMAs.
template <class C, bool SPLIT, bool MASKED, bool DROP>
__global__ void __maxnreg__(128)
    attn_fwd_tc_persist_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                       const __grid_constant__ CUtensorMap tmv, const TcFwdArgs a) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_addr(smem_raw);
    const uint32_t sb = (raw + 1023u) & ~1023u;
    uint8_t *sg = smem_raw + (sb - raw);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const AttnProblem &p = a.p;
    const int G = (int)gridDim.x, cta = (int)blockIdx.x;
    const int64_t T = a.num_tiles;
    constexpr int QS = C::QS, CPS = C::Q_CHUNKS_PER_SLOT;
    // Key blocks of the tile at q0 (causal tiles stop at their last row).
    auto tile_blocks = [&](int64_t q0) {
        const int64_t kv_end = p.causal ? min(p.S, q0 + C::BM) : p.S;
        return (int)((kv_end + C::BN - 1) / C::BN);
    };
    auto bar = [&](int i) { return sb + C::OFF_BAR + 8u * (uint32_t)i; };
    auto vslot = [&](int x) { return x % C::VST; };
    auto vpar = [&](int x) { return (uint32_t)((x / C::VST) & 1); };
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(sg + C::OFF_MISC);
    volatile int *abort = reinterpret_cast<volatile int *>(sg + C::OFF_MISC + 4);
    int *err = a.err;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::KST; s++) {
            mbar_init(bar(C::K_FULL + s), 1);
            mbar_init(bar(C::K_READY + s), 128);
            mbar_init(bar(C::K_EMPTY + s), 1);
        }
        for (int s = 0; s < C::VST; s++) {
            mbar_init(bar(C::V_FULL + s), 1);
            mbar_init(bar(C::V_READY + s), 128);
            mbar_init(bar(C::V_EMPTY + s), 1);
        }
        for (int s = 0; s < 2; s++) {
            mbar_init(bar(C::S_FULL + s), 1);
            mbar_init(bar(C::P_FULL + s), C::SOFTMAX_THREADS);
        }
        mbar_init(bar(C::PV_DONE_B), 1);
        mbar_init(bar(C::PV_DONE_B + 1), 1);
        mbar_init(bar(C::OB_FREE), C::SOFTMAX_THREADS);
        mbar_init(bar(C::OB_FREE + 1), C::SOFTMAX_THREADS);
        mbar_init(bar(C::XCH), C::SOFTMAX_THREADS);
        mbar_init(bar(C::XCH + 1), C::SOFTMAX_THREADS);
        mbar_init(bar(C::XSUM), C::SOFTMAX_THREADS);
        mbar_init(bar(C::DRAIN), 1);
        mbar_init(bar(C::DRAIN_PV), 1);
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == C::W_MMA) {
        tmem_alloc(smem_addr(tmem_slot), C::TMEM_COLS);
        tmem_relinquish();
    }
    if (warp == C::W_PROD && lane == 0) {
        prefetch_tmap(&tmq);
        prefetch_tmap(&tmk);
        prefetch_tmap(&tmv);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == C::W_PROD) {
        // ------------------------------------------------------------ TMA producer ----
        if (lane == 0) {
            int x = 0, kk = 0, x_last = -1, k_last = -1;
            bool ok = true;
            for (int64_t r = 0; ok; r++) {
                const int64_t t = fwd_tile_of(r, cta, G, T);
                if (t < 0) break;
                int64_t q0, h, b;
                fwd_tile(a, t, q0, h, b);
                const int64_t hk = h / p.group;
                const int nblk = tile_blocks(q0);
                // The raw Q tile into the next QS V-ring slots; the converters move it to TMEM.
                for (int s = 0; s < QS; s++, x++) {
                    const int vs = vslot(x);
                    if (x >= C::VST && !(ok = mbar_wait(bar(C::V_EMPTY + vs), vpar(x - C::VST), abort, err))) break;
                    mbar_expect_tx(bar(C::V_FULL + vs), C::KV_STAGE);
                    for (int c = 0; c < CPS; c++)
                        tma_load_4d(&tmq, sb + C::OFF_V + vs * C::KV_STAGE + c * C::Q_CHUNK, bar(C::V_FULL + vs),
                                    32 * (s * CPS + c), (int)q0, (int)h, (int)b);
                    x_last = x;
                }
                for (int j = 0; ok && j < nblk; j++) {
                    const int ks = kk % C::KST;
                    if (kk >= C::KST && !mbar_wait(bar(C::K_EMPTY + ks), (uint32_t)(((kk / C::KST) - 1) & 1), abort, err)) {
                        ok = false;
                        break;
                    }
                    mbar_expect_tx(bar(C::K_FULL + ks), C::KV_BYTES);
                    const uint32_t kd = sb + C::OFF_K + ks * C::KV_STAGE;
                    for (int c = 0; c < C::CHUNKS; c++)
                        tma_load_4d(&tmk, kd + c * C::KV_CHUNK, bar(C::K_FULL + ks), 32 * c, j * C::BN, (int)hk, (int)b);
                    k_last = kk++;
                    const int vs = vslot(x);
                    if (x >= C::VST && !mbar_wait(bar(C::V_EMPTY + vs), vpar(x - C::VST), abort, err)) {
                        ok = false;
                        break;
                    }
                    mbar_expect_tx(bar(C::V_FULL + vs), C::KV_BYTES);
                    const uint32_t vd = sb + C::OFF_V + vs * C::KV_STAGE;
                    for (int c = 0; c < C::CHUNKS; c++)
                        tma_load_4d(&tmv, vd + c * C::KV_CHUNK, bar(C::V_FULL + vs), 32 * c, j * C::BN, (int)hk, (int)b);
                    x_last = x++;
                }
            }
            if (*abort) {
                // Let the copies already in flight land before the CTA's memory goes away.
                volatile int never = 0;
                for (int i = max(0, k_last - C::KST + 1); i <= k_last; i++)
                    mbar_wait(bar(C::K_FULL + i % C::KST), (uint32_t)((i / C::KST) & 1), &never, nullptr);
                for (int i = max(0, x_last - C::VST + 1); i <= x_last; i++)
                    mbar_wait(bar(C::V_FULL + vslot(i)), vpar(i), &never, nullptr);
            }
        }
    } else if (warp == C::W_MMA) {
        // -------------------------------------------------------- MMA issuer: S = Q K^T ----
        // The whole warp runs the loop converged; one elected lane issues each MMA.
        {
            // Descriptor of K stage 0; stage and k-step offsets go into the address field.
            const uint64_t kdesc0 = sdesc_sw128(sb + C::OFF_K, 16, 1024);
            const uint32_t q_hi = tmem + C::COL_QHI, q_lo = tmem + C::COL_QLO;
            int x = 0, kk = 0, jg = 0;
            bool ok = true;
            for (int64_t r = 0; ok; r++) {
                const int64_t t = fwd_tile_of(r, cta, G, T);
                if (t < 0) break;
                int64_t q0, h, b;
                fwd_tile(a, t, q0, h, b);
                const int nblk = tile_blocks(q0);
                // This tile's Q is in TMEM once its V-ring slots are READY; those slots are then free.
                for (int s = 0; s < QS; s++)
                    if (!(ok = mbar_wait_warp(bar(C::V_READY + vslot(x + s)), vpar(x + s), abort, err))) break;
                if (!ok) break;
                if (lane == 0)
                    for (int s = 0; s < QS; s++) mbar_arrive(bar(C::V_EMPTY + vslot(x + s)));
                x += QS + nblk;
                tc_fence_after();
                for (int j = 0; j < nblk; j++, jg++, kk++) {
                    const int bb = jg & 1, ks = kk % C::KST;
                    // S buffer bb held P of block jg - 2, read by its PV.
                    if (jg >= 2 && !(ok = mbar_wait_warp(bar(C::PV_DONE_B + bb), (uint32_t)(((jg - 2) >> 1) & 1), abort, err)))
                        break;
                    if (!(ok = mbar_wait_warp(bar(C::K_READY + ks), (uint32_t)((kk / C::KST) & 1), abort, err))) break;
                    tc_fence_after();
                    const uint64_t kd = kdesc0 + ((ks * C::KV_STAGE) >> 4);
                    const uint32_t d_s = tmem + C::col_s(bb);
                    if (SPLIT) {  // Qhi Klo + Qlo Khi first, then Qhi Khi
#pragma unroll
                        for (int k8 = 0; k8 < C::D / 8; k8++) {
                            const uint32_t off = ((k8 >> 2) * C::KV_CHUNK + (k8 & 3) * 32) >> 4;
                            mma_tf32_ts_w(d_s, q_hi + k8 * 8, kd + ((C::KV_BYTES >> 4) + off), C::IDESC_S, k8 > 0 ? 1u : 0u);
                            mma_tf32_ts_w(d_s, q_lo + k8 * 8, kd + off, C::IDESC_S, 1u);
                        }
                    }
#pragma unroll
                    for (int k8 = 0; k8 < C::D / 8; k8++) {
                        const uint32_t off = ((k8 >> 2) * C::KV_CHUNK + (k8 & 3) * 32) >> 4;
                        mma_tf32_ts_w(d_s, q_hi + k8 * 8, kd + off, C::IDESC_S, (SPLIT || k8 > 0) ? 1u : 0u);
                    }
                    tc_commit_w(bar(C::S_FULL + bb));
                    tc_commit_w(bar(C::K_EMPTY + ks));
                }
            }
            // Every MMA this warp issued completes before TMEM is released.
            tc_commit_w(bar(C::DRAIN));
            volatile int never = 0;
            mbar_wait_warp(bar(C::DRAIN), 0, &never, nullptr);
        }
    } else if (warp == C::W_PV) {
        // ----------------------------------------------------- MMA issuer: O_blk = P V ----
        {
            const uint64_t vdesc0 = sdesc_mn_sw128_32b(sb + C::OFF_V, C::KV_CHUNK, 512);
            int x = 0, jg = 0;
            bool ok = true;
            for (int64_t r = 0; ok; r++) {
                const int64_t t = fwd_tile_of(r, cta, G, T);
                if (t < 0) break;
                int64_t q0, h, b;
                fwd_tile(a, t, q0, h, b);
                const int nblk = tile_blocks(q0);
                x += QS;
                for (int j = 0; j < nblk; j++, jg++, x++) {
                    const int bi = jg & 1, vs = vslot(x);
                    if (!(ok = mbar_wait_warp(bar(C::P_FULL + bi), (uint32_t)((jg >> 1) & 1), abort, err))) break;
                    if (!(ok = mbar_wait_warp(bar(C::V_READY + vs), vpar(x), abort, err))) break;
                    // O_blk buffer jg % NOB held block jg - NOB until the softmax threads folded it.
                    if (jg >= C::NOB &&
                        !(ok = mbar_wait_warp(bar(C::OB_FREE + (int)(jg % C::NOB)), (uint32_t)(((jg / C::NOB) - 1) & 1), abort, err)))
                        break;
                    const uint32_t d_ob = tmem + C::col_ob((int)(jg % C::NOB));
                    tc_fence_after();
                    const uint64_t vd = vdesc0 + ((vs * C::KV_STAGE) >> 4);
                    const uint32_t a_hi = tmem + C::col_s(bi), a_lo = tmem + C::col_plo(bi);
                    if (SPLIT) {  // the small cross terms first, then the main products
#pragma unroll
                        for (int k8 = 0; k8 < C::BN / 8; k8++) {
                            mma_tf32_ts_w(d_ob, a_hi + k8 * 8, vd + ((C::KV_BYTES + k8 * 1024) >> 4), C::IDESC_O,
                                          k8 > 0 ? 1u : 0u);
                            mma_tf32_ts_w(d_ob, a_lo + k8 * 8, vd + ((k8 * 1024) >> 4), C::IDESC_O, 1u);
                        }
                    }
#pragma unroll
                    for (int k8 = 0; k8 < C::BN / 8; k8++)
                        mma_tf32_ts_w(d_ob, a_hi + k8 * 8, vd + ((k8 * 1024) >> 4), C::IDESC_O, (SPLIT || k8 > 0) ? 1u : 0u);
                    tc_commit_w(bar(C::PV_DONE_B + bi));
                    tc_commit_w(bar(C::V_EMPTY + vs));
                }
            }
            tc_commit_w(bar(C::DRAIN_PV));
            volatile int never = 0;
            mbar_wait_warp(bar(C::DRAIN_PV), 0, &never, nullptr);
        }
    } else if (warp >= C::W_CVT && warp < C::W_PV) {
        // --------------------------------------------------------------- converters ----
        const int ct = threadIdx.x - 32 * C::W_CVT;
        const int quad = warp & 3;
        const uint32_t tl = tmem + ((uint32_t)(quad * 32) << 16);
        int x = 0, kk = 0, jg = 0;
        bool ok = true;
        for (int64_t r = 0; ok; r++) {
            const int64_t t = fwd_tile_of(r, cta, G, T);
            if (t < 0) break;
            int64_t q0, h, b;
            fwd_tile(a, t, q0, h, b);
            const int nblk = tile_blocks(q0);
            // The previous tile's last S MMA (block jg - 1) has read the old Q before the new one
            // overwrites it in TMEM. (S_FULL of that buffer cannot move on before this Q is in.)
            if (jg > 0 && !(ok = mbar_wait(bar(C::S_FULL + (int)((jg - 1) & 1)), (uint32_t)(((jg - 1) >> 1) & 1), abort, err)))
                break;
            tc_fence_after();
            for (int s = 0; s < QS; s++, x++) {
                const int vs = vslot(x);
                if (!(ok = mbar_wait(bar(C::V_FULL + vs), vpar(x), abort, err))) break;
                row_to_tmem<CPS, SPLIT>(sg + C::OFF_V + vs * C::KV_STAGE, C::Q_CHUNK, quad * 32 + lane, tl,
                                        C::COL_QHI + 32 * CPS * s, C::COL_QLO + 32 * CPS * s);
            }
            if (!ok) break;
            tmem_wait_st();
            tc_fence_before();
            for (int s = 0; s < QS; s++) mbar_arrive(bar(C::V_READY + vslot(x - QS + s)));
            for (int j = 0; j < nblk; j++, kk++, x++) {
                const int ks = kk % C::KST, vs = vslot(x);
                if (!(ok = mbar_wait(bar(C::K_FULL + ks), (uint32_t)((kk / C::KST) & 1), abort, err))) break;
                split_tile<SPLIT>(sg + C::OFF_K + ks * C::KV_STAGE, C::KV_BYTES, C::KV_BYTES, ct);
                fence_proxy_async_smem();
                mbar_arrive(bar(C::K_READY + ks));
                if (!(ok = mbar_wait(bar(C::V_FULL + vs), vpar(x), abort, err))) break;
                split_tile<SPLIT>(sg + C::OFF_V + vs * C::KV_STAGE, C::KV_BYTES, C::KV_BYTES, ct);
                fence_proxy_async_smem();
                mbar_arrive(bar(C::V_READY + vs));
            }
            jg += nblk;
        }
    } else {
        // ------------------------------------------------------------------ softmax ----
        const int row = threadIdx.x & 127, half = threadIdx.x >> 7;
        const uint32_t tl = tmem + ((uint32_t)((warp & 3) * 32) << 16);
        float *xmax = reinterpret_cast<float *>(sg + C::OFF_XMAX);  // [2][2][BM]
        float *xsum = reinterpret_cast<float *>(sg + C::OFF_XSUM);  // [2][BM]
        int jg = 0;
        bool ok = true;
        for (int64_t r = 0; ok; r++) {
            const int64_t t = fwd_tile_of(r, cta, G, T);
            if (t < 0) break;
            int64_t q0, h, b;
            fwd_tile(a, t, q0, h, b);
            const int nblk = tile_blocks(q0);
            const int64_t qrow = q0 + row;
            const bool row_ok = qrow < p.L;
            float m = -INFINITY, l = 0.0f;
            float o[C::HD];
#pragma unroll
            for (int x = 0; x < C::HD; x++) o[x] = 0.0f;
            for (int j = 0; j < nblk; j++, jg++) {
                const int bb = jg & 1;
                const int64_t k0 = (int64_t)j * C::BN + half * C::HB;
                // Rows past L (zero-filled by TMA) are computed but never stored. Column c is key
                // k0 + c: valid below S and, under causal masking, up to qrow (one bit per column
                // keeps the edge path as short as the fast one).
                const bool edge = MASKED || (k0 + C::HB > p.S) || (p.causal && k0 + C::HB - 1 > q0);
                uint32_t vbits = 0xFFFFFFFFu;
                if (edge) {
                    const int64_t lim = (p.causal ? min(p.S, qrow + 1) : p.S) - k0;
                    const int n = !row_ok || lim <= 0 ? 0 : (lim >= C::HB ? C::HB : (int)lim);
                    vbits = n == 0 ? 0u : (0xFFFFFFFFu >> (32 - n));
                }
                // The user mask's values for these columns, loaded before the wait for S so that
                // the wait hides their latency.
                float mk[MASKED ? C::HB : 1];
                if constexpr (MASKED) mask_run<C::HB>(p, b, h, qrow, k0, p.ms[3], vbits, mk);
                // Dropout: this row's keep bits for these columns (the weights that meet V are
                // P * keep_scale where kept, 0 where dropped; the row sum and lse stay undropped).
                uint32_t kbits = 0;
                if constexpr (DROP) kbits = row_ok ? keep_run32(p, b, h, qrow, k0) : 0u;
                if (!(ok = mbar_wait(bar(C::S_FULL + bb), (uint32_t)((jg >> 1) & 1), abort, err))) break;
                tc_fence_after();
                float s[C::HB];
                {
                    uint32_t rr[C::HB];
                    tmem_ld<C::HB>(tl + C::col_s(bb) + half * C::HB, rr);
                    tmem_wait_ld();
#pragma unroll
                    for (int x = 0; x < C::HB; x++) s[x] = __uint_as_float(rr[x]);
                }
                // Interior blocks keep the raw scores and fold the scale into the exponent's FFMA
                // (the max commutes with a positive scale); edge blocks scale, mask and fill first.
                const bool rawp = !edge && a.scale_log2 > 0.0f;
                const float smul = rawp ? a.scale_log2 : 1.0f;
                if (!rawp) {
#pragma unroll
                    for (int c = 0; c < C::HB; c++) {
                        float x = s[c] * a.scale_log2;
                        if (MASKED) x += mk[MASKED ? c : 0] * LOG2E;
                        s[c] = ((vbits >> c) & 1u) ? x : -INFINITY;
                    }
                }
                float bmax = max_tree<C::HB>(s) * smul;
                // The block's row max, shared with the partner thread (the other half) through
                // shared memory and an mbarrier (a bounded wait, unlike bar.sync).
                xmax[(bb * 2 + half) * C::BM + row] = bmax;
                mbar_arrive(bar(C::XCH + bb));
                if (!(ok = mbar_wait(bar(C::XCH + bb), (uint32_t)((jg >> 1) & 1), abort, err))) break;
                bmax = fmaxf(bmax, xmax[(bb * 2 + (half ^ 1)) * C::BM + row]);
                const float m_new = fmaxf(m, bmax);
                const bool rescale = m_new > m + 8.0f;
                float corr = 1.0f;
                if (rescale) {
                    corr = ex2_approx(m - m_new);
                    m = m_new;
                }
                const bool dead = (m == -INFINITY);
                float part[4] = {0.0f, 0.0f, 0.0f, 0.0f};  // four partial row sums: shorter chains
#pragma unroll
                for (int r0 = 0; r0 < C::HB; r0 += 16) {  // P in 16-column pieces
                    uint32_t phi[16], plo[16];
#pragma unroll
                    for (int c = 0; c < 16; c++) {
                        const float pc = dead ? 0.0f : ex2_approx(fmaf(s[r0 + c], smul, -m));
                        part[c & 3] += pc;
                        float pw = pc;
                        if constexpr (DROP) pw = ((kbits >> (r0 + c)) & 1u) ? pc * p.keep_scale : 0.0f;
                        if (SPLIT) {
                            phi[c] = __float_as_uint(pw);
                            plo[c] = tf32_lo_trunc(pw);
                        } else {
                            phi[c] = tf32_rna(pw);
                        }
                    }
                    tmem_st16(tl + C::col_s(bb) + half * C::HB + r0, phi);
                    if (SPLIT) tmem_st16(tl + C::col_plo(bb) + half * C::HB + r0, plo);
                }
                const float rs = (part[0] + part[1]) + (part[2] + part[3]);
                l = fmaf(l, corr, rs);
                tmem_wait_st();
                tc_fence_before();
                mbar_arrive(bar(C::P_FULL + bb));
                // Fold the previous block: o = (o + O_blk(jg-1)) * corr (both relative to the
                // previous max; corr moves them to m).
                if (j >= 1) {
                    // Per-buffer barrier: with two O_blk buffers PV_jg may finish before this wait,
                    // so a single barrier could be two phases ahead of it.
                    if (!(ok = mbar_wait(bar(C::PV_DONE_B + (int)((jg - 1) & 1)), (uint32_t)(((jg - 1) >> 1) & 1), abort, err)))
                        break;
                    tc_fence_after();
                    const bool scaled = __any_sync(0xffffffffu, corr != 1.0f);
#pragma unroll
                    for (int c = 0; c < C::HD / 16; c++) {
                        uint32_t rr[16];
                        tmem_ld16(tl + C::col_ob((int)((jg - 1) % C::NOB)) + half * C::HD + 16 * c, rr);
                        tmem_wait_ld();
                        if (scaled) {
#pragma unroll
                            for (int x = 0; x < 16; x++) o[16 * c + x] = (o[16 * c + x] + __uint_as_float(rr[x])) * corr;
                        } else {
#pragma unroll
                            for (int x = 0; x < 16; x++) o[16 * c + x] += __uint_as_float(rr[x]);
                        }
                    }
                    tc_fence_before();
                    mbar_arrive(bar(C::OB_FREE + (int)((jg - 1) % C::NOB)));
                }
            }
            // The tile's last block: its O_blk into the registers, its buffer freed for the next
            // tile's PV MMAs.
            const int jl = jg - 1;
            if (ok) {
                ok = mbar_wait(bar(C::PV_DONE_B + (int)(jl & 1)), (uint32_t)((jl >> 1) & 1), abort, err);
                tc_fence_after();
            }
            const bool read_o = __all_sync(0xffffffffu, ok);
            if (read_o) {
#pragma unroll
                for (int c = 0; c < C::HD / 32; c++) {
                    uint32_t rr[32];
                    tmem_ld32(tl + C::col_ob((int)(jl % C::NOB)) + half * C::HD + 32 * c, rr);
                    tmem_wait_ld();
#pragma unroll
                    for (int x = 0; x < 32; x++) o[32 * c + x] += __uint_as_float(rr[x]);
                }
                tc_fence_before();
                mbar_arrive(bar(C::OB_FREE + (int)(jl % C::NOB)));
            }
            if (!read_o) ok = false;
            const bool aborted = __any_sync(0xffffffffu, *abort != 0);
            // The row sum: this half's part plus the partner's. (A thread can only write the next
            // tile's sum after its partner passed the next tile's first max exchange, so after it
            // read this one.)
            xsum[half * C::BM + row] = l;
            mbar_arrive(bar(C::XSUM));
            const bool have_sum = mbar_wait(bar(C::XSUM), (uint32_t)(r & 1), abort, err);
            l += xsum[(half ^ 1) * C::BM + row];
            if (!have_sum) ok = false;
            if (ok && !aborted && row_ok) {
                const float lfin = l == 0.0f ? 1.0f : l;
                const float mnat = m == -INFINITY ? 0.0f : m * LN2;
                const float inv = 1.0f / lfin;
                float *orow = p.out + b * p.os[0] + h * p.os[1] + qrow * p.os[2] + (int64_t)half * C::HD * p.os[3];
                if (p.os[3] == 1 && (reinterpret_cast<uintptr_t>(orow) & 15u) == 0) {
#pragma unroll
                    for (int x = 0; x < C::HD; x += 4)
                        *reinterpret_cast<float4 *>(orow + x) =
                            make_float4(o[x] * inv, o[x + 1] * inv, o[x + 2] * inv, o[x + 3] * inv);
                } else {
#pragma unroll
                    for (int x = 0; x < C::HD; x++) orow[x * p.os[3]] = o[x] * inv;
                }
                if (half == 0) p.lse[b * p.ls[0] + h * p.ls[1] + qrow * p.ls[2]] = mnat + logf(lfin);
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == C::W_MMA) {
        tc_fence_after();
        tmem_dealloc(tmem, C::TMEM_COLS);
    }
}

// The forward instantiation for (split, masked, dropout): persistent, or one CTA per tile.
template <class C, bool PERSIST>
decltype(&attn_fwd_tc_kernel<C, true, true, true>) pick_fwd(bool split, bool masked, bool drop) {
#define DC_FWD(S, M, D) (PERSIST ? attn_fwd_tc_persist_kernel<C, S, M, D> : attn_fwd_tc_kernel<C, S, M, D>)
    if (drop)
        return split ? (masked ? DC_FWD(true, true, true) : DC_FWD(true, false, true))
                     : (masked ? DC_FWD(false, true, true) : DC_FWD(false, false, true));
    return split ? (masked ? DC_FWD(true, true, false) : DC_FWD(true, false, false))
                 : (masked ? DC_FWD(false, true, false) : DC_FWD(false, false, false));
#undef DC_FWD
}

template <class C>
int launch_fwd(const AttnProblem &p, int split, cudaStream_t stream) {
    CUtensorMap tq, tk, tv;
    int st = make_tmap(&tq, p.q, p.E, p.L, p.H, p.B, p.qs, C::BM);
    if (!st) st = make_tmap(&tk, p.k, p.E, p.S, p.Hkv, p.B, p.ks, C::BN);
    // V is the MN-major B operand of O += P V: tf32 needs the 32-byte-atom swizzle there.
    if (!st) st = make_tmap(&tv, p.v, p.Ev, p.S, p.Hkv, p.B, p.vs, C::BN, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
    if (st) return st;
    TcFwdArgs a;
    a.p = p;
    a.num_q_tiles = (int)((p.L + C::BM - 1) / C::BM);
    a.scale_log2 = p.scale * LOG2E;
    a.err = device_error_word();
    if (!a.err) return fail(DC_ERR_CUDA, "device error word is unavailable");
    const bool masked = p.mask_kind != MASK_NONE;
    const bool drop = p.keep != nullptr;
    a.num_tiles = (int64_t)a.num_q_tiles * p.H * p.B;
    // Groups of heads whose K and V (S * (E + Ev) floats each) fit in about 48 MB, within one of
    // the L2's two 63 MB partitions (at 67 MB, two of config 4's heads, the forward measured
    // 28 ms against 22 ms with one head at a time).
    const int64_t kv_bytes = p.S * (p.E + p.Ev) * 4, hb = p.H * p.B;
    a.group_heads = kv_bytes > 0 ? (48ll << 20) / kv_bytes : hb;
    a.group_heads = a.group_heads < 1 ? 1 : (a.group_heads > hb ? hb : a.group_heads);
    // Short tiles (up to 64 key blocks) run persistently, one CTA per SM (tensor and shared
    // memory admit one) walking the schedule, so that a tile's start-up overlaps the previous
    // tile's tail; long tiles take one CTA each, which the hardware hands out in schedule order.
    const int64_t sms = device_sm_count();
    const bool persistent = (p.S + C::BN - 1) / C::BN <= 64 && a.num_tiles < (1ll << 31);
    const int64_t ctas = persistent && a.num_tiles > sms ? sms : a.num_tiles;
    auto kernel = persistent ? pick_fwd<C, true>(split, masked, drop) : pick_fwd<C, false>(split, masked, drop);
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::SMEM);
    if (e != cudaSuccess) return cuda_fail(e, "attn_fwd_tc smem attribute");
    const dim3 grid = persistent ? dim3((unsigned)ctas) : dim3((unsigned)a.num_q_tiles, (unsigned)p.H, (unsigned)p.B);
    KernelTrace tr(C::D == 64 ? "fwd_tc_d64" : "fwd_tc_d128", stream);
    kernel<<<grid, C::THREADS, C::SMEM, stream>>>(tq, tk, tv, a);
    return check_launch("attn_fwd_tc");
}

using Fwd64 = FwdCfg<64, 64, 3, 3>;
using Fwd128 = FwdCfg<128, 32, 3, 3>;

bool aligned16(const void *ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

}  // namespace

int *device_error_word() {
    void *ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_tc_error) != cudaSuccess) return nullptr;
    return static_cast<int *>(ptr);
}

bool tc_forward_supported(const AttnProblem &p) {
    if (p.E != p.Ev || (p.E != 64 && p.E != 128)) return false;
    if (p.qs[3] != 1 || p.ks[3] != 1 || p.vs[3] != 1) return false;
    if (!tma_stride_ok(p.L, p.qs[2]) || !tma_stride_ok(p.H, p.qs[1]) || !tma_stride_ok(p.B, p.qs[0])) return false;
    if (!tma_stride_ok(p.S, p.ks[2]) || !tma_stride_ok(p.Hkv, p.ks[1]) || !tma_stride_ok(p.B, p.ks[0])) return false;
    if (!tma_stride_ok(p.S, p.vs[2]) || !tma_stride_ok(p.Hkv, p.vs[1]) || !tma_stride_ok(p.B, p.vs[0])) return false;
    if (!aligned16(p.q) || !aligned16(p.k) || !aligned16(p.v)) return false;
    if (p.L >= (1ll << 31) || p.S >= (1ll << 31) || p.L == 0 || p.S == 0) return false;
    return true;
}

int tc_forward(const AttnProblem &p, int precision, cudaStream_t stream) {
    const int split = precision == DC_PREC_TF32 ? 0 : 1;
    return p.E == 64 ? launch_fwd<Fwd64>(p, split, stream) : launch_fwd<Fwd128>(p, split, stream);
}

int device_error(int reset) {
    int v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_tc_error, sizeof(int));
    if (e != cudaSuccess) return -1;
    if (reset && v) {
        int z = 0;
        cudaMemcpyToSymbol(g_tc_error, &z, sizeof(int));
    }
    return v;
}

}  // namespace dc

