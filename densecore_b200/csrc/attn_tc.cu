// attn_tc.cu -- tcgen05 tensor-core attention forward for sm_100a.
//
// Replaces DenseCore's torch_attention::forward (src/torch_attention.rs:146-284) for head dim
// 64 and 128 with a warp-specialised kernel; one CTA computes a 128-row query tile of one
// (batch, head):
//
//   warp 4      TMA producer: the Q tile once, then K and V tiles of BN keys into rings of
//               shared-memory stages (128-byte swizzle, 4-D tensor maps over the caller's
//               strided (B, H, L, E) views, zero fill past the sequence end).
//   warps 6-9   converters (3xTF32): split each landed fp32 tile x into hi = tf32(x) in
//               place and lo = tf32(x - hi) beside it, so that a*b ~ ah*bh + ah*bl + al*bh
//               keeps fp32-class accuracy on the TF32 tensor cores.
//   warp 5      MMA issuer: S = Q K^T into TMEM (two S buffers), then O += P V with P read
//               from TMEM (A operand) and V from shared memory (MN-major B operand, which for
//               tf32 must use the 32-byte-atom 128-byte swizzle). Issue
//               order S0, S1, PV0, S2, PV1, ... so the tensor core works on S(j+1) while
//               the softmax warps handle block j.
//   warps 0-3   softmax: thread t owns query row t (TMEM lane t). Online softmax in base 2
//               with DenseCore's rules (a block whose running max is -inf adds nothing,
//               :218-226); P is written back to TMEM as tf32 hi/lo over the consumed S
//               columns. The running max moves only when it grows by more than 2^8 (the sum
//               and the output share the stale max, so the result is unchanged).
//               Each block's P V goes to a fresh TMEM accumulator (a handful of tensor-core
//               accumulation steps, whose internal rounding is coarser than fp32); the
//               softmax threads fold it into the running output with fp32 adds, one block
//               behind, while the tensor core works on the next block. Finalisation as the
//               reference: max -inf -> 0, sum 0 -> 1, out = acc/sum, lse = max + log(sum)
//               (:258-271).
//
// Every mbarrier wait is bounded (sm100::mbar_wait); a wait that times out sets a device
// error word and the CTA unwinds, frees its TMEM and exits.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <math.h>

#include <mutex>

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
    static constexpr int CHUNKS = D / 32;  // 128-byte column chunks of a row
    static constexpr uint32_t Q_CHUNK = BM * 128;
    static constexpr uint32_t KV_CHUNK = BN * 128;
    static constexpr uint32_t Q_BYTES = BM * D * 4;
    static constexpr uint32_t KV_BYTES = BN * D * 4;
    static constexpr uint32_t OFF_QHI = 0;
    static constexpr uint32_t OFF_QLO = Q_BYTES;
    static constexpr uint32_t OFF_K = 2 * Q_BYTES;
    static constexpr uint32_t OFF_V = OFF_K + KST * 2 * KV_BYTES;
    static constexpr uint32_t OFF_BAR = OFF_V + VST * 2 * KV_BYTES;
    // Barrier indices.
    static constexpr int Q_FULL = 0, Q_READY = 1, K_FULL = 2, K_READY = K_FULL + KST,
                         K_EMPTY = K_READY + KST, V_FULL = K_EMPTY + KST, V_READY = V_FULL + VST,
                         V_EMPTY = V_READY + VST, S_FULL = V_EMPTY + VST, P_FULL = S_FULL + 2,
                         PV_DONE = P_FULL + 2, OB_FREE = PV_DONE + 2, DRAIN = OB_FREE + 2,
                         NBAR = DRAIN + 1;
    static constexpr uint32_t OFF_MISC = OFF_BAR + NBAR * 8;
    static constexpr uint32_t SMEM = OFF_MISC + 16 + 1024;  // + slack for 1024-byte alignment
    // TMEM: the running output (fp32, folded by CUDA cores), two per-block P V accumulators,
    // then two (S / P_hi, P_lo) buffers.
    static constexpr uint32_t COL_O = 0;
    __host__ __device__ static constexpr uint32_t col_ob(int b) { return D + b * D; }
    static constexpr uint32_t COLS_USED = 3 * D + 4 * BN;
    static constexpr uint32_t TMEM_COLS = COLS_USED <= 128 ? 128 : COLS_USED <= 256 ? 256 : 512;
    static constexpr int THREADS = 320;
    static constexpr uint32_t IDESC_S = idesc_tf32(128, BN, 0, 0);
    static constexpr uint32_t IDESC_O = idesc_tf32(128, D, 0, 1);
    __host__ __device__ static constexpr uint32_t col_s(int b) { return 3 * D + b * 2 * BN; }
    __host__ __device__ static constexpr uint32_t col_plo(int b) { return 3 * D + b * 2 * BN + BN; }
    static_assert(SMEM <= 232448, "shared memory budget");
    static_assert(COLS_USED <= 512, "tensor memory budget");
};

struct TcFwdArgs {
    AttnProblem p;
    int split;  // 1: 3xTF32, 0: single-pass TF32
    int num_q_tiles;
    float scale_log2;
};

// hi = tf32(x) in place and, when split, lo = tf32(x - hi) at the same offset of the lo
// buffer. Single-pass TF32 rounds to nearest here rather than letting the tensor core drop
// the low mantissa bits (which would bias every operand toward zero).
__device__ __forceinline__ void split_tile(uint8_t *hi, uint8_t *lo, uint32_t bytes, int t, int nt, int split) {
    float4 *h = reinterpret_cast<float4 *>(hi);
    float4 *l = reinterpret_cast<float4 *>(lo);
    for (uint32_t i = t; i < bytes / 16; i += nt) {
        float4 x = h[i];
        uint32_t a0 = tf32_rna(x.x), a1 = tf32_rna(x.y), a2 = tf32_rna(x.z), a3 = tf32_rna(x.w);
        float4 hv = make_float4(__uint_as_float(a0), __uint_as_float(a1), __uint_as_float(a2),
                                __uint_as_float(a3));
        h[i] = hv;
        if (split)
            l[i] = make_float4(__uint_as_float(tf32_rna(x.x - hv.x)), __uint_as_float(tf32_rna(x.y - hv.y)),
                               __uint_as_float(tf32_rna(x.z - hv.z)), __uint_as_float(tf32_rna(x.w - hv.w)));
    }
}

template <class C>
__global__ void __launch_bounds__(C::THREADS, 1)
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
            mbar_init(bar(C::P_FULL + s), 128);
            mbar_init(bar(C::PV_DONE + s), 1);
            mbar_init(bar(C::OB_FREE + s), 128);
        }
        mbar_init(bar(C::DRAIN), 1);
        *abort = 0;
        fence_mbar_init();
    }
    if (warp == 5) {
        tmem_alloc(smem_addr(tmem_slot), C::TMEM_COLS);
        tmem_relinquish();
    }
    if (warp == 4 && lane == 0) {
        prefetch_tmap(&tmq);
        prefetch_tmap(&tmk);
        prefetch_tmap(&tmv);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 4) {
        // ------------------------------------------------------------ TMA producer ----
        if (lane == 0) {
            int k_issued = -1, v_issued = -1;
            mbar_expect_tx(bar(C::Q_FULL), C::Q_BYTES);
            for (int c = 0; c < C::CHUNKS; c++)
                tma_load_4d(&tmq, sb + C::OFF_QHI + c * C::Q_CHUNK, bar(C::Q_FULL), 32 * c, (int)q0,
                            (int)h, (int)b);
            for (int j = 0; j < nblk; j++) {
                const int ks = j % C::KST, vs = j % C::VST;
                if (j >= C::KST &&
                    !mbar_wait(bar(C::K_EMPTY + ks), ((j / C::KST) - 1) & 1, abort, &g_tc_error))
                    break;
                mbar_expect_tx(bar(C::K_FULL + ks), C::KV_BYTES);
                const uint32_t kd = sb + C::OFF_K + ks * 2 * C::KV_BYTES;
                for (int c = 0; c < C::CHUNKS; c++)
                    tma_load_4d(&tmk, kd + c * C::KV_CHUNK, bar(C::K_FULL + ks), 32 * c, j * C::BN,
                                (int)hk, (int)b);
                k_issued = j;
                if (j >= C::VST &&
                    !mbar_wait(bar(C::V_EMPTY + vs), ((j / C::VST) - 1) & 1, abort, &g_tc_error))
                    break;
                mbar_expect_tx(bar(C::V_FULL + vs), C::KV_BYTES);
                const uint32_t vd = sb + C::OFF_V + vs * 2 * C::KV_BYTES;
                for (int c = 0; c < C::CHUNKS; c++)
                    tma_load_4d(&tmv, vd + c * C::KV_CHUNK, bar(C::V_FULL + vs), 32 * c, j * C::BN,
                                (int)hk, (int)b);
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
    } else if (warp == 5) {
        // -------------------------------------------------------------- MMA issuer ----
        if (lane == 0) {
            const uint32_t qhi = sb + C::OFF_QHI, qlo = sb + C::OFF_QLO;
            bool ok = mbar_wait(bar(C::Q_READY), 0, abort, &g_tc_error);
            tc_fence_after();
            for (int j = 0; ok && j <= nblk; j++) {
                if (j < nblk) {
                    const int bb = j & 1, ks = j % C::KST;
                    if (!mbar_wait(bar(C::K_READY + ks), (j / C::KST) & 1, abort, &g_tc_error)) break;
                    if (j >= 2 && !mbar_wait(bar(C::PV_DONE + bb), ((j - 2) >> 1) & 1, abort, &g_tc_error))
                        break;
                    tc_fence_after();
                    const uint32_t khi = sb + C::OFF_K + ks * 2 * C::KV_BYTES, klo = khi + C::KV_BYTES;
                    const uint32_t d_s = tmem + C::col_s(bb);
                    if (a.split) {  // cross terms Qhi Klo + Qlo Khi first, then Qhi Khi
#pragma unroll
                        for (int kk = 0; kk < C::D / 8; kk++) {
                            const uint32_t oq = (kk >> 2) * C::Q_CHUNK + (kk & 3) * 32;
                            const uint32_t ok_ = (kk >> 2) * C::KV_CHUNK + (kk & 3) * 32;
                            mma_tf32_ss(d_s, sdesc_sw128(qhi + oq, 16, 1024), sdesc_sw128(klo + ok_, 16, 1024),
                                        C::IDESC_S, kk > 0 ? 1u : 0u);
                            mma_tf32_ss(d_s, sdesc_sw128(qlo + oq, 16, 1024), sdesc_sw128(khi + ok_, 16, 1024),
                                        C::IDESC_S, 1);
                        }
                    }
#pragma unroll
                    for (int kk = 0; kk < C::D / 8; kk++) {
                        const uint32_t oq = (kk >> 2) * C::Q_CHUNK + (kk & 3) * 32;
                        const uint32_t ok_ = (kk >> 2) * C::KV_CHUNK + (kk & 3) * 32;
                        mma_tf32_ss(d_s, sdesc_sw128(qhi + oq, 16, 1024), sdesc_sw128(khi + ok_, 16, 1024),
                                    C::IDESC_S, (a.split || kk > 0) ? 1u : 0u);
                    }
                    tc_commit(bar(C::S_FULL + bb));
                    tc_commit(bar(C::K_EMPTY + ks));
                }
                if (j >= 1) {
                    // O_blk(jp) = P(jp) V(jp) in a fresh accumulator: few tensor-core
                    // accumulation steps per block; the CUDA cores fold blocks in fp32.
                    const int jp = j - 1, bp = jp & 1, vs = jp % C::VST;
                    if (!mbar_wait(bar(C::P_FULL + bp), (jp >> 1) & 1, abort, &g_tc_error)) break;
                    if (!mbar_wait(bar(C::V_READY + vs), (jp / C::VST) & 1, abort, &g_tc_error)) break;
                    if (jp >= 2 && !mbar_wait(bar(C::OB_FREE + bp), ((jp - 2) >> 1) & 1, abort, &g_tc_error))
                        break;
                    tc_fence_after();
                    const uint32_t vhi = sb + C::OFF_V + vs * 2 * C::KV_BYTES, vlo = vhi + C::KV_BYTES;
                    const uint32_t d_o = tmem + C::col_ob(bp);
                    const uint32_t a_hi = tmem + C::col_s(bp), a_lo = tmem + C::col_plo(bp);
                    if (a.split) {  // the small cross terms first, then the main products
#pragma unroll
                        for (int kk = 0; kk < C::BN / 8; kk++) {
                            const uint64_t bv = sdesc_mn_sw128_32b(vhi + kk * 1024, C::KV_CHUNK, 512);
                            mma_tf32_ts(d_o, a_hi + kk * 8, sdesc_mn_sw128_32b(vlo + kk * 1024, C::KV_CHUNK, 512),
                                        C::IDESC_O, kk > 0 ? 1u : 0u);
                            mma_tf32_ts(d_o, a_lo + kk * 8, bv, C::IDESC_O, 1);
                        }
                    }
#pragma unroll
                    for (int kk = 0; kk < C::BN / 8; kk++) {
                        const uint64_t bv = sdesc_mn_sw128_32b(vhi + kk * 1024, C::KV_CHUNK, 512);
                        mma_tf32_ts(d_o, a_hi + kk * 8, bv, C::IDESC_O, (a.split || kk > 0) ? 1u : 0u);
                    }
                    tc_commit(bar(C::PV_DONE + bp));
                    tc_commit(bar(C::V_EMPTY + vs));
                }
            }
            // Every MMA issued so far completes before TMEM is released.
            tc_commit(bar(C::DRAIN));
            volatile int never = 0;
            mbar_wait(bar(C::DRAIN), 0, &never, nullptr);
        }
    } else if (warp >= 6) {
        // --------------------------------------------------------------- converters ----
        const int ct = threadIdx.x - 192;
        if (mbar_wait(bar(C::Q_FULL), 0, abort, &g_tc_error)) {
            split_tile(sg + C::OFF_QHI, sg + C::OFF_QLO, C::Q_BYTES, ct, 128, a.split);
            fence_proxy_async_smem();
            mbar_arrive(bar(C::Q_READY));
            for (int j = 0; j < nblk; j++) {
                const int ks = j % C::KST, vs = j % C::VST;
                if (!mbar_wait(bar(C::K_FULL + ks), (j / C::KST) & 1, abort, &g_tc_error)) break;
                {
                    uint8_t *kh = sg + C::OFF_K + ks * 2 * C::KV_BYTES;
                    split_tile(kh, kh + C::KV_BYTES, C::KV_BYTES, ct, 128, a.split);
                    fence_proxy_async_smem();
                }
                mbar_arrive(bar(C::K_READY + ks));
                if (!mbar_wait(bar(C::V_FULL + vs), (j / C::VST) & 1, abort, &g_tc_error)) break;
                {
                    uint8_t *vh = sg + C::OFF_V + vs * 2 * C::KV_BYTES;
                    split_tile(vh, vh + C::KV_BYTES, C::KV_BYTES, ct, 128, a.split);
                    fence_proxy_async_smem();
                }
                mbar_arrive(bar(C::V_READY + vs));
            }
        }
    } else {
        // ------------------------------------------------------------------ softmax ----
        const int row = threadIdx.x;
        const int64_t qrow = q0 + row;
        const bool row_ok = qrow < p.L;
        const uint32_t tl = tmem + ((uint32_t)(warp * 32) << 16);
        float m = -INFINITY, l = 0.0f;
        bool ok = true;
        for (int j = 0; j < nblk; j++) {
            const int bb = j & 1;
            if (!mbar_wait(bar(C::S_FULL + bb), (j >> 1) & 1, abort, &g_tc_error)) {
                ok = false;
                break;
            }
            tc_fence_after();
            float s[C::BN];
#pragma unroll
            for (int c = 0; c < C::BN / 32; c++) {
                uint32_t r[32];
                tmem_ld32(tl + C::col_s(bb) + 32 * c, r);
                tmem_wait_ld();
#pragma unroll
                for (int x = 0; x < 32; x++) s[32 * c + x] = __uint_as_float(r[x]);
            }
            const int64_t k0 = (int64_t)j * C::BN;
            // Rows past L (zero-filled by TMA) are computed but never stored.
            const bool edge = (k0 + C::BN > p.S) || (p.causal && k0 + C::BN - 1 > q0) ||
                              p.mask_kind != MASK_NONE;
            float bmax = -INFINITY;
            if (!edge) {
#pragma unroll
                for (int c = 0; c < C::BN; c++) {
                    s[c] *= a.scale_log2;
                    bmax = fmaxf(bmax, s[c]);
                }
            } else {
#pragma unroll
                for (int c = 0; c < C::BN; c++) {
                    const int64_t key = k0 + c;
                    float x = s[c] * a.scale_log2;
                    if (!row_ok || key >= p.S || (p.causal && key > qrow))
                        x = -INFINITY;
                    else if (p.mask_kind != MASK_NONE)
                        x += mask_value(p, b, h, qrow, key) * LOG2E;
                    s[c] = x;
                    bmax = fmaxf(bmax, x);
                }
            }
            const float m_new = fmaxf(m, bmax);
            const bool rescale = m_new > m + 8.0f;
            float corr = 1.0f;
            if (rescale) {
                corr = exp2f(m - m_new);
                m = m_new;
            }
            const bool dead = (m == -INFINITY);
            float rs = 0.0f;
#pragma unroll
            for (int c = 0; c < C::BN / 32; c++) {
                uint32_t hi[32], lo[32];
#pragma unroll
                for (int x = 0; x < 32; x++) {
                    const float pc = dead ? 0.0f : exp2f(s[32 * c + x] - m);
                    rs += pc;
                    if (a.split) {
                        hi[x] = tf32_rna(pc);
                        lo[x] = tf32_rna(pc - __uint_as_float(hi[x]));
                    } else {
                        hi[x] = tf32_rna(pc);
                    }
                }
                tmem_st32(tl + C::col_s(bb) + 32 * c, hi);
                if (a.split) tmem_st32(tl + C::col_plo(bb) + 32 * c, lo);
            }
            l = fmaf(l, corr, rs);
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(bar(C::P_FULL + bb));
            // Fold the previous block: O = (O + O_blk(j-1)) * corr, in fp32 on the CUDA cores
            // (O_blk(j-1) and O are both relative to the previous max; corr moves them to m).
            if (j >= 1) {
                const int jp = j - 1, bp = jp & 1;
                if (!mbar_wait(bar(C::PV_DONE + bp), (jp >> 1) & 1, abort, &g_tc_error)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
#pragma unroll
                for (int c = 0; c < C::CHUNKS; c++) {
                    uint32_t ob[32], o[32];
                    tmem_ld32(tl + C::col_ob(bp) + 32 * c, ob);
                    if (jp >= 1) tmem_ld32(tl + C::COL_O + 32 * c, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int x = 0; x < 32; x++) {
                        const float acc = jp >= 1 ? __uint_as_float(o[x]) + __uint_as_float(ob[x])
                                                  : __uint_as_float(ob[x]);
                        o[x] = __float_as_uint(acc * corr);
                    }
                    tmem_st32(tl + C::COL_O + 32 * c, o);
                }
                tmem_wait_st();
                tc_fence_before();
                mbar_arrive(bar(C::OB_FREE + bp));
            }
        }
        if (ok && nblk > 0) {
            ok = mbar_wait(bar(C::PV_DONE + ((nblk - 1) & 1)), ((nblk - 1) >> 1) & 1, abort, &g_tc_error);
            tc_fence_after();
        }
        const bool read_o = __all_sync(0xffffffffu, ok) && nblk > 0;
        const bool aborted = __any_sync(0xffffffffu, *abort != 0);
        if (!aborted) {
            const float lfin = l == 0.0f ? 1.0f : l;
            const float mnat = m == -INFINITY ? 0.0f : m * LN2;
            const float inv = 1.0f / lfin;
            float *orow = p.out + b * p.os[0] + h * p.os[1] + qrow * p.os[2];
            const int last = (nblk - 1) & 1;
#pragma unroll
            for (int c = 0; c < C::CHUNKS; c++) {
                uint32_t ob[32], o[32];
                if (read_o) {
                    tmem_ld32(tl + C::col_ob(last) + 32 * c, ob);
                    if (nblk >= 2) tmem_ld32(tl + C::COL_O + 32 * c, o);
                    tmem_wait_ld();
                } else {
#pragma unroll
                    for (int x = 0; x < 32; x++) ob[x] = 0u;
                }
                if (row_ok) {
#pragma unroll
                    for (int x = 0; x < 32; x++) {
                        const float acc = (read_o && nblk >= 2) ? __uint_as_float(o[x]) + __uint_as_float(ob[x])
                                                                : __uint_as_float(ob[x]);
                        orow[(32 * c + x) * p.os[3]] = acc * inv;
                    }
                }
            }
            if (row_ok) p.lse[b * p.ls[0] + h * p.ls[1] + qrow * p.ls[2]] = mnat + logf(lfin);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 5) {
        tc_fence_after();
        tmem_dealloc(tmem, C::TMEM_COLS);
    }
}

// ------------------------------------------------------------------- host side -------

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
    a.split = split;
    a.num_q_tiles = (int)((p.L + C::BM - 1) / C::BM);
    a.scale_log2 = p.scale * LOG2E;
    cudaError_t e = cudaFuncSetAttribute(attn_fwd_tc_kernel<C>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)C::SMEM);
    if (e != cudaSuccess) return cuda_fail(e, "attn_fwd_tc smem attribute");
    dim3 grid((unsigned)a.num_q_tiles, (unsigned)p.H, (unsigned)p.B);
    KernelTrace tr(C::D == 64 ? "fwd_tc_d64" : "fwd_tc_d128", stream);
    attn_fwd_tc_kernel<C><<<grid, C::THREADS, C::SMEM, stream>>>(tq, tk, tv, a);
    return check_launch("attn_fwd_tc");
}

using Fwd64 = FwdCfg<64, 64, 2, 2>;
using Fwd128 = FwdCfg<128, 32, 2, 1>;

bool aligned16(const void *ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

}  // namespace

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
