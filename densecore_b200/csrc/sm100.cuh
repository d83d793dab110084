// sm100.cuh -- inline-PTX wrappers for the Blackwell (sm_100a) features the tensor-core
// kernels use: mbarriers with bounded waits, TMA tile loads, tcgen05 MMA / TMEM access,
// shared-memory matrix descriptors and TF32 rounding. No cluster multicast anywhere.
#pragma once

#include <cuda.h>
#include <stdint.h>

namespace dc {
namespace sm100 {

// A wait that has not completed after this long is treated as a hang: the kernel records
// an error code and unwinds instead of spinning forever.
constexpr uint64_t WAIT_TIMEOUT_NS = 1000000000ull;  // 1 s

enum DeviceError : int { DEV_OK = 0, DEV_WAIT_TIMEOUT = 1, DEV_BAD_GENERATOR_STATE = 2 };

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// ---------------------------------------------------------------- mbarrier --------
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(bar),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Waits for the phase of `bar` with the given parity. Gives up (returns false) when *abort
// is set by another thread or after timeout_ns (WAIT_TIMEOUT_NS in every kernel; only the
// wait probe of selftest.cu passes a shorter bound), in which case it sets *abort and
// records DEV_WAIT_TIMEOUT in *err_flag.
//
// Only the first try_wait is inlined at each call site; the bounded spin after it is one
// out-of-line function, which keeps the kernels' many wait sites from crowding the hot loops
// out of the instruction cache.
static __device__ __noinline__ bool mbar_wait_spin(uint32_t bar, uint32_t parity, volatile int *abort, int *err_flag,
                                                   uint64_t timeout_ns);
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int *abort,
                                          int *err_flag, uint64_t timeout_ns = WAIT_TIMEOUT_NS) {
    if (mbar_try_wait(bar, parity)) return true;
    return mbar_wait_spin(bar, parity, abort, err_flag, timeout_ns);
}
static __device__ __noinline__ bool mbar_wait_spin(uint32_t bar, uint32_t parity, volatile int *abort, int *err_flag,
                                                   uint64_t timeout_ns) {
    const uint64_t t0 = globaltimer();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 63u) == 0) {
            if (*abort) return false;
            if (globaltimer() - t0 > timeout_ns) {
                *abort = 1;
                if (err_flag) atomicExch(err_flag, DEV_WAIT_TIMEOUT);
                return false;
            }
        }
    }
}

// mbar_wait by a whole converged warp with one outcome for every lane, so that the
// warp-collective instructions after it (tcgen05.ld / st, elect.sync issue) run converged.
__device__ __forceinline__ bool mbar_wait_warp(uint32_t bar, uint32_t parity, volatile int *abort, int *err_flag) {
    return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort, err_flag));
}

// ---------------------------------------------------------------------- TMA -------
// 4-D tiled load of a box into shared memory, completing on `bar` (transaction bytes).
__device__ __forceinline__ void tma_load_4d(const CUtensorMap *map, uint32_t dst, uint32_t bar,
                                            int c0, int c1, int c2, int c3) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar)
        : "memory");
}
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Generic-proxy shared-memory writes become visible to the async proxy (TMA, tcgen05).
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ----------------------------------------------------------------- tcgen05 --------
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc], kind::tf32, one CTA.
__device__ __forceinline__ void mma_tf32_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem desc], kind::tf32, one CTA.
__device__ __forceinline__ void mma_tf32_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrive once on `bar` when every tcgen05 op this thread issued so far has completed.
__device__ __forceinline__ void tc_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     bar)
                 : "memory");
}

// Warp-issued forms: all 32 lanes of a converged warp call these with the same arguments and
// one lane (elect.sync) issues. Measured on B200 (one CTA per SM, kind::tf32, M = 128): a
// converged warp issues back-to-back MMAs at the tensor core's own rate (about 18 cycles at
// N = 32, 33 at N = 64, N/2 beyond), while a single lane inside a divergent branch
// (`if (lane == 0)`) needs about 46 cycles per MMA whatever N.
__device__ __forceinline__ void mma_tf32_ts_w(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                              uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred e, p;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void mma_tf32_ss_w(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                              uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred e, p;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void tc_commit_w(uint32_t bar) {
    asm volatile(
        "{\n\t.reg .pred e;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(bar)
        : "memory");
}

#define DC_TMEM_REGS32(r)                                                                       \
    "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),         \
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), \
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),           \
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),           \
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
#define DC_TMEM_IN32(r)                                                                     \
    "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),   \
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),     \
        "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),   \
        "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),   \
        "r"(r[29]), "r"(r[30]), "r"(r[31])

// 32 consecutive 32-bit columns of this thread's TMEM lane (warp w reads lanes 32w..32w+31).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
        "%28, %29, %30, %31}, [%32];"
        : DC_TMEM_REGS32(r)
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
        "%28, %29, %30, %31, %32};" ::"r"(taddr),
        DC_TMEM_IN32(r)
        : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
        "%13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
        "%13, %14, %15, %16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
        "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// ------------------------------------------------------------- descriptors --------
// Instruction descriptor of kind::tf32 with fp32 accumulation (bit layout as in CUTLASS's
// UMMA::InstrDescriptor): c_format F32 [4,6), a/b_format TF32 [7,10)/[10,13), a/b major
// [15]/[16] (0 = K-major, 1 = MN-major), N>>3 [17,23), M>>4 [24,29).
__host__ __device__ constexpr uint32_t idesc_tf32(int M, int N, int a_mn_major, int b_mn_major) {
    return (1u << 4) | (2u << 7) | (2u << 10) | (uint32_t(a_mn_major) << 15) |
           (uint32_t(b_mn_major) << 16) | (uint32_t(N >> 3) << 17) | (uint32_t(M >> 4) << 24);
}

// Shared-memory matrix descriptor for a 128-byte-swizzled canonical layout: start address,
// leading / stride byte offsets (16-byte units), version 1 (sm_100), layout SWIZZLE_128B.
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr, uint32_t lbo_bytes,
                                                uint32_t sbo_bytes) {
    uint64_t d = 0;
    d |= uint64_t((saddr >> 4) & 0x3FFFu);
    d |= uint64_t((lbo_bytes >> 4) & 0x3FFFu) << 16;
    d |= uint64_t((sbo_bytes >> 4) & 0x3FFFu) << 32;
    d |= uint64_t(1) << 46;
    d |= uint64_t(2) << 61;
    return d;
}

// MN-major operands of 32-bit types (tf32) only take the 128-byte swizzle with 32-byte atoms
// (layout type 1, "SWIZZLE_128B_BASE32B"; a TMA load with CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B
// writes it): 128-byte rows along MN, 4-row K groups `sbo_bytes` apart, 32-element MN chunks
// `lbo_bytes` apart.
__device__ __forceinline__ uint64_t sdesc_mn_sw128_32b(uint32_t saddr, uint32_t lbo_bytes,
                                                       uint32_t sbo_bytes) {
    uint64_t d = sdesc_sw128(saddr, lbo_bytes, sbo_bytes);
    d &= ~(uint64_t(7) << 61);
    d |= uint64_t(1) << 61;
    return d;
}

// 2^x with the hardware approximation (MUFU.EX2, ~2 ulp, results below 2^-126 flushed to 0).
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// ---------------------------------------------------------------- TF32 ------------
// Round to the nearest TF32 value, ties away from zero (what cvt.rna.tf32.f32 computes): on
// the sign-magnitude encoding, add half a TF32 ulp (bit 12) to the magnitude and clear the 13
// low mantissa bits. A carry into the exponent gives the next power of two, as rounding
// should; +-Inf comes out unchanged, and so does every NaN with a payload bit above the 13 low
// bits (the quiet NaNs arithmetic produces). A NaN whose payload lies only in those bits turns
// into +-Inf here; its low part (x - hi) is NaN, so a 3xTF32 product still yields NaN. Two
// integer ops on the full-rate ALU pipe instead of a conversion instruction.
__device__ __forceinline__ uint32_t tf32_rna(float x) {
    return (__float_as_uint(x) + 0x1000u) & 0xFFFFE000u;
}

// The low part of a 3xTF32 split, lo = x - hi with hi = tf32_rna(x): exact in fp32 (at most
// 13 significant bits) and handed to the tensor core unrounded, which reads only its top 11
// significant bits. That truncation errs by less than 2^-10 of lo, below 2^-22 of x; as lo
// takes either sign (hi rounds to nearest), the errors do not accumulate in one direction.
// One FADD instead of a further round to nearest on the softmax warps' critical path.
__device__ __forceinline__ uint32_t tf32_lo(float x, uint32_t hi) {
    return __float_as_uint(x - __uint_as_float(hi));
}

// The 3xTF32 split with the high part truncated instead of rounded: hi = x itself (the
// tensor core reads only its top 19 bits, i.e. x with the 13 low mantissa bits cleared), lo =
// x minus that truncation, exact in fp32 and of x's sign, below one TF32 ulp of x. The tensor
// core truncates lo in turn, which errs by less than 2^-11 of lo (2^-21 of x) toward zero.
// One LOP and one FADD instead of the two integer ops of the rounding plus the FADD; used for
// the softmax warps' P and dS splits, where those ops sit on the critical path.
__device__ __forceinline__ uint32_t tf32_lo_trunc(float x) {
    return __float_as_uint(x - __uint_as_float(__float_as_uint(x) & 0xFFFFE000u));
}

}  // namespace sm100
}  // namespace dc
