// rng.cu -- dropout keep masks drawn from DenseCore's generator stream, in parallel.
//
// DenseCore's dropout (python/densecore/functional.py:229-244, :638-641) keeps element e when
// the e-th bernoulli draw of its CPU generator succeeds: PyTorch's mt19937
// (src/torch_random.rs:43-97) gives two 32-bit outputs per draw, random64 = (first << 32) |
// second, x = (random64 & (2^53 - 1)) * 2^-53 (:106-110), keep when x < 1 - p (:242-254).
// The draws of one call are consecutive outputs of that one stream, so a bit-exact mask on
// the GPU needs the stream at arbitrary offsets.
//
// The generator is linear over GF(2): writing X[k] for the k-th untempered state word
// (X[k + 624] = X[k + 397] ^ twist(X[k], X[k + 1])), every bit column of X[k], k >= 1, obeys
// the recurrence of the characteristic polynomial phi (degree 19937). If
// x^J = g(x) (mod phi) then X[b + J + w] = XOR over {i : g_i = 1} of X[b + i + w] for every
// window base b >= 1 -- the jump-ahead of Haramoto, Matsumoto, Nishimura, Panneton and
// L'Ecuyer, "Efficient jump ahead for F2-linear random number generators" (INFORMS J. on
// Computing 20(3), 2008). phi comes from Berlekamp-Massey on one bit column of the stream;
// the library computes it and the jump polynomials once per process on the host.
//
// Layout of a call (all indices relative to the first word of the given state block):
//   * pos = 625 - left is the next output; a seeded or fully used block (left == 1) is
//     twisted first, so the canonical block starts at B0 = 0 or 624 and pos >= B0;
//   * G = B0 + 624; chunk c >= 1 covers words [G + cJ, G + (c+1)J), chunk 0 covers
//     [pos, G + J) -- J = 624 * 1680 words, so every chunk start is a block start;
//   * a CTA owns the 32-element mask words whose first word lies in its chunk. CTA c >= 1
//     reaches its chunk start by at most two jumps (c = c1 * 32 + c0, tables x^(c0 J) and
//     x^(c1 32 J)), then generates 192 words per step in a 1024-word shared ring;
//   * the CTA whose chunk holds the block of the last consumed word writes the new state in
//     DenseCore's form (that block, left = 625 - next, next = words of it consumed).
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <string.h>

#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"
#include "kernels.h"
#include "sm100.cuh"

namespace dc {
namespace {

constexpr int MT_N = 624, MT_M = 397;
constexpr uint32_t MATRIX_A = 0x9908b0dfu, UMASK = 0x80000000u, LMASK = 0x7fffffffu;
constexpr int DEG = 19937;                  // degree of phi
constexpr int PW = (DEG + 63) / 64;         // 64-bit words of a reduced polynomial (312)
constexpr int64_t CHUNK = 624LL * 1680;     // words per chunk (1,048,320)
constexpr int LEVEL = 32;                   // chunk c = c1 * LEVEL + c0
constexpr int MAX_CHUNKS = LEVEL * LEVEL;
constexpr int RING = 1024;                  // shared ring of state words (power of two)
constexpr int STEP = 192;                   // words generated per step (6 warps; < 227)
constexpr int THREADS = 640;                // 624 jump accumulators, rounded up to warps

__host__ __device__ __forceinline__ int64_t imin(int64_t a, int64_t b) { return a < b ? a : b; }
__host__ __device__ __forceinline__ uint32_t twist(uint32_t u, uint32_t v) {
    return (((u & UMASK) | (v & LMASK)) >> 1) ^ ((v & 1u) ? MATRIX_A : 0u);
}
__host__ __device__ __forceinline__ uint32_t temper(uint32_t y) {
    y ^= y >> 11;
    y ^= (y << 7) & 0x9d2c5680u;
    y ^= (y << 15) & 0xefc60000u;
    y ^= y >> 18;
    return y;
}

// ------------------------------------------------------------------- host: GF(2)[x] ----

using Poly = std::vector<uint64_t>;

inline bool bit(const uint64_t *p, int64_t i) { return (p[i >> 6] >> (i & 63)) & 1u; }

// Minimal connection polynomial C (c_0 = 1) and its length L of the bit sequence s[0..n)
// (Berlekamp-Massey over GF(2)): s_k = XOR_{i=1..L} c_i s_{k-i} for k >= L.
int berlekamp_massey(const std::vector<uint8_t> &s, Poly &C) {
    const int64_t n = (int64_t)s.size();
    const int64_t W = n / 64 + 3;
    // R[j] = s[n - 1 - j], so s_{k-i} = R[n - 1 - k + i] and the discrepancy is the parity
    // of C AND (R >> (n - 1 - k)).
    Poly R(W + 1, 0), B(W, 0), T;
    C.assign(W, 0);
    for (int64_t j = 0; j < n; j++)
        if (s[n - 1 - j]) R[j >> 6] |= 1ull << (j & 63);
    C[0] = B[0] = 1;
    int64_t L = 0, m = 1;
    for (int64_t k = 0; k < n; k++) {
        const int64_t off = n - 1 - k;
        uint64_t acc = 0;
        for (int64_t w = 0; w <= L / 64; w++) {
            const int64_t bp = off + 64 * w, ww = bp >> 6, sh = bp & 63;
            uint64_t r = R[ww] >> sh;
            if (sh && ww + 1 <= W) r |= R[ww + 1] << (64 - sh);
            uint64_t c = C[w];
            if (w == L / 64 && ((L + 1) & 63)) c &= (1ull << ((L + 1) & 63)) - 1;  // bits 0..L
            acc ^= c & r;
        }
        if (!(__builtin_popcountll(acc) & 1)) {
            m++;
            continue;
        }
        // C ^= B << m
        const bool grow = 2 * L <= k;
        if (grow) T = C;
        const int64_t ws = m >> 6, bs = m & 63;
        for (int64_t w = W - 1; w >= ws; w--) {
            uint64_t v = B[w - ws] << bs;
            if (bs && w - ws - 1 >= 0) v |= B[w - ws - 1] >> (64 - bs);
            C[w] ^= v;
        }
        if (grow) {
            L = k + 1 - L;
            B.swap(T);
            m = 1;
        } else {
            m++;
        }
    }
    return (int)L;
}

struct Field {
    Poly phi;                // DEG + 1 bits
    std::vector<Poly> phs;   // phi << s, s = 0..63 (PW + 2 words each)

    // p (up to 2 DEG - 1 bits, any length) reduced mod phi into PW words.
    Poly reduce(Poly p) const {
        const int64_t top = (int64_t)p.size() * 64 - 1;
        for (int64_t k = top; k >= DEG; k--) {
            if (!bit(p.data(), k)) continue;
            const int64_t sft = k - DEG, w = sft >> 6;
            const Poly &q = phs[sft & 63];
            for (int j = 0; j < PW + 2 && w + j < (int64_t)p.size(); j++) p[w + j] ^= q[j];
        }
        p.resize(PW);
        return p;
    }
    Poly mul(const Poly &a, const Poly &b) const {
        std::vector<Poly> bs(64, Poly(PW + 1, 0));
        for (int s = 0; s < 64; s++)
            for (int k = 0; k <= PW; k++)
                bs[s][k] = (k < PW ? b[k] << s : 0) | (s && k > 0 ? b[k - 1] >> (64 - s) : 0);
        Poly prod(2 * PW + 2, 0);
        for (int64_t i = 0; i < DEG; i++) {
            if (!bit(a.data(), i)) continue;
            const int64_t w = i >> 6;
            const Poly &q = bs[i & 63];
            for (int k = 0; k <= PW; k++) prod[w + k] ^= q[k];
        }
        return reduce(std::move(prod));
    }
    Poly sqr(const Poly &a) const {
        Poly prod(2 * PW + 2, 0);
        for (int64_t i = 0; i < DEG; i++)
            if (bit(a.data(), i)) prod[(2 * i) >> 6] |= 1ull << ((2 * i) & 63);
        return reduce(std::move(prod));
    }
    // x^e mod phi by square-and-multiply.
    Poly powx(uint64_t e) const {
        Poly r(PW, 0);
        r[0] = 1;
        bool started = false;
        for (int b = 63; b >= 0; b--) {
            if (started) r = sqr(r);
            if ((e >> b) & 1u) {
                started = true;
                Poly t(PW + 1, 0);
                for (int k = 0; k <= PW; k++) t[k] = (k < PW ? r[k] << 1 : 0) | (k > 0 ? r[k - 1] >> 63 : 0);
                r = reduce(std::move(t));
            }
        }
        return r;
    }
};

struct JumpTables {
    bool ok = false;
    std::string error;
    Field f;
    std::vector<uint64_t> t0, t1;  // LEVEL polynomials of PW words: x^(c0 J), x^(c1 LEVEL J)
};

// The state words of a seeded generator (torch_random.rs:43-56), then enough outputs of its
// stream for Berlekamp-Massey.
void seed_block(uint64_t seed, uint32_t *st) {
    st[0] = (uint32_t)seed;
    for (uint32_t j = 1; j < MT_N; j++) st[j] = 1812433253u * (st[j - 1] ^ (st[j - 1] >> 30)) + j;
}

const JumpTables &tables() {
    static JumpTables T;
    static std::once_flag once;
    std::call_once(once, [] {
        // Bit 0 of X[k], k = 624 .. 624 + 2 DEG + 64, for the default seed.
        const int64_t n = 2 * DEG + 64;
        std::vector<uint32_t> X(MT_N + n);
        seed_block(67280421310721ull, X.data());
        for (int64_t k = MT_N; k < MT_N + n; k++)
            X[k] = X[k - MT_N + MT_M] ^ twist(X[k - MT_N], X[k - MT_N + 1]);
        std::vector<uint8_t> s(n);
        for (int64_t k = 0; k < n; k++) s[k] = X[MT_N + k] & 1u;
        Poly C;
        const int L = berlekamp_massey(s, C);
        if (L != DEG) {
            T.error = "generator jump tables: linear complexity " + std::to_string(L) + ", expected 19937";
            return;
        }
        // phi_j = c_{L-j}
        Poly phi(PW + 1, 0);
        for (int j = 0; j <= DEG; j++)
            if (bit(C.data(), DEG - j)) phi[j >> 6] |= 1ull << (j & 63);
        if (!(phi[0] & 1u)) {
            T.error = "generator jump tables: characteristic polynomial has no constant term";
            return;
        }
        T.f.phi = phi;
        T.f.phs.assign(64, Poly(PW + 2, 0));
        for (int sft = 0; sft < 64; sft++)
            for (int k = 0; k < PW + 2; k++) {
                uint64_t v = (k <= PW ? phi[k] << sft : 0);
                if (sft && k > 0 && k - 1 <= PW) v |= phi[k - 1] >> (64 - sft);
                T.f.phs[sft][k] = v;
            }
        T.t0.assign((size_t)LEVEL * PW, 0);
        T.t1.assign((size_t)LEVEL * PW, 0);
        Poly one(PW, 0);
        one[0] = 1;
        std::vector<Poly> a(LEVEL), b(LEVEL);
        a[0] = b[0] = one;
        a[1] = T.f.powx((uint64_t)CHUNK);
        for (int c = 2; c < LEVEL; c++) a[c] = T.f.mul(a[c - 1], a[1]);
        b[1] = T.f.mul(a[LEVEL - 1], a[1]);
        for (int c = 2; c < LEVEL; c++) b[c] = T.f.mul(b[c - 1], b[1]);
        for (int c = 0; c < LEVEL; c++) {
            memcpy(&T.t0[(size_t)c * PW], a[c].data(), PW * 8);
            memcpy(&T.t1[(size_t)c * PW], b[c].data(), PW * 8);
        }
        T.ok = true;
    });
    return T;
}

// ------------------------------------------------------------ host: the same walk ----
// A CPU restatement of the device walk, used by dc_rng_skip: the state after `words`
// outputs, found by jumping to the chunk of the last consumed word.

struct HostStream {
    std::vector<uint32_t> x;  // x[i] = X[base + i]
    int64_t base = 0;
    uint32_t at(int64_t k) const { return x[k - base]; }
    void extend_to(int64_t end) {  // X[.., end)
        while (base + (int64_t)x.size() < end) {
            const int64_t k = base + (int64_t)x.size();
            x.push_back(at(k - MT_N + MT_M) ^ twist(at(k - MT_N), at(k - MT_N + 1)));
        }
    }
    // Replace by the window at base + (jump of g), keeping nothing else.
    void jump(const uint64_t *g, int64_t dist) {
        extend_to(base + DEG + MT_N);
        std::vector<uint32_t> acc(MT_N, 0);
        for (int i = 0; i < DEG; i++)
            if (bit(g, i))
                for (int w = 0; w < MT_N; w++) acc[w] ^= x[i + w];
        x = acc;
        base += dist;
    }
};

}  // namespace

// ------------------------------------------------------------------------ device ----

namespace {

struct KeepArgs {
    const uint32_t *st_in;
    uint32_t *st_out;
    const uint64_t *t0, *t1;
    uint16_t *bits16;   // mask words as 16-bit halves (little-endian)
    int64_t n;          // elements
    int64_t nmask;      // 32-element mask words
    uint64_t thresh;    // keep when (random64 & (2^53 - 1)) < thresh
    int *err;           // the library's device error word
};

// Generates X[P, P + cnt) into the ring (cnt <= STEP), threads 0..cnt-1.
__device__ __forceinline__ void gen_step(uint32_t *ring, int64_t P, int cnt) {
    const int t = threadIdx.x;
    if (t < cnt) {
        const int64_t k = P + t;
        ring[k & (RING - 1)] =
            ring[(k - MT_N + MT_M) & (RING - 1)] ^ twist(ring[(k - MT_N) & (RING - 1)], ring[(k - MT_N + 1) & (RING - 1)]);
    }
}

// Jumps the window X[b, b + 624) in the ring (P == b + 624 on entry) by the polynomial g:
// on return the ring holds X[b + dist, b + dist + 624) and P == b + dist + 624.
__device__ void jump_window(uint32_t *ring, const uint64_t *__restrict__ g, int64_t &b, int64_t &P, int64_t dist) {
    const int w = threadIdx.x;
    uint32_t acc = 0;
    for (int j = 0; j * STEP < DEG; j++) {
        gen_step(ring, P, STEP);
        P += STEP;
        __syncthreads();
        if (w < MT_N) {
            const int64_t i0 = b + (int64_t)j * STEP + w;
#pragma unroll
            for (int u = 0; u < STEP / 64; u++) {
                uint64_t gw = __ldg(g + (j * STEP) / 64 + u);
                while (gw) {
                    const int t = __ffsll((long long)gw) - 1;
                    gw &= gw - 1;
                    acc ^= ring[(i0 + 64 * u + t) & (RING - 1)];
                }
            }
        }
    }
    __syncthreads();
    b += dist;
    if (w < MT_N) ring[(b + w) & (RING - 1)] = acc;
    P = b + MT_N;
    __syncthreads();
}

__global__ void __launch_bounds__(THREADS) keep_bits_kernel(KeepArgs a) {
    __shared__ uint32_t ring[RING];
    const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
    const int c = blockIdx.x;

    const uint32_t left = a.st_in[MT_N];
    if (left == 0 || left > (uint32_t)MT_N) {  // not a state DenseCore's engine can be in
        if (c == 0 && threadIdx.x == 0) atomicExch(a.err, sm100::DEV_BAD_GENERATOR_STATE);
        return;
    }
    const int64_t pos = 625 - (int64_t)left;          // 1..624
    const int64_t B0 = pos == MT_N ? MT_N : 0;        // canonical block start
    const int64_t G = B0 + MT_N;
    const int64_t W = 2 * a.n;                        // words consumed
    const int64_t last = pos + W - 1;                 // last consumed word
    const int64_t E = B0 + MT_N * ((last - B0) / MT_N);  // its block
    const int64_t lo = c == 0 ? pos : G + c * CHUNK, hi = G + (c + 1) * CHUNK;
    // Owned mask words: first word pos + 64 q in [lo, hi).
    int64_t q = c == 0 ? 0 : (lo - pos + 63) / 64;
    int64_t q_end = (hi - pos + 63) / 64;
    if (q_end > a.nmask) q_end = a.nmask;
    const bool owns_end = (E < G ? 0 : (E - G) / CHUNK) == c;
    if (q >= q_end && !owns_end) return;  // uniform across the CTA

    for (int i = tid; i < MT_N; i += THREADS) ring[i] = a.st_in[i];
    __syncthreads();
    int64_t b = 0, P = MT_N;  // window X[b, b + 624), produced up to P
    if (c > 0) {
        while (P < G + MT_N) {  // the base window at G
            const int cnt = (int)imin(STEP, G + MT_N - P);
            gen_step(ring, P, cnt);
            P += cnt;
            __syncthreads();
        }
        b = G;
        const int c0 = c % LEVEL, c1 = c / LEVEL;
        if (c0) jump_window(ring, a.t0 + (size_t)c0 * PW, b, P, c0 * CHUNK);
        if (c1) jump_window(ring, a.t1 + (size_t)c1 * PW, b, P, (int64_t)c1 * LEVEL * CHUNK);
    }
    bool captured = !owns_end;
    while (q < q_end || !captured) {
        gen_step(ring, P, STEP);
        P += STEP;
        __syncthreads();
        // Up to three mask words whose 64 words are produced.
        int64_t ready = (P - (pos + 64 * q)) / 64;
        int cnt = (int)imin(imin(3, q_end - q), ready);
        if (cnt < 0) cnt = 0;
        if (warp < 2 * cnt) {
            const int64_t qq = q + warp / 2, half = warp & 1;
            const uint32_t y = temper(ring[(pos + 64 * qq + 32 * half + lane) & (RING - 1)]);
            const uint32_t nxt = __shfl_down_sync(0xffffffffu, y, 1);
            const int64_t e = 32 * qq + 16 * half + lane / 2;
            const uint64_t m = ((uint64_t)(y & 0x1fffffu) << 32) | nxt;
            const bool keep = !(lane & 1) && e < a.n && m < a.thresh;
            uint32_t x = __ballot_sync(0xffffffffu, keep) & 0x55555555u;
            x = (x | (x >> 1)) & 0x33333333u;
            x = (x | (x >> 2)) & 0x0f0f0f0fu;
            x = (x | (x >> 4)) & 0x00ff00ffu;
            x = (x | (x >> 8)) & 0x0000ffffu;
            if (lane == 0) a.bits16[2 * qq + half] = (uint16_t)x;
        }
        q += cnt;
        if (!captured && P >= E + MT_N) {
            for (int i = tid; i < MT_N; i += THREADS) a.st_out[i] = ring[(E + i) & (RING - 1)];
            if (tid == 0) {
                const uint32_t next = (uint32_t)(last - E + 1);
                a.st_out[MT_N] = 625u - next;
                a.st_out[MT_N + 1] = next;
            }
            captured = true;
        }
    }
}

// Per-device copies of the jump tables.
constexpr int kTableDevices = 64;
std::mutex g_tab_mu;
uint64_t *g_tab_dev[kTableDevices];

int device_tables(const uint64_t **t0, const uint64_t **t1) {
    const JumpTables &T = tables();
    if (!T.ok) return fail(DC_ERR_RUNTIME, T.error);
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "dropout: current device");
    if (dev < 0 || dev >= kTableDevices)
        return fail(DC_ERR_UNSUPPORTED, "dropout: device ordinal " + std::to_string(dev) + " is above 63");
    std::lock_guard<std::mutex> lock(g_tab_mu);
    if (!g_tab_dev[dev]) {
        uint64_t *p = nullptr;
        const size_t bytes = 2 * (size_t)LEVEL * PW * 8;
        e = cudaMalloc(&p, bytes);
        if (e != cudaSuccess) return cuda_fail(e, "dropout: jump tables");
        e = cudaMemcpy(p, T.t0.data(), bytes / 2, cudaMemcpyHostToDevice);
        if (e == cudaSuccess) e = cudaMemcpy(p + (size_t)LEVEL * PW, T.t1.data(), bytes / 2, cudaMemcpyHostToDevice);
        if (e != cudaSuccess) {
            cudaFree(p);
            return cuda_fail(e, "dropout: jump tables upload");
        }
        g_tab_dev[dev] = p;
    }
    *t0 = g_tab_dev[dev];
    *t1 = g_tab_dev[dev] + (size_t)LEVEL * PW;
    return DC_OK;
}

}  // namespace

// Elements per launch: 1022 chunks of words (the two-level table reaches 1024 chunks; one
// chunk is lost to the head and one to the tail), rounded down to whole mask words.
constexpr int64_t kMaxElemsPerLaunch = ((MAX_CHUNKS - 2) * CHUNK / 2) / 32 * 32;

int keep_bits(const uint32_t *st_in, uint32_t *st_out, int64_t n, double keep_prob, uint32_t *bits,
              cudaStream_t stream) {
    if (!st_in || !st_out) return fail(DC_ERR_VALUE, "dropout: generator state pointers must not be null");
    if (n < 0) return fail(DC_ERR_VALUE, "dropout: negative element count");
    if (!(keep_prob >= 0.0 && keep_prob <= 1.0)) return fail(DC_ERR_VALUE, "dropout: keep probability must be in [0, 1]");
    if (n > 0 && !bits) return fail(DC_ERR_VALUE, "dropout: mask pointer must not be null");
    if ((reinterpret_cast<uintptr_t>(bits) & 3u) != 0)
        return fail(DC_ERR_VALUE, "dropout: mask words must be 4-byte aligned");
    if (n == 0) {
        if (st_out == st_in) return DC_OK;
        cudaError_t e = cudaMemcpyAsync(st_out, st_in, (MT_N + 2) * 4, cudaMemcpyDeviceToDevice, stream);
        return e == cudaSuccess ? DC_OK : cuda_fail(e, "dropout: state copy");
    }
    const uint64_t *t0 = nullptr, *t1 = nullptr;
    int st = device_tables(&t0, &t1);
    if (st) return st;
    int *err = device_error_word();
    if (!err) return fail(DC_ERR_CUDA, "device error word is unavailable");
    // keep iff m * 2^-53 < keep_prob  <=>  m < ceil(keep_prob * 2^53) (the scaling is exact)
    const uint64_t thresh = (uint64_t)ceil(keep_prob * 9007199254740992.0);
    const int64_t launches = (n + kMaxElemsPerLaunch - 1) / kMaxElemsPerLaunch;
    uint32_t *tmp = nullptr;
    if (launches > 1 || st_out == st_in) {
        st = pool_alloc(reinterpret_cast<void **>(&tmp), 2 * (MT_N + 2) * 4, stream);
        if (st) return st;
    }
    const uint32_t *src = st_in;
    for (int64_t l = 0; l < launches; l++) {
        const int64_t e0 = l * kMaxElemsPerLaunch, ne = imin(kMaxElemsPerLaunch, n - e0);
        uint32_t *dst = l == launches - 1 && st_out != st_in ? st_out : tmp + (l & 1) * (MT_N + 2);
        KeepArgs a{src, dst, t0, t1, reinterpret_cast<uint16_t *>(bits + e0 / 32), ne, (ne + 31) / 32, thresh, err};
        const int64_t grid = 2 + (2 * ne - 1) / CHUNK;
        keep_bits_kernel<<<(unsigned)grid, THREADS, 0, stream>>>(a);
        st = check_launch("dropout keep bits");
        if (st) {
            pool_free(tmp, stream);
            return st;
        }
        src = dst;
    }
    if (st_out == st_in) {
        cudaError_t e = cudaMemcpyAsync(st_out, src, (MT_N + 2) * 4, cudaMemcpyDeviceToDevice, stream);
        if (e != cudaSuccess) {
            pool_free(tmp, stream);
            return cuda_fail(e, "dropout: state copy");
        }
    }
    pool_free(tmp, stream);
    return DC_OK;
}

// CPU: the state after `outputs` 32-bit outputs, by the same chunked walk.
int rng_skip(const uint32_t *st_in, uint64_t outputs, uint32_t *st_out) {
    if (!st_in || !st_out) return fail(DC_ERR_VALUE, "generator skip: state pointers must not be null");
    const uint32_t left = st_in[MT_N], next = st_in[MT_N + 1];
    if (left == 0 || left > (uint32_t)MT_N || next > (uint32_t)MT_N)
        return fail(DC_ERR_VALUE, "generator skip: invalid generator state");
    if (outputs == 0) {
        if (st_out != st_in) memmove(st_out, st_in, (MT_N + 2) * 4);
        return DC_OK;
    }
    if (outputs > (1ull << 36)) return fail(DC_ERR_VALUE, "generator skip: more than 2^36 outputs");
    const JumpTables &T = tables();
    if (!T.ok) return fail(DC_ERR_RUNTIME, T.error);
    const int64_t pos = 625 - (int64_t)left;
    const int64_t B0 = pos == MT_N ? MT_N : 0, G = B0 + MT_N;
    const int64_t last = pos + (int64_t)outputs - 1;
    const int64_t E = B0 + MT_N * ((last - B0) / MT_N);
    const int64_t c = E < G ? 0 : (E - G) / CHUNK;
    HostStream s;
    s.x.assign(st_in, st_in + MT_N);
    if (c > 0) {
        s.extend_to(G + MT_N);
        s.x.erase(s.x.begin(), s.x.begin() + (G - s.base));
        s.x.resize(MT_N);
        s.base = G;
        int64_t cc = c;
        while (cc > 0) {  // chunks beyond one table reach walk in steps of the largest jump
            const int64_t step = cc >= (int64_t)MAX_CHUNKS ? (int64_t)(LEVEL - 1) * LEVEL : cc;
            const int64_t c0 = step % LEVEL, c1 = step / LEVEL;
            if (c0) s.jump(&T.t0[(size_t)c0 * PW], c0 * CHUNK);
            if (c1) s.jump(&T.t1[(size_t)c1 * PW], c1 * LEVEL * CHUNK);
            cc -= step;
        }
    }
    s.extend_to(E + MT_N);
    for (int i = 0; i < MT_N; i++) st_out[i] = s.at(E + i);
    const uint32_t nx = (uint32_t)(last - E + 1);
    st_out[MT_N] = 625u - nx;
    st_out[MT_N + 1] = nx;
    return DC_OK;
}

}  // namespace dc
