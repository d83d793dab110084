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
//     [pos, G + J) -- J = 624 * 840 words, so every chunk start is a block start;
//   * a CTA owns the 32-element mask words whose first word lies in its chunk. CTA c >= 1
//     reaches its chunk start by one jump with x^(c J) mod phi (a table computed on the host
//     as needed, 2048 entries at most), then generates 224 words per phase in a mirrored
//     2048-word shared ring while other warps turn earlier words into keep bits;
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
#include "trace.h"

namespace dc {
namespace {

constexpr int MT_N = 624, MT_M = 397;
constexpr uint32_t MATRIX_A = 0x9908b0dfu, UMASK = 0x80000000u, LMASK = 0x7fffffffu;
constexpr int DEG = 19937;                  // degree of phi
constexpr int PW = (DEG + 63) / 64;         // 64-bit words of a reduced polynomial (312)
constexpr int64_t CHUNK = 624LL * 840;      // words per chunk (524,160)
constexpr int MAX_CHUNKS = 2048;            // jump table entries x^(c J), c < MAX_CHUNKS
constexpr int RING = 2048;                  // shared ring of state words (power of two)
constexpr int GEN_WARPS = 7;                // warps generating the stream
constexpr int STEP = GEN_WARPS * 32;        // words generated per phase (224 <= 624 - 397)
constexpr int CONV_WARPS = 4;               // warps turning words into keep bits
constexpr int THREADS = (GEN_WARPS + CONV_WARPS) * 32;
constexpr int JW = 4;                       // window words per thread in a jump (156 threads)
static_assert(MT_N + 2 * STEP <= RING, "a jump phase must not overwrite words still being read");

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

// dst ^= src << sh (bits), over dst's words.
void xor_shifted(Poly &dst, const Poly &src, int64_t sh) {
    const int64_t ws = sh >> 6, bs = sh & 63;
    for (int64_t k = 0; k < (int64_t)src.size(); k++) {
        if (ws + k < (int64_t)dst.size()) dst[ws + k] ^= src[k] << bs;
        if (bs && ws + k + 1 < (int64_t)dst.size()) dst[ws + k + 1] ^= src[k] >> (64 - bs);
    }
}

uint32_t byte_at(const Poly &p, int64_t pos) {
    const int64_t w = pos >> 6, b = pos & 63;
    uint64_t v = p[w] >> b;
    if (b > 56 && w + 1 < (int64_t)p.size()) v |= p[w + 1] << (64 - b);
    return (uint32_t)(v & 0xffu);
}

// Arithmetic in GF(2)[x] / phi, eight coefficients at a time.
struct Field {
    Poly phi;                   // DEG + 1 bits
    // red[(o * 256 + t) * (PW + 1)]: the multiple q * phi (deg q < 8) whose coefficients
    // DEG .. DEG + 7 are the byte t, shifted left by 8 o bits. XORed in at word s / 8 it clears
    // coefficients DEG + 8 s .. DEG + 8 s + 7 of a product (o = s % 8).
    std::vector<uint64_t> red;

    void init(const Poly &phi_) {
        phi = phi_;
        red.assign((size_t)8 * 256 * (PW + 1), 0);
        for (int q = 0; q < 256; q++) {
            Poly m(PW + 2, 0);
            for (int i = 0; i < 8; i++)
                if ((q >> i) & 1) xor_shifted(m, phi, i);
            const uint32_t t = byte_at(m, DEG);  // a bijection of q (phi is monic)
            for (int o = 0; o < 8; o++) {
                Poly sh(PW + 2, 0);
                xor_shifted(sh, m, 8 * o);
                memcpy(&red[((size_t)o * 256 + t) * (PW + 1)], sh.data(), (PW + 1) * 8);
            }
        }
    }
    // p (2 PW + 2 words, degree <= 2 DEG - 2) reduced mod phi into PW words.
    Poly reduce(Poly p) const {
        p.resize(2 * PW + 2, 0);
        for (int64_t s = (DEG - 2) / 8; s >= 0; s--) {
            const uint32_t t = byte_at(p, DEG + 8 * s);
            if (!t) continue;
            const uint64_t *m = &red[((size_t)(s & 7) * 256 + t) * (PW + 1)];
            uint64_t *d = p.data() + (s >> 3);
            for (int j = 0; j <= PW; j++) d[j] ^= m[j];
        }
        p.resize(PW);
        return p;
    }
    Poly mul(const Poly &a, const Poly &b) const {
        Poly prod(2 * PW + 2, 0);
        std::vector<uint64_t> tab((size_t)256 * (PW + 1));
        for (int o = 0; o < 8; o++) {
            // tab[v] = (b * v) << 8 o for every byte v
            std::fill(tab.begin(), tab.begin() + (PW + 1), 0ull);
            for (int i = 0; i < 8; i++) {
                Poly sh(PW + 1, 0);
                xor_shifted(sh, b, 8 * o + i);
                memcpy(&tab[((size_t)1 << i) * (PW + 1)], sh.data(), (PW + 1) * 8);
            }
            for (int v = 3; v < 256; v++) {
                if (!(v & (v - 1))) continue;
                const uint64_t *x = &tab[(size_t)(v & (v - 1)) * (PW + 1)], *y = &tab[(size_t)(v & -v) * (PW + 1)];
                uint64_t *z = &tab[(size_t)v * (PW + 1)];
                for (int j = 0; j <= PW; j++) z[j] = x[j] ^ y[j];
            }
            for (int w = 0; w < PW; w++) {
                const uint32_t v = (uint32_t)(a[w] >> (8 * o)) & 0xffu;
                if (!v) continue;
                const uint64_t *m = &tab[(size_t)v * (PW + 1)];
                for (int j = 0; j <= PW; j++) prod[w + j] ^= m[j];
            }
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

// x^(c J) mod phi for c = 0 .. count - 1, PW words each, grown on demand. Storage for all
// MAX_CHUNKS entries is reserved up front, so entries never move once written.
struct JumpTables {
    bool ok = false;
    std::string error;
    Field f;
    std::mutex mu;
    std::vector<uint64_t> t;
    int count = 0;
};

// The state words of a seeded generator (torch_random.rs:43-56).
void seed_block(uint64_t seed, uint32_t *st) {
    st[0] = (uint32_t)seed;
    for (uint32_t j = 1; j < MT_N; j++) st[j] = 1812433253u * (st[j - 1] ^ (st[j - 1] >> 30)) + j;
}

JumpTables &tables() {
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
        T.f.init(phi);
        T.t.assign((size_t)MAX_CHUNKS * PW, 0);
        T.t[0] = 1;  // x^0
        T.count = 1;
        T.ok = true;
    });
    return T;
}

// Makes entries 0 .. need - 1 (need <= MAX_CHUNKS) available; returns the table.
const uint64_t *table_upto(JumpTables &T, int need) {
    std::lock_guard<std::mutex> lock(T.mu);
    while (T.count < need) {
        const int c = T.count;
        Poly r = c == 1 ? T.f.powx((uint64_t)CHUNK)
                        : T.f.mul(Poly(T.t.begin() + (size_t)(c - 1) * PW, T.t.begin() + (size_t)c * PW),
                                  Poly(T.t.begin() + PW, T.t.begin() + 2 * PW));
        memcpy(&T.t[(size_t)c * PW], r.data(), PW * 8);
        T.count = c + 1;
    }
    return T.t.data();
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
    const uint32_t *tab;  // x^(c J) mod phi, 2 PW 32-bit words per c
    uint32_t *bits;       // mask words
    int64_t n;            // elements
    int64_t nmask;        // 32-element mask words
    uint64_t thresh;      // keep when (random64 & (2^53 - 1)) < thresh
    int *err;             // the library's device error word
};

// Generates X[P, P + cnt) (cnt <= STEP) into both copies of the ring, threads 0..cnt-1. Ring
// slot k % RING and its mirror RING + k % RING hold X[k], so a run of up to RING words read
// from any slot below RING needs no wrap-around. Slot arithmetic is 32-bit (RING divides 2^32).
__device__ __forceinline__ void gen_step(uint32_t *ring, uint32_t P, int cnt) {
    const int t = threadIdx.x;
    if (t < cnt) {
        const uint32_t k = P + t;
        const uint32_t v = ring[(k - MT_N + MT_M) & (RING - 1)] ^
                           twist(ring[(k - MT_N) & (RING - 1)], ring[(k - MT_N + 1) & (RING - 1)]);
        ring[k & (RING - 1)] = v;
        ring[(k & (RING - 1)) + RING] = v;
    }
}

// Jumps the window X[b, b + 624) in the ring (P == b + 624 on entry) by the polynomial g
// (DEG bits in 2 PW 32-bit words): on return the ring holds X[b + dist, b + dist + 624) and
// P == b + dist + 624. Thread t < 156 accumulates window words t + 156 d, d < 4 (a warp reads
// consecutive words: no bank conflicts), two set bits of g per loop turn.
__device__ void jump_window(uint32_t *ring, const uint32_t *__restrict__ g, int64_t &b, int64_t &P, int64_t dist) {
    const int tid = threadIdx.x;
    constexpr int NT = MT_N / JW;
    uint32_t acc[JW] = {0u, 0u, 0u, 0u};
    const uint32_t b32 = (uint32_t)b;
    for (int j = 0; j * STEP < DEG; j++) {
        gen_step(ring, (uint32_t)P, STEP);
        P += STEP;
        __syncthreads();
        if (tid < NT) {
            // X[b + STEP j + i + w], i < STEP, w < 624: all below P and held (624 + 2 STEP <= RING).
            const uint32_t *p = ring + ((b32 + (uint32_t)(j * STEP)) & (RING - 1)) + tid;
#pragma unroll
            for (int u = 0; u < STEP / 32; u++) {
                const int gi = j * (STEP / 32) + u;
                uint32_t gw = gi < 2 * PW ? __ldg(g + gi) : 0u;
                while (gw) {
                    const int t1 = __ffs(gw) - 1;
                    gw &= gw - 1;
                    const int t2 = gw ? __ffs(gw) - 1 : t1;
                    const uint32_t m2 = gw ? ~0u : 0u;
                    gw &= gw - 1;
                    const uint32_t *r1 = p + 32 * u + t1, *r2 = p + 32 * u + t2;
#pragma unroll
                    for (int d = 0; d < JW; d++) acc[d] ^= r1[NT * d] ^ (r2[NT * d] & m2);
                }
            }
        }
    }
    __syncthreads();
    b += dist;
    if (tid < NT) {
#pragma unroll
        for (int d = 0; d < JW; d++) {
            const uint32_t k = ((uint32_t)b + tid + NT * d) & (RING - 1);
            ring[k] = acc[d];
            ring[k + RING] = acc[d];
        }
    }
    P = b + MT_N;
    __syncthreads();
}

// Warps 0..6 generate the stream, STEP words per phase; warps 7..10 turn words produced in
// earlier phases into keep bits (one element per lane, one 32-bit mask word per warp) and
// copy out the end state, so conversion overlaps generation.
__global__ void __launch_bounds__(THREADS) keep_bits_kernel(KeepArgs a) {
    __shared__ uint32_t ring[2 * RING];
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

    for (int i = tid; i < MT_N; i += THREADS) ring[i] = ring[i + RING] = a.st_in[i];
    __syncthreads();
    int64_t b = 0, P = MT_N;  // window X[b, b + 624), produced up to P
    if (c > 0) {
        while (P < G + MT_N) {  // the base window at G
            const int cnt = (int)imin(STEP, G + MT_N - P);
            gen_step(ring, (uint32_t)P, cnt);
            P += cnt;
            __syncthreads();
        }
        b = G;
        jump_window(ring, a.tab + (size_t)c * 2 * PW, b, P, c * CHUNK);
    }
    // Every phase: words below P are visible; generation writes X[P, P + STEP) over the slots
    // of X[P - RING, P - RING + STEP), while conversion reads at or above pos + 64 q >= P - 624
    // and the end-state copy at or above E > P - 624 - STEP.
    bool captured = !owns_end;
    while (q < q_end || !captured) {
        const int64_t ready = (P - (pos + 64 * q)) / 64;  // mask words whose words are all below P
        int cnt = (int)imin(imin(CONV_WARPS, q_end - q), ready);
        if (cnt < 0) cnt = 0;
        const bool capture = !captured && P >= E + MT_N;
        if (warp < GEN_WARPS) {
            gen_step(ring, (uint32_t)P, STEP);
        } else {
            const int cw = warp - GEN_WARPS;
            if (cw < cnt) {
                const int64_t e = 32 * (q + cw) + lane;
                const uint32_t k = (uint32_t)(pos + 2 * e) & (RING - 1);
                const uint32_t hi32 = temper(ring[k]), lo32 = temper(ring[k + 1]);  // k + 1 < 2 RING
                const uint64_t m = ((uint64_t)(hi32 & 0x1fffffu) << 32) | lo32;
                const uint32_t word = __ballot_sync(0xffffffffu, e < a.n && m < a.thresh);
                if (lane == 0) a.bits[q + cw] = word;
            }
            if (capture) {
                const int ct = tid - GEN_WARPS * 32;
                for (int i = ct; i < MT_N; i += THREADS - GEN_WARPS * 32)
                    a.st_out[i] = ring[((uint32_t)E + i) & (RING - 1)];
                if (ct == 0) {
                    const uint32_t next = (uint32_t)(last - E + 1);
                    a.st_out[MT_N] = 625u - next;
                    a.st_out[MT_N + 1] = next;
                }
            }
        }
        __syncthreads();
        P += STEP;
        q += cnt;
        captured = captured || capture;
    }
}

// Per-device copies of the jump table (MAX_CHUNKS entries reserved, filled on demand).
constexpr int kTableDevices = 64;
std::mutex g_tab_mu;
uint64_t *g_tab_dev[kTableDevices];
int g_tab_count[kTableDevices];

int device_table(int need, const uint32_t **tab) {
    JumpTables &T = tables();
    if (!T.ok) return fail(DC_ERR_RUNTIME, T.error);
    const uint64_t *host = table_upto(T, need);
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "dropout: current device");
    if (dev < 0 || dev >= kTableDevices)
        return fail(DC_ERR_UNSUPPORTED, "dropout: device ordinal " + std::to_string(dev) + " is above 63");
    std::lock_guard<std::mutex> lock(g_tab_mu);
    if (!g_tab_dev[dev]) {
        uint64_t *p = nullptr;
        e = cudaMalloc(&p, (size_t)MAX_CHUNKS * PW * 8);
        if (e != cudaSuccess) return cuda_fail(e, "dropout: jump table");
        g_tab_dev[dev] = p;
    }
    if (g_tab_count[dev] < need) {
        // Entries below the old count may be in use by launches in flight; only new ones are
        // written.
        const size_t from = (size_t)g_tab_count[dev] * PW;
        e = cudaMemcpy(g_tab_dev[dev] + from, host + from, ((size_t)need * PW - from) * 8, cudaMemcpyHostToDevice);
        if (e != cudaSuccess) return cuda_fail(e, "dropout: jump table upload");
        g_tab_count[dev] = need;
    }
    *tab = reinterpret_cast<const uint32_t *>(g_tab_dev[dev]);
    return DC_OK;
}

}  // namespace

// Elements per launch: MAX_CHUNKS - 2 chunks of words (one chunk may be taken by the head and
// one by the tail), rounded down to whole mask words.
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
    const int64_t launches = (n + kMaxElemsPerLaunch - 1) / kMaxElemsPerLaunch;
    const int64_t first = imin(kMaxElemsPerLaunch, n);
    const uint32_t *tab = nullptr;
    int st = device_table((int)(2 + (2 * first - 1) / CHUNK), &tab);
    if (st) return st;
    int *err = device_error_word();
    if (!err) return fail(DC_ERR_CUDA, "device error word is unavailable");
    // keep iff m * 2^-53 < keep_prob  <=>  m < ceil(keep_prob * 2^53) (the scaling is exact)
    const uint64_t thresh = (uint64_t)ceil(keep_prob * 9007199254740992.0);
    uint32_t *tmp = nullptr;
    if (launches > 1 || st_out == st_in) {
        st = pool_alloc(reinterpret_cast<void **>(&tmp), 2 * (MT_N + 2) * 4, stream);
        if (st) return st;
    }
    const uint32_t *src = st_in;
    for (int64_t l = 0; l < launches; l++) {
        const int64_t e0 = l * kMaxElemsPerLaunch, ne = imin(kMaxElemsPerLaunch, n - e0);
        uint32_t *dst = l == launches - 1 && st_out != st_in ? st_out : tmp + (l & 1) * (MT_N + 2);
        KeepArgs a{src, dst, tab, bits + e0 / 32, ne, (ne + 31) / 32, thresh, err};
        const int64_t grid = 2 + (2 * ne - 1) / CHUNK;
        {
            KernelTrace tr("dropout_keep_bits", stream);
            keep_bits_kernel<<<(unsigned)grid, THREADS, 0, stream>>>(a);
        }
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
    JumpTables &T = tables();
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
        while (cc > 0) {  // beyond the table, chain its largest jump
            const int step = (int)imin(cc, MAX_CHUNKS - 1);
            const uint64_t *tab = table_upto(T, step + 1);
            s.jump(tab + (size_t)step * PW, step * CHUNK);
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
