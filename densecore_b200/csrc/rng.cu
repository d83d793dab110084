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
//     [pos, G + J) -- J = 624 * 210 words, so every chunk start is a block start;
//   * the chunks are split into contiguous runs, one per CTA (at most one CTA per SM), and a
//     CTA owns the 32-element mask words whose first word lies in its run. A run that starts
//     at chunk c >= 1 is reached by one jump with x^(c J) mod phi (a table computed on the
//     host as needed, 2048 entries at most); the CTA then makes 576 words per phase in a
//     mirrored 8192-word shared ring (three words per thread, chained at distance 227), four
//     phases per CTA barrier, while other warps turn the words of the previous four phases
//     into keep bits;
//   * the CTA whose run holds the block of the last consumed word writes the new state in
//     DenseCore's form (that block, left = 625 - next, next = words of it consumed).
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <mutex>
#include <string>
#include <thread>
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
constexpr int64_t CHUNK = 624LL * 210;      // words per chunk (131,040): runs of chunks balance CTAs
constexpr int MAX_CHUNKS = 2048;            // jump table entries x^(c J), c < MAX_CHUNKS
constexpr int LAG = MT_N - MT_M;            // 227: X[k] = X[k - LAG] ^ twist(X[k - 624], X[k - 623])
constexpr int RING = 8192;                  // shared ring of state words (power of two), mirrored
constexpr int PHASE = 576;                  // words generated per barrier (nine 64-word mask words)
constexpr int GEN_WARPS = (LAG + 31) / 32;  // 8: thread t < LAG makes three chained words a phase
constexpr int NPH = 4;                      // phases per CTA barrier (the generating warps sync
constexpr int TURN = NPH * PHASE;           // among themselves between them): words per turn
constexpr int CONV_WARPS = PHASE / 64;      // 9: NPH mask words (one element per lane) a turn each
constexpr int WARPS = GEN_WARPS + CONV_WARPS;
constexpr int THREADS = WARPS * 32;         // 544
constexpr int JW = 2;                       // window words per thread in a jump
constexpr int JT = MT_N / JW;               // 312 threads accumulate a jump
constexpr int LIST_WARP = WARPS - 1;        // the warp that lists the nibbles of a jump block
// Dynamic shared memory, in 32-bit words: the mirrored ring, then the eleven jump tables (sums
// of two to four of four consecutive words, TABW each), then two lists of NIB 16-bit entries
// and their two counts.
constexpr int NIB = PHASE / 4;              // coefficient nibbles per jump block
constexpr int TABW = 1200;                  // >= 4 (NIB - 1) + MT_N: a table's words per block
constexpr int NTAB = 11;
constexpr int TAB0 = 2 * RING, LST0 = TAB0 + NTAB * TABW, CNT0 = LST0 + NIB;
constexpr int SMEM_WORDS = CNT0 + 2;
static_assert(SMEM_WORDS < 65536, "list entries are 16-bit word offsets");
static_assert(PHASE <= MT_N - 1 && PHASE - 2 * LAG <= MT_N - 1 - 2 * LAG,
              "a thread's third word must only read words made before the phase");
static_assert(PHASE % 64 == 0 && JT <= LIST_WARP * 32 && JT % 8 == 0, "warp roles");
static_assert(4 * (NIB - 1) + MT_N <= TABW && (LST0 % 2) == 0, "jump table layout");
static_assert(2 * PHASE + MT_N <= RING, "a jump phase must not overwrite words still being read");
static_assert(2 * TURN + MT_N <= RING, "a turn must not overwrite words still being read");

__host__ __device__ __forceinline__ int64_t imin(int64_t a, int64_t b) { return a < b ? a : b; }
__host__ __device__ __forceinline__ uint32_t twist(uint32_t u, uint32_t v) {
    // (v & 1) * MATRIX_A selects the constant with a multiply (the FMA pipe on the device; the
    // integer ALU pipe is the kernel's busiest)
    return (((u & UMASK) | (v & LMASK)) >> 1) ^ ((v & 1u) * MATRIX_A);
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
// Entries are x^(c J) = x^((c - 1) J) * x^J, one multiplication each (about a millisecond).
// Many new entries are shared out over host threads: each thread starts its range with
// x^(c0 J) by square-and-multiply and writes disjoint entries.
const uint64_t *table_upto(JumpTables &T, int need) {
    std::lock_guard<std::mutex> lock(T.mu);
    if (T.count >= need) return T.t.data();
    auto entry = [&](int c) { return Poly(T.t.begin() + (size_t)c * PW, T.t.begin() + (size_t)(c + 1) * PW); };
    auto store = [&](int c, const Poly &r) { memcpy(&T.t[(size_t)c * PW], r.data(), PW * 8); };
    if (T.count < 2) {
        store(1, T.f.powx((uint64_t)CHUNK));
        T.count = 2;
    }
    const int from = T.count, todo = need - from;
    if (todo <= 0) return T.t.data();
    const Poly xj = entry(1);
    auto run = [&](int a, int b) {  // entries [a, b)
        Poly cur = a - 1 < from ? T.f.mul(entry(a - 1), xj) : T.f.powx((uint64_t)a * (uint64_t)CHUNK);
        store(a, cur);
        for (int c = a + 1; c < b; c++) {
            cur = T.f.mul(cur, xj);
            store(c, cur);
        }
    };
    const unsigned hw = std::thread::hardware_concurrency();
    const int nth = (int)std::min<int64_t>({(int64_t)todo / 64, hw > 0 ? (int64_t)hw : 1, 16});
    if (nth <= 1) {
        run(from, need);
    } else {
        std::vector<std::thread> pool;
        for (int i = 0; i < nth; i++) {
            const int a = from + (int)((int64_t)todo * i / nth), b = from + (int)((int64_t)todo * (i + 1) / nth);
            if (a < b) pool.emplace_back(run, a, b);
        }
        for (auto &t : pool) t.join();
    }
    T.count = need;
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

// Writes X[k] into slot k % RING and its mirror RING + k % RING, so that a run of up to RING
// words read from any slot below RING needs no wrap-around. Slot arithmetic is 32-bit (RING
// divides 2^32).
__device__ __forceinline__ void put(uint32_t *ring, uint32_t k, uint32_t v) {
    const uint32_t s = k & (RING - 1);
    ring[s] = v;
    ring[s + RING] = v;
}

// Generates X[P, P + cnt), cnt <= PHASE, with every word below P already in the ring. Thread
// t < LAG makes the chain X[P + t], X[P + t + LAG], X[P + t + 2 LAG] (those below P + cnt):
// a chain word takes X[k - LAG] from the thread's previous word and X[k - 624], X[k - 623]
// from below P (t + 2 LAG < PHASE keeps the third word's operands there), so no thread reads
// a word made in the same phase by another thread, and all reads come before the writes.
__device__ __forceinline__ void gen_words(uint32_t *ring, uint32_t P, int cnt) {
    const int t = threadIdx.x;
    if (t >= LAG || t >= cnt) return;
    const uint32_t k = P + (uint32_t)t;
    const uint32_t *r = ring + (k & (RING - 1)) + RING;  // r[-d] = X[k - d], 0 < d <= RING
    const bool two = t + LAG < cnt, three = t + 2 * LAG < cnt;
    const uint32_t a0 = r[-LAG], a1 = r[-MT_N], a2 = r[-MT_N + 1];
    const uint32_t b1 = two ? r[LAG - MT_N] : 0u, b2 = two ? r[LAG - MT_N + 1] : 0u;
    const uint32_t c1 = three ? r[2 * LAG - MT_N] : 0u, c2 = three ? r[2 * LAG - MT_N + 1] : 0u;
    uint32_t x = a0 ^ twist(a1, a2);
    put(ring, k, x);
    if (two) {
        x ^= twist(b1, b2);
        put(ring, k + LAG, x);
        if (three) {
            x ^= twist(c1, c2);
            put(ring, k + 2 * LAG, x);
        }
    }
}

// Mask word q from the ring: element 32 q + lane uses the words k + 2 lane (high half of the
// 64-bit draw) and k + 2 lane + 1, where k = pos + 64 q and `slot` = k + 2 lane (mod 2^32).
__device__ __forceinline__ void load_pair(const uint32_t *ring, uint32_t slot, uint32_t &hi, uint32_t &lo) {
    const uint32_t s = slot & (RING - 1);
    hi = ring[s];
    lo = ring[s + 1];  // s + 1 <= RING: the mirror
}

// Stores mask word q from the untempered pair (hi, lo) of each lane. The draw is
// m = (temper(hi) & (2^21 - 1)) 2^32 + temper(lo), kept when m < thresh: the high 21 bits
// decide unless they equal those of thresh (probability 2^-21), so the low word is tempered
// only then. Elements past n are cleared in the last word. One warp, all lanes.
__device__ __forceinline__ void store_word(const KeepArgs &a, uint32_t hi, uint32_t lo, int64_t q, int lane) {
    const uint32_t th_hi = (uint32_t)(a.thresh >> 32), h = temper(hi) & 0x1fffffu;
    bool keep = h < th_hi;
    if (h == th_hi) keep = temper(lo) < (uint32_t)a.thresh;
    uint32_t word = __ballot_sync(0xffffffffu, keep);
    if (lane == 0) {
        if (q == a.nmask - 1 && (a.n & 31)) word &= (1u << (a.n & 31)) - 1u;
        a.bits[q] = word;
    }
}

// The nonzero nibbles of jump block j (coefficients PHASE j .. PHASE j + PHASE - 1 of g), as
// 16-bit word offsets into shared memory: a nibble v at coefficient 4 n reads X[B + 4 n + s + w]
// from the ring when v has one bit s, and word 4 n + w of table v otherwise (B = the block's
// first word, at ring slot sB). Their number goes to `count`. One warp.
__device__ __forceinline__ void list_nibbles(const uint32_t *__restrict__ g, int j, uint32_t sB, uint16_t *list,
                                             int *count, int lane) {
    constexpr int GW = PHASE / 32;
    const int gi = j * GW + lane;
    const uint32_t mine = lane < GW && gi < 2 * PW ? __ldg(g + gi) : 0u;
    int c = 0;
#pragma unroll
    for (int u = 0; u < GW; u++) {
        const uint32_t w = __shfl_sync(0xffffffffu, mine, u);
        const uint32_t v = lane < 8 ? (w >> (4 * lane)) & 15u : 0u;
        const uint32_t bal = __ballot_sync(0xffffffffu, v != 0u);
        if (v) {
            const int n = 8 * u + lane;
            // tables hold the values with two or more bits: 3, 5, 6, 7, 9, ..., 15 -> 0 .. 10
            const int idx = (int)v - 1 - (v > 1u) - (v > 2u) - (v > 4u) - (v > 8u);
            const uint32_t base = __popc(v) == 1 ? sB + (uint32_t)(__ffs(v) - 1) : (uint32_t)(TAB0 + idx * TABW);
            list[c + __popc(bal & ((1u << lane) - 1u))] = (uint16_t)(base + 4u * (uint32_t)n);
        }
        c += __popc(bal);
    }
    if (lane == 0) *count = c;
}

// Jumps the window X[b, b + 624) in the ring (P == b + 624 on entry) by the polynomial g
// (DEG coefficients in 2 PW 32-bit words): on return the ring holds X[b + dist, b + dist + 624)
// and P == b + dist + 624. Block j of g (coefficients [PHASE j, PHASE j + PHASE), first word
// B = b + PHASE j) is taken four coefficients at a time (the method of four Russians): once
// the phase that makes X[.., B + 1200) is done, the CTA writes the eleven tables
// T_v[k] = XOR over the bits s of v of X[B + k + s], then thread t < JT adds, for each nonzero
// nibble v at 4 n, the word 4 n + w of T_v (or of the ring when v has one bit) into window
// words w = t + JT d, d < JW. A warp reads consecutive words: no bank conflicts. The list warp
// writes block j's entries while the phase is made (two list buffers: a buffer is rewritten
// two barriers after its last reader finished).
__device__ void jump_window(uint32_t *sm, const uint32_t *__restrict__ g, int64_t &b, int64_t &P, int64_t dist) {
    const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
    constexpr int NBLK = (DEG + PHASE - 1) / PHASE;
    uint16_t *lists = reinterpret_cast<uint16_t *>(sm + LST0);
    int *counts = reinterpret_cast<int *>(sm + CNT0);
    uint32_t acc[JW] = {};
    for (int j = 0; j < NBLK; j++) {
        const uint32_t sB = ((uint32_t)b + (uint32_t)(j * PHASE)) & (RING - 1);
        gen_words(sm, (uint32_t)P, PHASE);
        if (warp == LIST_WARP) list_nibbles(g, j, sB, lists + (j & 1) * NIB, &counts[j & 1], lane);
        __syncthreads();
        P += PHASE;
        // X[B + k + s], k < TABW, s < 4: below P = B + 1200 + 4... made; sB + k + s < 2 RING.
        for (int k = tid; k < TABW; k += THREADS) {
            const uint32_t *x = sm + sB + k;
            const uint32_t x0 = x[0], x1 = x[1], x2 = x[2], x3 = x[3];
            const uint32_t t3 = x0 ^ x1, t5 = x0 ^ x2, t6 = x1 ^ x2, t7 = t3 ^ x2;
            uint32_t *t = sm + TAB0 + k;
            t[0 * TABW] = t3;
            t[1 * TABW] = t5;
            t[2 * TABW] = t6;
            t[3 * TABW] = t7;
            t[4 * TABW] = x0 ^ x3;
            t[5 * TABW] = x1 ^ x3;
            t[6 * TABW] = t3 ^ x3;
            t[7 * TABW] = x2 ^ x3;
            t[8 * TABW] = t5 ^ x3;
            t[9 * TABW] = t6 ^ x3;
            t[10 * TABW] = t7 ^ x3;
        }
        __syncthreads();
        if (warp < JT / 32 + (JT % 32 != 0)) {
            // Lanes past JT (warp 9, lanes 24..31) read in-bounds words and keep no result. A
            // warp loads 32 entries at once and broadcasts them, so the word loads of 32
            // entries are in flight together.
            const uint32_t *p = sm + tid;
            const uint16_t *L = lists + (j & 1) * NIB;
            const int cnt = counts[j & 1];
            int i0 = 0;
            for (; i0 + 32 <= cnt; i0 += 32) {
                const uint32_t mine = L[i0 + lane];
#pragma unroll
                for (int e = 0; e < 32; e++) {
                    const uint32_t o = __shfl_sync(0xffffffffu, mine, e);
#pragma unroll
                    for (int d = 0; d < JW; d++) acc[d] ^= p[o + JT * d];
                }
            }
            if (i0 < cnt) {
                const uint32_t mine = i0 + lane < cnt ? L[i0 + lane] : 0u;
                for (int e = 0; e < cnt - i0; e++) {
                    const uint32_t o = __shfl_sync(0xffffffffu, mine, e);
#pragma unroll
                    for (int d = 0; d < JW; d++) acc[d] ^= p[o + JT * d];
                }
            }
        }
    }
    __syncthreads();
    b += dist;
    if (tid < JT) {
#pragma unroll
        for (int d = 0; d < JW; d++) put(sm, (uint32_t)b + (uint32_t)(tid + JT * d), acc[d]);
    }
    P = b + MT_N;
    __syncthreads();
}

// CTA c of K owns the chunks [c nch / K, (c + 1) nch / K) of the call's nch chunks: it reaches
// the first one's start by one jump (none for chunk 0), then makes TURN words per CTA barrier
// (eight generating warps) and turns each turn's words into 9 NPH mask words in the next turn
// of the loop (nine conversion warps), while the following turn is made. The CTA whose
// chunks hold the block of the last consumed word copies out the end state.
__global__ void __launch_bounds__(THREADS) keep_bits_kernel(KeepArgs a) {
    extern __shared__ __align__(16) uint32_t sm[];
    uint32_t *ring = sm;
    const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;

    const uint32_t left = a.st_in[MT_N];
    if (left == 0 || left > (uint32_t)MT_N) {  // not a state DenseCore's engine can be in
        if (blockIdx.x == 0 && threadIdx.x == 0) atomicExch(a.err, sm100::DEV_BAD_GENERATOR_STATE);
        return;
    }
    const int64_t pos = 625 - (int64_t)left;          // 1..624
    const int64_t B0 = pos == MT_N ? MT_N : 0;        // canonical block start
    const int64_t G = B0 + MT_N;
    const int64_t last = pos + 2 * a.n - 1;           // last consumed word
    const int64_t E = B0 + MT_N * ((last - B0) / MT_N);  // its block
    // Chunk 0 is [pos, G + CHUNK), chunk c >= 1 is [G + c CHUNK, G + (c + 1) CHUNK); a mask
    // word belongs to the chunk of its first word pos + 64 q.
    const int64_t cE = E < G ? 0 : (E - G) / CHUNK;
    const int64_t qlast = pos + 64 * (a.nmask - 1);
    const int64_t cQ = qlast < G ? 0 : (qlast - G) / CHUNK;
    const int64_t nch = 1 + (cE > cQ ? cE : cQ);
    const int64_t K = gridDim.x, c0 = blockIdx.x * nch / K, c1 = (blockIdx.x + 1) * nch / K;
    if (c0 >= c1) return;  // uniform across the CTA
    const int64_t lo = c0 == 0 ? pos : G + c0 * CHUNK, hi = G + c1 * CHUNK;
    const int64_t q_lo = c0 == 0 ? 0 : (lo - pos + 63) / 64;
    const int64_t q_hi = imin((hi - pos + 63) / 64, a.nmask);
    const bool owns_end = cE >= c0 && cE < c1;
    if (q_lo >= q_hi && !owns_end) return;

    for (int i = tid; i < MT_N; i += THREADS) ring[i] = ring[i + RING] = a.st_in[i];
    __syncthreads();
    int64_t b = 0, P = MT_N;  // window X[b, b + 624), produced up to P
    if (c0 > 0) {
        while (P < G + MT_N) {  // the base window at G
            const int cnt = (int)imin(PHASE, G + MT_N - P);
            gen_words(ring, (uint32_t)P, cnt);
            __syncthreads();
            P += cnt;
        }
        b = G;
        jump_window(sm, a.tab + (size_t)c0 * 2 * PW, b, P, c0 * CHUNK);
    }
    // Phases start at P = pos (mod 64), so that each one holds nine whole mask words.
    const int align = (int)((pos - P) & 63);
    if (align) {
        gen_words(ring, (uint32_t)P, align);
        __syncthreads();
        P += align;
    }
    // Owned mask words whose words are already made: those of the window.
    const int64_t q_pre = imin(q_hi, (P - pos) / 64);
    for (int64_t q = q_lo + warp; q < q_pre; q += WARPS) {
        uint32_t hi, lo;
        load_pair(ring, (uint32_t)(pos + 64 * q) + 2u * (uint32_t)lane, hi, lo);
        store_word(a, hi, lo, q, lane);
    }

    int64_t target = pos + 64 * q_hi;
    if (owns_end && E + MT_N > target) target = E + MT_N;
    const int64_t nturn = target > P ? (target - P + TURN - 1) / TURN : 0;
    bool captured = !owns_end;
    // Turn u: copy out the end state once its block is made; the generating warps make the NPH
    // phases of [P, P + TURN) (a named barrier of their own between them; the slots written are
    // those of words at least RING - TURN below P: neither read nor copied here) while each
    // conversion warp turns NPH mask words of the words of turn u - 1 ([P - TURN, P)), NPH
    // independent chains.
    const int cw = warp - GEN_WARPS;
    int64_t qw = (P - pos) / 64 + cw;  // this conversion warp's first mask word in turn 1
    uint32_t slot = (uint32_t)(pos + 64 * qw) + 2u * (uint32_t)lane;
    uint32_t P32 = (uint32_t)P;
    for (int64_t u = 0; u <= nturn; u++) {
        if (!captured && P >= E + MT_N) {
            for (int i = tid; i < MT_N; i += THREADS) a.st_out[i] = ring[((uint32_t)E + (uint32_t)i) & (RING - 1)];
            if (tid == 0) {
                const uint32_t next = (uint32_t)(last - E + 1);
                a.st_out[MT_N] = 625u - next;
                a.st_out[MT_N + 1] = next;
            }
            captured = true;
        }
        if (warp < GEN_WARPS) {
            if (u < nturn) {
#pragma unroll
                for (int f = 0; f < NPH; f++) {
                    if (f > 0) asm volatile("bar.sync 1, %0;" ::"r"(GEN_WARPS * 32) : "memory");
                    gen_words(ring, P32 + (uint32_t)(f * PHASE), PHASE);
                }
            }
        } else if (u > 0) {
            uint32_t hi[NPH], lo[NPH];
#pragma unroll
            for (int f = 0; f < NPH; f++) {
                const int64_t q = qw + f * CONV_WARPS;
                hi[f] = lo[f] = 0u;
                if (q >= q_lo && q < q_hi) load_pair(ring, slot + 64u * CONV_WARPS * (uint32_t)f, hi[f], lo[f]);
            }
#pragma unroll
            for (int f = 0; f < NPH; f++) {
                const int64_t q = qw + f * CONV_WARPS;
                if (q >= q_lo && q < q_hi) store_word(a, hi[f], lo[f], q, lane);
            }
            qw += NPH * CONV_WARPS;
            slot += 64u * NPH * CONV_WARPS;
        }
        __syncthreads();
        P += TURN;
        P32 += TURN;
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

// The kernel's shared memory (above the 48 KB default), granted once per device.
int allow_keep_smem() {
    static std::mutex mu;
    static bool done[kTableDevices];
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "dropout: current device");
    if (dev < 0 || dev >= kTableDevices)
        return fail(DC_ERR_UNSUPPORTED, "dropout: device ordinal " + std::to_string(dev) + " is above 63");
    std::lock_guard<std::mutex> lock(mu);
    if (!done[dev]) {
        e = cudaFuncSetAttribute(keep_bits_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_WORDS * 4);
        if (e != cudaSuccess) return cuda_fail(e, "dropout: keep-bits shared memory");
        done[dev] = true;
    }
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
    st = allow_keep_smem();
    if (st) return st;
    // keep iff m * 2^-53 < keep_prob  <=>  m < ceil(keep_prob * 2^53) (the scaling is exact)
    const uint64_t thresh = (uint64_t)ceil(keep_prob * 9007199254740992.0);
    uint32_t *tmp = nullptr;
    if (launches > 1 || st_out == st_in) {
        st = pool_alloc(reinterpret_cast<void **>(&tmp), 2 * (MT_N + 2) * 4, stream);
        if (st) return st;
    }
    // One CTA per SM at most: each CTA pays one jump (shared-memory bound, the same for every
    // distance); a second CTA per SM measured no faster.
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const uint32_t *src = st_in;
    for (int64_t l = 0; l < launches; l++) {
        const int64_t e0 = l * kMaxElemsPerLaunch, ne = imin(kMaxElemsPerLaunch, n - e0);
        uint32_t *dst = l == launches - 1 && st_out != st_in ? st_out : tmp + (l & 1) * (MT_N + 2);
        KeepArgs a{src, dst, tab, bits + e0 / 32, ne, (ne + 31) / 32, thresh, err};
        const int64_t grid = imin(1 + (2 * ne - 1) / CHUNK, sms > 0 ? sms : 1);  // >= the chunks' count
        {
            KernelTrace tr("dropout_keep_bits", stream);
            keep_bits_kernel<<<(unsigned)grid, THREADS, SMEM_WORDS * 4, stream>>>(a);
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
