// Counter-based randomness of the B200 POV shuffle.
//
// The reference draws every iteration's randomness on the host with a serial
// std::mt19937 (src/povs/__cuda/lib/povs.cu:396-430, lib/utils.h:51-60) and
// copies it to the device.  Here every random quantity is a pure function of
// (seed, iteration, vblock, element), so any thread can compute the values it
// needs without a host round trip:
//
//   * offset index         philox(seed; {0, 0, DOMAIN_OFFSET<<24, it}).x
//   * pblock -> vblock map  a keyed Feistel bijection of [0, n_v*V) whose
//                           12 round keys come from philox(seed; {c, 0,
//                           DOMAIN_ASSIGN<<24, it}), c = 0..2; slot s of
//                           vblock v holds pblock pi(v*V + s); ids >= n_p are
//                           padding.
//   * per-vblock order      element e of vblock v gets the 32-bit key
//                           philox(seed; {e>>2, v_lo, v_hi|DOMAIN_PERM<<24,
//                           it}).word[e&3]; sorting (key, e) ascending gives
//                           the source slot of every destination slot.
//
// Philox4x32-10 is the generator of Salmon, Moraes, Dror and Shaw, "Parallel
// random numbers: as easy as 1, 2, 3" (SC'11).  The Feistel round function
// is the "lowbias32" integer hash from Wellons' hash-prospector.  The
// bijection with cycle walking follows the construction of Mitchell, Stokes,
// Frank and Holmes, "Bandwidth-optimal random shuffling for GPUs" (2022).
#pragma once

#include <stdint.h>

#if defined(__CUDACC__)
#define POVS_HD __host__ __device__ __forceinline__
#else
#define POVS_HD inline
#endif

namespace povs {

enum : uint32_t {
    DOMAIN_OFFSET = 1u,
    DOMAIN_ASSIGN = 2u,
    DOMAIN_PERM = 3u,
    DOMAIN_VSEED = 4u,
};

// Randomness modes.
enum : int {
    RNG_UNIFORM = 0,        // uniform per-vblock permutations (sorted Philox keys), padding anywhere
    RNG_REFERENCE_CUDA = 1, // the reference CUDA path's distribution: per-vblock seeds 1..999,
                            // xorshift32 forward Fisher-Yates, padding in the last vblock
    RNG_REFERENCE_NUMPY = 2, // the reference NumPy path's distribution: padding anywhere, members in
                             // slot order, per-vblock seeds 1..999 and RandomState(seed).shuffle
};

constexpr int FEISTEL_ROUNDS = 12;

struct U32x4 {
    uint32_t x, y, z, w;
};

POVS_HD void mul_hilo(uint32_t a, uint32_t b, uint32_t& hi, uint32_t& lo)
{
#if defined(__CUDA_ARCH__)
    hi = __umulhi(a, b);
    lo = a * b;
#else
    const uint64_t p = static_cast<uint64_t>(a) * b;
    hi = static_cast<uint32_t>(p >> 32);
    lo = static_cast<uint32_t>(p);
#endif
}

// Philox4x32 with 10 rounds (SC'11 paper, table of constants in section 5).
POVS_HD U32x4 philox4x32_10(U32x4 c, uint32_t k0, uint32_t k1)
{
    constexpr uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u;
    constexpr uint32_t W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
#pragma unroll
    for (int r = 0; r < 10; ++r) {
        uint32_t hi0, lo0, hi1, lo1;
        mul_hilo(M0, c.x, hi0, lo0);
        mul_hilo(M1, c.z, hi1, lo1);
        c = U32x4{hi1 ^ c.y ^ k0, lo1, hi0 ^ c.w ^ k1, lo0};
        k0 += W0;
        k1 += W1;
    }
    return c;
}

POVS_HD uint32_t pick_word(const U32x4& v, int i)
{
    return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

// Unbiased-enough range reduction of a 32-bit draw to [0, n) (multiply-shift).
POVS_HD uint32_t reduce_range(uint32_t r, uint32_t n)
{
    return static_cast<uint32_t>((static_cast<uint64_t>(r) * n) >> 32);
}

POVS_HD uint32_t seed_lo(uint64_t seed) { return static_cast<uint32_t>(seed); }
POVS_HD uint32_t seed_hi(uint64_t seed) { return static_cast<uint32_t>(seed >> 32); }

POVS_HD uint32_t offset_draw(uint64_t seed, uint32_t iteration)
{
    return philox4x32_10(U32x4{0u, 0u, DOMAIN_OFFSET << 24, iteration}, seed_lo(seed), seed_hi(seed)).x;
}

POVS_HD uint32_t perm_key(uint64_t seed, uint32_t iteration, uint64_t vblock, uint32_t element)
{
    const U32x4 c{element >> 2, static_cast<uint32_t>(vblock),
                  (static_cast<uint32_t>(vblock >> 32) & 0x00FFFFFFu) | (DOMAIN_PERM << 24), iteration};
    return pick_word(philox4x32_10(c, seed_lo(seed), seed_hi(seed)), static_cast<int>(element & 3u));
}

// Four consecutive element keys (elements 4q .. 4q+3) of one vblock in one call.
POVS_HD U32x4 perm_key4(uint64_t seed, uint32_t iteration, uint64_t vblock, uint32_t quad)
{
    const U32x4 c{quad, static_cast<uint32_t>(vblock),
                  (static_cast<uint32_t>(vblock >> 32) & 0x00FFFFFFu) | (DOMAIN_PERM << 24), iteration};
    return philox4x32_10(c, seed_lo(seed), seed_hi(seed));
}

// Per-vblock seed in [1, 999] of the reference-CUDA mode (the reference draws
// uniform_int_distribution(1, 999), src/povs/__cuda/lib/povs.cu:398,425-426).
POVS_HD uint32_t vblock_seed(uint64_t seed, uint32_t iteration, uint64_t vblock)
{
    const U32x4 c{0u, static_cast<uint32_t>(vblock),
                  (static_cast<uint32_t>(vblock >> 32) & 0x00FFFFFFu) | (DOMAIN_VSEED << 24), iteration};
    return 1u + reduce_range(philox4x32_10(c, seed_lo(seed), seed_hi(seed)).x, 999u);
}

POVS_HD uint32_t lowbias32(uint32_t x)
{
    x ^= x >> 16;
    x *= 0x7feb352du;
    x ^= x >> 15;
    x *= 0x846ca68bu;
    x ^= x >> 16;
    return x;
}

// Keyed bijection of [0, domain) used for the physical -> virtual block map.
struct Feistel {
    uint32_t keys[FEISTEL_ROUNDS];
    uint64_t domain; // number of assignment slots, n_v * V
    int lbits, rbits; // widths of the two halves, lbits + rbits = ceil(log2(domain)) (>= 2)

    POVS_HD void init(uint64_t seed, uint32_t iteration, uint64_t n_slots)
    {
#pragma unroll
        for (uint32_t c = 0; c < FEISTEL_ROUNDS / 4; ++c) {
            const U32x4 r = philox4x32_10(U32x4{c, 0u, DOMAIN_ASSIGN << 24, iteration}, seed_lo(seed), seed_hi(seed));
            keys[4 * c + 0] = r.x;
            keys[4 * c + 1] = r.y;
            keys[4 * c + 2] = r.z;
            keys[4 * c + 3] = r.w;
        }
        domain = n_slots;
        int bits = 2;
        while (bits < 64 && (uint64_t{1} << bits) < n_slots) ++bits;
        lbits = bits / 2;
        rbits = bits - lbits;
    }

    // One pass of the network over [0, 2^(lbits+rbits)).
    POVS_HD uint64_t round_trip(uint64_t x) const
    {
        int wl = lbits, wr = rbits;
        uint64_t L = x >> wr;
        uint64_t R = x & ((uint64_t{1} << wr) - 1);
#pragma unroll
        for (int i = 0; i < FEISTEL_ROUNDS; ++i) {
            // Round function on the low 32 bits of R, widened by a second hash for halves > 32 bits.
            const uint32_t h0 = lowbias32(static_cast<uint32_t>(R) ^ keys[i]);
            const uint32_t h1 = lowbias32(static_cast<uint32_t>(R >> 32) ^ h0 ^ keys[(i + 1) % FEISTEL_ROUNDS]);
            const uint64_t f = (static_cast<uint64_t>(h1) << 32) | h0;
            const uint64_t nl = R;
            const uint64_t nr = (L ^ f) & ((uint64_t{1} << wl) - 1);
            L = nl;
            R = nr;
            const int t = wl;
            wl = wr;
            wr = t;
        }
        return (L << wr) | R;
    }

    // Same network when both halves fit 32 bits: the high word of the round function is
    // masked away there, so only the low hash is needed.
    POVS_HD uint32_t round_trip32(uint32_t x) const
    {
        int wl = lbits, wr = rbits;
        uint32_t L = x >> wr;
        uint32_t R = x & ((1u << wr) - 1u);
#pragma unroll
        for (int i = 0; i < FEISTEL_ROUNDS; ++i) {
            const uint32_t nr = (L ^ lowbias32(R ^ keys[i])) & ((1u << wl) - 1u);
            L = R;
            R = nr;
            const int t = wl;
            wl = wr;
            wr = t;
        }
        return (L << wr) | R;
    }

    // Inverse of round_trip32: undo rounds 11..0.  Round i starts with widths (lbits, rbits) when
    // i is even and (rbits, lbits) when odd, and maps (L, R) to (R, (L ^ F_i(R)) & mask).
    POVS_HD uint32_t round_trip32_inverse(uint32_t y) const
    {
        uint32_t L = y >> rbits;
        uint32_t R = y & ((1u << rbits) - 1u);
#pragma unroll
        for (int i = FEISTEL_ROUNDS - 1; i >= 0; --i) {
            const int wl_i = (i & 1) ? rbits : lbits;
            const uint32_t prev_r = L;
            const uint32_t prev_l = (R ^ lowbias32(prev_r ^ keys[i])) & ((1u << wl_i) - 1u);
            L = prev_l;
            R = prev_r;
        }
        return (L << rbits) | R;
    }

    POVS_HD uint64_t round_trip_inverse(uint64_t y) const
    {
        uint64_t L = y >> rbits;
        uint64_t R = y & ((uint64_t{1} << rbits) - 1);
#pragma unroll
        for (int i = FEISTEL_ROUNDS - 1; i >= 0; --i) {
            const int wl_i = (i & 1) ? rbits : lbits;
            const uint64_t prev_r = L;
            const uint32_t h0 = lowbias32(static_cast<uint32_t>(prev_r) ^ keys[i]);
            const uint32_t h1 = lowbias32(static_cast<uint32_t>(prev_r >> 32) ^ h0 ^ keys[(i + 1) % FEISTEL_ROUNDS]);
            const uint64_t f = (static_cast<uint64_t>(h1) << 32) | h0;
            const uint64_t prev_l = (R ^ f) & ((uint64_t{1} << wl_i) - 1);
            L = prev_l;
            R = prev_r;
        }
        return (L << rbits) | R;
    }

    // pi^-1(y) for y in [0, domain): the inverse cycle walk.
    POVS_HD uint64_t inverse(uint64_t y) const
    {
        if (lbits + rbits <= 32) {
            uint32_t x = round_trip32_inverse(static_cast<uint32_t>(y));
            while (x >= domain) x = round_trip32_inverse(x);
            return x;
        }
        uint64_t x = round_trip_inverse(y);
        while (x >= domain) x = round_trip_inverse(x);
        return x;
    }

    // pi(x) for x in [0, domain): cycle-walk until the image falls inside the domain.
    // Terminates because round_trip is a permutation of [0, 2^bits) and x is inside the domain.
    POVS_HD uint64_t operator()(uint64_t x) const
    {
        if (lbits + rbits <= 32) {
            uint32_t y = round_trip32(static_cast<uint32_t>(x));
            while (y >= domain) y = round_trip32(y);
            return y;
        }
        uint64_t y = round_trip(x);
        while (y >= domain) y = round_trip(y);
        return y;
    }
};

} // namespace povs
