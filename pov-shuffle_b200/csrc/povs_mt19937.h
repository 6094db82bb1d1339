// Host-side permutations of the reference's NumPy path: numpy.random.RandomState(seed).shuffle of
// arange(n) (src/povs/numpy.py:125-136 applies it to every vblock's rows, with seed drawn from 1..999).
//
// Restated from the published algorithms, not from any implementation's source:
//   * MT19937 (Matsumoto and Nishimura, ACM TOMACS 8(1), 1998): 624-word state seeded by the
//     recurrence x[i] = 1812433253 * (x[i-1] ^ (x[i-1] >> 30)) + i from x[0] = seed, regenerated in
//     blocks of 624 (twist with matrix 0x9908b0df), outputs tempered with shifts 11, 7 (mask
//     0x9d2c5680), 15 (mask 0xefc60000) and 18;
//   * NumPy's legacy bounded integers: a draw in [0, m] masks a 32-bit output to the smallest
//     all-ones mask covering m and rejects values above m;
//   * the legacy shuffle: for i = n-1 down to 1, swap element i with element draw(i).
// The library's tests check the result against numpy.random.RandomState itself.
#pragma once

#include <cstdint>

namespace povs {

class Mt19937 {
public:
    explicit Mt19937(uint32_t seed)
    {
        x_[0] = seed;
        for (uint32_t i = 1; i < N; ++i) x_[i] = 1812433253u * (x_[i - 1] ^ (x_[i - 1] >> 30)) + i;
        at_ = N;
    }

    uint32_t next()
    {
        if (at_ >= N) regenerate();
        uint32_t y = x_[at_++];
        y ^= y >> 11;
        y ^= (y << 7) & 0x9d2c5680u;
        y ^= (y << 15) & 0xefc60000u;
        y ^= y >> 18;
        return y;
    }

    // Uniform integer in [0, m] by masked rejection (m < 2^32).
    uint32_t bounded(uint32_t m)
    {
        if (m == 0) return 0;
        uint32_t mask = m;
        mask |= mask >> 1;
        mask |= mask >> 2;
        mask |= mask >> 4;
        mask |= mask >> 8;
        mask |= mask >> 16;
        uint32_t v;
        do {
            v = next() & mask;
        } while (v > m);
        return v;
    }

private:
    static constexpr uint32_t N = 624, M = 397;
    uint32_t x_[N];
    uint32_t at_;

    void regenerate()
    {
        for (uint32_t i = 0; i < N; ++i) {
            const uint32_t y = (x_[i] & 0x80000000u) | (x_[(i + 1) % N] & 0x7fffffffu);
            x_[i] = x_[(i + M) % N] ^ (y >> 1) ^ ((y & 1u) ? 0x9908b0dfu : 0u);
        }
        at_ = 0;
    }
};

// numpy.random.RandomState(seed).shuffle(arange(n)) into out[0 .. n-1].
template <typename T>
inline void numpy_legacy_shuffle(uint32_t seed, int n, T* out)
{
    for (int i = 0; i < n; ++i) out[i] = static_cast<T>(i);
    Mt19937 g(seed);
    for (int i = n - 1; i >= 1; --i) {
        const uint32_t j = g.bounded(static_cast<uint32_t>(i));
        const T t = out[i];
        out[i] = out[j];
        out[j] = t;
    }
}

} // namespace povs
