// ORACLE - test infrastructure only (not part of the product).
//
// C++ restatement of the randomness of the reference's CUDA path, so that its offsets,
// pblock -> vblock assignments and per-vblock permutations can be injected into the B200
// kernels (povs_apply_v1) and into the C oracle:
//   * host loop, src/povs/__cuda/lib/povs.cu:396-430: std::mt19937 seeded with the call seed;
//     a persistent assignment array initialised to 0..n_p-1 followed by -1 padding
//     (povs.cu:401-404) and re-shuffled every iteration by a forward Fisher-Yates whose draws
//     are std::uniform_int_distribution<long>(i, n_p-1) (lib/utils.h:51-60); then one
//     std::uniform_int_distribution<int>(1, 999) seed per vblock; then the offset index from
//     std::uniform_int_distribution<long>(0, n_offsets-1).  libstdc++'s <random> is used
//     directly, not restated.
//   * kernel Stage 0 + Stage 2, povs.cu:203-221 and :282-321: members sorted ascending with
//     padding last; slots 0..B valid (B = valid rows - 1); forward Fisher-Yates of the identity
//     with xorshift32 (13, 17, 5) seeded by the vblock seed and Lemire's multiply-shift range
//     j = i + ((uint64)rng * (B - i + 1)) >> 32.
#include <cstdint>
#include <random>
#include <utility>
#include <vector>

namespace {

void fisher_yates_forward(std::vector<long>& a, long n, std::mt19937& rng)
{
    for (long i = 0; i < n; ++i) {
        std::uniform_int_distribution<long> d(i, n - 1);
        long j = d(rng);
        std::swap(a[i], a[j]);
    }
}

// Kernel Stage 0 + Stage 2 for one vblock: members m[0..V) (padding -1, any order) and its seed;
// writes V*P entries of pv (entries beyond the valid rows are -1).
void vblock_perm(const long* members, int V, int P, int64_t N, int seed, std::vector<uint32_t>& idx, int32_t* pv)
{
    // Stage 0: insertion sort ascending, -1 sinks to the end.
    std::vector<long> m(members, members + V);
    for (int i = 1; i < V; ++i) {
        long key = m[i];
        int j = i - 1;
        while (j >= 0 && key != -1 && (m[j] == -1 || m[j] > key)) {
            m[j + 1] = m[j];
            --j;
        }
        m[j + 1] = key;
    }
    int n_valid = 0;
    for (int k = 0; k < V; ++k) {
        if (m[k] == -1) break;
        const int64_t left = N - static_cast<int64_t>(m[k]) * P;
        n_valid += left < P ? static_cast<int>(left) : P;
    }
    // Stage 2: Fisher-Yates over the gap-free slots 0..B.
    for (int f = 0; f < n_valid; ++f) idx[f] = static_cast<uint32_t>(f);
    const int B = n_valid - 1;
    uint32_t r = static_cast<uint32_t>(seed);
    for (int i = 0; i <= B; ++i) {
        r ^= r << 13;
        r ^= r >> 17;
        r ^= r << 5;
        const int j = i + static_cast<int>((static_cast<uint64_t>(r) * static_cast<uint64_t>(B - i + 1)) >> 32);
        std::swap(idx[i], idx[j]);
    }
    for (int f = 0; f < V * P; ++f) pv[f] = f < n_valid ? static_cast<int32_t>(idx[f]) : -1;
}

} // namespace

extern "C" {

// Outputs: out_offsets[iterations], out_assign[iterations][n_v*V] (padding -1),
// out_perms[iterations][n_v][V*P] (entries beyond the valid rows are -1).
int oracle_refcuda_randomness(int32_t seed, int64_t N, int32_t P, int32_t V, const int64_t* offsets,
                              int32_t n_offsets, int32_t iterations, int64_t* out_offsets, int64_t* out_assign,
                              int32_t* out_perms)
{
    if (N < 1 || P < 1 || V < 1 || n_offsets < 1) return -1;
    const long n_p = static_cast<long>((N + P - 1) / P);
    const long n_v = (n_p + V - 1) / V;
    const long n_assign = n_v * V;
    const int VP = V * P;

    std::mt19937 rng(static_cast<std::mt19937::result_type>(seed));
    std::uniform_int_distribution<long> offset_dist(0l, static_cast<long>(n_offsets) - 1);
    std::uniform_int_distribution<int> seed_dist(1, 999);

    std::vector<long> a(static_cast<size_t>(n_assign));
    for (long i = 0; i < n_assign; ++i) a[i] = i < n_p ? i : -1;
    std::vector<int> seeds(static_cast<size_t>(n_v));
    std::vector<uint32_t> idx(static_cast<size_t>(VP));

    for (int it = 0; it < iterations; ++it) {
        fisher_yates_forward(a, n_p, rng);
        for (long v = 0; v < n_v; ++v) seeds[v] = seed_dist(rng);
        const long offset = offsets[offset_dist(rng)];
        out_offsets[it] = offset;
        int64_t* asg = out_assign + static_cast<int64_t>(it) * n_assign;
        for (long i = 0; i < n_assign; ++i) asg[i] = a[i];
        int32_t* perms = out_perms + static_cast<int64_t>(it) * n_v * VP;
        for (long v = 0; v < n_v; ++v) vblock_perm(a.data() + v * V, V, P, N, seeds[v], idx, perms + v * VP);
    }
    return 0;
}

// Stage 0 + Stage 2 for given members and seeds (any member order, padding anywhere):
// assign int64 [n_v][V], seeds int32 [n_v], out_perms int32 [n_v][V*P].
int oracle_refcuda_perms(int64_t N, int32_t P, int32_t V, const int64_t* assign, const int32_t* seeds,
                         int32_t* out_perms)
{
    if (N < 1 || P < 1 || V < 1) return -1;
    const long n_p = static_cast<long>((N + P - 1) / P);
    const long n_v = (n_p + V - 1) / V;
    std::vector<uint32_t> idx(static_cast<size_t>(V) * P);
    std::vector<long> m(static_cast<size_t>(V));
    for (long v = 0; v < n_v; ++v) {
        for (int k = 0; k < V; ++k) {
            const int64_t x = assign[v * V + k];
            m[k] = (x < 0 || x >= n_p) ? -1 : static_cast<long>(x);
        }
        vblock_perm(m.data(), V, P, N, seeds[v], idx, out_perms + v * V * P);
    }
    return 0;
}

} // extern "C"
