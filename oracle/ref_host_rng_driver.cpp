// ORACLE - test infrastructure only (not part of the product).
//
// Driver compiled against the reference's own header src/povs/__cuda/lib/utils.h, in place
// under the reference tree (see oracle/build.py), into oracle/_ref/libref_host_rng.so.  It runs
// the reference's compiled `shuffle_array` (lib/utils.h:51-60) inside the draw sequence of the
// reference host loop (src/povs/__cuda/lib/povs.cu:396-430: assignment shuffle, one seed draw
// per vblock, one offset-index draw), so the C++ restatement in ref_cuda_rng.cpp can be pinned
// against the reference's code for the assignment sequence.
#include <cstdint>
#include <random>
#include <type_traits>
#include <utility>
#include <vector>

#include "utils.h"

extern "C" int ref_assign_sequence(int32_t seed, int64_t N, int32_t P, int32_t V, int32_t n_offsets,
                                   int32_t iterations, int64_t* out_assign, int64_t* out_offset_index)
{
    const long n_p = div_round_up(static_cast<long>(N), P);
    const long n_v = div_round_up(n_p, V);
    const long n_assign = n_v * V;
    std::mt19937 rng(seed);
    std::uniform_int_distribution offset_dist(0l, static_cast<long>(n_offsets) - 1);
    std::uniform_int_distribution seed_dist(1, 999);
    std::vector<long> a(static_cast<size_t>(n_assign));
    for (long i = 0; i < n_assign; ++i) a[i] = i < n_p ? i : -1;
    for (int it = 0; it < iterations; ++it) {
        shuffle_array(a.data(), n_p, rng);
        for (long v = 0; v < n_v; ++v) (void)seed_dist(rng);
        out_offset_index[it] = offset_dist(rng);
        for (long i = 0; i < n_assign; ++i) out_assign[static_cast<int64_t>(it) * n_assign + i] = a[i];
    }
    return 0;
}
