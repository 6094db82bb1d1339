// Shuffle-bias metrics on the GPU: histograms of travel distances and n-gram keys over many
// shuffled episodes (each episode a permutation of the ids 0 .. deck-1).
//
// Definitions follow the reference's metric module (src/povs/eval/metrics.py):
//  * positional travel distance of the element at position i holding id v: (i - v) mod deck
//    (get_tvd, metrics.py:38-87);
//  * relative travel distance of the k-th n-gram element, the n-gram anchored at position i with
//    elements spaced `step` = skip + 1 apart (wrapping around the deck):
//    ((v[i + k*step] - v[i]) - k*step) mod deck (_relative_travel_distances, metrics.py:250-278,
//    reduced modulo deck as in get_ngram_tvd, metrics.py:90-248);
//  * an n-gram key for n >= 3 is the base-deck number of its n-1 reduced distances, first
//    distance most significant (metrics.py:196-236).
// The distributions' TVDs are finished on the host from these counts (O(deck) work).
#pragma once

#include <cstdint>

namespace povs {

constexpr int HIST_SMEM_MAX_BINS = 49152; // uint32 bins staged per CTA (192 KiB of shared memory)

struct MetricParams {
    const void* ids;        // episode e, position i at ids[e * episode_stride + i * element_stride]
    int32_t id_bytes;       // 4 (int32) or 8 (int64)
    int32_t kind;           // histograms: 0 positional, 1 pair distance (n = 2); keys: n
    int64_t n_episodes;
    int64_t deck;
    int64_t episode_stride; // in ids
    int64_t element_stride; // in ids
    int64_t step;           // skip + 1
    const int64_t* positions; // keys: anchor positions (NULL = every position)
    int64_t n_positions;
    unsigned long long* counts; // histograms: deck bins, added to
    int64_t* keys;              // keys: n_episodes * (n_positions or deck) outputs
    int32_t smem_bins;          // histograms: deck when staged in shared memory, else 0
};

__device__ __forceinline__ int64_t metric_id(const MetricParams& q, int64_t e, int64_t i)
{
    const int64_t at = e * q.episode_stride + i * q.element_stride;
    return q.id_bytes == 4 ? static_cast<int64_t>(static_cast<const int32_t*>(q.ids)[at])
                           : static_cast<const int64_t*>(q.ids)[at];
}

__device__ __forceinline__ int64_t floor_mod(int64_t a, int64_t m)
{
    const int64_t r = a % m;
    return r < 0 ? r + m : r;
}

__global__ void __launch_bounds__(256) povs_travel_histogram_kernel(const __grid_constant__ MetricParams q)
{
    extern __shared__ uint32_t bins[];
    const bool staged = q.smem_bins > 0;
    if (staged) {
        for (int i = threadIdx.x; i < q.smem_bins; i += blockDim.x) bins[i] = 0;
        __syncthreads();
    }
    const int64_t total = q.n_episodes * q.deck;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t o = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; o < total; o += stride) {
        const int64_t e = o / q.deck;
        const int64_t i = o - e * q.deck;
        const int64_t v = metric_id(q, e, i);
        int64_t t;
        if (q.kind == 0) {
            t = floor_mod(i - v, q.deck);
        } else {
            const int64_t v1 = metric_id(q, e, floor_mod(i + q.step, q.deck));
            t = floor_mod((v1 - v) - q.step, q.deck);
        }
        if (staged)
            atomicAdd(&bins[t], 1u);
        else
            atomicAdd(&q.counts[t], 1ull);
    }
    if (staged) {
        __syncthreads();
        for (int i = threadIdx.x; i < q.smem_bins; i += blockDim.x)
            if (bins[i] != 0) atomicAdd(&q.counts[i], static_cast<unsigned long long>(bins[i]));
    }
}

// Key of observation o (episode o / per_episode, anchor o % per_episode).
__device__ __forceinline__ uint64_t ngram_key(const MetricParams& q, int64_t o, int64_t per_episode)
{
    const int64_t e = o / per_episode;
    const int64_t j = o - e * per_episode;
    const int64_t anchor = q.positions != nullptr ? floor_mod(q.positions[j], q.deck) : j;
    const int64_t v0 = metric_id(q, e, anchor);
    const uint64_t base = static_cast<uint64_t>(q.deck);
    uint64_t key = 0; // wraps modulo 2^64 like the reference's int64 key arithmetic
    for (int k = 1; k < q.kind; ++k) {
        const int64_t vk = metric_id(q, e, floor_mod(anchor + k * q.step, q.deck));
        key = key * base + static_cast<uint64_t>(floor_mod((vk - v0) - k * q.step, q.deck));
    }
    return key;
}

__global__ void __launch_bounds__(256) povs_ngram_keys_kernel(const __grid_constant__ MetricParams q)
{
    const int64_t per_episode = q.positions != nullptr ? q.n_positions : q.deck;
    const int64_t total = q.n_episodes * per_episode;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t o = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; o < total; o += stride)
        q.keys[o] = static_cast<int64_t>(ngram_key(q, o, per_episode));
}

// ---------------------------------------------------------------------------------------------
// Distinct n-gram keys and their counts without sorting: an open-addressing hash table in global
// memory (keys[slots] then counts[slots + 1]; the extra count is for the one key value that marks
// an empty slot), linear probing from a 64-bit mix of the key, then the multiplicities of the counts.
// ---------------------------------------------------------------------------------------------

constexpr unsigned long long NGRAM_EMPTY = ~0ull;

struct NgramTable {
    unsigned long long* keys;   // slots entries, NGRAM_EMPTY when free
    unsigned long long* counts; // slots + 1 entries
    int64_t slots;              // a power of two, more than the distinct keys
    unsigned long long* mult;   // mult[c]: distinct keys seen exactly c times (1 <= c < mult_bins);
                                // mult[0]: distinct keys seen mult_bins times or more
    int64_t mult_bins;
    unsigned long long* overflow; // counts of the keys tallied in mult[0], first overflow_cap of them
    int64_t overflow_cap;
    int* status;                  // device status word: DEV_ERR_TABLE_FULL if a key found no free slot
};

// A 64-bit finaliser (xor-shift / multiply rounds) spreading keys over the table.
__device__ __forceinline__ uint64_t mix64(uint64_t x)
{
    x ^= x >> 31;
    x *= 0x7fb5d329728ea185ull;
    x ^= x >> 27;
    x *= 0x81dadef4bc2dd44dull;
    x ^= x >> 33;
    return x;
}

__global__ void __launch_bounds__(256) povs_ngram_table_clear_kernel(NgramTable t)
{
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    const int64_t n = t.slots + 1 > t.mult_bins ? t.slots + 1 : t.mult_bins;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
        if (i < t.slots) t.keys[i] = NGRAM_EMPTY;
        if (i <= t.slots) t.counts[i] = 0;
        if (i < t.mult_bins) t.mult[i] = 0;
    }
}

__global__ void __launch_bounds__(256) povs_ngram_count_kernel(const __grid_constant__ MetricParams q, NgramTable t)
{
    const int64_t per_episode = q.positions != nullptr ? q.n_positions : q.deck;
    const int64_t total = q.n_episodes * per_episode;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    const uint64_t mask = static_cast<uint64_t>(t.slots) - 1;
    for (int64_t o = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; o < total; o += stride) {
        const unsigned long long key = ngram_key(q, o, per_episode);
        if (key == NGRAM_EMPTY) {
            atomicAdd(&t.counts[t.slots], 1ull);
            continue;
        }
        uint64_t h = mix64(key) & mask;
        bool placed = false;
        for (int64_t probe = 0; probe < t.slots; ++probe) {
            unsigned long long k = t.keys[h];
            if (k == NGRAM_EMPTY) k = atomicCAS(&t.keys[h], NGRAM_EMPTY, key);
            if (k == NGRAM_EMPTY || k == key) {
                atomicAdd(&t.counts[h], 1ull);
                placed = true;
                break;
            }
            h = (h + 1) & mask;
        }
        if (!placed) atomicOr(t.status, DEV_ERR_TABLE_FULL);
    }
}

__global__ void __launch_bounds__(256) povs_ngram_tally_kernel(NgramTable t)
{
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i <= t.slots; i += stride) {
        const unsigned long long c = t.counts[i];
        if (c == 0) continue;
        if (c < static_cast<unsigned long long>(t.mult_bins)) {
            atomicAdd(&t.mult[c], 1ull);
        } else {
            const unsigned long long at = atomicAdd(&t.mult[0], 1ull);
            if (at < static_cast<unsigned long long>(t.overflow_cap)) t.overflow[at] = c;
        }
    }
}

} // namespace povs
