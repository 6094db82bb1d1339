// One POV-shuffle iteration over a deck resident in HBM, for sm_100a.
//
// Reference semantics (src/povs/__cuda/lib/povs.cu:116-349, one CTA per vblock there):
//   * logical row L lives at storage row (L + offset) mod N;
//   * pblock b covers logical rows [b*P, min((b+1)*P, N));
//   * the V member pblocks of a vblock are ordered ascending with padding last
//     (povs.cu:203-221), which puts a truncated last pblock at the end and keeps
//     the slots 0..n_valid-1 gap free;
//   * slot f = r*P + i is row i of the r-th member; after the iteration
//     slot f holds what slot perm[f] held before (povs.cu:325-348).
//
// B200 design.  The kernel is persistent and every warp is an independent
// worker with its own ring of shared-memory stages.  For a work unit (one
// vblock, or one column slab of one vblock when V*P rows do not fit a stage)
// the warp
//   1. computes the member pblocks (device Feistel bijection, or the injected
//      assignment), orders them and derives each member's storage run;
//   2. issues cp.async.bulk (TMA, non-multicast, local HBM only) copies of the
//      <= 2 wrapped runs per member into the stage, completing on an mbarrier;
//   3. builds the permutation of the unit's rows with a register bitonic sort
//      of Philox keys over warp shuffles (or copies the injected one);
//   4. once the stage's mbarrier flips, writes every destination row from
//      shared memory with 16-byte vector stores, lanes covering consecutive
//      bytes of consecutive destination rows (full 128-byte lines).
// Steps 1-3 of unit j+NST-1 overlap the loads in flight for units j..j+NST-2.
// Rows whose size is not a multiple of 16 bytes (or decks that are not 16-byte
// aligned) take the same pipeline with plain vector loads of the widest
// aligned width instead of TMA.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "povs_rng.cuh"

namespace povs {

constexpr int MAX_INLINE_OFFSETS = 256;
constexpr int MAX_VBLOCK = 32;
constexpr unsigned FULL_MASK = 0xffffffffu;

// Device status bits (sticky, OR-ed into the per-device status word).
enum : int {
    DEV_ERR_WAIT_TIMEOUT = 1, // an mbarrier wait gave up after the time limit
    DEV_ERR_BAD_INJECTED = 2, // an injected permutation entry was out of range (identity used instead)
};

constexpr unsigned long long WAIT_LIMIT_NS = 2000000000ull; // 2 s: far beyond any legitimate copy

struct IterParams {
    uint8_t* data;
    int64_t n_rows;    // N
    int64_t row_bytes; // R
    int64_t n_pblocks; // ceil(N / P)
    int64_t n_vblocks; // ceil(n_pblocks / V)
    int32_t pblock;    // P, power of two
    int32_t pblock_shift;
    int32_t vblock; // V, power of two <= MAX_VBLOCK
    int32_t vp;     // V * P
    int32_t slab_bytes; // S: bytes of each row staged per unit (== R when rows fit)
    int32_t n_slabs;    // ceil(R / S)
    int32_t stage_bytes;   // bytes of one data stage (>= vp * S, 128-aligned)
    int32_t n_stages;      // NST
    int32_t warp_bytes;    // bytes of shared memory owned by one warp
    int32_t vec_bytes;     // chunk width of the plain-load path (1, 2, 4, 8 or 16)
    uint32_t iteration;
    uint64_t seed;
    int32_t n_offsets;
    int32_t sort_members; // injected mode: 1 = ascending, padding last (CUDA path); 0 = given order (NumPy path)
    int64_t offset;       // injected mode: this iteration's offset
    const int64_t* assign; // injected mode: [n_vblocks][V] pblock ids, padding < 0 or >= n_pblocks
    const int32_t* perms;  // injected mode: [n_vblocks][V*P] source slot of each destination slot
    int* status;
    int64_t offsets[MAX_INLINE_OFFSETS];
};

// ---------------------------------------------------------------------------------------------
// PTX wrappers (mbarrier + bulk async copy).
// ---------------------------------------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_addr(const void* p)
{
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init()
{
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok)
                 : "r"(smem_addr(bar)), "r"(parity)
                 : "memory");
    return ok != 0;
}

__device__ __forceinline__ void bulk_load(void* dst_smem, const void* src_gmem, uint32_t bytes, uint64_t* bar)
{
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_addr(dst_smem)),
                 "l"(src_gmem), "r"(bytes), "r"(smem_addr(bar))
                 : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem()
{
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ unsigned long long global_timer_ns()
{
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Warp-uniform bounded wait on one phase of a stage barrier.  Returns false (and
// records DEV_ERR_WAIT_TIMEOUT) if the phase did not complete within the limit.
__device__ __forceinline__ bool warp_wait_stage(uint64_t* bar, uint32_t parity, int* status)
{
    if (__all_sync(FULL_MASK, mbar_try_wait(bar, parity))) return true;
    const unsigned long long t0 = global_timer_ns();
    while (true) {
        if (__all_sync(FULL_MASK, mbar_try_wait(bar, parity))) return true;
        const unsigned long long dt = __shfl_sync(FULL_MASK, global_timer_ns() - t0, 0);
        if (dt > WAIT_LIMIT_NS) {
            if ((threadIdx.x & 31) == 0) atomicOr(status, DEV_ERR_WAIT_TIMEOUT);
            return false;
        }
    }
}

// ---------------------------------------------------------------------------------------------
// Register bitonic sort over one warp: n = 32 * EPL 64-bit values, lane l owns
// elements l*EPL .. l*EPL+EPL-1.  Ascending.
// ---------------------------------------------------------------------------------------------

template <int EPL>
__device__ __forceinline__ void warp_bitonic_sort(uint64_t (&x)[EPL], int lane)
{
    constexpr int N = 32 * EPL;
#pragma unroll
    for (int k = 2; k <= N; k <<= 1) {
#pragma unroll
        for (int j = k >> 1; j > 0; j >>= 1) {
            if (j >= EPL) {
                const int lm = j / EPL;
#pragma unroll
                for (int r = 0; r < EPL; ++r) {
                    const uint64_t y = __shfl_xor_sync(FULL_MASK, x[r], lm);
                    const int e = lane * EPL + r;
                    const bool up = (e & k) == 0;
                    const bool lower = (e & j) == 0;
                    const bool take_min = (lower == up);
                    const uint64_t lo = x[r] < y ? x[r] : y;
                    const uint64_t hi = x[r] < y ? y : x[r];
                    x[r] = take_min ? lo : hi;
                }
            } else {
#pragma unroll
                for (int r = 0; r < EPL; ++r) {
                    if ((r & j) == 0) {
                        const int e = lane * EPL + r;
                        const bool up = (e & k) == 0;
                        const uint64_t a = x[r], b = x[r | j];
                        const bool swap = up ? (a > b) : (a < b);
                        x[r] = swap ? b : a;
                        x[r | j] = swap ? a : b;
                    }
                }
            }
        }
    }
}

// Generates the permutation of one vblock: perm[f] = source slot of destination slot f, f < n_valid.
template <int EPL>
__device__ __forceinline__ void warp_make_perm(const IterParams& p, uint64_t vblock, int n_valid, uint16_t* perm,
                                               int lane)
{
    uint64_t x[EPL];
    if constexpr (EPL >= 4) {
#pragma unroll
        for (int q = 0; q < EPL / 4; ++q) {
            const uint32_t quad = static_cast<uint32_t>((lane * EPL) / 4 + q);
            const U32x4 k = perm_key4(p.seed, p.iteration, vblock, quad);
            const uint32_t w[4] = {k.x, k.y, k.z, k.w};
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const uint32_t e = quad * 4u + t;
                x[4 * q + t] = (static_cast<int>(e) < n_valid) ? ((static_cast<uint64_t>(w[t]) << 32) | e) : ~uint64_t{0};
            }
        }
    } else {
        const uint32_t e0 = static_cast<uint32_t>(lane * EPL);
        const U32x4 k = perm_key4(p.seed, p.iteration, vblock, e0 >> 2);
#pragma unroll
        for (int r = 0; r < EPL; ++r) {
            const uint32_t e = e0 + r;
            x[r] = (static_cast<int>(e) < n_valid) ? ((static_cast<uint64_t>(pick_word(k, static_cast<int>(e & 3u))) << 32) | e)
                                                   : ~uint64_t{0};
        }
    }
    warp_bitonic_sort<EPL>(x, lane);
#pragma unroll
    for (int r = 0; r < EPL; ++r) {
        const int f = lane * EPL + r;
        if (f < n_valid) perm[f] = static_cast<uint16_t>(x[r] & 0xffffu);
    }
}

// ---------------------------------------------------------------------------------------------
// Per-warp shared-memory layout.
// ---------------------------------------------------------------------------------------------

struct StageMeta {
    int64_t start[MAX_VBLOCK]; // storage row of the first row of the r-th ordered member
    int32_t n_valid;           // valid rows (slots) of the unit
    int32_t pad;
};

struct WarpSmem {
    uint8_t* data;     // n_stages * stage_bytes
    uint16_t* perm;    // n_stages * vp
    StageMeta* meta;   // n_stages
    uint64_t* bars;    // n_stages
};

__host__ __device__ inline int perm_bytes_per_stage(int vp) { return ((vp * 2 + 15) / 16) * 16; }

__host__ __device__ inline int warp_smem_bytes(int n_stages, int stage_bytes, int vp)
{
    const int bytes = n_stages * stage_bytes + n_stages * perm_bytes_per_stage(vp) +
                      n_stages * static_cast<int>(sizeof(StageMeta)) + n_stages * 8;
    return ((bytes + 127) / 128) * 128;
}

__device__ __forceinline__ WarpSmem carve_warp_smem(uint8_t* base, const IterParams& p)
{
    WarpSmem w;
    w.data = base;
    uint8_t* q = base + static_cast<size_t>(p.n_stages) * p.stage_bytes;
    w.perm = reinterpret_cast<uint16_t*>(q);
    q += static_cast<size_t>(p.n_stages) * perm_bytes_per_stage(p.vp);
    w.meta = reinterpret_cast<StageMeta*>(q);
    q += static_cast<size_t>(p.n_stages) * sizeof(StageMeta);
    w.bars = reinterpret_cast<uint64_t*>(q);
    return w;
}

// ---------------------------------------------------------------------------------------------
// Vector chunk copies of the plain-load path.
// ---------------------------------------------------------------------------------------------

template <int W>
struct VecOf;
template <>
struct VecOf<16> {
    using T = uint4;
};
template <>
struct VecOf<8> {
    using T = uint2;
};
template <>
struct VecOf<4> {
    using T = uint32_t;
};
template <>
struct VecOf<2> {
    using T = uint16_t;
};
template <>
struct VecOf<1> {
    using T = uint8_t;
};

__device__ __forceinline__ int64_t slot_row(const StageMeta& m, int f, int pshift, int pmask, int64_t n_rows)
{
    int64_t row = m.start[f >> pshift] + (f & pmask);
    if (row >= n_rows) row -= n_rows;
    return row;
}

// Identity-order copy global -> stage of the unit's valid rows (plain loads).
template <int W>
__device__ __forceinline__ void lsu_load_unit(const IterParams& p, const StageMeta& m, uint8_t* stage, int slab,
                                              int slen, int lane)
{
    using T = typename VecOf<W>::T;
    const int cpr = slen / W;
    const int pmask = p.pblock - 1;
    const int64_t col = static_cast<int64_t>(slab) * p.slab_bytes;
    const int n_valid = m.n_valid;
    if (cpr >= 32) {
        for (int f = 0; f < n_valid; ++f) {
            const int64_t row = slot_row(m, f, p.pblock_shift, pmask, p.n_rows);
            const T* src = reinterpret_cast<const T*>(p.data + row * p.row_bytes + col);
            T* dst = reinterpret_cast<T*>(stage + static_cast<size_t>(f) * p.slab_bytes);
            for (int q = lane; q < cpr; q += 32) dst[q] = src[q];
        }
    } else {
        const int g = 32 / cpr;
        const int lrow = lane / cpr, lq = lane - lrow * cpr;
        if (lrow < g) {
            for (int f = lrow; f < n_valid; f += g) {
                const int64_t row = slot_row(m, f, p.pblock_shift, pmask, p.n_rows);
                const T* src = reinterpret_cast<const T*>(p.data + row * p.row_bytes + col);
                T* dst = reinterpret_cast<T*>(stage + static_cast<size_t>(f) * p.slab_bytes);
                dst[lq] = src[lq];
            }
        }
    }
}

// Permuted copy stage -> global: destination slot f receives source slot perm[f].
template <int W>
__device__ __forceinline__ void store_unit(const IterParams& p, const StageMeta& m, const uint8_t* stage,
                                           const uint16_t* perm, int slab, int slen, int lane)
{
    using T = typename VecOf<W>::T;
    const int cpr = slen / W;
    const int pmask = p.pblock - 1;
    const int64_t col = static_cast<int64_t>(slab) * p.slab_bytes;
    const int n_valid = m.n_valid;
    if (cpr >= 32) {
        for (int f = 0; f < n_valid; ++f) {
            const int64_t row = slot_row(m, f, p.pblock_shift, pmask, p.n_rows);
            const T* src = reinterpret_cast<const T*>(stage + static_cast<size_t>(perm[f]) * p.slab_bytes);
            T* dst = reinterpret_cast<T*>(p.data + row * p.row_bytes + col);
#pragma unroll 4
            for (int q = lane; q < cpr; q += 32) dst[q] = src[q];
        }
    } else {
        const int g = 32 / cpr;
        const int lrow = lane / cpr, lq = lane - lrow * cpr;
        if (lrow < g) {
            constexpr int U = 4;
            int f = lrow;
            for (; f + (U - 1) * g < n_valid; f += U * g) {
                T v[U];
                int64_t rows[U];
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    const int fu = f + u * g;
                    rows[u] = slot_row(m, fu, p.pblock_shift, pmask, p.n_rows);
                    v[u] = reinterpret_cast<const T*>(stage + static_cast<size_t>(perm[fu]) * p.slab_bytes)[lq];
                }
#pragma unroll
                for (int u = 0; u < U; ++u) reinterpret_cast<T*>(p.data + rows[u] * p.row_bytes + col)[lq] = v[u];
            }
            for (; f < n_valid; f += g) {
                const int64_t row = slot_row(m, f, p.pblock_shift, pmask, p.n_rows);
                const T v = reinterpret_cast<const T*>(stage + static_cast<size_t>(perm[f]) * p.slab_bytes)[lq];
                reinterpret_cast<T*>(p.data + row * p.row_bytes + col)[lq] = v;
            }
        }
    }
}

template <int W>
__device__ __forceinline__ void store_unit_dispatch(const IterParams& p, const StageMeta& m, const uint8_t* stage,
                                                    const uint16_t* perm, int slab, int slen, int lane)
{
    store_unit<W>(p, m, stage, perm, slab, slen, lane);
}

// ---------------------------------------------------------------------------------------------
// The iteration kernel.
// EPL: elements per lane of the permutation sort (32 * EPL >= V * P).
// INJECTED: members, permutation and offset come from the caller instead of the device RNG.
// BULK: rows are 16-byte multiples on a 16-byte aligned deck -> TMA bulk loads.
// ---------------------------------------------------------------------------------------------

template <int EPL, bool INJECTED, bool BULK>
__global__ void __launch_bounds__(512) povs_iteration_kernel(const __grid_constant__ IterParams p)
{
    extern __shared__ __align__(128) uint8_t smem_raw[];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int warps_per_cta = blockDim.x >> 5;
    WarpSmem ws = carve_warp_smem(smem_raw + static_cast<size_t>(warp) * p.warp_bytes, p);

    if (BULK) {
        if (lane < p.n_stages) mbar_init(&ws.bars[lane], 1);
        mbar_fence_init();
    }
    __syncwarp();

    // Iteration-wide randomness.
    int64_t offset;
    if constexpr (INJECTED) {
        offset = p.offset;
    } else {
        offset = p.offsets[reduce_range(offset_draw(p.seed, p.iteration), static_cast<uint32_t>(p.n_offsets))];
    }
    Feistel pi;
    if constexpr (!INJECTED) pi.init(p.seed, p.iteration, static_cast<uint64_t>(p.n_vblocks) * p.vblock);

    const int64_t gw = static_cast<int64_t>(blockIdx.x) * warps_per_cta + warp;
    const int64_t total_warps = static_cast<int64_t>(gridDim.x) * warps_per_cta;
    if (gw >= p.n_vblocks) return;
    const int64_t my_vblocks = (p.n_vblocks - gw + total_warps - 1) / total_warps;
    const int64_t n_units = my_vblocks * p.n_slabs;
    const int nst = p.n_stages;
    const int pmask = p.pblock - 1;

    // Prepares unit j in stage j % nst: metadata, permutation, and (bulk path) the async loads.
    auto issue = [&](int64_t j) {
        const int st = static_cast<int>(j % nst);
        const int64_t v = gw + (j / p.n_slabs) * total_warps;
        const int slab = static_cast<int>(j % p.n_slabs);
        StageMeta& m = ws.meta[st];
        uint16_t* perm = ws.perm + static_cast<size_t>(st) * (perm_bytes_per_stage(p.vp) / 2);
        if (slab == 0) {
            int64_t mem = -1;
            if (lane < p.vblock) {
                const int64_t slot = v * p.vblock + lane;
                int64_t a;
                if constexpr (INJECTED) {
                    a = p.assign[slot];
                } else {
                    a = static_cast<int64_t>(pi(static_cast<uint64_t>(slot)));
                }
                mem = (a >= 0 && a < p.n_pblocks) ? a : -1;
            }
            const bool valid = mem >= 0;
            int rows = 0;
            if (valid) {
                const int64_t left = p.n_rows - mem * p.pblock;
                rows = left < p.pblock ? static_cast<int>(left) : p.pblock;
            }
            // Ordering key: ascending member ids with padding last (CUDA path), or the given order
            // with padding last and a truncated member moved behind the full ones (NumPy path).
            uint64_t key;
            if (lane >= p.vblock) {
                key = ~uint64_t{0};
            } else if (!INJECTED || p.sort_members) {
                key = valid ? static_cast<uint64_t>(mem) : ((uint64_t{1} << 63) | static_cast<uint64_t>(lane));
            } else {
                key = static_cast<uint64_t>(lane) + (valid ? (rows == p.pblock ? 0u : 64u) : 128u);
            }
            int rank = 0;
            for (int l2 = 0; l2 < p.vblock; ++l2) {
                const uint64_t k2 = __shfl_sync(FULL_MASK, key, l2);
                rank += (k2 < key || (k2 == key && l2 < lane)) ? 1 : 0;
            }
            const int n_valid = __reduce_add_sync(FULL_MASK, rows);
            if (lane < p.vblock && valid) {
                int64_t s0 = mem * p.pblock + offset;
                if (s0 >= p.n_rows) s0 -= p.n_rows;
                m.start[rank] = s0;
            }
            if (lane == 0) m.n_valid = n_valid;
            if constexpr (INJECTED) {
                const int32_t* src = p.perms + v * static_cast<int64_t>(p.vp);
                for (int f = lane; f < n_valid; f += 32) {
                    int32_t sf = src[f];
                    if (sf < 0 || sf >= n_valid) {
                        atomicOr(p.status, DEV_ERR_BAD_INJECTED);
                        sf = f;
                    }
                    perm[f] = static_cast<uint16_t>(sf);
                }
            } else {
                warp_make_perm<EPL>(p, static_cast<uint64_t>(v), n_valid, perm, lane);
            }
        } else {
            // Same vblock as unit j-1, whose stage still holds its metadata and permutation.
            const int prev = static_cast<int>((j - 1) % nst);
            const StageMeta& pm = ws.meta[prev];
            const uint16_t* pp = ws.perm + static_cast<size_t>(prev) * (perm_bytes_per_stage(p.vp) / 2);
            if (lane < p.vblock) m.start[lane] = pm.start[lane];
            if (lane == 0) m.n_valid = pm.n_valid;
            for (int f = lane; f < pm.n_valid; f += 32) perm[f] = pp[f];
        }
        __syncwarp();
        const int n_valid = m.n_valid;
        const int64_t col = static_cast<int64_t>(slab) * p.slab_bytes;
        const int slen = static_cast<int>(min(static_cast<int64_t>(p.slab_bytes), p.row_bytes - col));
        uint8_t* stage = ws.data + static_cast<size_t>(st) * p.stage_bytes;
        if constexpr (BULK) {
            if (lane == 0) mbar_arrive_expect_tx(&ws.bars[st], static_cast<uint32_t>(n_valid) * static_cast<uint32_t>(slen));
            __syncwarp();
            if (p.n_slabs == 1) {
                // Whole rows: each member is <= 2 contiguous runs (split where the offset wraps).
                const int n_mem = (n_valid + pmask) >> p.pblock_shift;
                if (lane < n_mem) {
                    const int first = lane << p.pblock_shift;
                    const int rows = min(p.pblock, n_valid - first);
                    const int64_t s0 = m.start[lane];
                    const int64_t until_end = p.n_rows - s0;
                    const int n1 = until_end < rows ? static_cast<int>(until_end) : rows;
                    bulk_load(stage + static_cast<size_t>(first) * p.slab_bytes, p.data + s0 * p.row_bytes,
                              static_cast<uint32_t>(n1) * static_cast<uint32_t>(p.row_bytes), &ws.bars[st]);
                    if (rows > n1)
                        bulk_load(stage + static_cast<size_t>(first + n1) * p.slab_bytes, p.data,
                                  static_cast<uint32_t>(rows - n1) * static_cast<uint32_t>(p.row_bytes), &ws.bars[st]);
                }
            } else {
                for (int f = lane; f < n_valid; f += 32) {
                    const int64_t row = slot_row(m, f, p.pblock_shift, pmask, p.n_rows);
                    bulk_load(stage + static_cast<size_t>(f) * p.slab_bytes, p.data + row * p.row_bytes + col,
                              static_cast<uint32_t>(slen), &ws.bars[st]);
                }
            }
        }
    };

    auto consume = [&](int64_t j) -> bool {
        const int st = static_cast<int>(j % nst);
        const int slab = static_cast<int>(j % p.n_slabs);
        const StageMeta& m = ws.meta[st];
        const uint16_t* perm = ws.perm + static_cast<size_t>(st) * (perm_bytes_per_stage(p.vp) / 2);
        uint8_t* stage = ws.data + static_cast<size_t>(st) * p.stage_bytes;
        const int64_t col = static_cast<int64_t>(slab) * p.slab_bytes;
        const int slen = static_cast<int>(min(static_cast<int64_t>(p.slab_bytes), p.row_bytes - col));
        if constexpr (BULK) {
            if (!warp_wait_stage(&ws.bars[st], static_cast<uint32_t>((j / nst) & 1), p.status)) return false;
            store_unit<16>(p, m, stage, perm, slab, slen, lane);
        } else {
            switch (p.vec_bytes) {
            case 16:
                lsu_load_unit<16>(p, m, stage, slab, slen, lane);
                __syncwarp();
                store_unit<16>(p, m, stage, perm, slab, slen, lane);
                break;
            case 8:
                lsu_load_unit<8>(p, m, stage, slab, slen, lane);
                __syncwarp();
                store_unit<8>(p, m, stage, perm, slab, slen, lane);
                break;
            case 4:
                lsu_load_unit<4>(p, m, stage, slab, slen, lane);
                __syncwarp();
                store_unit<4>(p, m, stage, perm, slab, slen, lane);
                break;
            case 2:
                lsu_load_unit<2>(p, m, stage, slab, slen, lane);
                __syncwarp();
                store_unit<2>(p, m, stage, perm, slab, slen, lane);
                break;
            default:
                lsu_load_unit<1>(p, m, stage, slab, slen, lane);
                __syncwarp();
                store_unit<1>(p, m, stage, perm, slab, slen, lane);
                break;
            }
        }
        __syncwarp();
        // The stage is reused by a later async copy: order this warp's shared reads before it.
        fence_proxy_async_smem();
        return true;
    };

    const int64_t ahead = nst - 1;
    for (int64_t j = 0; j < ahead && j < n_units; ++j) issue(j);
    for (int64_t j = 0; j < n_units; ++j) {
        if (j + ahead < n_units) issue(j + ahead);
        if (!consume(j)) {
            // A stage never completed: stop, after giving the other in-flight stages the same bounded wait.
            if constexpr (BULK) {
                for (int64_t k = j + 1; k < n_units && k <= j + ahead; ++k)
                    warp_wait_stage(&ws.bars[k % nst], static_cast<uint32_t>((k / nst) & 1), p.status);
            }
            return;
        }
    }
}

} // namespace povs
