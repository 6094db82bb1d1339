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
// B200 design (warp-specialized persistent CTA).
//   * Permuter warps compute, for each unit (a vblock, or one column slab of a
//     vblock whose V*P rows do not fit a stage), the member pblocks (device
//     Feistel bijection, or the injected assignment), their order and storage
//     runs, and the permutation (register bitonic sort of Philox keys over warp
//     shuffles, or the injected one) into a ring of KP small slots, running up
//     to KP units ahead (mbarriers pfull / pempty).
//   * Mover warps own a ring of NST shared-memory data stages.  Unit u is issued
//     by mover u % n_movers: it waits for its permutation slot and for every
//     mover to have read the stage's previous unit (mbarrier `empty`), then
//     starts cp.async.bulk copies (non-multicast; from local HBM, or from a peer
//     GPU's shard in the sharded in-place order) of the <= 2 wrapped runs per
//     member into the stage, completing on `full`.
//     Every mover then takes its share of every unit: it waits for `full` and
//     writes its destination rows from shared memory with 16-byte vector stores
//     (lanes cover consecutive bytes of consecutive destination rows, so each
//     warp store is 4 full 128-byte lines), and arrives on `empty` and `pempty`.
//     Issuing runs NST-1 units ahead, so NST-1 stages are normally loading while
//     one is being written.
// Rows whose size is not a multiple of 16 bytes (or decks that are not 16-byte
// aligned) take the same pipeline with plain vector loads by the issuing mover.
//
// Every wait is bounded (WAIT_LIMIT_NS); a wait that gives up records
// DEV_ERR_WAIT_TIMEOUT in the status word, waits once more (bounded) for the
// copies this warp started, and the warp returns.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "povs_rng.cuh"

// Cache-hint variants of the data path, off: on B200 both were slower (32 GiB bf16 and 256 MiB fp16
// decks, same box: streaming stores -7 to -10 %, evict-first bulk loads about -1 %; neutral on 12 KiB
// and 64-byte rows).
#ifndef POVS_LOAD_EVICT_FIRST
#define POVS_LOAD_EVICT_FIRST 0
#endif
#ifndef POVS_STREAM_STORES
#define POVS_STREAM_STORES 0
#endif

namespace povs {

constexpr int MAX_INLINE_OFFSETS = 256;
constexpr int MAX_VBLOCK = 32;
constexpr int MAX_STAGES = 16;
constexpr int MAX_SLOTS = 32;
constexpr int MAX_SHARDS = 8;
constexpr unsigned FULL_MASK = 0xffffffffu;
constexpr uint16_t HOLE = 0xFFFFu; // packed units: a destination slot past its vblock's valid rows

// Device status bits (sticky, OR-ed into the per-device status word).
enum : int {
    DEV_ERR_WAIT_TIMEOUT = 1, // an mbarrier wait gave up after the time limit
    DEV_ERR_BAD_INJECTED = 2, // an injected permutation entry was out of range (identity used instead)
    DEV_ERR_PEER_TIMEOUT = 4, // a cross-GPU barrier gave up waiting for a peer
    DEV_ERR_TABLE_FULL = 8,   // an n-gram count table had no free slot for a key (key not counted)
};

constexpr unsigned long long PEER_WAIT_LIMIT_NS = 20000000000ull; // default: 20 s for a peer GPU to reach the barrier

constexpr unsigned long long WAIT_LIMIT_NS = 2000000000ull; // 2 s: far beyond any legitimate wait

struct IterParams {
    uint8_t* data;
    int64_t n_rows;    // N
    int64_t row_bytes; // R
    int64_t n_pblocks; // ceil(N / P)
    int64_t n_vblocks; // ceil(n_pblocks / V)
    int32_t pblock;    // P, power of two
    int32_t pblock_shift;
    int32_t vblock;     // V, power of two <= MAX_VBLOCK
    int32_t vp;         // V * P
    int32_t slab_bytes; // S: bytes of each row staged per unit (== R when rows fit)
    int32_t n_slabs;    // ceil(R / S)
    int32_t stage_bytes; // bytes of one data stage (>= vp * S, 128-aligned)
    int32_t n_stages;    // NST
    int32_t vec_bytes;   // chunk width of the plain-load path (1, 2, 4, 8 or 16)
    int32_t copy_rows;   // whole-row path: rows per bulk copy (runs are split into pieces this long)
    int32_t n_slots;     // KP: permutation slots in the CTA's permutation ring
    int32_t n_movers;    // warps that issue copies and write rows
    int32_t n_permuters; // warps that compute members and permutations
    uint32_t iteration;
    uint64_t seed;
    int32_t n_offsets;
    int32_t sort_members; // injected mode: 1 = ascending, padding last (CUDA path); 0 = given order (NumPy path)
    int32_t rng_mode;     // RNG_UNIFORM, RNG_REFERENCE_CUDA or RNG_REFERENCE_NUMPY (device randomness only)
    int64_t offset;       // injected mode: this iteration's offset
    const int64_t* assign; // injected mode: [n_vblocks][V] pblock ids, padding < 0 or >= n_pblocks
    const int32_t* perms;  // injected mode: [n_vblocks][V*P] source slot of each destination slot
    int* status;
    // The deck as a table of shards: rows [shard_start[s], shard_start[s+1]) live at shard_base[s]
    // (one shard for a single-GPU deck; the shards of other GPUs are peer addresses).
    int32_t n_shards;
    uint8_t* shard_base[MAX_SHARDS];
    int64_t shard_start[MAX_SHARDS + 1];
    // vblocks handled by this launch: vb_begin, vb_begin + vb_step, ...
    int64_t vb_begin;
    int64_t vb_step;
    // Push mode (double-buffered decks): rows are read from shard_base and written to dst_base.
    // A launch moves the pblocks whose first storage row lies in shard push_rank (all pblocks if -1).
    uint8_t* dst_base[MAX_SHARDS];
    int32_t push_rank;
    // Batched decks (device randomness, in place, one shard): n_decks independent decks of the same
    // geometry at data + d * deck_stride, deck d shuffled with seed deck_seeds[d] (device array).
    // n_decks == 1: the single deck of `data` with `seed`.
    int64_t n_decks;
    int64_t deck_stride;
    const uint64_t* deck_seeds;
    // Packed units (small vblocks): a unit is `pack` consecutive vblocks of one deck (pack == 1: one
    // vblock, or one column slab of it).  Unit slot f = s * vp + (slot of the s-th vblock), so the
    // unit has unit_vp = pack * vp slots; slots past a vblock's valid rows are holes.
    int32_t async_plain;     // plain-load path: asynchronous copies (whole rows, 4-byte multiples)
    // RNG_REFERENCE_NUMPY: the permutation of a vblock of n valid rows drawing seed s (1..999) is
    // np_table[np_off[class(n)] + (s - 1) * n + f], f < n, where class(n) = n / P - 1 for whole
    // members and V + (n - np_trunc) / P when the deck's truncated last pblock is one of them.
    const uint16_t* np_table;
    int32_t np_trunc;        // n_rows % P
    int64_t np_off[2 * MAX_VBLOCK];
    int32_t pack;
    int32_t unit_vp;
    int32_t vp_shift;        // log2(vp)
    int32_t vblock_shift;    // log2(V)
    int32_t idx_bits;        // index bits of a vblock's permutation sort keys: max(5, log2(vp))
    int64_t groups_per_deck; // ceil(n_vblocks / pack)
    // Packed units of plain-loaded rows (R a multiple of 4, R < 128) launched with the CHUNK kernels:
    // stores go out as 16-byte chunks of each member's destination run (store_unit_chunked);
    // row_magic = ceil(2^32 / R).
    int32_t chunked_store;
    uint32_t row_magic;
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

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes)
{
    asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar)
{
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
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

// Same, but the thread may sleep up to `hint_ns` waiting for the phase instead of returning at once.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns)
{
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok)
                 : "r"(smem_addr(bar)), "r"(parity), "r"(hint_ns)
                 : "memory");
    return ok != 0;
}

__device__ __forceinline__ void bulk_load(void* dst_smem, const void* src_gmem, uint32_t bytes, uint64_t* bar)
{
#if POVS_LOAD_EVICT_FIRST
    uint64_t policy;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_addr(dst_smem)),
        "l"(src_gmem), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
#else
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_addr(dst_smem)),
                 "l"(src_gmem), "r"(bytes), "r"(smem_addr(bar))
                 : "memory");
#endif
}

// Row stores of the write-back pass (POVS_STREAM_STORES: streaming cache hint).
template <typename T>
__device__ __forceinline__ void store_row_chunk(T* dst, const T& v)
{
#if POVS_STREAM_STORES
    if constexpr (sizeof(T) == 16) {
        __stcs(reinterpret_cast<uint4*>(dst), *reinterpret_cast<const uint4*>(&v));
        return;
    }
#endif
    *dst = v;
}

// Per-thread asynchronous copies global -> shared of 4 or 8 bytes (both addresses aligned to the
// size), and the arrival of this thread on `bar` once all of its earlier such copies have landed
// (.noinc: the arrival counts as one of the barrier's expected arrivals).
__device__ __forceinline__ void cp_async4(void* dst_smem, const void* src)
{
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_addr(dst_smem)), "l"(src) : "memory");
}

__device__ __forceinline__ void cp_async8(void* dst_smem, const void* src)
{
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_addr(dst_smem)), "l"(src) : "memory");
}

__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t* bar)
{
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Programmatic dependent launch: the next kernel of a chain may start its CTAs (set-up and
// permutations, which read no data) while this grid drains; its movers wait for this grid's
// completion and memory flush before touching the deck.  Both are no-ops for ordinary launches.
__device__ __forceinline__ void allow_dependent_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void wait_for_prior_grid() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

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

// Warp-uniform bounded wait on one phase of a barrier.  Returns false (and records
// DEV_ERR_WAIT_TIMEOUT) if the phase did not complete within the limit.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int* status)
{
    if (__all_sync(FULL_MASK, mbar_try_wait(bar, parity))) return true;
    const unsigned long long t0 = global_timer_ns();
    while (true) {
        // Sleeping waits leave the issue slots to the warps that have work.
        if (__all_sync(FULL_MASK, mbar_try_wait_sleep(bar, parity, 20000u))) return true;
        const unsigned long long dt = __shfl_sync(FULL_MASK, global_timer_ns() - t0, 0);
        if (dt > WAIT_LIMIT_NS) {
            if ((threadIdx.x & 31) == 0) atomicOr(status, DEV_ERR_WAIT_TIMEOUT);
            return false;
        }
    }
}

// ---------------------------------------------------------------------------------------------
// Register sorting networks over one warp: n = 32 * EPL values (T = uint32_t), lane l owns
// elements l*EPL .. l*EPL+EPL-1.  Ascending.
// ---------------------------------------------------------------------------------------------

// Ascending compare-exchange of registers r < s: the smaller key goes to r.
template <int EPL, typename T>
__device__ __forceinline__ void cx_asc(T (&x)[EPL], int r, int s)
{
    const T a = x[r], b = x[s];
    x[r] = min(a, b);
    x[s] = max(a, b);
}

// Sorts every aligned block of `seg` elements ascending (seg a power of two, 2 <= seg <= 32 * EPL);
// element e = lane * EPL + r is register r of lane `lane`, and elements of different blocks are
// never compared.  Every comparator keeps the smaller key at the lower index.  Blocks inside a
// lane are sorted by a fixed network of register pairs (a min and a max each); larger blocks by
// bitonic merging in the form whose comparators all point one way (Batcher's network with the
// first stage of every merge mirrored): phase k = 2 EPL, .., seg compares element e with
// e ^ (k - 1), its mirror image inside its block of k (which merges two ascending halves without
// reversing one of them), then with e ^ j for j = k/4, .., 1; across lanes a stage is one shuffle
// per register.  The keys are distinct, so the order equals that of any other correct sort.
template <int EPL, typename T>
__device__ __forceinline__ void warp_sort_blocks(T (&x)[EPL], int lane, int seg)
{
    // Blocks of up to EPL elements, inside each lane's registers: Batcher's odd-even merge sort,
    // cut after its merges into blocks of min(seg, EPL) (191 comparators for 32 elements where the
    // bitonic network takes 240).  Merge of blocks of pp into 2 pp: distances kk = pp, pp/2, .., 1;
    // element a meets a + kk when a - (kk mod pp) lies in the lower half of a run of 2 kk and both
    // are in the same block of 2 pp.
    // Loops of fixed trip counts, so that every register index is a compile-time constant.
    constexpr int LOG_EPL = EPL >= 32 ? 5 : EPL >= 16 ? 4 : EPL >= 8 ? 3 : EPL >= 4 ? 2 : EPL >= 2 ? 1 : 0;
#pragma unroll
    for (int lp = 0; lp < LOG_EPL; ++lp) {
        const int pp = 1 << lp;
        if (2 * pp <= seg) {
#pragma unroll
            for (int lk = lp; lk >= 0; --lk) {
                const int kk = 1 << lk;
                const int j0 = kk % pp;
#pragma unroll
                for (int a = 0; a < EPL; ++a) {
                    const int b = a + kk;
                    if (a >= j0 && (a - j0) % (2 * kk) < kk && b < EPL && a / (2 * pp) == b / (2 * pp))
                        cx_asc<EPL, T>(x, a, b);
                }
            }
        }
    }
    // Phases k = 2 * EPL .. seg: blocks of lk = k / EPL lanes (a runtime loop keeps the code small).
#pragma unroll 1
    for (int k = 2 * EPL; k <= seg; k <<= 1) {
        const int lk = k / EPL;
        const bool low = (lane & (lk >> 1)) == 0; // this lane holds the lower half of its block
        // Mirror stage: register r pairs with register EPL - 1 - r of lane ^ (lk - 1).
        if constexpr (EPL == 1) {
            const T y = __shfl_xor_sync(FULL_MASK, x[0], lk - 1);
            x[0] = low ? min(x[0], y) : max(x[0], y);
        } else {
#pragma unroll
            for (int r = 0; r < EPL / 2; ++r) {
                const int s = EPL - 1 - r;
                const T ya = __shfl_xor_sync(FULL_MASK, x[s], lk - 1);
                const T yb = __shfl_xor_sync(FULL_MASK, x[r], lk - 1);
                x[r] = low ? min(x[r], ya) : max(x[r], ya);
                x[s] = low ? min(x[s], yb) : max(x[s], yb);
            }
        }
        // Distances j = k/4 .. EPL: register r with the same register of lane ^ (j / EPL).
#pragma unroll 1
        for (int lm = lk >> 2; lm >= 1; lm >>= 1) {
            const bool keep_min = (lane & lm) == 0;
#pragma unroll
            for (int r = 0; r < EPL; ++r) {
                const T y = __shfl_xor_sync(FULL_MASK, x[r], lm);
                x[r] = keep_min ? min(x[r], y) : max(x[r], y);
            }
        }
        // Distances j = EPL/2 .. 1: inside the lane.
#pragma unroll
        for (int j = EPL >> 1; j > 0; j >>= 1) {
#pragma unroll
            for (int r = 0; r < EPL; ++r)
                if ((r & j) == 0) cx_asc<EPL, T>(x, r, r | j);
        }
    }
}

// All 32 * EPL elements of the warp in one ascending order.
template <int EPL, typename T>
__device__ __forceinline__ void warp_bitonic_sort(T (&x)[EPL], int lane)
{
    warp_sort_blocks<EPL, T>(x, lane, 32 * EPL);
}

// A lane's EPL consecutive uint16 entries (register r -> dst[r]) in as few stores as their
// alignment allows: dst is 2 * EPL-byte aligned (a permutation slot is 16-byte aligned and the
// lane's run starts at lane * EPL).  Lanes 64 bytes apart (EPL = 32) touch 2 bank groups per
// 16-byte store instead of 2 banks per 2-byte store.
template <int EPL>
__device__ __forceinline__ void store_u16_run(uint16_t* dst, const uint32_t (&v)[EPL])
{
    if constexpr (EPL == 1) {
        dst[0] = static_cast<uint16_t>(v[0]);
    } else if constexpr (EPL == 2) {
        *reinterpret_cast<uint32_t*>(dst) = (v[0] & 0xFFFFu) | (v[1] << 16);
    } else if constexpr (EPL == 4) {
        *reinterpret_cast<uint2*>(dst) = make_uint2((v[0] & 0xFFFFu) | (v[1] << 16), (v[2] & 0xFFFFu) | (v[3] << 16));
    } else {
#pragma unroll
        for (int c = 0; c < EPL / 8; ++c) {
            const uint32_t* w = v + 8 * c;
            *reinterpret_cast<uint4*>(dst + 8 * c) =
                make_uint4((w[0] & 0xFFFFu) | (w[1] << 16), (w[2] & 0xFFFFu) | (w[3] << 16),
                           (w[4] & 0xFFFFu) | (w[5] << 16), (w[6] & 0xFFFFu) | (w[7] << 16));
        }
    }
}

// Sort keys of a vblock's elements e = 0 .. 32*EPL-1: the element's 32-bit Philox word with its
// low IDX_BITS bits replaced by e (so keys are distinct and the sort is a permutation).  Elements
// past n_valid get all high bits set: they sort after every valid element (same high bits: the
// larger index).  The order of the valid keys is a uniformly random permutation except where two
// elements' high bits tie (probability below n^2 / 2^(33 - IDX_BITS) per vblock), whose relative
// order is then their index order.
template <int EPL>
struct PermKey {
    static constexpr int IDX_BITS = EPL >= 32 ? 10 : EPL >= 16 ? 9 : EPL >= 8 ? 8 : EPL >= 4 ? 7 : EPL >= 2 ? 6 : 5;
    static constexpr uint32_t IDX_MASK = (1u << IDX_BITS) - 1u;
};

template <int EPL>
__device__ __forceinline__ void perm_sort_keys(const IterParams& p, uint64_t seed, uint64_t vblock, int n_valid,
                                               uint32_t (&x)[EPL], int lane)
{
    constexpr uint32_t M = PermKey<EPL>::IDX_MASK;
    if constexpr (EPL >= 4) {
#pragma unroll
        for (int q = 0; q < EPL / 4; ++q) {
            const uint32_t quad = static_cast<uint32_t>((lane * EPL) / 4 + q);
            const U32x4 k = perm_key4(seed, p.iteration, vblock, quad);
            const uint32_t w[4] = {k.x, k.y, k.z, k.w};
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const uint32_t e = quad * 4u + t;
                x[4 * q + t] = ((static_cast<int>(e) < n_valid) ? (w[t] & ~M) : ~M) | e;
            }
        }
    } else {
        const uint32_t e0 = static_cast<uint32_t>(lane * EPL);
        const U32x4 k = perm_key4(seed, p.iteration, vblock, e0 >> 2);
#pragma unroll
        for (int r = 0; r < EPL; ++r) {
            const uint32_t e = e0 + r;
            x[r] = ((static_cast<int>(e) < n_valid) ? (pick_word(k, static_cast<int>(e & 3u)) & ~M) : ~M) | e;
        }
    }
}

// Generates the permutation of one vblock: perm[f] = source slot of destination slot f, f < n_valid.
template <int EPL>
__device__ __forceinline__ void warp_make_perm(const IterParams& p, uint64_t seed, uint64_t vblock, int n_valid,
                                               uint16_t* perm, int lane)
{
    uint32_t x[EPL];
    perm_sort_keys<EPL>(p, seed, vblock, n_valid, x, lane);
    warp_bitonic_sort<EPL, uint32_t>(x, lane);
#pragma unroll
    for (int r = 0; r < EPL; ++r) x[r] &= PermKey<EPL>::IDX_MASK;
    // Entries n_valid .. vp-1 get the invalid elements' indices, which no mover reads; lanes past
    // the slot's vp entries (vp < 32, one entry per lane) store nothing.
    if (lane * EPL < p.unit_vp) store_u16_run<EPL>(perm + lane * EPL, x);
}

// The reference kernel's permutation (src/povs/__cuda/lib/povs.cu:282-321): identity over the
// gap-free slots 0..n_valid-1, then a forward Fisher-Yates on one thread with xorshift32
// (13, 17, 5) seeded by the vblock seed and Lemire's multiply-shift range reduction.
__device__ __forceinline__ void warp_make_perm_xorshift(const IterParams& p, uint64_t seed, uint64_t vblock,
                                                        int n_valid, uint16_t* perm, int lane)
{
    for (int f = lane; f < n_valid; f += 32) perm[f] = static_cast<uint16_t>(f);
    __syncwarp();
    if (lane == 0) {
        uint32_t r = vblock_seed(seed, p.iteration, vblock);
        const int last = n_valid - 1;
        for (int i = 0; i <= last; ++i) {
            r ^= r << 13;
            r ^= r >> 17;
            r ^= r << 5;
            const int j = i + static_cast<int>((static_cast<uint64_t>(r) * static_cast<uint64_t>(last - i + 1)) >> 32);
            const uint16_t t = perm[i];
            perm[i] = perm[j];
            perm[j] = t;
        }
    }
    __syncwarp();
}

// The reference NumPy path's permutation of a vblock of n valid rows under per-vblock seed s:
// numpy.random.RandomState(s).shuffle(arange(n)), precomputed on the host (povs_mt19937.h).
__device__ __forceinline__ const uint16_t* np_perm(const IterParams& p, int n, uint32_t s)
{
    const int cls = (n & (p.pblock - 1)) == 0 ? (n >> p.pblock_shift) - 1
                                              : p.vblock + ((n - p.np_trunc) >> p.pblock_shift);
    return p.np_table + p.np_off[cls] + static_cast<int64_t>(s - 1u) * n;
}

__device__ __forceinline__ void warp_copy_np_perm(const IterParams& p, uint64_t seed, uint64_t vblock, int n_valid,
                                                  uint16_t* perm, int lane)
{
    if (n_valid <= 0) return;
    const uint16_t* src = np_perm(p, n_valid, vblock_seed(seed, p.iteration, vblock));
    for (int f = lane; f < n_valid; f += 32) perm[f] = src[f];
    __syncwarp();
}

// ---------------------------------------------------------------------------------------------
// CTA shared-memory layout:
//   [NST data stages][KP permutations][KP metas][NST full][NST empty][KP pfull][KP pempty]
// Data stage u % NST and permutation slot u % KP belong to unit u.
// ---------------------------------------------------------------------------------------------

struct StageMeta {
    // Row i of the r-th ordered member is at (i < n_a[r] ? run_a[r] : run_b[r]) + i * row_bytes:
    // run_a is the member's first row, run_b is where the run continues past a shard or deck end,
    // pre-shifted back by n_a rows so that both cases index with i (a select, not a branch).
    uintptr_t run_a[MAX_VBLOCK];
    uintptr_t run_b[MAX_VBLOCK];
    int32_t n_a[MAX_VBLOCK]; // rows of the member stored contiguously from run_a
    int16_t mrows[MAX_VBLOCK]; // packed units: rows of every ordered member (0 = padding or no vblock)
    int32_t n_valid;         // valid rows (slots) of the unit
    int32_t rows_mine;       // push mode: rows of the unit's own member
    // push mode: the unit's own member in the source buffer, same (a, b, n_a) convention
    uintptr_t src_a;
    uintptr_t src_b;
    int32_t src_na;
    int32_t pad;
};

__host__ __device__ inline int perm_bytes_per_slot(int vp) { return ((vp * 2 + 15) / 16) * 16; }

__host__ __device__ inline int cta_smem_bytes(int n_stages, int stage_bytes, int n_slots, int vp, int pblock)
{
    return n_stages * stage_bytes +
           n_slots * (perm_bytes_per_slot(vp) + perm_bytes_per_slot(pblock) + static_cast<int>(sizeof(StageMeta))) +
           (2 * n_stages + 2 * n_slots) * 8;
}

struct CtaSmem {
    uint8_t* data;
    uint16_t* perm;   // per slot: source slot of every destination slot (in-place mode, and scratch)
    uint16_t* pos;    // per slot, push mode: destination slot of every row of the unit's own member
    StageMeta* meta;
    uint64_t* full;   // data stage loaded (TMA bytes + issuer arrivals)
    uint64_t* empty;  // data stage read by every mover thread
    uint64_t* pfull;  // permutation slot written by its permuter warp
    uint64_t* pempty; // permutation slot read by every mover thread
    int perm_stride;  // uint16 entries per slot
    int pos_stride;
};

__device__ __forceinline__ CtaSmem carve_smem(uint8_t* base, const IterParams& p)
{
    CtaSmem s;
    s.data = base;
    uint8_t* q = base + static_cast<size_t>(p.n_stages) * p.stage_bytes;
    s.perm = reinterpret_cast<uint16_t*>(q);
    s.perm_stride = perm_bytes_per_slot(p.unit_vp) / 2;
    q += static_cast<size_t>(p.n_slots) * perm_bytes_per_slot(p.unit_vp);
    s.pos = reinterpret_cast<uint16_t*>(q);
    s.pos_stride = perm_bytes_per_slot(p.pblock) / 2;
    q += static_cast<size_t>(p.n_slots) * perm_bytes_per_slot(p.pblock);
    s.meta = reinterpret_cast<StageMeta*>(q);
    q += static_cast<size_t>(p.n_slots) * sizeof(StageMeta);
    s.full = reinterpret_cast<uint64_t*>(q);
    s.empty = s.full + p.n_stages;
    s.pfull = s.empty + p.n_stages;
    s.pempty = s.pfull + p.n_slots;
    return s;
}

// ---------------------------------------------------------------------------------------------
// Vector chunks.
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

// Address of the first byte of destination/source slot f's row.
__device__ __forceinline__ uint8_t* slot_ptr(const StageMeta& m, int f, int pshift, int pmask, int64_t row_bytes)
{
    const int r = f >> pshift, i = f & pmask;
    const uintptr_t a = m.run_a[r], b = m.run_b[r];
    const uintptr_t base = i < m.n_a[r] ? a : b;
    return reinterpret_cast<uint8_t*>(base + static_cast<uintptr_t>(static_cast<int64_t>(i) * row_bytes));
}

// Push mode: row i of the unit's own member in the source buffer.
__device__ __forceinline__ const uint8_t* src_row_ptr(const StageMeta& m, int i, int64_t row_bytes)
{
    const uintptr_t base = i < m.src_na ? m.src_a : m.src_b;
    return reinterpret_cast<const uint8_t*>(base + static_cast<uintptr_t>(static_cast<int64_t>(i) * row_bytes));
}

// A slab of slen bytes per row as W-byte chunks over a warp: cpr chunks per row, g rows per warp
// instruction, lane -> (row lrow, chunk lq).  Shifts instead of divisions when cpr is a power of two.
struct LaneGeom {
    int cpr, g, lrow, lq, g_shift; // g_shift = log2(g), or -1 when g is not a power of two
    __device__ __forceinline__ int passes(int n) const { return g_shift >= 0 ? (n + g - 1) >> g_shift : (n + g - 1) / g; }
};

template <int W>
__device__ __forceinline__ LaneGeom lane_geom(int slen, int lane)
{
    LaneGeom lg;
    lg.cpr = slen / W;
    if (lg.cpr >= 32) {
        lg.g = 1;
        lg.lrow = 0;
        lg.lq = lane;
        lg.g_shift = 0;
    } else if ((lg.cpr & (lg.cpr - 1)) == 0) {
        const int cs = __ffs(lg.cpr) - 1;
        lg.g = 32 >> cs;
        lg.lrow = lane >> cs;
        lg.lq = lane & (lg.cpr - 1);
        lg.g_shift = 5 - cs;
    } else {
        lg.g = 32 / lg.cpr;
        lg.lrow = lane / lg.cpr;
        lg.lq = lane - lg.lrow * lg.cpr;
        lg.g_shift = -1;
    }
    return lg;
}

// Identity-order copy global -> stage by one warp (plain loads): the unit's valid rows (in place),
// or the rows of the unit's own member (push).  Several loads per lane are in flight.
template <int W, bool PUSH, bool PACK = false>
__device__ __forceinline__ void lsu_load_unit(const IterParams& p, const StageMeta& m, uint8_t* stage, int64_t col,
                                              int slen, int lane)
{
    using T = typename VecOf<W>::T;
    const LaneGeom lg = lane_geom<W>(slen, lane);
    const int pmask = p.pblock - 1;
    // Packed units: every slot of the unit, skipping the holes (rows past a member's row count).
    const int n = PACK ? p.unit_vp : (PUSH ? m.rows_mine : m.n_valid);
    auto live = [&](int f) -> bool {
        if constexpr (PACK) return (f & pmask) < m.mrows[f >> p.pblock_shift];
        else return true;
    };
    auto src_of = [&](int f) -> const uint8_t* {
        if constexpr (PUSH) return src_row_ptr(m, f, p.row_bytes) + col;
        else return slot_ptr(m, f, p.pblock_shift, pmask, p.row_bytes) + col;
    };
    if (lg.cpr >= 32) {
        for (int f = 0; f < n; ++f) {
            if (!live(f)) continue;
            const T* src = reinterpret_cast<const T*>(src_of(f));
            T* dst = reinterpret_cast<T*>(stage + static_cast<size_t>(f) * p.slab_bytes);
            for (int q = lane; q < lg.cpr; q += 32) dst[q] = src[q];
        }
    } else if (lg.lrow < lg.g) {
        constexpr int UL = W >= 8 ? 4 : 8; // loads in flight per lane (wide chunks cost registers)
        for (int f0 = lg.lrow; f0 < n; f0 += UL * lg.g) {
            T v[UL];
#pragma unroll
            for (int u = 0; u < UL; ++u) {
                const int f = f0 + u * lg.g;
                if (f < n && live(f)) v[u] = reinterpret_cast<const T*>(src_of(f))[lg.lq];
            }
#pragma unroll
            for (int u = 0; u < UL; ++u) {
                const int f = f0 + u * lg.g;
                if (f < n && live(f)) reinterpret_cast<T*>(stage + static_cast<size_t>(f) * p.slab_bytes)[lg.lq] = v[u];
            }
        }
    }
}

// One contiguous piece (len bytes, a multiple of 4; both addresses 4-byte aligned) global -> stage,
// asynchronously, by the whole warp.  When the two addresses agree modulo 16, the 16-byte aligned
// middle is one bulk copy (TMA, no multicast) issued by lane `piece % 32` after it registers the
// bytes on `bar`, and the unaligned head and tail (< 16 bytes each) are 4-byte copies; otherwise the
// piece goes as 8-byte copies (addresses agreeing modulo 8) or 4-byte copies spread over the lanes.
__device__ __forceinline__ void async_copy_piece(uint8_t* dst, uintptr_t src, uint32_t len, uint64_t* bar, int lane,
                                                 int piece)
{
    const uint32_t d = smem_addr(dst);
    const uint32_t mis = d ^ static_cast<uint32_t>(src);
    if ((mis & 15u) == 0) {
        const uint32_t head = min(len, (16u - (static_cast<uint32_t>(src) & 15u)) & 15u);
        const uint32_t body = (len - head) & ~15u;
        const uint32_t tail_at = head + body;
        if (body != 0 && lane == (piece & 31)) {
            mbar_expect_tx(bar, body);
            bulk_load(dst + head, reinterpret_cast<const void*>(src + head), body, bar);
        }
        const uint32_t n_head = head >> 2;
        const uint32_t n_tail = (len - tail_at) >> 2;
        if (static_cast<uint32_t>(lane) < n_head) {
            cp_async4(dst + 4 * lane, reinterpret_cast<const void*>(src + 4 * lane));
        } else if (lane >= 4 && static_cast<uint32_t>(lane - 4) < n_tail) {
            const uint32_t o = tail_at + 4 * (lane - 4);
            cp_async4(dst + o, reinterpret_cast<const void*>(src + o));
        }
    } else if ((mis & 7u) == 0) {
        const uint32_t head = min(len, (8u - (static_cast<uint32_t>(src) & 7u)) & 7u); // 0 or 4
        const uint32_t body = (len - head) & ~7u;
        if (lane == 0 && head != 0) cp_async4(dst, reinterpret_cast<const void*>(src));
        for (uint32_t o = head + 8u * lane; o < head + body; o += 256u)
            cp_async8(dst + o, reinterpret_cast<const void*>(src + o));
        if (lane == 1 && head + body < len) {
            const uint32_t o = head + body;
            cp_async4(dst + o, reinterpret_cast<const void*>(src + o));
        }
    } else {
        for (uint32_t o = 4u * lane; o < len; o += 128u) cp_async4(dst + o, reinterpret_cast<const void*>(src + o));
    }
}

// Whole-row units whose rows are a multiple of 4 bytes but not of 16 (or a deck that is not 16-byte
// aligned): every member's <= 2 contiguous runs copied asynchronously into the stage
// (async_copy_piece), so the issuing warp does not wait for its loads.  Each lane then arrives on
// `bar` when its own copies have landed (the 32 arrivals the barrier expects), and the bulk bytes
// keep the phase open until they land too.
template <bool PUSH, bool PACK>
__device__ __forceinline__ void async_load_unit(const IterParams& p, const StageMeta& m, uint8_t* stage, uint64_t* bar,
                                                int lane)
{
    const int pmask = p.pblock - 1;
    const int n_load = PUSH ? m.rows_mine : m.n_valid;
    const int n_mem = PACK ? (p.pack << p.vblock_shift) : (PUSH ? 1 : (n_load + pmask) >> p.pblock_shift);
    const uint32_t R = static_cast<uint32_t>(p.row_bytes);
    int piece = 0;
    for (int r = 0; r < n_mem; ++r) {
        const int first = PUSH ? 0 : (r << p.pblock_shift);
        const int rows_r = PACK ? static_cast<int>(m.mrows[r]) : (PUSH ? m.rows_mine : min(p.pblock, n_load - first));
        if (rows_r <= 0) continue;
        const int na = PUSH ? m.src_na : m.n_a[r];
        const uintptr_t ra = PUSH ? m.src_a : m.run_a[r];
        const uintptr_t rb = PUSH ? m.src_b : m.run_b[r];
        const int n1 = min(rows_r, na);
        if (n1 > 0)
            async_copy_piece(stage + static_cast<size_t>(first) * R, ra, static_cast<uint32_t>(n1) * R, bar, lane, piece++);
        if (rows_r > n1)
            async_copy_piece(stage + static_cast<size_t>(first + n1) * R, rb + static_cast<uintptr_t>(n1) * R,
                             static_cast<uint32_t>(rows_r - n1) * R, bar, lane, piece++);
    }
    cp_async_arrive_noinc(bar);
}

// Rows (or slabs) of at most 32 * C chunks of T, this warp's share (rows f = warp, warp + n_warps,
// ..): lane l moves chunks l, l + 32, .. of a row, and the chunks of U rows are loaded before any
// is stored, so that each lane has up to U * C loads in flight (a row-by-row loop waited for every
// row's loads: 512-byte rows moved 3.4-3.9 TB/s that way).  Packed units skip holes.
template <int C, int U, typename T, bool PACK, typename SrcRow, typename DstSlot>
__device__ __forceinline__ void store_wide_rows(const IterParams& p, const StageMeta& m, const uint8_t* stage,
                                                int64_t col, int n, int cpr, int lane, int warp, int n_warps,
                                                SrcRow src_row, DstSlot dst_slot)
{
    const int pmask = p.pblock - 1;
    for (int f = warp; f < n; f += U * n_warps) {
        T v[U][C];
        T* dst[U];
        bool ok[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int fu = f + u * n_warps;
            ok[u] = fu < n;
            int s = 0, d = 0;
            if (ok[u]) {
                s = src_row(fu);
                d = dst_slot(fu);
                if constexpr (PACK) ok[u] = s != HOLE;
            }
            if (!ok[u]) s = d = 0;
            const T* src = reinterpret_cast<const T*>(stage + static_cast<size_t>(s) * p.slab_bytes);
            dst[u] = reinterpret_cast<T*>(slot_ptr(m, d, p.pblock_shift, pmask, p.row_bytes) + col);
#pragma unroll
            for (int c = 0; c < C; ++c) {
                const int q = lane + 32 * c;
                if (ok[u] && q < cpr) v[u][c] = src[q];
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
#pragma unroll
            for (int c = 0; c < C; ++c) {
                const int q = lane + 32 * c;
                if (ok[u] && q < cpr) store_row_chunk(dst[u] + q, v[u][c]);
            }
        }
    }
}

// store_share with the lane geometry computed by divisions: the form the bulk (TMA) path uses,
// where it measured faster than the shift form below (the per-unit share of this arithmetic is
// small there).  This warp's share of the copy stage -> global.  In place: destination slot f receives stage row
// idx[f] (idx = the permutation).  Push: stage row f (the unit's own member) goes to destination
// slot idx[f] (idx = the member's destination slots).  Work items are interleaved over the warps.
template <int W, bool PUSH, bool WIDE = false>
__device__ __forceinline__ void store_share_div(const IterParams& p, const StageMeta& m, const uint8_t* stage,
                                            const uint16_t* idx, int64_t col, int slen, int lane, int warp,
                                            int n_warps)
{
    using T = typename VecOf<W>::T;
    const int cpr = slen / W;
    const int pmask = p.pblock - 1;
    const int n = PUSH ? m.rows_mine : m.n_valid;
    auto src_row = [&](int f) -> int {
        if constexpr (PUSH) return f;
        else return idx[f];
    };
    auto dst_slot = [&](int f) -> int {
        if constexpr (PUSH) return idx[f];
        else return f;
    };
    if (cpr >= 32) {
        bool done = false;
        if constexpr (WIDE) {
            if (cpr <= 64) {
                store_wide_rows<2, 2, T, false>(p, m, stage, col, n, cpr, lane, warp, n_warps, src_row, dst_slot);
                done = true;
            }
        }
        if (!done) {
            for (int f = warp; f < n; f += n_warps) {
                const T* src = reinterpret_cast<const T*>(stage + static_cast<size_t>(src_row(f)) * p.slab_bytes);
                T* dst = reinterpret_cast<T*>(slot_ptr(m, dst_slot(f), p.pblock_shift, pmask, p.row_bytes) + col);
#pragma unroll 4
                for (int q = lane; q < cpr; q += 32) store_row_chunk(dst + q, src[q]);
            }
        }
    } else {
        const int g = 32 / cpr;
        const int lrow = lane / cpr, lq = lane - lrow * cpr;
        if (lrow >= g) return;
        const int n_pass = (n + g - 1) / g;
        constexpr int U = 4;
        int t = warp;
        for (; t + (U - 1) * n_warps < n_pass; t += U * n_warps) {
            T v[U];
            T* dst[U];
            bool ok[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int f = (t + u * n_warps) * g + lrow;
                ok[u] = f < n;
                const int fs = ok[u] ? f : 0;
                dst[u] = reinterpret_cast<T*>(slot_ptr(m, dst_slot(fs), p.pblock_shift, pmask, p.row_bytes) + col) + lq;
                v[u] = reinterpret_cast<const T*>(stage + static_cast<size_t>(src_row(fs)) * p.slab_bytes)[lq];
            }
#pragma unroll
            for (int u = 0; u < U; ++u)
                if (ok[u]) store_row_chunk(dst[u], v[u]);
        }
        for (; t < n_pass; t += n_warps) {
            const int f = t * g + lrow;
            if (f < n) {
                const T v = reinterpret_cast<const T*>(stage + static_cast<size_t>(src_row(f)) * p.slab_bytes)[lq];
                reinterpret_cast<T*>(slot_ptr(m, dst_slot(f), p.pblock_shift, pmask, p.row_bytes) + col)[lq] = v;
            }
        }
    }
}

// This warp's share of the copy stage -> global.  In place: destination slot f receives stage row
// idx[f] (idx = the permutation).  Push: stage row f (the unit's own member) goes to destination
// slot idx[f] (idx = the member's destination slots).  Work items are interleaved over the warps.
// WIDE (kernels launched for slabs of 512 to 1024 bytes): rows of 32 to 64 chunks keep four chunk
// loads per lane in flight (store_wide_rows; 512- to 1024-byte rows moved 1.1-1.7x faster).  The
// other kernels keep the row-by-row loop: compiled into them, the wide form cost the 256-byte-row
// kernels 1-2 % (more registers), and 2 KiB slabs ran 1 % slower with it.
template <int W, bool PUSH, bool PACK = false, bool WIDE = false, bool FAST = false>
__device__ __forceinline__ void store_share(const IterParams& p, const StageMeta& m, const uint8_t* stage,
                                            const uint16_t* idx, int64_t col, int slen, int lane, int warp,
                                            int n_warps)
{
    using T = typename VecOf<W>::T;
    const LaneGeom lg = lane_geom<W>(slen, lane);
    const int cpr = lg.cpr;
    const int pmask = p.pblock - 1;
    // Packed units: every slot of the unit; holes (idx == HOLE) are skipped.
    const int n = PACK ? p.unit_vp : (PUSH ? m.rows_mine : m.n_valid);
    auto src_row = [&](int f) -> int {
        if constexpr (PUSH) return f;
        else return idx[f];
    };
    auto dst_slot = [&](int f) -> int {
        if constexpr (PUSH) return idx[f];
        else return f;
    };
    if (cpr >= 32) {
        bool done = false;
        if constexpr (WIDE) {
            if (cpr <= 64) {
                store_wide_rows<2, 2, T, PACK>(p, m, stage, col, n, cpr, lane, warp, n_warps, src_row, dst_slot);
                done = true;
            }
        }
        if (!done) {
            for (int f = warp; f < n; f += n_warps) {
                if (PACK && idx[f] == HOLE) continue;
                const T* src = reinterpret_cast<const T*>(stage + static_cast<size_t>(src_row(f)) * p.slab_bytes);
                T* dst = reinterpret_cast<T*>(slot_ptr(m, dst_slot(f), p.pblock_shift, pmask, p.row_bytes) + col);
#pragma unroll 4
                for (int q = lane; q < cpr; q += 32) store_row_chunk(dst + q, src[q]);
            }
        }
    } else {
        const int g = lg.g, lrow = lg.lrow, lq = lg.lq;
        if (lrow >= g) return;
        if constexpr (FAST) {
            if (m.n_valid == p.unit_vp && lg.g_shift >= 0 && g <= p.pblock) {
                // A packed unit without holes whose passes (g rows each) lie inside one member: the
                // member of a pass and its run bases are the same for the whole warp, and no slot
                // needs the hole test.
                const int n_pass = n >> lg.g_shift;
                constexpr int U = 4;
                for (int t = warp; t < n_pass; t += U * n_warps) {
                    T v[U];
                    T* dst[U];
                    bool ok[U];
#pragma unroll
                    for (int u = 0; u < U; ++u) {
                        const int pass = t + u * n_warps;
                        ok[u] = pass < n_pass;
                        const int fb = (ok[u] ? pass : 0) << lg.g_shift;
                        const int r = fb >> p.pblock_shift;
                        const int i = (fb & pmask) + lrow;
                        const int src = idx[fb + lrow];
                        const uintptr_t base = i < m.n_a[r] ? m.run_a[r] : m.run_b[r];
                        dst[u] = reinterpret_cast<T*>(base + static_cast<uintptr_t>(i) * static_cast<uintptr_t>(p.row_bytes) +
                                                      static_cast<uintptr_t>(col)) + lq;
                        v[u] = reinterpret_cast<const T*>(stage + static_cast<size_t>(src) * p.slab_bytes)[lq];
                    }
#pragma unroll
                    for (int u = 0; u < U; ++u)
                        if (ok[u]) store_row_chunk(dst[u], v[u]);
                }
                return;
            }
        }
        const int n_pass = lg.passes(n);
        constexpr int U = 4;
        int t = warp;
        for (; t + (U - 1) * n_warps < n_pass; t += U * n_warps) {
            T v[U];
            T* dst[U];
            bool ok[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int f = (t + u * n_warps) * g + lrow;
                int src = 0, slot = 0;
                ok[u] = f < n;
                if (ok[u]) {
                    src = src_row(f);
                    slot = dst_slot(f);
                    if constexpr (PACK) ok[u] = src != HOLE;
                }
                if (!ok[u]) src = slot = 0;
                dst[u] = reinterpret_cast<T*>(slot_ptr(m, slot, p.pblock_shift, pmask, p.row_bytes) + col) + lq;
                v[u] = reinterpret_cast<const T*>(stage + static_cast<size_t>(src) * p.slab_bytes)[lq];
            }
#pragma unroll
            for (int u = 0; u < U; ++u)
                if (ok[u]) store_row_chunk(dst[u], v[u]);
        }
        for (; t < n_pass; t += n_warps) {
            const int f = t * g + lrow;
            if (f < n) {
                const int src = src_row(f);
                if (PACK && src == HOLE) continue;
                const T v = reinterpret_cast<const T*>(stage + static_cast<size_t>(src) * p.slab_bytes)[lq];
                reinterpret_cast<T*>(slot_ptr(m, dst_slot(f), p.pblock_shift, pmask, p.row_bytes) + col)[lq] = v;
            }
        }
    }
}

// Packed units of rows that are a multiple of 4 bytes (plain loads, R < 128), this warp's share:
// members r = warp, warp + n_warps, .. of the unit.  A member's valid rows are at most two
// contiguous destination runs (rows before n_a at run a, the rest at run b); the lanes write each
// run's 16-byte aligned chunks, lane l chunks l, l + 32, .., each assembled from four 4-byte words
// of the stage rows that land there (word at byte o of the run: destination row o / R, byte o % R
// of stage row perm[row]; the division is a multiply by row_magic, exact for o < 2^17).  The
// unaligned head and tail of a run (< 16 bytes each) go out as word stores.  Against one lane per
// 4-byte piece of a row, this stores 16 bytes per lane and computes no per-row global addresses.
__device__ __forceinline__ void store_unit_chunked(const IterParams& p, const StageMeta& m, const uint8_t* stage,
                                                   const uint16_t* perm, int lane, int warp, int n_warps)
{
    const uint32_t R = static_cast<uint32_t>(p.row_bytes);
    const uint32_t magic = p.row_magic;
    const int n_mem = p.pack << p.vblock_shift;
    for (int r = warp; r < n_mem; r += n_warps) {
        const int rows = m.mrows[r];
        if (rows <= 0) continue;
        const int na = m.n_a[r];
        for (int piece = 0; piece < 2; ++piece) {
            const int i_lo = piece == 0 ? 0 : na;
            const int i_hi = piece == 0 ? min(rows, na) : rows;
            if (i_lo >= i_hi) continue;
            const uintptr_t g0 = (piece == 0 ? m.run_a[r] : m.run_b[r]) + static_cast<uintptr_t>(i_lo) * R;
            const uint16_t* pr = perm + (r << p.pblock_shift) + i_lo;
            const uint32_t len = static_cast<uint32_t>(i_hi - i_lo) * R;
            const uint32_t head = min(len, (16u - static_cast<uint32_t>(g0 & 15u)) & 15u);
            const uint32_t n_chunks = (len - head) >> 4;
            const uint32_t tail_at = head + (n_chunks << 4);
            auto word = [&](uint32_t o) -> uint32_t {
                const uint32_t q = __umulhi(o, magic);
                return *reinterpret_cast<const uint32_t*>(stage + static_cast<size_t>(pr[q]) * R + (o - q * R));
            };
            for (uint32_t c = static_cast<uint32_t>(lane); c < n_chunks; c += 32u) {
                const uint32_t o = head + (c << 4);
                uint4 v;
                v.x = word(o);
                v.y = word(o + 4u);
                v.z = word(o + 8u);
                v.w = word(o + 12u);
                store_row_chunk(reinterpret_cast<uint4*>(g0 + o), v);
            }
            if (static_cast<uint32_t>(lane) * 4u < head) {
                const uint32_t o = static_cast<uint32_t>(lane) * 4u;
                *reinterpret_cast<uint32_t*>(g0 + o) = word(o);
            } else if (lane >= 4 && tail_at + static_cast<uint32_t>(lane - 4) * 4u < len) {
                const uint32_t o = tail_at + static_cast<uint32_t>(lane - 4) * 4u;
                *reinterpret_cast<uint32_t*>(g0 + o) = word(o);
            }
        }
    }
}

// Push mode: the destination slot of every element of the unit's own member (elements
// first .. first+count-1 of the vblock) under the uniform permutation; same sort as warp_make_perm.
template <int EPL>
__device__ __forceinline__ void warp_make_pos(const IterParams& p, uint64_t seed, uint64_t vblock, int n_valid,
                                              int first, int count, uint16_t* pos, int lane)
{
    uint32_t x[EPL];
    perm_sort_keys<EPL>(p, seed, vblock, n_valid, x, lane);
    warp_bitonic_sort<EPL, uint32_t>(x, lane);
#pragma unroll
    for (int r = 0; r < EPL; ++r) {
        const int f = lane * EPL + r;
        const int e = static_cast<int>(x[r] & PermKey<EPL>::IDX_MASK) - first;
        if (f < n_valid && e >= 0 && e < count) pos[e] = static_cast<uint16_t>(f);
    }
}

// ---------------------------------------------------------------------------------------------
// The iteration kernel.
// EPL: elements per lane of the permutation sort (32 * EPL >= V * P; packed: = pack * V * P).
// INJECTED: members, permutation and offset come from the caller instead of the device RNG.
// BULK: rows are 16-byte multiples on a 16-byte aligned deck -> TMA bulk loads.
//
// Warps 0 .. n_movers-1 move data; warps n_movers .. n_movers+n_permuters-1 compute, for unit
// u (permuter (u % n_permuters)), the ordered members, their storage runs and the permutation
// into slot u % KP, running up to KP units ahead of the movers.
// ---------------------------------------------------------------------------------------------

// Push-mode work list: the pblocks whose first storage row lies in shard `push_rank` (all pblocks
// when push_rank < 0).  Logical row L is stored at (L + offset) mod N, so these are the pblocks
// whose first logical row falls in the shard's rows shifted back by the offset: at most two ranges.
struct PushList {
    int64_t first, cnt1, cnt2; // [first, first + cnt1) then [0, cnt2)
    __device__ __forceinline__ int64_t size() const { return cnt1 + cnt2; }
    __device__ __forceinline__ int64_t at(int64_t k) const { return k < cnt1 ? first + k : k - cnt1; }
};

__device__ __forceinline__ PushList push_list(const IterParams& p, int64_t offset)
{
    PushList l{0, p.n_pblocks, 0};
    if (p.push_rank < 0) return l;
    const int64_t s0 = p.shard_start[p.push_rank];
    const int64_t len = p.shard_start[p.push_rank + 1] - s0;
    int64_t ls = s0 - offset;
    if (ls < 0) ls += p.n_rows;
    const int64_t P = p.pblock;
    l.first = (ls + P - 1) / P;
    const int64_t hi = ls + len;
    if (hi <= p.n_rows) {
        const int64_t end = min(p.n_pblocks, (hi + P - 1) / P);
        l.cnt1 = end > l.first ? end - l.first : 0;
        l.cnt2 = 0;
    } else {
        l.cnt1 = p.n_pblocks > l.first ? p.n_pblocks - l.first : 0;
        l.cnt2 = min(p.n_pblocks, (hi - p.n_rows + P - 1) / P);
    }
    return l;
}

// Storage run (a, pre-shifted b, n_a) of `rows` rows starting at storage row s0 in a table of shards.
__device__ __forceinline__ void locate_run(const IterParams& p, uint8_t* const* base, int64_t s0, int rows,
                                           uintptr_t& run_a, uintptr_t& run_b, int32_t& n_a)
{
    int sa = 0;
    while (sa + 1 < p.n_shards && s0 >= p.shard_start[sa + 1]) ++sa;
    const int64_t until_end = p.shard_start[sa + 1] - s0;
    const int na = until_end < rows ? static_cast<int>(until_end) : rows;
    run_a = reinterpret_cast<uintptr_t>(base[sa] + (s0 - p.shard_start[sa]) * p.row_bytes);
    run_b = reinterpret_cast<uintptr_t>(base[sa + 1 == p.n_shards ? 0 : sa + 1]) -
            static_cast<uintptr_t>(static_cast<int64_t>(na) * p.row_bytes);
    n_a = na;
}

// Position of unit u in a ring of n entries: i = u % n and the phase bit ph = (u / n) & 1,
// advanced one unit at a time without divisions.
struct RingPos {
    uint32_t i, ph;
    __device__ __forceinline__ void next(uint32_t n)
    {
        if (++i == n) {
            i = 0;
            ph ^= 1u;
        }
    }
};

__device__ __forceinline__ RingPos ring_at(uint64_t u, uint32_t n)
{
    return RingPos{static_cast<uint32_t>(u % n), static_cast<uint32_t>((u / n) & 1u)};
}

// ---------------------------------------------------------------------------------------------
// Packed units: the permuter warp's work for `n_seg` (<= pack) consecutive vblocks v0 .. v0+n_seg-1
// of one deck, written to permutation slot `slot`.  Lane l computes member (l mod V) of vblock
// v0 + l / V (pack * V <= 32), ranks it inside its vblock and records its storage run at ordered
// member index (l / V) * V + rank.  The permutation is every vblock's own, unchanged: the same sort
// keys as a vblock processed alone (same Philox words, same index bits), sorted in aligned blocks
// of vp elements by one warp; destination slots past a vblock's valid rows get HOLE.
// ---------------------------------------------------------------------------------------------

template <int EPL, typename PI>
__device__ __forceinline__ void make_packed_unit(const IterParams& p, StageMeta& m, uint16_t* perm, int64_t v0,
                                                 int n_seg, uint64_t seed, int64_t deck_offset, uintptr_t deck_shift,
                                                 const PI& pi, bool ref_rng, bool np_rng, int lane)
{
    const int vshift = p.vblock_shift;
    const int seg = lane >> vshift;          // this lane's vblock within the unit
    const int j = lane & (p.vblock - 1);     // this lane's member within its vblock
    int64_t mem = -1;
    if (seg < n_seg) {
        const int64_t slot = (v0 + seg) * p.vblock + j;
        const int64_t a = (ref_rng && slot >= p.n_pblocks) ? -1 : static_cast<int64_t>(pi(static_cast<uint64_t>(slot)));
        mem = (a >= 0 && a < p.n_pblocks) ? a : -1;
    }
    const bool valid = mem >= 0;
    int rows = 0;
    if (valid) {
        const int64_t left = p.n_rows - mem * p.pblock;
        rows = left < p.pblock ? static_cast<int>(left) : p.pblock;
    }
    // Ascending member ids with padding last (the reference kernel's order, povs.cu:203-221), or for
    // the NumPy path's distribution the slot order with full members first, then a truncated one,
    // then padding (numpy.py:125-136).
    const uint64_t key = np_rng ? static_cast<uint64_t>(j) + (valid ? (rows == p.pblock ? 0u : 64u) : 128u)
                         : valid ? static_cast<uint64_t>(mem) : ((uint64_t{1} << 63) | static_cast<uint64_t>(j));
    const int grp = seg << vshift;
    int rank = 0;
    for (int t = 0; t < p.vblock; ++t) {
        const uint64_t k2 = __shfl_sync(FULL_MASK, key, grp + t);
        rank += (k2 < key || (k2 == key && t < j)) ? 1 : 0;
    }
    int nv = rows; // valid rows of this lane's vblock (sum over its V lanes)
    for (int o = p.vblock >> 1; o > 0; o >>= 1) nv += __shfl_xor_sync(FULL_MASK, nv, o);
    const int total = __reduce_add_sync(FULL_MASK, rows);
    const int mi = grp + rank; // ordered member index within the unit
    m.mrows[mi] = static_cast<int16_t>(rows);
    if (valid) {
        int64_t s0 = mem * p.pblock + deck_offset;
        if (s0 >= p.n_rows) s0 -= p.n_rows;
        locate_run(p, p.shard_base, s0, rows, m.run_a[mi], m.run_b[mi], m.n_a[mi]);
        m.run_a[mi] += deck_shift;
        m.run_b[mi] += deck_shift;
    }
    if (lane == 0) m.n_valid = total;
    // Lane s (< pack) holds the valid rows of vblock s.
    const int pack_last = p.pack - 1;
    const int nv_lane = __shfl_sync(FULL_MASK, nv, min(lane, pack_last) << vshift);
    const int vpm = p.vp - 1;
    if (np_rng) {
        // Lane s (< n_seg) finds vblock s's precomputed permutation; every lane copies its share.
        int64_t base = 0;
        if (lane < n_seg && nv_lane > 0)
            base = np_perm(p, nv_lane, vblock_seed(seed, p.iteration, static_cast<uint64_t>(v0 + lane))) - p.np_table;
        for (int f = lane; f < p.unit_vp; f += 32) {
            const int sf = f >> p.vp_shift;
            const int nvf = __shfl_sync(FULL_MASK, nv_lane, sf);
            const int64_t bf = __shfl_sync(FULL_MASK, base, sf);
            const int fl = f & vpm;
            perm[f] = fl < nvf ? static_cast<uint16_t>((sf << p.vp_shift) + p.np_table[bf + fl]) : HOLE;
        }
        __syncwarp();
        return;
    }
    if (ref_rng) {
        // The reference kernel's xorshift32 Fisher-Yates, one vblock per lane (povs.cu:282-321).
        for (int f = lane; f < p.unit_vp; f += 32) {
            const int nvf = __shfl_sync(FULL_MASK, nv_lane, f >> p.vp_shift);
            perm[f] = (f & vpm) < nvf ? static_cast<uint16_t>(f) : HOLE;
        }
        __syncwarp();
        if (lane < n_seg) {
            uint16_t* pv = perm + (lane << p.vp_shift);
            uint32_t r = vblock_seed(seed, p.iteration, static_cast<uint64_t>(v0 + lane));
            const int last = nv_lane - 1;
            for (int i = 0; i <= last; ++i) {
                r ^= r << 13;
                r ^= r >> 17;
                r ^= r << 5;
                const int jj = i + static_cast<int>((static_cast<uint64_t>(r) * static_cast<uint64_t>(last - i + 1)) >> 32);
                const uint16_t t = pv[i];
                pv[i] = pv[jj];
                pv[jj] = t;
            }
        }
        __syncwarp();
        return;
    }
    const uint32_t M = (1u << p.idx_bits) - 1u;
    uint32_t x[EPL];
    // Keys come in quads of Philox words (elements 4c .. 4c+3 of a vblock); vp >= 8, so a quad never
    // straddles two vblocks.  With fewer than 4 keys per lane, the lane's keys share one quad.
    constexpr int QPL = EPL >= 4 ? EPL / 4 : 1; // quads per lane
#pragma unroll
    for (int q = 0; q < QPL; ++q) {
        const int e0g = lane * EPL + 4 * q;       // unit element of the lane's first key in the quad
        const int sq = e0g >> p.vp_shift;         // its vblock within the unit
        const int e0 = e0g & vpm;                 // its element index within the vblock
        const int nvq = __shfl_sync(FULL_MASK, nv_lane, sq);
        const U32x4 k = perm_key4(seed, p.iteration, static_cast<uint64_t>(v0 + sq), static_cast<uint32_t>(e0 >> 2));
#pragma unroll
        for (int t = 0; t < (EPL >= 4 ? 4 : EPL); ++t) {
            const uint32_t e = static_cast<uint32_t>(e0 + t);
            x[4 * q + t] = ((static_cast<int>(e) < nvq) ? (pick_word(k, static_cast<int>(e & 3u)) & ~M) : ~M) | e;
        }
    }
    warp_sort_blocks<EPL, uint32_t>(x, lane, p.vp);
    // Destination slot fg = lane * EPL + r of the unit takes unit row (fg & ~vpm) + (x[r] & M), or
    // HOLE past its vblock's valid rows (only in units with a short or missing vblock).
    if (total == p.unit_vp) {
#pragma unroll
        for (int r = 0; r < EPL; ++r) x[r] = ((lane * EPL + r) & ~vpm) | (x[r] & M);
    } else {
#pragma unroll
        for (int r = 0; r < EPL; ++r) {
            const int fg = lane * EPL + r;
            const int sr = fg >> p.vp_shift;
            const int nvr = __shfl_sync(FULL_MASK, nv_lane, sr);
            x[r] = (fg & vpm) < nvr ? static_cast<uint32_t>((sr << p.vp_shift) + static_cast<int>(x[r] & M)) : HOLE;
        }
    }
    store_u16_run<EPL>(perm + lane * EPL, x);
}

// RING: the permuter and mover warps carry their units' stage / slot ring positions from unit to
// unit (small units, where per-unit bookkeeping is a visible share of the work, and every
// plain-load kernel); otherwise they recompute them per unit, which measured faster on large
// bulk-loaded units.
// PACK: units are groups of `pack` small vblocks (device randomness, in place, whole rows).
template <int EPL, bool INJECTED, bool BULK, bool PUSH, bool RING, bool PACK = false, bool WIDE = false,
          bool CHUNK = false, bool FAST = false>
__global__ void __launch_bounds__(512, 1) povs_iteration_kernel(const __grid_constant__ IterParams p)
{
    static_assert(!FAST || (PACK && BULK), "the uniform-member store form is built into packed TMA-loaded kernels");
    static_assert(!WIDE || (BULK && !PACK), "the wide-row store form is built into TMA-loaded, unpacked kernels");
    static_assert(!CHUNK || (PACK && !BULK), "chunked stores are built into packed plain-load kernels");
    static_assert(BULK || RING, "plain-load kernels carry ring positions");
    static_assert(!(PUSH && INJECTED), "push mode draws its randomness on the device");
    static_assert(!PACK || (RING && !PUSH && !INJECTED), "packed units: device randomness, in place, ring positions");
    extern __shared__ __align__(128) uint8_t smem_raw[];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int n_movers = p.n_movers;
    const int nst = p.n_stages;
    const int kp = p.n_slots;
    const uint32_t mover_threads = static_cast<uint32_t>(n_movers) * 32u;
    CtaSmem sm = carve_smem(smem_raw, p);

    for (int i = threadIdx.x; i < nst; i += blockDim.x) {
        mbar_init(&sm.full[i], 32);
        mbar_init(&sm.empty[i], mover_threads);
    }
    for (int i = threadIdx.x; i < kp; i += blockDim.x) {
        mbar_init(&sm.pfull[i], 32);
        mbar_init(&sm.pempty[i], mover_threads);
    }
    mbar_fence_init();
    __syncthreads();
    allow_dependent_launch();

    // Iteration-wide randomness (identical in every thread).
    int64_t offset;
    if constexpr (INJECTED) {
        offset = p.offset;
    } else {
        offset = p.offsets[reduce_range(offset_draw(p.seed, p.iteration), static_cast<uint32_t>(p.n_offsets))];
    }

    // Work list.  In place: vblocks vb_begin + vb_step * k, k < n_list.  Push: the pblocks of
    // push_list.  CTA b takes list entries b, b + grid, ...; a unit is (entry, slab).
    int64_t n_list;
    PushList plist{};
    if constexpr (PUSH) {
        plist = push_list(p, offset);
        n_list = plist.size();
    } else if constexpr (PACK) {
        n_list = p.groups_per_deck * p.n_decks;
    } else {
        const int64_t total = p.n_vblocks * p.n_decks;
        n_list = p.vb_begin < total ? (total - p.vb_begin + p.vb_step - 1) / p.vb_step : 0;
    }
    if (blockIdx.x >= n_list) return;
    const int64_t my_entries = (n_list - blockIdx.x + gridDim.x - 1) / gridDim.x;
    const int64_t n_units = my_entries * p.n_slabs;
    const int pmask = p.pblock - 1;

    if (warp >= n_movers) {
        // ------------------------------------------------------------------ permuter warps
        Feistel pi;
        // Uniform mode maps all n_v*V slots (padding ids anywhere); the reference-CUDA mode maps
        // slots [0, n_p) and leaves the padding in the last slots, as the reference does.
        const bool ref_rng = p.rng_mode == RNG_REFERENCE_CUDA;
        const bool np_rng = p.rng_mode == RNG_REFERENCE_NUMPY;
        const uint64_t domain = ref_rng ? static_cast<uint64_t>(p.n_pblocks) : static_cast<uint64_t>(p.n_vblocks) * p.vblock;
        if constexpr (!INJECTED) pi.init(p.seed, p.iteration, domain);
        // Batched decks: the randomness of the deck of the current unit.
        uint64_t seed = p.seed;
        int64_t deck = -1; // batched decks: none drawn yet
        int64_t deck_offset = offset;
        const int q = warp - n_movers;
        // Unit u = q, q + n_permuters, ...: its slot (u % kp, phase) and its list entry / slab
        // (u / n_slabs, u % n_slabs) advance without divisions (n_permuters < kp).
        const uint32_t step_e = static_cast<uint32_t>(p.n_permuters / p.n_slabs);
        const uint32_t step_s = static_cast<uint32_t>(p.n_permuters % p.n_slabs);
        RingPos kr = ring_at(static_cast<uint64_t>(q), static_cast<uint32_t>(kp));
        if constexpr (PACK) {
            // Unit u = group u of this CTA's list (one slab): groups blockIdx.x + u * gridDim.x.
            for (int64_t u = q; u < n_units; u += p.n_permuters) {
                const int k = static_cast<int>(kr.i);
                if (u >= kp && !warp_wait(&sm.pempty[k], kr.ph ^ 1u, p.status)) return;
                for (int t = 0; t < p.n_permuters; ++t) kr.next(static_cast<uint32_t>(kp));
                const int64_t group = blockIdx.x + u * static_cast<int64_t>(gridDim.x);
                const int64_t d = p.n_decks > 1 ? group / p.groups_per_deck : 0;
                const int64_t v0 = (group - d * p.groups_per_deck) * p.pack;
                const int n_seg = static_cast<int>(min(static_cast<int64_t>(p.pack), p.n_vblocks - v0));
                uintptr_t deck_shift = 0;
                if (p.n_decks > 1) {
                    if (d != deck) {
                        deck = d;
                        seed = p.deck_seeds[d];
                        pi.init(seed, p.iteration, domain);
                        deck_offset = p.offsets[reduce_range(offset_draw(seed, p.iteration),
                                                             static_cast<uint32_t>(p.n_offsets))];
                    }
                    deck_shift = static_cast<uintptr_t>(d * p.deck_stride);
                }
                make_packed_unit<EPL>(p, sm.meta[k], sm.perm + static_cast<size_t>(k) * sm.perm_stride, v0, n_seg,
                                      seed, deck_offset, deck_shift, pi, ref_rng, np_rng, lane);
                __syncwarp();
                mbar_arrive(&sm.pfull[k]); // each lane publishes its writes to the slot
            }
            return;
        }
        int64_t entry_local = q / p.n_slabs;
        uint32_t slab_q = static_cast<uint32_t>(q % p.n_slabs);
        for (int64_t u = q; u < n_units; u += p.n_permuters) {
            int k;
            int64_t entry;
            if constexpr (!RING) {
                // Large bulk units: positions recomputed per unit (measured faster there).
                k = static_cast<int>(u % kp);
                if (u >= kp && !warp_wait(&sm.pempty[k], static_cast<uint32_t>(((u / kp) - 1) & 1), p.status)) return;
                entry = blockIdx.x + (u / p.n_slabs) * static_cast<int64_t>(gridDim.x);
            } else {
                k = static_cast<int>(kr.i);
                if (u >= kp && !warp_wait(&sm.pempty[k], kr.ph ^ 1u, p.status)) return;
                entry = blockIdx.x + entry_local * static_cast<int64_t>(gridDim.x);
                // Advance to this warp's next unit.
                kr.i += static_cast<uint32_t>(p.n_permuters);
                if (kr.i >= static_cast<uint32_t>(kp)) {
                    kr.i -= static_cast<uint32_t>(kp);
                    kr.ph ^= 1u;
                }
                entry_local += step_e;
                slab_q += step_s;
                if (slab_q >= static_cast<uint32_t>(p.n_slabs)) {
                    slab_q -= static_cast<uint32_t>(p.n_slabs);
                    ++entry_local;
                }
            }
            int64_t v;
            int64_t own = -1;  // push: the unit's own pblock
            int own_lane = 0;  // push: its slot within the vblock
            if constexpr (PUSH) {
                own = plist.at(entry);
                const int64_t slot_of_own = static_cast<int64_t>(pi.inverse(static_cast<uint64_t>(own)));
                v = slot_of_own / p.vblock;
                own_lane = static_cast<int>(slot_of_own - v * p.vblock);
            } else {
                v = p.vb_begin + p.vb_step * entry;
            }
            uintptr_t deck_shift = 0; // batched decks: byte offset of the unit's deck
            if constexpr (!PUSH && !INJECTED) {
                if (p.n_decks > 1) {
                    const int64_t d = v / p.n_vblocks;
                    v -= d * p.n_vblocks;
                    if (d != deck) {
                        deck = d;
                        seed = p.deck_seeds[d];
                        pi.init(seed, p.iteration, domain);
                        deck_offset = p.offsets[reduce_range(offset_draw(seed, p.iteration),
                                                             static_cast<uint32_t>(p.n_offsets))];
                    }
                    deck_shift = static_cast<uintptr_t>(d * p.deck_stride);
                }
            }
            StageMeta& m = sm.meta[k];
            uint16_t* perm = sm.perm + static_cast<size_t>(k) * sm.perm_stride;

            int64_t mem = -1;
            if (lane < p.vblock) {
                const int64_t slot = v * p.vblock + lane;
                int64_t a;
                if constexpr (INJECTED) {
                    a = p.assign[slot];
                } else {
                    a = (ref_rng && slot >= p.n_pblocks) ? -1 : static_cast<int64_t>(pi(static_cast<uint64_t>(slot)));
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
            } else if (INJECTED ? p.sort_members != 0 : !np_rng) {
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
                // Storage run of the member (in the destination buffer in push mode): from row s0, split
                // at most once where its shard (or the deck) ends.
                int64_t s0 = mem * p.pblock + deck_offset;
                if (s0 >= p.n_rows) s0 -= p.n_rows;
                locate_run(p, PUSH ? p.dst_base : p.shard_base, s0, rows, m.run_a[rank], m.run_b[rank], m.n_a[rank]);
                m.run_a[rank] += deck_shift;
                m.run_b[rank] += deck_shift;
                if (PUSH && lane == own_lane) {
                    locate_run(p, p.shard_base, s0, rows, m.src_a, m.src_b, m.src_na);
                    m.rows_mine = rows;
                }
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
            } else if constexpr (PUSH) {
                const int own_rank = __shfl_sync(FULL_MASK, rank, own_lane);
                const int own_rows = __shfl_sync(FULL_MASK, rows, own_lane);
                const int first = own_rank << p.pblock_shift;
                uint16_t* pos = sm.pos + static_cast<size_t>(k) * sm.pos_stride;
                if (ref_rng || np_rng) {
                    if (ref_rng)
                        warp_make_perm_xorshift(p, seed, static_cast<uint64_t>(v), n_valid, perm, lane);
                    else
                        warp_copy_np_perm(p, seed, static_cast<uint64_t>(v), n_valid, perm, lane);
                    for (int f = lane; f < n_valid; f += 32) {
                        const int e = static_cast<int>(perm[f]) - first;
                        if (e >= 0 && e < own_rows) pos[e] = static_cast<uint16_t>(f);
                    }
                } else {
                    warp_make_pos<EPL>(p, seed, static_cast<uint64_t>(v), n_valid, first, own_rows, pos, lane);
                }
            } else {
                if (ref_rng)
                    warp_make_perm_xorshift(p, seed, static_cast<uint64_t>(v), n_valid, perm, lane);
                else if (np_rng)
                    warp_copy_np_perm(p, seed, static_cast<uint64_t>(v), n_valid, perm, lane);
                else
                    warp_make_perm<EPL>(p, seed, static_cast<uint64_t>(v), n_valid, perm, lane);
            }
            __syncwarp();
            mbar_arrive(&sm.pfull[k]); // each lane publishes its writes to the slot
        }
        return;
    }

    // ---------------------------------------------------------------------- mover warps
    const int mw = warp;
    // Nothing of the deck is read or written before the previous iteration's grid has finished.
    wait_for_prior_grid();
    const int64_t ahead = nst - 1;
    int64_t last_issued = -1;

    if constexpr (!RING) {
        // Large TMA-loaded units.  Unit u's stage (u % nst), permutation slot (u % kp) and phases are
        // recomputed per unit (on large units this measured faster than carrying ring counters).
        auto issue = [&](int64_t u) -> bool {
            const int st = static_cast<int>(u % nst);
            const int k = static_cast<int>(u % kp);
            if (!warp_wait(&sm.pfull[k], static_cast<uint32_t>((u / kp) & 1), p.status)) return false;
            if (u >= nst && !warp_wait(&sm.empty[st], static_cast<uint32_t>(((u / nst) - 1) & 1), p.status))
                return false;
            fence_proxy_async_smem();
            const StageMeta& m = sm.meta[k];
            const int n_load = PUSH ? m.rows_mine : m.n_valid;
            const int slab = static_cast<int>(u % p.n_slabs);
            const int64_t col = static_cast<int64_t>(slab) * p.slab_bytes;
            const int slen = static_cast<int>(min(static_cast<int64_t>(p.slab_bytes), p.row_bytes - col));
            uint8_t* stage = sm.data + static_cast<size_t>(st) * p.stage_bytes;
            if (lane == 0) mbar_expect_tx(&sm.full[st], static_cast<uint32_t>(n_load) * static_cast<uint32_t>(slen));
            __syncwarp();
            if (p.n_slabs == 1) {
                // Whole rows: each member is <= 2 contiguous runs (split where its shard or the deck
                // ends), copied in pieces of at most copy_rows rows; pieces are spread over the lanes.
                const int pieces_per_member = (p.pblock + p.copy_rows - 1) / p.copy_rows;
                const int n_mem = PUSH ? 1 : (n_load + pmask) >> p.pblock_shift;
                for (int q = lane; q < n_mem * pieces_per_member; q += 32) {
                    const int r = q / pieces_per_member;
                    const int i0 = (q - r * pieces_per_member) * p.copy_rows;
                    const int first = r << p.pblock_shift;
                    const int rows_r = min(p.pblock, n_load - first);
                    if (i0 >= rows_r) continue;
                    const int len = min(p.copy_rows, rows_r - i0);
                    const int na = PUSH ? m.src_na : m.n_a[r];
                    const uintptr_t ra = PUSH ? m.src_a : m.run_a[r];
                    const uintptr_t rb = PUSH ? m.src_b : m.run_b[r];
                    // Rows [i0, i0+len) of the member: the part before n_a from run a, the rest from run b.
                    const int n1 = i0 < na ? min(len, na - i0) : 0;
                    uint8_t* dst = stage + static_cast<size_t>(first + i0) * p.slab_bytes;
                    if (n1 > 0)
                        bulk_load(dst, reinterpret_cast<const uint8_t*>(ra + static_cast<uintptr_t>(i0) * p.row_bytes),
                                  static_cast<uint32_t>(n1) * static_cast<uint32_t>(p.row_bytes), &sm.full[st]);
                    if (len > n1)
                        bulk_load(dst + static_cast<size_t>(n1) * p.slab_bytes,
                                  reinterpret_cast<const uint8_t*>(rb + static_cast<uintptr_t>(i0 + n1) * p.row_bytes),
                                  static_cast<uint32_t>(len - n1) * static_cast<uint32_t>(p.row_bytes), &sm.full[st]);
                }
            } else {
                for (int f = lane; f < n_load; f += 32) {
                    const uint8_t* src = PUSH ? src_row_ptr(m, f, p.row_bytes) + col
                                              : slot_ptr(m, f, p.pblock_shift, pmask, p.row_bytes) + col;
                    bulk_load(stage + static_cast<size_t>(f) * p.slab_bytes, src, static_cast<uint32_t>(slen),
                              &sm.full[st]);
                }
            }
            mbar_arrive(&sm.full[st]);
            return true;
        };
        auto store = [&](int64_t j) -> bool {
            const int st = static_cast<int>(j % nst);
            const int k = static_cast<int>(j % kp);
            if (!warp_wait(&sm.full[st], static_cast<uint32_t>((j / nst) & 1), p.status)) return false;
            const StageMeta& m = sm.meta[k];
            const uint16_t* idx = PUSH ? sm.pos + static_cast<size_t>(k) * sm.pos_stride
                                       : sm.perm + static_cast<size_t>(k) * sm.perm_stride;
            const uint8_t* stage = sm.data + static_cast<size_t>(st) * p.stage_bytes;
            const int slab = static_cast<int>(j % p.n_slabs);
            const int64_t col = static_cast<int64_t>(slab) * p.slab_bytes;
            const int slen = static_cast<int>(min(static_cast<int64_t>(p.slab_bytes), p.row_bytes - col));
            store_share_div<16, PUSH, WIDE>(p, m, stage, idx, col, slen, lane, mw, n_movers);
            mbar_arrive(&sm.empty[st]);  // this thread's reads of the data stage are done
            mbar_arrive(&sm.pempty[k]);  // ... and of the permutation slot
            return true;
        };
        // On a timeout: wait (bounded) for the copies of the units this warp issued and stop.
        auto drain_and_stop = [&](int64_t from) {
            for (int64_t u = from; u <= last_issued; ++u)
                if (u % n_movers == mw) warp_wait(&sm.full[u % nst], static_cast<uint32_t>((u / nst) & 1), p.status);
        };
        for (int64_t u = mw; u < ahead && u < n_units; u += n_movers) {
            if (!issue(u)) {
                drain_and_stop(0);
                return;
            }
            last_issued = u;
        }
        // Store before issuing: the issue of unit j+NST-1 waits for every mover's share of unit j-1.
        for (int64_t j = 0; j < n_units; ++j) {
            if (!store(j)) {
                drain_and_stop(j);
                return;
            }
            const int64_t u = j + ahead;
            if (u < n_units && u % n_movers == mw) {
                if (!issue(u)) {
                    drain_and_stop(j + 1);
                    return;
                }
                last_issued = u;
            }
        }
    } else {
        // Ring positions carried from unit to unit.  Loads: TMA bulk copies (BULK) or plain vector
        // loads (rows not a multiple of 16 bytes, or an unaligned deck).
        auto issue = [&](RingPos sr, RingPos kr, int slab, bool wait_empty) -> bool {
            const int st = static_cast<int>(sr.i);
            const int k = static_cast<int>(kr.i);
            if (!warp_wait(&sm.pfull[k], kr.ph, p.status)) return false;
            if (wait_empty && !warp_wait(&sm.empty[st], sr.ph ^ 1u, p.status)) return false;
            const StageMeta& m = sm.meta[k];
            const int64_t col = static_cast<int64_t>(slab) * p.slab_bytes;
            const int slen = static_cast<int>(min(static_cast<int64_t>(p.slab_bytes), p.row_bytes - col));
            uint8_t* stage = sm.data + static_cast<size_t>(st) * p.stage_bytes;
            if constexpr (BULK) {
                fence_proxy_async_smem();
                const int n_load = PUSH ? m.rows_mine : m.n_valid;
                if (lane == 0)
                    mbar_expect_tx(&sm.full[st], static_cast<uint32_t>(n_load) * static_cast<uint32_t>(slen));
                __syncwarp();
                if (p.n_slabs == 1) {
                    // Whole rows: each member is <= 2 contiguous runs, copied in pieces of at most
                    // copy_rows rows; pieces are spread over the lanes.  Packed units: every member
                    // slot of the unit, with its own row count (0 for padding).
                    const int ppm = (p.pblock + p.copy_rows - 1) / p.copy_rows;
                    const int n_mem = PACK ? (p.pack << p.vblock_shift)
                                           : (PUSH ? 1 : (n_load + pmask) >> p.pblock_shift);
                    for (int q = lane; q < n_mem * ppm; q += 32) {
                        const int r = ppm == 1 ? q : q / ppm;
                        const int i0 = (q - r * ppm) * p.copy_rows;
                        const int first = r << p.pblock_shift;
                        const int rows_r = PACK ? static_cast<int>(m.mrows[r]) : min(p.pblock, n_load - first);
                        if (i0 >= rows_r) continue;
                        const int len = min(p.copy_rows, rows_r - i0);
                        const int na = PUSH ? m.src_na : m.n_a[r];
                        const uintptr_t ra = PUSH ? m.src_a : m.run_a[r];
                        const uintptr_t rb = PUSH ? m.src_b : m.run_b[r];
                        const int n1 = i0 < na ? min(len, na - i0) : 0;
                        uint8_t* dst = stage + static_cast<size_t>(first + i0) * p.slab_bytes;
                        if (n1 > 0)
                            bulk_load(dst, reinterpret_cast<const uint8_t*>(ra + static_cast<uintptr_t>(i0) * p.row_bytes),
                                      static_cast<uint32_t>(n1) * static_cast<uint32_t>(p.row_bytes), &sm.full[st]);
                        if (len > n1)
                            bulk_load(dst + static_cast<size_t>(n1) * p.slab_bytes,
                                      reinterpret_cast<const uint8_t*>(rb + static_cast<uintptr_t>(i0 + n1) * p.row_bytes),
                                      static_cast<uint32_t>(len - n1) * static_cast<uint32_t>(p.row_bytes), &sm.full[st]);
                    }
                } else {
                    for (int f = lane; f < n_load; f += 32) {
                        const uint8_t* src = PUSH ? src_row_ptr(m, f, p.row_bytes) + col
                                                  : slot_ptr(m, f, p.pblock_shift, pmask, p.row_bytes) + col;
                        bulk_load(stage + static_cast<size_t>(f) * p.slab_bytes, src, static_cast<uint32_t>(slen),
                                  &sm.full[st]);
                    }
                }
            } else if (p.async_plain) {
                // Whole rows of 4-byte multiples: asynchronous copies; each lane's arrival on `full`
                // comes when its copies land (no separate arrival below).
                fence_proxy_async_smem();
                async_load_unit<PUSH, PACK>(p, m, stage, &sm.full[st], lane);
                return true;
            } else {
                switch (p.vec_bytes) {
                case 16: lsu_load_unit<16, PUSH, PACK>(p, m, stage, col, slen, lane); break;
                case 8: lsu_load_unit<8, PUSH, PACK>(p, m, stage, col, slen, lane); break;
                case 4: lsu_load_unit<4, PUSH, PACK>(p, m, stage, col, slen, lane); break;
                case 2: lsu_load_unit<2, PUSH, PACK>(p, m, stage, col, slen, lane); break;
                default: lsu_load_unit<1, PUSH, PACK>(p, m, stage, col, slen, lane); break;
                }
                __syncwarp();
            }
            mbar_arrive(&sm.full[st]);
            return true;
        };
        auto store = [&](RingPos sr, RingPos kr, int slab) -> bool {
            const int st = static_cast<int>(sr.i);
            const int k = static_cast<int>(kr.i);
            if (!warp_wait(&sm.full[st], sr.ph, p.status)) return false;
            const StageMeta& m = sm.meta[k];
            const uint16_t* idx = PUSH ? sm.pos + static_cast<size_t>(k) * sm.pos_stride
                                       : sm.perm + static_cast<size_t>(k) * sm.perm_stride;
            const uint8_t* stage = sm.data + static_cast<size_t>(st) * p.stage_bytes;
            const int64_t col = static_cast<int64_t>(slab) * p.slab_bytes;
            const int slen = static_cast<int>(min(static_cast<int64_t>(p.slab_bytes), p.row_bytes - col));
            if constexpr (BULK) {
                store_share<16, PUSH, PACK, WIDE, FAST>(p, m, stage, idx, col, slen, lane, mw, n_movers);
            } else if (CHUNK && p.chunked_store) {
                // The CHUNK kernels keep the piecewise stores below compiled in as well: with both
                // forms in one kernel the chunked stores measured 5-22 % faster than in a kernel
                // with the chunked form alone (same plans, same box).
                store_unit_chunked(p, m, stage, idx, lane, mw, n_movers);
            } else {
                switch (p.vec_bytes) {
                case 16: store_share<16, PUSH, PACK>(p, m, stage, idx, col, slen, lane, mw, n_movers); break;
                case 8: store_share<8, PUSH, PACK>(p, m, stage, idx, col, slen, lane, mw, n_movers); break;
                case 4: store_share<4, PUSH, PACK>(p, m, stage, idx, col, slen, lane, mw, n_movers); break;
                case 2: store_share<2, PUSH, PACK>(p, m, stage, idx, col, slen, lane, mw, n_movers); break;
                default: store_share<1, PUSH, PACK>(p, m, stage, idx, col, slen, lane, mw, n_movers); break;
                }
            }
            mbar_arrive(&sm.empty[st]);  // this thread's reads of the data stage are done
            mbar_arrive(&sm.pempty[k]);  // ... and of the permutation slot
            return true;
        };
        // On a timeout: wait (bounded) for the asynchronous copies of the units this warp issued and
        // stop (synchronous plain loads complete before a unit's `full` arrival: nothing to wait for).
        auto drain_and_stop = [&](int64_t from) {
            if (BULK || p.async_plain) {
                for (int64_t u = from; u <= last_issued; ++u)
                    if (u % n_movers == mw)
                        warp_wait(&sm.full[u % nst], static_cast<uint32_t>((u / nst) & 1), p.status);
                cp_async_wait_all(); // this thread's 4/8-byte copies (they always complete)
            }
        };
        const uint32_t n_slabs = static_cast<uint32_t>(p.n_slabs);
        for (int64_t u = mw; u < ahead && u < n_units; u += n_movers) {
            if (!issue(ring_at(static_cast<uint64_t>(u), static_cast<uint32_t>(nst)),
                       ring_at(static_cast<uint64_t>(u), static_cast<uint32_t>(kp)),
                       static_cast<int>(static_cast<uint64_t>(u) % n_slabs), u >= nst)) {
                drain_and_stop(0);
                return;
            }
            last_issued = u;
        }
        // Store before issuing: the issue of unit j+NST-1 waits for every mover's share of unit j-1.
        // Ring positions of unit j (stores) and of unit j + ahead (issues) advance one unit per step.
        RingPos sj{0u, 0u}, kj{0u, 0u};
        uint32_t slab_j = 0;
        RingPos su = ring_at(static_cast<uint64_t>(ahead), static_cast<uint32_t>(nst));
        RingPos ku = ring_at(static_cast<uint64_t>(ahead), static_cast<uint32_t>(kp));
        uint32_t slab_u = static_cast<uint32_t>(static_cast<uint64_t>(ahead) % n_slabs);
        uint32_t mover_u = static_cast<uint32_t>(ahead % n_movers);
        for (int64_t j = 0; j < n_units; ++j) {
            if (!store(sj, kj, static_cast<int>(slab_j))) {
                drain_and_stop(j);
                return;
            }
            const int64_t u = j + ahead;
            if (u < n_units && mover_u == static_cast<uint32_t>(mw)) {
                if (!issue(su, ku, static_cast<int>(slab_u), u >= nst)) {
                    drain_and_stop(j + 1);
                    return;
                }
                last_issued = u;
            }
            sj.next(static_cast<uint32_t>(nst));
            kj.next(static_cast<uint32_t>(kp));
            su.next(static_cast<uint32_t>(nst));
            ku.next(static_cast<uint32_t>(kp));
            if (++slab_j == n_slabs) slab_j = 0;
            if (++slab_u == n_slabs) slab_u = 0;
            if (++mover_u == static_cast<uint32_t>(n_movers)) mover_u = 0;
        }
    }
}

// ---------------------------------------------------------------------------------------------
// Cross-GPU barrier between iterations of a sharded deck (one launch of one CTA per GPU).
// Rank r writes `epoch` into slot r of every rank's flag array (system-scope release after a
// system fence, so this GPU's earlier writes to peer shards are visible first), then waits until
// every slot of its own array holds at least `epoch` (system-scope acquire).  The wait is bounded:
// past limit_ns (default PEER_WAIT_LIMIT_NS) it records DEV_ERR_PEER_TIMEOUT and returns.
// ---------------------------------------------------------------------------------------------

struct PeerBarrierParams {
    uint32_t* flags[MAX_SHARDS]; // flags[r]: rank r's array of n_ranks words, as mapped in this process
    int32_t n_ranks;
    int32_t rank;
    uint32_t epoch;
    int* status;
    unsigned long long limit_ns;
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v)
{
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p)
{
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__global__ void __launch_bounds__(32) povs_peer_barrier_kernel(const __grid_constant__ PeerBarrierParams q)
{
    const int t = threadIdx.x;
    __threadfence_system();
    __syncwarp();
    if (t < q.n_ranks) st_release_sys(q.flags[t] + q.rank, q.epoch);
    if (t < q.n_ranks) {
        const uint32_t* mine = q.flags[q.rank] + t;
        const unsigned long long t0 = global_timer_ns();
        while (static_cast<int32_t>(ld_acquire_sys(mine) - q.epoch) < 0) {
            __nanosleep(200);
            if (global_timer_ns() - t0 > q.limit_ns) {
                atomicOr(q.status, DEV_ERR_PEER_TIMEOUT);
                return;
            }
        }
    }
}

} // namespace povs
