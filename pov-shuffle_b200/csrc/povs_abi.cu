// C ABI of the B200 POV shuffle: argument checks, launch planning, per-device
// context and CUDA-graph chaining of iterations.  Declarations and the
// reference interfaces each entry replaces are in include/povs.h.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <unordered_map>
#include <vector>

#include <unistd.h>

#include "../../include/povs.h"
#include "povs_kernel.cuh"
#include "povs_metrics.cuh"
#include "povs_mt19937.h"

using povs::IterParams;

namespace {

thread_local char g_err[512] = "";

int fail(int code, const char* fmt, ...)
{
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
    return code;
}

int cuda_fail(cudaError_t e, const char* what)
{
    return fail(POVS_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

#define POVS_CUDA_TRY(expr)                                \
    do {                                                   \
        cudaError_t e_ = (expr);                           \
        if (e_ != cudaSuccess) return cuda_fail(e_, #expr); \
    } while (0)

bool is_pow2(int64_t x) { return x > 0 && (x & (x - 1)) == 0; }

int ilog2(int64_t x)
{
    int s = 0;
    while ((int64_t{1} << s) < x) ++s;
    return s;
}

// ------------------------------------------------------------------------------------------
// Kernel table.
// ------------------------------------------------------------------------------------------

using KernelFn = void (*)(IterParams);

template <bool INJ, bool BULK, bool PUSH, bool RING, bool WIDE = false>
KernelFn kernel_for_epl(int epl)
{
    switch (epl) {
    case 1: return povs::povs_iteration_kernel<1, INJ, BULK, PUSH, RING, false, WIDE>;
    case 2: return povs::povs_iteration_kernel<2, INJ, BULK, PUSH, RING, false, WIDE>;
    case 4: return povs::povs_iteration_kernel<4, INJ, BULK, PUSH, RING, false, WIDE>;
    case 8: return povs::povs_iteration_kernel<8, INJ, BULK, PUSH, RING, false, WIDE>;
    case 16: return povs::povs_iteration_kernel<16, INJ, BULK, PUSH, RING, false, WIDE>;
    case 32: return povs::povs_iteration_kernel<32, INJ, BULK, PUSH, RING, false, WIDE>;
    default: return nullptr;
    }
}

// wide: slabs of 512 to 1024 bytes (TMA loads only), whose stores keep several loads in flight.
template <bool INJ, bool PUSH>
KernelFn kernel_for(int epl, bool bulk, bool ring, bool wide)
{
    if (!bulk) return kernel_for_epl<INJ, false, PUSH, true>(epl);
    if (wide)
        return ring ? kernel_for_epl<INJ, true, PUSH, true, true>(epl) : kernel_for_epl<INJ, true, PUSH, false, true>(epl);
    return ring ? kernel_for_epl<INJ, true, PUSH, true>(epl) : kernel_for_epl<INJ, true, PUSH, false>(epl);
}

// Packed units (device randomness, in place, ring positions): 2 to 32 sort elements per lane.
// CHUNK: plain-load rows stored as 16-byte chunks of each member's run.
template <bool BULK, bool CHUNK = false, bool FAST = false>
KernelFn packed_kernel_for_epl(int epl)
{
    switch (epl) {
    case 2: return povs::povs_iteration_kernel<2, false, BULK, false, true, true, false, CHUNK, FAST>;
    case 4: return povs::povs_iteration_kernel<4, false, BULK, false, true, true, false, CHUNK, FAST>;
    case 8: return povs::povs_iteration_kernel<8, false, BULK, false, true, true, false, CHUNK, FAST>;
    case 16: return povs::povs_iteration_kernel<16, false, BULK, false, true, true, false, CHUNK, FAST>;
    case 32: return povs::povs_iteration_kernel<32, false, BULK, false, true, true, false, CHUNK, FAST>;
    default: return nullptr;
    }
}

// Push mode exists for device randomness only.  Plain-load kernels always carry ring positions.
KernelFn select_kernel(int epl, bool injected, bool bulk, bool push = false, bool ring = false, bool packed = false,
                       bool wide = false, bool chunk = false, bool fast = false)
{
    if (packed)
        return bulk ? (fast ? packed_kernel_for_epl<true, false, true>(epl) : packed_kernel_for_epl<true>(epl))
                    : (chunk ? packed_kernel_for_epl<false, true>(epl) : packed_kernel_for_epl<false>(epl));
    if (push) return kernel_for<false, true>(epl, bulk, ring, wide);
    if (injected) return kernel_for<true, false>(epl, bulk, ring, wide);
    return kernel_for<false, false>(epl, bulk, ring, wide);
}

// Decks (all decks of a batch together) of at least this many bytes are launched one iteration
// at a time with programmatic dependent launches; smaller ones replay a cached CUDA graph.
constexpr int64_t GRAPH_MAX_BYTES = int64_t{32} << 20;

// Bulk-loaded units (stages) of at most this many bytes use the ring-position kernels.
constexpr int RING_STAGE_BYTES = 16 * 1024;

// Packed plain-load units write 16-byte chunks of each member's destination run (0: one lane per
// vector piece of a row, as unpacked units do).
#ifndef POVS_CHUNKED_STORES
#define POVS_CHUNKED_STORES 1
#endif

// Packed TMA-loaded units of power-of-two rows take their FAST kernel variants (0: never).
#ifndef POVS_UNIFORM_MEMBER_STORES
#define POVS_UNIFORM_MEMBER_STORES 1
#endif

// ------------------------------------------------------------------------------------------
// Tuning knobs (process-wide; defaults chosen by measurement on B200).
// ------------------------------------------------------------------------------------------

struct Tuning {
    int stage_cap = 32 * 1024; // max bytes of one stage; larger vblocks are split into column slabs
    int n_stages = 8;          // max shared-memory data stages per CTA
    int movers = 4;            // warps that copy rows
    int permuters = 4;         // warps that compute members and permutations
    int force_plain = 0;       // 1 = never use TMA bulk loads
    int copy_bytes = 8192;     // target bytes per bulk copy on the whole-row path
    int pack_bytes = 16 * 1024; // packed units: several small vblocks per unit up to this size (0 = off)
};
Tuning g_tuning;
std::mutex g_tuning_mu;
std::atomic<unsigned long long> g_peer_wait_ns{povs::PEER_WAIT_LIMIT_NS};

// ------------------------------------------------------------------------------------------
// Per-device context.
// ------------------------------------------------------------------------------------------

struct GraphKey {
    KernelFn fn;
    int grid, block, smem, iterations;
    bool pdl;
    bool operator==(const GraphKey& o) const
    {
        return fn == o.fn && grid == o.grid && block == o.block && smem == o.smem && iterations == o.iterations &&
               pdl == o.pdl;
    }
};
struct GraphKeyHash {
    size_t operator()(const GraphKey& k) const
    {
        size_t h = reinterpret_cast<size_t>(k.fn);
        h = h * 1000003u ^ static_cast<size_t>(k.grid);
        h = h * 1000003u ^ static_cast<size_t>(k.block);
        h = h * 1000003u ^ static_cast<size_t>(k.smem);
        h = h * 1000003u ^ static_cast<size_t>(k.iterations);
        h = h * 1000003u ^ static_cast<size_t>(k.pdl);
        return h;
    }
};
struct CachedGraph {
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    std::vector<cudaGraphNode_t> nodes;
};

// Permutation tables of the reference NumPy path's distribution for one (P, V, n_rows % P).
struct NpTable {
    uint16_t* dev = nullptr;
    std::vector<int64_t> off; // 2 * MAX_VBLOCK entries, -1 where a class cannot occur
};

struct DeviceCtx {
    bool ready = false;
    int sm_count = 0;
    int smem_optin = 0;  // max dynamic shared memory per block
    int smem_per_sm = 0; // shared memory per multiprocessor
    int max_threads_per_sm = 0;
    int* status = nullptr;
    std::mutex mu; // guards the graph cache and launches that reuse it
    std::unordered_map<GraphKey, CachedGraph, GraphKeyHash> graphs;
    std::mutex np_mu; // guards np_tables
    std::unordered_map<uint64_t, NpTable> np_tables;
};

constexpr int MAX_DEVICES = 64;
constexpr int64_t SLAB_FLOOR_BYTES = 2048; // preferred minimum width of a column slab
DeviceCtx g_ctx[MAX_DEVICES];
std::mutex g_ctx_mu;

struct DeviceGuard {
    int prev = -1;
    bool changed = false;
    int enter(int dev)
    {
        cudaError_t e = cudaGetDevice(&prev);
        if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
        if (prev != dev) {
            e = cudaSetDevice(dev);
            if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
            changed = true;
        }
        return POVS_OK;
    }
    ~DeviceGuard()
    {
        if (changed) cudaSetDevice(prev);
    }
};

int set_smem_attr_all(int smem)
{
    for (int mode = 0; mode < 3; ++mode)
        for (int bulk = 0; bulk < 2; ++bulk)
            for (int ring = 0; ring < 2; ++ring)
                for (int wide = 0; wide <= bulk; ++wide)
                    for (int epl = 1; epl <= 32; epl <<= 1) {
                        KernelFn fn = select_kernel(epl, mode == 1, bulk != 0, mode == 2, ring != 0, false, wide != 0);
                        cudaError_t e = cudaFuncSetAttribute(reinterpret_cast<const void*>(fn),
                                                             cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
                        if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute");
                    }
    for (int kind = 0; kind < 4; ++kind) // packed: TMA loads (kind 3: uniform-member stores), plain loads, chunked
        for (int epl = 2; epl <= 32; epl <<= 1) {
            KernelFn fn = select_kernel(epl, false, kind == 0 || kind == 3, false, true, true, false, kind == 2, kind == 3);
            cudaError_t e = cudaFuncSetAttribute(reinterpret_cast<const void*>(fn),
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
            if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute");
        }
    return POVS_OK;
}

// Called with the device current.
int get_ctx(int dev, DeviceCtx** out)
{
    if (dev < 0 || dev >= MAX_DEVICES) return fail(POVS_ERR_INVALID_ARGUMENT, "device %d out of range", dev);
    std::lock_guard<std::mutex> lk(g_ctx_mu);
    DeviceCtx& c = g_ctx[dev];
    if (!c.ready) {
        cudaDeviceProp prop;
        POVS_CUDA_TRY(cudaGetDeviceProperties(&prop, dev));
        if (prop.major < 10)
            return fail(POVS_ERR_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a (B200)", dev,
                        prop.major, prop.minor);
        c.sm_count = prop.multiProcessorCount;
        c.smem_optin = static_cast<int>(prop.sharedMemPerBlockOptin);
        c.smem_per_sm = static_cast<int>(prop.sharedMemPerMultiprocessor);
        c.max_threads_per_sm = prop.maxThreadsPerMultiProcessor;
        int r = set_smem_attr_all(c.smem_optin);
        if (r != POVS_OK) return r;
        POVS_CUDA_TRY(cudaFuncSetAttribute(reinterpret_cast<const void*>(povs::povs_travel_histogram_kernel),
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           povs::HIST_SMEM_MAX_BINS * static_cast<int>(sizeof(uint32_t))));
        POVS_CUDA_TRY(cudaMalloc(&c.status, sizeof(int)));
        POVS_CUDA_TRY(cudaMemset(c.status, 0, sizeof(int)));
        c.ready = true;
    }
    *out = &c;
    return POVS_OK;
}

// ------------------------------------------------------------------------------------------
// Launch planning.
// ------------------------------------------------------------------------------------------

struct Plan {
    KernelFn fn = nullptr;
    int grid = 0, block = 0, smem = 0, epl = 0;
    bool bulk = false;
    int pack = 1;
    bool wide = false;  // the WIDE kernel variant (slabs of 512 to 1024 bytes)
    bool chunk = false; // the CHUNK kernel variant (packed plain-load rows, chunked stores)
    bool fast = false;  // the FAST kernel variant (packed TMA-loaded rows, uniform-member stores)
};

int plan_launch(IterParams& p, const DeviceCtx& c, bool injected, Plan& out, bool push = false,
                bool plain_loads = false)
{
    Tuning t;
    {
        std::lock_guard<std::mutex> lk(g_tuning_mu);
        t = g_tuning;
    }
    const int64_t vp = static_cast<int64_t>(p.vblock) * p.pblock;
    if (vp > POVS_MAX_VP)
        return fail(POVS_ERR_UNSUPPORTED, "virtual_block_size * physical_block_size = %lld exceeds %d",
                    static_cast<long long>(vp), POVS_MAX_VP);
    // Packed units: small vblocks (device randomness, in place over the whole list of vblocks)
    // travel `pack` at a time, so the per-unit costs (barrier round trips, member ranks, the sort
    // network, copy issue) are paid once per pack * V * P rows.  One member per lane (pack * V <= 32),
    // one sort of pack * V * P <= 1024 keys, at least 2 keys per lane, unit bytes <= pack_bytes.
    uintptr_t addr = 0;
    for (int i = 0; i < p.n_shards; ++i) addr |= reinterpret_cast<uintptr_t>(p.shard_base[i]);
    if (push)
        for (int i = 0; i < p.n_shards; ++i) addr |= reinterpret_cast<uintptr_t>(p.dst_base[i]);
    if (p.n_decks > 1) addr |= static_cast<uintptr_t>(p.deck_stride);
    int vec = 16;
    while (vec > 1 && ((p.row_bytes % vec) != 0 || (addr % vec) != 0)) vec >>= 1;
    const bool bulk = (vec == 16) && !t.force_plain && !plain_loads;

    // TMA-loaded rows whose 16-byte chunk count is not a power of two (48, 80, 96, .. bytes) spread
    // over the lanes unevenly, and ran best in larger units (measured on B200, 2 GiB decks: 48-byte
    // rows, P = 64, 3,756 GB/s in 12 KiB units, 5,387 in 48 KiB; 96-byte rows, P = 32, 4,418 in 12
    // KiB, 5,359 in 24 KiB), so their packs may grow to three times pack_bytes.
    const int64_t pack_limit =
        (bulk && (p.row_bytes & (p.row_bytes - 1)) != 0) ? 3 * static_cast<int64_t>(t.pack_bytes) : t.pack_bytes;
    // A packed unit is always staged as whole rows: beyond the stage cap it must still fit three
    // whole-row stages next to their permutation slots (the slab rule below then keeps whole rows).
    auto packed_fits = [&](int64_t pk) {
        const int64_t urows = pk * vp;
        const int64_t ubytes = urows * p.row_bytes;
        if (ubytes <= t.stage_cap) return true;
        const int mv = std::max(1, std::min(!bulk ? std::min(t.movers, 2) : t.movers, 15));
        const int pm = std::max(1, std::min(!bulk ? std::min(t.permuters, 2) : t.permuters, 16 - mv));
        const int slots = std::min(povs::MAX_SLOTS, 3 + 2 * pm);
        const int64_t fixed = povs::cta_smem_bytes(0, 0, slots, static_cast<int>(urows), p.pblock);
        return fixed + 3 * (((ubytes + 127) / 128) * 128 + 16) <= c.smem_optin;
    };
    int pack = 1;
    if (!injected && !push && p.vb_begin == 0 && p.vb_step == 1 && t.pack_bytes > 0 && vp >= 8) {
        while (2 * pack * p.vblock <= 32 && 2 * pack * vp <= POVS_MAX_VP &&
               2 * pack * vp * p.row_bytes <= pack_limit && pack < p.n_vblocks && packed_fits(2 * pack))
            pack *= 2;
        if (pack * vp < 64) pack = 1;
    }
    const int64_t unit_vp = pack * vp;
    int epl = 1;
    while (32 * epl < unit_vp) epl <<= 1;
    p.pack = pack;
    p.unit_vp = static_cast<int32_t>(unit_vp);
    p.groups_per_deck = (p.n_vblocks + pack - 1) / pack;

    // Slab width: whole rows when a vblock fits a stage, else the widest 128-byte (or vec) multiple that does.
    // A stage holds a unit's rows: the vblock's V*P rows in place (pack of them when packed), one
    // member's P rows in push mode.
    const int64_t stage_rows = push ? p.pblock : unit_vp;
    // Packed units run best as several small CTAs per SM, each its own pipeline (measured on B200,
    // 2 GiB decks of 16- to 256-byte rows): at most 4 stages with TMA loads (5 or 6 stages were
    // 0-14 % slower on every shape tried, 3 or 2 slower still); with plain loads, whose issuing warp
    // waits for its loads, 2 mover and 2 permuter warps and at most 3 stages.
    const int stage_limit = pack == 1 ? t.n_stages : std::min(t.n_stages, bulk ? 4 : 3);
    const int max_stages = std::max(2, std::min(stage_limit, povs::MAX_STAGES));
    const int movers = std::max(1, std::min(pack > 1 && !bulk ? std::min(t.movers, 2) : t.movers, 15));
    const int permuters =
        std::max(1, std::min(pack > 1 && !bulk ? std::min(t.permuters, 2) : t.permuters, 16 - movers));
    // Permutation slots: the stages' worth plus room for every permuter to work ahead.
    auto slots_for = [&](int stages) { return std::min(povs::MAX_SLOTS, stages + 2 * permuters); };
    // The most stages (<= max_stages) of slabs of sl bytes per row that fit next to their
    // permutation slots (slots_for(n) of them for n stages).
    auto stages_for = [&](int64_t sl, int64_t& stage_bytes) {
        stage_bytes = ((stage_rows * sl + 127) / 128) * 128;
        const int64_t per_stage = stage_bytes + 16;
        int n = max_stages;
        while (n > 0 && povs::cta_smem_bytes(0, 0, slots_for(n), static_cast<int>(unit_vp), p.pblock) + n * per_stage >
                            c.smem_optin)
            --n;
        return n;
    };
    int64_t slab = p.row_bytes;
    if (stage_rows * p.row_bytes > t.stage_cap) {
        const int64_t fit = t.stage_cap / stage_rows;
        const int64_t gran = fit >= 128 ? 128 : vec;
        slab = std::max<int64_t>(vec, (fit / gran) * gran);
        // Wide rows: pieces of at least SLAB_FLOOR bytes per row and stage when three such stages
        // fit (per-row copies of 1 KiB and less leave the DRAM well short of its copy bandwidth).
        const int64_t wide = std::min<int64_t>(p.row_bytes, ((SLAB_FLOOR_BYTES / vec) * vec));
        int64_t sb = 0;
        if (slab < wide && stages_for(wide, sb) >= 3) slab = wide;
        // Narrow rows in a vblock of many rows: per-row copies under 128 bytes are slow (measured on
        // B200: 64-byte rows in 1024-row vblocks moved 0.59 TB/s as 32-byte slabs), so take the
        // fewest slabs per row, whole rows first, with which two stages fit.
        if (slab < std::min<int64_t>(p.row_bytes, 128)) {
            for (int64_t n = 1; n * vec <= p.row_bytes; ++n) {
                const int64_t cand = (((p.row_bytes + n - 1) / n + vec - 1) / vec) * vec;
                if (cand <= slab) break;
                if (stages_for(cand, sb) >= 2) {
                    slab = cand;
                    break;
                }
            }
        }
    }
    if (pack > 1 && slab != p.row_bytes)
        return fail(POVS_ERR_UNSUPPORTED, "packed units of %lld bytes do not fit as whole rows",
                    static_cast<long long>(stage_rows * p.row_bytes));
    int64_t stage_bytes = 0;
    int nst = stages_for(slab, stage_bytes);
    // Shrink the slab until at least two stages fit.
    while (nst < 2 && slab > vec) {
        slab = std::max<int64_t>(vec, ((slab / 2) / vec) * vec);
        nst = stages_for(slab, stage_bytes);
    }
    if (nst < 2)
        return fail(POVS_ERR_UNSUPPORTED, "a vblock of %lld rows does not fit shared memory", static_cast<long long>(vp));
    const int kp = slots_for(nst);

    const int warps = movers + permuters;
    const int cta_smem =
        povs::cta_smem_bytes(nst, static_cast<int>(stage_bytes), kp, static_cast<int>(unit_vp), p.pblock);
    const int per_sm_by_smem = std::max(1, c.smem_per_sm / (cta_smem + 1024));
    const int per_sm_by_threads = std::max(1, c.max_threads_per_sm / (warps * 32));
    const int ctas_per_sm = std::min(per_sm_by_smem, per_sm_by_threads);
    const int64_t n_mine = push ? (p.push_rank < 0 ? p.n_pblocks : p.n_pblocks / std::max(1, p.n_shards) + 1)
                           : pack > 1 ? p.groups_per_deck * p.n_decks
                                      : (p.vb_begin < p.n_vblocks * p.n_decks
                                             ? (p.n_vblocks * p.n_decks - p.vb_begin + p.vb_step - 1) / p.vb_step
                                             : 0);
    const int grid = static_cast<int>(std::min<int64_t>(std::max<int64_t>(1, n_mine), static_cast<int64_t>(c.sm_count) * ctas_per_sm));

    p.slab_bytes = static_cast<int32_t>(slab);
    p.n_slabs = static_cast<int32_t>((p.row_bytes + slab - 1) / slab);
    p.stage_bytes = static_cast<int32_t>(stage_bytes);
    p.n_stages = nst;
    p.vec_bytes = vec;
    // Plain-load plans of whole rows in 4-byte multiples copy asynchronously when a pblock's run is at
    // least 192 bytes (measured on B200: 12- to 1020-byte rows 1.2-18x faster; with runs of 64-128
    // bytes the many small copies lost to the issuing warp's synchronous loads).  force_plain = 2
    // keeps the synchronous loads, for comparison.
    p.async_plain =
        (!bulk && vec >= 4 && p.n_slabs == 1 && static_cast<int64_t>(p.pblock) * p.row_bytes >= 192 && t.force_plain != 2)
            ? 1 : 0;
    p.copy_rows = static_cast<int32_t>(std::max<int64_t>(1, std::min<int64_t>(p.pblock, t.copy_bytes / p.row_bytes)));
    // Packed plain-load units of 4-byte-multiple rows under 128 bytes store 16-byte chunks of each
    // member's destination run.  A run is at most one packed unit, which three whole-row stages
    // must fit in shared memory (under 76 KiB): inside the 2^17 bytes for which the kernel's
    // division by multiplication with row_magic is exact.
    // Each lane takes 16-byte chunks of one member run at a time, so members of fewer than 32
    // chunks, or of 33 to 63, leave lanes idle: measured on B200 (2 GiB decks, GB/s, one lane per
    // piece -> chunks) 12-byte rows P = 64 (768-byte members) 1769 -> 1724 and V = 4, P = 16 (192 bytes)
    // 947 -> 720, against 4 B P = 128 (512 bytes) 879 -> 997, 20 B P = 64 1716 -> 2126, 24 B P = 128
    // 3200 -> 3872, 28 B P = 64 2667 -> 3563, 56 B P = 64 3998 -> 5168.
    const int64_t member_bytes = static_cast<int64_t>(p.pblock) * p.row_bytes;
    p.chunked_store = (pack > 1 && !bulk && vec >= 4 && p.row_bytes < 128 && POVS_CHUNKED_STORES &&
                       (member_bytes == 512 || member_bytes >= 1024))
                          ? 1
                          : 0;
    p.row_magic = p.chunked_store
                      ? static_cast<uint32_t>(((uint64_t{1} << 32) + static_cast<uint64_t>(p.row_bytes) - 1) /
                                              static_cast<uint64_t>(p.row_bytes))
                      : 0u;
    p.n_slots = kp;
    p.n_movers = movers;
    p.n_permuters = permuters;

    out.wide = bulk && pack == 1 && slab >= 512 && slab <= 1024;
    out.chunk = p.chunked_store != 0;
    // Packed TMA-loaded rows of a power-of-two count of 16-byte chunks, at most a pblock per warp
    // store pass: the FAST kernels, whose full units take the member of each pass once per warp.
    const int64_t chunks_per_row = p.row_bytes / 16;
    const int64_t rows_per_pass = chunks_per_row > 0 && chunks_per_row < 32 ? 32 / chunks_per_row : 1;
    out.fast = bulk && pack > 1 && chunks_per_row > 0 && (chunks_per_row & (chunks_per_row - 1)) == 0 &&
               rows_per_pass <= p.pblock && POVS_UNIFORM_MEMBER_STORES;
    out.fn = select_kernel(epl, injected, bulk, push, stage_bytes <= RING_STAGE_BYTES || pack > 1, pack > 1,
                           out.wide, out.chunk, out.fast);
    out.grid = std::max(1, grid);
    out.block = warps * 32;
    out.smem = cta_smem;
    out.epl = epl;
    out.bulk = bulk;
    out.pack = pack;
    return POVS_OK;
}

int check_common(void* data, int64_t n_rows, int64_t row_bytes, int32_t pblock, int32_t vblock, int32_t iterations)
{
    if (data == nullptr) return fail(POVS_ERR_INVALID_ARGUMENT, "data is NULL");
    if (n_rows < 2) return fail(POVS_ERR_INVALID_ARGUMENT, "deck must have at least 2 rows, has %lld", static_cast<long long>(n_rows));
    if (row_bytes < 1) return fail(POVS_ERR_INVALID_ARGUMENT, "row_bytes must be positive");
    if (iterations < 0) return fail(POVS_ERR_INVALID_ARGUMENT, "iterations (%d) must be non-negative", iterations);
    if (!is_pow2(pblock)) return fail(POVS_ERR_INVALID_ARGUMENT, "pblock size (%d) must be a power of 2", pblock);
    if (!is_pow2(vblock) || vblock < 2)
        return fail(POVS_ERR_INVALID_ARGUMENT, "vblock size (%d) must be a power of 2 and at least 2", vblock);
    if (vblock > POVS_MAX_VBLOCK)
        return fail(POVS_ERR_UNSUPPORTED, "vblock size (%d) exceeds %d", vblock, POVS_MAX_VBLOCK);
    if (row_bytes > (int64_t{1} << 40)) return fail(POVS_ERR_UNSUPPORTED, "row_bytes too large");
    return POVS_OK;
}

// Randomness mode of a flag set (POVS_ERR_INVALID_ARGUMENT when both reference modes are asked for).
int rng_mode_of(uint32_t flags, int32_t* mode)
{
    const bool cuda_rng = (flags & POVS_FLAG_REFERENCE_RNG) != 0;
    const bool numpy_rng = (flags & POVS_FLAG_REFERENCE_NUMPY) != 0;
    if (cuda_rng && numpy_rng)
        return fail(POVS_ERR_INVALID_ARGUMENT, "POVS_FLAG_REFERENCE_RNG and POVS_FLAG_REFERENCE_NUMPY exclude each other");
    *mode = cuda_rng ? povs::RNG_REFERENCE_CUDA : numpy_rng ? povs::RNG_REFERENCE_NUMPY : povs::RNG_UNIFORM;
    return POVS_OK;
}

constexpr int64_t NP_TABLE_MAX_BYTES = int64_t{128} << 20;

// For the NumPy path's distribution: numpy.random.RandomState(s).shuffle(arange(n)) for every seed
// s in 1..999 and every valid-row count n a vblock can have (m whole pblocks, or m-1 whole ones and
// the deck's truncated last pblock, m = 1..V), built on the host once per geometry and device and
// kept until povs_release_v1.  Sets the launch parameters that point at it.
int prepare_np_table(DeviceCtx& c, povs::IterParams& p)
{
    if (p.rng_mode != povs::RNG_REFERENCE_NUMPY) return POVS_OK;
    const int P = p.pblock, V = p.vblock;
    const int t = static_cast<int>(p.n_rows % P);
    const uint64_t key = (static_cast<uint64_t>(P) << 40) | (static_cast<uint64_t>(V) << 32) | static_cast<uint32_t>(t);
    std::lock_guard<std::mutex> lk(c.np_mu);
    auto it = c.np_tables.find(key);
    if (it == c.np_tables.end()) {
        NpTable tab;
        tab.off.assign(2 * povs::MAX_VBLOCK, -1);
        std::vector<int> sizes(2 * V, 0);
        int64_t total = 0;
        for (int m = 1; m <= V; ++m) {
            sizes[m - 1] = m * P;
            if (t > 0) sizes[V + m - 1] = (m - 1) * P + t;
        }
        for (int n : sizes) total += static_cast<int64_t>(n) * 999;
        if (total * 2 > NP_TABLE_MAX_BYTES)
            return fail(POVS_ERR_UNSUPPORTED, "the NumPy-path permutation tables for P = %d, V = %d need %lld bytes "
                        "(limit %lld)", P, V, static_cast<long long>(total * 2), static_cast<long long>(NP_TABLE_MAX_BYTES));
        std::vector<uint16_t> host(static_cast<size_t>(total));
        int64_t at = 0;
        for (int cls = 0; cls < 2 * V; ++cls) {
            const int n = sizes[cls];
            if (n <= 0) continue;
            tab.off[cls] = at;
            for (uint32_t sd = 1; sd <= 999; ++sd) {
                povs::numpy_legacy_shuffle(sd, n, host.data() + at);
                at += n;
            }
        }
        POVS_CUDA_TRY(cudaMalloc(&tab.dev, static_cast<size_t>(total) * sizeof(uint16_t)));
        const cudaError_t e = cudaMemcpy(tab.dev, host.data(), static_cast<size_t>(total) * sizeof(uint16_t),
                                         cudaMemcpyHostToDevice);
        if (e != cudaSuccess) {
            cudaFree(tab.dev);
            return cuda_fail(e, "cudaMemcpy(NumPy-path tables)");
        }
        it = c.np_tables.emplace(key, std::move(tab)).first;
    }
    p.np_table = it->second.dev;
    p.np_trunc = t;
    for (int i = 0; i < 2 * povs::MAX_VBLOCK; ++i) p.np_off[i] = it->second.off[i];
    return POVS_OK;
}

int64_t sum_rows(const int64_t* shard_rows, int32_t n_shards)
{
    int64_t n = 0;
    for (int i = 0; i < n_shards; ++i) n += shard_rows[i] > 0 ? shard_rows[i] : 0;
    return n;
}

void fill_geometry(IterParams& p, void* data, int64_t n_rows, int64_t row_bytes, int32_t pblock, int32_t vblock,
                   int* status)
{
    std::memset(&p, 0, sizeof(p));
    p.data = static_cast<uint8_t*>(data);
    p.n_rows = n_rows;
    p.row_bytes = row_bytes;
    p.pblock = pblock;
    p.pblock_shift = ilog2(pblock);
    p.vblock = vblock;
    p.vp = pblock * vblock;
    p.n_pblocks = (n_rows + pblock - 1) / pblock;
    p.n_vblocks = (p.n_pblocks + vblock - 1) / vblock;
    p.pack = 1;
    p.unit_vp = p.vp;
    p.vp_shift = ilog2(p.vp);
    p.vblock_shift = ilog2(vblock);
    p.idx_bits = std::max(5, ilog2(p.vp));
    p.groups_per_deck = p.n_vblocks;
    p.status = status;
    p.n_shards = 1;
    p.shard_base[0] = p.data;
    p.shard_start[0] = 0;
    p.shard_start[1] = n_rows;
    p.vb_begin = 0;
    p.vb_step = 1;
    p.push_rank = -1;
    p.n_decks = 1;
    p.deck_stride = 0;
    p.deck_seeds = nullptr;
}

// `chained`: launch as a programmatic dependent launch of the kernel before it on `s` (the
// iteration kernel waits for that grid to complete before any data access; a predecessor that is
// not a kernel keeps ordinary stream order).
int launch_direct(const Plan& pl, const IterParams& p, cudaStream_t s, bool chained = false)
{
    void* args[] = {const_cast<IterParams*>(&p)};
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(pl.grid);
    cfg.blockDim = dim3(pl.block);
    cfg.dynamicSmemBytes = static_cast<size_t>(pl.smem);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = chained ? 1 : 0;
    cudaError_t e = cudaLaunchKernelExC(&cfg, reinterpret_cast<const void*>(pl.fn), args);
    if (e != cudaSuccess) return cuda_fail(e, "cudaLaunchKernelExC");
    return POVS_OK;
}

// Replays `iters` chained iteration kernels as one CUDA graph (cached per launch shape).
int launch_graph(DeviceCtx& c, const Plan& pl, std::vector<IterParams>& ps, cudaStream_t s, bool pdl)
{
    const int iters = static_cast<int>(ps.size());
    std::lock_guard<std::mutex> lk(c.mu);
    GraphKey key{pl.fn, pl.grid, pl.block, pl.smem, iters, pdl};
    auto it = c.graphs.find(key);
    if (it == c.graphs.end()) {
        CachedGraph g;
        POVS_CUDA_TRY(cudaGraphCreate(&g.graph, 0));
        cudaGraphNode_t prev = nullptr;
        for (int i = 0; i < iters; ++i) {
            cudaKernelNodeParams kp{};
            void* args[] = {&ps[i]};
            kp.func = reinterpret_cast<void*>(pl.fn);
            kp.gridDim = dim3(pl.grid);
            kp.blockDim = dim3(pl.block);
            kp.sharedMemBytes = static_cast<unsigned>(pl.smem);
            kp.kernelParams = args;
            cudaGraphNode_t node;
            if (pdl) {
                // Programmatic edge: iteration i+1 may launch once every CTA of iteration i has
                // signalled (its movers still wait for iteration i to complete).
                POVS_CUDA_TRY(cudaGraphAddKernelNode(&node, g.graph, nullptr, 0, &kp));
                if (prev) {
                    cudaGraphEdgeData ed{};
                    ed.from_port = cudaGraphKernelNodePortProgrammatic;
                    ed.to_port = 0;
                    ed.type = cudaGraphDependencyTypeProgrammatic;
                    POVS_CUDA_TRY(cudaGraphAddDependencies_v2(g.graph, &prev, &node, &ed, 1));
                }
            } else {
                POVS_CUDA_TRY(cudaGraphAddKernelNode(&node, g.graph, prev ? &prev : nullptr, prev ? 1 : 0, &kp));
            }
            g.nodes.push_back(node);
            prev = node;
        }
        POVS_CUDA_TRY(cudaGraphInstantiate(&g.exec, g.graph, 0));
        it = c.graphs.emplace(key, std::move(g)).first;
    } else {
        for (int i = 0; i < iters; ++i) {
            cudaKernelNodeParams kp{};
            void* args[] = {&ps[i]};
            kp.func = reinterpret_cast<void*>(pl.fn);
            kp.gridDim = dim3(pl.grid);
            kp.blockDim = dim3(pl.block);
            kp.sharedMemBytes = static_cast<unsigned>(pl.smem);
            kp.kernelParams = args;
            POVS_CUDA_TRY(cudaGraphExecKernelNodeSetParams(it->second.exec, it->second.nodes[i], &kp));
        }
    }
    POVS_CUDA_TRY(cudaGraphLaunch(it->second.exec, s));
    return POVS_OK;
}

int read_status(DeviceCtx& c, int32_t* out)
{
    POVS_CUDA_TRY(cudaDeviceSynchronize());
    int v = 0;
    POVS_CUDA_TRY(cudaMemcpy(&v, c.status, sizeof(int), cudaMemcpyDeviceToHost));
    POVS_CUDA_TRY(cudaMemset(c.status, 0, sizeof(int)));
    if (out) *out = v;
    return POVS_OK;
}

// Applies a shard table (pointers + row counts) to launch parameters; checks the layout.
int set_shards(IterParams& p, void* const* shard_ptrs, const int64_t* shard_rows, int32_t n_shards)
{
    if (shard_ptrs == nullptr || shard_rows == nullptr || n_shards < 1 || n_shards > povs::MAX_SHARDS)
        return fail(POVS_ERR_INVALID_ARGUMENT, "between 1 and %d shards are supported", povs::MAX_SHARDS);
    int64_t start = 0;
    for (int i = 0; i < n_shards; ++i) {
        if (shard_ptrs[i] == nullptr) return fail(POVS_ERR_INVALID_ARGUMENT, "shard %d pointer is NULL", i);
        if (shard_rows[i] < p.pblock)
            return fail(POVS_ERR_UNSUPPORTED, "shard %d has %lld rows; every shard needs at least P = %d rows", i,
                        static_cast<long long>(shard_rows[i]), p.pblock);
        p.shard_base[i] = static_cast<uint8_t*>(shard_ptrs[i]);
        p.shard_start[i] = start;
        start += shard_rows[i];
    }
    p.shard_start[n_shards] = start;
    p.n_shards = n_shards;
    p.data = p.shard_base[0];
    return POVS_OK;
}

int shuffle_on_device(void* data, int64_t n_rows, int64_t row_bytes, const int64_t* offsets, int32_t n_offsets,
                      int32_t iterations, int32_t pblock, int32_t vblock, uint64_t seed, DeviceCtx& c,
                      cudaStream_t s, uint32_t flags, void* const* shard_ptrs = nullptr,
                      const int64_t* shard_rows = nullptr, int32_t n_shards = 1, int64_t n_decks = 1,
                      int64_t deck_stride = 0, const uint64_t* deck_seeds = nullptr, bool plain_loads = false,
                      bool chain_first = true)
{
    IterParams base;
    fill_geometry(base, data, n_rows, row_bytes, pblock, vblock, c.status);
    if (shard_ptrs != nullptr) {
        int rs = set_shards(base, shard_ptrs, shard_rows, n_shards);
        if (rs != POVS_OK) return rs;
    }
    base.n_decks = n_decks;
    base.deck_stride = deck_stride;
    base.deck_seeds = deck_seeds;
    base.seed = seed;
    int r = rng_mode_of(flags, &base.rng_mode);
    if (r != POVS_OK) return r;
    r = prepare_np_table(c, base);
    if (r != POVS_OK) return r;
    base.n_offsets = n_offsets;
    for (int i = 0; i < n_offsets; ++i) base.offsets[i] = offsets[i];
    Plan pl;
    r = plan_launch(base, c, false, pl, false, plain_loads);
    if (r != POVS_OK) return r;
    if (iterations == 0) return POVS_OK;
    std::vector<IterParams> ps(static_cast<size_t>(iterations), base);
    for (int i = 0; i < iterations; ++i) ps[i].iteration = static_cast<uint32_t>(i);
    const bool pdl = (flags & POVS_FLAG_NO_PDL) == 0;
    // With programmatic dependent launches, decks of GRAPH_MAX_BYTES and more are launched one
    // iteration at a time, every launch (the first too) chained to the kernel before it on the
    // stream: the first iteration then overlaps the previous call's last one (measured +1-3 % on
    // 64-256 MiB decks against one graph per call).  Smaller decks, whose iterations take a few
    // microseconds, replay a cached graph to keep the host's launch cost off the GPU's timeline.
    // Routes whose stream holds copies or event waits before the first iteration (host decks) pass
    // chain_first = false: their first launch keeps ordinary stream order.  So does a batch with a
    // device seed array: the permuter warps read it before they wait for the prior grid, and the
    // caller may have written it with the kernel just before this call.
    if (deck_seeds != nullptr) chain_first = false;
    const int64_t deck_bytes = n_rows * row_bytes * std::max<int64_t>(1, n_decks);
    const bool direct = iterations == 1 || (flags & POVS_FLAG_NO_GRAPH) || (pdl && deck_bytes >= GRAPH_MAX_BYTES);
    if (direct) {
        for (int i = 0; i < iterations; ++i) {
            r = launch_direct(pl, ps[i], s, pdl && (i > 0 || chain_first));
            if (r != POVS_OK) return r;
        }
    } else {
        r = launch_graph(c, pl, ps, s, pdl);
        if (r != POVS_OK) return r;
    }
    if (flags & POVS_FLAG_SYNC) {
        POVS_CUDA_TRY(cudaStreamSynchronize(s));
        int32_t st = 0;
        r = read_status(c, &st);
        if (r != POVS_OK) return r;
        if (st != 0) return fail(POVS_ERR_DEVICE_STATUS, "device status 0x%x after shuffle", st);
    }
    return POVS_OK;
}

int check_offsets(const int64_t* offsets, int32_t n_offsets, int64_t n_rows)
{
    if (offsets == nullptr || n_offsets < 1) return fail(POVS_ERR_INVALID_ARGUMENT, "at least one offset is required");
    if (n_offsets > POVS_MAX_OFFSETS)
        return fail(POVS_ERR_UNSUPPORTED, "%d offsets exceed the limit of %d", n_offsets, POVS_MAX_OFFSETS);
    for (int i = 0; i < n_offsets; ++i)
        if (offsets[i] < 0 || offsets[i] >= n_rows)
            return fail(POVS_ERR_INVALID_ARGUMENT, "offset at index %d (%lld) must be in [0, %lld)", i,
                        static_cast<long long>(offsets[i]), static_cast<long long>(n_rows));
    return POVS_OK;
}

} // namespace

// ------------------------------------------------------------------------------------------
// Exported entry points.
// ------------------------------------------------------------------------------------------

extern "C" int povs_shuffle_v1(void* data, int64_t n_rows, int64_t row_bytes, const int64_t* offsets,
                               int32_t n_offsets, int32_t iterations, int32_t pblock, int32_t vblock, uint64_t seed,
                               int32_t device, void* stream, uint32_t flags)
{
    g_err[0] = '\0';
    int r = check_common(data, n_rows, row_bytes, pblock, vblock, iterations);
    if (r != POVS_OK) return r;
    r = check_offsets(offsets, n_offsets, n_rows);
    if (r != POVS_OK) return r;
    DeviceGuard dg;
    r = dg.enter(device);
    if (r != POVS_OK) return r;
    DeviceCtx* c = nullptr;
    r = get_ctx(device, &c);
    if (r != POVS_OK) return r;
    return shuffle_on_device(data, n_rows, row_bytes, offsets, n_offsets, iterations, pblock, vblock, seed, *c,
                             static_cast<cudaStream_t>(stream), flags);
}

extern "C" int povs_shuffle_host_v1(void* host_data, void* device_buffer, int64_t n_rows, int64_t row_bytes,
                                    const int64_t* offsets, int32_t n_offsets, int32_t iterations, int32_t pblock,
                                    int32_t vblock, uint64_t seed, int32_t device, void* stream, uint32_t flags)
{
    g_err[0] = '\0';
    if (host_data == nullptr) return fail(POVS_ERR_INVALID_ARGUMENT, "host_data is NULL");
    int r = check_common(device_buffer, n_rows, row_bytes, pblock, vblock, iterations);
    if (r != POVS_OK) return r;
    r = check_offsets(offsets, n_offsets, n_rows);
    if (r != POVS_OK) return r;
    DeviceGuard dg;
    r = dg.enter(device);
    if (r != POVS_OK) return r;
    DeviceCtx* c = nullptr;
    r = get_ctx(device, &c);
    if (r != POVS_OK) return r;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const size_t bytes = static_cast<size_t>(n_rows) * static_cast<size_t>(row_bytes);
    POVS_CUDA_TRY(cudaMemcpyAsync(device_buffer, host_data, bytes, cudaMemcpyHostToDevice, s));
    r = shuffle_on_device(device_buffer, n_rows, row_bytes, offsets, n_offsets, iterations, pblock, vblock, seed, *c,
                          s, flags & ~POVS_FLAG_SYNC, nullptr, nullptr, 1, 1, 0, nullptr, false, false);
    if (r != POVS_OK) return r;
    POVS_CUDA_TRY(cudaMemcpyAsync(host_data, device_buffer, bytes, cudaMemcpyDeviceToHost, s));
    POVS_CUDA_TRY(cudaStreamSynchronize(s));
    if (flags & POVS_FLAG_SYNC) {
        int32_t st = 0;
        r = read_status(*c, &st);
        if (r != POVS_OK) return r;
        if (st != 0) return fail(POVS_ERR_DEVICE_STATUS, "device status 0x%x after shuffle", st);
    }
    return POVS_OK;
}

extern "C" int povs_shuffle_host_batch_v1(void* const* host_decks, int32_t n_decks, void* const* device_buffers,
                                          int32_t n_buffers, int64_t n_rows, int64_t row_bytes,
                                          const int64_t* offsets, int32_t n_offsets, int32_t iterations,
                                          int32_t pblock, int32_t vblock, const uint64_t* seeds, int32_t device,
                                          void* stream, uint32_t flags)
{
    g_err[0] = '\0';
    if (host_decks == nullptr || device_buffers == nullptr || seeds == nullptr || n_decks < 0 || n_buffers < 1 ||
        n_buffers > 8)
        return fail(POVS_ERR_INVALID_ARGUMENT, "host_decks, seeds and 1..8 device_buffers are required");
    for (int i = 0; i < n_decks; ++i)
        if (host_decks[i] == nullptr) return fail(POVS_ERR_INVALID_ARGUMENT, "host deck %d is NULL", i);
    for (int b = 0; b < n_buffers; ++b) {
        int r = check_common(device_buffers[b], n_rows, row_bytes, pblock, vblock, iterations);
        if (r != POVS_OK) return r;
    }
    int r = check_offsets(offsets, n_offsets, n_rows);
    if (r != POVS_OK) return r;
    DeviceGuard dg;
    r = dg.enter(device);
    if (r != POVS_OK) return r;
    DeviceCtx* c = nullptr;
    r = get_ctx(device, &c);
    if (r != POVS_OK) return r;
    if (n_decks == 0) return POVS_OK;

    // Deck d uses buffer d % n_buffers.  Copies in, the iterations and copies out run on three
    // streams ordered by events, so deck d's copy out overlaps deck d+1's copy in and iterations.
    // Deck d's copy in waits for the copy out of the deck that last used its buffer and of the
    // previous deck with the same host pointer (a deck listed twice is shuffled twice in order).
    cudaStream_t user = static_cast<cudaStream_t>(stream);
    cudaStream_t s_in = nullptr, s_out = nullptr, s_cmp = nullptr;
    std::vector<cudaEvent_t> ev;
    const size_t bytes = static_cast<size_t>(n_rows) * static_cast<size_t>(row_bytes);
    auto cleanup = [&]() {
        for (cudaEvent_t e : ev)
            if (e) cudaEventDestroy(e);
        if (s_in) cudaStreamDestroy(s_in);
        if (s_out) cudaStreamDestroy(s_out);
        if (s_cmp) cudaStreamDestroy(s_cmp);
    };
    auto run = [&]() -> int {
        POVS_CUDA_TRY(cudaStreamCreateWithFlags(&s_in, cudaStreamNonBlocking));
        POVS_CUDA_TRY(cudaStreamCreateWithFlags(&s_out, cudaStreamNonBlocking));
        POVS_CUDA_TRY(cudaStreamCreateWithFlags(&s_cmp, cudaStreamNonBlocking));
        ev.assign(static_cast<size_t>(2 * n_buffers + n_decks + 1), nullptr);
        for (auto& e : ev) POVS_CUDA_TRY(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
        cudaEvent_t start = ev[2 * n_buffers];
        auto out_done = [&](int d) { return ev[static_cast<size_t>(2 * n_buffers + 1 + d)]; };
        std::unordered_map<void*, int> last_use;
        // Work already queued on the caller's stream (e.g. writes to the buffers) comes first.
        POVS_CUDA_TRY(cudaEventRecord(start, user));
        POVS_CUDA_TRY(cudaStreamWaitEvent(s_in, start, 0));
        POVS_CUDA_TRY(cudaStreamWaitEvent(s_cmp, start, 0));
        POVS_CUDA_TRY(cudaStreamWaitEvent(s_out, start, 0));
        for (int d = 0; d < n_decks; ++d) {
            const int b = d % n_buffers;
            cudaEvent_t in_done = ev[2 * b], cmp_done = ev[2 * b + 1];
            if (d >= n_buffers) POVS_CUDA_TRY(cudaStreamWaitEvent(s_in, out_done(d - n_buffers), 0));
            auto prev = last_use.find(host_decks[d]);
            if (prev != last_use.end()) POVS_CUDA_TRY(cudaStreamWaitEvent(s_in, out_done(prev->second), 0));
            last_use[host_decks[d]] = d;
            POVS_CUDA_TRY(cudaMemcpyAsync(device_buffers[b], host_decks[d], bytes, cudaMemcpyHostToDevice, s_in));
            POVS_CUDA_TRY(cudaEventRecord(in_done, s_in));
            POVS_CUDA_TRY(cudaStreamWaitEvent(s_cmp, in_done, 0));
            int rc = shuffle_on_device(device_buffers[b], n_rows, row_bytes, offsets, n_offsets, iterations, pblock,
                                       vblock, seeds[d], *c, s_cmp, flags & ~POVS_FLAG_SYNC, nullptr, nullptr, 1,
                                       1, 0, nullptr, false, false);
            if (rc != POVS_OK) return rc;
            POVS_CUDA_TRY(cudaEventRecord(cmp_done, s_cmp));
            POVS_CUDA_TRY(cudaStreamWaitEvent(s_out, cmp_done, 0));
            POVS_CUDA_TRY(cudaMemcpyAsync(host_decks[d], device_buffers[b], bytes, cudaMemcpyDeviceToHost, s_out));
            POVS_CUDA_TRY(cudaEventRecord(out_done(d), s_out));
        }
        POVS_CUDA_TRY(cudaStreamSynchronize(s_in));
        POVS_CUDA_TRY(cudaStreamSynchronize(s_cmp));
        POVS_CUDA_TRY(cudaStreamSynchronize(s_out));
        if (flags & POVS_FLAG_SYNC) {
            int32_t st = 0;
            int rs = read_status(*c, &st);
            if (rs != POVS_OK) return rs;
            if (st != 0) return fail(POVS_ERR_DEVICE_STATUS, "device status 0x%x after shuffle", st);
        }
        return POVS_OK;
    };
    r = run();
    cleanup();
    return r;
}

extern "C" int povs_apply_v1(void* data, int64_t n_rows, int64_t row_bytes, int32_t pblock, int32_t vblock,
                             int32_t iterations, const int64_t* offsets_per_iter, const int64_t* assign,
                             const int32_t* perms, int32_t sort_members, int32_t device, void* stream)
{
    g_err[0] = '\0';
    int r = check_common(data, n_rows, row_bytes, pblock, vblock, iterations);
    if (r != POVS_OK) return r;
    if (iterations > 0 && (offsets_per_iter == nullptr || assign == nullptr || perms == nullptr))
        return fail(POVS_ERR_INVALID_ARGUMENT, "offsets_per_iter, assign and perms are required");
    for (int i = 0; i < iterations; ++i)
        if (offsets_per_iter[i] < 0 || offsets_per_iter[i] >= n_rows)
            return fail(POVS_ERR_INVALID_ARGUMENT, "offset of iteration %d (%lld) must be in [0, %lld)", i,
                        static_cast<long long>(offsets_per_iter[i]), static_cast<long long>(n_rows));
    DeviceGuard dg;
    r = dg.enter(device);
    if (r != POVS_OK) return r;
    DeviceCtx* c = nullptr;
    r = get_ctx(device, &c);
    if (r != POVS_OK) return r;
    IterParams base;
    fill_geometry(base, data, n_rows, row_bytes, pblock, vblock, c->status);
    base.sort_members = sort_members ? 1 : 0;
    Plan pl;
    r = plan_launch(base, *c, true, pl);
    if (r != POVS_OK) return r;
    const int64_t n_slots = base.n_vblocks * vblock;
    const int64_t n_perm = base.n_vblocks * static_cast<int64_t>(base.vp);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    for (int i = 0; i < iterations; ++i) {
        IterParams p = base;
        p.iteration = static_cast<uint32_t>(i);
        p.offset = offsets_per_iter[i];
        p.assign = assign + i * n_slots;
        p.perms = perms + i * n_perm;
        r = launch_direct(pl, p, s);
        if (r != POVS_OK) return r;
    }
    return POVS_OK;
}

extern "C" int povs_device_status_v1(int32_t device, int32_t* status)
{
    g_err[0] = '\0';
    DeviceGuard dg;
    int r = dg.enter(device);
    if (r != POVS_OK) return r;
    DeviceCtx* c = nullptr;
    r = get_ctx(device, &c);
    if (r != POVS_OK) return r;
    return read_status(*c, status);
}

extern "C" int povs_release_v1(void)
{
    g_err[0] = '\0';
    std::lock_guard<std::mutex> lk(g_ctx_mu);
    int prev = -1;
    cudaGetDevice(&prev);
    for (int d = 0; d < MAX_DEVICES; ++d) {
        DeviceCtx& c = g_ctx[d];
        if (!c.ready) continue;
        cudaSetDevice(d);
        std::lock_guard<std::mutex> lk2(c.mu);
        for (auto& kv : c.graphs) {
            if (kv.second.exec) cudaGraphExecDestroy(kv.second.exec);
            if (kv.second.graph) cudaGraphDestroy(kv.second.graph);
        }
        c.graphs.clear();
        {
            std::lock_guard<std::mutex> lk3(c.np_mu);
            for (auto& kv : c.np_tables)
                if (kv.second.dev) cudaFree(kv.second.dev);
            c.np_tables.clear();
        }
        if (c.status) cudaFree(c.status);
        c.status = nullptr;
        c.ready = false;
    }
    if (prev >= 0) cudaSetDevice(prev);
    return POVS_OK;
}

extern "C" const char* povs_last_error_string(void) { return g_err; }

extern "C" int32_t povs_version(void) { return 100; }

// Tuning and introspection.
extern "C" int povs_set_tuning_v1(int32_t stage_cap, int32_t n_stages, int32_t movers, int32_t permuters,
                                  int32_t force_plain, int32_t copy_bytes)
{
    g_err[0] = '\0';
    if (stage_cap < 1024 || n_stages < 2 || n_stages > povs::MAX_STAGES || movers < 1 || permuters < 1 ||
        movers + permuters > 16 || copy_bytes < 16)
        return fail(POVS_ERR_INVALID_ARGUMENT, "tuning out of range");
    std::lock_guard<std::mutex> lk(g_tuning_mu);
    g_tuning.stage_cap = stage_cap;
    g_tuning.n_stages = n_stages;
    g_tuning.movers = movers;
    g_tuning.permuters = permuters;
    g_tuning.copy_bytes = copy_bytes;
    g_tuning.force_plain = force_plain < 0 ? 0 : (force_plain > 2 ? 2 : force_plain);
    return POVS_OK;
}

extern "C" int povs_set_pack_bytes_v1(int32_t pack_bytes)
{
    g_err[0] = '\0';
    if (pack_bytes < 0) return fail(POVS_ERR_INVALID_ARGUMENT, "pack_bytes (%d) must be non-negative", pack_bytes);
    std::lock_guard<std::mutex> lk(g_tuning_mu);
    g_tuning.pack_bytes = pack_bytes;
    return POVS_OK;
}

namespace {
// The values povs_describe_plan_v1 and povs_plan_for_resources_v1 report, in the header's order.
int plan_values(const IterParams& p, const Plan& pl, int sm_count, int64_t* out, int32_t n_out)
{
    const int64_t vals[] = {pl.grid,       pl.block,     pl.smem,       pl.epl,        pl.bulk ? 1 : 0,
                            p.slab_bytes,  p.n_slabs,    p.n_stages,    p.stage_bytes, p.vec_bytes,
                            p.n_vblocks,   sm_count,     p.copy_rows,   p.n_slots,     p.n_movers,
                            p.n_permuters, pl.pack,      p.unit_vp,     pl.wide ? 1 : 0, pl.chunk ? 1 : 0};
    const int n = std::min<int>(n_out, static_cast<int>(sizeof(vals) / sizeof(vals[0])));
    for (int i = 0; i < n; ++i) out[i] = vals[i];
    return n;
}
} // namespace

extern "C" int povs_describe_plan_v1(void* data, int64_t n_rows, int64_t row_bytes, int32_t pblock, int32_t vblock,
                                     int32_t device, int64_t* out, int32_t n_out)
{
    g_err[0] = '\0';
    int r = check_common(data, n_rows, row_bytes, pblock, vblock, 1);
    if (r != POVS_OK) return r;
    DeviceGuard dg;
    r = dg.enter(device);
    if (r != POVS_OK) return r;
    DeviceCtx* c = nullptr;
    r = get_ctx(device, &c);
    if (r != POVS_OK) return r;
    IterParams p;
    fill_geometry(p, data, n_rows, row_bytes, pblock, vblock, c->status);
    Plan pl;
    r = plan_launch(p, *c, false, pl);
    if (r != POVS_OK) return r;
    return plan_values(p, pl, c->sm_count, out, n_out);
}

extern "C" int povs_plan_for_resources_v1(uint64_t data_address, int64_t n_rows, int64_t row_bytes, int32_t pblock,
                                          int32_t vblock, int32_t sm_count, int32_t smem_optin, int32_t smem_per_sm,
                                          int32_t max_threads_per_sm, int64_t* out, int32_t n_out)
{
    g_err[0] = '\0';
    void* data = reinterpret_cast<void*>(static_cast<uintptr_t>(data_address));
    int r = check_common(data, n_rows, row_bytes, pblock, vblock, 1);
    if (r != POVS_OK) return r;
    if (out == nullptr || n_out < 0) return fail(POVS_ERR_INVALID_ARGUMENT, "out is NULL");
    if (sm_count < 1 || smem_optin < 1024 || smem_per_sm < smem_optin || max_threads_per_sm < 512)
        return fail(POVS_ERR_INVALID_ARGUMENT, "device resources out of range");
    DeviceCtx c;
    c.sm_count = sm_count;
    c.smem_optin = smem_optin;
    c.smem_per_sm = smem_per_sm;
    c.max_threads_per_sm = max_threads_per_sm;
    IterParams p;
    fill_geometry(p, data, n_rows, row_bytes, pblock, vblock, nullptr);
    Plan pl;
    r = plan_launch(p, c, false, pl);
    if (r != POVS_OK) return r;
    return plan_values(p, pl, c.sm_count, out, n_out);
}

// ------------------------------------------------------------------------------------------
// Allocation-free injected-randomness entry (povs_apply_static_v1).
//
// Some callers cannot call cudaMalloc once they are running: a process whose memory pool has
// already reserved the GPU's memory (a framework caching allocator holding every free byte), or
// a service that allows no allocation after start-up so that its memory use stays fixed.  For
// them this entry point stages the injected randomness in a fixed scratch array that is part of
// the library image (a file-scope __device__ array, present on every GPU that loads the library
// until the process exits) instead of in buffers the caller would have to allocate, keeps its
// status word there too, and launches the kernels directly (no CUDA graph, no per-device context).
//
// Layout of the array: [status word, 256 bytes][assignment, int64][permutations, int32].  Every
// call reuses it and it keeps the last call's contents; the status word is cleared at the start
// of every call.  Calls that overlap on the GPU (different streams, or different host threads
// without ordering) race on the array.
// ------------------------------------------------------------------------------------------

namespace {

constexpr size_t STATIC_SCRATCH_BYTES = size_t{POVS_STATIC_SCRATCH_BYTES};
constexpr size_t STATIC_STATUS_BYTES = 256;

static __device__ __align__(256) unsigned char g_static_scratch[STATIC_SCRATCH_BYTES];

struct StaticDevice {
    bool ready = false;
    unsigned char* scratch = nullptr; // device address of g_static_scratch on this device
    DeviceCtx props;                  // SM count and shared-memory limits only (nothing allocated)
};
StaticDevice g_static_dev[MAX_DEVICES];
std::mutex g_static_mu;

// First call on a device: look up the scratch array's device address (with that device current)
// and read the launch limits.  No allocation happens here or later.
int static_setup(int dev, StaticDevice** out)
{
    if (dev < 0 || dev >= MAX_DEVICES) return fail(POVS_ERR_INVALID_ARGUMENT, "device %d out of range", dev);
    std::lock_guard<std::mutex> lk(g_static_mu);
    StaticDevice& s = g_static_dev[dev];
    if (!s.ready) {
        cudaDeviceProp prop;
        POVS_CUDA_TRY(cudaGetDeviceProperties(&prop, dev));
        if (prop.major < 10)
            return fail(POVS_ERR_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a (B200)", dev,
                        prop.major, prop.minor);
        void* ptr = nullptr;
        POVS_CUDA_TRY(cudaGetSymbolAddress(&ptr, g_static_scratch));
        s.props.sm_count = prop.multiProcessorCount;
        s.props.smem_optin = static_cast<int>(prop.sharedMemPerBlockOptin);
        s.props.smem_per_sm = static_cast<int>(prop.sharedMemPerMultiprocessor);
        s.props.max_threads_per_sm = prop.maxThreadsPerMultiProcessor;
        int r = set_smem_attr_all(s.props.smem_optin);
        if (r != POVS_OK) return r;
        s.scratch = static_cast<unsigned char*>(ptr);
        s.ready = true;
    }
    *out = &s;
    return POVS_OK;
}

} // namespace

extern "C" int povs_apply_static_v1(void* data, int64_t n_rows, int64_t row_bytes, int32_t pblock, int32_t vblock,
                                    int32_t iterations, const int64_t* offsets_per_iter, const int64_t* assign_host,
                                    const int32_t* perms_host, int32_t sort_members, int32_t device, void* stream,
                                    uint32_t flags)
{
    g_err[0] = '\0';
    if (flags & ~POVS_FLAG_SYNC)
        return fail(POVS_ERR_INVALID_ARGUMENT, "povs_apply_static_v1 accepts only POVS_FLAG_SYNC (flags 0x%x)", flags);
    int r = check_common(data, n_rows, row_bytes, pblock, vblock, iterations);
    if (r != POVS_OK) return r;
    if (iterations > 0 && (offsets_per_iter == nullptr || assign_host == nullptr || perms_host == nullptr))
        return fail(POVS_ERR_INVALID_ARGUMENT, "offsets_per_iter, assign_host and perms_host are required");
    for (int i = 0; i < iterations; ++i)
        if (offsets_per_iter[i] < 0 || offsets_per_iter[i] >= n_rows)
            return fail(POVS_ERR_INVALID_ARGUMENT, "offset of iteration %d (%lld) must be in [0, %lld)", i,
                        static_cast<long long>(offsets_per_iter[i]), static_cast<long long>(n_rows));
    const int64_t n_pblocks = (n_rows + pblock - 1) / pblock;
    const int64_t n_vblocks = (n_pblocks + vblock - 1) / vblock;
    const int64_t n_slots = n_vblocks * vblock;
    const int64_t n_perm = n_vblocks * static_cast<int64_t>(pblock) * vblock;
    const size_t assign_bytes = static_cast<size_t>(n_slots) * sizeof(int64_t);
    const size_t perm_offset = STATIC_STATUS_BYTES + ((assign_bytes + 255) / 256) * 256;
    const size_t need = perm_offset + static_cast<size_t>(n_perm) * sizeof(int32_t);
    if (need > STATIC_SCRATCH_BYTES)
        return fail(POVS_ERR_UNSUPPORTED,
                    "one iteration's injected randomness needs %zu bytes of scratch; povs_apply_static_v1 holds at "
                    "most %zu (use povs_apply_v1 with caller-allocated device buffers)",
                    need, STATIC_SCRATCH_BYTES);
    DeviceGuard dg;
    r = dg.enter(device);
    if (r != POVS_OK) return r;
    StaticDevice* sd = nullptr;
    r = static_setup(device, &sd);
    if (r != POVS_OK) return r;

    int* status = reinterpret_cast<int*>(sd->scratch);
    int64_t* assign_dev = reinterpret_cast<int64_t*>(sd->scratch + STATIC_STATUS_BYTES);
    int32_t* perms_dev = reinterpret_cast<int32_t*>(sd->scratch + perm_offset);
    IterParams base;
    fill_geometry(base, data, n_rows, row_bytes, pblock, vblock, status);
    base.sort_members = sort_members ? 1 : 0;
    Plan pl;
    r = plan_launch(base, sd->props, true, pl);
    if (r != POVS_OK) return r;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    POVS_CUDA_TRY(cudaMemsetAsync(status, 0, sizeof(int), s));
    for (int i = 0; i < iterations; ++i) {
        // Stream order keeps each iteration's copies behind the previous iteration's kernel.
        POVS_CUDA_TRY(cudaMemcpyAsync(assign_dev, assign_host + i * n_slots, assign_bytes, cudaMemcpyHostToDevice, s));
        POVS_CUDA_TRY(cudaMemcpyAsync(perms_dev, perms_host + i * n_perm, static_cast<size_t>(n_perm) * sizeof(int32_t),
                                      cudaMemcpyHostToDevice, s));
        IterParams p = base;
        p.iteration = static_cast<uint32_t>(i);
        p.offset = offsets_per_iter[i];
        p.assign = assign_dev;
        p.perms = perms_dev;
        r = launch_direct(pl, p, s);
        if (r != POVS_OK) return r;
    }
    if (flags & POVS_FLAG_SYNC) {
        POVS_CUDA_TRY(cudaStreamSynchronize(s));
        int v = 0;
        POVS_CUDA_TRY(cudaMemcpy(&v, status, sizeof(int), cudaMemcpyDeviceToHost));
        if (v != 0) return fail(POVS_ERR_DEVICE_STATUS, "device status 0x%x after povs_apply_static_v1", v);
    }
    return POVS_OK;
}

// ------------------------------------------------------------------------------------------
// Decks split into shards.
// ------------------------------------------------------------------------------------------

namespace {

// Points the launch at source and destination shard tables (push mode) for iteration `it`:
// even iterations read the decks and write the scratch buffers, odd ones the other way round.
void set_push_direction(IterParams& p, void* const* shard_ptrs, void* const* scratch_ptrs, int32_t n_shards, int it)
{
    for (int i = 0; i < n_shards; ++i) {
        uint8_t* deck = static_cast<uint8_t*>(shard_ptrs[i]);
        uint8_t* scratch = static_cast<uint8_t*>(scratch_ptrs[i]);
        p.shard_base[i] = (it % 2 == 0) ? deck : scratch;
        p.dst_base[i] = (it % 2 == 0) ? scratch : deck;
    }
}

int check_scratch(void* const* scratch_ptrs, int32_t n_shards)
{
    for (int i = 0; i < n_shards; ++i)
        if (scratch_ptrs[i] == nullptr) return fail(POVS_ERR_INVALID_ARGUMENT, "scratch buffer %d is NULL", i);
    return POVS_OK;
}

} // namespace

extern "C" int povs_shuffle_shards_v1(void* const* shard_ptrs, void* const* scratch_ptrs, const int64_t* shard_rows,
                                      int32_t n_shards, int64_t row_bytes, const int64_t* offsets, int32_t n_offsets,
                                      int32_t iterations, int32_t pblock, int32_t vblock, uint64_t seed,
                                      int32_t device, void* stream, uint32_t flags)
{
    g_err[0] = '\0';
    if (shard_ptrs == nullptr || shard_rows == nullptr || n_shards < 1 || n_shards > povs::MAX_SHARDS)
        return fail(POVS_ERR_INVALID_ARGUMENT, "between 1 and %d shards are supported", povs::MAX_SHARDS);
    const int64_t n_rows = sum_rows(shard_rows, n_shards);
    int r = check_common(shard_ptrs[0], n_rows, row_bytes, pblock, vblock, iterations);
    if (r != POVS_OK) return r;
    r = check_offsets(offsets, n_offsets, n_rows);
    if (r != POVS_OK) return r;
    if (scratch_ptrs != nullptr && (r = check_scratch(scratch_ptrs, n_shards)) != POVS_OK) return r;
    DeviceGuard dg;
    r = dg.enter(device);
    if (r != POVS_OK) return r;
    DeviceCtx* c = nullptr;
    r = get_ctx(device, &c);
    if (r != POVS_OK) return r;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (scratch_ptrs == nullptr)
        return shuffle_on_device(shard_ptrs[0], n_rows, row_bytes, offsets, n_offsets, iterations, pblock, vblock, seed,
                                 *c, s, flags, shard_ptrs, shard_rows, n_shards);

    // Double-buffered (push) mode in one launch per iteration over every pblock.
    IterParams base;
    fill_geometry(base, shard_ptrs[0], n_rows, row_bytes, pblock, vblock, c->status);
    r = set_shards(base, shard_ptrs, shard_rows, n_shards);
    if (r != POVS_OK) return r;
    base.seed = seed;
    r = rng_mode_of(flags, &base.rng_mode);
    if (r != POVS_OK) return r;
    r = prepare_np_table(*c, base);
    if (r != POVS_OK) return r;
    base.n_offsets = n_offsets;
    for (int i = 0; i < n_offsets; ++i) base.offsets[i] = offsets[i];
    base.push_rank = -1;
    set_push_direction(base, shard_ptrs, scratch_ptrs, n_shards, 0);
    Plan pl;
    r = plan_launch(base, *c, false, pl, true);
    if (r != POVS_OK) return r;
    for (int i = 0; i < iterations; ++i) {
        IterParams p = base;
        p.iteration = static_cast<uint32_t>(i);
        set_push_direction(p, shard_ptrs, scratch_ptrs, n_shards, i);
        r = launch_direct(pl, p, s);
        if (r != POVS_OK) return r;
    }
    if (iterations % 2 == 1)
        for (int i = 0; i < n_shards; ++i)
            POVS_CUDA_TRY(cudaMemcpyAsync(shard_ptrs[i], scratch_ptrs[i],
                                          static_cast<size_t>(shard_rows[i]) * static_cast<size_t>(row_bytes),
                                          cudaMemcpyDeviceToDevice, s));
    if (flags & POVS_FLAG_SYNC) {
        POVS_CUDA_TRY(cudaStreamSynchronize(s));
        int32_t st = 0;
        r = read_status(*c, &st);
        if (r != POVS_OK) return r;
        if (st != 0) return fail(POVS_ERR_DEVICE_STATUS, "device status 0x%x after shuffle", st);
    }
    return POVS_OK;
}

extern "C" int povs_shuffle_sharded_v1(void* const* shard_ptrs, void* const* scratch_ptrs, const int64_t* shard_rows,
                                       int32_t n_shards, int32_t rank, int64_t row_bytes, const int64_t* offsets,
                                       int32_t n_offsets, int32_t iterations, int32_t pblock, int32_t vblock,
                                       uint64_t seed, void* const* peer_flags, uint32_t epoch_base, int32_t device,
                                       void* stream, uint32_t flags)
{
    g_err[0] = '\0';
    if (shard_ptrs == nullptr || shard_rows == nullptr || n_shards < 1 || n_shards > povs::MAX_SHARDS)
        return fail(POVS_ERR_INVALID_ARGUMENT, "between 1 and %d shards are supported", povs::MAX_SHARDS);
    if (rank < 0 || rank >= n_shards) return fail(POVS_ERR_INVALID_ARGUMENT, "rank %d out of range", rank);
    if (peer_flags == nullptr) return fail(POVS_ERR_INVALID_ARGUMENT, "peer_flags is NULL");
    for (int i = 0; i < n_shards; ++i)
        if (peer_flags[i] == nullptr) return fail(POVS_ERR_INVALID_ARGUMENT, "flag array of rank %d is NULL", i);
    const int64_t n_rows = sum_rows(shard_rows, n_shards);
    int r = check_common(shard_ptrs[rank], n_rows, row_bytes, pblock, vblock, iterations);
    if (r != POVS_OK) return r;
    r = check_offsets(offsets, n_offsets, n_rows);
    if (r != POVS_OK) return r;
    const bool push = scratch_ptrs != nullptr;
    if (push && (r = check_scratch(scratch_ptrs, n_shards)) != POVS_OK) return r;
    DeviceGuard dg;
    r = dg.enter(device);
    if (r != POVS_OK) return r;
    DeviceCtx* c = nullptr;
    r = get_ctx(device, &c);
    if (r != POVS_OK) return r;

    IterParams base;
    fill_geometry(base, shard_ptrs[rank], n_rows, row_bytes, pblock, vblock, c->status);
    r = set_shards(base, shard_ptrs, shard_rows, n_shards);
    if (r != POVS_OK) return r;
    base.seed = seed;
    r = rng_mode_of(flags, &base.rng_mode);
    if (r != POVS_OK) return r;
    r = prepare_np_table(*c, base);
    if (r != POVS_OK) return r;
    base.n_offsets = n_offsets;
    for (int i = 0; i < n_offsets; ++i) base.offsets[i] = offsets[i];
    if (push) {
        // Every rank moves the rows of the pblocks stored in its own shard, each straight to its
        // destination slot in the other buffer: a row crosses NVLink at most once.
        base.push_rank = rank;
        set_push_direction(base, shard_ptrs, scratch_ptrs, n_shards, 0);
    } else {
        // Every rank reads and writes back whole vblocks rank, rank + n_shards, ...
        base.vb_begin = rank;
        base.vb_step = n_shards;
    }
    Plan pl;
    r = plan_launch(base, *c, false, pl, push);
    if (r != POVS_OK) return r;

    povs::PeerBarrierParams q{};
    for (int i = 0; i < n_shards; ++i) q.flags[i] = static_cast<uint32_t*>(peer_flags[i]);
    q.n_ranks = n_shards;
    q.rank = rank;
    q.status = c->status;
    q.limit_ns = g_peer_wait_ns.load();
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    auto barrier = [&](uint32_t epoch) -> int {
        q.epoch = epoch;
        void* args[] = {&q};
        cudaError_t e = cudaLaunchKernel(reinterpret_cast<const void*>(povs::povs_peer_barrier_kernel), dim3(1),
                                         dim3(32), args, 0, s);
        return e == cudaSuccess ? POVS_OK : cuda_fail(e, "cudaLaunchKernel(barrier)");
    };
    // Every shard must be ready before any rank reads it, and every rank must have finished writing
    // before anyone goes on: a barrier before the first iteration and after each one.
    r = barrier(epoch_base + 1);
    if (r != POVS_OK) return r;
    for (int i = 0; i < iterations; ++i) {
        IterParams p = base;
        p.iteration = static_cast<uint32_t>(i);
        if (push) set_push_direction(p, shard_ptrs, scratch_ptrs, n_shards, i);
        r = launch_direct(pl, p, s);
        if (r != POVS_OK) return r;
        r = barrier(epoch_base + 2 + static_cast<uint32_t>(i));
        if (r != POVS_OK) return r;
    }
    // After an odd number of push iterations the rows are in the scratch buffers; every peer has
    // finished writing this rank's scratch (last barrier), so copy it back locally.
    if (push && iterations % 2 == 1)
        POVS_CUDA_TRY(cudaMemcpyAsync(shard_ptrs[rank], scratch_ptrs[rank],
                                      static_cast<size_t>(shard_rows[rank]) * static_cast<size_t>(row_bytes),
                                      cudaMemcpyDeviceToDevice, s));
    if (flags & POVS_FLAG_SYNC) {
        POVS_CUDA_TRY(cudaStreamSynchronize(s));
        int32_t st = 0;
        r = read_status(*c, &st);
        if (r != POVS_OK) return r;
        if (st != 0) return fail(POVS_ERR_DEVICE_STATUS, "device status 0x%x after sharded shuffle", st);
    }
    return POVS_OK;
}

// ------------------------------------------------------------------------------------------
// CUDA IPC: map another process's shard (or flag array) into this one.
// ------------------------------------------------------------------------------------------

namespace {
using GetAddressRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

int address_range(const void* ptr, CUdeviceptr* base)
{
    static GetAddressRangeFn fn = nullptr;
    static std::mutex mu;
    {
        std::lock_guard<std::mutex> lk(mu);
        if (fn == nullptr) {
            void* f = nullptr;
            cudaDriverEntryPointQueryResult q;
            cudaError_t e = cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q);
            if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || f == nullptr)
                return fail(POVS_ERR_CUDA, "cuMemGetAddressRange entry point unavailable");
            fn = reinterpret_cast<GetAddressRangeFn>(f);
        }
    }
    size_t size = 0;
    if (fn(base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
        return fail(POVS_ERR_INVALID_ARGUMENT, "pointer %p is not device memory", ptr);
    return POVS_OK;
}
} // namespace

extern "C" int povs_ipc_export_v1(const void* ptr, int32_t device, void* handle_out, int64_t* offset_out)
{
    g_err[0] = '\0';
    if (ptr == nullptr || handle_out == nullptr || offset_out == nullptr)
        return fail(POVS_ERR_INVALID_ARGUMENT, "NULL argument");
    DeviceGuard dg;
    int r = dg.enter(device);
    if (r != POVS_OK) return r;
    CUdeviceptr base = 0;
    r = address_range(ptr, &base);
    if (r != POVS_OK) return r;
    cudaIpcMemHandle_t h;
    POVS_CUDA_TRY(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)));
    std::memcpy(handle_out, &h, sizeof(h));
    *offset_out = static_cast<int64_t>(reinterpret_cast<uintptr_t>(ptr) - static_cast<uintptr_t>(base));
    return POVS_OK;
}

extern "C" int povs_ipc_import_v1(const void* handle, int64_t offset, int32_t device, void** ptr_out, void** base_out)
{
    g_err[0] = '\0';
    if (handle == nullptr || ptr_out == nullptr || base_out == nullptr || offset < 0)
        return fail(POVS_ERR_INVALID_ARGUMENT, "invalid argument");
    DeviceGuard dg;
    int r = dg.enter(device);
    if (r != POVS_OK) return r;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    void* base = nullptr;
    POVS_CUDA_TRY(cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess));
    *base_out = base;
    *ptr_out = static_cast<uint8_t*>(base) + offset;
    return POVS_OK;
}

extern "C" int povs_ipc_close_v1(void* base, int32_t device)
{
    g_err[0] = '\0';
    DeviceGuard dg;
    int r = dg.enter(device);
    if (r != POVS_OK) return r;
    POVS_CUDA_TRY(cudaIpcCloseMemHandle(base));
    return POVS_OK;
}

extern "C" int povs_enable_peer_access_v1(int32_t device, int32_t peer)
{
    g_err[0] = '\0';
    if (device == peer) return POVS_OK;
    int can = 0;
    POVS_CUDA_TRY(cudaDeviceCanAccessPeer(&can, device, peer));
    if (!can) return fail(POVS_ERR_UNSUPPORTED, "device %d cannot access device %d's memory", device, peer);
    DeviceGuard dg;
    int r = dg.enter(device);
    if (r != POVS_OK) return r;
    const cudaError_t e = cudaDeviceEnablePeerAccess(peer, 0);
    if (e == cudaErrorPeerAccessAlreadyEnabled) {
        cudaGetLastError(); // clear the recorded error so that a later cudaGetLastError does not report it
        return POVS_OK;
    }
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceEnablePeerAccess");
    return POVS_OK;
}

// ------------------------------------------------------------------------------------------
// Batched decks and shuffle-bias metrics.
// ------------------------------------------------------------------------------------------

extern "C" int povs_shuffle_batch_v1(void* data, int64_t n_decks, int64_t deck_stride, int64_t n_rows,
                                     int64_t row_bytes, const int64_t* offsets, int32_t n_offsets, int32_t iterations,
                                     int32_t pblock, int32_t vblock, const uint64_t* seeds, int32_t device,
                                     void* stream, uint32_t flags)
{
    g_err[0] = '\0';
    int r = check_common(data, n_rows, row_bytes, pblock, vblock, iterations);
    if (r != POVS_OK) return r;
    r = check_offsets(offsets, n_offsets, n_rows);
    if (r != POVS_OK) return r;
    if (n_decks < 1) return fail(POVS_ERR_INVALID_ARGUMENT, "n_decks (%lld) must be positive", static_cast<long long>(n_decks));
    if (seeds == nullptr) return fail(POVS_ERR_INVALID_ARGUMENT, "seeds is NULL");
    if (n_decks > 1 && deck_stride < n_rows * row_bytes)
        return fail(POVS_ERR_INVALID_ARGUMENT, "deck_stride (%lld) is smaller than a deck (%lld bytes)",
                    static_cast<long long>(deck_stride), static_cast<long long>(n_rows * row_bytes));
    if ((flags & ~uint32_t{POVS_FLAG_NO_GRAPH | POVS_FLAG_SYNC | POVS_FLAG_REFERENCE_RNG | POVS_FLAG_NO_PDL |
                           POVS_FLAG_REFERENCE_NUMPY}) != 0)
        return fail(POVS_ERR_INVALID_ARGUMENT, "unknown flags 0x%x", flags);
    DeviceGuard dg;
    r = dg.enter(device);
    if (r != POVS_OK) return r;
    DeviceCtx* c = nullptr;
    r = get_ctx(device, &c);
    if (r != POVS_OK) return r;
    return shuffle_on_device(data, n_rows, row_bytes, offsets, n_offsets, iterations, pblock, vblock, 0, *c,
                             static_cast<cudaStream_t>(stream), flags, nullptr, nullptr, 1, n_decks,
                             n_decks > 1 ? deck_stride : 0, seeds);
}

namespace {

int check_metric_args(const void* ids, int32_t id_bytes, int64_t n_episodes, int64_t deck)
{
    if (ids == nullptr) return fail(POVS_ERR_INVALID_ARGUMENT, "ids is NULL");
    if (id_bytes != 4 && id_bytes != 8) return fail(POVS_ERR_INVALID_ARGUMENT, "id_bytes must be 4 or 8, is %d", id_bytes);
    if (n_episodes < 1 || deck < 1)
        return fail(POVS_ERR_INVALID_ARGUMENT, "episodes (%lld) and deck size (%lld) must be positive",
                    static_cast<long long>(n_episodes), static_cast<long long>(deck));
    return POVS_OK;
}

int metric_grid(const DeviceCtx& c, int64_t total, int64_t min_blocks)
{
    const int64_t want = std::max<int64_t>(1, (total + 255) / 256);
    return static_cast<int>(std::max<int64_t>(min_blocks, std::min<int64_t>(want, int64_t{4} * c.sm_count)));
}

} // namespace

extern "C" int povs_travel_histogram_v1(const void* ids, int32_t id_bytes, int64_t n_episodes, int64_t deck,
                                        int64_t episode_stride, int64_t element_stride, int32_t kind, int64_t step,
                                        uint64_t* counts, int32_t device, void* stream)
{
    g_err[0] = '\0';
    int r = check_metric_args(ids, id_bytes, n_episodes, deck);
    if (r != POVS_OK) return r;
    if (counts == nullptr) return fail(POVS_ERR_INVALID_ARGUMENT, "counts is NULL");
    if (kind != 0 && kind != 1) return fail(POVS_ERR_INVALID_ARGUMENT, "kind must be 0 (positional) or 1 (pairs)");
    if (kind == 1 && step < 1) return fail(POVS_ERR_INVALID_ARGUMENT, "step (%lld) must be positive", static_cast<long long>(step));
    DeviceGuard dg;
    r = dg.enter(device);
    if (r != POVS_OK) return r;
    DeviceCtx* c = nullptr;
    r = get_ctx(device, &c);
    if (r != POVS_OK) return r;
    povs::MetricParams q{};
    q.ids = ids;
    q.id_bytes = id_bytes;
    q.kind = kind;
    q.n_episodes = n_episodes;
    q.deck = deck;
    q.episode_stride = episode_stride;
    q.element_stride = element_stride;
    q.step = step;
    q.counts = reinterpret_cast<unsigned long long*>(counts);
    q.smem_bins = deck <= povs::HIST_SMEM_MAX_BINS ? static_cast<int32_t>(deck) : 0;
    const int64_t total = n_episodes * deck;
    // Shared-memory bins are uint32: keep every CTA below 2^32 observations.
    const int grid = metric_grid(*c, total, total / (int64_t{1} << 31) + 1);
    void* args[] = {&q};
    cudaError_t e = cudaLaunchKernel(reinterpret_cast<const void*>(povs::povs_travel_histogram_kernel), dim3(grid),
                                     dim3(256), args, static_cast<size_t>(q.smem_bins) * sizeof(uint32_t),
                                     static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "cudaLaunchKernel(histogram)");
    return POVS_OK;
}

extern "C" int povs_ngram_keys_v1(const void* ids, int32_t id_bytes, int64_t n_episodes, int64_t deck,
                                  int64_t episode_stride, int64_t element_stride, int32_t n, int64_t step,
                                  const int64_t* positions, int64_t n_positions, int64_t* keys, int32_t device,
                                  void* stream)
{
    g_err[0] = '\0';
    int r = check_metric_args(ids, id_bytes, n_episodes, deck);
    if (r != POVS_OK) return r;
    if (keys == nullptr) return fail(POVS_ERR_INVALID_ARGUMENT, "keys is NULL");
    if (n < 2) return fail(POVS_ERR_INVALID_ARGUMENT, "n-gram degree (%d) must be at least 2", n);
    if (step < 1) return fail(POVS_ERR_INVALID_ARGUMENT, "step (%lld) must be positive", static_cast<long long>(step));
    if (positions != nullptr && n_positions < 1) return fail(POVS_ERR_INVALID_ARGUMENT, "n_positions must be positive");
    DeviceGuard dg;
    r = dg.enter(device);
    if (r != POVS_OK) return r;
    DeviceCtx* c = nullptr;
    r = get_ctx(device, &c);
    if (r != POVS_OK) return r;
    povs::MetricParams q{};
    q.ids = ids;
    q.id_bytes = id_bytes;
    q.kind = n;
    q.n_episodes = n_episodes;
    q.deck = deck;
    q.episode_stride = episode_stride;
    q.element_stride = element_stride;
    q.step = step;
    q.positions = positions;
    q.n_positions = positions != nullptr ? n_positions : 0;
    q.keys = keys;
    const int64_t total = n_episodes * (positions != nullptr ? n_positions : deck);
    const int grid = metric_grid(*c, total, 1);
    void* args[] = {&q};
    cudaError_t e = cudaLaunchKernel(reinterpret_cast<const void*>(povs::povs_ngram_keys_kernel), dim3(grid), dim3(256),
                                     args, 0, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "cudaLaunchKernel(ngram keys)");
    return POVS_OK;
}

extern "C" int povs_ngram_count_v1(const void* ids, int32_t id_bytes, int64_t n_episodes, int64_t deck,
                                   int64_t episode_stride, int64_t element_stride, int32_t n, int64_t step,
                                   const int64_t* positions, int64_t n_positions, uint64_t* table, int64_t slots,
                                   uint64_t* mult, int64_t mult_bins, uint64_t* overflow, int64_t overflow_cap,
                                   int32_t device, void* stream)
{
    g_err[0] = '\0';
    int r = check_metric_args(ids, id_bytes, n_episodes, deck);
    if (r != POVS_OK) return r;
    if (n < 2) return fail(POVS_ERR_INVALID_ARGUMENT, "n-gram degree (%d) must be at least 2", n);
    if (step < 1) return fail(POVS_ERR_INVALID_ARGUMENT, "step (%lld) must be positive", static_cast<long long>(step));
    if (positions != nullptr && n_positions < 1) return fail(POVS_ERR_INVALID_ARGUMENT, "n_positions must be positive");
    if (table == nullptr || mult == nullptr) return fail(POVS_ERR_INVALID_ARGUMENT, "table and mult are required");
    const int64_t total = n_episodes * (positions != nullptr ? n_positions : deck);
    if (!is_pow2(slots) || slots <= total)
        return fail(POVS_ERR_INVALID_ARGUMENT, "slots (%lld) must be a power of two above the %lld keys",
                    static_cast<long long>(slots), static_cast<long long>(total));
    if (mult_bins < 2) return fail(POVS_ERR_INVALID_ARGUMENT, "mult_bins (%lld) must be at least 2", static_cast<long long>(mult_bins));
    if (overflow_cap < 0 || (overflow_cap > 0 && overflow == nullptr))
        return fail(POVS_ERR_INVALID_ARGUMENT, "overflow must hold overflow_cap entries");
    DeviceGuard dg;
    r = dg.enter(device);
    if (r != POVS_OK) return r;
    DeviceCtx* c = nullptr;
    r = get_ctx(device, &c);
    if (r != POVS_OK) return r;
    povs::MetricParams q{};
    q.ids = ids;
    q.id_bytes = id_bytes;
    q.kind = n;
    q.n_episodes = n_episodes;
    q.deck = deck;
    q.episode_stride = episode_stride;
    q.element_stride = element_stride;
    q.step = step;
    q.positions = positions;
    q.n_positions = positions != nullptr ? n_positions : 0;
    povs::NgramTable t{};
    t.keys = reinterpret_cast<unsigned long long*>(table);
    t.counts = reinterpret_cast<unsigned long long*>(table) + slots;
    t.slots = slots;
    t.mult = reinterpret_cast<unsigned long long*>(mult);
    t.mult_bins = mult_bins;
    t.overflow = reinterpret_cast<unsigned long long*>(overflow);
    t.overflow_cap = overflow_cap;
    t.status = c->status;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int grid_t = metric_grid(*c, std::max<int64_t>(slots + 1, mult_bins), 1);
    const int grid_k = metric_grid(*c, total, 1);
    povs::povs_ngram_table_clear_kernel<<<grid_t, 256, 0, s>>>(t);
    povs::povs_ngram_count_kernel<<<grid_k, 256, 0, s>>>(q, t);
    povs::povs_ngram_tally_kernel<<<grid_t, 256, 0, s>>>(t);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "n-gram count kernels");
    return POVS_OK;
}

extern "C" int povs_numpy_path_perm_v1(uint32_t seed, int32_t n, int32_t* out)
{
    g_err[0] = '\0';
    if (n < 0 || (n > 0 && out == nullptr)) return fail(POVS_ERR_INVALID_ARGUMENT, "n must be >= 0 and out given");
    povs::numpy_legacy_shuffle(seed, n, out);
    return POVS_OK;
}

extern "C" int povs_set_peer_wait_limit_v1(uint64_t limit_ns)
{
    g_err[0] = '\0';
    g_peer_wait_ns.store(limit_ns == 0 ? povs::PEER_WAIT_LIMIT_NS : static_cast<unsigned long long>(limit_ns));
    return POVS_OK;
}

// ------------------------------------------------------------------------------------------
// Decks that stay in host memory (mapped, page-locked).
// ------------------------------------------------------------------------------------------

extern "C" int povs_shuffle_mapped_v1(void* host_data, int64_t n_rows, int64_t row_bytes, const int64_t* offsets,
                                      int32_t n_offsets, int32_t iterations, int32_t pblock, int32_t vblock,
                                      uint64_t seed, int32_t device, void* stream, uint32_t flags)
{
    g_err[0] = '\0';
    int r = check_common(host_data, n_rows, row_bytes, pblock, vblock, iterations);
    if (r != POVS_OK) return r;
    r = check_offsets(offsets, n_offsets, n_rows);
    if (r != POVS_OK) return r;
    DeviceGuard dg;
    r = dg.enter(device);
    if (r != POVS_OK) return r;
    DeviceCtx* c = nullptr;
    r = get_ctx(device, &c);
    if (r != POVS_OK) return r;
    cudaStream_t s = static_cast<cudaStream_t>(stream);

    // Page-lock and map the deck for the call unless the caller already did (pinned memory).
    cudaPointerAttributes attr{};
    POVS_CUDA_TRY(cudaPointerGetAttributes(&attr, host_data));
    void* registered = nullptr;
    if (attr.type == cudaMemoryTypeUnregistered) {
        const long sys_page = sysconf(_SC_PAGESIZE);
        const uintptr_t page = sys_page > 0 ? static_cast<uintptr_t>(sys_page) : 4096u;
        const uintptr_t begin = reinterpret_cast<uintptr_t>(host_data) & ~(page - 1);
        const uintptr_t end = (reinterpret_cast<uintptr_t>(host_data) + static_cast<uintptr_t>(n_rows * row_bytes) +
                               page - 1) & ~(page - 1);
        registered = reinterpret_cast<void*>(begin);
        POVS_CUDA_TRY(cudaHostRegister(registered, end - begin, cudaHostRegisterMapped | cudaHostRegisterPortable));
        cudaError_t q = cudaPointerGetAttributes(&attr, host_data);
        if (q != cudaSuccess) {
            cudaHostUnregister(registered);
            return cuda_fail(q, "cudaPointerGetAttributes");
        }
    } else if (attr.type != cudaMemoryTypeHost) {
        return fail(POVS_ERR_INVALID_ARGUMENT, "host_data is not host memory (use povs_shuffle_v1 for device decks)");
    }
    // The device-side address of this very byte (interior pointers into a pinned block included).
    void* mapped = attr.devicePointer;
    cudaError_t e = mapped != nullptr ? cudaSuccess : cudaErrorInvalidValue;
    if (e == cudaSuccess) {
        // Plain vector loads and stores over the interconnect; TMA copies are not used on host memory.
        r = shuffle_on_device(mapped, n_rows, row_bytes, offsets, n_offsets, iterations, pblock, vblock, seed, *c, s,
                              flags & ~uint32_t{POVS_FLAG_SYNC}, nullptr, nullptr, 1, 1, 0, nullptr, true, false);
        if (r == POVS_OK) {
            e = cudaStreamSynchronize(s);
            if (e != cudaSuccess) r = cuda_fail(e, "cudaStreamSynchronize");
        }
    } else {
        r = fail(POVS_ERR_INVALID_ARGUMENT, "host_data is page-locked but not mapped into the device's address space");
    }
    if (registered != nullptr) {
        if (r != POVS_OK) cudaStreamSynchronize(s);  // the deck must not be unmapped under a running kernel
        cudaError_t u = cudaHostUnregister(registered);
        if (r == POVS_OK && u != cudaSuccess) r = cuda_fail(u, "cudaHostUnregister");
    }
    if (r != POVS_OK) return r;
    if (flags & POVS_FLAG_SYNC) {
        int32_t st = 0;
        r = read_status(*c, &st);
        if (r != POVS_OK) return r;
        if (st != 0) return fail(POVS_ERR_DEVICE_STATUS, "device status 0x%x after shuffle", st);
    }
    return POVS_OK;
}
