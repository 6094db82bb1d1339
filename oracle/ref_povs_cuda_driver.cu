// ORACLE - test infrastructure only (not part of the product).
//
// Driver that compiles the reference's own CUDA path, src/povs/__cuda/lib/povs.cu, where it lies in
// the reference checkout (recipe: oracle/build.py), into oracle/_ref/libref_povs_cuda.so, so that the
// GPU parity tests can run the reference kernel and its host loop next to this library's kernels.
//
// Compiled with -DPOVS_H: the reference's povs.h only declares the host template and pulls in ATen
// for c10::Half; the template is defined in povs.cu itself, and the 2-byte rows here use uint16_t,
// which the reference's copies treat exactly like c10::Half (both are 16-bit values moved as
// cute::uint_bit_t words; the kernel never does arithmetic on them).  The reference's generated
// instantiation file (povs_cuda_template_instances.gen.inc, written by its setup.py:134-163) is
// replaced by oracle/ref_gen/povs_cuda_template_instances.gen.inc, which instantiates nothing: the
// shapes below are instantiated by this file instead.
//
// Safe shapes only.  The reference's Stage 1 copy (povs.cu:80-91, 225-278) tiles a pblock's
// (InstanceSize, PBlockSize) elements with a (BlockSize, copy width) tile.  When InstanceSize is not
// a multiple of BlockSize the tile's instance coordinate runs past the row, and the predicates
// (povs.cu:239-259) only test the row index, so threads read past the pblock in global memory and
// write past the vblock's shared-memory array.  Every shape in the table keeps InstanceSize a
// multiple of BlockSize, and ref_povs_layout_check() re-derives the tile partition on the host and
// verifies that every copied coordinate lies inside the pblock and that each element is copied once;
// the run entry points refuse a shape that fails it.
#include <cstdint>
#include <cstdio>
#include <vector>

#include "povs.cu"

namespace {

// One instantiated shape: (VBlockSize, PBlockSize, InstanceSize, element type, GPU thread-block size).
template <int V, int P, int Inst, typename T, int BS>
struct RefShape {
    static constexpr int kRowBytes = Inst * static_cast<int>(sizeof(T));

    // The reference's full host loop (povs.cu:356-467): mt19937 randomness, per-call device
    // allocations, blocking copies and one kernel per iteration on the legacy default stream.
    static void run(void* data, int64_t n_rows, const int64_t* offsets, int64_t n_offsets, int iterations, int seed,
                    int device)
    {
        povs_cuda<V, P, Inst, T>(static_cast<T*>(data), static_cast<long>(n_rows),
                                 reinterpret_cast<const long*>(offsets), static_cast<long>(n_offsets), iterations,
                                 seed, static_cast<int8_t>(device), BS);
    }

    // The reference kernel alone (povs.cu:116-349) with injected assignments, seeds and offset.
    static int kernel(void* data, int64_t n_rows, const int64_t* assign, const int32_t* seeds, int64_t offset,
                      cudaStream_t stream)
    {
        const long n_p = (static_cast<long>(n_rows) + P - 1) / P;
        const long n_v = (n_p + V - 1) / V;
        povs_kernel<T, P, V, Inst, BS><<<static_cast<unsigned>(n_v), BS, 0, stream>>>(
            static_cast<T*>(data), reinterpret_cast<const long*>(assign), seeds, static_cast<long>(offset),
            static_cast<long>(n_rows));
        return cudaGetLastError() == cudaSuccess ? 0 : -3;
    }

    // Host re-derivation of the Stage 1 tile partition (povs.cu:68-91): returns 0 when every thread's
    // coordinates lie inside (InstanceSize, PBlockSize) and cover each element exactly once.
    static int layout_check()
    {
        using namespace cute;
        constexpr int InstanceBits = Inst * static_cast<int>(sizeof(T)) * 8;
        constexpr int BitWidth = InstanceBits % 128 == 0 ? 128 : InstanceBits % 64 == 0 ? 64
                                                             : InstanceBits % 32 == 0   ? 32
                                                                                        : 16;
        constexpr int CW = BitWidth / 8 / static_cast<int>(sizeof(T));
        auto atom = Copy_Atom<UniversalCopy<uint_bit_t<BitWidth>>, T>{};
        auto thr_layout = make_layout(make_shape(Int<BS / CW>{}, Int<CW>{}));
        auto val_layout = make_layout(make_shape(Int<CW>{}));
        auto tiled = make_tiled_copy(atom, thr_layout, val_layout);
        auto ident = make_identity_tensor(make_shape(Int<Inst>{}, Int<P>{}));
        std::vector<int> seen(static_cast<size_t>(Inst) * P, 0);
        for (int t = 0; t < BS; ++t) {
            auto part = tiled.get_slice(t).partition_S(ident);
            for (int k = 0; k < size(part); ++k) {
                auto c = part(k);
                const int i = get<0>(c), j = get<1>(c);
                if (i < 0 || i >= Inst || j < 0 || j >= P) return 1;
                seen[static_cast<size_t>(i) + static_cast<size_t>(Inst) * j] += 1;
            }
        }
        for (int s : seen)
            if (s != 1) return 2;
        // Stage 2/3 partition of the (PBlockSize, VBlockSize) slots over the threads (povs.cu:151,177).
        if (BS > P * V || (P * V) % BS != 0 || P % (BS / V) != 0) return 3;
        // The kernel's static shared memory must fit the 48 KB static limit.
        if (static_cast<long>(V) * P * kRowBytes + 4l * V * P > 48 * 1024) return 4;
        return 0;
    }
};

using Shape0 = RefShape<2, 16, 32, uint16_t, 32>;   // 64 B rows (the bias deck's rows)
using Shape1 = RefShape<4, 16, 32, uint16_t, 32>;   // 64 B rows, V = 4
using Shape2 = RefShape<2, 64, 128, uint16_t, 64>;  // 256 B rows, the 1,048,576 x 128 fp16 deck
using Shape3 = RefShape<4, 32, 128, uint16_t, 64>;  // 256 B rows, the 134,217,728 x 128 bf16 deck
using Shape4 = RefShape<4, 64, 32, float, 32>;      // 128 B rows, the fp32 x 32 sharded deck's rows
using Shape5 = RefShape<8, 16, 64, uint16_t, 32>;   // 128 B rows, V = 8
using Shape6 = RefShape<2, 32, 64, double, 64>;     // 512 B rows
using Shape7 = RefShape<16, 16, 32, int32_t, 32>;   // 128 B rows, V = 16

struct Entry {
    int V, P, inst, elem_bytes, block;
    void (*run)(void*, int64_t, const int64_t*, int64_t, int, int, int);
    int (*kernel)(void*, int64_t, const int64_t*, const int32_t*, int64_t, cudaStream_t);
    int (*check)();
};

template <int V, int P, int Inst, typename T, int BS>
constexpr Entry entry(RefShape<V, P, Inst, T, BS>)
{
    using S = RefShape<V, P, Inst, T, BS>;
    return Entry{V, P, Inst, static_cast<int>(sizeof(T)), BS, &S::run, &S::kernel, &S::layout_check};
}

const Entry kShapes[] = {entry(Shape0{}), entry(Shape1{}), entry(Shape2{}), entry(Shape3{}),
                         entry(Shape4{}), entry(Shape5{}), entry(Shape6{}), entry(Shape7{})};
constexpr int kNumShapes = static_cast<int>(sizeof(kShapes) / sizeof(kShapes[0]));

bool valid(int shape) { return shape >= 0 && shape < kNumShapes; }

} // namespace

extern "C" {

// Number of shapes; writes min(n, count) rows of {V, P, InstanceSize, element bytes, block size}.
int ref_povs_shapes(int32_t* out, int32_t n)
{
    for (int s = 0; s < kNumShapes && s < n; ++s) {
        const Entry& e = kShapes[s];
        out[5 * s + 0] = e.V;
        out[5 * s + 1] = e.P;
        out[5 * s + 2] = e.inst;
        out[5 * s + 3] = e.elem_bytes;
        out[5 * s + 4] = e.block;
    }
    return kNumShapes;
}

// Host-only check of a shape's copy partition (no GPU needed); 0 = in bounds.
int ref_povs_layout_check(int32_t shape) { return valid(shape) ? kShapes[shape].check() : -1; }

// Host-only check of the options the reference picks on a B200 for a float32 deck of 32-byte rows
// (V = 2, P = 64, block size 64, from its chooser, src/povs/torch.py:154-241): InstanceSize 8 is
// not a multiple of the block size, so the check reports coordinates outside the pblock (nonzero).
// Only the check is instantiated; this shape has no run entry.
int ref_povs_layout_check_small_rows() { return RefShape<2, 64, 8, float, 64>::layout_check(); }

// The reference's CUDA path for one shape: povs_cuda<V,P,Inst,T>(data, ...) with the given seed.
// Synchronous with respect to the host only through the reference's own blocking copies and frees.
int ref_povs_cuda(int32_t shape, void* data, int64_t n_rows, const int64_t* offsets, int64_t n_offsets,
                  int32_t iterations, int32_t seed, int32_t device)
{
    if (!valid(shape) || kShapes[shape].check() != 0) return -1;
    if (data == nullptr || n_rows < 1 || offsets == nullptr || n_offsets < 1 || iterations < 0) return -1;
    for (int64_t i = 0; i < n_offsets; ++i)
        if (offsets[i] < 0 || offsets[i] >= n_rows) return -1;
    kShapes[shape].run(data, n_rows, offsets, n_offsets, iterations, seed, device);
    return cudaDeviceSynchronize() == cudaSuccess ? 0 : -3;
}

// The reference kernel alone, one iteration: assign (device, int64 [n_v][V], -1 padding) and seeds
// (device, int32 [n_v]) as the reference's host loop would upload them (povs.cu:420-430).
int ref_povs_kernel(int32_t shape, void* data, int64_t n_rows, const int64_t* assign, const int32_t* seeds,
                    int64_t offset, void* stream)
{
    if (!valid(shape) || kShapes[shape].check() != 0) return -1;
    if (data == nullptr || assign == nullptr || seeds == nullptr || n_rows < 1 || offset < 0 || offset >= n_rows)
        return -1;
    return kShapes[shape].kernel(data, n_rows, assign, seeds, offset, static_cast<cudaStream_t>(stream));
}

} // extern "C"
