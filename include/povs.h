/*
 * C ABI of the B200-native POV shuffle (libpovs_sm100.so).
 *
 * Every entry point takes plain pointers and sizes, returns 0 on success or a
 * negative POVS_ERR_* code, never terminates the process, and records a
 * message retrievable with povs_last_error_string() (per calling thread).
 * Device work is enqueued on the caller's stream (a cudaStream_t passed as
 * void*; NULL means the legacy default stream) and is asynchronous unless
 * stated otherwise.  The caller owns every data buffer; the library only keeps
 * a small per-device context (a status word and cached CUDA graphs), created
 * on first use and freed by povs_release_v1().
 *
 * Rows ("instances") are opaque byte vectors of row_bytes bytes; the deck is
 * n_rows rows, contiguous.  Shuffling is in place along axis 0.
 */
#ifndef POVS_H
#define POVS_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Return codes. */
#define POVS_OK 0
#define POVS_ERR_INVALID_ARGUMENT (-1) /* a size, option or pointer is out of range */
#define POVS_ERR_UNSUPPORTED (-2)      /* valid for the algorithm but outside this library's limits */
#define POVS_ERR_CUDA (-3)             /* a CUDA runtime call failed */
#define POVS_ERR_DEVICE_STATUS (-4)    /* a kernel reported a failure through the device status word */

/* Device status bits reported by povs_device_status_v1(). */
#define POVS_DEV_WAIT_TIMEOUT 1 /* an async-copy barrier wait gave up after its time limit */
#define POVS_DEV_BAD_INJECTED 2 /* an injected permutation entry was out of range and was ignored */

/* Flags of povs_shuffle_v1(). */
/* Launch the iterations one by one (by default decks under 32 MiB replay a cached CUDA graph and
 * larger decks are launched one by one). */
#define POVS_FLAG_NO_GRAPH 1u
#define POVS_FLAG_SYNC 2u     /* synchronize the stream and check the device status before returning */
/* Draw the randomness with the distribution of the reference's CUDA path (per-vblock seeds 1..999,
 * xorshift32 forward Fisher-Yates, padding in the last vblock; src/povs/__cuda/lib/povs.cu:396-430,
 * 294-316) instead of uniform per-vblock permutations.  For statistical comparisons with it. */
#define POVS_FLAG_REFERENCE_RNG 4u
/* Order the iteration kernels with ordinary stream order instead of programmatic dependent
 * launches (by default each iteration kernel's CTAs start their set-up while the kernel before it
 * on the stream drains - the previous iteration, or for decks of 32 MiB and more the previous
 * call's last iteration - and wait for it to complete before touching the deck). */
#define POVS_FLAG_NO_PDL 8u
/* Draw the randomness with the distribution of the reference's NumPy path (padding ids anywhere,
 * members in slot order, per-vblock seeds 1..999 and numpy.random.RandomState(seed).shuffle of the
 * vblock's rows; src/povs/numpy.py:43-61,125-136).  The permutations come from tables built on the
 * host once per (P, V, n_rows % P) and device (at most 128 MiB; a larger geometry is rejected with
 * POVS_ERR_UNSUPPORTED), freed by povs_release_v1.  Excludes POVS_FLAG_REFERENCE_RNG. */
#define POVS_FLAG_REFERENCE_NUMPY 16u

/* Limits of this library. */
#define POVS_MAX_OFFSETS 256 /* offsets are passed to the device inline in the launch parameters */
#define POVS_MAX_VBLOCK 32   /* one warp lane per member pblock */
#define POVS_MAX_VP 1024     /* V * P rows per vblock: one warp sorts the permutation in registers */

/*
 * Shuffle a deck in place: `iterations` POV iterations, all randomness drawn on
 * the device from `seed` (Philox4x32-10 counters: offset choice, a keyed
 * bijection of pblocks onto vblock slots, per-vblock permutations).
 *
 * Replaces the reference's native entry `torch_binding(X, O, iterations,
 * pblock, vblock, block_size, seed)` (src/povs/_cuda.pyi:9-17,
 * src/povs/__cuda/binds/torch.cpp:19-60) and the host loop it dispatches to
 * (src/povs/__cuda/lib/povs.cu:356-467).  Differences: the device pointer and
 * the row size replace the typed tensor (any dtype); offsets are a host array;
 * the GPU thread-block size is not needed; the stream is explicit; errors are
 * return codes instead of exit().
 *
 *   data        device pointer to n_rows * row_bytes bytes
 *   offsets     host array of n_offsets (1..POVS_MAX_OFFSETS) row offsets, each in [0, n_rows)
 *   pblock      P, a power of two >= 1;  vblock: V, a power of two in [2, POVS_MAX_VBLOCK]
 *   device      CUDA ordinal the data lives on
 *   stream      cudaStream_t of that device, or NULL
 */
int povs_shuffle_v1(void* data, int64_t n_rows, int64_t row_bytes, const int64_t* offsets, int32_t n_offsets,
                    int32_t iterations, int32_t pblock, int32_t vblock, uint64_t seed, int32_t device, void* stream,
                    uint32_t flags);

/*
 * Same as povs_shuffle_v1 for a deck in HOST memory: the rows are copied to a
 * device buffer supplied by the caller (`device_buffer`, at least n_rows *
 * row_bytes bytes on `device`), shuffled there and copied back, all on
 * `stream`, and the call returns after the stream has synchronized.  Pinned
 * host memory gives full PCIe / C2C bandwidth; pageable memory works.
 *
 * Serves the reference's CPU route (`povs.shuffle` on a numpy array or a CPU
 * tensor, src/povs/__init__.py:36-42 -> src/povs/numpy.py:18-61) on the GPU.
 */
int povs_shuffle_host_v1(void* host_data, void* device_buffer, int64_t n_rows, int64_t row_bytes,
                         const int64_t* offsets, int32_t n_offsets, int32_t iterations, int32_t pblock,
                         int32_t vblock, uint64_t seed, int32_t device, void* stream, uint32_t flags);

/*
 * Same as povs_shuffle_v1 for a deck that STAYS in host memory, for decks larger than the
 * device's memory: the kernels read and write the rows in place over PCIe / C2C through mapped
 * page-locked memory (plain vector loads and stores, no TMA).  Memory from cudaHostAlloc /
 * cudaMallocHost or already registered is used as is; any other host range is page-locked and
 * mapped for the duration of the call (cudaHostRegister of the enclosing pages) and released
 * before returning.  The call returns after the stream has synchronized.  Throughput is bound by
 * the interconnect (each iteration moves the deck across it twice).
 * Serves the reference's roadmap item of decks larger than memory (CONTRIBUTING.md:16) on the
 * reference's CPU route (src/povs/numpy.py:18-61).
 */
int povs_shuffle_mapped_v1(void* host_data, int64_t n_rows, int64_t row_bytes, const int64_t* offsets,
                           int32_t n_offsets, int32_t iterations, int32_t pblock, int32_t vblock, uint64_t seed,
                           int32_t device, void* stream, uint32_t flags);

/*
 * Shuffle n_decks host decks of the same shape through n_buffers device buffers (>= 2 for
 * overlap; each at least n_rows * row_bytes bytes on `device`): deck d is copied into buffer
 * d % n_buffers, shuffled with seeds[d], and copied back, on internal streams ordered by events so
 * that deck d's copy back overlaps deck d+1's copy in and iterations (the PCIe directions and the
 * SMs work at the same time).  Work queued on `stream` before the call is ordered first; the call
 * returns when every deck is back in host memory.  A host deck may appear more than once in the
 * list (it is then shuffled again, after its previous copy back).  Use pinned host memory for
 * overlap.  Batched form of povs_shuffle_host_v1 (same reference route).
 */
int povs_shuffle_host_batch_v1(void* const* host_decks, int32_t n_decks, void* const* device_buffers, int32_t n_buffers,
                               int64_t n_rows, int64_t row_bytes, const int64_t* offsets, int32_t n_offsets,
                               int32_t iterations, int32_t pblock, int32_t vblock, const uint64_t* seeds,
                               int32_t device, void* stream, uint32_t flags);

/*
 * Apply externally supplied randomness (test hook for bit-exact parity with the
 * reference's CPU and CUDA paths).  For each iteration t:
 *   offsets_per_iter[t]        (host)   the iteration's row offset, in [0, n_rows)
 *   assign + t*n_v*V           (device) int64 [n_v][V] member pblock ids; values < 0 or
 *                                       >= ceil(n_rows/P) are padding
 *   perms  + t*n_v*V*P         (device) int32 [n_v][V*P]; destination slot f of a vblock
 *                                       receives source slot perms[f] (f < valid rows)
 * sort_members = 1 orders each vblock's members ascending with padding last, as the
 * reference kernel does (src/povs/__cuda/lib/povs.cu:203-221); 0 keeps the given order
 * (the NumPy path, src/povs/numpy.py:120-136), except that padding goes last and a
 * truncated last pblock is placed after the full ones.
 * n_v = ceil(ceil(n_rows/P)/V).  Replaces no single reference function: it is the
 * reference kernel's body (povs.cu:116-349) with the host RNG (povs.cu:415-431) cut out.
 */
int povs_apply_v1(void* data, int64_t n_rows, int64_t row_bytes, int32_t pblock, int32_t vblock,
                  int32_t iterations, const int64_t* offsets_per_iter, const int64_t* assign, const int32_t* perms,
                  int32_t sort_members, int32_t device, void* stream);

/*
 * Shuffle a deck stored as up to POVS_MAX_SHARDS shards (one process, one device): rows
 * [sum(shard_rows[0..i-1]), +shard_rows[i]) live at shard_ptrs[i].  The result equals
 * povs_shuffle_v1 on the concatenated deck with the same seed.  Every shard must be addressable
 * from `device` (allocations on it, or peer memory with peer access enabled) and hold at least
 * `pblock` rows; the caller orders any writes to the shards before the call.  scratch_ptrs is NULL
 * (in place: each vblock is read into shared memory and written back) or one buffer per shard of
 * the same size (double-buffered "push" order: each pblock's rows are read once from the buffer
 * holding them and stored straight into their destination slots in the other buffer; an odd
 * number of iterations ends with a copy back).  Both orders give the same result.
 * No reference counterpart: the reference shuffles one contiguous tensor (src/povs/torch.py:20-50).
 */
int povs_shuffle_shards_v1(void* const* shard_ptrs, void* const* scratch_ptrs, const int64_t* shard_rows,
                           int32_t n_shards, int64_t row_bytes, const int64_t* offsets, int32_t n_offsets,
                           int32_t iterations, int32_t pblock, int32_t vblock, uint64_t seed, int32_t device,
                           void* stream, uint32_t flags);

/*
 * Sharded mode, one process per GPU, over the deck whose shards are shard_ptrs (this rank's own
 * shard and the peers' shards as mapped into this process with povs_ipc_import_v1).  With
 * scratch_ptrs NULL, rank `rank` reads the vblocks rank, rank + n_shards, ... from local or peer
 * memory (bulk copies over NVLink, no multicast) and writes them back with peer stores.  With one
 * scratch buffer per shard (same sizes, mapped the same way), rank `rank` moves the pblocks stored
 * in its own shard, reading them locally and storing every row straight into its destination slot
 * in the other buffer, so a row crosses NVLink at most once per iteration (half the traffic).
 * A device barrier over the ranks' flag arrays (peer_flags[r]: n_shards uint32 words of rank r,
 * zero-initialised, mapped here) runs before the first iteration and after each one, with epochs
 * epoch_base + 1 .. epoch_base + iterations + 1; every rank must call with the same arguments
 * (except rank, device, stream) and the caller advances epoch_base by iterations + 1 per call.
 * Same result as povs_shuffle_v1 on the concatenated deck with the same seed.
 * No reference counterpart (the reference has no multi-GPU code).
 */
#define POVS_MAX_SHARDS 8
#define POVS_DEV_PEER_TIMEOUT 4 /* device status bit: a peer GPU did not reach the barrier in time */
int povs_shuffle_sharded_v1(void* const* shard_ptrs, void* const* scratch_ptrs, const int64_t* shard_rows,
                            int32_t n_shards, int32_t rank, int64_t row_bytes, const int64_t* offsets,
                            int32_t n_offsets, int32_t iterations, int32_t pblock, int32_t vblock, uint64_t seed,
                            void* const* peer_flags, uint32_t epoch_base, int32_t device, void* stream,
                            uint32_t flags);

/*
 * Time limit of the cross-GPU barrier between iterations of povs_shuffle_sharded_v1 (process-wide;
 * 0 restores the default of 20 s).  A barrier that gives up sets POVS_DEV_PEER_TIMEOUT in the
 * device status word and returns, so the context stays usable.  No reference counterpart.
 */
int povs_set_peer_wait_limit_v1(uint64_t limit_ns);

/*
 * Let kernels on `device` read and write `peer`'s memory (cudaDeviceEnablePeerAccess; enabling it
 * twice is not an error).  Needed before povs_shuffle_shards_v1 gets shards on other GPUs of the
 * node.  No reference counterpart (the reference is single-GPU).
 */
int povs_enable_peer_access_v1(int32_t device, int32_t peer);

/*
 * Host only (no GPU needed): numpy.random.RandomState(seed).shuffle(arange(n)) into out[0 .. n-1],
 * the permutation the reference's NumPy path applies to a vblock of n rows under per-vblock seed
 * `seed` (src/povs/numpy.py:125-136).  The tables of the POVS_FLAG_REFERENCE_NUMPY mode are built
 * from it.
 */
int povs_numpy_path_perm_v1(uint32_t seed, int32_t n, int32_t* out);

/* CUDA IPC of device memory between the processes of a sharded deck (64-byte handles). */
int povs_ipc_export_v1(const void* ptr, int32_t device, void* handle_out, int64_t* offset_out);
int povs_ipc_import_v1(const void* handle, int64_t offset, int32_t device, void** ptr_out, void** base_out);
int povs_ipc_close_v1(void* base, int32_t device);

/* Read and clear the device status word of `device` (synchronizes the device's context). Writes bits to *status. */
int povs_device_status_v1(int32_t device, int32_t* status);

/* Free the per-device context (status word, cached graphs) of every device touched. */
int povs_release_v1(void);

/* Message describing the last error returned on the calling thread ("" if none). */
const char* povs_last_error_string(void);

/* Library version: major * 10000 + minor * 100 + patch. */
int32_t povs_version(void);

/*
 * Advanced: process-wide launch tuning (no reference counterpart; the reference
 * fixes these at compile time through template parameters, povs.cu:116,433-436).
 *   stage_cap   max bytes of one shared-memory data stage; vblocks whose V*P rows exceed it
 *               are processed in column slabs (default 32768)
 *   n_stages    max data stages in a CTA's ring, 2..16 (default 8; fewer when shared memory is short)
 *   movers      warps per CTA that copy rows (default 4)
 *   permuters   warps per CTA that compute members and permutations (default 4); movers + permuters <= 16
 *   force_plain 1 = plain vector loads instead of TMA bulk copies (whole rows of 4-byte multiples
 *               are then copied asynchronously); 2 = plain loads issued synchronously
 *   copy_bytes  target bytes of one bulk copy when whole rows are staged (default 8192)
 */
int povs_set_tuning_v1(int32_t stage_cap, int32_t n_stages, int32_t movers, int32_t permuters, int32_t force_plain,
                       int32_t copy_bytes);

/*
 * Advanced: largest packed unit, in bytes (process-wide; no reference counterpart).  Vblocks of
 * device-randomness in-place shuffles whose V*P rows are small travel several per unit (up to 32 / V
 * vblocks, 1024 rows and this many bytes per unit), so that per-unit costs are paid once for all of
 * them; the result is the same.  0 turns packing off; the default is 16384.
 */
int povs_set_pack_bytes_v1(int32_t pack_bytes);

/*
 * Advanced: report the launch plan povs_shuffle_v1 would use, as int64 values
 * {grid, block, dynamic smem, sort elements per lane, bulk (0/1), slab bytes, slabs,
 *  stages per CTA, stage bytes, vector bytes, vblocks, SM count, rows per bulk copy,
 *  permutation slots, mover warps, permuter warps, vblocks per unit, rows per unit,
 *  wide-row store kernel (0/1), chunked store kernel (0/1)}; returns how many were written.
 */
int povs_describe_plan_v1(void* data, int64_t n_rows, int64_t row_bytes, int32_t pblock, int32_t vblock,
                          int32_t device, int64_t* out, int32_t n_out);

/*
 * Advanced: the same plan computed on the host for given device resources, without a GPU: SM
 * count, the opt-in maximum of dynamic shared memory per block, shared memory per SM and threads
 * per SM (B200: 148, 232448, 233472, 2048).  data_address only sets the alignment the plan sees
 * (nonzero).  Same output as povs_describe_plan_v1, under the process-wide tuning.  For checking
 * plans in tests and tools; replaces nothing in the reference.
 */
int povs_plan_for_resources_v1(uint64_t data_address, int64_t n_rows, int64_t row_bytes, int32_t pblock,
                               int32_t vblock, int32_t sm_count, int32_t smem_optin, int32_t smem_per_sm,
                               int32_t max_threads_per_sm, int64_t* out, int32_t n_out);

/*
 * Allocation-free variant of povs_apply_v1 (no counterpart in the reference).
 *
 * For callers that cannot allocate GPU memory while they run - for example a process whose
 * memory pool has already reserved the GPU's free memory, or a service that forbids allocation
 * after start-up to keep its footprint fixed.  The injected randomness is passed in HOST memory
 * (same layouts as povs_apply_v1: assign_host int64 [iterations][n_v][V], perms_host int32
 * [iterations][n_v][V*P]) and staged, one iteration at a time, in a scratch array that is part
 * of the library image: POVS_STATIC_SCRATCH_BYTES of device memory that every GPU which loads
 * the library holds until the process exits.  The call allocates nothing (no cudaMalloc, no
 * CUDA graph); it launches the same kernels as povs_apply_v1 and gives the same bytes.
 *
 * Limit: one iteration needs 256 + round_up(8 * n_v * V, 256) + 4 * n_v * V * P bytes; larger
 * decks are rejected with POVS_ERR_UNSUPPORTED (use povs_apply_v1 then).
 * The first call on a device looks up the scratch array's device address (with that device
 * current) and reads its limits; make that first call before any stream capture.  With lazy
 * module loading (the CUDA 12 default) the array and the kernels come into being on the library's
 * first use on a device, so make one povs call there (iterations = 0 is enough: the set-up still
 * runs) before a memory pool reserves the GPU's free memory or the process stops allocating.
 * Every call shares the one array, which keeps the last call's contents (the status word in it is
 * cleared at the start of each call): calls that overlap on the GPU race.  Device failures (a
 * wait that timed out, an out-of-range injected permutation entry) are reported only with
 * POVS_FLAG_SYNC, the one flag accepted: the call then synchronizes `stream` and returns
 * POVS_ERR_DEVICE_STATUS; povs_device_status_v1 does not see this entry's status word.  Without it
 * the call returns after enqueueing, and the host arrays must stay unchanged until the stream has
 * run the work (pinned host memory is read asynchronously).
 */
#define POVS_STATIC_SCRATCH_BYTES (8u * 1024u * 1024u)
int povs_apply_static_v1(void* data, int64_t n_rows, int64_t row_bytes, int32_t pblock, int32_t vblock,
                         int32_t iterations, const int64_t* offsets_per_iter, const int64_t* assign_host,
                         const int32_t* perms_host, int32_t sort_members, int32_t device, void* stream,
                         uint32_t flags);

/*
 * Batched decks: n_decks independent decks of the same geometry, deck d at
 * data + d * deck_stride (bytes; deck_stride >= n_rows * row_bytes), all shuffled by one launch
 * per iteration.  Deck d ends exactly as povs_shuffle_v1 on it alone with seed seeds[d] would
 * leave it.  `seeds` is a DEVICE array of n_decks seeds that must stay unchanged until the stream
 * has run the work.  Flags as povs_shuffle_v1.
 * Replaces the reference's loop of one povs.shuffle call per episode in its bias exercises
 * (src/povs/eval/exercises.py:387-389, 247-249).
 */
int povs_shuffle_batch_v1(void* data, int64_t n_decks, int64_t deck_stride, int64_t n_rows, int64_t row_bytes,
                          const int64_t* offsets, int32_t n_offsets, int32_t iterations, int32_t pblock,
                          int32_t vblock, const uint64_t* seeds, int32_t device, void* stream, uint32_t flags);

/*
 * Travel-distance histogram over shuffled episodes (all pointers are device memory; asynchronous
 * on `stream`).  ids: int32 (id_bytes 4) or int64 (id_bytes 8); element i of episode e at
 * ids[e * episode_stride + i * element_stride], each episode a permutation of 0 .. deck-1.
 * kind 0: counts[(i - v) mod deck] += 1 for every element (positional travel distance,
 * get_tvd, src/povs/eval/metrics.py:38-87).  kind 1: counts[((v[(i + step) mod deck] - v[i]) - step)
 * mod deck] += 1 for every position (2-gram relative travel distance with step = skip + 1,
 * get_ngram_tvd with n = 2, metrics.py:147-172).  counts: deck uint64 bins, ADDED to.
 */
int povs_travel_histogram_v1(const void* ids, int32_t id_bytes, int64_t n_episodes, int64_t deck,
                             int64_t episode_stride, int64_t element_stride, int32_t kind, int64_t step,
                             uint64_t* counts, int32_t device, void* stream);

/*
 * n-gram keys (n >= 2) over shuffled episodes, for the sparse n-gram TVD (get_ngram_tvd with
 * n > 2, metrics.py:173-248): for every episode e and anchor a (positions[j] for j < n_positions,
 * or every position 0 .. deck-1 when positions is NULL), keys[e * count + j] =
 * sum over k = 1 .. n-1 of (((v[(a + k*step) mod deck] - v[a]) - k*step) mod deck) * deck^(n-1-k),
 * in wrapping 64-bit arithmetic.  Same id layout as povs_travel_histogram_v1.
 */
int povs_ngram_keys_v1(const void* ids, int32_t id_bytes, int64_t n_episodes, int64_t deck, int64_t episode_stride,
                       int64_t element_stride, int32_t n, int64_t step, const int64_t* positions,
                       int64_t n_positions, int64_t* keys, int32_t device, void* stream);

/*
 * The distinct n-gram keys of povs_ngram_keys_v1 (same arguments) counted without sorting, for the
 * sparse n-gram TVD (metrics.py:173-248, which sorts the keys with np.unique): an open-addressing
 * hash table in `table` (device, 2 * slots + 1 uint64, overwritten; slots a power of two above the
 * number of keys, twice it or more keeps probes short), then the multiplicities of the counts:
 * mult[c] (device, mult_bins uint64, overwritten) = distinct keys seen exactly c times for
 * 1 <= c < mult_bins, mult[0] = distinct keys seen mult_bins times or more, whose counts go to
 * overflow[0 .. min(mult[0], overflow_cap) - 1] (device, any order).  The TVD needs only these:
 * observed keys = sum of mult, and sum over keys of |count / observations - p_ref|.  A key that
 * finds no free slot sets POVS_DEV_TABLE_FULL in the device status word.  No reference
 * counterpart as an entry point (the reference counts on the host).
 */
#define POVS_DEV_TABLE_FULL 8
int povs_ngram_count_v1(const void* ids, int32_t id_bytes, int64_t n_episodes, int64_t deck, int64_t episode_stride,
                        int64_t element_stride, int32_t n, int64_t step, const int64_t* positions,
                        int64_t n_positions, uint64_t* table, int64_t slots, uint64_t* mult, int64_t mult_bins,
                        uint64_t* overflow, int64_t overflow_cap, int32_t device, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* POVS_H */
