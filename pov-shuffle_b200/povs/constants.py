"""Constants of the option model (names as in src/povs/constants.py of the reference).

Values that differ from the reference, and why:
  * ``MAX_SEED``: a ``numpy.random.Generator`` / ``torch.Generator`` seed is drawn from
    [1, 2**63 - 1) instead of [1, 1000).  The reference narrowed it so that its 32-bit per-vblock
    seeds matched between CPU and CUDA (constants.py:1-4 there); the device RNG here is keyed
    by the full 64-bit seed, so a generator no longer collapses to 999 distinct shuffles.  With
    ``randomness="reference_cuda"`` or ``"reference_numpy"`` (the reference's distributions) a
    generator draws from the reference's [1, 1000) again (``REFERENCE_MAX_SEED``).
  * ``MIN_PBLOCK_SIZE`` is 8 (the reference has 16).  With 8-bit instances and P = 8 the offset
    chooser still finds the two offsets [0, 4], which is the invariant the reference's bound
    protects; P = 8 is needed by the bias suite (deck 1000, V = 2, P = 8).
  * ``CUDA_CC_IDEAL_OCCUPANCY`` keeps the reference table; the B200 kernel plans its own launch
    and only uses ``physical_block_size`` / ``virtual_block_size`` from the options.
"""

MIN_SEED = 1
MAX_SEED = 2**63 - 1
REFERENCE_MAX_SEED = 1000

# At least two offsets so that the per-iteration offset draw is not a constant.
MIN_OFFSETS = 2

MIN_PBLOCK_SIZE = 8

# Physical block size the CPU-data route picks when none is given (the reference's NumPy default).
DEFAULT_CPU_PBLOCK_SIZE = 16

MIN_VBLOCK_SIZE = 2

# Offsets must keep each pblock start aligned to at least this many bits.
MIN_MEM_ALIGNMENT_BITS = 16

# Preferred alignment of pblock starts (16-byte vector copies).
MAX_MEM_ALIGNMENT_BITS = 128

MIN_CUDA_ARCH = (10, 0)
MAX_BLOCK_SIZE = 1024
MIN_BLOCK_SIZE = 32

# Limits of the native library (include/povs.h).
MAX_VBLOCK_SIZE = 32
MAX_VP = 1024
MAX_OFFSETS = 256

CUDA_CC_IDEAL_OCCUPANCY: dict[tuple[int, int], tuple[int, int]] = {
    (12, 0): (64, 24),
    (11, 0): (64, 24),
    (10, 3): (64, 32),
    (10, 0): (64, 32),
    (9, 0): (64, 32),
    (8, 9): (64, 24),
    (8, 7): (96, 16),
    (8, 6): (96, 16),
    (8, 0): (64, 16),
    (7, 5): (64, 16),
}
CUDA_DEFAULT_IDEAL_OCCUPANCY = (64, 24)
