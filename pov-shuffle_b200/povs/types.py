"""Public option types (same names and fields as src/povs/types.py:4-32 of the reference)."""

from typing import NamedTuple


class BuildParams(NamedTuple):
    """Build-time parameters of the native library.

    The reference compiles one template instantiation per (vblock, pblock, instance size, dtype)
    and lists them here; this library's kernels are runtime-general, so the instantiation lists are
    empty and ``cartesian_instancing`` is False.
    """

    debug_mode: bool
    cuda_arch: list[str]
    vblock_sizes: list[int]
    pblock_sizes: list[int]
    instance_sizes: list[int]
    cartesian_instancing: bool
    instantiations: list
    instantiations_all_types: list


class Options(NamedTuple):
    """POV Shuffle algorithm options.

    :param virtual_block_size: Virtual block size, in number of physical blocks.
    :param physical_block_size: Physical block size, in number of instances.
    :param offsets: List of valid offsets to sample at random in each shuffling iteration, in number of instances.
    :param gpu_thread_block_size: Accepted for compatibility; the B200 kernels size their launch themselves.
    :param randomness: ``"uniform"`` (default: uniformly random permutation of every virtual block),
                       ``"reference_cuda"`` (the reference CUDA implementation's distribution: per-block seeds
                       1..999 and an xorshift32 Fisher-Yates, padding in the last virtual block) or
                       ``"reference_numpy"`` (the reference NumPy implementation's distribution: padding
                       anywhere, per-block seeds 1..999 and ``numpy.random.RandomState(seed).shuffle``), for
                       statistical comparisons with them.  Not part of the reference's options.
    """

    virtual_block_size: int | None = None
    physical_block_size: int | None = None
    offsets: list[int] | None = None

    gpu_thread_block_size: int | None = None

    randomness: str | None = None
