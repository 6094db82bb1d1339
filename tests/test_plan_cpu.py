"""Launch plans computed on the host (povs_plan_for_resources_v1), no GPU needed.

The planner (`povs_abi.cu: plan_launch`) decides unit sizes, packing, column slabs, stage counts
and kernel variants from the deck geometry and the device's resources.  These tests check its
invariants over a grid of row sizes and vblock shapes for B200's resources, and pin the plans of
the bench workloads to the ones `povs_describe_plan_v1` reported on a B200.
"""

from __future__ import annotations

import pytest

from povs import _native

SMEM_OPTIN, SMEM_PER_SM, SMS = 232448, 233472, 148

ROW_BYTES = [1, 2, 3, 4, 8, 12, 16, 20, 24, 28, 32, 48, 56, 64, 80, 96, 100, 112, 128, 144, 256, 512, 768, 1024,
             1040, 1536, 2048, 4096, 12288]
SHAPES = [(V, P) for V in (2, 4, 8, 16, 32) for P in (8, 16, 32, 64, 128, 256, 512, 1024) if V * P <= 1024]


def _plan(R: int, V: int, P: int, n_rows: int | None = None) -> dict[str, int]:
    n = n_rows if n_rows is not None else max(4 * V * P, (1 << 30) // R)
    return _native.plan_for_resources(n, R, P, V)


@pytest.mark.parametrize("R", ROW_BYTES)
def test_plan_invariants(R):
    for V, P in SHAPES:
        try:
            pl = _plan(R, V, P)
        except RuntimeError as e:  # only geometries outside the library's limits may be refused
            assert "unsupported" in str(e) or "does not fit" in str(e), (R, V, P, e)
            continue
        where = (R, V, P, pl)
        assert pl["stages_per_cta"] >= 2 and pl["smem"] <= SMEM_OPTIN, where
        assert pl["block"] == 32 * (pl["movers"] + pl["permuters"]) <= 512, where
        assert 1 <= pl["grid"] <= SMS * max(1, SMEM_PER_SM // (pl["smem"] + 1024)), where
        assert pl["rows_per_unit"] == pl["vblocks_per_unit"] * V * P <= 1024, where
        assert 32 * pl["sort_elems_per_lane"] >= pl["rows_per_unit"], where
        slab, n_slabs = pl["slab_bytes"], pl["n_slabs"]
        assert slab * n_slabs >= R > slab * (n_slabs - 1), where
        assert pl["stage_bytes"] % 128 == 0 and pl["stage_bytes"] >= pl["rows_per_unit"] * slab, where
        if pl["vblocks_per_unit"] > 1:  # packed units are always whole rows
            assert n_slabs == 1 and slab == R, where
        if pl["bulk"]:
            assert R % 16 == 0 and slab % 16 == 0, where
        if pl["chunked_kernel"]:
            assert not pl["bulk"] and R % 4 == 0 and R < 128 and pl["vblocks_per_unit"] > 1, where
            assert P * R == 512 or P * R >= 1024, where
        if pl["wide_kernel"]:
            assert pl["bulk"] and pl["vblocks_per_unit"] == 1 and 512 <= slab <= 1024, where


# Plans reported by povs_describe_plan_v1 on a B200 for the bench workloads (grid, smem, stages,
# permutation slots, vblocks per unit, slab bytes).
BENCH_PLANS = [
    ((134_217_728, 256, 32, 4), (148, 211712, 6, 14, 1, 256)),  # bf16_32GiB
    ((1_048_576, 256, 64, 2), (148, 212608, 6, 14, 1, 256)),  # fp16_256MiB
    ((1_000_000, 12288, 16, 2), (148, 205984, 3, 11, 1, 2048)),  # u8_12KiB: 2 KiB column slabs
    ((134_217_728, 16, 64, 2), (296, 100736, 4, 12, 8, 16)),  # f32x4_2GiB: 8 vblocks per unit
]


@pytest.mark.parametrize("args,want", BENCH_PLANS)
def test_bench_workload_plans_match_the_device(args, want):
    n, R, P, V = args
    pl = _plan(R, V, P, n)
    got = (pl["grid"], pl["smem"], pl["stages_per_cta"], pl["perm_slots"], pl["vblocks_per_unit"], pl["slab_bytes"])
    assert got == want


def test_planner_argument_checks():
    with pytest.raises(RuntimeError):
        _native.plan_for_resources(1000, 64, 8, 2, resources=(0, SMEM_OPTIN, SMEM_PER_SM, 2048))
    with pytest.raises(RuntimeError):
        _native.plan_for_resources(1000, 64, 8, 2, address=0)
    with pytest.raises(RuntimeError):
        _native.plan_for_resources(1000, 64, 12, 2)  # pblock not a power of two
