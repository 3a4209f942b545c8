"""Host-side K-split planning of the grouped decode GEMV (sbq_gemv_plan_parts): no GPU involved.

A launch cuts its 16-row tiles into K parts only when the tiles alone cannot keep the GPU's CTAs
busy; a one-GPU decode step of the stack never splits (its results stay those of whole-tile
sums), a sharded step cuts its largest tiles, and no part is smaller than 32 KiB.
"""

import ctypes

import pytest

from conftest import load_package

SLOTS = 3 * 148  # CTA slots of a B200 at m <= 8


def plan(jobs, slots=SLOTS, m=1):
    L = load_package()._lib
    lib = L.load()
    flat = (ctypes.c_int64 * (3 * len(jobs)))(*[v for job in jobs for v in job])
    parts = (ctypes.c_int * len(jobs))()
    status = lib.sbq_gemv_plan_parts(flat, len(jobs), slots, m, parts)
    return status, list(parts)


def stack_launches(world):
    h, inter = 4096, 12288
    return ([(inter // world, h, 2), (4 * h // world, h, 1)],
            [(h // world, inter, 1), (h // world, h, 1), (h // world, h, 1)])


def test_one_gpu_stack_never_splits():
    for jobs in stack_launches(1):
        status, parts = plan(jobs)
        assert status == 0 and parts == [1] * len(jobs)


@pytest.mark.parametrize("world", [4, 8])
def test_sharded_stack_splits_its_largest_tiles(world):
    l1, l2 = stack_launches(world)
    _, p2 = plan(l2)
    assert p2[0] > 1  # the down projection's 192 KiB tiles
    if world == 8:
        _, p1 = plan(l1)
        assert p1[0] > 1  # the fused gate/up job's 128 KiB tiles


def test_parts_are_at_least_32_kib_of_whole_chunks():
    jobs = [(64, 12288, 1), (16, 4096, 2), (32, 2048, 1), (4, 128, 1)]
    status, parts = plan(jobs)
    assert status == 0
    for (n, k, nmat), p in zip(jobs, parts):
        tile_bytes = 16 * (-(-k // 64)) * 64 * nmat
        assert 1 <= p <= 8 and tile_bytes // p >= 32 * 1024 or p == 1


def test_few_tiles_are_cut():
    status, parts = plan([(64, 12288, 1)])
    assert status == 0 and parts == [6]  # four 192 KiB tiles -> 24 parts of 32 KiB


def test_plan_is_deterministic_and_cached():
    jobs = [(1536, 4096, 2), (2048, 4096, 1)]
    assert plan(jobs) == plan(jobs) == plan(list(jobs))


def test_invalid_plans_rejected():
    L = load_package()._lib
    status, _ = plan([(0, 4096, 1)])
    assert status == L.ERR_INVALID_ARGUMENT
    status, _ = plan([(16, 100, 1)])  # k not a multiple of 16
    assert status == L.ERR_INVALID_ARGUMENT
    status, _ = plan([(16, 128, 3)])
    assert status == L.ERR_INVALID_ARGUMENT
    status, _ = plan([(16, 128, 1)], m=17)
    assert status == L.ERR_INVALID_ARGUMENT
