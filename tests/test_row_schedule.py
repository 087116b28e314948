"""Launch plan of the overlapped row-parallel reduction (CPU).

Every chunk's reduce-scatter (phase A) and all-gather (phase B) must each be
carried exactly once; phase A only after the chunk's second GEMM (its
partial is complete in stream order), phase B only after phase A was carried
by an earlier launch (every rank's slab announced) or in the same final
launch; a first-GEMM launch before the second GEMMs of its chunks; launches
of their own only at the end.  Row chunks start and end on multiples of the
world size and cover the rows once.
"""
import pytest

from deepx_op_gpukernelcompiler_b200.shard import first_groups, row_chunks, row_schedule


@pytest.mark.parametrize("n", [1, 2, 3, 4, 5, 8, 13, 64])
@pytest.mark.parametrize("groups", [None, 1, 2, 3, 4])
def test_schedule_invariants(n, groups):
    plan = row_schedule(n, first_groups(n, groups))
    where_a, where_b, second_at, first_at = {}, {}, {}, {}
    seen_reduce = False
    for i, launch in enumerate(plan):
        kind = launch[0]
        a, b = launch[-1]
        if kind == "reduce":
            seen_reduce = True
        else:
            assert not seen_reduce, "GEMM launch after a launch of its own"
        if kind == "first":
            for c in range(launch[1], launch[2]):
                assert c not in first_at
                first_at[c] = i
        if kind == "second":
            second_at[launch[1]] = i
        if a is not None:
            assert a not in where_a
            where_a[a] = i
        if b is not None:
            assert b not in where_b
            where_b[b] = i
    assert sorted(first_at) == sorted(second_at) == list(range(n))
    assert sorted(where_a) == sorted(where_b) == list(range(n))
    for c in range(n):
        assert first_at[c] < second_at[c]
        assert where_a[c] > second_at[c]
        assert where_b[c] > where_a[c] or (where_b[c] == where_a[c] and plan[where_a[c]][0] == "reduce")
    # at most two launches of their own end a step
    assert sum(1 for p in plan if p[0] == "reduce") <= 2


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
@pytest.mark.parametrize("M", [8, 24, 1000, 1024, 16384, 16392])
@pytest.mark.parametrize("chunks", [1, 3, 4, 8, 100])
def test_row_chunks_cover_rows(world, M, chunks):
    if M % world:
        with pytest.raises(ValueError):
            row_chunks(M, world, chunks)
        return
    ch = row_chunks(M, world, chunks)
    assert 1 <= len(ch) <= min(chunks, 64)
    pos = 0
    for r0, rn in ch:
        assert r0 == pos and rn > 0 and r0 % world == 0 and rn % world == 0
        pos += rn
    assert pos == M
    if M % (32 * world) == 0:
        assert all(rn % (32 * world) == 0 for _, rn in ch)
