"""Host logic of the split output head (pipeline.py): vocab slices and the per-stage program, checked on the CPU.

The programs are run through a model of the ranks in which each rank executes its operations one at a time, in
program order, and a transfer or broadcast completes only when every rank taking part has reached it: the worst
case NCCL allows when several communicators share a GPU. They must always complete there; the earlier order
(every activation receive posted first) is shown to deadlock in the same model."""

import pytest

from forgeserve_b200.pipeline import HEAD_TILE, head_bounds, split_head_program


@pytest.mark.parametrize("vocab,size", [(128256, 8), (128256, 3), (1000, 2), (256, 4), (5, 2), (32000, 7)])
def test_head_bounds_tile_the_vocab(vocab, size):
    b = head_bounds(vocab, size)
    assert len(b) == size and b[0][0] == 0 and b[-1][1] == vocab
    assert all(b[i][1] == b[i + 1][0] for i in range(size - 1))
    assert all((lo % HEAD_TILE == 0 or lo == vocab) and lo <= hi for lo, hi in b)
    tiles = [-(-(hi - lo) // HEAD_TILE) for lo, hi in b]
    assert max(tiles) - min(tiles) <= 1 and tiles == sorted(tiles, reverse=True)


@pytest.mark.parametrize("size", [2, 3, 4, 8])
@pytest.mark.parametrize("m", [1, 2, 5, 16])
def test_program_does_every_piece_once_in_order(size, m):
    for rank in range(size):
        prog = split_head_program(rank, size, m)
        kinds = ["layers", "head", "bcast"] + (["recv"] if rank > 0 else []) + (["send"] if rank < size - 1 else [])
        for kind in kinds:
            assert [j for k, j in prog if k == kind] == list(range(m)), (rank, kind)
        assert set(k for k, _ in prog) == set(kinds)
        for j in range(m):
            at = prog.index
            assert at(("bcast", j)) < at(("head", j))
            if rank > 0:
                assert at(("recv", j)) < at(("layers", j))
            if rank < size - 1:
                assert at(("layers", j)) < at(("send", j))
            else:
                assert at(("layers", j)) < at(("bcast", j))


def _op(kind, j, rank):
    return {"send": ("S", rank, j), "recv": ("S", rank - 1, j), "bcast": ("B", j)}.get(kind)


def run_serialised(progs):
    """True if every rank gets through its program when each rank runs one operation at a time."""
    size = len(progs)
    pc = [0] * size
    while True:
        for r in range(size):   # local work runs as soon as it is reached
            while pc[r] < len(progs[r]) and _op(*progs[r][pc[r]], r) is None:
                pc[r] += 1
        if all(pc[r] == len(progs[r]) for r in range(size)):
            return True
        waiting = {}
        for r in range(size):
            if pc[r] < len(progs[r]):
                waiting.setdefault(_op(*progs[r][pc[r]], r), []).append(r)
        fired = False
        for op, ranks in waiting.items():
            if len(ranks) == (2 if op[0] == "S" else size):
                for r in ranks:
                    pc[r] += 1
                fired = True
        if not fired:
            return False


@pytest.mark.parametrize("size", [2, 3, 4, 5, 8])
@pytest.mark.parametrize("m", [1, 2, 3, 7, 16, 32])
def test_program_completes_when_every_rank_is_serialised(size, m):
    assert run_serialised([split_head_program(r, size, m) for r in range(size)])


def test_receives_posted_up_front_deadlock_in_the_model():
    """The order that hung: the last stage posts all its activation receives before its first broadcast."""
    size, m = 2, 3
    progs = [split_head_program(r, size, m) for r in range(size)]
    last = progs[-1]
    progs[-1] = [op for op in last if op[0] == "recv"] + [op for op in last if op[0] != "recv"]
    assert not run_serialised(progs)
