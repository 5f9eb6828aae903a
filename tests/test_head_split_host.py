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
@pytest.mark.parametrize("m", [1, 2, 3, 7, 16, 32, 64])     # 64: 16 micro-batches in 4 sequence pieces
def test_program_completes_when_every_rank_is_serialised(size, m):
    assert run_serialised([split_head_program(r, size, m) for r in range(size)])


def test_receives_posted_up_front_deadlock_in_the_model():
    """The order that hung: the last stage posts all its activation receives before its first broadcast."""
    size, m = 2, 3
    progs = [split_head_program(r, size, m) for r in range(size)]
    last = progs[-1]
    progs[-1] = [op for op in last if op[0] == "recv"] + [op for op in last if op[0] != "recv"]
    assert not run_serialised(progs)


# ------------------------------------------------------------------------ overlapped decoding (token ring)
from forgeserve_b200.pipeline import ring_program


def _ring_op(kind, k, rank, size):
    if kind in ("tok_send", "tok_recv"):
        return ("T", k)
    if kind == "act_send":
        return ("A", rank, k)
    if kind == "act_recv":
        return ("A", rank - 1, k)
    return None


def run_ring_serialised(size, progs):
    pc = [0] * size
    while True:
        for r in range(size):
            while pc[r] < len(progs[r]) and _ring_op(*progs[r][pc[r]], r, size) is None:
                pc[r] += 1
        if all(pc[r] == len(progs[r]) for r in range(size)):
            return True
        waiting = {}
        for r in range(size):
            if pc[r] < len(progs[r]):
                waiting.setdefault(_ring_op(*progs[r][pc[r]], r, size), []).append(r)
        fired = [op for op, ranks in waiting.items() if len(ranks) == 2]
        if not fired:
            return False
        for op in fired:
            for r in waiting[op]:
                pc[r] += 1


@pytest.mark.parametrize("size,m", [(2, 2), (2, 3), (2, 5), (3, 3), (3, 4), (4, 4), (4, 7), (8, 8), (8, 16)])
@pytest.mark.parametrize("steps", [1, 2, 5])
def test_ring_program_is_complete_ordered_and_completes_serialised(size, m, steps):
    items = steps * m
    progs = [ring_program(r, size, m, items) for r in range(size)]
    for r, prog in enumerate(progs):
        assert [k for op, k in prog if op == "compute"] == list(range(items))
        for k in range(items):
            c = prog.index(("compute", k))
            if r == 0:
                assert prog.index(("tok_recv", k)) < c
            else:
                assert prog.index(("act_recv", k)) < c
            if r < size - 1:
                assert c < prog.index(("act_send", k))
            elif k + m < items:
                assert c < prog.index(("tok_send", k + m))
    sends = [k for op, k in progs[-1] if op == "tok_send"]
    assert sorted(sends) == list(range(items)) and [k for op, k in progs[0] if op == "tok_recv"] == sends
    assert run_ring_serialised(size, progs)


def test_ring_program_needs_enough_microbatches():
    with pytest.raises(ValueError):
        ring_program(0, 4, 3, 10)
