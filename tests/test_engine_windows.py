"""Decode windows of the continuous-batching scheduler (Scheduler._window_steps / _window_step / _window_end, and
PipelineEngine._decode_window over gloo ranks): taking several decode steps at once must give the outputs, block
tables, positions and counters (steps, preemptions, peaks) of the reference's one-step-at-a-time scheduler
(forgeserve/engine.py:80-139).

The model is a deterministic stand-in whose next token depends on the previous token and its position, so a
token routed to the wrong row or step changes every later token; the scheduling is the product's."""

import pytest
import torch

from forgeserve_b200 import ModelConfig
from forgeserve_b200.engine import Scheduler
from forgeserve_b200.paged import PagedKVPool

V = 61


def next_token(prev: int, pos: int) -> int:
    return (prev * 7 + pos * 3 + 1) % V


class FakeScheduler(Scheduler):
    """Scheduler over a stand-in model; `windowed` lets run() take decode windows, computed on the host."""

    def __init__(self, cfg, num_blocks, block_size, max_batch, windowed):
        self.cfg = cfg
        self.pool = PagedKVPool(cfg, num_blocks, block_size, n_layers=1)
        self.windowed, self.trace, self.windows = windowed, [], 0
        self._init_scheduler(max_batch, seed=0)

    def _forward_rows(self, reqs, idx, positions, tables):
        self.trace.append((tables.tolist(), positions.tolist()))
        last = positions[:, -1].tolist()
        out = []
        for r, req in enumerate(reqs):
            if req.temperature != 0:      # consume the generator as sampling does (row order, once per row)
                torch.rand(1, generator=self.generator)
            out.append(next_token(int(idx[r, -1]), last[r]))
        return out

    def _windowed(self):
        return self.windowed

    def _decode_window(self, w):
        rows = list(self.running)
        cached = [r.cached for r in rows]
        prev = [r.output[-1] for r in rows]
        tokens = []
        for t in range(w):
            tables, positions = self._window_step(rows, cached, t, last=t == w - 1)
            self.trace.append((tables.tolist(), positions.tolist()))
            prev = [next_token(p, c + t) for p, c in zip(prev, cached)]
            tokens.append(prev)
        self._window_end(rows, tokens)
        self.windows += 1


def _requests(seed, n, max_len):
    g = torch.Generator().manual_seed(seed)
    out = []
    for i in range(n):
        plen = int(torch.randint(1, max_len // 2, (1,), generator=g))
        prompt = torch.randint(0, V, (plen,), generator=g).tolist()
        new = int(torch.randint(1, max_len, (1,), generator=g))
        eos = None if i % 4 else int(torch.randint(0, V, (1,), generator=g))     # some rows stop on eos
        temp = 0.7 if i % 5 == 3 else 0.0
        out.append((prompt, new, eos, temp))
    return out


def _run(windowed, requests, num_blocks, block_size, max_batch, max_seq_len):
    cfg = ModelConfig(vocab_size=V, d_model=16, n_layers=1, n_heads=2, n_kv_heads=1, max_seq_len=max_seq_len)
    s = FakeScheduler(cfg, num_blocks, block_size, max_batch, windowed)
    for prompt, new, eos, temp in requests:
        s.add_request(prompt, new, eos, temp)
    out = s.run()
    return out, s


@pytest.mark.parametrize("seed,n,num_blocks,block_size,max_batch,max_seq_len", [
    (0, 6, 64, 4, 3, 48),          # roomy pool, waiting requests
    (1, 9, 14, 4, 6, 40),          # small pool: preemptions, windows cut before a grant finds it empty
    (2, 5, 40, 8, 5, 30),          # rows reaching max_seq_len
    (3, 12, 30, 2, 12, 24),        # block size 2: grants inside most windows
])
def test_windows_reproduce_stepwise_scheduling(seed, n, num_blocks, block_size, max_batch, max_seq_len):
    reqs = _requests(seed, n, max_seq_len)
    want, a = _run(False, reqs, num_blocks, block_size, max_batch, max_seq_len)
    got, b = _run(True, reqs, num_blocks, block_size, max_batch, max_seq_len)
    assert got == want
    assert b.trace == a.trace                      # every step's block tables and positions
    assert (b.steps, b.preemptions, b.peak_running, b.peak_blocks) == (a.steps, a.preemptions, a.peak_running,
                                                                        a.peak_blocks)
    assert b.pool.allocator.num_free == num_blocks
    assert b.windows > 0


def test_window_length_rules():
    cfg = ModelConfig(vocab_size=V, d_model=16, n_layers=1, n_heads=2, n_kv_heads=1, max_seq_len=32)
    s = FakeScheduler(cfg, num_blocks=8, block_size=4, max_batch=2, windowed=False)
    a = s.add_request([1, 2, 3], 10)
    b = s.add_request([4, 5, 6, 7, 8], 6)
    s.step()
    s.step()                                       # both prefilled: cached 3 and 5, one token each
    assert [r.cached for r in s.running] == [3, 5]
    assert s._window_steps() == 5                  # b finishes after 5 more tokens (6 new in all)
    s.requests[b].eos_id = 9
    assert s._window_steps() == 0                  # a row that may stop on eos: no window
    s.requests[b].eos_id = None
    s.requests[a].temperature = 0.5
    assert s._window_steps() == 0                  # a sampled row: no window
    s.requests[a].temperature = 0.0
    s.pool.allocator.allocate(s.pool.allocator.num_free - 1)   # one free block left
    # step 0: a writes position 3, b position 5 (no grants); step 1: a takes the last free block at position 4;
    # step 3: b needs a block at position 8 and the pool is empty (the stepwise scheduler preempts): steps 0-2
    assert s._window_steps() == 3
    s.add_request([1], 3)
    assert s._window_steps() == 3                  # a request waits, but running == max_batch: still decodes


# ------------------------------------------------------------------------------ PipelineEngine over gloo
def _fake_stage_class():
    from forgeserve_b200 import PipelineStage

    class FakeStage(PipelineStage):
        """Stage s adds (s + 1) * position to an accumulator; the head turns (token, accumulator) into the next
        token. Each stage records the block tables and positions it was given."""

        def embed(self, idx):
            x = torch.zeros(*idx.shape, self.cfg.d_model)
            x[..., 0] = idx.float()
            return x

        def run_layers_(self, x, positions, caches):
            self.seen.append((caches[0].tables.tolist(), positions.tolist()))
            x[..., 1] += (self.rank + 1) * positions.float()
            return x

        def head(self, x, out=None):
            tok = (x[..., 0].long() * 7 + x[..., 1].long() * 3 + 1) % self.cfg.vocab_size
            y = torch.nn.functional.one_hot(tok, self.cfg.vocab_size).float()
            if out is None:
                return y
            out.copy_(y)
            return out

    return FakeStage


def window_worker(rank, size, cfg_dict, requests, num_blocks, max_batch, microbatches, prefill_chunks=1):
    import forgeserve_b200.pipeline as P
    from forgeserve_b200.pipeline_engine import PipelineEngine
    P.SEQ_PIECE_QUANTUM = 4                    # test-only: prompts here are shorter than 128 tokens
    P.PIECE_MIN_ROWS = 1

    class CpuEngine(PipelineEngine):
        def _argmax(self, logits):
            return logits.argmax(-1)

    cfg = ModelConfig(**cfg_dict)
    res = []
    for overlap in (False, None):
        stage = _fake_stage_class()(cfg, rank, size, device="cpu")
        stage.seen = []
        eng = CpuEngine(stage, num_blocks=num_blocks, block_size=4, max_batch=max_batch, microbatches=microbatches,
                        overlap=overlap, prefill_chunks=prefill_chunks)
        for prompt, new, eos, temp in requests:
            eng.add_request(prompt, new, eos, temp)
        out = eng.run()
        res.append((out, eng.steps, eng.preemptions, eng.peak_running, eng.peak_blocks, eng.pool.allocator.num_free,
                    stage.seen, eng.windows))
    return res


@pytest.mark.parametrize("size,microbatches", [(2, 2), (3, 3), (3, 4)])
def test_pipeline_engine_windows_over_gloo(size, microbatches):
    """The ring order, the per-step grants on every stage and the token flow of PipelineEngine._decode_window, as
    processes over gloo: the same outputs, counters and per-stage tables/positions as stepping one by one."""
    from forgeserve_b200.tensor_parallel import run_distributed
    cfg = ModelConfig(vocab_size=V, d_model=16, n_layers=3, n_heads=2, n_kv_heads=1, max_seq_len=48)
    reqs = [(p, n, None, 0.0) for p, n, _, _ in _requests(5, 8, 48)]
    reqs[1] = (reqs[1][0], 3, 17, 0.0)             # an eos row and a sampled row, both short: windows come after
    reqs[2] = (reqs[2][0], 4, None, 0.9)
    res = run_distributed(window_worker, size, cfg.to_dict(), reqs, 30, 6, microbatches, backend="gloo",
                          timeout=240)
    _, ref = _run(False, reqs, 30, 4, 6, 48)        # the host-only scheduler with the same stand-in arithmetic
    for stepwise, windowed in res:
        assert stepwise[7] == 0 and windowed[7] > 0
        assert windowed[:6] == stepwise[:6]
        assert windowed[6] == stepwise[6]          # this stage's tables and positions, step by step
    assert res[0][0][1] == ref.steps and res[0][0][2] == ref.preemptions


try:
    from hypothesis import given, settings, strategies as st
except ImportError:                       # hypothesis is optional
    given = None

if given is not None:
    @settings(max_examples=150, deadline=None)
    @given(seed=st.integers(0, 10_000), n=st.integers(1, 10), num_blocks=st.integers(6, 60),
           block_size=st.sampled_from([1, 2, 4, 8]), max_batch=st.integers(1, 8),
           max_seq_len=st.sampled_from([16, 24, 40]), eos_every=st.sampled_from([0, 2, 5]),
           temp_every=st.sampled_from([0, 3]))
    def test_windows_match_stepping_on_random_workloads(seed, n, num_blocks, block_size, max_batch, max_seq_len,
                                                        eos_every, temp_every):
        """Any mix of requests, pools and limits: windowed scheduling gives the outputs, per-step tables and
        positions, and counters of stepping one by one (or both refuse the same unschedulable pool)."""
        g = torch.Generator().manual_seed(seed)
        reqs = []
        for i in range(n):
            plen = int(torch.randint(1, max_seq_len - 1, (1,), generator=g))
            new = int(torch.randint(1, max_seq_len, (1,), generator=g))
            eos = int(torch.randint(0, V, (1,), generator=g)) if eos_every and i % eos_every == 0 else None
            temp = 0.8 if temp_every and i % temp_every == 1 else 0.0
            reqs.append((torch.randint(0, V, (plen,), generator=g).tolist(), new, eos, temp))
        runs = []
        for windowed in (False, True):
            try:
                out, s = _run(windowed, reqs, num_blocks, block_size, max_batch, max_seq_len)
                runs.append((out, s.trace, s.steps, s.preemptions, s.peak_running, s.peak_blocks,
                             s.pool.allocator.num_free))
            except (ValueError, RuntimeError) as e:
                runs.append(("error", type(e).__name__, str(e)))
        assert runs[0] == runs[1]


def test_pipeline_engine_prefill_pieces_over_gloo():
    """A prefill step pushed through the stages in pieces of the prompt (PipelineEngine's prefill_chunks): the
    outputs and counters of whole prefills; every stage sees the pieces' positions in order."""
    from forgeserve_b200.tensor_parallel import run_distributed
    cfg = ModelConfig(vocab_size=V, d_model=16, n_layers=3, n_heads=2, n_kv_heads=1, max_seq_len=48)
    reqs = [(p, n, None, 0.0) for p, n, _, _ in _requests(5, 8, 48)]
    whole = run_distributed(window_worker, 2, cfg.to_dict(), reqs, 30, 6, 2, 1, backend="gloo", timeout=240)
    pieces = run_distributed(window_worker, 2, cfg.to_dict(), reqs, 30, 6, 2, 3, backend="gloo", timeout=240)
    for w, p in zip(whole, pieces):
        for a, b in zip(w, p):
            assert a[:6] == b[:6]                      # outputs, steps, preemptions, peaks, free blocks
        seen_w, seen_p = w[0][6], p[0][6]
        assert len(seen_p) > len(seen_w)               # prefills arrived in several pieces
        starts = [pos[0][0] for _, pos in seen_p if len(pos[0]) > 1]
        assert any(s0 > 0 for s0 in starts)            # pieces after the first start past position 0
