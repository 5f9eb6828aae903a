"""The multi-process pipeline path on CPU: forgeserve_b200's own pipeline_forward / pipeline_generate schedule,
stage split, micro-batch rows, transports and run_distributed, over gloo with world_size 2 and 3.

The decoder math inside each stage is the oracle's (injected by subclassing the stage in this test file),
because the product's kernels need a GPU; what is under test is everything around them. The logits are
compared with the reference's own pipeline output (tests/golden/small.pt)."""

from pathlib import Path

import pytest
import torch

from oracle import forge_oracle as O

GOLDEN = Path(__file__).resolve().parent / "golden"


def _oracle_stage_class():
    from forgeserve_b200 import PipelineStage

    class OracleStage(PipelineStage):
        """A PipelineStage whose compute is the CPU oracle (test-only)."""

        def _ocfg(self):
            return O.Cfg(**self.cfg.to_dict())

        def embed(self, idx):
            return self.tok_emb.weight.detach()[idx.cpu()].clone()

        def run_layers_(self, x, positions, caches):
            cfg = self._ocfg()
            cos, sin = O.rope_tables(cfg.head_dim, cfg.max_seq_len, cfg.rope_theta)
            for j, (layer, kv) in enumerate(zip(self.layers, caches)):
                sd = {f"layers.0.{k}": v.detach() for k, v in layer.state_dict().items()}
                x.copy_(O.block(sd, 0, x, cfg, cos, sin, positions, kv))
            return x

        def head(self, x, out=None):
            y = O.head({"norm.weight": self.norm.weight.detach(), "lm_head.weight": self.lm_head.weight.detach()}, x,
                       self._ocfg())
            if out is None:
                return y
            out.copy_(y)
            return out

    return OracleStage


def forward_worker(rank, size, cfg_dict, full_sd, idx, more, microbatches):
    from forgeserve_b200 import ModelConfig, PipelineState, pipeline_forward
    cfg = ModelConfig(**cfg_dict)
    stage = _oracle_stage_class()(cfg, rank, size, device="cpu")
    stage.load_from_full(full_sd)
    state = PipelineState(stage, idx.shape[0], microbatches)
    logits = pipeline_forward(stage, state, idx if rank == 0 else None, idx.shape[1])
    logits2 = pipeline_forward(stage, state, more if rank == 0 else None, more.shape[1])
    layer_params = sum(p.numel() for p in stage.layers.parameters())
    return logits, logits2, layer_params


def pieces_worker(rank, size, cfg_dict, full_sd, idx, more, microbatches, pieces, quantum):
    import forgeserve_b200.pipeline as P
    from forgeserve_b200 import ModelConfig, PipelineState, pipeline_forward
    P.SEQ_PIECE_QUANTUM = quantum     # test-only: the golden model's sequences are shorter than 128 tokens
    P.PIECE_MIN_ROWS = 1
    P.sample = lambda logits, temperature=0.0, generator=None: logits.argmax(-1)   # CPU greedy, test-only
    cfg = ModelConfig(**cfg_dict)
    stage = _oracle_stage_class()(cfg, rank, size, device="cpu")
    stage.load_from_full(full_sd)
    res = []
    for c in (1, pieces):
        state = PipelineState(stage, idx.shape[0], microbatches)
        first = pipeline_forward(stage, state, idx if rank == 0 else None, idx.shape[1], seq_chunks=c)
        cont = pipeline_forward(stage, state, more if rank == 0 else None, more.shape[1], seq_chunks=c)
        state = PipelineState(stage, idx.shape[0], microbatches)
        last = pipeline_forward(stage, state, idx if rank == 0 else None, idx.shape[1], last_only=True, seq_chunks=c)
        res.append((first, cont, last, state.length, P.pipeline_generate(stage, idx[:, :5], 6, microbatches,
                                                                         seq_chunks=c)))
    return res


def generate_worker(rank, size, cfg_dict, full_sd, prompt, microbatches, n):
    import forgeserve_b200.pipeline as P
    from forgeserve_b200 import ModelConfig
    P.sample = lambda logits, temperature=0.0, generator=None: logits.argmax(-1)   # CPU greedy, test-only
    cfg = ModelConfig(**cfg_dict)
    stage = _oracle_stage_class()(cfg, rank, size, device="cpu")
    stage.load_from_full(full_sd)
    return P.pipeline_generate(stage, prompt, n, microbatches)


def empty_microbatch_worker(rank, size, cfg_dict, full_sd, idx):
    from forgeserve_b200 import ModelConfig, PipelineState, pipeline_forward
    cfg = ModelConfig(**cfg_dict)
    stage = _oracle_stage_class()(cfg, rank, size, device="cpu")
    stage.load_from_full(full_sd)
    state = PipelineState(stage, idx.shape[0], idx.shape[0] + 2)
    return pipeline_forward(stage, state, idx if rank == 0 else None, idx.shape[1])


@pytest.fixture(scope="module")
def golden():
    g = torch.load(GOLDEN / "small.pt", weights_only=False)
    sd = O.test_model_weights(O.Cfg(**g["cfg"]), *g["weights"][1:])
    return g, sd


@pytest.mark.parametrize("size,microbatches", [(2, 1), (3, 2), (3, 4)])
def test_pipeline_schedule_over_gloo_matches_reference(golden, size, microbatches):
    from forgeserve_b200.tensor_parallel import run_distributed
    g, sd = golden
    res = run_distributed(forward_worker, size, g["cfg"], sd, g["idx"], g["more"], microbatches, backend="gloo")
    logits, logits2, _ = res[-1]
    want, want2 = g["pipeline"][(size, microbatches)]
    torch.testing.assert_close(logits, want, atol=1e-4, rtol=1e-4)
    torch.testing.assert_close(logits2, want2, atol=1e-4, rtol=1e-4)    # continued through the stage caches
    assert all(r[0] is None and r[1] is None for r in res[:-1])
    total = sum(v.numel() for k, v in sd.items() if k.startswith("layers."))
    assert sum(r[2] for r in res) == total


def test_pipeline_generation_over_gloo_matches_reference(golden):
    from forgeserve_b200.tensor_parallel import run_distributed
    g, sd = golden
    res = run_distributed(generate_worker, 2, g["cfg"], sd, g["prompt"], 2, 10, backend="gloo")
    for out in res:
        assert torch.equal(out, g["generate"])


def test_more_microbatches_than_rows_is_refused_on_every_rank(golden):
    from forgeserve_b200.tensor_parallel import run_distributed
    g, sd = golden
    with pytest.raises(RuntimeError, match="micro-batches"):
        run_distributed(empty_microbatch_worker, 2, g["cfg"], sd, g["idx"][:2], backend="gloo", timeout=60)


@pytest.mark.parametrize("size,microbatches,pieces,quantum", [(2, 1, 2, 4), (3, 2, 3, 1), (3, 4, 2, 2)])
def test_sequence_pieces_give_the_same_logits(golden, size, microbatches, pieces, quantum):
    """pipeline_forward with each micro-batch split into pieces along the sequence (more items in the schedule,
    every piece after the earlier ones of its rows on every stage): the logits of every position, of a forward
    continued through the caches, and of last_only, as with whole micro-batches and as the reference's."""
    from forgeserve_b200.pipeline import seq_pieces
    from forgeserve_b200.tensor_parallel import run_distributed
    g, sd = golden
    t = g["idx"].shape[1]
    res = run_distributed(pieces_worker, size, g["cfg"], sd, g["idx"], g["more"], microbatches, pieces, quantum,
                          backend="gloo")
    (first, cont, last, n, gen), (first_p, cont_p, last_p, n_p, gen_p) = res[-1]
    assert all(torch.equal(r[1][4], gen) and torch.equal(r[0][4], gen) for r in res)   # generation, prompt in pieces
    want, want2 = g["pipeline"][(size, microbatches)]
    # the fp32 bar: the CPU stand-in's attention sums in another order for another number of queries
    for got, ref in ((first_p, first), (first_p, want), (cont_p, cont), (cont_p, want2), (last_p, first[:, -1:])):
        torch.testing.assert_close(got, ref, atol=1e-4, rtol=1e-4)
    assert last.shape == last_p.shape and n == n_p == t
    assert all(r[1][0] is None for r in res[:-1])


def test_seq_pieces_bounds():
    import forgeserve_b200.pipeline as P
    assert P.SEQ_PIECE_QUANTUM == 128 and P.PIECE_MIN_ROWS == 129
    assert P.seq_pieces(2048, 4, 4) == [(0, 512), (512, 1024), (1024, 1536), (1536, 2048)]     # config 3
    assert P.seq_pieces(2048, 3, 4) == [(0, 768), (768, 1536), (1536, 2048)]
    assert P.seq_pieces(1000, 4, 4) == [(0, 256), (256, 512), (512, 768), (768, 1000)]
    assert P.seq_pieces(200, 4, 4) == [(0, 200)] and P.seq_pieces(2048, 1, 4) == [(0, 2048)]
    assert P.seq_pieces(512, 4, 1) == [(0, 256), (256, 512)]          # one row: pieces of 256 tokens at least
    assert P.seq_pieces(520, 2, 1) == [(0, 384), (384, 520)]
    assert P.seq_pieces(300, 2, 1) == [(0, 300)]
    for t in range(1, 3000, 37):
        for n in (1, 2, 3, 5, 8):
            for rows in (1, 2, 4):
                b = P.seq_pieces(t, n, rows)
                assert b[0][0] == 0 and b[-1][1] == t and len(b) <= n
                assert all(c1 == d0 and c0 % 128 == 0 and c1 > c0 for (c0, c1), (d0, _) in zip(b, b[1:] + [(t, t)]))
                assert len(b) == 1 or all(rows * (c1 - c0) >= 129 for c0, c1 in b)   # every GEMM > 128 rows


def _oracle_tp_stage_class():
    """A PipelineStage whose layers are computed by the oracle on this process's tensor-parallel shard: each shard's
    partial attention and MLP outputs summed over the stage's shards by the all-reduce (test-only compute; the
    grid, the groups, the weight cutting and the schedule are the product's)."""
    import torch.distributed as dist
    base = _oracle_stage_class()

    class OracleTPStage(base):
        def run_layers_(self, x, positions, caches):
            cfg = self._ocfg()
            c = O.shard_cfg(cfg, self.tp.size)
            cos, sin = O.rope_tables(cfg.head_dim, cfg.max_seq_len, cfg.rope_theta)
            for layer, kv in zip(self.layers, caches):
                sd = {f"layers.0.{k}": v.detach() for k, v in layer.state_dict().items()}
                h = O.rms_norm(x, sd["layers.0.attn_norm.weight"], cfg.norm_eps)
                part = O.attention(sd, "layers.0.", h, c, cos, sin, positions, kv)
                dist.all_reduce(part, group=self.tp.group)
                x.add_(part)
                part = O.swiglu(sd, "layers.0.", O.rms_norm(x, sd["layers.0.mlp_norm.weight"], cfg.norm_eps))
                dist.all_reduce(part, group=self.tp.group)
                x.add_(part)
            return x

    return OracleTPStage


def grid_worker(rank, size, cfg_dict, full_sd, idx, more, microbatches, stages, prompt, pieces=1):
    import forgeserve_b200.pipeline as P
    from forgeserve_b200 import ModelConfig, PipelineState, pipeline_forward
    from forgeserve_b200.transport import make_grid
    P.sample = lambda logits, temperature=0.0, generator=None: logits.argmax(-1)   # CPU greedy, test-only
    P.SEQ_PIECE_QUANTUM, P.PIECE_MIN_ROWS = 2, 1      # test-only: short sequences
    cfg = ModelConfig(**cfg_dict)
    stage_idx, tp, transport = make_grid(stages, size // stages)
    stage = _oracle_tp_stage_class()(cfg, stage_idx, stages, device="cpu", tp=tp, transport=transport)
    stage.load_from_full(full_sd)
    state = PipelineState(stage, idx.shape[0], microbatches)
    first = pipeline_forward(stage, state, idx if stage.is_first else None, idx.shape[1], seq_chunks=pieces)
    cont = pipeline_forward(stage, state, more if stage.is_first else None, more.shape[1], seq_chunks=pieces)
    gen = P.pipeline_generate(stage, prompt, 10, microbatches, seq_chunks=pieces)
    shapes = {k: tuple(v.shape) for k, v in stage.state_dict().items()}
    return stage_idx, tp.rank, first, cont, gen, shapes


@pytest.mark.parametrize("stages,shards,microbatches,pieces",
                         [(2, 2, 1, 1), (2, 2, 2, 1), (3, 2, 4, 1), (3, 1, 2, 1), (1, 4, 2, 1), (2, 2, 2, 3)])
def test_tensor_parallel_stages_over_gloo(golden, stages, shards, microbatches, pieces):
    """A stages x shards grid (transport.make_grid): every shard of the last stage returns the reference pipeline's
    logits, continued through the shards' caches, and every rank generates the reference's tokens; each shard holds
    its cut of its stage's layers."""
    from forgeserve_b200.tensor_parallel import run_distributed
    g, sd = golden
    res = run_distributed(grid_worker, stages * shards, g["cfg"], sd, g["idx"], g["more"], microbatches, stages,
                          g["prompt"], pieces, backend="gloo", timeout=300)
    for rank, (stage_idx, shard, first, cont, gen, shapes) in enumerate(res):
        assert (stage_idx, shard) == divmod(rank, shards)
        if stage_idx == stages - 1:
            torch.testing.assert_close(first, g["logits"], atol=1e-4, rtol=1e-4)
            torch.testing.assert_close(cont, g["logits_more"], atol=1e-4, rtol=1e-4)
        else:
            assert first is None and cont is None
        assert torch.equal(gen, g["generate"])
        assert shapes["layers.0.attn.wq.weight"][0] == g["cfg"]["d_model"] // shards
        assert shapes["layers.0.mlp.w_down.weight"][1] == O.Cfg(**g["cfg"]).ffn_dim // shards
