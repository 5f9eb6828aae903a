"""Multi-GPU tests of paths whose single-GPU and CPU tests have passed, but which have not yet run on several GPUs:
sequence pieces with the split head, prefill pieces in the pipeline engine, and the stage x shard grid. They skip
without enough GPUs. They sit in the last test file, after the suites already run on a B200, so that with -x a
failure here stops nothing else."""

from pathlib import Path

import pytest
import torch

from forgeserve_b200 import ModelConfig, PipelineStage, PipelineState, pipeline_forward
from forgeserve_b200.tensor_parallel import run_distributed
from oracle import forge_oracle as O

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"


def load_small():
    g = torch.load(GOLDEN / "small.pt", weights_only=False)
    sd = O.test_model_weights(O.Cfg(**g["cfg"]), *g["weights"][1:])
    return g, sd


def pieces_split_head_worker(rank, size, cfg_dict, batch, t, microbatches, pieces):
    from forgeserve_b200 import _lib
    from forgeserve_b200.weights import init_stage_
    cfg = ModelConfig(**cfg_dict)
    stage = PipelineStage(cfg, rank, size, dtype=torch.bfloat16).eval()
    init_stage_(stage, seed=17, std=0.05)
    idx = torch.randint(0, cfg.vocab_size, (batch, t), generator=torch.Generator().manual_seed(4))

    def run(n):
        out = pipeline_forward(stage, PipelineState(stage, batch, microbatches), idx if rank == 0 else None, t,
                               seq_chunks=n)
        return None if out is None else out.cpu()

    whole = run(1)
    stage.split_head_()
    return whole, run(1), run(pieces), _lib.device_error(clear=True)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("microbatches,pieces", [(1, 3), (3, 2)])
def test_nccl_sequence_pieces_with_split_head(microbatches, pieces):
    """Two stages over NCCL with the split head: sequence pieces (more items in split_head_program's order, each
    head slice copied row by row into the last stage's logits) give the logits of whole micro-batches, bit for
    bit."""
    cfg = dict(vocab_size=1000, d_model=256, n_layers=4, n_heads=4, n_kv_heads=2, max_seq_len=512)
    res = run_distributed(pieces_split_head_worker, 2, cfg, 6, 384, microbatches, pieces, backend="nccl",
                          timeout=300)
    assert res[0][:3] == (None, None, None)
    whole, split, split_pieces, err = res[1]
    assert torch.equal(whole, split) and torch.equal(whole, split_pieces)
    assert err == 0 and res[0][3] == 0


def grid_worker(rank, size, cfg_dict, full_sd, idx, more, stages):
    from forgeserve_b200 import _lib
    from forgeserve_b200.transport import make_grid
    cfg = ModelConfig(**cfg_dict)
    stage_idx, tp, transport = make_grid(stages, size // stages)
    stage = PipelineStage(cfg, stage_idx, stages, tp=tp, transport=transport).eval()
    stage.load_from_full(full_sd)
    state = PipelineState(stage, idx.shape[0], 2)
    first = pipeline_forward(stage, state, idx if stage.is_first else None, idx.shape[1])
    cont = pipeline_forward(stage, state, more if stage.is_first else None, more.shape[1])
    return (None if first is None else first.cpu()), (None if cont is None else cont.cpu()), \
        _lib.device_error(clear=True)


@pytest.mark.skipif(torch.cuda.device_count() < 4, reason="needs 4 GPUs")
def test_nccl_tensor_parallel_stages_match_reference():
    """A 2 x 2 grid over NCCL (two stages, each split over two shards; transport.make_grid): the last stage's
    shards return the reference's logits (fp32, 1e-4), continued through the shards' caches."""
    g, sd = load_small()
    res = run_distributed(grid_worker, 4, g["cfg"], sd, g["idx"], g["more"], 2, backend="nccl", timeout=300)
    for rank, (first, cont, err) in enumerate(res):
        assert err == 0
        if rank >= 2:
            torch.testing.assert_close(first, g["logits"], atol=1e-4, rtol=1e-4)
            torch.testing.assert_close(cont, g["logits_more"], atol=1e-4, rtol=1e-4)
        else:
            assert first is None and cont is None


def prefill_pieces_worker(rank, size, cfg_dict, sd, requests, num_blocks, max_batch, pieces):
    from forgeserve_b200 import PipelineEngine, PipelineStage, _lib
    cfg = ModelConfig(**cfg_dict)
    res = []
    for n in (1, pieces):
        stage = PipelineStage(cfg, rank, size)
        stage.load_from_full(sd)
        stage = stage.to(torch.bfloat16).eval()
        eng = PipelineEngine(stage, num_blocks=num_blocks, block_size=16, max_batch=max_batch, microbatches=2,
                             prefill_chunks=n)
        ids = [eng.add_request(p, k) for p, k in requests]
        out = eng.run()
        res.append(([out[i] for i in ids], eng.steps, eng.preemptions))
    return res, _lib.device_error(clear=True)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_nccl_pipeline_engine_prefill_pieces_match_whole_prefills():
    """PipelineEngine over NCCL ranks with each prefill's prompt in pieces (every piece's GEMMs above 128 rows, the
    attention rows independent): the same tokens and counters as whole prefills, in bf16 at head_dim 128."""
    cfg = ModelConfig(vocab_size=512, d_model=512, n_layers=4, n_heads=4, n_kv_heads=2, max_seq_len=1024)
    sd = O.test_model_weights(O.Cfg(**cfg.to_dict()), seed=11, scale=0.05)
    gen = torch.Generator().manual_seed(7)
    requests = [(torch.randint(0, 512, (n,), generator=gen).tolist(), k) for n, k in ((700, 12), (300, 20), (520, 9))]
    res = run_distributed(prefill_pieces_worker, 2, cfg.to_dict(), sd, requests, 160, 3, 4, backend="nccl",
                          timeout=300)
    for (whole, pieces), err in res:
        assert err == 0
        assert pieces == whole
    assert len({t for out in res[0][0][0][0] for t in out}) > 5
