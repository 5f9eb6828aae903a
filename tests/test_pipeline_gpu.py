"""forgeserve_b200's pipeline on the GPU: stages as threads on one GPU (run_in_threads), NCCL ranks when the
box has several GPUs, and a full-size 8B-shape decoder layer against the oracle."""

from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

from forgeserve_b200 import ModelConfig, PipelineStage, PipelineState, pipeline_forward, pipeline_generate
from forgeserve_b200.tensor_parallel import run_distributed, run_in_threads
from oracle import forge_oracle as O

GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(autouse=True)
def _no_device_errors():
    from forgeserve_b200 import _lib
    _lib.device_error(clear=True)
    yield
    assert _lib.device_error(clear=True) == 0, "a kernel flagged bad input or a wait timeout"


def load_small():
    g = torch.load(GOLDEN / "small.pt", weights_only=False)
    sd = O.test_model_weights(O.Cfg(**g["cfg"]), *g["weights"][1:])
    return g, sd


def forward_worker(rank, size, cfg_dict, full_sd, idx, more, microbatches):
    cfg = ModelConfig(**cfg_dict)
    stage = PipelineStage(cfg, rank, size).eval()
    stage.load_from_full(full_sd)
    state = PipelineState(stage, idx.shape[0], microbatches)
    logits = pipeline_forward(stage, state, idx if rank == 0 else None, idx.shape[1])
    logits2 = pipeline_forward(stage, state, more if rank == 0 else None, more.shape[1])
    n = sum(p.numel() for p in stage.layers.parameters())
    return (None if logits is None else logits.cpu()), (None if logits2 is None else logits2.cpu()), n


def generate_worker(rank, size, cfg_dict, full_sd, prompt, microbatches, n):
    cfg = ModelConfig(**cfg_dict)
    stage = PipelineStage(cfg, rank, size).eval()
    stage.load_from_full(full_sd)
    return pipeline_generate(stage, prompt, n, microbatches).cpu()


@pytest.mark.parametrize("size,microbatches", [(2, 1), (3, 2), (3, 4)])
def test_threaded_stages_match_reference_pipeline(size, microbatches):
    g, sd = load_small()
    res = run_in_threads(forward_worker, size, g["cfg"], sd, g["idx"], g["more"], microbatches)
    want, want2 = g["pipeline"][(size, microbatches)]
    torch.testing.assert_close(res[-1][0], want, atol=1e-4, rtol=1e-4)
    torch.testing.assert_close(res[-1][1], want2, atol=1e-4, rtol=1e-4)
    assert all(r[0] is None for r in res[:-1])
    assert sum(r[2] for r in res) == sum(v.numel() for k, v in sd.items() if k.startswith("layers."))


@pytest.mark.parametrize("size,microbatches", [(2, 1), (3, 2)])
def test_threaded_generation_matches_reference(size, microbatches):
    g, sd = load_small()
    res = run_in_threads(generate_worker, size, g["cfg"], sd, g["prompt"], microbatches, 10)
    for out in res:
        assert torch.equal(out, g["generate"])


def test_config1_two_stages_four_microbatches():
    g = torch.load(GOLDEN / "c1.pt", weights_only=False)
    sd = O.test_model_weights(O.Cfg(**g["cfg"]), *g["weights"][1:])
    res = run_in_threads(forward_worker, 2, g["cfg"], sd, g["idx"], g["idx"][:, :3].clone(), 4)
    torch.testing.assert_close(res[-1][0], g["pipeline_logits"], atol=1e-4, rtol=1e-4)
    torch.testing.assert_close(res[-1][1], g["pipeline_logits2"], atol=1e-4, rtol=1e-4)
    gen = run_in_threads(generate_worker, 2, g["cfg"], sd, g["prompt"], 4, 8)
    assert torch.equal(gen[0], g["pipeline_generate"])


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_nccl_two_gpu_pipeline_matches_reference():
    g, sd = load_small()
    res = run_distributed(forward_worker, 2, g["cfg"], sd, g["idx"], g["more"], 2, backend="nccl", timeout=300)
    want, want2 = g["pipeline"][(2, 1)]
    torch.testing.assert_close(res[-1][0], want, atol=1e-4, rtol=1e-4)
    torch.testing.assert_close(res[-1][1], want2, atol=1e-4, rtol=1e-4)
    gen = run_distributed(generate_worker, 2, g["cfg"], sd, g["prompt"], 2, 10, backend="nccl", timeout=300)
    for out in gen:
        assert torch.equal(out, g["generate"])


def split_head_worker(rank, size, cfg_dict, batch, t, microbatches, transfer):
    from forgeserve_b200 import _lib
    from forgeserve_b200.weights import init_stage_
    cfg = ModelConfig(**cfg_dict)
    stage = PipelineStage(cfg, rank, size, dtype=torch.bfloat16).eval()
    init_stage_(stage, seed=11, std=0.05)
    idx = torch.randint(0, cfg.vocab_size, (batch, t), generator=torch.Generator().manual_seed(3))

    def run():
        state = PipelineState(stage, batch, microbatches)
        out = pipeline_forward(stage, state, idx if rank == 0 else None, t)
        return None if out is None else out.cpu()

    whole = run()
    stage.split_head_(transfer)
    split, again = run(), run()   # the second call reuses the mapping of the last stage's logits
    return whole, split, again, _lib.device_error(clear=True)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("microbatches,transfer", [(1, "copy"), (3, "copy"), (3, "store")])
def test_nccl_split_head_matches_whole_head(microbatches, transfer):
    """Head slices computed on every stage and moved into the last stage's logits over NVLink (by the copy
    engine, or stored by the GEMM epilogue) give the same logits, bit for bit, as the whole head on the last
    stage (ragged last slice: vocab 1000 = 3 x 256 + 232)."""
    cfg = dict(vocab_size=1000, d_model=256, n_layers=4, n_heads=4, n_kv_heads=2, max_seq_len=128)
    res = run_distributed(split_head_worker, 2, cfg, 6, 64, microbatches, transfer, backend="nccl", timeout=300)
    assert res[0][:3] == (None, None, None)
    whole, split, again, err = res[1]
    assert whole.shape == (6, 64, 1000) and torch.isfinite(whole.float()).all()
    assert torch.equal(whole, split) and torch.equal(whole, again)
    assert err == 0 and res[0][3] == 0


def test_sequence_pieces_are_bit_identical_on_one_gpu():
    """bf16, head_dim 128: micro-batches pushed through in 4 pieces of 256 tokens give exactly the logits of whole
    micro-batches (every kernel treats rows independently; every GEMM has more than 128 rows either way, so the
    same 2-SM kernel runs), for all positions, continued through the caches, and with last_only."""
    from forgeserve_b200 import _lib
    from forgeserve_b200.weights import init_stage_
    cfg = ModelConfig(vocab_size=1000, d_model=512, n_layers=2, n_heads=4, n_kv_heads=2, max_seq_len=2048)
    stage = PipelineStage(cfg, 0, 1, dtype=torch.bfloat16).eval()
    init_stage_(stage, seed=13, std=0.05)
    g = torch.Generator().manual_seed(2)
    idx = torch.randint(0, 1000, (6, 1024), generator=g)
    more = torch.randint(0, 1000, (6, 1024), generator=g)

    def run(pieces):
        state = PipelineState(stage, 6, 2)
        a = pipeline_forward(stage, state, idx, 1024, seq_chunks=pieces)
        b = pipeline_forward(stage, state, more, 1024, seq_chunks=pieces)
        c = pipeline_forward(stage, PipelineState(stage, 6, 2), idx, 1024, last_only=True, seq_chunks=pieces)
        return a, b, c

    whole, pieces = run(1), run(4)
    for x, y in zip(whole, pieces):
        assert torch.isfinite(x.float()).all() and torch.equal(x, y)
    assert _lib.device_error(clear=True) == 0


def overlap_worker(rank, size, cfg_dict, prompt, n, microbatches):
    from forgeserve_b200 import _lib
    from forgeserve_b200.weights import init_stage_
    cfg = ModelConfig(**cfg_dict)
    stage = PipelineStage(cfg, rank, size, dtype=torch.bfloat16).eval()
    init_stage_(stage, seed=5, std=0.08)
    plain = pipeline_generate(stage, prompt, n, microbatches, overlap=False).cpu()
    ring = pipeline_generate(stage, prompt, n, microbatches, overlap=True).cpu()
    auto = pipeline_generate(stage, prompt, n, microbatches).cpu()     # picks the overlapped path
    return plain, ring, auto, _lib.device_error(clear=True)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("microbatches", [2, 3])
def test_nccl_overlapped_generation_matches_step_by_step(microbatches):
    """Greedy generation with the token ring (no pipeline drain per token) gives the same tokens on every stage as
    the step-by-step loop (pipeline.py:121-137)."""
    cfg = dict(vocab_size=1000, d_model=256, n_layers=4, n_heads=4, n_kv_heads=2, max_seq_len=128)
    prompt = torch.randint(0, 1000, (6, 11), generator=torch.Generator().manual_seed(8))
    res = run_distributed(overlap_worker, 2, cfg, prompt, 9, microbatches, backend="nccl", timeout=300)
    for plain, ring, auto, err in res:
        assert plain.shape == (6, 20) and torch.equal(plain[:, :11], prompt)
        assert torch.equal(plain, ring) and torch.equal(plain, auto)
        assert err == 0
    assert torch.equal(res[0][0], res[1][0])
    assert len(set(res[0][0][:, 11:].flatten().tolist())) > 3          # tokens vary


def test_8b_shape_layer_bf16_against_oracle():
    """One 8B-shape decoder layer (d 4096, 32/8 heads, ffn 14336, theta 5e5) at B=1, T=1024 in bf16, against the
    oracle's fp32 layer on the same bf16 weights (run on the GPU with plain torch as the checker)."""
    from forgeserve_b200.weights import layer_shapes, seeded_state_dict
    cfg = ModelConfig(vocab_size=128256, d_model=4096, n_layers=1, n_heads=32, n_kv_heads=8, ffn_dim=14336,
                      max_seq_len=2048, rope_theta=500000.0)
    names = list(layer_shapes(cfg, 0))
    sd = seeded_state_dict(cfg, seed=5, std=0.02, names=names, device="cuda", dtype=torch.bfloat16)
    stage = PipelineStage(cfg, 0, 1, dtype=torch.bfloat16)
    stage.layers[0].load_state_dict({k.replace("layers.0.", ""): v for k, v in sd.items()})
    x = torch.randn(1, 1024, 4096, device="cuda").bfloat16()
    pos = torch.arange(1024, device="cuda")[None]
    from forgeserve_b200.kv import ContiguousKV
    got = stage.run_layers(x, pos, [ContiguousKV()]).float()
    ocfg = O.Cfg(**cfg.to_dict())
    cos, sin = O.rope_tables(ocfg.head_dim, ocfg.max_seq_len, ocfg.rope_theta)
    sd32 = {k: v.float() for k, v in sd.items()}
    want = O.block(sd32, 0, x.float(), ocfg, cos.cuda(), sin.cuda(), pos, O.ContiguousCache())
    err = (got - want).abs().max().item()
    assert err < 0.05 * want.abs().max().item(), err
    rel = ((got - want).norm() / want.norm()).item()
    assert rel < 1e-2, rel
