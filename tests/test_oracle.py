"""Pin the oracle (oracle/forge_oracle.py) to outputs of the reference forgeserve (tests/golden/*.pt)."""

from pathlib import Path

import pytest
import torch

from oracle import forge_oracle as O

GOLDEN = Path(__file__).resolve().parent / "golden"


def load(name):
    return torch.load(GOLDEN / name, weights_only=False)


@pytest.fixture(scope="module")
def small():
    g = load("small.pt")
    cfg = O.Cfg(**g["cfg"])
    sd = O.test_model_weights(cfg, *g["weights"][1:])
    return g, cfg, sd


@pytest.fixture(scope="module")
def c1():
    g = load("c1.pt")
    cfg = O.Cfg(**g["cfg"])
    sd = O.test_model_weights(cfg, *g["weights"][1:])
    return g, cfg, sd


def close(a, b, tol=1e-5):
    torch.testing.assert_close(a, b, atol=tol, rtol=tol)


def test_weight_recipes_match_the_reference_models(small, c1):
    for g, _, sd in (small, c1):
        want = g["checksum"]
        got = O.checksum(sd)
        assert set(got) == set(want)
        for k in want:
            assert got[k] == pytest.approx(want[k], rel=1e-12, abs=1e-9), k


def test_forward(small):
    g, cfg, sd = small
    close(O.model_forward(sd, cfg, g["idx"]), g["logits"])
    close(O.model_forward(sd, cfg, torch.cat([g["idx"], g["more"]], 1))[:, 9:], g["logits_more"])


def test_one_token_cache_steps(small):
    g, cfg, sd = small
    kv = [O.ContiguousCache() for _ in range(cfg.n_layers)]
    steps = torch.cat([O.model_forward(sd, cfg, g["steps_idx"][:, i : i + 1], kv=kv) for i in range(20)], dim=1)
    close(steps, g["steps_logits"])


def test_explicit_positions(small):
    g, cfg, sd = small
    close(O.model_forward(sd, cfg, g["idx"][:1, :5], positions=torch.arange(5)[None] + 11), g["shifted_logits"])


@pytest.mark.parametrize("size,mbs", [(2, 1), (3, 2), (3, 4)])
def test_pipeline_schedule(small, size, mbs):
    g, cfg, sd = small
    sim = O.PipelineSim(cfg, 4, size, mbs)
    logits = O.pipeline_forward(sd, sim, g["idx"], 9)
    logits2 = O.pipeline_forward(sd, sim, g["more"], 3)
    want, want2 = g["pipeline"][(size, mbs)]
    close(logits, want)
    close(logits2, want2)


def test_greedy_generation(small):
    g, cfg, sd = small
    out = O.greedy_generate(sd, cfg, g["prompt"], 10)
    assert torch.equal(out, g["generate"])
    for (size, mbs), toks in g["pipeline_generate"].items():
        assert torch.equal(out, toks), (size, mbs)
    assert len(set(out[:, 5:].flatten().tolist())) > 5        # the fixture model really produces varied tokens


def test_generation_stops_at_max_seq_len(small):
    g, cfg, sd = small
    prompt = g["generate_long"][:, :60]
    out = O.greedy_generate(sd, cfg, prompt, 100)
    assert out.shape[1] == cfg.max_seq_len
    assert torch.equal(out, g["generate_long"])


def test_paged_scatter_gather(small):
    g, cfg, sd = small
    pool = O.PagedPool(cfg, 16, 4)
    table = torch.tensor([g["paged_blocks"]])
    idx = g["paged_idx"]
    pos = torch.arange(12)[None]
    got = [O.model_forward(sd, cfg, idx[:, :12], pos, [pool.view(i, table, pos) for i in range(cfg.n_layers)])]
    for i in range(12, 30):
        pos = torch.tensor([[i]])
        got.append(O.model_forward(sd, cfg, idx[:, i : i + 1], pos, [pool.view(l, table, pos) for l in range(cfg.n_layers)]))
    close(torch.cat(got, 1), g["paged_logits"])


def test_engine_outputs_equal_per_request_generation(small):
    """The reference engine's outputs (with and without preemption) are per-request greedy generations."""
    g, cfg, sd = small
    for key in ("engine", "engine_preempt"):
        e = g[key]
        for (prompt, n), got in zip(e["requests"], e["outputs"]):
            want = O.greedy_generate(sd, cfg, torch.tensor([prompt]), n)[0, len(prompt):].tolist()
            assert got == want
    assert g["engine_preempt"]["preemptions"] > 0


def test_bf16_rounding_points(small):
    g, cfg, sd = small
    r = g["bf16_rmsnorm"]
    assert torch.equal(O.rms_norm(r["x"], r["w"], 1e-5), r["y"])
    q = g["bf16_rope"]
    cos, sin = O.rope_tables(16, 64, 10000.0)
    assert torch.equal(O.apply_rope(q["x"], cos, sin, q["positions"]), q["y"])
    # one bf16 decoder layer: equal up to one bf16 ulp of the output magnitude (SDPA's internal order differs)
    sd16 = {k: v.to(torch.bfloat16) for k, v in sd.items()}
    x0 = sd16["tok_emb.weight"][g["idx"]]
    pos = torch.arange(9)[None].expand(4, 9)
    cos, sin = O.rope_tables(cfg.head_dim, cfg.max_seq_len, cfg.rope_theta)
    got = O.block(sd16, 0, x0, cfg, cos, sin, pos, O.ContiguousCache())
    want = g["bf16_block0"]
    assert (got.float() - want.float()).abs().max() <= 2 ** -7 * want.float().abs().max()


def test_bf16_model_within_tolerance(c1):
    """bf16 mode tolerance (2e-2 max-abs after log-softmax) at the reference's init scale."""
    g, cfg, sd = c1
    sd16 = {k: v.to(torch.bfloat16) for k, v in sd.items()}
    assert O.log_softmax_maxabs(O.model_forward(sd16, cfg, g["idx"]), g["bf16_logits"]) < 2e-2


def test_empty_microbatches_are_an_error_in_the_reference(small):
    assert small[0]["empty_microbatch_raises"]


def test_config1_pipeline(c1):
    g, cfg, sd = c1
    close(O.model_forward(sd, cfg, g["idx"]), g["logits"])
    sim = O.PipelineSim(cfg, 8, 2, 4)
    close(O.pipeline_forward(sd, sim, g["idx"], 16), g["pipeline_logits"])
    close(O.pipeline_forward(sd, sim, g["idx"][:, :3], 3), g["pipeline_logits2"])
    assert torch.equal(O.greedy_generate(sd, cfg, g["prompt"], 8), g["generate"])
    assert torch.equal(g["generate"], g["pipeline_generate"])


def test_known_answers_from_the_reference_tests():
    assert O.stage_layers(3, 3) == [(0, 1), (1, 2), (2, 3)]
    assert O.stage_layers(7, 3) == [(0, 3), (3, 5), (5, 7)]
    with pytest.raises(ValueError):
        O.stage_layers(2, 3)
    assert O.microbatch_sizes(2, 4) == [1, 1, 0, 0]
    assert O.microbatch_sizes(8, 4) == [2, 2, 2, 2]


@pytest.mark.parametrize("size", [2, 4])
def test_tensor_parallel_restatement(size):
    """The oracle's tensor-parallel forward (shards' partial outputs summed at the two all-reduce points) against
    the reference's own tensor parallelism over gloo: forward and a chunk continued through the shards' caches."""
    g = load("tp.pt")
    cfg = O.Cfg(**g["cfg"])
    sd = O.test_model_weights(cfg, *g["weights"][1:])
    assert O.checksum(sd) == g["checksum"]
    shards = [O.shard(sd, r, size) for r in range(size)]
    kvs = [[O.ContiguousCache() for _ in range(cfg.n_layers)] for _ in range(size)]
    close(O.model_forward_tp(shards, cfg, g["idx"], kvs), g["tp"][size]["logits"], tol=5e-5)
    close(O.model_forward_tp(shards, cfg, g["more"], kvs), g["tp"][size]["logits_more"], tol=5e-5)
    assert g["tp"][size]["all_reduces"] == 2 * 2 * cfg.n_layers      # two forwards, two per layer
    # the reference's shards give the single-process model's tokens
    assert torch.equal(g["tp"][size]["generate"], O.greedy_generate(sd, cfg, g["prompt"], 10))


def test_reference_attention_call_matches_the_written_out_one_in_fp32():
    """oracle.sdpa_torch (the reference's own scaled_dot_product_attention call, model.py:76) and the written-out
    softmax give the reference's golden logits alike in fp32."""
    g = torch.load(GOLDEN / "small.pt", weights_only=False)
    cfg = O.Cfg(**g["cfg"])
    sd = O.test_model_weights(cfg, *g["weights"][1:])
    got = O.model_forward(sd, cfg, g["idx"], attn_core=O.sdpa_torch)
    torch.testing.assert_close(got, g["logits"], atol=1e-4, rtol=1e-4)
    assert torch.equal(O.greedy_generate(sd, cfg, g["prompt"], 10, attn_core=O.sdpa_torch), g["generate"])


def test_pp8_fixture_weights_and_outputs():
    """The multi-GPU bench's parity fixture: the product's restatement of the test suite's weight recipe gives the
    recorded checksums, and the oracle reproduces the reference's fp32 logits and greedy tokens."""
    from forgeserve_b200 import ModelConfig
    from forgeserve_b200.weights import checksum, test_suite_state_dict
    g = torch.load(GOLDEN / "pp8.pt", weights_only=False)
    cfg = O.Cfg(**g["cfg"])
    sd = test_suite_state_dict(ModelConfig(**g["cfg"]), *g["weights"][1:])
    assert checksum(sd) == g["checksum"]
    assert checksum(test_suite_state_dict(ModelConfig(**g["cfg"]), *g["bf16_weights"][1:])) == g["bf16_checksum"]
    for k, v in O.test_model_weights(cfg, *g["weights"][1:]).items():
        assert torch.equal(v, sd[k]), k
    got = O.model_forward(sd, cfg, g["idx"])[:, g["positions"]]
    torch.testing.assert_close(got, g["logits"], atol=1e-4, rtol=1e-4)
    assert torch.equal(O.greedy_generate(sd, cfg, g["prompt"], 16), g["generate"])
    assert 0 < g["bf16_spread"] < 0.05
