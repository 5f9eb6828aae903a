"""Tensor parallelism on the GPU: ForgeModel shards (TPContext(rank, size), shard_state_dict) against the
reference's own tensor-parallel run (tests/golden/tp.pt, forgeserve/model.py:47-106 with parallel.py and
tensor_parallel.py) in fp32: logits within 1e-4 for a forward and a chunk continued through the shards' caches,
the all-reduce count, greedy tokens, and the Engine's outputs and counters over 2 shards.

The shards run as processes: over NCCL with one GPU each when the machine has enough GPUs, else over gloo with
every shard on the one GPU (the all-reduce then goes through host memory; no kernel waits on another process)."""

from pathlib import Path

import pytest
import torch

from forgeserve_b200.tensor_parallel import run_distributed
from oracle import forge_oracle as O

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"


def _model(rank, size, cfg_dict, full_sd):
    from forgeserve_b200 import ForgeModel, ModelConfig, TPContext
    from forgeserve_b200.tensor_parallel import shard_state_dict
    cfg = ModelConfig(**cfg_dict)
    tp = TPContext(rank, size)
    m = ForgeModel(cfg, tp)
    m.load_state_dict(shard_state_dict(full_sd, cfg, rank, size))
    return m.to("cuda").eval(), tp


def tp_worker(rank, size, cfg_dict, full_sd, idx, more, prompt):
    from forgeserve_b200 import _lib, generate, new_contiguous_cache
    m, tp = _model(rank, size, cfg_dict, full_sd)
    kv = new_contiguous_cache(m.cfg.n_layers, m.cfg.max_seq_len)
    first = m(idx, kv=kv).cpu()
    cont = m(more, kv=kv).cpu()
    n_all_reduces = tp.num_all_reduces
    return first, cont, n_all_reduces, generate(m, prompt, 10).cpu(), _lib.device_error(clear=True)


def tp_engine_worker(rank, size, cfg_dict, full_sd, requests, num_blocks, max_batch):
    from forgeserve_b200 import Engine, _lib
    m, _ = _model(rank, size, cfg_dict, full_sd)
    eng = Engine(m, num_blocks=num_blocks, block_size=4, max_batch=max_batch)
    ids = [eng.add_request(p, n) for p, n in requests]
    out = eng.run()
    return ([out[i] for i in ids], eng.steps, eng.preemptions, tuple(eng.pool.k[0].shape),
            _lib.device_error(clear=True))


@pytest.fixture(scope="module")
def golden():
    g = torch.load(GOLDEN / "tp.pt", weights_only=False)
    cfg = O.Cfg(**g["cfg"])
    sd = O.test_model_weights(cfg, *g["weights"][1:])
    assert O.checksum(sd) == g["checksum"]
    return g, sd


@pytest.mark.parametrize("size", [2, 4])
def test_tensor_parallel_shards_match_the_reference(golden, size):
    g, sd = golden
    want = g["tp"][size]
    res = run_distributed(tp_worker, size, g["cfg"], sd, g["idx"], g["more"], g["prompt"], timeout=300)
    for first, cont, n_all_reduces, gen, err in res:
        torch.testing.assert_close(first, want["logits"], atol=1e-4, rtol=1e-4)
        torch.testing.assert_close(cont, want["logits_more"], atol=1e-4, rtol=1e-4)
        assert n_all_reduces == want["all_reduces"]
        assert torch.equal(gen, want["generate"])
        assert err == 0


def test_engine_under_tensor_parallelism_matches_the_reference(golden):
    """Every shard runs the same Engine; the pool holds the shard's KV heads; the small pool preempts."""
    g, sd = golden
    e = g["tp_engine"]
    res = run_distributed(tp_engine_worker, 2, g["cfg"], sd, e["requests"], e["num_blocks"], e["max_batch"],
                          timeout=300)
    for outputs, steps, preemptions, pool_shape, err in res:
        assert outputs == e["outputs"]
        assert (steps, preemptions, pool_shape) == (e["steps"], e["preemptions"], e["pool_shape"])
        assert err == 0
    assert e["preemptions"] > 0
