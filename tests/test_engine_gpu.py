"""The serving engine on the GPU against the reference engine's outputs (tests/golden/small.pt)."""

from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

from forgeserve_b200 import Engine, ForgeModel, ModelConfig, generate
from oracle import forge_oracle as O

GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(autouse=True)
def _no_device_errors():
    from forgeserve_b200 import _lib
    _lib.device_error(clear=True)
    yield
    assert _lib.device_error(clear=True) == 0, "a kernel flagged bad input or a wait timeout"


@pytest.fixture(scope="module")
def setup():
    g = torch.load(GOLDEN / "small.pt", weights_only=False)
    cfg = ModelConfig(**g["cfg"])
    m = ForgeModel(cfg, device="cuda")
    m.load_state_dict(O.test_model_weights(O.Cfg(**g["cfg"]), *g["weights"][1:]))
    return g, m.eval()


@pytest.mark.parametrize("key,num_blocks,max_batch", [("engine", 64, 3), ("engine_preempt", 12, 5)])
def test_engine_outputs_equal_reference_engine(setup, key, num_blocks, max_batch):
    g, m = setup
    e = g[key]
    eng = Engine(m, num_blocks=num_blocks, block_size=4, max_batch=max_batch)
    ids = [eng.add_request(p, n) for p, n in e["requests"]]
    out = eng.run()
    assert [out[i] for i in ids] == e["outputs"]
    assert eng.steps == e["steps"] and eng.preemptions == e["preemptions"]
    assert eng.pool.allocator.num_free == num_blocks


def test_engine_eos_and_temperature(setup):
    g, m = setup
    full = generate(m, torch.tensor([[3, 1, 4, 1, 5]]), 10)[0, 5:].tolist()
    eos = full[3]
    eng = Engine(m, num_blocks=32, block_size=4)
    rid = eng.add_request([3, 1, 4, 1, 5], 10, eos_id=eos)
    assert eng.run()[rid] == full[: full.index(eos) + 1]

    def run(seed):
        e = Engine(m, num_blocks=32, block_size=4, seed=seed)
        rid = e.add_request([1, 2, 3], 10, temperature=1.0)
        return e.run()[rid]
    a, b, c = run(0), run(0), run(1)
    assert a == b and len(a) == 10 and all(0 <= t < 64 for t in a) and a != c


def test_engine_bf16_matches_own_generate():
    """bf16 model: engine (paged cache, batched decode) and plain generation give the same greedy tokens."""
    cfg = ModelConfig(vocab_size=512, d_model=256, n_layers=2, n_heads=4, n_kv_heads=2, max_seq_len=256)
    torch.manual_seed(0)
    m = ForgeModel(cfg, device="cuda").to(torch.bfloat16).eval()
    g = torch.Generator().manual_seed(3)
    for p in m.parameters():
        if p.ndim >= 2:
            p.data.copy_((torch.randn(p.shape, generator=g) * 0.1).to(p.device, p.dtype))
    prompts = [torch.randint(0, 512, (n,), generator=g).tolist() for n in (5, 40, 17)]
    eng = Engine(m, num_blocks=64, block_size=16, max_batch=3)
    ids = [eng.add_request(p, 12) for p in prompts]
    out = eng.run()
    for rid, p in zip(ids, prompts):
        want = generate(m, torch.tensor([p]), 12)[0, len(p):].tolist()
        agree = sum(a == b for a, b in zip(out[rid], want))
        assert agree >= 10, (out[rid], want)       # bf16: paged/batched and contiguous paths may flip a near-tie
