"""forgeserve_b200's decoder on the GPU against the reference's outputs (tests/golden) and the oracle.

fp32 mode: logits within 1e-4 and identical greedy tokens. bf16 mode: within 2e-2 max-abs after log-softmax
(the tolerance of the bf16 mode), rounding points bit-exact."""

from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

from forgeserve_b200 import ForgeModel, ModelConfig, PagedKVPool, generate, new_contiguous_cache, ops
from forgeserve_b200 import _lib as L
from oracle import forge_oracle as O

GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(autouse=True)
def _no_device_errors():
    from forgeserve_b200 import _lib
    _lib.device_error(clear=True)
    yield
    assert _lib.device_error(clear=True) == 0, "a kernel flagged bad input or a wait timeout"


DEV = "cuda"


def golden(name):
    g = torch.load(GOLDEN / name, weights_only=False)
    cfg = ModelConfig(**g["cfg"])
    sd = O.test_model_weights(O.Cfg(**g["cfg"]), *g["weights"][1:])
    return g, cfg, sd


def model_from(cfg, sd, dtype=torch.float32):
    m = ForgeModel(cfg, device=DEV)
    m.load_state_dict(sd)
    return m.to(dtype).eval()


@pytest.fixture(scope="module")
def small():
    g, cfg, sd = golden("small.pt")
    return g, cfg, sd, model_from(cfg, sd)


def close(a, b, tol=1e-4):
    torch.testing.assert_close(a.float().cpu(), b.float().cpu(), atol=tol, rtol=tol)


def test_forward_and_continued_chunk(small):
    g, cfg, sd, m = small
    close(m(g["idx"]), g["logits"])
    kv = new_contiguous_cache(cfg.n_layers)
    m(g["idx"], kv=kv)
    close(m(g["more"], kv=kv), g["logits_more"])


def test_one_token_cache_steps(small):
    g, cfg, sd, m = small
    kv = new_contiguous_cache(cfg.n_layers)
    steps = torch.cat([m(g["steps_idx"][:, i : i + 1], kv=kv) for i in range(20)], dim=1)
    close(steps, g["steps_logits"])


def test_explicit_positions_and_no_future_leakage(small):
    g, cfg, sd, m = small
    close(m(g["idx"][:1, :5], positions=torch.arange(5)[None] + 11), g["shifted_logits"])
    a = g["idx"][:1]
    b = a.clone()
    b[0, 6:] = (b[0, 6:] + 1) % 64
    la, lb = m(a), m(b)
    close(la[:, :6], lb[:, :6], 1e-5)
    assert not torch.allclose(la[:, 6:], lb[:, 6:])


def test_rows_at_different_positions(small):
    """One step with rows at their own positions, each continuing its own cached prefix (model.py:140-159)."""
    g, cfg, sd, m = small
    a, b = g["steps_idx"][:1, :7], g["steps_idx"][1:, :3]
    want_a, want_b = m(a)[:, -1], m(b)[:, -1]
    kv_a, kv_b = new_contiguous_cache(3), new_contiguous_cache(3)
    m(a[:, :-1], kv=kv_a)
    m(b[:, :-1], kv=kv_b)
    close(m(a[:, -1:], kv=kv_a)[:, -1], want_a)
    close(m(b[:, -1:], kv=kv_b)[:, -1], want_b)


def test_greedy_generation_and_length_limit(small):
    g, cfg, sd, m = small
    assert torch.equal(generate(m, g["prompt"], 10), g["generate"])
    assert torch.equal(generate(m, g["generate_long"][:, :60], 100), g["generate_long"])
    with pytest.raises(ValueError):
        m(torch.randint(0, 64, (1, 65)))


def test_paged_views_match_reference(small):
    g, cfg, sd, m = small
    pool = PagedKVPool(cfg, num_blocks=16, block_size=4, dtype=torch.float32, device=DEV)
    table = torch.tensor([g["paged_blocks"]])
    idx = g["paged_idx"]
    got = [m(idx[:, :12], torch.arange(12)[None], pool.views(table, torch.arange(12)[None]))]
    for i in range(12, 30):
        pos = torch.tensor([[i]])
        got.append(m(idx[:, i : i + 1], pos, pool.views(table, pos)))
    close(torch.cat(got, 1), g["paged_logits"])


def test_paged_view_protocol_update(small):
    """PagedLayerView.update stores at the table slots and returns the rows' blocks in table order."""
    g, cfg, sd, m = small
    pool = PagedKVPool(cfg, num_blocks=10, block_size=4, device=DEV)
    table = torch.tensor([[7, 2, 9]])
    k = torch.randn(1, cfg.n_kv_heads, 10, cfg.head_dim, device=DEV)
    v = torch.randn_like(k)
    k_all, v_all = pool.views(table, torch.arange(10)[None])[0].update(k, v)
    assert k_all.shape == (1, cfg.n_kv_heads, 12, cfg.head_dim)
    close(k_all[:, :, :10], k, 0)
    close(v_all[:, :, :10], v, 0)
    close(pool.k[0][2, :, 1], k[0, :, 5], 0)


def test_foreign_view_protocol(small):
    """Any object with update(k, v) works as a cache view (the reference's KV view protocol)."""
    g, cfg, sd, m = small

    class CatCache:
        def __init__(self):
            self.k = self.v = None

        @property
        def length(self):
            return 0 if self.k is None else self.k.shape[2]

        def update(self, k, v):
            self.k = k if self.k is None else torch.cat([self.k, k], 2)
            self.v = v if self.v is None else torch.cat([self.v, v], 2)
            return self.k, self.v

    kv = [CatCache() for _ in range(cfg.n_layers)]
    m(g["idx"], kv=kv)
    close(m(g["more"], kv=kv), g["logits_more"])


def test_config1_fp32(tmp_path):
    g, cfg, sd = golden("c1.pt")
    m = model_from(cfg, sd)
    close(m(g["idx"]), g["logits"])
    assert torch.equal(generate(m, g["prompt"], 8), g["generate"])


def test_config1_bf16_tolerance():
    g, cfg, sd = golden("c1.pt")
    m = model_from(cfg, sd, torch.bfloat16)
    got = m(g["idx"]).cpu()
    assert O.log_softmax_maxabs(got, g["bf16_logits"]) < 2e-2         # vs the reference in bf16
    assert O.log_softmax_maxabs(got, g["logits"]) < 2e-2              # vs the reference in fp32


def test_bf16_rounding_points_bit_exact():
    g, _, _ = golden("small.pt")
    r = g["bf16_rmsnorm"]
    got = ops.rmsnorm(r["x"].to(DEV), r["w"].to(DEV), 1e-5).cpu()
    assert torch.equal(got, r["y"])
    q = g["bf16_rope"]
    x, pos = q["x"], q["positions"]                                    # (2, 4, 7, 16)
    B, H, T, D = x.shape
    cos, sin = O.rope_tables(16, 64, 10000.0)
    # through the RoPE+KV kernel: put x in the q slot of a qkv buffer (H query heads, 1 KV head)
    qkv = torch.zeros(B * T, (H + 2) * D, dtype=torch.bfloat16, device=DEV)
    qkv[:, : H * D] = x.transpose(1, 2).reshape(B * T, H * D).to(DEV)
    kc = torch.zeros(B, 1, 64, D, dtype=torch.bfloat16, device=DEV)
    desc = ops.contiguous_desc(kc, kc.clone(), torch.arange(B, device=DEV))
    ops.rope_kv_write(qkv, cos.to(DEV), sin.to(DEV), pos.to(DEV), desc, B, T, H, 1, D, slot_base=0,
                      slot_from_pos=False)
    got = qkv[:, : H * D].view(B, T, H, D).transpose(1, 2).cpu()
    assert torch.equal(got, q["y"])


def test_no_device_errors_after_model_runs(small):
    g, cfg, sd, m = small
    m(g["idx"])
    assert L.device_error(clear=True) == 0
