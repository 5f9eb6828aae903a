"""Full-depth parity on the benchmarked model: the 32-layer 8B-shape decoder of BASELINE config 3 (d_model 4096,
32 query / 8 KV heads of head_dim 128, ffn 14336, vocab 128256, RoPE theta 5e5) in bf16, with the bench's seeded
N(0, 0.02) weights (forgeserve_b200.weights, seed 1234), against the oracle run with plain torch on the same GPU
and the same weights.

The references, all on the same bf16 weights:
  r16  the reference's module in bf16: the oracle with the reference's own scaled_dot_product_attention call
       (forgeserve/model.py:76) in bf16 (oracle.sdpa_torch);
  o16  another bf16 rendering of the same module: the oracle's written-out fp32 softmax attention, rounded to bf16;
  o32  the oracle in fp32 on the same weights (the exact algebra the bf16 renderings approximate).

Tolerance. Max-abs after log-softmax between r16 and o16 (two renderings of the reference itself) is about 0.06
after one layer and 0.42 after 32 (measured on a B200; the bf16 logits alone are quantised to 2^-5 at magnitude
4-8), so the 2e-2 bar of the bf16 mode cannot hold at this depth for any bf16 implementation; it is met on the
smaller bf16 models (config 1's golden bf16 logits, smoke()). Here the bar is the reference's own spread:
  * max-abs(log_softmax(product) - log_softmax(r16)) <= 1.1 * max-abs(log_softmax(o16) - log_softmax(r16));
  * max-abs against o32 <= 1.25 * r16's max-abs against o32 (the product is about as close to the exact algebra as
    the reference's own bf16 module; measured 1.04, and a variant of the attention kernel that only summed each
    softmax row in two halves moved it to 1.16, so the figure is sensitive to the order of fp32 sums).

* ForgeModel's forward over 2 x 512 tokens (forgeserve/model.py:140-159), against all three.
* Greedy generation of 16 tokens per row (forgeserve/sampling.py:24-35): the product's logits at every step (the
  cached decode path: split-K GEMMs and split-KV decode attention) lie within the reference's own spread of r16 at
  the same prefix, and every token is r16's greedy choice given that prefix, up to near-ties: a step may take
  another candidate only where r16's two log-probs are closer than twice the step's measured distance to r16; at
  least 75 % of the steps must be exact. The generated tokens must vary (std 0.02 weights can degenerate to one
  repeated token; forgeserve README.md:161-165).
* The same weights as 4 pipeline stages (threads on this GPU) with 4 micro-batches of 1 x 256 tokens
  (forgeserve/pipeline.py:95-118): the last stage's logits equal the single-process model's bit for bit, since
  every kernel treats rows alike at any row count above 128.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu

from forgeserve_b200 import ForgeModel, ModelConfig, PipelineStage, PipelineState, pipeline_forward
from forgeserve_b200 import _lib
from forgeserve_b200.kv import new_contiguous_cache
from forgeserve_b200.sampling import generate
from forgeserve_b200.tensor_parallel import run_in_threads
from forgeserve_b200.weights import init_model_, init_stage_
from oracle import forge_oracle as O

CFG = dict(vocab_size=128256, d_model=4096, n_layers=32, n_heads=32, n_kv_heads=8, ffn_dim=14336, max_seq_len=1024,
           rope_theta=500000.0)
SEED, STD = 1234, 0.02


@pytest.fixture(scope="module")
def model8b():
    cfg = ModelConfig(**CFG)
    model = ForgeModel(cfg, device="cuda", dtype=torch.bfloat16).eval()
    init_model_(model, seed=SEED, std=STD)
    sd16 = dict(model.state_dict())            # the oracle reads the very same bf16 tensors
    yield cfg, model, sd16
    del model, sd16
    torch.cuda.empty_cache()


def lsm_err(a: torch.Tensor, b: torch.Tensor) -> float:
    return float((torch.log_softmax(a.float(), -1) - torch.log_softmax(b.float(), -1)).abs().max())


SPREAD = 1.1           # the product may differ from r16 by 1.1x what o16 does
EXACT_SPREAD = 1.25    # ... and from o32 by 1.25x what r16 does


def test_8b_full_model_logits_match_the_oracle(model8b):
    cfg, model, sd16 = model8b
    ocfg = O.Cfg(**CFG)
    idx = torch.randint(0, cfg.vocab_size, (2, 512), generator=torch.Generator().manual_seed(21)).cuda()
    _lib.device_error(clear=True)
    got = model(idx)
    assert _lib.device_error(clear=True) == 0
    r16 = O.model_forward(sd16, ocfg, idx, attn_core=O.sdpa_torch)
    o16 = O.model_forward(sd16, ocfg, idx)
    e_pr, e_or = lsm_err(got, r16), lsm_err(o16, r16)
    del o16
    sd32 = {k: v.float() for k, v in sd16.items()}
    o32 = O.model_forward(sd32, ocfg, idx)
    e_p32, e_r32 = lsm_err(got, o32), lsm_err(r16, o32)
    del sd32, o32, r16
    torch.cuda.empty_cache()
    print(f"\n8B full model, 2 x 512 tokens, log-softmax max-abs: product vs r16 {e_pr:.4f} (o16 vs r16 {e_or:.4f}); "
          f"product vs o32 {e_p32:.4f} (r16 vs o32 {e_r32:.4f})")
    assert e_pr <= SPREAD * e_or, (e_pr, e_or)
    assert e_p32 <= EXACT_SPREAD * e_r32, (e_p32, e_r32)


def test_8b_full_model_greedy_tokens_match_the_oracle(model8b):
    cfg, model, sd16 = model8b
    ocfg = O.Cfg(**CFG)
    n_new = 16
    prompt = torch.randint(0, cfg.vocab_size, (2, 128), generator=torch.Generator().manual_seed(22))
    got = generate(model, prompt.cuda(), n_new)
    assert got.shape == (2, 128 + n_new) and torch.equal(got[:, :128].cpu(), prompt)
    new = got[:, 128:]
    assert len(set(new.flatten().tolist())) > 4, new            # tokens vary
    # the product's own logits at every step (the prefill's last position, then each cached decode step), which
    # its greedy choices came from
    kv = new_contiguous_cache(cfg.n_layers, cfg.max_seq_len)
    steps = [model(got[:, :128], kv=kv)[:, -1:]]
    for i in range(n_new - 1):
        steps.append(model(got[:, 128 + i : 129 + i], kv=kv))
    mine = torch.log_softmax(torch.cat(steps, 1).float(), -1)                                    # (2, 16, V)
    assert torch.equal(mine.argmax(-1), new)                    # generate() took these logits' argmax
    # r16 and o16 at the same prefixes (teacher-forced over the product's tokens)
    r16 = torch.log_softmax(O.model_forward(sd16, ocfg, got[:, :-1], attn_core=O.sdpa_torch)[:, 127:].float(), -1)
    o16 = torch.log_softmax(O.model_forward(sd16, ocfg, got[:, :-1])[:, 127:].float(), -1)
    err = (mine - r16).abs().amax(-1)                           # per step, over the vocab
    spread = float((o16 - r16).abs().max())
    best = r16.max(-1)
    gap = best.values - r16.gather(-1, new[..., None])[..., 0]
    exact = int((new == best.indices).sum())
    free = O.greedy_generate(sd16, ocfg, prompt.cuda(), n_new, attn_core=O.sdpa_torch)
    same = int((free[:, 128:] == new).sum())
    print(f"\n8B greedy, 2 rows x {n_new} tokens: {exact}/{2 * n_new} steps are r16's argmax given the same prefix; "
          f"step log-softmax max-abs vs r16 {float(err.max()):.4f} (o16 vs r16 {spread:.4f}); largest log-prob gap "
          f"to r16's choice {float(gap.max()):.4f}; free-running r16 tokens equal at {same}/{2 * n_new} steps")
    assert float(err.max()) <= SPREAD * spread, (float(err.max()), spread)
    # a step may differ from r16's choice only where r16's two candidates are closer than the two log-prob vectors
    # differ at that step (if |mine - r16| <= e everywhere, mine's argmax has r16 log-prob >= r16's best - 2e)
    assert bool((gap <= 2 * err + 1e-6).all()), (gap, err)
    assert exact >= 0.75 * 2 * n_new, (exact, gap)


def stage_worker(rank, size, cfg_dict, idx, microbatches):
    cfg = ModelConfig(**cfg_dict)
    stage = PipelineStage(cfg, rank, size, device="cuda", dtype=torch.bfloat16).eval()
    init_stage_(stage, seed=SEED, std=STD)
    state = PipelineState(stage, idx.shape[0], microbatches)
    logits = pipeline_forward(stage, state, idx if rank == 0 else None, idx.shape[1])
    torch.cuda.synchronize()
    out = None if logits is None else logits.clone()
    del stage, state, logits
    return out


def test_8b_four_stages_four_microbatches_equal_the_single_process_model(model8b):
    cfg, model, sd16 = model8b
    idx = torch.randint(0, cfg.vocab_size, (4, 256), generator=torch.Generator().manual_seed(23)).cuda()
    want = model(idx)
    res = run_in_threads(stage_worker, 4, CFG, idx, 4, timeout=600)
    assert all(r is None for r in res[:-1])
    got = res[-1]
    assert got.shape == want.shape
    assert torch.equal(got, want), float((got.float() - want.float()).abs().max())
    r16 = O.model_forward(sd16, O.Cfg(**CFG), idx, attn_core=O.sdpa_torch)
    e_pr, e_or = lsm_err(got, r16), lsm_err(O.model_forward(sd16, O.Cfg(**CFG), idx), r16)
    print(f"\n8B, 4 stages x 4 micro-batches: bit-identical to the single-process model; log-softmax max-abs "
          f"vs r16 {e_pr:.4f} (o16 vs r16 {e_or:.4f})")
    assert e_pr <= SPREAD * e_or, (e_pr, e_or)
    assert _lib.device_error(clear=True) == 0
