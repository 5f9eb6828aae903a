"""Generate the golden fixtures of tests/golden/ by running the reference forgeserve itself.

Run in a container that has the reference checkout (read-only is fine):

    python tests/golden/make_golden.py --reference /path/to/forgeserve

Weights are not stored: each fixture records the recipe (the reference test suite's randn * 0.25 model, or the
reference's own std-0.02 init from a torch seed) and a per-tensor checksum, and tests rebuild the weights with
oracle.forge_oracle and check the checksum first. Everything runs on the CPU in fp32 unless noted (one bf16
single-process fixture: the reference pipeline path itself only runs fp32, forgeserve/pipeline.py:108).
"""

import argparse
import os
import random
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
# The reference checkout to import (its `forgeserve` package): --reference <dir> or FORGESERVE_REFERENCE.
REF = os.environ.get("FORGESERVE_REFERENCE")
if "--reference" in sys.argv:
    REF = sys.argv[sys.argv.index("--reference") + 1]
if not REF:
    raise SystemExit("make_golden.py: pass --reference <reference checkout> or set FORGESERVE_REFERENCE")
sys.path.insert(0, REF)
sys.path.insert(0, str(ROOT))

from forgeserve import (Engine, ForgeModel, ModelConfig, PagedKVPool, PipelineStage, PipelineState,  # noqa: E402
                        generate, new_contiguous_cache, pipeline_forward, pipeline_generate)
from forgeserve.model import apply_rope, precompute_rope, RMSNorm  # noqa: E402
from forgeserve.parallel import TPContext  # noqa: E402
from forgeserve.tensor_parallel import run_distributed, shard_state_dict  # noqa: E402

from oracle import forge_oracle as O  # noqa: E402

SMALL = dict(vocab_size=64, d_model=64, n_layers=3, n_heads=8, n_kv_heads=4, max_seq_len=64)
C1 = dict(vocab_size=256, d_model=128, n_layers=4, n_heads=8, n_kv_heads=4)


def small_model():
    """The reference test suite's model (its tests/conftest.py: seed 0, then randn * 0.25 from generator 1)."""
    torch.manual_seed(0)
    model = ForgeModel(ModelConfig(**SMALL)).eval()
    g = torch.Generator().manual_seed(1)
    for p in model.parameters():
        if p.ndim >= 2:
            p.data = torch.randn(p.shape, generator=g) * 0.25
    return model


def forward_worker(rank, size, cfg_dict, full_sd, idx, more, microbatches):
    cfg = ModelConfig(**cfg_dict)
    stage = PipelineStage(cfg, rank, size).eval()
    stage.load_from_full(full_sd)
    state = PipelineState(stage, idx.shape[0], microbatches)
    logits = pipeline_forward(stage, state, idx if rank == 0 else None, idx.shape[1])
    logits2 = pipeline_forward(stage, state, more if rank == 0 else None, more.shape[1])
    return logits, logits2


def generate_worker(rank, size, cfg_dict, full_sd, prompt, microbatches, n):
    cfg = ModelConfig(**cfg_dict)
    stage = PipelineStage(cfg, rank, size).eval()
    stage.load_from_full(full_sd)
    return pipeline_generate(stage, prompt, n, microbatches)


def tp_worker(rank, size, cfg_dict, full_sd, idx, more, prompt, n_new):
    """One tensor-parallel shard of the reference model: a forward, a chunk continued through its cache, the number
    of all-reduces those two took, and a greedy generation."""
    cfg = ModelConfig(**cfg_dict)
    tp = TPContext(rank, size)
    model = ForgeModel(cfg, tp).eval()
    model.load_state_dict(shard_state_dict(full_sd, cfg, rank, size))
    kv = new_contiguous_cache(cfg.n_layers)
    first = model(idx, kv=kv)
    cont = model(more, kv=kv)
    # numpy copies travel by value through the launcher's queue (a tensor would be passed as a shared-memory handle,
    # which the parent cannot open once the worker has exited)
    gen = generate(model, prompt, n_new)
    return first.numpy().copy(), cont.numpy().copy(), tp.num_all_reduces, gen.numpy().copy()


def tp_engine_worker(rank, size, cfg_dict, full_sd, requests, num_blocks, max_batch):
    """The reference Engine over one tensor-parallel shard."""
    cfg = ModelConfig(**cfg_dict)
    model = ForgeModel(cfg, TPContext(rank, size)).eval()
    model.load_state_dict(shard_state_dict(full_sd, cfg, rank, size))
    eng = Engine(model, num_blocks=num_blocks, block_size=4, max_batch=max_batch)
    ids = [eng.add_request(p, n) for p, n in requests]
    res = eng.run()
    return [res[i] for i in ids], eng.steps, eng.preemptions, tuple(eng.pool.k[0].shape)


def make_requests(n=6, seed=1):
    g = torch.Generator().manual_seed(seed)
    reqs = []
    for _ in range(n):
        plen = int(torch.randint(2, 20, (1,), generator=g))
        reqs.append((torch.randint(0, 64, (plen,), generator=g).tolist(), int(torch.randint(3, 15, (1,), generator=g))))
    return reqs


def small_fixture():
    torch.manual_seed(0)
    model = small_model()
    sd = {k: v.detach().clone() for k, v in model.state_dict().items()}
    cfg = ModelConfig(**SMALL)
    out = {"cfg": SMALL, "weights": ("test_model_weights", 1, 0.25), "checksum": O.checksum(sd)}

    # single-process forward, a continued chunk, one-token cache steps
    idx = torch.randint(0, 64, (4, 9), generator=torch.Generator().manual_seed(2))
    more = torch.randint(0, 64, (4, 3), generator=torch.Generator().manual_seed(9))
    out["idx"], out["more"] = idx, more
    out["logits"] = model(idx)
    out["logits_more"] = model(torch.cat([idx, more], 1))[:, 9:]
    steps_idx = torch.randint(0, 64, (2, 20), generator=torch.Generator().manual_seed(3))
    kv = new_contiguous_cache(cfg.n_layers)
    out["steps_idx"] = steps_idx
    out["steps_logits"] = torch.cat([model(steps_idx[:, i : i + 1], kv=kv) for i in range(20)], dim=1)
    out["shifted_logits"] = model(idx[:1, :5], positions=torch.arange(5)[None] + 11)

    # the reference pipeline over gloo at (stages, micro-batches)
    out["pipeline"] = {}
    for size, mbs in [(2, 1), (3, 2), (3, 4)]:
        res = run_distributed(forward_worker, size, cfg.to_dict(), sd, idx, more, mbs)
        out["pipeline"][(size, mbs)] = res[-1]
        assert all(r[0] is None for r in res[:-1])
    # more micro-batches than rows: the reference fails on the empty micro-batch (a RuntimeError on a rank)
    try:
        run_distributed(forward_worker, 2, cfg.to_dict(), sd, idx, more, 8, timeout=60)
        out["empty_microbatch_raises"] = False
    except RuntimeError:
        out["empty_microbatch_raises"] = True

    # greedy generation: single process and pipelined
    prompt = torch.randint(0, 64, (4, 5), generator=torch.Generator().manual_seed(4))
    out["prompt"] = prompt
    out["generate"] = generate(model, prompt, 10)
    out["pipeline_generate"] = {}
    for size, mbs in [(2, 1), (3, 2)]:
        res = run_distributed(generate_worker, size, cfg.to_dict(), sd, prompt, mbs, 10)
        out["pipeline_generate"][(size, mbs)] = res[0]
        assert all(torch.equal(r, res[0]) for r in res)
    out["generate_long"] = generate(model, torch.randint(0, 64, (1, 60), generator=torch.Generator().manual_seed(5)), 100)

    # paged: prefill 12 then 18 decode steps through shuffled blocks
    pidx = torch.randint(0, 64, (1, 30), generator=torch.Generator().manual_seed(6))
    pool = PagedKVPool(cfg, num_blocks=16, block_size=4)
    blocks = pool.allocator.allocate(8)
    random.Random(0).shuffle(blocks)
    table = torch.tensor([blocks])
    got = [model(pidx[:, :12], torch.arange(12)[None], pool.views(table, torch.arange(12)[None]))]
    for i in range(12, 30):
        pos = torch.tensor([[i]])
        got.append(model(pidx[:, i : i + 1], pos, pool.views(table, pos)))
    out["paged_idx"], out["paged_blocks"], out["paged_logits"] = pidx, blocks, torch.cat(got, 1)

    # the serving engine: outputs per request, with and without preemption
    reqs = make_requests()
    eng = Engine(model, num_blocks=64, block_size=4, max_batch=3)
    ids = [eng.add_request(p, n) for p, n in reqs]
    res = eng.run()
    out["engine"] = {"requests": reqs, "outputs": [res[i] for i in ids], "steps": eng.steps,
                     "peak_running": eng.peak_running, "preemptions": eng.preemptions}
    reqs5 = make_requests(5)
    eng = Engine(model, num_blocks=12, block_size=4, max_batch=5)
    ids = [eng.add_request(p, n) for p, n in reqs5]
    res = eng.run()
    out["engine_preempt"] = {"requests": reqs5, "outputs": [res[i] for i in ids], "steps": eng.steps,
                             "preemptions": eng.preemptions}

    # bf16: the reference single-process model in bf16 (CPU), and its bf16 RMSNorm / RoPE on random inputs
    mb = small_model().to(torch.bfloat16)
    out["bf16_logits"] = mb(idx)
    x0 = mb.embed(idx)
    out["bf16_block0"] = mb.layers[0](x0, mb.rope_cos, mb.rope_sin, torch.arange(9)[None].expand(4, 9),
                                      new_contiguous_cache(1)[0])
    x = torch.randn(5, 64, generator=torch.Generator().manual_seed(7)).to(torch.bfloat16) * 3
    w = (torch.rand(64, generator=torch.Generator().manual_seed(8)) + 0.5).to(torch.bfloat16)
    norm = RMSNorm(64).to(torch.bfloat16)
    norm.weight.data = w
    out["bf16_rmsnorm"] = {"x": x, "w": w, "y": norm(x)}
    cos, sin = precompute_rope(16, 64, 10000.0)
    q = torch.randn(2, 4, 7, 16, generator=torch.Generator().manual_seed(10)).to(torch.bfloat16)
    pos = torch.tensor([[0, 3, 9, 20, 33, 40, 63], [5, 6, 7, 8, 9, 10, 11]])
    out["bf16_rope"] = {"x": q, "positions": pos, "y": apply_rope(q, cos.to(torch.bfloat16), sin.to(torch.bfloat16), pos)}
    return out


def tp_fixture():
    """The reference's tensor parallelism (model.py:47-106, parallel.py, tensor_parallel.py) over gloo on the test
    suite's model: 2 and 4 shards (n_kv_heads 4), forward + continued chunk + greedy generation, and the Engine
    over 2 shards with a pool small enough to preempt."""
    cfg = ModelConfig(**SMALL)
    sd = {k: v.detach().clone() for k, v in small_model().state_dict().items()}
    idx = torch.randint(0, 64, (4, 9), generator=torch.Generator().manual_seed(2))
    more = torch.randint(0, 64, (4, 3), generator=torch.Generator().manual_seed(9))
    prompt = torch.randint(0, 64, (4, 5), generator=torch.Generator().manual_seed(4))
    out = {"cfg": SMALL, "weights": ("test_model_weights", 1, 0.25), "checksum": O.checksum(sd), "idx": idx,
           "more": more, "prompt": prompt, "tp": {}}
    for size in (2, 4):
        res = [tuple(torch.from_numpy(a) if not isinstance(a, int) else a for a in r)
               for r in run_distributed(tp_worker, size, cfg.to_dict(), sd, idx, more, prompt, 10)]
        first, cont, n_ar, gen = res[0]
        for r in res[1:]:
            assert torch.equal(r[0], first) and torch.equal(r[3], gen) and r[2] == n_ar
        out["tp"][size] = {"logits": first, "logits_more": cont, "all_reduces": n_ar, "generate": gen}
    reqs = make_requests(5)
    res = run_distributed(tp_engine_worker, 2, cfg.to_dict(), sd, reqs, 12, 5)
    assert all(r[:3] == res[0][:3] for r in res)
    out["tp_engine"] = {"requests": reqs, "outputs": res[0][0], "steps": res[0][1], "preemptions": res[0][2],
                        "pool_shape": res[0][3], "num_blocks": 12, "max_batch": 5}
    return out


def c1_fixture():
    """tiny fp32 decoder, 2 pipeline stages over gloo, 4 micro-batches of 2 x 16 tokens."""
    cfg = ModelConfig(**C1)
    model = ForgeModel(cfg).eval()
    # seeded N(0, 0.02) weights (the reference's init scale), norms ones; rebuilt by the tests from the recipe
    model.load_state_dict(O.test_model_weights(O.Cfg(**C1), seed=1234, scale=0.02))
    sd = {k: v.detach().clone() for k, v in model.state_dict().items()}
    idx = torch.randint(0, 256, (8, 16), generator=torch.Generator().manual_seed(11))
    res = run_distributed(forward_worker, 2, cfg.to_dict(), sd, idx, idx[:, :3].clone(), 4)
    prompt = idx[:, :6].clone()
    gen = run_distributed(generate_worker, 2, cfg.to_dict(), sd, prompt, 4, 8)
    bf16_logits = ForgeModel(cfg).eval()
    bf16_logits.load_state_dict(sd)
    bf16_logits = bf16_logits.to(torch.bfloat16)(idx)
    return {"cfg": C1, "weights": ("test_model_weights", 1234, 0.02), "checksum": O.checksum(sd), "idx": idx,
            "logits": model(idx), "bf16_logits": bf16_logits,
            "pipeline_logits": res[-1][0], "pipeline_logits2": res[-1][1], "prompt": prompt,
            "generate": generate(model, prompt, 8), "pipeline_generate": gen[0]}


PP8 = dict(vocab_size=2048, d_model=512, n_layers=8, n_heads=4, n_kv_heads=2, max_seq_len=544)
PP8_POSITIONS = [0, 1, 127, 128, 255, 256, 300, 383, 384, 511]


def pp8_fixture():
    """A head_dim-128 model that splits into 1, 2, 4 or 8 pipeline stages (8 layers) with a vocab of 8 head tiles of
    256 (one per stage at 8). The multi-GPU bench checks its own NCCL pipeline against these before timing; the
    reference's pipeline matches its single-process model within 1e-4 (its tests/test_pipeline.py:44-68), so the
    single-process outputs are what a pipeline of any depth must give.
    fp32: the reference test suite's randn recipe at scale 0.05 (greedy tokens vary; fp32 rounding stays near
    2e-5, inside the 1e-4 bar, where 0.25 reaches 2.4e-4 at this depth), logits at positions that
    straddle 128-token boundaries (where sequence pieces start) for 8 rows x 512 tokens, and 16 greedy tokens.
    bf16: the same recipe at scale 0.02, the reference's module in bf16 on the CPU, logits at the same positions."""
    cfg = ModelConfig(**PP8)
    model = ForgeModel(cfg).eval()
    model.load_state_dict(O.test_model_weights(O.Cfg(**PP8), seed=4321, scale=0.05))
    sd = {k: v.detach().clone() for k, v in model.state_dict().items()}
    idx = torch.randint(0, PP8["vocab_size"], (8, 512), generator=torch.Generator().manual_seed(31))
    pos = torch.tensor(PP8_POSITIONS)
    logits = model(idx)[:, pos]
    prompt = torch.randint(0, PP8["vocab_size"], (8, 32), generator=torch.Generator().manual_seed(32))
    m16 = ForgeModel(cfg).eval()
    sd16 = O.test_model_weights(O.Cfg(**PP8), seed=4321, scale=0.02)
    m16.load_state_dict(sd16)
    bf16_logits = m16.to(torch.bfloat16)(idx)[:, pos]
    # the spread between two bf16 renderings of the reference's module (its own attention call, and the oracle's
    # written-out fp32 softmax rounded to bf16): a bf16 implementation is held to this (or 2e-2 if larger)
    o16 = O.model_forward({k: v.bfloat16() for k, v in sd16.items()}, O.Cfg(**PP8), idx)[:, pos]
    spread = O.log_softmax_maxabs(o16, bf16_logits)
    return {"cfg": PP8, "weights": ("test_model_weights", 4321, 0.05), "checksum": O.checksum(sd), "idx": idx,
            "positions": pos, "logits": logits, "prompt": prompt, "generate": generate(model, prompt, 16),
            "bf16_weights": ("test_model_weights", 4321, 0.02), "bf16_checksum": O.checksum(sd16),
            "bf16_logits": bf16_logits, "bf16_spread": spread}


FIXTURES = {"small": small_fixture, "c1": c1_fixture, "tp": tp_fixture, "pp8": pp8_fixture}

if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=REF)
    ap.add_argument("--only", default="", help="comma-separated fixture names (default: all)")
    args = ap.parse_args()
    for name in (args.only.split(",") if args.only else FIXTURES):
        torch.save(FIXTURES[name](), HERE / f"{name}.pt")
    print("wrote", sorted(p.name for p in HERE.glob("*.pt")))
