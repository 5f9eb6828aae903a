"""Pipeline-parallel prefill throughput of an 8B-shaped bf16 decoder on 1-8 B200s (one pipeline stage per GPU).

Workload: LLaMA-3-8B shape — 32 layers, d_model 4096, 32 query / 8 KV heads (head_dim 128),
ffn 14336, vocab 128256, RoPE theta 5e5 — seeded N(0, 0.02) weights, uniform random token ids; one step is one
`pipeline_forward` of 16 micro-batches x (4 x 2048) tokens through p = N stages, logits for every position on the
last stage, exactly as the reference's pipeline_forward computes them.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...     (one rank per GPU, NCCL)

Other workloads (not the headline): `--workload c2` (config 2: the same prefill on the 1B shape, 8 micro-batches of
4 x 1024 tokens), `--workload c4` (config 4: continuous-batching decode of 64 requests over a
paged cache; one step is the whole batch) and `--workload c5` (config 5: the 70B shape, a micro-batch sweep of
generation; one step is one generation per sweep point, so `--steps 1 --warmup 1` at 8 GPUs takes about a minute).

Prints one JSON line on rank 0. `value` is device-timed (CUDA events, max over ranks) with the token ids already
on the GPU; `e2e` is the same through the public API with the token ids copied from pinned host memory and the
last-position logits copied back every step. `--impl reference` times the CPU oracle (a restatement of the
reference's algorithm) on the host cores on a bounded sample of the same workload.
"""

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "PP prefill tokens/s, 8B-shape bf16"
CFG = dict(vocab_size=128256, d_model=4096, n_layers=32, n_heads=32, n_kv_heads=8, ffn_dim=14336, max_seq_len=8192,
           rope_theta=500000.0)
MICROBATCHES, MB_ROWS, SEQ = 16, 4, 2048
WORKLOAD = ("C3: 8B-shape prefill (32 layers, d4096, 32/8 heads, ffn 14336, vocab 128256, theta 5e5), "
            "16 micro-batches x (4 x 2048 tokens), one pipeline stage per GPU")

# Pipeline-prefill workloads: config 3 (the headline) and config 2 (the 1B shape; its RoPE theta is not given,
# so it keeps the reference's default).
PREFILL = {
    "c3": dict(cfg=CFG, microbatches=MICROBATCHES, rows=MB_ROWS, seq=SEQ, metric=METRIC, workload=WORKLOAD),
    "c2": dict(cfg=dict(vocab_size=128256, d_model=2048, n_layers=16, n_heads=32, n_kv_heads=8, ffn_dim=8192,
                        max_seq_len=1024),
               microbatches=8, rows=4, seq=1024, metric="PP prefill tokens/s, 1B-shape bf16 (config 2)",
               workload=("C2: 1B-shape prefill (16 layers, d2048, 32/8 heads, head_dim 64, ffn 8192, vocab 128256), "
                         "8 micro-batches x (4 x 1024 tokens), one pipeline stage per GPU")),
}


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["bf16_tflops_sustained"], "measured (bf16_tflops_sustained, MEASURED_PEAKS.json)"
    return 1400.0, "fallback (1.4 PFLOP/s sustained)"


class ClockSampler:
    """nvidia-smi samples every 200 ms while running (reads clocks only; changes nothing)."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus):
        self.gpus = set(gpus)
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9 or not f[0].isdigit() or int(f[0]) not in self.gpus:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        under = [s for s in sm if mx and s > 0.3 * mx] or sm
        return {"sm_mhz": statistics.median(under) if under else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------------------------------------ parity prologue
PARITY_FIXTURE = ROOT / "tests" / "golden" / "pp8.pt"


def parity_check(world, rank, dev, split_head: bool, seq_chunks: int):
    """Before any timing: the pipeline this run times (N stages over NCCL, the same head split and sequence pieces)
    on the 8-layer golden model of tests/golden/pp8.pt, against the reference's own outputs recorded there
    (its single-process model, which its pipeline matches within 1e-4): fp32 logits at 10 positions of 8 rows x
    512 tokens within atol = rtol = 1e-4, its 16 greedy tokens per row through pipeline_generate, and the bf16
    logits (tensor-core path) within max(2e-2, 1.1 x the spread between two bf16 renderings of the reference) after
    log-softmax. Outside the timed region; the result goes into the JSON line."""
    import torch.distributed as dist

    from forgeserve_b200 import ModelConfig, PipelineStage, PipelineState, pipeline_forward, pipeline_generate
    from forgeserve_b200.weights import checksum, test_suite_state_dict

    g = torch.load(PARITY_FIXTURE, weights_only=False)
    cfg = ModelConfig(**g["cfg"])
    B, T = g["idx"].shape
    mbs = 4
    res = {"model": "tests/golden/pp8.pt: 8 layers, d_model 512, 4/2 heads (head_dim 128), vocab 2048; reference "
                    "outputs", "stages": world, "microbatches": mbs,
           "seq_pieces": seq_chunks, "head": "split over the stages" if split_head else "on the last stage"}
    for mode, dtype in (("fp32", torch.float32), ("bf16", torch.bfloat16)):
        recipe, ck = (g["weights"], g["checksum"]) if mode == "fp32" else (g["bf16_weights"], g["bf16_checksum"])
        sd = test_suite_state_dict(cfg, recipe[1], recipe[2])
        got_ck = checksum(sd)      # fp64 sums: equal up to the host's reduction order
        if set(got_ck) != set(ck) or any(abs(a - b) > 1e-9 * max(1.0, abs(b))
                                         for k in ck for a, b in zip(got_ck[k], ck[k])):
            raise RuntimeError("parity fixture: the weight recipe does not reproduce the recorded checksums")
        stage = PipelineStage(cfg, rank, world, device=dev, dtype=dtype).eval()
        stage.load_from_full(sd)
        if split_head:
            stage.split_head_()
        state = PipelineState(stage, B, mbs)
        logits = pipeline_forward(stage, state, g["idx"].to(dev) if stage.is_first else None, T,
                                  seq_chunks=seq_chunks)
        err = torch.zeros(2, dtype=torch.float64, device=dev)
        if stage.is_last:
            got = logits[:, g["positions"].to(dev)].float().cpu()
            if mode == "fp32":
                want = g["logits"]
                err[0] = float(((got - want).abs() / (1e-4 + 1e-4 * want.abs())).max())   # <= 1 passes
                err[1] = float((got - want).abs().max())
            else:
                lg = torch.log_softmax(got, -1) - torch.log_softmax(g["bf16_logits"].float(), -1)
                err[0] = float(lg.abs().max())
        if world > 1:
            dist.broadcast(err, src=world - 1)
        if mode == "fp32":
            res["fp32_logits_maxabs"] = round(float(err[1]), 7)
            res["fp32_within_1e-4"] = bool(float(err[0]) <= 1.0)
            toks = pipeline_generate(stage, g["prompt"], 16, microbatches=mbs)
            res["greedy_tokens_equal"] = bool(torch.equal(toks.cpu(), g["generate"]))
        else:
            bar = max(2e-2, 1.1 * g["bf16_spread"])
            res.update({"bf16_logsoftmax_maxabs": round(float(err[0]), 5), "bf16_bar": round(bar, 5),
                        "bf16_within_bar": bool(float(err[0]) <= bar)})
        del stage, state, logits
    if world > 1:
        flag = torch.tensor([float(res["greedy_tokens_equal"])], device=dev)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        res["greedy_tokens_equal"] = bool(float(flag) == 1.0)
    res["ok"] = res["fp32_within_1e-4"] and res["greedy_tokens_equal"] and res["bf16_within_bar"]
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return res


# --------------------------------------------------------------------------------------------------- ours
def run_ours(args, spec):
    import torch.distributed as dist

    from forgeserve_b200 import ModelConfig, PipelineStage, PipelineState, bubble_fraction, ops, pipeline_forward
    from forgeserve_b200 import _lib
    from forgeserve_b200.pipeline import seq_pieces
    from forgeserve_b200.weights import init_stage_

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=600))

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def allreduce(x, op):
        t = torch.tensor([float(x)], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=op)
        return float(t)

    cfg = ModelConfig(**spec["cfg"])
    microbatches, mb_rows, seq = spec["microbatches"], spec["rows"], spec["seq"]
    split_head = world > 1 and not args.whole_head
    parity = parity_check(world, rank, dev, split_head, args.seq_chunks)
    stage = PipelineStage(cfg, rank, world, device=dev, dtype=torch.bfloat16).eval()
    init_stage_(stage, seed=1234, std=0.02)
    weight_gb = allreduce(sum(p.numel() * p.element_size() for p in stage.parameters()),
                          dist.ReduceOp.SUM if world > 1 else None) / 1e9
    if split_head:
        stage.split_head_()   # every stage computes a vocab slice of the head (logits still land on the last stage)
    batch = microbatches * mb_rows
    g = torch.Generator(device="cpu").manual_seed(7)
    idx_host = torch.randint(0, cfg.vocab_size, (batch, seq), generator=g).pin_memory()
    idx_dev = idx_host.to(dev)
    tokens_per_step = batch * seq

    def step(idx):
        state = PipelineState(stage, batch, microbatches)
        return pipeline_forward(stage, state, idx if stage.is_first else None, seq, seq_chunks=args.seq_chunks)

    for _ in range(args.warmup):
        step(idx_dev)
    barrier()

    # ---- device-timed region (token ids already on the GPU)
    stream = torch.cuda.current_stream(dev)
    stage.trace = []
    ops.gemm_events = []
    launches0 = _lib.launch_count()
    sampler = ClockSampler([local] if world == 1 else range(world))
    with sampler:
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            out = step(idx_dev)
            del out
        e1.record(stream)
        torch.cuda.synchronize()
    launches = _lib.launch_count() - launches0
    ms_total = e0.elapsed_time(e1)
    ms_max = allreduce(ms_total, dist.ReduceOp.MAX if world > 1 else None)
    busy_ms = sum(a.elapsed_time(b) for _, a, b in stage.trace)
    busy_sum = allreduce(busy_ms, dist.ReduceOp.SUM if world > 1 else None)
    gemm_flops = sum(f for _, _, f in ops.gemm_events)
    gemm_ms = sum(a.elapsed_time(b) for a, b, _ in ops.gemm_events)
    gemm_n = len(ops.gemm_events)
    per_rank = {"rank": rank, "gemm_tflops": round(gemm_flops / max(gemm_ms, 1e-9) / 1e9, 1),
                "busy_ms": round(busy_ms, 1), "elapsed_ms": round(ms_total, 1)}
    if world > 1:
        gathered = [None] * world
        dist.all_gather_object(gathered, per_rank)
    else:
        gathered = [per_rank]
    gemm_flops = allreduce(gemm_flops, dist.ReduceOp.SUM if world > 1 else None)
    gemm_ms = allreduce(gemm_ms, dist.ReduceOp.SUM if world > 1 else None)
    gemm_n = allreduce(gemm_n, dist.ReduceOp.SUM if world > 1 else None)
    launches = allreduce(launches, dist.ReduceOp.SUM if world > 1 else None)
    stage.trace = None
    ops.gemm_events = None

    # ---- end to end through the public API: host token ids in, last-position logits out
    barrier()
    out_host = torch.empty(batch, cfg.vocab_size, dtype=torch.bfloat16).pin_memory() if stage.is_last else None
    e2 = torch.cuda.Event(enable_timing=True)
    e3 = torch.cuda.Event(enable_timing=True)
    e2.record(stream)
    for _ in range(args.steps):
        idx = idx_host.to(dev, non_blocking=True) if stage.is_first else None
        logits = step(idx)
        if stage.is_last:
            out_host.copy_(logits[:, -1], non_blocking=True)
        del logits
    e3.record(stream)
    torch.cuda.synchronize()
    e2e_ms = allreduce(e2.elapsed_time(e3), dist.ReduceOp.MAX if world > 1 else None)

    clocks = sampler.summary()
    result = None
    if rank == 0:
        value = tokens_per_step * args.steps / (ms_max / 1e3)
        peak, peak_src = peaks()
        achieved = gemm_flops / (gemm_ms / 1e3) / 1e12 if gemm_ms > 0 else None
        flops_per_token = 2 * (cfg.d_model * (cfg.n_heads + 2 * cfg.n_kv_heads) * cfg.head_dim +
                               cfg.n_heads * cfg.head_dim * cfg.d_model + 3 * cfg.d_model * cfg.ffn_dim) \
            * cfg.n_layers \
            + 2 * cfg.d_model * cfg.vocab_size
        attn_flops = 2 * mb_rows * cfg.n_heads * seq * seq * cfg.head_dim * cfg.n_layers * microbatches  # causal
        step_flops = flops_per_token * tokens_per_step + attn_flops
        n_pieces = len(seq_pieces(seq, args.seq_chunks, mb_rows))
        result = {
            "metric": spec["metric"], "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 3), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: uniform token ids, seeded N(0, 0.02) weights (no checkpoint or dataset)",
            "config": {"workload": spec["workload"], "global_batch": batch, "seq_len": seq,
                       "microbatches": microbatches,
                       "stages": world, "parallelism": f"pp{world}",
                       "head": "split over the stages by vocab range" if split_head else "on the last stage",
                       "seq_pieces": n_pieces,
                       "l2": f"no flush needed: every step streams {weight_gb:.1f} GB of weights (> 126 MB L2)"},
            "bubble": {"measured": round(1.0 - busy_sum / (world * ms_max), 4),
                       "analytic": round(bubble_fraction(world, microbatches * n_pieces), 4),
                       "analytic_whole_microbatches": round(bubble_fraction(world, microbatches), 4)},
            "model_tflops": round(step_flops * args.steps / (ms_max / 1e3) / 1e12, 1),
            # the whole step against the pipeline's peak: model FLOP/s / (stages x the measured GEMM peak)
            "model_frac": round(step_flops * args.steps / (ms_max / 1e3) / 1e12 / (world * peak), 4),
            "roofline": {"bound": "tensor",
                         "kernel": "gemm_tc2_kernel, the 2-SM tcgen05 GEMM (every projection GEMM of the timed region)",
                         "achieved": round(achieved, 1) if achieved else None, "peak": peak, "unit": "TFLOP/s",
                         "frac": round(achieved / peak, 4) if achieved else None, "peak_source": peak_src,
                         "launches": int(gemm_n), "traffic": gemm_traffic() if spec["cfg"] is CFG else None},
            "e2e": {"value": round(tokens_per_step * args.steps / (e2e_ms / 1e3), 1), "unit": "tokens/s",
                    "h2d_bytes_per_step": idx_host.numel() * idx_host.element_size(),
                    "d2h_bytes_per_step": batch * cfg.vocab_size * 2,
                    "io": "token ids from pinned host memory in; the last position's logits of every row "
                          "(B x vocab bf16) back to pinned host memory; all-position logits stay on the device"},
            "parity": parity,
            "per_rank": gathered,
            "gpu_launches": int(launches),
            "clocks": clocks,
        }
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return result


# --------------------------------------------------------------------------------------- config 4 (decode)
C4 = dict(requests=64, new_tokens=256, prompt_lo=512, prompt_hi=4096, num_blocks=16384, block_size=16)
C4_WORKLOAD = ("C4: 8B-shape continuous-batching decode over a paged KV cache (block size 16, 16384 blocks per "
               "GPU, free list shuffled by a seed), 64 requests, prompts uniform in [512, 4096], 256 greedy new "
               "tokens each, one pipeline stage per GPU")


def run_c4(args):
    """Config 4 through the Engine (1 GPU) or PipelineEngine (one stage per GPU): one step is the whole batch of
    64 requests from submission to the last token. Reports generated tokens/s over the run and over the decode
    phase (every request prefilled), and the decode steps' HBM bytes against the measured bandwidth."""
    import random
    import torch.distributed as dist

    from forgeserve_b200 import Engine, ForgeModel, ModelConfig, PipelineStage, _lib
    from forgeserve_b200.pipeline_engine import PipelineEngine
    from forgeserve_b200.weights import init_model_, init_stage_

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=600))
    cfg = ModelConfig(**CFG)
    if world == 1:
        model = ForgeModel(cfg, device=dev, dtype=torch.bfloat16).eval()
        init_model_(model, seed=1234, std=0.02)
        engine = Engine(model, C4["num_blocks"], C4["block_size"], max_batch=C4["requests"], seed=0,
                        cuda_graphs=not args.no_graphs)
        weight_bytes = sum(p.numel() * p.element_size() for p in model.parameters())
    else:
        stage = PipelineStage(cfg, rank, world, device=dev, dtype=torch.bfloat16).eval()
        init_stage_(stage, seed=1234, std=0.02)
        engine = PipelineEngine(stage, C4["num_blocks"], C4["block_size"], max_batch=C4["requests"], seed=0,
                                microbatches=args.microbatches or world, overlap=False if args.no_windows else None,
                                prefill_chunks=args.seq_chunks, cuda_graphs=not args.no_graphs)
        weight_bytes = sum(p.numel() * p.element_size() for p in stage.parameters())
    rng = random.Random(11)
    lengths = [rng.randint(C4["prompt_lo"], C4["prompt_hi"]) for _ in range(C4["requests"])]
    g = torch.Generator().manual_seed(12)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in lengths]
    stream = torch.cuda.current_stream(dev)

    def one_run(prompts, new_tokens):
        random.Random(5).shuffle(engine.pool.allocator._free)   # non-contiguous block tables
        for pr in prompts:
            engine.add_request(pr, new_tokens)
        e0 = torch.cuda.Event(enable_timing=True)
        e_dec = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        while engine.waiting:            # prefill phase: one request per step (decodes only while blocks lack)
            engine.step()
        e_dec.record(stream)
        steps0 = engine.steps
        engine.run()                     # decode phase (on a pipeline: decode windows, unless --no-windows)
        decode_steps = engine.steps - steps0
        e1.record(stream)
        torch.cuda.synchronize()
        outs = {rid: r.output for rid, r in engine.requests.items()}
        engine.requests.clear()
        return e0.elapsed_time(e1), e_dec.elapsed_time(e1), decode_steps, outs

    for _ in range(max(args.warmup, 1)):
        one_run(prompts[:8], 16)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    launches0 = _lib.launch_count()
    sampler = ClockSampler([local] if world == 1 else range(world))
    total_ms = dec_ms = 0.0
    steps_dec = 0
    with sampler:
        for _ in range(args.steps):
            t, td, nd, outs = one_run(prompts, C4["new_tokens"])
            total_ms, dec_ms, steps_dec = total_ms + t, dec_ms + td, steps_dec + nd
    launches = _lib.launch_count() - launches0

    def red(x, op):
        t = torch.tensor([float(x)], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=op)
        return float(t)

    total_ms = red(total_ms, dist.ReduceOp.MAX if world > 1 else None)
    dec_ms = red(dec_ms, dist.ReduceOp.MAX if world > 1 else None)
    weight_bytes = red(weight_bytes, dist.ReduceOp.SUM if world > 1 else None)
    launches = red(launches, dist.ReduceOp.SUM if world > 1 else None)
    clocks = sampler.summary()
    result = None
    if rank == 0:
        n_req, n_new = C4["requests"], C4["new_tokens"]
        generated = n_req * n_new * args.steps
        dec_tokens = n_req * (n_new - 1) * args.steps
        # bytes a decode step must move: every weight once (all stages) and the K/V of every cached token of
        # every layer; the mean context over the decode phase is prompt + half the generated tokens
        kv_token = cfg.n_layers * cfg.n_kv_heads * cfg.head_dim * 2 * 2
        mean_ctx = sum(lengths) / n_req + n_new / 2
        step_bytes = weight_bytes + n_req * mean_ctx * kv_token
        step_ms = dec_ms / max(steps_dec, 1)
        hbm, src = (json.loads((ROOT / "MEASURED_PEAKS.json").read_text())["hbm_gbs"], "measured") \
            if (ROOT / "MEASURED_PEAKS.json").exists() else (6650.0, "fallback")
        achieved = step_bytes / (step_ms / 1e3) / 1e9
        result = {
            "metric": "continuous-batching decode tokens/s, 8B-shape bf16 (config 4)",
            "value": round(generated / (total_ms / 1e3), 1), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": max(args.warmup, 1), "ms_per_step": round(total_ms / args.steps, 1),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: seeded prompt lengths and token ids, seeded N(0, 0.02) weights",
            "config": {"workload": C4_WORKLOAD, "stages": world, "parallelism": f"pp{world}",
                       "microbatches": 1 if world == 1 else (args.microbatches or world),
                       "decode_cuda_graphs": (not args.no_graphs) and (world == 1 or not args.no_windows),
                       "prefill_pieces": args.seq_chunks if world > 1 else 1,
                       "decode_windows": getattr(engine, "windows", 0)},
            "decode": {"tokens_per_s": round(dec_tokens / (dec_ms / 1e3), 1), "steps": steps_dec,
                       "ms_per_step": round(step_ms, 3)},
            "roofline": {"bound": "hbm", "kernel": "whole decode step (weights + K/V of every cached token)",
                         "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(achieved / hbm, 4), "peak_source": src,
                         "bytes_per_step": int(step_bytes)},
            "gpu_launches": int(launches), "clocks": clocks,
        }
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return result


# --------------------------------------------------------------------------------------- config 5 (70B)
C5_CFG = dict(vocab_size=128256, d_model=8192, n_layers=80, n_heads=64, n_kv_heads=8, ffn_dim=28672,
              max_seq_len=2048 + 128, rope_theta=500000.0)
C5 = dict(rows=2, seq=2048, new_tokens=128, sweep=(4, 8, 16, 32))
C5_WORKLOAD = ("C5: 70B-shape generation (80 layers, d8192, 64/8 heads, ffn 28672, vocab 128256, theta 5e5), "
               "micro-batches of 2 prompts x 2048 tokens, swept over 4/8/16/32 micro-batches, 128 greedy new tokens "
               "each, one pipeline stage per GPU")


def c5_stage_bytes(cfg, world: int, rank: int, m: int) -> int:
    """Device bytes a stage needs for one sweep point: its weights, the contiguous K/V of its layers for 2m rows
    (capacity up to twice the length, as the caches grow), and the largest activations (gate/up of one
    micro-batch's prefill)."""
    from forgeserve_b200.pipeline import stage_layers
    lo, hi = stage_layers(cfg.n_layers, world)[rank]
    d, f, hd = cfg.d_model, cfg.ffn_dim, cfg.head_dim
    layer = d * (cfg.n_heads + 2 * cfg.n_kv_heads) * hd + cfg.n_heads * hd * d + 3 * d * f + 2 * d
    weights = (hi - lo) * layer * 2 + cfg.vocab_size * d * 2 * ((rank == 0) + (rank == world - 1)) \
        + (d * 2 if rank == world - 1 else 0)                   # embedding, head, final norm
    kv = (hi - lo) * 2 * C5["rows"] * m * 2 * cfg.max_seq_len * cfg.n_kv_heads * hd * 2
    act = C5["rows"] * C5["seq"] * (3 * f + 2 * d) * 2
    return weights + kv + act


def run_c5(args):
    """Config 5: for each micro-batch count m of the sweep, pipeline_generate of 2m prompts (2048 tokens) and 128
    greedy new tokens through p = N stages (with the overlapped token ring when m >= p, else the reference's
    step-by-step loop), after a pipeline_forward of the prompts alone (the prefill phase). Reports per m the tokens/s
    of the whole generation (prompt + new tokens), of the prefill, of the decode (generation minus prefill time), and
    the measured bubble of the generation beside the analytic (p - 1) / (m + p - 1). A sweep point whose stage would
    not fit in device memory is reported as skipped."""
    import torch.distributed as dist

    from forgeserve_b200 import ModelConfig, PipelineStage, PipelineState, _lib, bubble_fraction, pipeline_forward
    from forgeserve_b200 import pipeline_generate
    from forgeserve_b200.weights import init_stage_

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=900))
    cfg = ModelConfig(**C5_CFG)
    sweep = [int(x) for x in args.c5_sweep.split(",")] if args.c5_sweep else list(C5["sweep"])

    def red(x, op):
        t = torch.tensor([float(x)], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=op)
        return float(t)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    free0 = torch.cuda.mem_get_info(dev)[0]
    fits = [red(c5_stage_bytes(cfg, world, rank, m) < 0.92 * free0, dist.ReduceOp.MIN if world > 1 else None) > 0
            for m in sweep]
    stage = PipelineStage(cfg, rank, world, device=dev, dtype=torch.bfloat16).eval()
    init_stage_(stage, seed=1234, std=0.02)
    stream = torch.cuda.current_stream(dev)
    launches0 = _lib.launch_count()
    points, total_tokens, total_ms = [], 0, 0.0
    sampler = ClockSampler([local] if world == 1 else range(world))
    with sampler:
        for m, ok in zip(sweep, fits):
            B = C5["rows"] * m
            if not ok:
                points.append({"microbatches": m, "rows": B, "skipped": "the stage does not fit in device memory"})
                continue
            g = torch.Generator().manual_seed(100 + m)
            prompt = torch.randint(0, cfg.vocab_size, (B, C5["seq"]), generator=g)
            for _ in range(max(args.warmup, 1)):
                pipeline_generate(stage, prompt, 2, m, seq_chunks=args.seq_chunks)
            barrier()
            pre_ms = gen_ms = 0.0
            busy = 0.0
            for _ in range(args.steps):
                state = PipelineState(stage, B, m)
                e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
                e0.record(stream)
                pipeline_forward(stage, state, prompt.to(dev) if stage.is_first else None, C5["seq"], last_only=True,
                                 seq_chunks=args.seq_chunks)
                e1.record(stream)
                del state
                barrier()
                stage.trace = []
                e1b = torch.cuda.Event(enable_timing=True)
                e1b.record(stream)
                pipeline_generate(stage, prompt, C5["new_tokens"], m, seq_chunks=args.seq_chunks)
                e2.record(stream)
                torch.cuda.synchronize()
                busy += sum(a.elapsed_time(b) for _, a, b in stage.trace)
                stage.trace = None
                pre_ms += e0.elapsed_time(e1)
                gen_ms += e1b.elapsed_time(e2)
                barrier()
            pre_ms = red(pre_ms, dist.ReduceOp.MAX if world > 1 else None)
            gen_ms = red(gen_ms, dist.ReduceOp.MAX if world > 1 else None)
            busy = red(busy, dist.ReduceOp.SUM if world > 1 else None)
            n_tok = B * (C5["seq"] + C5["new_tokens"]) * args.steps
            total_tokens += n_tok
            total_ms += gen_ms
            points.append({
                "microbatches": m, "rows": B, "overlapped": m >= world > 1,
                "tokens_per_s": round(n_tok / (gen_ms / 1e3), 1),
                "prefill_tokens_per_s": round(B * C5["seq"] * args.steps / (pre_ms / 1e3), 1),
                "decode_tokens_per_s": round(B * C5["new_tokens"] * args.steps / (max(gen_ms - pre_ms, 1e-6) / 1e3), 1),
                "ms_per_generation": round(gen_ms / args.steps, 1),
                "bubble": {"measured": round(1.0 - busy / (world * gen_ms), 4),
                           "analytic": round(bubble_fraction(world, m), 4)}})
    launches = red(_lib.launch_count() - launches0, dist.ReduceOp.SUM if world > 1 else None)
    result = None
    if rank == 0:
        result = {
            "metric": "PP generation tokens/s (prompt + new tokens), 70B-shape bf16 (config 5)",
            "value": round(total_tokens / (total_ms / 1e3), 1) if total_ms > 0 else None, "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": max(args.warmup, 1),
            "ms_per_step": round(total_ms / max(args.steps, 1), 1), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: seeded token ids, seeded N(0, 0.02) weights (no checkpoint or dataset)",
            "config": {"workload": C5_WORKLOAD, "stages": world, "parallelism": f"pp{world}",
                       "head": "on the last stage (last position only)", "prompt_pieces": args.seq_chunks},
            "sweep": points, "gpu_launches": int(launches), "clocks": sampler.summary(),
        }
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return result


def gemm_traffic():
    """DRAM bytes per launch of the profiled gate/up GEMM launch, from the committed ncu summary (or None)."""
    p = ROOT / "profiles" / "gemm_tc_8b_gateup.txt"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.startswith("dram_bytes_per_launch:"):
            try:
                return int(line.split(":")[1].split()[0])
            except (ValueError, IndexError):
                return None
    return None


# ------------------------------------------------------------------------------------------- CPU baseline
def cpu_sample(steps: int, warmup: int, spec=None):
    """The oracle (CPU restatement of the reference path, fp32, all host threads) on a bounded sample of the
    workload: one decoder layer and the head on one row of the workload's sequence length; tokens/s for the whole
    model is seq / (n_layers * t_layer + t_head)."""
    from oracle import forge_oracle as O
    spec = spec or PREFILL["c3"]
    seq = spec["seq"]
    cfg = O.Cfg(**spec["cfg"])
    threads = torch.get_num_threads()
    g = torch.Generator().manual_seed(0)
    names = O.param_order(cfg)
    sd = {}
    for name, shape in names:
        if name.startswith("layers.0.") or name in ("norm.weight",):
            sd[name] = torch.randn(shape, generator=g) * 0.02 if len(shape) > 1 else torch.ones(shape)
    sd["lm_head.weight"] = torch.randn(cfg.vocab_size, cfg.d_model, generator=g) * 0.02
    cos, sin = O.rope_tables(cfg.head_dim, cfg.max_seq_len, cfg.rope_theta)
    x = torch.randn(1, seq, cfg.d_model, generator=g)
    pos = torch.arange(seq)[None]
    times = []
    for i in range(warmup + steps):
        t0 = time.perf_counter()
        y = O.block(sd, 0, x, cfg, cos, sin, pos, O.ContiguousCache())
        t1 = time.perf_counter()
        O.head(sd, y, cfg)
        t2 = time.perf_counter()
        if i >= warmup:
            times.append((t1 - t0, t2 - t1))
    t_layer = statistics.median(t for t, _ in times)
    t_head = statistics.median(h for _, h in times)
    per_row = cfg.n_layers * t_layer + t_head
    return {"value": round(seq / per_row, 2), "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"oracle fp32: 1 of {cfg.n_layers} layers + final norm/head on 1 x {seq} tokens per step "
                      f"(measured: t_layer {t_layer:.3f} s, t_head {t_head:.3f} s per step), value extrapolated "
                      f"to the {cfg.n_layers}-layer model: {seq} tokens / ({cfg.n_layers} t_layer + t_head)",
            "sample_ms_per_step": round((t_layer + t_head) * 1e3, 3),
            "extrapolated_ms_per_row": round(per_row * 1e3, 3)}


def run_reference(args, spec):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    t0 = time.perf_counter()
    cb = cpu_sample(args.steps, args.warmup, spec)
    wall = time.perf_counter() - t0
    seq = spec["seq"]
    # ms_per_step is the measured time of one step of the sample that ran (one layer and the head on one row);
    # the whole model's time for that row, from which `value` comes, is extrapolated_ms_per_row
    return {"metric": spec["metric"], "value": cb["value"], "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": cb["sample_ms_per_step"],
            "extrapolated_ms_per_row": cb["extrapolated_ms_per_row"], "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "impl": "reference",
            "data": "synthetic: random fp32 weights (std 0.02) and activations",
            "config": {"workload": spec["workload"], "global_batch": spec["microbatches"] * spec["rows"],
                       "seq_len": seq, "microbatches": spec["microbatches"], "stages": world, "parallelism": "cpu"},
            "cpu_baseline": cb,
            "e2e": {"value": cb["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "wall_s": round(wall, 1)}


def profile_case(name: str, reps: int, timed: bool = False):
    """A few launches of one kernel on a small case (inputs larger than L2, a few GB at most) for ncu captures."""
    from forgeserve_b200 import _lib as L
    from forgeserve_b200 import ops
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)

    def rnd(*shape, scale=1.0):
        return (torch.randn(*shape, device=dev, generator=g) * scale).bfloat16()

    M, d, F, nh, nkv, hd, V = MB_ROWS * SEQ, CFG["d_model"], CFG["ffn_dim"], CFG["n_heads"], CFG["n_kv_heads"], 128, \
        CFG["vocab_size"]
    if name == "gemm_gateup":          # one micro-batch's gate/up projection: M 8192, N 2 x 14336, K 4096
        a, w = rnd(M, d), rnd(2 * F, d, scale=0.02)
        fn = lambda: ops.linear(a, w, L.FS_EPI_SWIGLU)
        work = (2.0 * M * 2 * F * d, "FLOP")
    elif name == "gemm_qkv":
        a, w = rnd(M, d), rnd((nh + 2 * nkv) * hd, d, scale=0.02)
        fn = lambda: ops.linear(a, w)
        work = (2.0 * M * w.shape[0] * d, "FLOP")
    elif name == "gemm_down":
        a, w, x = rnd(M, F), rnd(d, F, scale=0.02), rnd(M, d)
        fn = lambda: ops.linear(a, w, L.FS_EPI_RESIDUAL, residual=x, out=x)
        work = (2.0 * M * d * F, "FLOP")
    elif name == "gemm_head":
        a, w = rnd(M, d), rnd(V, d, scale=0.02)
        out = torch.empty(M, V, device=dev, dtype=torch.bfloat16)
        fn = lambda: ops.linear(a, w, out=out)
        work = (2.0 * M * V * d, "FLOP")
    elif name.startswith(("gemm_decode_", "cublas_decode_")) and not name.endswith("_projections"):
        # a C4 decode step's projections (gemm_decode_<proj>[@rows], 64 rows); gateup4k: gate/up with 4x the K (a
        # longer weight stream, to separate the per-launch cost from the streaming rate); cublas_decode_<proj>:
        # the same product by torch's cuBLAS matmul, store only, for comparison
        lib = name.startswith("cublas_")
        proj, _, r = name[len("cublas_decode_" if lib else "gemm_decode_"):].partition("@")
        rows = int(r) if r else 64
        n_k = {"qkv": ((nh + 2 * nkv) * hd, d), "o": (d, nh * hd), "gateup": (2 * F, d), "down": (d, F),
               "gateup4k": (2 * F, 4 * d)}
        if proj not in n_k:
            raise SystemExit(f"unknown profile case {name}")
        n, k = n_k[proj]
        a, w = rnd(rows, k), rnd(n, k, scale=0.02)
        if lib:
            out = torch.empty(rows, n, device=dev, dtype=torch.bfloat16)
            fn = lambda: torch.matmul(a, w.t(), out=out)
        elif proj in ("o", "down"):
            x = rnd(rows, n)
            fn = lambda: ops.linear(a, w, L.FS_EPI_RESIDUAL, residual=x, out=x)
        elif proj.startswith("gateup"):
            fn = lambda: ops.linear(a, w, L.FS_EPI_SWIGLU)
        else:
            fn = lambda: ops.linear(a, w)
        work = (2.0 * n * k + 2.0 * rows * (k + n), "B")    # the weights once, the rows in and out
    elif name == "attention":          # one micro-batch's causal prefill attention: 4 x 2048 queries, 32/8 heads
        kc, vc = rnd(MB_ROWS, nkv, SEQ, hd), rnd(MB_ROWS, nkv, SEQ, hd)
        q = rnd(M, (nh + 2 * nkv) * hd)
        pos = torch.arange(SEQ, device=dev)[None].expand(MB_ROWS, SEQ).contiguous()
        out = torch.empty(M, nh * hd, device=dev, dtype=torch.bfloat16)
        table = torch.arange(MB_ROWS, device=dev)
        desc = ops.contiguous_desc(kc, vc, table)
        fn = lambda: ops.attention(q[:, : nh * hd], desc, SEQ, pos, out, MB_ROWS, SEQ, nh, nkv, hd)
        work = (4.0 * MB_ROWS * nh * hd * SEQ * (SEQ + 1) / 2, "FLOP")
    elif name == "rope_kv":
        kc, vc = rnd(MB_ROWS, nkv, SEQ, hd), rnd(MB_ROWS, nkv, SEQ, hd)
        q = rnd(M, (nh + 2 * nkv) * hd)
        pos = torch.arange(SEQ, device=dev)[None].expand(MB_ROWS, SEQ).contiguous()
        from forgeserve_b200.model import precompute_rope
        cos, sin = (t.to(dev) for t in precompute_rope(hd, CFG["max_seq_len"], CFG["rope_theta"]))
        desc = ops.contiguous_desc(kc, vc, torch.arange(MB_ROWS, device=dev))
        fn = lambda: ops.rope_kv_write(q, cos, sin, pos, desc, MB_ROWS, SEQ, nh, nkv, hd, 0, False)
        work = (2.0 * M * (nh + 2 * nkv) * hd * 2, "B")     # q rotated in place; k, v read and stored
    elif name == "rmsnorm":
        x, w = rnd(M, d), rnd(d)
        fn = lambda: ops.rmsnorm(x, w, 1e-5)
        work = (2.0 * M * d * 2, "B")
    elif name == "decode":             # one layer's decode attention of the C4 batch: 64 rows, paged bs 16
        import random
        rng = random.Random(0)
        bs, rows = 16, 64
        lengths = [rng.randint(512, 4096) + 128 for _ in range(rows)]       # mid-generation context lengths
        widths = [-(-(n + 1) // bs) for n in lengths]
        nblk = sum(widths) + 64
        blocks = list(range(nblk))
        rng.shuffle(blocks)
        it = iter(blocks)
        W = max(widths)
        table = torch.tensor([[next(it) for _ in range(w)] + [0] * (W - w) for w in widths], device=dev)
        pool_k, pool_v = rnd(nblk, nkv, bs, hd), rnd(nblk, nkv, bs, hd)
        q = rnd(rows, nh * hd)
        out = torch.empty_like(q)
        positions = torch.tensor([[n] for n in lengths], device=dev)
        desc = ops.paged_desc(pool_k, pool_v, table)
        kv_bytes = sum(n + 1 for n in lengths) * nkv * hd * 2 * 2
        print(json.dumps({"decode_kv_bytes": kv_bytes, "keys": sum(n + 1 for n in lengths),
                          "splits_workspace": L.load().fs_attention_decode_workspace(rows, nh, nkv, hd, W * bs)}))
        fn = lambda: ops.attention_decode(q, desc, W * bs, positions, out, rows, nh, nkv, hd)
        work = (kv_bytes + 2.0 * rows * nh * hd * 2, "B")  # K and V of every key, q in, o out
    elif name in ("prefill_paged", "prefill_contiguous"):   # one config-4 prefill step: 1 prompt of 2300 tokens
        from forgeserve_b200 import ForgeModel, ModelConfig
        from forgeserve_b200.kv import new_contiguous_cache
        from forgeserve_b200.paged import PagedKVPool
        from forgeserve_b200.weights import init_model_
        import random
        cfg = ModelConfig(**CFG)
        model = ForgeModel(cfg, device=dev, dtype=torch.bfloat16).eval()
        init_model_(model, seed=1234, std=0.02)
        T = 2300
        idx = torch.randint(0, cfg.vocab_size, (1, T), generator=torch.Generator().manual_seed(3)).to(dev)
        pos = torch.arange(T, device=dev)[None]
        if name == "prefill_paged":
            bs = 16
            nblk = -(-T // bs)
            pool = PagedKVPool(cfg, 4 * nblk, bs, dtype=torch.bfloat16, device=dev)
            blocks = list(range(4 * nblk))
            random.Random(5).shuffle(blocks)
            table = torch.tensor([blocks[:nblk]], device=dev)
            fn = lambda: model(idx, pos, pool.views(table, pos), last_only=True)
        else:
            fn = lambda: model(idx, kv=new_contiguous_cache(cfg.n_layers, cfg.max_seq_len), last_only=True)
        flops = T * (2 * (d * (nh + 2 * nkv) * hd + nh * hd * d + 3 * d * F) * cfg.n_layers + 2 * d * V / T) \
            + 2 * nh * T * T * hd * cfg.n_layers
        work = (float(flops), "FLOP")
    elif name in ("decode_projections", "cublas_decode_projections"):
        # a decode layer's four projections back to back, 64 rows, 8 layers per replay; the cublas_ form makes the
        # same four products with torch's cuBLAS matmul, store only (no residual add, no SwiGLU), for comparison
        rows, per_replay = 64, 8
        wqkv, wo = rnd((nh + 2 * nkv) * hd, d, scale=0.02), rnd(d, nh * hd, scale=0.02)
        wgu, wd = rnd(2 * F, d, scale=0.02), rnd(d, F, scale=0.02)
        x, h, a = rnd(rows, d), rnd(rows, d), rnd(rows, nh * hd)
        outs = [torch.empty(rows, n, device=dev, dtype=torch.bfloat16) for n in (wqkv.shape[0], d, 2 * F, d)]
        gin = rnd(rows, F)

        def projections():
            for _ in range(per_replay):
                if name.startswith("cublas_"):
                    torch.matmul(h, wqkv.t(), out=outs[0])
                    torch.matmul(a, wo.t(), out=outs[1])
                    torch.matmul(h, wgu.t(), out=outs[2])
                    torch.matmul(gin, wd.t(), out=outs[3])
                    continue
                ops.linear(h, wqkv)
                ops.linear(a, wo, L.FS_EPI_RESIDUAL, residual=x, out=x)
                gg = ops.linear(h, wgu, L.FS_EPI_SWIGLU)
                ops.linear(gg, wd, L.FS_EPI_RESIDUAL, residual=x, out=x)

        cap = torch.cuda.Stream(dev)
        cap.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(cap):
            projections()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=cap):
            projections()

        def fn():
            graph.replay()
        wbytes = sum(t.numel() * 2 for t in (wqkv, wo, wgu, wd))
        work = (per_replay * wbytes, "B")
    elif name == "decode_layer":       # one whole decode layer of the C4 batch (8 layers per CUDA graph replay)
        import random
        from forgeserve_b200 import ModelConfig
        from forgeserve_b200.model import Block, RopeTables, layer_forward_
        from forgeserve_b200.paged import PagedKVPool
        from forgeserve_b200.weights import layer_shapes, seeded_tensor
        rng = random.Random(0)
        bs, rows, per_replay = 16, 64, 8
        cfg = ModelConfig(**CFG)
        lengths = [rng.randint(512, 4096) + 128 for _ in range(rows)]
        widths = [-(-(n + 1) // bs) for n in lengths]
        nblk = sum(widths) + 64
        blocks = list(range(nblk))
        rng.shuffle(blocks)
        it = iter(blocks)
        W = max(widths)
        table = torch.tensor([[next(it) for _ in range(w)] + [0] * (W - w) for w in widths], device=dev)
        pool = PagedKVPool(cfg, nblk, bs, dtype=torch.bfloat16, device=dev, n_layers=1)
        pool.k[0].normal_(generator=g)
        pool.v[0].normal_(generator=g)
        blk = Block(cfg, device=dev, dtype=torch.bfloat16)
        with torch.no_grad():
            for pname, prm in blk.named_parameters():
                full = "layers.0." + pname
                prm.copy_(seeded_tensor(full, layer_shapes(cfg, 0)[full], 1234, 0.02, device=dev, dtype=prm.dtype))
        positions = torch.tensor([[n] for n in lengths], device=dev)
        view = pool.views(table, positions)[0]
        cos, sin = RopeTables(cfg).on(dev)
        x = rnd(rows, 1, d)
        x0 = x.clone()

        def layers():
            for _ in range(per_replay):
                layer_forward_(blk, x, positions, view, cos, sin)

        cap = torch.cuda.Stream(dev)                      # warm-up on the capture stream: its per-stream GEMM
        cap.wait_stream(torch.cuda.current_stream(dev))   # counters and workspaces exist before the capture
        with torch.cuda.stream(cap):
            layers()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=cap):
            layers()
        x.copy_(x0)

        def fn():
            graph.replay()
        weight_bytes = sum(prm.numel() * prm.element_size() for prm in blk.parameters())
        kv_bytes = sum(n + 1 for n in lengths) * nkv * hd * 2 * 2
        print(json.dumps({"decode_layer_weight_bytes": weight_bytes, "kv_bytes": kv_bytes, "layers_per_launch": 8}))
        work = (per_replay * (weight_bytes + kv_bytes + 4.0 * rows * d * 2), "B")
    else:
        raise SystemExit(f"unknown profile case {name}")
    for _ in range(reps):
        fn()
    torch.cuda.synchronize()
    res = {"profile_case": name, "reps": reps}
    if timed:
        # cold-L2 launches timed with CUDA events on the launching stream (a 256 MB write between launches)
        flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
        st = torch.cuda.current_stream(dev)
        times = []
        for _ in range(max(reps, 3) * 4):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            fn()
            e1.record(st)
            e1.synchronize()
            times.append(e0.elapsed_time(e1) * 1e3)
        us = statistics.median(times)
        amount, unit = work
        res.update({"us_median": round(us, 2), "us_min": round(min(times), 2),
                    ("TFLOP/s" if unit == "FLOP" else "GB/s"):
                        round(amount / (us * 1e-6) / (1e12 if unit == "FLOP" else 1e9), 1),
                    "work_per_launch": amount, "work_unit": unit})
    res["device_error"] = L.device_error()
    print(json.dumps(res))


def auto_seq_chunks(workload: str, gpus: int) -> int:
    """Sequence pieces per micro-batch for the prefill workloads by default: pieces cut the pipeline's fill and drain
    from (p - 1) / (m + p - 1) to (p - 1) / (m s + p - 1), but every piece's GEMMs have s times fewer rows. Measured on
    config 3: at 2 GPUs 4 pieces gave 132.4k tokens/s against 137.9k whole; at 4 GPUs 248.6k against 242.5k (with one
    NCCL channel per stage pair; with two, the middle stages lost 12 % of their GEMM rate and pieces gave 238.7k); at
    8 GPUs 445.0k against 406.4k (two channels). So pieces from 4 stages on, while a piece keeps >= 2048 GEMM rows."""
    if workload not in PREFILL or gpus < 4:
        return 1
    spec = PREFILL[workload]
    rows = spec["rows"] * spec["seq"]
    return max(1, min(4, rows // 2048))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--whole-head", action="store_true", help="N > 1: keep the whole output head on the last stage")
    ap.add_argument("--seq-chunks", type=int, default=0,
                    help="c3, c2, c5: pieces per micro-batch along the sequence in the prompt's forward; c4 with "
                         "N > 1: pieces per prefill (pipeline_forward's seq_chunks, PipelineEngine's "
                         "prefill_chunks). 0 (default): auto_seq_chunks (4 for c3 and 2 for c2 from 4 GPUs on, else 1)")
    ap.add_argument("--workload", choices=["c3", "c2", "c4", "c5"], default="c3",
                    help="c3: 8B-shape pipeline prefill (the headline metric); c2: 1B-shape pipeline prefill; "
                         "c4: continuous-batching decode; c5: 70B-shape generation, micro-batch sweep")
    ap.add_argument("--c5-sweep", default="", help="c5: comma-separated micro-batch counts (default 4,8,16,32)")
    ap.add_argument("--microbatches", type=int, default=0, help="c4 with N > 1: micro-batches per engine step")
    ap.add_argument("--no-graphs", action="store_true", help="c4: launch every decode kernel from Python")
    ap.add_argument("--no-windows", action="store_true", help="c4 with N > 1: drain the pipeline after every step")
    ap.add_argument("--profile-case", default=None,
                    help="run a few launches of one kernel (for ncu) and exit; a comma-separated list runs several")
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--timed", action="store_true", help="with --profile-case: also time cold-L2 launches")
    args = ap.parse_args()
    if args.seq_chunks <= 0:
        args.seq_chunks = auto_seq_chunks(args.workload, args.gpus)
    if args.profile_case:
        for name in args.profile_case.split(","):
            profile_case(name, args.reps, args.timed)
        return
    if args.warmup < 3 and args.impl == "ours":
        print("warning: fewer than 3 warm-up steps", file=sys.stderr)
    if args.workload == "c5":
        if args.impl == "reference":
            res = None if int(os.environ.get("RANK", "0")) else {
                "impl": "reference",
                "metric": "PP generation tokens/s (prompt + new tokens), 70B-shape bf16 (config 5)",
                "unavailable": "config 5 is not run on the CPU (a 70B fp32 model is about 280 GB)"}
        else:
            res = run_c5(args)
    elif args.workload == "c4":
        if args.impl == "reference":
            res = None if int(os.environ.get("RANK", "0")) else {
                "impl": "reference", "metric": "continuous-batching decode tokens/s, 8B-shape bf16 (config 4)",
                "unavailable": "config 4 is not run on the CPU (the reference's Engine is fp32 on the host cores)"}
        else:
            res = run_c4(args)
    elif args.impl == "reference":
        res = run_reference(args, PREFILL[args.workload])
    else:
        res = run_ours(args, PREFILL[args.workload])
        if res is not None and args.gpus == 1 and not args.no_cpu_baseline:
            torch.cuda.empty_cache()
            res["cpu_baseline"] = cpu_sample(steps=2, warmup=1, spec=PREFILL[args.workload])
    if res is not None:
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
