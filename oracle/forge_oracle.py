"""ORACLE — test infrastructure only. A CPU restatement of forgeserve's pipeline-parallel forward path, used by
tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference arm as the checker and the timed
CPU baseline. The product (forgeserve_b200) never imports this module.

Restated from the reference (omkarbhad/forgeserve; file:line of that project):
  rms_norm            forgeserve/model.py:29-31
  rope_tables         forgeserve/model.py:34-37
  apply_rope          forgeserve/model.py:40-45
  attention           forgeserve/model.py:62-78 (repeat_interleave :70-71, mask :75, SDPA :76 written out as
                      softmax(QK^T / sqrt(hd) + mask) V in fp32; or, with attn_core=sdpa_torch, the reference's
                      own torch scaled_dot_product_attention call in the inputs' dtype)
  swiglu              forgeserve/model.py:92-93
  block               forgeserve/model.py:104-106
  model_forward       forgeserve/model.py:140-159 (tied head :120, :137-138)
  ContiguousCache     forgeserve/kv.py:10-29
  PagedPool           forgeserve/paged.py:42-82 (scatter :74-78, gather :80-81)
  stage_layers        forgeserve/pipeline.py:26-36
  microbatch_sizes    forgeserve/pipeline.py:86-87 (torch.tensor_split rows)
  pipeline_forward    forgeserve/pipeline.py:95-118 (stages simulated in order in one process: every
                      micro-batch visits stage 0 .. p-1, the data each stage would send is what the next receives)
  greedy_generate     forgeserve/sampling.py:24-35 with temperature 0 (argmax, first index on ties)
  shard               forgeserve/tensor_parallel.py:25-39 (q/k/v/gate/up by output rows, wo/down by input columns)
  shard_cfg           forgeserve/model.py:54,87 (a shard's head and hidden counts; head_dim unchanged)
  model_forward_tp    forgeserve/model.py:77,93,104-106 with parallel.py:20-26 (the shards' partial outputs of
                      attention and of the MLP summed before each residual add; shards simulated in one process)

Arithmetic is plain torch on whatever device the tensors are on (CPU in every CPU test), in the dtype of the
weights passed in: fp32 for the 1e-4 parity mode; bf16 reproduces the reference's bf16 rounding points.
Parity pin: tests/test_oracle.py checks this file against golden outputs of the reference itself
(tests/golden/, made by tests/golden/make_golden.py).
"""

import math
from typing import Dict, List, Optional, Tuple

import torch


class Cfg:
    """The subset of ModelConfig the oracle needs (built from a plain dict)."""

    def __init__(self, vocab_size, d_model, n_layers, n_heads, n_kv_heads, ffn_dim=None, max_seq_len=256,
                 rope_theta=10000.0, norm_eps=1e-5):
        self.vocab_size, self.d_model, self.n_layers = vocab_size, d_model, n_layers
        self.n_heads, self.n_kv_heads = n_heads, n_kv_heads
        self.ffn_dim = ffn_dim if ffn_dim is not None else (int(8 / 3 * d_model) + 63) // 64 * 64
        self.max_seq_len, self.rope_theta, self.norm_eps = max_seq_len, rope_theta, norm_eps
        self.head_dim = d_model // n_heads


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    x32 = x.float()
    return (x32 * torch.rsqrt(x32.pow(2).mean(-1, keepdim=True) + eps)).to(x.dtype) * w


def rope_tables(head_dim: int, max_len: int, theta: float) -> Tuple[torch.Tensor, torch.Tensor]:
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2).float() / head_dim))
    ang = torch.outer(torch.arange(max_len).float(), inv_freq)
    return ang.cos(), ang.sin()


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, positions: torch.Tensor) -> torch.Tensor:
    """x (B, H, T, D), positions (B, T); half-split rotation in x's dtype."""
    c = cos[positions][:, None].to(x.dtype)
    s = sin[positions][:, None].to(x.dtype)
    half = x.shape[-1] // 2
    x1, x2 = x[..., :half], x[..., half:]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)


def sdpa(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, mask: torch.Tensor) -> torch.Tensor:
    """softmax(q k^T / sqrt(D), masked) v, accumulated in fp32, result in q's dtype."""
    scale = 1.0 / math.sqrt(q.shape[-1])
    s = torch.matmul(q.float(), k.float().transpose(-1, -2)) * scale
    s = s.masked_fill(~mask, float("-inf"))
    p = torch.softmax(s, dim=-1)
    return torch.matmul(p, v.float()).to(q.dtype)


def sdpa_torch(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, mask: torch.Tensor) -> torch.Tensor:
    """The reference's own attention call (model.py:76): torch's fused scaled_dot_product_attention with the
    boolean mask, in the inputs' dtype. In fp32 on the CPU it equals `sdpa` within rounding; in bf16 on a GPU it is
    the kernel the reference's module itself would run there (bf16 probabilities into P V), one of several valid
    bf16 renderings of the same algebra."""
    return torch.nn.functional.scaled_dot_product_attention(q, k, v, attn_mask=mask)


class ContiguousCache:
    def __init__(self):
        self.k: Optional[torch.Tensor] = None
        self.v: Optional[torch.Tensor] = None

    @property
    def length(self) -> int:
        return 0 if self.k is None else self.k.shape[2]

    def update(self, k, v):
        self.k = k if self.k is None else torch.cat([self.k, k], dim=2)
        self.v = v if self.v is None else torch.cat([self.v, v], dim=2)
        return self.k, self.v


class PagedPool:
    """Per-layer pools (num_blocks, n_kv, block_size, hd) and the scatter/gather view of one step."""

    def __init__(self, cfg: Cfg, num_blocks: int, block_size: int, dtype=torch.float32):
        shape = (num_blocks, cfg.n_kv_heads, block_size, cfg.head_dim)
        self.k = [torch.zeros(shape, dtype=dtype) for _ in range(cfg.n_layers)]
        self.v = [torch.zeros(shape, dtype=dtype) for _ in range(cfg.n_layers)]
        self.block_size = block_size

    def view(self, layer: int, tables: torch.Tensor, positions: torch.Tensor):
        pool = self

        class _View:
            def update(self, k, v):
                bs = pool.block_size
                b, h, t, d = k.shape
                phys = tables.gather(1, positions // bs).reshape(-1)
                off = (positions % bs).reshape(-1)
                pool.k[layer][phys, :, off, :] = k.permute(0, 2, 1, 3).reshape(b * t, h, d)
                pool.v[layer][phys, :, off, :] = v.permute(0, 2, 1, 3).reshape(b * t, h, d)
                k_all = pool.k[layer][tables].permute(0, 2, 1, 3, 4).reshape(b, h, -1, d)
                v_all = pool.v[layer][tables].permute(0, 2, 1, 3, 4).reshape(b, h, -1, d)
                return k_all, v_all

        return _View()


def attention(sd: Dict[str, torch.Tensor], p: str, x: torch.Tensor, cfg: Cfg, cos, sin, positions, kv,
              attn_core=None) -> torch.Tensor:
    b, t, _ = x.shape
    nh, nkv, hd = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
    q = (x @ sd[p + "attn.wq.weight"].t()).view(b, t, nh, hd).transpose(1, 2)
    k = (x @ sd[p + "attn.wk.weight"].t()).view(b, t, nkv, hd).transpose(1, 2)
    v = (x @ sd[p + "attn.wv.weight"].t()).view(b, t, nkv, hd).transpose(1, 2)
    q, k = apply_rope(q, cos, sin, positions), apply_rope(k, cos, sin, positions)
    k_all, v_all = kv.update(k, v)
    rep = nh // nkv
    k_all = k_all.repeat_interleave(rep, dim=1)
    v_all = v_all.repeat_interleave(rep, dim=1)
    s = k_all.shape[2]
    mask = (torch.arange(s, device=positions.device)[None, None, :] <= positions[:, :, None])[:, None]
    out = (attn_core or sdpa)(q, k_all, v_all, mask)
    return out.transpose(1, 2).reshape(b, t, -1) @ sd[p + "attn.wo.weight"].t()


def swiglu(sd, p: str, x: torch.Tensor) -> torch.Tensor:
    g = x @ sd[p + "mlp.w_gate.weight"].t()
    u = x @ sd[p + "mlp.w_up.weight"].t()
    return (torch.nn.functional.silu(g) * u) @ sd[p + "mlp.w_down.weight"].t()


def block(sd, i: int, x, cfg: Cfg, cos, sin, positions, kv, attn_core=None):
    p = f"layers.{i}."
    x = x + attention(sd, p, rms_norm(x, sd[p + "attn_norm.weight"], cfg.norm_eps), cfg, cos, sin, positions, kv,
                      attn_core)
    return x + swiglu(sd, p, rms_norm(x, sd[p + "mlp_norm.weight"], cfg.norm_eps))


def head(sd, x, cfg: Cfg):
    w = sd["lm_head.weight"] if "lm_head.weight" in sd else sd["tok_emb.weight"]
    return rms_norm(x, sd["norm.weight"], cfg.norm_eps) @ w.t()


def model_forward(sd: Dict[str, torch.Tensor], cfg: Cfg, idx: torch.Tensor, positions: Optional[torch.Tensor] = None,
                  kv: Optional[List] = None, layers: Optional[range] = None, attn_core=None) -> torch.Tensor:
    """Single-process forward: idx (B, T) -> logits (B, T, V), on idx's device (the reference's model is
    device-agnostic: its positions follow idx.device, model.py:153, and its RoPE buffers move with it)."""
    b, t = idx.shape
    cos, sin = (x.to(idx.device) for x in rope_tables(cfg.head_dim, cfg.max_seq_len, cfg.rope_theta))
    if kv is None:
        kv = [ContiguousCache() for _ in range(cfg.n_layers)]
    if positions is None:
        positions = (kv[0].length + torch.arange(t, device=idx.device))[None, :].expand(b, t)
    positions = positions.to(idx.device)
    if int(positions.max()) >= cfg.max_seq_len:
        raise ValueError("position exceeds max_seq_len")
    x = sd["tok_emb.weight"][idx]
    for i in (layers if layers is not None else range(cfg.n_layers)):
        x = block(sd, i, x, cfg, cos, sin, positions, kv[i], attn_core)
    return head(sd, x, cfg)


_BY_ROWS = ("attn.wq.weight", "attn.wk.weight", "attn.wv.weight", "mlp.w_gate.weight", "mlp.w_up.weight")
_BY_COLUMNS = ("attn.wo.weight", "mlp.w_down.weight")


def shard(sd: Dict[str, torch.Tensor], rank: int, size: int) -> Dict[str, torch.Tensor]:
    """Tensor-parallel shard `rank` of `size` of a full state dict (embedding, norms and head replicated)."""
    out = {}
    for name, w in sd.items():
        if name.endswith(_BY_ROWS):
            n = w.shape[0] // size
            out[name] = w[rank * n : (rank + 1) * n]
        elif name.endswith(_BY_COLUMNS):
            n = w.shape[1] // size
            out[name] = w[:, rank * n : (rank + 1) * n]
        else:
            out[name] = w
    return out


def shard_cfg(cfg: Cfg, size: int) -> Cfg:
    """The head and hidden-feature counts one shard holds (head_dim stays the model's)."""
    c = Cfg(cfg.vocab_size, cfg.d_model, cfg.n_layers, cfg.n_heads, cfg.n_kv_heads, cfg.ffn_dim, cfg.max_seq_len,
            cfg.rope_theta, cfg.norm_eps)
    c.n_heads, c.n_kv_heads, c.ffn_dim = cfg.n_heads // size, cfg.n_kv_heads // size, cfg.ffn_dim // size
    return c


def model_forward_tp(shards: List[Dict[str, torch.Tensor]], cfg: Cfg, idx: torch.Tensor,
                     kvs: Optional[List[List]] = None) -> torch.Tensor:
    """The reference's tensor-parallel forward with every shard in this process: shard r attends over its own
    heads with its own caches (kvs[r]); the partial attention and MLP outputs are summed in rank order (what the
    all-reduce computes) and added to the replicated residual stream."""
    size = len(shards)
    c = shard_cfg(cfg, size)
    b, t = idx.shape
    cos, sin = rope_tables(cfg.head_dim, cfg.max_seq_len, cfg.rope_theta)
    if kvs is None:
        kvs = [[ContiguousCache() for _ in range(cfg.n_layers)] for _ in range(size)]
    positions = (kvs[0][0].length + torch.arange(t))[None, :].expand(b, t)
    x = shards[0]["tok_emb.weight"][idx]
    for i in range(cfg.n_layers):
        p = f"layers.{i}."
        h = rms_norm(x, shards[0][p + "attn_norm.weight"], cfg.norm_eps)
        parts = [attention(sd, p, h, c, cos, sin, positions, kvs[r][i]) for r, sd in enumerate(shards)]
        x = x + sum(parts[1:], parts[0])
        h = rms_norm(x, shards[0][p + "mlp_norm.weight"], cfg.norm_eps)
        parts = [swiglu(sd, p, h) for sd in shards]
        x = x + sum(parts[1:], parts[0])
    return head(shards[0], x, cfg)


def stage_layers(n_layers: int, size: int) -> List[Tuple[int, int]]:
    if size > n_layers:
        raise ValueError("more pipeline stages than layers")
    base, extra = divmod(n_layers, size)
    out, lo = [], 0
    for r in range(size):
        hi = lo + base + (1 if r < extra else 0)
        out.append((lo, hi))
        lo = hi
    return out


def microbatch_sizes(batch: int, microbatches: int) -> List[int]:
    return [len(c) for c in torch.arange(batch).tensor_split(microbatches)]


class PipelineSim:
    """State of a p-stage pipeline simulated in one process: one cache per (micro-batch, layer)."""

    def __init__(self, cfg: Cfg, batch: int, stages: int, microbatches: int):
        self.cfg, self.stages = cfg, stages
        self.sizes = microbatch_sizes(batch, microbatches)
        self.split = stage_layers(cfg.n_layers, stages)
        self.caches = [[ContiguousCache() for _ in range(cfg.n_layers)] for _ in self.sizes]

    @property
    def length(self) -> int:
        return self.caches[0][0].length


def pipeline_forward(sd, sim: PipelineSim, idx: torch.Tensor, t: int) -> torch.Tensor:
    """What the last stage returns: logits (B, t, V), micro-batch by micro-batch, stage by stage."""
    cfg = sim.cfg
    cos, sin = rope_tables(cfg.head_dim, cfg.max_seq_len, cfg.rope_theta)
    start = sim.length
    outs, row = [], 0
    for mb, size in enumerate(sim.sizes):
        positions = (start + torch.arange(t))[None, :].expand(size, t)
        x = sd["tok_emb.weight"][idx[row : row + size]]
        for lo, hi in sim.split:                           # stage s receives what stage s-1 sent
            for i in range(lo, hi):
                x = block(sd, i, x, cfg, cos, sin, positions, sim.caches[mb][i])
        outs.append(head(sd, x, cfg))
        row += size
    return torch.cat(outs, dim=0)


def greedy_generate(sd, cfg: Cfg, prompt: torch.Tensor, max_new_tokens: int, attn_core=None) -> torch.Tensor:
    kv = [ContiguousCache() for _ in range(cfg.n_layers)]
    max_new_tokens = min(max_new_tokens, cfg.max_seq_len - prompt.shape[1])
    out = prompt
    logits = model_forward(sd, cfg, prompt, kv=kv, attn_core=attn_core)
    for _ in range(max_new_tokens):
        nxt = logits[:, -1].argmax(-1)[:, None]
        out = torch.cat([out, nxt], dim=1)
        logits = model_forward(sd, cfg, nxt, kv=kv, attn_core=attn_core)
    return out


def log_softmax_maxabs(a: torch.Tensor, b: torch.Tensor) -> float:
    """max |log_softmax(a) - log_softmax(b)| over the vocab axis, in fp32 (the bf16-mode tolerance metric)."""
    la = torch.log_softmax(a.float(), dim=-1)
    lb = torch.log_softmax(b.float(), dim=-1)
    return float((la - lb).abs().max())


# ------------------------------------------------------------------------------------------- test weights
def param_order(cfg: Cfg) -> List[Tuple[str, Tuple[int, ...]]]:
    """State-dict keys and shapes in ForgeModel.parameters() order (model.py:112-122; the tied head is the
    embedding and is listed once)."""
    d, hd = cfg.d_model, cfg.head_dim
    out = [("tok_emb.weight", (cfg.vocab_size, d))]
    for i in range(cfg.n_layers):
        p = f"layers.{i}."
        out += [(p + "attn_norm.weight", (d,)), (p + "attn.wq.weight", (cfg.n_heads * hd, d)),
                (p + "attn.wk.weight", (cfg.n_kv_heads * hd, d)), (p + "attn.wv.weight", (cfg.n_kv_heads * hd, d)),
                (p + "attn.wo.weight", (d, cfg.n_heads * hd)), (p + "mlp_norm.weight", (d,)),
                (p + "mlp.w_gate.weight", (cfg.ffn_dim, d)), (p + "mlp.w_up.weight", (cfg.ffn_dim, d)),
                (p + "mlp.w_down.weight", (d, cfg.ffn_dim))]
    out.append(("norm.weight", (d,)))
    return out


def test_model_weights(cfg: Cfg, seed: int = 1, scale: float = 0.25) -> Dict[str, torch.Tensor]:
    """The reference test suite's model (tests/conftest.py:18-27 of the reference): every parameter with 2+ dims
    replaced, in parameters() order, by randn(generator seeded `seed`) * scale; norms stay ones."""
    g = torch.Generator().manual_seed(seed)
    sd = {}
    for name, shape in param_order(cfg):
        sd[name] = torch.randn(shape, generator=g) * scale if len(shape) >= 2 else torch.ones(shape)
    sd["lm_head.weight"] = sd["tok_emb.weight"]
    return sd


def checksum(sd: Dict[str, torch.Tensor]) -> Dict[str, Tuple[float, float]]:
    return {k: (float(v.double().sum()), float(v.double().pow(2).sum())) for k, v in sd.items()}
