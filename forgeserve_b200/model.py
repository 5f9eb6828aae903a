"""LLaMA-style decoder (forgeserve/model.py:23-159) whose layers run as sm_100a kernels.

Modules and parameter names are the reference's (`layers.{i}.attn.{wq,wk,wv,wo}.weight`,
`layers.{i}.{attn_norm,mlp_norm}.weight`, `layers.{i}.mlp.{w_gate,w_up,w_down}.weight`, `tok_emb.weight`,
`norm.weight`, `lm_head.weight` tied to the embedding), so a reference state dict loads unchanged. Inside a
Block the q/k/v weights are row slices of one fused [Wq; Wk; Wv] tensor and gate/up of one [W_gate; W_up]
tensor (the parameters are views into them, so nothing is stored twice), and one decoder layer is:

    h   = rmsnorm(x)                              fs_rmsnorm
    qkv = h @ [Wq;Wk;Wv]^T                        fs_gemm (tcgen05)
    rope(q, k); k, v -> cache slots               fs_rope_kv_write
    a   = attention(q, cache)                     fs_attention (reads the cache through its block table)
    x  += a @ Wo^T                                fs_gemm, residual epilogue, in place
    h   = rmsnorm(x)                              fs_rmsnorm
    g   = silu(h @ Wg^T) * (h @ Wu^T)             fs_gemm, SwiGLU epilogue
    x  += g @ Wd^T                                fs_gemm, residual epilogue, in place

with the reference's rounding points kept in every kernel (see csrc/). Tensors must live on a CUDA device;
there is no CPU implementation.
"""

from typing import List, Optional

import torch
import torch.nn as nn

from . import _lib as L
from . import ops
from .config import ModelConfig
from .kv import ContiguousKV, new_contiguous_cache, row_table
from .paged import PagedLayerView
from .parallel import SINGLE, TPContext


class RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float = 1e-5, device=None, dtype=None):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim, device=device, dtype=dtype))

    def forward(self, x):
        return ops.rmsnorm(x, self.weight, self.eps)


def precompute_rope(head_dim: int, max_len: int, theta: float):
    """cos/sin tables (max_len, head_dim/2) in fp32, angles pos * theta^(-2i/head_dim) (model.py:34-37)."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2).float() / head_dim))
    angles = torch.outer(torch.arange(max_len).float(), inv_freq)
    return angles.cos(), angles.sin()


class RopeTables:
    """fp32 cos/sin tables per device; the kernels round them to the activation dtype as the reference does."""

    def __init__(self, cfg: ModelConfig):
        self.cos, self.sin = precompute_rope(cfg.head_dim, cfg.max_seq_len, cfg.rope_theta)
        self._dev = {}

    def on(self, device: torch.device):
        key = str(device)
        if key not in self._dev:
            self._dev[key] = (self.cos.to(device), self.sin.to(device))
        return self._dev[key]


def _fused(parts: List[nn.Parameter], cache_attr: str, owner: nn.Module) -> torch.Tensor:
    """Return one tensor whose consecutive row blocks are `parts`, re-pointing the parameters at views of it.

    Re-fuses when a parameter no longer aliases the fused tensor (after .to(), or replaced storage)."""
    fused = getattr(owner, cache_attr, None)
    if fused is not None and fused.dtype == parts[0].dtype and fused.device == parts[0].device:
        off, ok = 0, True
        for p in parts:
            n = p.shape[0]
            if p.data_ptr() != fused.data_ptr() + off * fused.stride(0) * fused.element_size() or p.shape[1:] != fused.shape[1:]:
                ok = False
                break
            off += n
        if ok and off == fused.shape[0]:
            return fused
    with torch.no_grad():
        fused = torch.cat([p.detach() for p in parts], dim=0).contiguous()
        off = 0
        for p in parts:
            n = p.shape[0]
            p.data = fused[off : off + n]
            off += n
    object.__setattr__(owner, cache_attr, fused)
    return fused


class Attention(nn.Module):
    """q/k/v/o projections of one layer (model.py:48-78); the computation lives in `layer_forward_`. Under tensor
    parallelism (tp.size > 1) this shard holds n_heads / size query heads and n_kv_heads / size KV heads (whole
    heads: q/k/v split by output rows, wo by input columns, model.py:47-58)."""

    def __init__(self, cfg: ModelConfig, tp: TPContext = SINGLE, device=None, dtype=None):
        super().__init__()
        cfg.check_tensor_parallel(tp.size)
        self.tp = tp
        self.hd = cfg.head_dim
        self.nh, self.nkv = cfg.n_heads // tp.size, cfg.n_kv_heads // tp.size
        self.rep = cfg.n_heads // cfg.n_kv_heads
        f = dict(bias=False, device=device, dtype=dtype)
        self.wq = nn.Linear(cfg.d_model, self.nh * self.hd, **f)
        self.wk = nn.Linear(cfg.d_model, self.nkv * self.hd, **f)
        self.wv = nn.Linear(cfg.d_model, self.nkv * self.hd, **f)
        self.wo = nn.Linear(self.nh * self.hd, cfg.d_model, **f)

    def wqkv(self) -> torch.Tensor:
        return _fused([self.wq.weight, self.wk.weight, self.wv.weight], "_wqkv", self)


class SwiGLU(nn.Module):
    """gate/up/down projections of one layer (model.py:81-93); under tensor parallelism ffn_dim / size hidden
    features of them (gate/up split by output rows, down by input columns)."""

    def __init__(self, cfg: ModelConfig, tp: TPContext = SINGLE, device=None, dtype=None):
        super().__init__()
        cfg.check_tensor_parallel(tp.size)
        self.tp = tp
        hidden = cfg.ffn_dim // tp.size
        f = dict(bias=False, device=device, dtype=dtype)
        self.w_gate = nn.Linear(cfg.d_model, hidden, **f)
        self.w_up = nn.Linear(cfg.d_model, hidden, **f)
        self.w_down = nn.Linear(hidden, cfg.d_model, **f)

    def w_gate_up(self) -> torch.Tensor:
        return _fused([self.w_gate.weight, self.w_up.weight], "_wgu", self)


def _bind_kv(kv, B: int, T: int, nkv: int, hd: int, dtype, device, positions: torch.Tensor):
    """Resolve a KV view into (descriptor, n_slots, slot_base, slot_from_pos, commit, keepalive)."""
    if isinstance(kv, ContiguousKV):
        base = kv.reserve(B, nkv, hd, T, dtype, device)
        k, v = kv.buffers()
        table = row_table(B, device)
        return ops.contiguous_desc(k, v, table), base + T, base, False, (lambda: kv.commit(T)), (k, v, table)
    if isinstance(kv, PagedLayerView):
        if kv.pool.k[kv.layer].dtype != dtype or kv.pool.device != torch.device(device):
            raise ValueError("paged pool dtype/device differs from the model's")
        if kv.positions.shape != positions.shape:
            raise ValueError("paged view positions must match the step's positions")
        return kv.descriptor(), kv.n_slots, 0, True, (lambda: None), (kv.tables,)
    return None


def layer_forward_(blk: "Block", x: torch.Tensor, positions: torch.Tensor, kv, rope_cos: torch.Tensor,
                   rope_sin: torch.Tensor) -> torch.Tensor:
    """One decoder layer (model.py:104-106) on x (B, T, d) in place. positions: (B, T) int64 on x's device."""
    B, T, d = x.shape
    a = blk.attn
    nh, nkv, hd = a.nh, a.nkv, a.hd
    M = B * T
    h = ops.rmsnorm(x, blk.attn_norm.weight, blk.attn_norm.eps)
    qkv = ops.linear(h, a.wqkv())
    qkv2 = qkv.view(M, (nh + 2 * nkv) * hd)
    bound = _bind_kv(kv, B, T, nkv, hd, x.dtype, x.device, positions)
    if bound is None:
        # Any other object with the view protocol: rotate into a scratch cache, hand k/v to kv.update(), and
        # attend over what it returns (keys at slots 0..S-1, as model.py:69-76).
        ks = torch.empty(B, nkv, T, hd, dtype=x.dtype, device=x.device)
        vs = torch.empty_like(ks)
        table = row_table(B, x.device)
        ops.rope_kv_write(qkv2, rope_cos, rope_sin, positions, ops.contiguous_desc(ks, vs, table), B, T, nh, nkv,
                          hd, slot_base=0, slot_from_pos=False)
        k_all, v_all = kv.update(ks, vs)
        k_all, v_all = k_all.contiguous(), v_all.contiguous()
        desc, n_slots = ops.contiguous_desc(k_all, v_all, table), k_all.shape[2]
        keep = (k_all, v_all, table)
    else:
        desc, n_slots, base, from_pos, commit, keep = bound
        ops.rope_kv_write(qkv2, rope_cos, rope_sin, positions, desc, B, T, nh, nkv, hd, slot_base=base,
                          slot_from_pos=from_pos)
    attn = torch.empty(B, T, nh * hd, dtype=x.dtype, device=x.device)
    if T == 1 and hd in (64, 128) and nh // nkv <= 8:
        # one new token per row (decode): split-KV kernel reading each K/V row once per KV head
        ops.attention_decode(qkv2[:, : nh * hd], desc, n_slots, positions, attn.view(M, nh * hd), B, nh, nkv, hd)
    else:
        ops.attention(qkv2[:, : nh * hd], desc, n_slots, positions, attn.view(M, nh * hd), B, T, nh, nkv, hd)
    if bound is not None:
        commit()
    del keep
    if a.tp.size == 1:
        ops.linear(attn, a.wo.weight, L.FS_EPI_RESIDUAL, residual=x, out=x)
    else:
        # row-parallel: this shard's partial sum (rounded as nn.Linear rounds), summed over the shards, then added
        # to the residual stream (x + all_reduce(wo(a)), model.py:77,105)
        x.add_(a.tp.all_reduce(ops.linear(attn, a.wo.weight)))
    ops.rmsnorm(x, blk.mlp_norm.weight, blk.mlp_norm.eps, out=h)
    g = ops.linear(h, blk.mlp.w_gate_up(), L.FS_EPI_SWIGLU)
    if blk.mlp.tp.size == 1:
        ops.linear(g, blk.mlp.w_down.weight, L.FS_EPI_RESIDUAL, residual=x, out=x)
    else:
        x.add_(blk.mlp.tp.all_reduce(ops.linear(g, blk.mlp.w_down.weight)))
    return x


class Block(nn.Module):
    def __init__(self, cfg: ModelConfig, tp: TPContext = SINGLE, device=None, dtype=None):
        super().__init__()
        self.attn_norm = RMSNorm(cfg.d_model, cfg.norm_eps, device=device, dtype=dtype)
        self.attn = Attention(cfg, tp, device=device, dtype=dtype)
        self.mlp_norm = RMSNorm(cfg.d_model, cfg.norm_eps, device=device, dtype=dtype)
        self.mlp = SwiGLU(cfg, tp, device=device, dtype=dtype)

    @torch.no_grad()
    def forward(self, x, cos, sin, positions, kv):
        """x + attn(attn_norm(x)), then + mlp(mlp_norm(x)) (model.py:104-106); x is not modified."""
        dev = x.device
        ops.require_cuda(x)
        pos = torch.as_tensor(positions).to(device=dev, dtype=torch.int64).contiguous()
        return layer_forward_(self, x.contiguous().clone(), pos, kv, cos.to(dev, torch.float32).contiguous(),
                              sin.to(dev, torch.float32).contiguous())


def check_positions(positions: torch.Tensor, max_seq_len: int) -> None:
    if positions.numel() and int(positions.max()) >= max_seq_len:
        raise ValueError(f"position {int(positions.max())} exceeds max_seq_len {max_seq_len}")


class ForgeModel(nn.Module):
    """Embeddings and the output head are tied (model.py:109-159). `device`/`dtype` build it in place
    (the reference builds on the CPU in fp32; move it with .to(device, dtype) before running).

    tp: this process's shard of a tensor-parallel model (load it with tensor_parallel.shard_state_dict); the
    embedding, norms and head are replicated, and the two row-parallel projections of each layer end in one
    all-reduce each (2 * n_layers per forward, TPContext counts them)."""

    def __init__(self, cfg: ModelConfig, tp: TPContext = SINGLE, device=None, dtype=None):
        super().__init__()
        cfg.check_tensor_parallel(tp.size)
        self.cfg, self.tp = cfg, tp
        self.tok_emb = nn.Embedding(cfg.vocab_size, cfg.d_model, device=device, dtype=dtype)
        self.layers = nn.ModuleList(Block(cfg, tp, device=device, dtype=dtype) for _ in range(cfg.n_layers))
        self.norm = RMSNorm(cfg.d_model, cfg.norm_eps, device=device, dtype=dtype)
        self.lm_head = nn.Linear(cfg.d_model, cfg.vocab_size, bias=False, device=device, dtype=dtype)
        self.lm_head.weight = self.tok_emb.weight
        self._rope = RopeTables(cfg)
        self.register_buffer("rope_cos", self._rope.cos.to(device or "cpu"), persistent=False)
        self.register_buffer("rope_sin", self._rope.sin.to(device or "cpu"), persistent=False)
        self.apply(self._init_weights)

    @staticmethod
    def _init_weights(m):
        if isinstance(m, (nn.Linear, nn.Embedding)):
            nn.init.normal_(m.weight, mean=0.0, std=0.02)

    @property
    def device(self) -> torch.device:
        return self.tok_emb.weight.device

    @property
    def dtype(self) -> torch.dtype:
        return self.tok_emb.weight.dtype

    def num_params(self) -> int:
        return sum(p.numel() for p in self.parameters())

    def embed(self, idx):
        return ops.embed(torch.as_tensor(idx).to(self.device), self.tok_emb.weight)

    def head(self, x):
        return ops.linear(self.norm(x), self.lm_head.weight)

    @torch.no_grad()
    def forward(self, idx, positions: Optional[torch.Tensor] = None, kv: Optional[List] = None,
                last_only: bool = False):
        """idx: (B, T) token ids -> logits (B, T, vocab) on the model's device.

        positions: (B, T) absolute positions; default continues after whatever `kv` already holds.
        kv: one cache view per layer; None runs with a fresh contiguous cache.
        last_only: compute the head for the last position only (logits (B, 1, vocab))."""
        dev = self.device
        ops.require_cuda(self.tok_emb.weight)
        idx = torch.as_tensor(idx)
        b, t = idx.shape
        if kv is None:
            kv = new_contiguous_cache(self.cfg.n_layers, self.cfg.max_seq_len)
        if positions is None:
            start = kv[0].length
            if start + t > self.cfg.max_seq_len:
                raise ValueError(f"position {start + t - 1} exceeds max_seq_len {self.cfg.max_seq_len}")
            positions = (start + torch.arange(t))[None, :].expand(b, t)
        else:
            positions = torch.as_tensor(positions)
            check_positions(positions, self.cfg.max_seq_len)
        if idx.device.type == "cpu" and idx.numel() and (int(idx.min()) < 0 or int(idx.max()) >= self.cfg.vocab_size):
            raise IndexError("token id out of range for the embedding")
        pos = positions.to(device=dev, dtype=torch.int64, non_blocking=True).expand(b, t).contiguous()
        cos, sin = self._rope.on(dev)
        x = self.embed(idx)
        for layer, view in zip(self.layers, kv):
            layer_forward_(layer, x, pos, view, cos, sin)
        return self.head(x[:, -1:] if last_only else x)
