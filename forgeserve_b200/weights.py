"""Weights in the reference's state-dict format: seeded per tensor, or memory-mapped from a saved state dict.

Every tensor is drawn from its own generator, seeded from (seed, tensor name), so a pipeline stage can build
exactly its own layers — on its GPU, without materialising the full model — and still hold the same values
as a single-process model built from the same seed. Names are the reference's state-dict keys
(forgeserve/model.py:109-138; `lm_head.weight` equals `tok_emb.weight`, as ForgeModel ties them).

A saved model is a `torch.save` of `ForgeModel.state_dict()` (the reference's format; any subset of its keys
works too). `open_state_dict` maps such a file instead of reading it, so a stage that loads from it with
`PipelineStage.load_from_full` reads only its own tensors' pages: at the 70B shape the full fp32 dict is about
274 GB, more than a host holds, while one of 8 stages needs about 35 GB of it.
"""

import hashlib
from typing import Dict, Iterable, Optional

import torch

from .config import ModelConfig


def layer_shapes(cfg: ModelConfig, i: int) -> Dict[str, tuple]:
    d, hd = cfg.d_model, cfg.head_dim
    p = f"layers.{i}."
    return {
        p + "attn_norm.weight": (d,),
        p + "attn.wq.weight": (cfg.n_heads * hd, d),
        p + "attn.wk.weight": (cfg.n_kv_heads * hd, d),
        p + "attn.wv.weight": (cfg.n_kv_heads * hd, d),
        p + "attn.wo.weight": (d, cfg.n_heads * hd),
        p + "mlp_norm.weight": (d,),
        p + "mlp.w_gate.weight": (cfg.ffn_dim, d),
        p + "mlp.w_up.weight": (cfg.ffn_dim, d),
        p + "mlp.w_down.weight": (d, cfg.ffn_dim),
    }


def model_shapes(cfg: ModelConfig) -> Dict[str, tuple]:
    shapes = {"tok_emb.weight": (cfg.vocab_size, cfg.d_model)}
    for i in range(cfg.n_layers):
        shapes.update(layer_shapes(cfg, i))
    shapes["norm.weight"] = (cfg.d_model,)
    shapes["lm_head.weight"] = (cfg.vocab_size, cfg.d_model)
    return shapes


def _tensor_seed(seed: int, name: str) -> int:
    h = hashlib.sha256(f"{seed}:{name}".encode()).digest()
    return int.from_bytes(h[:8], "little") & ((1 << 63) - 1)


def seeded_tensor(name: str, shape: tuple, seed: int, std: float, device="cpu", dtype=torch.float32) -> torch.Tensor:
    """Norm weights are ones (the reference's RMSNorm init); matrices are N(0, std^2)."""
    if name.endswith("norm.weight"):
        return torch.ones(shape, device=device, dtype=dtype)
    if name == "lm_head.weight":
        name = "tok_emb.weight"
    g = torch.Generator(device=device).manual_seed(_tensor_seed(seed, name))
    t = torch.empty(shape, device=device, dtype=torch.float32)
    t.normal_(0.0, std, generator=g)
    return t.to(dtype)


def seeded_state_dict(cfg: ModelConfig, seed: int = 0, std: float = 0.02, names: Optional[Iterable[str]] = None,
                      device="cpu", dtype=torch.float32) -> Dict[str, torch.Tensor]:
    shapes = model_shapes(cfg)
    keys = list(shapes) if names is None else list(names)
    return {k: seeded_tensor(k, shapes[k], seed, std, device, dtype) for k in keys}


def open_state_dict(path) -> Dict[str, torch.Tensor]:
    """The state dict saved at `path`, memory-mapped: CPU tensors that are views of the file's pages (tied
    tensors, such as the reference's `lm_head.weight` and `tok_emb.weight`, stay one storage). Nothing is read
    until a tensor's elements are used."""
    return torch.load(path, map_location="cpu", mmap=True, weights_only=True)


def _own_part(name: str, full: torch.Tensor, cfg: ModelConfig, tp) -> torch.Tensor:
    """The part of a full tensor that a tensor-parallel shard holds (all of it without tensor parallelism)."""
    if tp is None or tp.size == 1:
        return full
    from .tensor_parallel import shard_state_dict
    return shard_state_dict({name: full}, cfg, tp.rank, tp.size)[name]


@torch.no_grad()
def init_stage_(stage, seed: int = 0, std: float = 0.02) -> None:
    """Fill a PipelineStage with the seeded weights of its own layers (global layer numbering), on its device; a
    tensor-parallel stage takes its shard of each tensor."""
    shapes = model_shapes(stage.cfg)
    for name, p in stage.named_parameters():
        if name.startswith("layers."):
            i = int(name.split(".")[1])
            gname = name.replace(f"layers.{i}.", f"layers.{i + stage.lo}.", 1)
        else:
            gname = name
        full = seeded_tensor(gname, shapes[gname], seed, std, device=p.device, dtype=p.dtype)
        p.copy_(_own_part(gname, full, stage.cfg, getattr(stage, "tp", None)))


@torch.no_grad()
def init_model_(model, seed: int = 0, std: float = 0.02) -> None:
    """Fill a ForgeModel with the same seeded weights (tied head = embedding); a tensor-parallel model takes its
    shard of each tensor."""
    shapes = model_shapes(model.cfg)
    for name, p in model.named_parameters():
        full = seeded_tensor(name, shapes[name], seed, std, device=p.device, dtype=p.dtype)
        p.copy_(_own_part(name, full, model.cfg, getattr(model, "tp", None)))


def test_suite_state_dict(cfg: ModelConfig, seed: int, scale: float) -> Dict[str, torch.Tensor]:
    """The weights the reference's test suite gives its models (forgeserve tests/conftest.py:18-27): every
    parameter of two or more dimensions, in ForgeModel.parameters() order (model.py:109-122: embedding, then per
    layer attn_norm, wq, wk, wv, wo, mlp_norm, w_gate, w_up, w_down, then the final norm), replaced by
    randn(shape, generator seeded `seed`) * scale; norms stay ones; the head is the embedding (tied). fp32, CPU."""
    g = torch.Generator().manual_seed(seed)
    sd = {}
    for name, shape in model_shapes(cfg).items():
        if name == "lm_head.weight":
            continue
        sd[name] = torch.randn(shape, generator=g) * scale if len(shape) >= 2 else torch.ones(shape)
    sd["lm_head.weight"] = sd["tok_emb.weight"]
    return sd


def checksum(sd: Dict[str, torch.Tensor]) -> Dict[str, tuple]:
    """Per-tensor (sum, sum of squares) in fp64: how a recorded fixture names the weights it was made with."""
    return {k: (float(v.double().sum()), float(v.double().pow(2).sum())) for k, v in sd.items()}
