"""Token sampling and the plain generator (forgeserve/sampling.py:9-35).

Greedy sampling (temperature 0) runs the fs_argmax kernel on the logits' device: the first maximal index,
as torch.argmax. Temperature sampling draws with torch.multinomial from the caller's generator, on the
generator's device (a CPU generator gets CPU probabilities), so a seeded CPU generator gives the same stream
of draws as the reference for the same probabilities."""

import torch
import torch.nn.functional as F

from . import ops
from .kv import new_contiguous_cache


def probs_from_logits(logits: torch.Tensor, temperature: float) -> torch.Tensor:
    """Softmax of logits / temperature. temperature 0 gives a one-hot on the argmax."""
    if temperature == 0:
        idx = ops.argmax(logits) if logits.is_cuda else logits.argmax(-1)
        return F.one_hot(idx, logits.shape[-1]).to(logits.dtype)
    return F.softmax(logits.float() / temperature, dim=-1)


def sample(logits: torch.Tensor, temperature: float = 0.0, generator=None) -> torch.Tensor:
    """logits (..., V) -> token ids (...,), on the logits' device."""
    if temperature == 0:
        ops.require_cuda(logits)
        return ops.argmax(logits)
    probs = probs_from_logits(logits, temperature)
    if generator is not None and generator.device != probs.device:
        probs = probs.to(generator.device)
    out = torch.multinomial(probs.reshape(-1, probs.shape[-1]), 1, generator=generator).reshape(probs.shape[:-1])
    return out.to(logits.device)


@torch.no_grad()
def generate(model, prompt: torch.Tensor, max_new_tokens: int, temperature: float = 0.0, generator=None):
    """Reference generator for rows of equal length: prefill, then one token at a time with a plain cache.

    Returns (B, T + n) on the prompt's device."""
    kv = new_contiguous_cache(model.cfg.n_layers, model.cfg.max_seq_len)
    max_new_tokens = min(max_new_tokens, model.cfg.max_seq_len - prompt.shape[1])
    dev = model.device
    out = prompt.to(dev)
    logits = model(out, kv=kv)
    for _ in range(max_new_tokens):
        nxt = sample(logits[:, -1], temperature, generator)[:, None]
        out = torch.cat([out, nxt], dim=1)
        logits = model(nxt, kv=kv)
    return out.to(prompt.device)
