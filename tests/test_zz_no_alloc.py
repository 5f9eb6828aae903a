"""fs_attention_decode_static — decode attention for callers that cannot allocate device memory when they run a
decode step (a host that owns all device memory through its own pool, a plugin handed only device pointers, a
loop that cannot take a cudaMalloc's synchronisation mid-step) — must give the same output as fs_attention_decode
with a caller-owned workspace. Two calls in a row, with different shapes, both needing several key splits so that
the fixed scratch array holds partial results; the second call must not see anything the first one left behind.

This file's name makes pytest collect it last, so a failure here stops an `-x` run only after every other test."""

import ctypes
import random

import pytest
import torch

pytestmark = pytest.mark.gpu

from forgeserve_b200 import _lib as L
from forgeserve_b200 import ops

DEV = "cuda"


def paged_case(seed, lengths, nh, nkv, hd, bs=16):
    rng = random.Random(seed)
    g = torch.Generator(device="cpu").manual_seed(seed)
    B = len(lengths)
    widths = [-(-(n + 1) // bs) for n in lengths]
    nblk = sum(widths) + 5
    blocks = list(range(nblk))
    rng.shuffle(blocks)
    it = iter(blocks)
    W = max(widths)
    table = torch.tensor([[next(it) for _ in range(w)] + [0] * (W - w) for w in widths], device=DEV)
    pool_k = torch.randn(nblk, nkv, bs, hd, generator=g).bfloat16().to(DEV)
    pool_v = torch.randn(nblk, nkv, bs, hd, generator=g).bfloat16().to(DEV)
    q = torch.randn(B, nh * hd, generator=g).bfloat16().to(DEV)
    positions = torch.tensor([[n] for n in lengths], device=DEV)
    return pool_k, pool_v, table, q, positions, W * bs


def decode_static(q, desc, n_slots, positions, B, nh, nkv, hd):
    out = torch.empty_like(q)
    rc = L.load().fs_attention_decode_static(
        ctypes.c_void_p(q.data_ptr()), nh * hd, ctypes.byref(desc), n_slots, ctypes.c_void_p(positions.data_ptr()),
        ctypes.c_void_p(out.data_ptr()), nh * hd, B, nh, nkv, hd, ctypes.c_float(hd ** -0.5), L.FS_BF16,
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    L.check(rc, "fs_attention_decode_static")
    return out


def test_static_scratch_decode_matches_workspace_decode():
    cases = [  # (seed, lengths, nh, nkv, hd): both need more than one key split
        (1, [3000, 1200], 32, 8, 128),
        (2, [5000, 40, 2600], 16, 2, 64),
    ]
    for seed, lengths, nh, nkv, hd in cases:
        B = len(lengths)
        pool_k, pool_v, table, q, positions, n_slots = paged_case(seed, lengths, nh, nkv, hd)
        assert L.load().fs_attention_decode_workspace(B, nh, nkv, hd, n_slots) > 0   # the scratch is really used
        desc = ops.paged_desc(pool_k, pool_v, table)
        got = decode_static(q, desc, n_slots, positions, B, nh, nkv, hd)
        want = torch.empty_like(q)
        ops.attention_decode(q, desc, n_slots, positions, want, B, nh, nkv, hd)
        torch.cuda.synchronize()
        assert torch.isfinite(got.float()).all()
        assert (got.float() - want.float()).abs().max().item() < 2e-2
    assert L.device_error(clear=True) == 0
