"""fs_attention_decode_static: decode attention for callers that cannot allocate device memory when they run a
decode step (a host that owns all device memory through its own pool, a plugin handed only device pointers, a loop
that cannot take a cudaMalloc's synchronisation mid-step). It runs the same kernels, with the same key splits in the
same order, as fs_attention_decode with a caller-owned workspace, so its output must be bit-identical. Two calls in
a row, with different shapes, both needing several key splits so that the fixed scratch array holds partial
results: the second call must not see anything the first one left behind. A call whose partials would not fit the
4 MiB array is refused, and once the entry point has been set up on a device a call takes no device memory.

This file's name makes pytest collect it last, so a failure here stops an `-x` run only after every other test."""

import ctypes
import os
import random
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

from forgeserve_b200 import _lib as L
from forgeserve_b200 import ops

DEV = "cuda"
ROOT = Path(__file__).resolve().parents[1]
STATIC_BYTES = 4 << 20


def paged_case(seed, lengths, nh, nkv, hd, bs=16, dtype=torch.bfloat16):
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
    pool_k = torch.randn(nblk, nkv, bs, hd, generator=g).to(dtype).to(DEV)
    pool_v = torch.randn(nblk, nkv, bs, hd, generator=g).to(dtype).to(DEV)
    q = torch.randn(B, nh * hd, generator=g).to(dtype).to(DEV)
    positions = torch.tensor([[n] for n in lengths], device=DEV)
    return pool_k, pool_v, table, q, positions, W * bs


def decode_static(q, desc, n_slots, positions, B, nh, nkv, hd, out=None):
    out = torch.empty_like(q) if out is None else out
    rc = L.load().fs_attention_decode_static(
        ctypes.c_void_p(q.data_ptr()), nh * hd, ctypes.byref(desc), n_slots, ctypes.c_void_p(positions.data_ptr()),
        ctypes.c_void_p(out.data_ptr()), nh * hd, B, nh, nkv, hd, ctypes.c_float(hd ** -0.5),
        L.FS_BF16 if q.dtype == torch.bfloat16 else L.FS_F32,
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    L.check(rc, "fs_attention_decode_static")
    return out


CASES = [  # (seed, lengths, nh, nkv, hd, dtype): each needs more than one key split
    (1, [3000, 1200], 32, 8, 128, torch.bfloat16),    # tensor-core decode kernel
    (2, [5000, 40, 2600], 16, 2, 64, torch.bfloat16),
    (3, [2100, 700], 8, 4, 64, torch.float32),        # CUDA-core kernel (fp32 parity mode)
]


def test_static_scratch_decode_matches_workspace_decode():
    L.device_error(clear=True)
    for seed, lengths, nh, nkv, hd, dtype in CASES:
        B = len(lengths)
        pool_k, pool_v, table, q, positions, n_slots = paged_case(seed, lengths, nh, nkv, hd, dtype=dtype)
        assert L.load().fs_attention_decode_workspace(B, nh, nkv, hd, n_slots) > 0   # the scratch is really used
        desc = ops.paged_desc(pool_k, pool_v, table)
        got = decode_static(q, desc, n_slots, positions, B, nh, nkv, hd)
        want = torch.empty_like(q)
        ops.attention_decode(q, desc, n_slots, positions, want, B, nh, nkv, hd)
        torch.cuda.synchronize()
        assert torch.isfinite(got.float()).all()
        assert torch.equal(got, want), (seed, (got.float() - want.float()).abs().max().item())
    assert L.device_error(clear=True) == 0


def test_static_scratch_decode_takes_no_device_memory_after_setup():
    seed, lengths, nh, nkv, hd, dtype = CASES[0]
    B = len(lengths)
    pool_k, pool_v, table, q, positions, n_slots = paged_case(seed, lengths, nh, nkv, hd, dtype=dtype)
    desc = ops.paged_desc(pool_k, pool_v, table)
    out = torch.empty_like(q)
    decode_static(q, desc, n_slots, positions, B, nh, nkv, hd, out)     # set-up call
    torch.cuda.synchronize()
    first = out.clone()
    free0 = torch.cuda.mem_get_info()[0]
    for _ in range(3):
        decode_static(q, desc, n_slots, positions, B, nh, nkv, hd, out)
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0
    assert torch.equal(out, first)


def test_static_scratch_refuses_calls_that_do_not_fit():
    B, nh, nkv, hd, n_slots = 64, 32, 8, 128, 2048        # 4 splits: 64 * 32 * 4 * 130 * 4 bytes > 4 MiB
    need = L.load().fs_attention_decode_workspace(B, nh, nkv, hd, n_slots)
    assert need > STATIC_BYTES
    assert L.load().fs_attention_decode_workspace(B, nh, nkv, hd, 1536) <= STATIC_BYTES
    nblk = n_slots // 16
    pool = torch.zeros(nblk, nkv, 16, hd, device=DEV, dtype=torch.bfloat16)
    table = torch.arange(nblk, device=DEV).repeat(B, 1)
    q = torch.zeros(B, nh * hd, device=DEV, dtype=torch.bfloat16)
    positions = torch.full((B, 1), n_slots - 1, device=DEV)
    desc = ops.paged_desc(pool, pool, table)
    with pytest.raises(RuntimeError, match=f"needs {need} bytes of scratch"):
        decode_static(q, desc, n_slots, positions, B, nh, nkv, hd)


FRESH = r"""
import sys, torch
sys.path.insert(0, sys.argv[1])
sys.path.insert(0, sys.argv[1] + "/tests")
from test_zz_no_alloc import CASES, paged_case, decode_static
from forgeserve_b200 import ops, _lib as L
for seed, lengths, nh, nkv, hd, dtype in CASES:
    pool_k, pool_v, table, q, positions, n_slots = paged_case(seed, lengths, nh, nkv, hd, dtype=dtype)
    desc = ops.paged_desc(pool_k, pool_v, table)
    got = decode_static(q, desc, n_slots, positions, len(lengths), nh, nkv, hd)   # first library work in the process
    want = torch.empty_like(q)
    ops.attention_decode(q, desc, n_slots, positions, want, len(lengths), nh, nkv, hd)
    torch.cuda.synchronize()
    assert torch.equal(got, want), seed
assert L.device_error(clear=True) == 0
print("fresh ok")
"""


def test_static_scratch_decode_in_a_fresh_process():
    """The entry point as the first work of the library in a new process, under CUDA's lazy module loading."""
    env = dict(os.environ, CUDA_MODULE_LOADING="LAZY")
    res = subprocess.run([sys.executable, "-c", FRESH, str(ROOT)], capture_output=True, text=True, timeout=300,
                         env=env)
    assert res.returncode == 0, res.stdout + res.stderr
    assert "fresh ok" in res.stdout
