"""Each sm_100a kernel against a plain PyTorch fp32 statement of the same op, through the C ABI."""

import math
import random

import pytest
import torch

pytestmark = pytest.mark.gpu

from forgeserve_b200 import _lib as L
from forgeserve_b200 import ops

DEV = "cuda"


@pytest.fixture(autouse=True)
def _clean_device_errors():
    if torch.cuda.is_available():
        L.device_error(clear=True)
    yield
    if torch.cuda.is_available():
        assert L.device_error(clear=True) == 0


def bf16_close(got, want, rel=2 ** -7):
    got, want = got.float(), want.float()
    err = (got - want).abs().max().item()
    scale = want.abs().max().item()
    assert err <= rel * scale + 1e-3, f"max err {err} vs scale {scale}"


# ----------------------------------------------------------------------------------------------- GEMM
GEMM_SHAPES = [(128, 256, 64), (1, 64, 64), (77, 320, 192), (300, 520, 128), (1024, 1024, 1024), (256, 6144, 4096),
               (64, 4096, 14336), (4, 128256, 128)]


@pytest.mark.parametrize("M,N,K", GEMM_SHAPES)
def test_gemm_tcgen05_store(M, N, K):
    a = torch.randn(M, K, device=DEV).bfloat16()
    w = (torch.randn(N, K, device=DEV) / math.sqrt(K)).bfloat16()
    got = ops.linear(a, w)
    want = (a.double() @ w.double().t()).float()
    bf16_close(got, want)


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (77, 320, 192), (513, 4096, 4096)])
def test_gemm_tcgen05_residual_inplace(M, N, K):
    a = torch.randn(M, K, device=DEV).bfloat16()
    w = (torch.randn(N, K, device=DEV) / math.sqrt(K)).bfloat16()
    x = torch.randn(M, N, device=DEV).bfloat16()
    want = (x.float() + (a.float() @ w.float().t()).bfloat16().float())
    ops.linear(a, w, L.FS_EPI_RESIDUAL, residual=x, out=x)   # in place, as the residual stream is updated
    bf16_close(x, want)


@pytest.mark.parametrize("M,F,K", [(128, 128, 64), (77, 200, 192), (300, 384, 128), (256, 14336, 4096)])
def test_gemm_tcgen05_swiglu(M, F, K):
    a = torch.randn(M, K, device=DEV).bfloat16()
    wg = (torch.randn(F, K, device=DEV) / math.sqrt(K)).bfloat16()
    wu = (torch.randn(F, K, device=DEV) / math.sqrt(K)).bfloat16()
    got = ops.linear(a, torch.cat([wg, wu]), L.FS_EPI_SWIGLU)
    g = (a.float() @ wg.float().t()).bfloat16()
    u = (a.float() @ wu.float().t()).bfloat16()
    want = torch.nn.functional.silu(g) * u
    bf16_close(got, want, rel=2 ** -6)


@pytest.mark.parametrize("epi", [L.FS_EPI_STORE, L.FS_EPI_RESIDUAL, L.FS_EPI_SWIGLU])
@pytest.mark.parametrize("M,N,K", [(64, 6144, 4096), (1, 512, 4096), (100, 768, 2048), (64, 4096, 14336),
                                   (33, 1002, 1024)])
def test_gemm_split_k_small_m(epi, M, N, K):
    """Few rows (decode steps): K is split over more CTAs and a second kernel sums the partials and applies the
    epilogue (ragged N, N/2 not a multiple of 4 for SwiGLU, a single row)."""
    a = torch.randn(M, K, device=DEV).bfloat16()
    w = (torch.randn(N, K, device=DEV) / math.sqrt(K)).bfloat16()
    if epi == L.FS_EPI_SWIGLU:
        F = N // 2
        got = ops.linear(a, w, epi)
        g = (a.float() @ w[:F].float().t()).bfloat16()
        u = (a.float() @ w[F:].float().t()).bfloat16()
        bf16_close(got, torch.nn.functional.silu(g) * u, rel=2 ** -6)
    elif epi == L.FS_EPI_RESIDUAL:
        x = torch.randn(M, N, device=DEV).bfloat16()
        want = x.float() + (a.float() @ w.float().t()).bfloat16().float()
        ops.linear(a, w, epi, residual=x, out=x)
        bf16_close(x, want)
    else:
        bf16_close(ops.linear(a, w), (a.double() @ w.double().t()).float())


@pytest.mark.parametrize("epi", [L.FS_EPI_STORE, L.FS_EPI_RESIDUAL, L.FS_EPI_SWIGLU])
def test_split_k_reduce_paths_agree_bitwise(epi):
    """The split-K sums are reduced four outputs per thread when the output rows allow 8-byte stores, else one
    output per thread (here forced by a row stride that is not a multiple of 4); both sum the K chunks in the same
    order with the same rounding points, so they give the same bits."""
    M, N, K = 64, 2048, 4096
    a = torch.randn(M, K, device=DEV).bfloat16()
    w = (torch.randn(N, K, device=DEV) / math.sqrt(K)).bfloat16()
    n_out = N // 2 if epi == L.FS_EPI_SWIGLU else N
    wide = torch.zeros(M, n_out + 2, device=DEV).bfloat16()
    narrow = wide[:, :n_out]
    if epi == L.FS_EPI_RESIDUAL:
        x = torch.randn(M, n_out, device=DEV).bfloat16()
        narrow.copy_(x)
        ops.linear(a, w, epi, residual=x, out=x)
        ops.linear(a, w, epi, residual=narrow, out=narrow)
        assert torch.equal(x, narrow)
    else:
        assert torch.equal(ops.linear(a, w, epi), ops.linear(a, w, epi, out=narrow))
    assert L.device_error(clear=True) == 0


@pytest.mark.parametrize("epi", [L.FS_EPI_STORE, L.FS_EPI_RESIDUAL, L.FS_EPI_SWIGLU])
@pytest.mark.parametrize("M,N,K", [(64, 2048, 4096), (17, 1002, 4096), (1, 512, 256), (50, 768, 320)])
def test_gemm_thin_rows_match_full_tile_bitwise(epi, M, N, K):
    """Up to 64 rows run the thin form (64-row A boxes, five stages); the same rows inside a 100-row product run
    the full 128-row form. Each row is the same MMA chain over the same weights and the same split of K, so the
    two give the same bits, with and without split K."""
    a = torch.randn(100, K, device=DEV).bfloat16()
    w = (torch.randn(N, K, device=DEV) / math.sqrt(K)).bfloat16()
    n_out = N // 2 if epi == L.FS_EPI_SWIGLU else N
    r = torch.randn(100, n_out, device=DEV).bfloat16() if epi == L.FS_EPI_RESIDUAL else None
    full = ops.linear(a, w, epi, residual=r)
    thin = ops.linear(a[:M], w, epi, residual=None if r is None else r[:M])
    assert torch.equal(thin, full[:M])
    assert L.device_error(clear=True) == 0


def test_gemm_tcgen05_strided_rows():
    """A operand that is a column slice of a wider buffer (row stride > K), as the q part of a qkv buffer."""
    buf = torch.randn(200, 384, device=DEV).bfloat16()
    a = buf[:, 64:320]
    w = (torch.randn(256, 256, device=DEV) / 16).bfloat16()
    got = ops.linear(a, w)
    bf16_close(got, a.float() @ w.float().t())


@pytest.mark.parametrize("epi", [L.FS_EPI_STORE, L.FS_EPI_RESIDUAL, L.FS_EPI_SWIGLU])
@pytest.mark.parametrize("M,N,K", [(1, 16, 8), (37, 96, 64), (130, 200, 72)])
def test_gemm_simt_fp32(epi, M, N, K):
    a = torch.randn(M, K, device=DEV)
    w = torch.randn(N, K, device=DEV)
    ref = (a.double() @ w.double().t())
    if epi == L.FS_EPI_SWIGLU:
        F = N // 2
        got = ops.linear(a, w[: 2 * F], epi)
        want = torch.nn.functional.silu(ref[:, :F]) * ref[:, F : 2 * F]
    elif epi == L.FS_EPI_RESIDUAL:
        r = torch.randn(M, N, device=DEV)
        got = ops.linear(a, w, epi, residual=r)
        want = r.double() + ref
    else:
        got = ops.linear(a, w)
        want = ref
    torch.testing.assert_close(got.double(), want, atol=1e-4, rtol=1e-4)


def test_gemm_simt_matches_tcgen05_bf16():
    a = torch.randn(300, 512, device=DEV).bfloat16()
    w = (torch.randn(640, 512, device=DEV) / 22).bfloat16()
    bf16_close(ops.linear(a, w, simt=True), ops.linear(a, w).float())


# -------------------------------------------------------------------------------------------- RMSNorm
def rmsnorm_ref(x, w, eps):
    x32 = x.float()
    return (x32 * torch.rsqrt(x32.pow(2).mean(-1, keepdim=True) + eps)).to(x.dtype) * w


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("rows,dim", [(1, 64), (7, 128), (300, 4096), (5, 100), (33, 256), (17, 8192), (9, 768)])
def test_rmsnorm(dtype, rows, dim):
    x = torch.randn(rows, dim, device=DEV).to(dtype) * 3
    w = (torch.rand(dim, device=DEV) + 0.5).to(dtype)
    got = ops.rmsnorm(x, w, 1e-5)
    want = rmsnorm_ref(x, w, 1e-5)
    if dtype == torch.float32:
        torch.testing.assert_close(got, want, atol=1e-5, rtol=1e-5)
    else:
        bf16_close(got, want)


# --------------------------------------------------------------------------------- RoPE + KV store
def rope_tables(hd, max_len, theta):
    inv = 1.0 / (theta ** (torch.arange(0, hd, 2).float() / hd))
    ang = torch.outer(torch.arange(max_len).float(), inv)
    return ang.cos(), ang.sin()


def rope_ref(x, cos, sin, positions):
    c = cos[positions][:, None].to(x.dtype)
    s = sin[positions][:, None].to(x.dtype)
    x1, x2 = x.chunk(2, dim=-1)
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("nh,nkv,hd", [(8, 4, 8), (32, 8, 128),
                                       # bf16 vector path: fewer heads than one group of threads (hd 16: one chunk
                                       # per half head; hd 64), more heads than four groups (70B shape), v wider
                                       # than the block, and hd 48 (chunks do not divide the block: generic path)
                                       (4, 2, 16), (4, 2, 64), (64, 8, 128), (16, 16, 128), (6, 2, 48)])
def test_rope_kv_write_contiguous(dtype, nh, nkv, hd):
    B, T, start, cap = 3, 5, 4, 16
    cos, sin = rope_tables(hd, 64, 10000.0)
    qkv = torch.randn(B * T, (nh + 2 * nkv) * hd, device=DEV).to(dtype)
    orig = qkv.clone()
    positions = (start + torch.arange(T))[None].expand(B, T).contiguous()
    k = torch.zeros(B, nkv, cap, hd, device=DEV, dtype=dtype)
    v = torch.zeros_like(k)
    table = torch.arange(B, device=DEV)
    desc = ops.contiguous_desc(k, v, table)
    ops.rope_kv_write(qkv, cos.to(DEV), sin.to(DEV), positions.to(DEV), desc, B, T, nh, nkv, hd, slot_base=start,
                      slot_from_pos=False)
    q0 = orig[:, : nh * hd].view(B, T, nh, hd).transpose(1, 2).cpu()
    k0 = orig[:, nh * hd : (nh + nkv) * hd].view(B, T, nkv, hd).transpose(1, 2).cpu()
    v0 = orig[:, (nh + nkv) * hd :].view(B, T, nkv, hd).transpose(1, 2).cpu()
    q_want = rope_ref(q0, cos, sin, positions)
    k_want = rope_ref(k0, cos, sin, positions)
    q_got = qkv[:, : nh * hd].view(B, T, nh, hd).transpose(1, 2).cpu()
    tol = dict(atol=1e-6, rtol=1e-6) if dtype == torch.float32 else dict(atol=0, rtol=0)
    torch.testing.assert_close(q_got, q_want, **tol)   # bf16: bit-exact with the reference rounding order
    torch.testing.assert_close(k[:, :, start : start + T].cpu(), k_want, **tol)
    torch.testing.assert_close(v[:, :, start : start + T].cpu(), v0, atol=0, rtol=0)
    assert k[:, :, :start].abs().sum() == 0 and k[:, :, start + T :].abs().sum() == 0


def test_rope_kv_write_paged_slots():
    """Paged cache: token at position p of row r goes to block table[r, p // bs], slot p % bs."""
    nh, nkv, hd, bs = 4, 2, 16, 4
    B, T = 2, 6
    cos, sin = rope_tables(hd, 64, 10000.0)
    pool_k = torch.zeros(12, nkv, bs, hd, device=DEV)
    pool_v = torch.zeros_like(pool_k)
    table = torch.tensor([[7, 2, 9], [0, 11, 5]], device=DEV)
    positions = torch.tensor([[0, 1, 2, 3, 4, 5], [3, 4, 5, 6, 7, 8]], device=DEV)
    qkv = torch.randn(B * T, (nh + 2 * nkv) * hd, device=DEV)
    v_src = qkv[:, (nh + nkv) * hd :].clone().view(B, T, nkv, hd)
    ops.rope_kv_write(qkv, cos.to(DEV), sin.to(DEV), positions, ops.paged_desc(pool_k, pool_v, table), B, T, nh, nkv,
                      hd, slot_base=0, slot_from_pos=True)
    for r in range(B):
        for j in range(T):
            p = int(positions[r, j])
            blk = int(table[r, p // bs])
            torch.testing.assert_close(pool_v[blk, :, p % bs], v_src[r, j])


@pytest.mark.parametrize("hd", [16, 128])
def test_rope_kv_write_bad_slot_and_position_bf16(hd):
    """bf16 vector path, paged: a token whose block-table entry is -1 still has its q rotated, stores no k or v,
    and raises FS_ERR_BAD_SLOT; a position past the RoPE table raises FS_ERR_BAD_POSITION and writes nothing."""
    nh, nkv, bs = 8, 2, 16
    cos, sin = rope_tables(hd, 64, 10000.0)
    cos, sin = cos.to(DEV), sin.to(DEV)
    pool_k = torch.zeros(4, nkv, bs, hd, device=DEV, dtype=torch.bfloat16)
    pool_v = torch.zeros_like(pool_k)
    table = torch.tensor([[1, -1]], device=DEV)
    positions = torch.tensor([[3, 20]], device=DEV)             # block 1, then the missing block
    qkv = torch.randn(2, (nh + 2 * nkv) * hd, device=DEV).bfloat16()
    orig = qkv.clone()
    ops.rope_kv_write(qkv, cos, sin, positions, ops.paged_desc(pool_k, pool_v, table), 1, 2, nh, nkv, hd,
                      slot_base=0, slot_from_pos=True)
    assert L.device_error(clear=True) & L.FS_ERR_BAD_SLOT
    q0 = orig[:, : nh * hd].view(1, 2, nh, hd).transpose(1, 2).cpu()
    q_want = rope_ref(q0, cos.cpu(), sin.cpu(), positions.cpu())
    torch.testing.assert_close(qkv[:, : nh * hd].view(1, 2, nh, hd).transpose(1, 2).cpu(), q_want, atol=0, rtol=0)
    v_src = orig[:, (nh + nkv) * hd :].view(2, nkv, hd)
    torch.testing.assert_close(pool_v[1, :, 3], v_src[0], atol=0, rtol=0)
    assert pool_k[[0, 2, 3]].abs().sum() == 0 and pool_v[[0, 2, 3]].abs().sum() == 0
    assert int((pool_v[1].abs().sum(-1) != 0).sum()) == nkv      # only slot 3 of block 1 was written

    bad = torch.tensor([[3, 64]], device=DEV)                    # 64 = the table's length: out of range
    qkv2 = orig.clone()
    pool_k.zero_()
    pool_v.zero_()
    ops.rope_kv_write(qkv2, cos, sin, bad, ops.paged_desc(pool_k, pool_v, torch.tensor([[1, 2, 3, 0, 0]], device=DEV)),
                      1, 2, nh, nkv, hd, slot_base=0, slot_from_pos=True)
    assert L.device_error(clear=True) & L.FS_ERR_BAD_POSITION
    assert torch.equal(qkv2[1], orig[1])                          # the bad token is left as it was
    assert int((pool_v.abs().sum(-1) != 0).sum()) == nkv          # only the good token's v was stored


# ------------------------------------------------------------------------------------------ attention
def attention_ref(q, k_all, v_all, positions, rep):
    """q (B, nh, T, hd); k_all/v_all (B, nkv, S, hd); SDPA with the reference's mask, in fp64."""
    k_all = k_all.repeat_interleave(rep, dim=1).double()
    v_all = v_all.repeat_interleave(rep, dim=1).double()
    S = k_all.shape[2]
    mask = (torch.arange(S, device=q.device)[None, None, :] <= positions[:, :, None])[:, None]
    return torch.nn.functional.scaled_dot_product_attention(q.double(), k_all, v_all, attn_mask=mask)


def run_contiguous_attention(dtype, B, T, start, nh, nkv, hd, impl=L.FS_ATTN_AUTO, cap_multiple=1):
    S = start + T
    cap = -(-(S + 3) // cap_multiple) * cap_multiple
    k = torch.randn(B, nkv, cap, hd, device=DEV).to(dtype)
    v = torch.randn(B, nkv, cap, hd, device=DEV).to(dtype)
    q = torch.randn(B * T, nh * hd, device=DEV).to(dtype)
    positions = (start + torch.arange(T, device=DEV))[None].expand(B, T).contiguous()
    out = torch.empty(B * T, nh * hd, device=DEV, dtype=dtype)
    desc = ops.contiguous_desc(k, v, torch.arange(B, device=DEV))
    ops.attention(q, desc, S, positions, out, B, T, nh, nkv, hd, impl=impl)
    want = attention_ref(q.view(B, T, nh, hd).transpose(1, 2), k[:, :, :S], v[:, :, :S], positions, nh // nkv)
    return out.view(B, T, nh, hd).transpose(1, 2), want


@pytest.mark.parametrize("B,T,start,nh,nkv,hd", [(2, 9, 0, 8, 4, 8), (1, 16, 0, 8, 4, 16), (3, 1, 20, 8, 4, 16),
                                                 (2, 5, 7, 4, 4, 64)])
def test_attention_generic_fp32(B, T, start, nh, nkv, hd):
    got, want = run_contiguous_attention(torch.float32, B, T, start, nh, nkv, hd)
    torch.testing.assert_close(got.double(), want, atol=1e-5, rtol=1e-5)


@pytest.mark.parametrize("B,T,start,nh,nkv,hd", [(1, 128, 0, 4, 1, 128), (2, 200, 0, 8, 2, 128), (2, 64, 33, 4, 2, 64),
                                                 (1, 2048, 0, 4, 1, 128), (2, 17, 100, 4, 4, 128), (1, 1000, 24, 2, 1, 64)])
def test_attention_tensorcore_bf16(B, T, start, nh, nkv, hd):
    got, want = run_contiguous_attention(torch.bfloat16, B, T, start, nh, nkv, hd)
    err = (got.double() - want).abs().max().item()
    assert err < 2e-2, err


def test_attention_generic_bf16_matches_tensorcore():
    got_tc, want = run_contiguous_attention(torch.bfloat16, 2, 96, 5, 8, 2, 128, impl=L.FS_ATTN_MMA_SYNC)
    assert (got_tc.double() - want).abs().max().item() < 2e-2
    got_gen, want2 = run_contiguous_attention(torch.bfloat16, 2, 96, 5, 8, 2, 128, impl=L.FS_ATTN_CUDA_CORE)
    assert (got_gen.double() - want2).abs().max().item() < 2e-2


@pytest.mark.parametrize("B,T,start,nh,nkv,hd", [(1, 128, 0, 4, 1, 128), (2, 300, 0, 8, 2, 128), (1, 2048, 0, 8, 2, 128),
                                                 (2, 200, 37, 4, 4, 128), (2, 64, 0, 4, 2, 64), (1, 333, 21, 8, 2, 64),
                                                 (3, 1, 50, 4, 1, 128), (1, 17, 0, 8, 8, 128)])
def test_attention_tcgen05(B, T, start, nh, nkv, hd):
    got, want = run_contiguous_attention(torch.bfloat16, B, T, start, nh, nkv, hd, impl=L.FS_ATTN_TCGEN05,
                                         cap_multiple=16)
    err = (got.double() - want).abs().max().item()
    assert err < 2e-2, err


def test_attention_tcgen05_large_logits():
    """Scores far apart (the running max jumps by more than 2^8 between key tiles): the lazy rescale path."""
    B, T, nh, nkv, hd = 1, 512, 4, 1, 128
    k = torch.randn(B, nkv, 512, hd, device=DEV)
    k[:, :, 300:] *= 40.0                                    # later keys dominate by a wide margin
    k, v = k.bfloat16(), torch.randn(B, nkv, 512, hd, device=DEV).bfloat16()
    q = (torch.randn(B * T, nh * hd, device=DEV) * 2).bfloat16()
    positions = torch.arange(T, device=DEV)[None]
    out = torch.empty(B * T, nh * hd, device=DEV, dtype=torch.bfloat16)
    ops.attention(q, ops.contiguous_desc(k, v, torch.arange(B, device=DEV)), T, positions, out, B, T, nh, nkv, hd,
                  impl=L.FS_ATTN_TCGEN05)
    want = attention_ref(q.view(B, T, nh, hd).transpose(1, 2), k, v, positions, nh)
    got = out.view(B, T, nh, hd).transpose(1, 2).double()
    assert torch.isfinite(got).all()
    assert (got - want).abs().max().item() < 3e-2


def test_attention_tcgen05_paged_scattered_blocks():
    """Prefill of rows with different lengths into 16-slot blocks taken from a shuffled free list."""
    nh, nkv, hd, bs = 8, 2, 128, 16
    lengths = [200, 77, 130]
    B, T = len(lengths), max(lengths)
    nblk = 64
    blocks = list(range(nblk))
    random.Random(1).shuffle(blocks)
    it = iter(blocks)
    width = -(-T // bs)
    table = torch.tensor([[next(it) for _ in range(width)] for _ in lengths], device=DEV)
    pool_k = torch.randn(nblk, nkv, bs, hd, device=DEV).bfloat16()
    pool_v = torch.randn(nblk, nkv, bs, hd, device=DEV).bfloat16()
    positions = torch.stack([torch.arange(T) for _ in lengths]).to(DEV)
    q = torch.randn(B * T, nh * hd, device=DEV).bfloat16()
    out = torch.empty_like(q)
    ops.attention(q, ops.paged_desc(pool_k, pool_v, table), width * bs, positions, out, B, T, nh, nkv, hd,
                  impl=L.FS_ATTN_TCGEN05)
    k_all = pool_k[table].permute(0, 2, 1, 3, 4).reshape(B, nkv, -1, hd)
    v_all = pool_v[table].permute(0, 2, 1, 3, 4).reshape(B, nkv, -1, hd)
    want = attention_ref(q.view(B, T, nh, hd).transpose(1, 2), k_all, v_all, positions, nh // nkv)
    got = out.view(B, T, nh, hd).transpose(1, 2).double()
    assert (got - want).abs().max().item() < 2e-2


def test_attention_kernel_selector_refuses_unsupported_layouts():
    q = torch.randn(4, 8 * 16, device=DEV).bfloat16()
    k = torch.randn(1, 4, 8, 16, device=DEV).bfloat16()
    out = torch.empty_like(q)
    desc = ops.contiguous_desc(k, k.clone(), torch.arange(1, device=DEV))
    with pytest.raises(RuntimeError, match="tcgen05"):
        ops.attention(q, desc, 4, torch.arange(4, device=DEV)[None], out, 1, 4, 8, 4, 16, impl=L.FS_ATTN_TCGEN05)


@pytest.mark.parametrize("dtype,hd", [(torch.float32, 16), (torch.bfloat16, 128), (torch.bfloat16, 64)])
def test_attention_paged_per_row_positions(dtype, hd):
    """Decode-style step: rows at different positions, scattered blocks, padded tables (padding = block 0)."""
    nh, nkv, bs, nblk = 8, 2, 16, 40
    lengths = [37, 5, 70]                                   # keys already in the cache per row
    B = len(lengths)
    blocks = list(range(1, nblk))
    random.Random(0).shuffle(blocks)
    tables, it = [], iter(blocks)
    for n in lengths:
        tables.append([next(it) for _ in range(-(-(n + 1) // bs))])
    width = max(len(t) for t in tables)
    table = torch.tensor([t + [0] * (width - len(t)) for t in tables], device=DEV)
    pool_k = torch.randn(nblk, nkv, bs, hd, device=DEV).to(dtype)
    pool_v = torch.randn(nblk, nkv, bs, hd, device=DEV).to(dtype)
    positions = torch.tensor([[n] for n in lengths], device=DEV)
    q = torch.randn(B, nh * hd, device=DEV).to(dtype)
    out = torch.empty_like(q)
    ops.attention(q, ops.paged_desc(pool_k, pool_v, table), width * bs, positions, out, B, 1, nh, nkv, hd)
    k_all = pool_k[table].permute(0, 2, 1, 3, 4).reshape(B, nkv, -1, hd)
    v_all = pool_v[table].permute(0, 2, 1, 3, 4).reshape(B, nkv, -1, hd)
    want = attention_ref(q.view(B, 1, nh, hd).transpose(1, 2), k_all, v_all, positions, nh // nkv)
    got = out.view(B, 1, nh, hd).transpose(1, 2).double()
    tol = 1e-5 if dtype == torch.float32 else 2e-2
    assert (got - want).abs().max().item() < tol


def test_attention_paged_prefill_tensorcore():
    """Prefill of 40 tokens into scattered 16-slot blocks, read back through the table by the tensor-core kernel."""
    nh, nkv, hd, bs = 8, 2, 128, 16
    T = 40
    table = torch.tensor([[5, 1, 3]], device=DEV)
    pool_k = torch.randn(6, nkv, bs, hd, device=DEV).bfloat16()
    pool_v = torch.randn(6, nkv, bs, hd, device=DEV).bfloat16()
    positions = torch.arange(T, device=DEV)[None]
    q = torch.randn(T, nh * hd, device=DEV).bfloat16()
    out = torch.empty_like(q)
    ops.attention(q, ops.paged_desc(pool_k, pool_v, table), 3 * bs, positions, out, 1, T, nh, nkv, hd)
    k_all = pool_k[table].permute(0, 2, 1, 3, 4).reshape(1, nkv, -1, hd)
    v_all = pool_v[table].permute(0, 2, 1, 3, 4).reshape(1, nkv, -1, hd)
    want = attention_ref(q.view(1, T, nh, hd).transpose(1, 2), k_all, v_all, positions, nh // nkv)
    assert (out.view(1, T, nh, hd).transpose(1, 2).double() - want).abs().max().item() < 2e-2


# ------------------------------------------------------------------------------ embedding, argmax, gather
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_embed(dtype):
    table = torch.randn(1000, 136, device=DEV).to(dtype)
    ids = torch.randint(0, 1000, (3, 7), device=DEV)
    torch.testing.assert_close(ops.embed(ids, table), table[ids], atol=0, rtol=0)


def test_embed_bad_id_sets_device_error():
    table = torch.randn(10, 16, device=DEV)
    ops.embed(torch.tensor([3, 10], device=DEV), table)
    assert L.device_error(clear=True) & L.FS_ERR_BAD_TOKEN


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_argmax_ties_lowest_index(dtype):
    x = torch.randn(5, 128256, device=DEV).to(dtype)
    x[1, 7] = x[1, 99] = 50.0
    x[2, :] = 0
    x[3, 128255] = 60.0
    got = ops.argmax(x)
    torch.testing.assert_close(got.cpu(), x.cpu().argmax(-1))
    assert int(got[1]) == 7 and int(got[2]) == 0


def test_kv_store_and_paged_gather_round_trip():
    nkv, bs, hd = 4, 4, 8
    pool_k = torch.zeros(10, nkv, bs, hd, device=DEV)
    pool_v = torch.zeros_like(pool_k)
    table = torch.tensor([[7, 2, 9]], device=DEV)
    k = torch.randn(1, nkv, 10, hd, device=DEV)
    v = torch.randn_like(k)
    positions = torch.arange(10, device=DEV)[None]
    ops.kv_store(k, v, positions, ops.paged_desc(pool_k, pool_v, table))
    k_all = ops.paged_gather(pool_k, table)
    assert k_all.shape == (1, nkv, 12, hd)
    torch.testing.assert_close(k_all[:, :, :10], k, atol=0, rtol=0)
    torch.testing.assert_close(pool_k[2, :, 1], k[0, :, 5], atol=0, rtol=0)
    torch.testing.assert_close(ops.paged_gather(pool_v, table)[:, :, :10], v, atol=0, rtol=0)


@pytest.mark.parametrize("epi", [L.FS_EPI_STORE, L.FS_EPI_RESIDUAL, L.FS_EPI_SWIGLU])
@pytest.mark.parametrize("M,N,K", [(256, 512, 192), (300, 1000, 256), (1000, 768, 4096), (8192, 1024, 512)])
def test_gemm_pair_kernel_matches_single_cta_kernel(epi, M, N, K):
    """The 2-SM (CTA pair) GEMM and the 1-SM GEMM give the same result on the same inputs."""
    a = torch.randn(M, K, device=DEV).bfloat16()
    w = (torch.randn(N, K, device=DEV) / math.sqrt(K)).bfloat16()
    r = torch.randn(M, N, device=DEV).bfloat16()
    kw = dict(residual=r) if epi == L.FS_EPI_RESIDUAL else {}
    try:
        ops.set_gemm_pair_mode(False)
        single = ops.linear(a, w, epi, **kw)
    finally:
        ops.set_gemm_pair_mode(True)
    pair = ops.linear(a, w, epi, **kw)
    bf16_close(pair, single.float(), rel=2 ** -8)
    if epi == L.FS_EPI_STORE:
        bf16_close(pair, a.double() @ w.double().t())


# ------------------------------------------------------------------------------------- decode attention
@pytest.mark.parametrize("dtype,hd,nh,nkv,lengths,bs", [
    (torch.bfloat16, 128, 32, 8, [3000, 17, 700, 1], 16),    # long rows: several splits
    (torch.bfloat16, 128, 32, 8, [200] * 64, 16),            # a full decode batch
    (torch.bfloat16, 64, 8, 8, [513, 64, 65], 16),           # no GQA sharing
    (torch.bfloat16, 128, 8, 1, [1000], 16),                 # one KV head for 8 query heads
    (torch.bfloat16, 128, 32, 8, [900, 31, 2], 32),          # 16-key tiles inside 32-slot blocks
    (torch.bfloat16, 128, 32, 8, [900, 31, 2], 8),           # blocks smaller than a tile: CUDA-core kernel
    (torch.bfloat16, 128, 12, 4, [4000, 2500, 130, 17, 8, 3000, 600, 1], 16),   # rep 3, ragged lengths
    (torch.float32, 128, 16, 4, [333, 2048, 5], 16),
])
def test_attention_decode_paged(dtype, hd, nh, nkv, lengths, bs):
    """One query per row at its own position, over scattered blocks (padded tables), against fp64 SDPA."""
    B = len(lengths)
    widths = [-(-(n + 1) // bs) for n in lengths]
    nblk = sum(widths) + 3
    blocks = list(range(nblk))
    random.Random(2).shuffle(blocks)
    it = iter(blocks)
    W = max(widths)
    table = torch.tensor([[next(it) for _ in range(w)] + [0] * (W - w) for w in widths], device=DEV)
    pool_k = torch.randn(nblk, nkv, bs, hd, device=DEV).to(dtype)
    pool_v = torch.randn(nblk, nkv, bs, hd, device=DEV).to(dtype)
    positions = torch.tensor([[n] for n in lengths], device=DEV)
    q = torch.randn(B, nh * hd, device=DEV).to(dtype)
    out = torch.empty_like(q)
    ops.attention_decode(q, ops.paged_desc(pool_k, pool_v, table), W * bs, positions, out, B, nh, nkv, hd)
    k_all = pool_k[table].permute(0, 2, 1, 3, 4).reshape(B, nkv, -1, hd)
    v_all = pool_v[table].permute(0, 2, 1, 3, 4).reshape(B, nkv, -1, hd)
    want = attention_ref(q.view(B, 1, nh, hd).transpose(1, 2), k_all, v_all, positions, nh // nkv)
    got = out.view(B, 1, nh, hd).transpose(1, 2).double()
    tol = 1e-5 if dtype == torch.float32 else 2e-2
    assert (got - want).abs().max().item() < tol


def test_attention_decode_long_rows_reload_block_ids():
    """Rows past 64 splits x 512 keys: a split then covers more than 32 of a warp's 16-key tiles, and the warp
    reloads its lanes' block ids every 32 tiles. A sharper softmax (q x 2) makes a wrong block show as an error of
    the order of the output itself."""
    dtype, hd, nh, nkv, bs = torch.bfloat16, 128, 2, 1, 16
    lengths = [140000, 40000]
    B = len(lengths)
    widths = [-(-(n + 1) // bs) for n in lengths]
    nblk = sum(widths) + 3
    blocks = list(range(nblk))
    random.Random(7).shuffle(blocks)
    it = iter(blocks)
    W = max(widths)
    table = torch.tensor([[next(it) for _ in range(w)] + [0] * (W - w) for w in widths], device=DEV)
    pool_k = torch.randn(nblk, nkv, bs, hd, device=DEV).to(dtype)
    pool_v = torch.randn(nblk, nkv, bs, hd, device=DEV).to(dtype)
    positions = torch.tensor([[n] for n in lengths], device=DEV)
    q = (torch.randn(B, nh * hd, device=DEV) * 2).to(dtype)
    out = torch.empty_like(q)
    assert L.load().fs_attention_decode_workspace(B, nh, nkv, hd, W * bs) > 0
    ops.attention_decode(q, ops.paged_desc(pool_k, pool_v, table), W * bs, positions, out, B, nh, nkv, hd)
    k_all = pool_k[table].permute(0, 2, 1, 3, 4).reshape(B, nkv, -1, hd)
    v_all = pool_v[table].permute(0, 2, 1, 3, 4).reshape(B, nkv, -1, hd)
    want = attention_ref(q.view(B, 1, nh, hd).transpose(1, 2), k_all, v_all, positions, nh // nkv)
    got = out.view(B, 1, nh, hd).transpose(1, 2).double()
    err, scale = (got - want).abs().max().item(), want.abs().max().item()
    assert err <= 3e-2 * scale, f"max err {err} vs output scale {scale}"


def test_attention_decode_ignores_stale_slots():
    """Slots past each row's position (in the last block, and whole unused blocks) hold NaN: they must not leak."""
    B, nh, nkv, hd, bs = 3, 32, 8, 128, 16
    lengths = [37, 16, 250]
    widths = [-(-(n + 1) // bs) + 1 for n in lengths]          # one extra (unused) block per row
    nblk = sum(widths)
    table = torch.arange(nblk, device=DEV).flip(0)
    rows, at = [], 0
    for w in widths:
        rows.append(table[at : at + w].tolist())
        at += w
    W = max(widths)
    table = torch.tensor([r + [0] * (W - len(r)) for r in rows], device=DEV)
    pool_k = torch.full((nblk, nkv, bs, hd), float("nan"), device=DEV).bfloat16()
    pool_v = torch.full((nblk, nkv, bs, hd), float("nan"), device=DEV).bfloat16()
    for r, n in enumerate(lengths):
        for s in range(n + 1):
            blk = int(table[r, s // bs])
            pool_k[blk, :, s % bs] = torch.randn(nkv, hd, device=DEV).bfloat16()
            pool_v[blk, :, s % bs] = torch.randn(nkv, hd, device=DEV).bfloat16()
    q = torch.randn(B, nh * hd, device=DEV).bfloat16()
    positions = torch.tensor([[n] for n in lengths], device=DEV)
    out = torch.empty_like(q)
    ops.attention_decode(q, ops.paged_desc(pool_k, pool_v, table), W * bs, positions, out, B, nh, nkv, hd)
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()
    k_all = torch.nan_to_num(pool_k[table].permute(0, 2, 1, 3, 4).reshape(B, nkv, -1, hd).double())
    v_all = torch.nan_to_num(pool_v[table].permute(0, 2, 1, 3, 4).reshape(B, nkv, -1, hd).double())
    want = attention_ref(q.view(B, 1, nh, hd).transpose(1, 2), k_all, v_all, positions, nh // nkv)
    got = out.view(B, 1, nh, hd).transpose(1, 2).double()
    assert (got - want).abs().max().item() < 2e-2


def test_attention_decode_flags_a_bad_block():
    """A block id outside the pool inside the visible range sets the device error bit; nothing is read there."""
    B, nh, nkv, hd, bs = 1, 32, 8, 128, 16
    pool = torch.randn(4, nkv, bs, hd, device=DEV).bfloat16()
    table = torch.tensor([[0, 1, 9]], device=DEV)             # block 9 does not exist
    q = torch.randn(B, nh * hd, device=DEV).bfloat16()
    out = torch.empty_like(q)
    L.device_error(clear=True)
    ops.attention_decode(q, ops.paged_desc(pool, pool, table), 3 * bs, torch.tensor([[40]], device=DEV), out, B, nh,
                         nkv, hd)
    torch.cuda.synchronize()
    assert L.device_error(clear=True) & L.FS_ERR_BAD_SLOT


def test_attention_decode_contiguous_matches_generic():
    """Contiguous cache (one block per row), the decode kernel against the CUDA-core kernel."""
    B, nh, nkv, hd, S = 3, 32, 8, 128, 1500
    k = torch.randn(B, nkv, 1504, hd, device=DEV).bfloat16()
    v = torch.randn(B, nkv, 1504, hd, device=DEV).bfloat16()
    q = torch.randn(B, nh * hd, device=DEV).bfloat16()
    positions = torch.tensor([[S - 1], [10], [700]], device=DEV)
    desc = ops.contiguous_desc(k, v, torch.arange(B, device=DEV))
    a, b = torch.empty_like(q), torch.empty_like(q)
    ops.attention_decode(q, desc, S, positions, a, B, nh, nkv, hd)
    ops.attention(q, desc, S, positions, b, B, 1, nh, nkv, hd, impl=L.FS_ATTN_CUDA_CORE)
    assert (a.float() - b.float()).abs().max().item() < 2e-2


def test_attention_decode_refuses_a_small_workspace():
    B, nh, nkv, hd = 1, 32, 8, 128
    k = torch.zeros(1, nkv, 4096, hd, device=DEV).bfloat16()
    q = torch.zeros(B, nh * hd, device=DEV).bfloat16()
    desc = ops.contiguous_desc(k, k, torch.arange(1, device=DEV))
    need = L.load().fs_attention_decode_workspace(B, nh, nkv, hd, 4096)
    assert need > 0
    import ctypes
    rc = L.load().fs_attention_decode(ctypes.c_void_p(q.data_ptr()), nh * hd, ctypes.byref(desc), 4096,
                                      ctypes.c_void_p(torch.zeros(1, 1, dtype=torch.int64, device=DEV).data_ptr()),
                                      ctypes.c_void_p(q.data_ptr()), nh * hd, B, nh, nkv, hd, 0.1, None, 0, L.FS_BF16,
                                      None)
    assert rc != 0 and b"workspace" in L.load().fs_last_error()
