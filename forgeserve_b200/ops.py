"""Tensor-level wrappers of the C ABI: each function checks its torch tensors (CUDA, dtype, layout), passes raw
pointers and the caller's current CUDA stream to libforgeserve_b200.so, and returns torch tensors it allocated
(the caller owns them). Nothing here computes on the CPU."""

import ctypes
import math
from typing import List, Optional

import torch

from . import _lib as L

_DTYPES = {torch.float32: L.FS_F32, torch.bfloat16: L.FS_BF16}

# When set to a list, every projection GEMM appends (start_event, end_event, flops) recorded on its stream.
gemm_events: Optional[List] = None


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _DTYPES[dtype]
    except KeyError:
        raise TypeError(f"forgeserve_b200 kernels support float32 and bfloat16, not {dtype}") from None


def require_cuda(*tensors) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError(
                "forgeserve_b200 runs its path as CUDA kernels only (no CPU fallback); "
                f"got a tensor on {t.device}. Move the module and inputs to a CUDA device.")


def _p(t: Optional[torch.Tensor]) -> ctypes.c_void_p:
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def _stream(t: torch.Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _rows(t: torch.Tensor):
    """View a (..., n) tensor whose last dim is contiguous as rows: returns (num_rows, row_stride)."""
    n = t.shape[-1]
    if t.stride(-1) != 1 and n > 1:
        raise ValueError("last dimension must be contiguous")
    if t.dim() == 1:
        return 1, n
    rows = 1
    for s in t.shape[:-1]:
        rows *= s
    # leading dims must collapse to uniformly strided rows (size-1 dims impose nothing)
    for i in range(t.dim() - 2):
        if t.shape[i] > 1 and t.shape[i + 1] > 1 and t.stride(i) != t.stride(i + 1) * t.shape[i + 1]:
            raise ValueError("leading dimensions must collapse to uniformly strided rows")
    # the row stride is the stride of the innermost leading dim that has more than one entry
    row_stride = next((t.stride(i) for i in range(t.dim() - 2, -1, -1) if t.shape[i] > 1), n)
    return rows, max(row_stride, n)


def set_persistent_sms(n: int) -> None:
    """Cap the persistent GEMM grid of the current CUDA device to n SMs (0 = all)."""
    L.check(L.load().fs_set_persistent_sms(int(n)), "fs_set_persistent_sms")


def set_gemm_pair_mode(on: bool) -> None:
    """Choose the 2-SM (CTA pair) GEMM for M > 128 (default) or always the 1-SM GEMM."""
    L.check(L.load().fs_set_gemm_pair_mode(int(bool(on))), "fs_set_gemm_pair_mode")


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """RMSNorm over the last dim (forgeserve/model.py:29-31)."""
    require_cuda(x, w)
    if w.dtype != x.dtype:
        raise TypeError("rmsnorm weight and input must have the same dtype")
    out = torch.empty_like(x, memory_format=torch.contiguous_format) if out is None else out
    rows, xs = _rows(x)
    _, ys = _rows(out)
    lib = L.load()
    L.check(lib.fs_rmsnorm(_p(x), xs, _p(w), _p(out), ys, rows, x.shape[-1], float(eps), dtype_code(x.dtype),
                           _stream(x)), "fs_rmsnorm")
    return out


def linear(x: torch.Tensor, w: torch.Tensor, epilogue: int = L.FS_EPI_STORE, residual: Optional[torch.Tensor] = None,
           out: Optional[torch.Tensor] = None, simt: bool = False) -> torch.Tensor:
    """x (..., K) @ w (N, K)^T with a fused epilogue (see fs_gemm). Returns (..., n_out)."""
    require_cuda(x, w, residual, out)
    if w.dtype != x.dtype or (residual is not None and residual.dtype != x.dtype):
        raise TypeError("linear: all operands must share one dtype")
    if w.dim() != 2 or w.stride(1) != 1:
        raise ValueError("linear: weight must be 2-D with contiguous rows")
    K = x.shape[-1]
    N = w.shape[0]
    if w.shape[1] != K:
        raise ValueError(f"linear: weight has {w.shape[1]} input features, input has {K}")
    n_out = N // 2 if epilogue == L.FS_EPI_SWIGLU else N
    if out is None:
        out = torch.empty(*x.shape[:-1], n_out, dtype=x.dtype, device=x.device)
    M, lda = _rows(x)
    _, ldc = _rows(out)
    ldr = _rows(residual)[1] if residual is not None else 0
    fn = L.load().fs_gemm_simt if simt else L.load().fs_gemm
    ev = gemm_events
    if ev is not None:
        st = torch.cuda.current_stream(x.device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
    L.check(fn(_p(x), lda, _p(w), w.stride(0), _p(out), ldc, _p(residual), ldr, M, N, K, n_out, epilogue,
               dtype_code(x.dtype), _stream(x)), "fs_gemm")
    if ev is not None:
        e1.record(st)
        ev.append((e0, e1, 2.0 * M * N * K))
    return out


def linear_to(x: torch.Tensor, w: torch.Tensor, c_ptr: int, ldc: int, system_fence: bool = False) -> None:
    """x (..., K) @ w (N, K)^T stored at device address c_ptr, rows of ldc elements apart (no residual, no
    SwiGLU). c_ptr may be another GPU's buffer mapped with ipc_open; system_fence=True then makes the kernel end
    with a system-scope fence, so its stores are performed by the time the kernel completes."""
    require_cuda(x, w)
    if w.dtype != x.dtype or w.dim() != 2 or w.stride(1) != 1 or w.shape[1] != x.shape[-1]:
        raise ValueError("linear_to: weight must be (N, K) with contiguous rows, in the input's dtype")
    M, lda = _rows(x)
    N, K = w.shape
    if ldc < N:
        raise ValueError("linear_to: output row stride smaller than N")
    epi = L.FS_EPI_STORE | (L.FS_EPI_SYSTEM_FENCE if system_fence else 0)
    ev = gemm_events
    if ev is not None:
        st = torch.cuda.current_stream(x.device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
    L.check(L.load().fs_gemm(_p(x), lda, _p(w), w.stride(0), ctypes.c_void_p(c_ptr), ldc, None, 0, M, N, K, N, epi,
                             dtype_code(x.dtype), _stream(x)), "fs_gemm")
    if ev is not None:
        e1.record(st)
        ev.append((e0, e1, 2.0 * M * N * K))


def ipc_handle(t: torch.Tensor) -> bytes:
    """CUDA IPC handle of the allocation holding t, followed by t's byte offset in it (8 bytes, little-endian)."""
    require_cuda(t)
    h = (ctypes.c_char * L.FS_IPC_HANDLE_BYTES)()
    off = ctypes.c_int64()
    L.check(L.load().fs_ipc_handle(_p(t), h, ctypes.byref(off)), "fs_ipc_handle")
    return bytes(h) + int(off.value).to_bytes(8, "little", signed=True)


def ipc_open(handle: bytes) -> int:
    """Map another process's allocation (the first FS_IPC_HANDLE_BYTES bytes of an ipc_handle); returns its base."""
    base = ctypes.c_void_p()
    L.check(L.load().fs_ipc_open(handle[: L.FS_IPC_HANDLE_BYTES], ctypes.byref(base)), "fs_ipc_open")
    return int(base.value)


def copy_2d_to(dst_ptr: int, dpitch: int, src: torch.Tensor) -> None:
    """Copy the rows of a 2-D view `src` (last dim contiguous) to device address dst_ptr, rows dpitch bytes apart,
    on the current stream by the copy engine (dst_ptr may be another GPU's buffer mapped with ipc_open)."""
    require_cuda(src)
    rows, ld = _rows(src)
    width = src.shape[-1] * src.element_size()
    L.check(L.load().fs_copy_2d(ctypes.c_void_p(dst_ptr), int(dpitch), _p(src), ld * src.element_size(), width, rows,
                                _stream(src)), "fs_copy_2d")


def ipc_close(base: int) -> None:
    L.check(L.load().fs_ipc_close(ctypes.c_void_p(base)), "fs_ipc_close")


def rope_kv_write(qkv: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, positions: torch.Tensor,
                  kv: L.KVCacheDesc, B: int, T: int, nh: int, nkv: int, hd: int, slot_base: int, slot_from_pos: bool,
                  apply_rope: bool = True) -> None:
    require_cuda(qkv, cos, sin, positions)
    rows, ld = _rows(qkv)
    L.check(L.load().fs_rope_kv_write(_p(qkv), ld, _p(cos), _p(sin), cos.shape[0], _p(positions), ctypes.byref(kv), B,
                                      T, nh, nkv, hd, slot_base, int(slot_from_pos), int(apply_rope),
                                      dtype_code(qkv.dtype), _stream(qkv)), "fs_rope_kv_write")


def attention(q: torch.Tensor, kv: L.KVCacheDesc, n_slots: int, positions: torch.Tensor, out: torch.Tensor, B: int,
              T: int, nh: int, nkv: int, hd: int, impl: int = L.FS_ATTN_AUTO) -> torch.Tensor:
    """GQA attention over a cache; impl selects the kernel (FS_ATTN_*), automatic by default."""
    require_cuda(q, positions, out)
    _, ldq = _rows(q)
    _, ldo = _rows(out)
    L.check(L.load().fs_attention_impl(_p(q), ldq, ctypes.byref(kv), n_slots, _p(positions), _p(out), ldo, B, T, nh,
                                       nkv, hd, 1.0 / math.sqrt(hd), int(impl), dtype_code(q.dtype), _stream(q)),
            "fs_attention")
    return out


_DECODE_WS = {}
_DECODE_WS_RETIRED: List[torch.Tensor] = []


def decode_workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """A scratch buffer for split decode attention per (device, current stream), grown on demand and reused by the
    calls on that stream (which run one after another). A buffer that is outgrown stays allocated: a CUDA graph
    captured earlier may still address it."""
    key = (str(device), torch.cuda.current_stream(device).cuda_stream)
    ws = _DECODE_WS.get(key)
    if ws is None or ws.numel() < nbytes:
        if ws is not None:
            _DECODE_WS_RETIRED.append(ws)
        ws = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _DECODE_WS[key] = ws
    return ws


def attention_decode(q: torch.Tensor, kv: L.KVCacheDesc, n_slots: int, positions: torch.Tensor, out: torch.Tensor,
                     B: int, nh: int, nkv: int, hd: int) -> torch.Tensor:
    """Split-KV decode attention: one query per row (positions (B,) or (B, 1))."""
    require_cuda(q, positions, out)
    _, ldq = _rows(q)
    _, ldo = _rows(out)
    lib = L.load()
    need = int(lib.fs_attention_decode_workspace(B, nh, nkv, hd, n_slots))
    ws = decode_workspace(q.device, need) if need > 0 else None
    L.check(lib.fs_attention_decode(_p(q), ldq, ctypes.byref(kv), n_slots, _p(positions), _p(out), ldo, B, nh, nkv, hd,
                                    1.0 / math.sqrt(hd), _p(ws), 0 if ws is None else ws.numel(),
                                    dtype_code(q.dtype), _stream(q)), "fs_attention_decode")
    return out


def kv_store(k: torch.Tensor, v: torch.Tensor, positions: torch.Tensor, kv: L.KVCacheDesc) -> None:
    require_cuda(k, v, positions)
    B, nkv, T, hd = k.shape
    k, v = k.contiguous(), v.contiguous()
    L.check(L.load().fs_kv_store(_p(k), _p(v), _p(positions), ctypes.byref(kv), B, T, nkv, hd, dtype_code(k.dtype),
                                 _stream(k)), "fs_kv_store")


def paged_gather(pool: torch.Tensor, table: torch.Tensor) -> torch.Tensor:
    """pool (num_blocks, nkv, bs, hd), table (B, nb) int64 -> (B, nkv, nb*bs, hd)."""
    require_cuda(pool, table)
    nblk, nkv, bs, hd = pool.shape
    B, nb = table.shape
    out = torch.empty(B, nkv, nb * bs, hd, dtype=pool.dtype, device=pool.device)
    L.check(L.load().fs_paged_gather(_p(pool), _p(table), B, nb, nblk, nkv, bs, hd, _p(out), dtype_code(pool.dtype),
                                     _stream(pool)), "fs_paged_gather")
    return out


def embed(ids: torch.Tensor, table: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """table[ids] for int64 ids on the table's device (nn.Embedding)."""
    require_cuda(ids, table)
    ids = ids.contiguous()
    if ids.dtype != torch.int64:
        ids = ids.long()
    V, d = table.shape
    if out is None:
        out = torch.empty(*ids.shape, d, dtype=table.dtype, device=table.device)
    L.check(L.load().fs_embed(_p(ids), ids.numel(), _p(table), V, d, _p(out), dtype_code(table.dtype), _stream(table)),
            "fs_embed")
    return out


def argmax(x: torch.Tensor) -> torch.Tensor:
    """argmax over the last dim (lowest index on ties), int64 result of shape x.shape[:-1]."""
    require_cuda(x)
    rows, rs = _rows(x)
    out = torch.empty(x.shape[:-1], dtype=torch.int64, device=x.device)
    L.check(L.load().fs_argmax(_p(x), rows, x.shape[-1], rs, _p(out), dtype_code(x.dtype), _stream(x)), "fs_argmax")
    return out


def contiguous_desc(k: torch.Tensor, v: torch.Tensor, table: torch.Tensor) -> L.KVCacheDesc:
    """Descriptor of a per-row cache k, v of shape (B, nkv, capacity, hd) (contiguous); table = arange(B)."""
    B, nkv, cap, hd = k.shape
    desc = L.KVCacheDesc(k.data_ptr(), v.data_ptr(), table.data_ptr(), 1, 1, cap, nkv * cap * hd, cap * hd, B)
    desc.keep = (k, v, table)          # the descriptor holds raw pointers: keep the tensors alive with it
    return desc


def paged_desc(k: torch.Tensor, v: torch.Tensor, table: torch.Tensor) -> L.KVCacheDesc:
    """Descriptor of a paged pool k, v of shape (num_blocks, nkv, block_size, hd); table (B, nb) int64."""
    nblk, nkv, bs, hd = k.shape
    desc = L.KVCacheDesc(k.data_ptr(), v.data_ptr(), table.data_ptr(), table.stride(0), table.shape[1], bs,
                         nkv * bs * hd, bs * hd, nblk)
    desc.keep = (k, v, table)
    return desc
