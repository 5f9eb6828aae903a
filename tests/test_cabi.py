"""The C ABI library loads and exports every entry point include/forgeserve_b200.h declares; host-side argument
checks answer with a status and a message (no GPU needed for these)."""

import ctypes
import re
from pathlib import Path

import pytest

from forgeserve_b200 import _lib as L

HEADER = Path(__file__).resolve().parents[1] / "include" / "forgeserve_b200.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(fs_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    if not L.LIB_PATH.exists():
        from forgeserve_b200 import build
        build.build()
    return L.load()


def test_every_declared_symbol_is_exported_and_bound(lib):
    names = declared_functions()
    assert len(names) >= 14
    for name in names:
        assert hasattr(lib, name), name
        assert name in L.SIGNATURES, f"{name} has no ctypes signature"
    assert set(L.SIGNATURES) == set(names)


def test_version_and_empty_error(lib):
    assert lib.fs_version() == 100
    assert lib.fs_last_error() in (b"",) or isinstance(lib.fs_last_error(), bytes)


def test_null_pointers_are_refused_with_a_message(lib):
    rc = lib.fs_gemm(None, 64, None, 64, None, 64, None, 0, 4, 64, 64, 64, L.FS_EPI_STORE, L.FS_BF16, None)
    assert rc != 0
    assert b"NULL" in lib.fs_last_error()
    rc = lib.fs_rmsnorm(None, 8, None, None, 8, 3, 8, 1e-5, L.FS_F32, None)
    assert rc != 0 and b"NULL" in lib.fs_last_error()


def test_shape_checks(lib):
    p = ctypes.c_void_p(16)          # never dereferenced: the checks fail before any launch
    rc = lib.fs_gemm(p, 64, p, 64, p, 64, None, 0, 4, 96, 64, 40, L.FS_EPI_SWIGLU, L.FS_BF16, None)
    assert rc != 0 and b"swiglu" in lib.fs_last_error()
    rc = lib.fs_gemm(p, 32, p, 64, p, 64, None, 0, 4, 64, 64, 64, L.FS_EPI_STORE, L.FS_BF16, None)
    assert rc != 0 and b"stride" in lib.fs_last_error()
    rc = lib.fs_gemm(p, 64, p, 64, p, 64, None, 0, 4, 64, 64, 64, L.FS_EPI_RESIDUAL, L.FS_BF16, None)
    assert rc != 0 and b"residual" in lib.fs_last_error()
    rc = lib.fs_gemm(p, 64, p, 64, p, 64, None, 0, 4, 64, 64, 64, 7, L.FS_BF16, None)
    assert rc != 0
    with pytest.raises(RuntimeError, match="fs_gemm failed"):
        L.check(rc, "fs_gemm")


def test_empty_work_is_a_no_op(lib):
    assert lib.fs_gemm(None, 64, None, 64, None, 64, None, 0, 0, 64, 64, 64, 0, 1, None) == 0
    assert lib.fs_argmax(None, 0, 10, 10, None, 1, None) == 0
    assert lib.fs_embed(None, 0, None, 10, 8, None, 1, None) == 0


def test_static_decode_refuses_a_call_beyond_its_fixed_scratch_on_the_host(lib):
    """fs_attention_decode_static answers a call whose split partials exceed its fixed 4 MiB array with an error
    naming the size, before any device work (the pointers below are never dereferenced)."""
    p = 4096
    B, nh, nkv, hd, n_slots = 64, 32, 8, 128, 2048
    need = lib.fs_attention_decode_workspace(B, nh, nkv, hd, n_slots)
    assert need == B * nh * 4 * (hd + 2) * 4 > 4 << 20
    assert lib.fs_attention_decode_workspace(B, nh, nkv, hd, 1536) == B * nh * 3 * (hd + 2) * 4 <= 4 << 20
    desc = L.KVCacheDesc(k=p, v=p, table=p, table_stride=128, table_cols=128, block_size=16,
                         block_stride=nkv * 16 * hd, head_stride=16 * hd, num_blocks=128)
    rc = lib.fs_attention_decode_static(ctypes.c_void_p(p), nh * hd, ctypes.byref(desc), n_slots, ctypes.c_void_p(p),
                                        ctypes.c_void_p(p), nh * hd, B, nh, nkv, hd, ctypes.c_float(hd ** -0.5),
                                        L.FS_BF16, None)
    assert rc == -1
    assert f"needs {need} bytes of scratch".encode() in lib.fs_last_error()


def test_rope_refuses_non_positive_head_shapes_on_the_host(lib):
    """A zero head_dim or head count is refused with a message before any device work (the vectorised path's
    chunk arithmetic divides by head_dim / 16); the pointers below are never dereferenced."""
    p = 4096
    desc = L.KVCacheDesc(k=p, v=p, table=p, table_stride=4, table_cols=4, block_size=16, block_stride=2 * 16 * 128,
                         head_stride=16 * 128, num_blocks=4)
    for nh, nkv, hd in ((4, 2, 0), (0, 2, 128), (4, 0, 128)):
        rc = lib.fs_rope_kv_write(ctypes.c_void_p(p), 1024, ctypes.c_void_p(p), ctypes.c_void_p(p), 64,
                                  ctypes.c_void_p(p), ctypes.byref(desc), 1, 1, nh, nkv, hd, 0, 1, 1, L.FS_BF16, None)
        assert rc == -1
        assert b"must be positive" in lib.fs_last_error()
