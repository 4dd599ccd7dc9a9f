"""The C-ABI library loads and exports every symbol include/*.h declares.

CPU only: nothing here launches a kernel.  Argument validation happens on the
host before any CUDA call, so invalid calls can be checked without a GPU.
"""
import ctypes
import importlib.util
import pathlib
import re

import pytest

ROOT = pathlib.Path(__file__).resolve().parent.parent
PKG = ROOT / "adaptive-specdec_b200"


@pytest.fixture(scope="module")
def lib():
    spec = importlib.util.spec_from_file_location("sd_build", PKG / "build.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    mod.build()
    from specdec import _lib
    return _lib.lib()


def _declared():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        src = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names |= set(re.findall(r"\b(sd_[a-z0-9_]+)\s*\(", src))
    return sorted(names)


def test_every_declared_symbol_is_exported(lib):
    declared = _declared()
    assert len(declared) >= 12
    missing = [n for n in declared if not hasattr(lib, n)]
    assert not missing, missing


def test_bindings_cover_the_header(lib):
    from specdec import _lib
    assert set(_declared()) <= set(_lib._SIGNATURES)


def test_version_and_workspace_sizes(lib):
    assert lib.sd_version() >= 1
    small = lib.sd_sampling_workspace_bytes(8, 72, 32, 0)
    big = lib.sd_sampling_workspace_bytes(64, 576, 151936, 2)
    assert small > 0 and big > 0
    # the small-V path materialises probabilities: bytes grow with n_vec * V
    assert lib.sd_sampling_workspace_bytes(64, 576, 2048, 0) > 576 * 2048 * 4


def test_invalid_arguments_rejected_on_host(lib):
    n = ctypes.c_void_p(0)
    # B = 0, NULL pointers: rejected before any launch
    rc = lib.sd_verify_sample(n, 0, 0, n, 0, 0, 2, n, 0, n, 0, n, n, 0, 4, 151936, 0.7, 0.9, 0,
                              n, n, n, n, n, 0, n)
    assert rc == -22
    rc = lib.sd_to_probs(n, 0, 7, 1, 10, 1.0, 1.0, 0, n, 10, n, 0, n)    # bad dtype
    assert rc == -22
    rc = lib.sd_kv_commit(n, n, 4, 1, n, n)
    assert rc == -22
    rc = lib.sd_verify_attn(n, 0, 0, 0, n, n, n, n, 1, 32, 8, 128, 100, 5, 0.1, n, 0, 0, 0, 2, n,
                            0, n)
    assert rc == -22


def test_new_entry_points_validate_on_host(lib):
    """The fused QK-norm / RoPE / append, the paged K/V calls and the layer
    kernels reject bad arguments (or do nothing for empty batches) before
    any CUDA call."""
    n = ctypes.c_void_p(0)
    d = ctypes.c_void_p(256)                            # a non-null stand-in never dereferenced
    qkv = lambda **kw: lib.sd_qkv_norm_rope_append(   # noqa: E731
        kw.get("q", d), 0, d, 0, d, 0, kw.get("qw", n), kw.get("kw", n), 1e-6, d, d, 0, 0, d, d,
        kw.get("bt", n), kw.get("bts", 0), kw.get("npages", 0), d, kw.get("B", 2), 3, 4, 2,
        kw.get("D", 128), kw.get("C", 64), d, n, n)
    assert qkv(q=n) == -22                              # NULL input
    assert qkv(D=7) == -95                              # odd head dimension
    assert qkv(D=512) == -95                            # above 256
    assert qkv(qw=d) == -22                             # one norm weight without the other
    assert qkv(bt=d, bts=0, npages=4) == -22            # paged without a table width
    assert qkv(bt=d, bts=1, npages=4, C=200) == -22     # C beyond bt_stride * SD_KV_PAGE
    assert qkv(B=0) == 0                                # nothing to do
    assert lib.sd_kv_append_paged(d, d, d, d, 0, 0, 0, n, 4, 8, d, 2, 2, 128, 1, 2, n, n) == -22
    assert lib.sd_kv_append_paged(d, d, d, d, 0, 0, 0, d, 0, 8, d, 2, 2, 128, 1, 2, n, n) == -22
    assert lib.sd_verify_attn_paged(d, 0, 0, 0, d, d, n, 4, 8, d, n, 1, 32, 8, 128, 5, 0.1, d,
                                    0, 0, 0, 2, d, 1 << 20, n) == -22
    assert lib.sd_rmsnorm(n, 0, d, 1e-6, d, 0, 4, 128, n) == -22
    assert lib.sd_rmsnorm(d, 0, d, 1e-6, d, 0, 0, 128, n) == 0          # no rows
    assert lib.sd_add_rmsnorm(d, 0, d, 0, d, 1e-6, d, 0, d, 0, 4, 9000, n) == -95
    assert lib.sd_add_rmsnorm(d, 0, d, 0, d, 1e-6, d, 0, d, 0, 0, 4096, n) == 0
    assert lib.sd_silu_mul(d, 0, d, 0, 4, 0, n) == -22
