"""The C-ABI extension builds, loads without a GPU, and exports every symbol of include/eesd.h.
No compute call here (CPU suite)."""

import ctypes as C
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def L():
    from thesis_b200 import build, lib

    build.build()
    return lib.load()


def _declared():
    text = (ROOT / "include" / "eesd.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(eesd_\w+)\s*\(", text)))


def test_every_declared_symbol_is_exported_and_bound(L):
    from thesis_b200 import lib

    names = _declared()
    assert len(names) >= 20
    for n in names:
        assert hasattr(L, n), n                      # exported by the .so
        assert n in lib.SIGNATURES, n                 # bound by the ctypes layer


def test_library_metadata(L):
    assert L.eesd_version() >= 100
    assert L.eesd_attn_item_tokens(32, 8) == 8        # 32 query rows per attention work item
    assert L.eesd_attn_item_tokens(32, 32) == 32
    assert L.eesd_attn_item_tokens(6, 4) == -1        # heads must be a multiple of KV heads


def test_workspace_sizes(L):
    from thesis_b200 import lib

    d = lib.ModelDesc()
    d.dtype, d.n_layers, d.dim, d.n_heads, d.n_kv_heads, d.head_dim = lib.BF16, 32, 4096, 32, 8, 128
    d.intermediate, d.vocab, d.max_batch, d.max_seq, d.max_tokens = 14336, 128256, 64, 1088, 2048
    ws = L.eesd_model_workspace_bytes(C.byref(d))
    acts = 2048 * (4096 + 6144 + 4096 + 14336) * 2
    # split-K partial tiles: output tiles x token tiles x splits x 128 rows x columns x fp32; the
    # largest is O / W2 at 2048 tokens (32 row tiles, 6 token tiles of 352, 4 splits)
    partials = 32 * 6 * 4 * 128 * 352 * 4
    assert acts + partials < ws < acts + partials + (1 << 22)
    # status word + QKV partials (48 row tiles, 2 splits, 64 tokens)
    assert L.eesd_gemm_workspace_bytes(64, 6144, 4096, lib.EPI_STORE) == 256 + 48 * 2 * 128 * 64 * 4
    # status word + fp32-path scratch + SwiGLU partials (4 row tiles, 4 splits, gate + up columns)
    assert L.eesd_gemm_workspace_bytes(64, 512, 4096, lib.EPI_SWIGLU) == 256 + 64 * 1024 * 4 + 4 * 4 * 128 * 128 * 4
    # the LM-head-sized weight is never split
    assert L.eesd_gemm_workspace_bytes(64, 128256, 4096, lib.EPI_STORE) == 256
    assert L.eesd_gemm_workspace_bytes(0, 6144, 4096, lib.EPI_STORE) == 0


def test_argument_errors_are_reported_before_any_launch(L):
    from thesis_b200 import lib

    d = lib.ModelDesc()
    d.dtype, d.n_layers, d.dim, d.n_heads, d.n_kv_heads, d.head_dim = lib.BF16, 2, 256, 4, 2, 96
    h = C.c_void_p()
    assert L.eesd_model_create(C.byref(d), C.byref(h)) == lib.ERR_ARG
    assert b"head_dim" in L.eesd_last_error()
    d.head_dim, d.intermediate, d.vocab, d.max_batch, d.max_seq, d.max_tokens = 64, 512, 512, 2, 128, 64
    assert L.eesd_model_create(C.byref(d), C.byref(h)) == lib.ERR_ARG
    assert b"workspace" in L.eesd_last_error()
    assert L.eesd_set_option(lib.OPT_MMA_N, 24) == lib.ERR_ARG
    assert L.eesd_gemm(lib.BF16, 7, None, None, None, None, 1, 1, 1, 0, None, 0, None) == lib.ERR_ARG


def test_sources_contain_no_cluster_multicast_loads():
    """Every kernel may run in the 8-GPU configuration: no multicast TMA forms anywhere."""
    for p in (ROOT / "thesis_b200" / "csrc").iterdir():
        assert "multicast" not in p.read_text(), p
