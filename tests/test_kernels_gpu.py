"""Kernel-level numerics on the B200 through the C ABI, against plain PyTorch fp32 references.

bf16 tolerances: every output is rounded to bf16 (relative step 2^-8), so a kernel agrees with
the fp32 reference within 1e-2 of the output's max magnitude; fp32 kernels within 1e-5.
"""

import ctypes as C

import numpy as np
import pytest
import torch

from thesis_b200 import lib

pytestmark = pytest.mark.gpu


def _gemm(x, w, epi=lib.EPI_STORE, residual=None, n_out=None, up_offset=0):
    n_tok, k = x.shape
    n_out = n_out or w.shape[0]
    dt = lib.BF16 if x.dtype == torch.bfloat16 else lib.F32
    y = torch.empty(n_tok, n_out, dtype=x.dtype, device=x.device)
    L = lib.load()
    ws_bytes = L.eesd_gemm_workspace_bytes(n_tok, n_out, k, epi)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=x.device)
    lib.call("eesd_gemm", dt, epi, x.data_ptr(), w.data_ptr(), lib.ptr(residual), y.data_ptr(), n_tok, n_out, k,
             up_offset, ws.data_ptr(), ws_bytes, lib.stream_ptr())
    bits = C.c_int(0)
    lib.check(L.eesd_status_read(ws.data_ptr(), C.byref(bits), lib.stream_ptr()), "status")
    return y


def _close(got, ref, tol):
    got, ref = got.float(), ref.float()
    err = (got - ref).abs().max().item() / max(ref.abs().max().item(), 1e-30)
    assert err < tol, err


@pytest.mark.parametrize("n_out,k", [(256, 512), (6144, 4096), (4096, 14336), (1000, 1024)])
@pytest.mark.parametrize("n_tok", [1, 7, 64, 320, 600])
def test_gemm_bf16_store(cuda_dev, n_out, k, n_tok):
    g = torch.Generator(device=cuda_dev).manual_seed(n_tok + n_out)
    x = torch.randn(n_tok, k, device=cuda_dev, generator=g).bfloat16()
    w = (torch.randn(n_out, k, device=cuda_dev, generator=g) * 0.02).bfloat16()
    _close(_gemm(x, w), x.float() @ w.float().T, 1e-2)


@pytest.mark.parametrize("n_tok", [3, 64, 320])
def test_gemm_bf16_residual_and_swiglu(cuda_dev, n_tok):
    g = torch.Generator(device=cuda_dev).manual_seed(7)
    k, n_out, inter = 1024, 512, 768
    x = torch.randn(n_tok, k, device=cuda_dev, generator=g).bfloat16()
    w = (torch.randn(n_out, k, device=cuda_dev, generator=g) * 0.02).bfloat16()
    r = torch.randn(n_tok, n_out, device=cuda_dev, generator=g).bfloat16()
    ref = (r.float() + (x.float() @ w.float().T).bfloat16().float()).bfloat16()
    _close(_gemm(x, w, lib.EPI_RESIDUAL, residual=r), ref, 1e-2)
    w13 = (torch.randn(2 * inter, k, device=cuda_dev, generator=g) * 0.05).bfloat16()
    gu = (x.float() @ w13.float().T).bfloat16().float()
    gg, uu = gu[:, :inter], gu[:, inter:]
    ref = (torch.nn.functional.silu(gg).bfloat16().float() * uu).bfloat16()
    _close(_gemm(x, w13, lib.EPI_SWIGLU, n_out=inter, up_offset=inter), ref, 1e-2)


@pytest.mark.parametrize("mma_n", [0, 64])
def test_gemm_bf16_is_batch_invariant(cuda_dev, mma_n):
    """A token row's result is bit-identical whatever the number of tokens in the launch."""
    g = torch.Generator(device=cuda_dev).manual_seed(3)
    k, n_out = 4096, 6144
    x = torch.randn(640, k, device=cuda_dev, generator=g).bfloat16()
    w = (torch.randn(n_out, k, device=cuda_dev, generator=g) * 0.02).bfloat16()
    lib.call("eesd_set_option", lib.OPT_MMA_N, mma_n)
    try:
        full = _gemm(x, w)
        for n in (1, 4, 16, 64, 100, 320, 333):
            assert torch.equal(_gemm(x[:n].contiguous(), w), full[:n]), n
    finally:
        lib.call("eesd_set_option", lib.OPT_MMA_N, 0)


@pytest.mark.parametrize("n_tok", [257, 320, 352, 384])
def test_gemm_two_mma_split_is_bit_identical(cuda_dev, n_tok):
    """A token tile above 256 tokens takes two MMAs per k-step; their N split (192 + rest by
    default, equal halves, 256 + rest) changes no bit of the result."""
    g = torch.Generator(device=cuda_dev).manual_seed(n_tok)
    k, n_out = 4096, 4096
    x = torch.randn(n_tok, k, device=cuda_dev, generator=g).bfloat16()
    w = (torch.randn(n_out, k, device=cuda_dev, generator=g) * 0.02).bfloat16()
    r = torch.randn(n_tok, n_out, device=cuda_dev, generator=g).bfloat16()
    outs = []
    try:
        for split in (192, 0, 256, 128):
            lib.call("eesd_set_option", lib.OPT_MMA_SPLIT, split)
            outs.append((_gemm(x, w), _gemm(x, w, lib.EPI_RESIDUAL, residual=r)))
    finally:
        lib.call("eesd_set_option", lib.OPT_MMA_SPLIT, 192)
    for y, z in outs[1:]:
        assert torch.equal(y, outs[0][0]) and torch.equal(z, outs[0][1])
    _close(outs[0][0], x.float() @ w.float().T, 1e-2)


def test_gemm_swiglu_on_cta_pairs(cuda_dev):
    """W13 + SwiGLU at the 8B shape runs on CTA pairs (cta_group::2, M = 256, each CTA loading half
    of the token tile): it matches the fp32 reference and the single-CTA kernel, and a token row's
    result is bit-identical whatever the number of tokens in the launch."""
    g = torch.Generator(device=cuda_dev).manual_seed(11)
    k, inter = 4096, 14336
    x = torch.randn(333, k, device=cuda_dev, generator=g).bfloat16()
    w13 = (torch.randn(2 * inter, k, device=cuda_dev, generator=g) * 0.02).bfloat16()

    def swiglu(xx):
        return _gemm(xx, w13, lib.EPI_SWIGLU, n_out=inter, up_offset=inter)

    full = swiglu(x)
    gu = (x.float() @ w13.float().T).bfloat16().float()
    ref = (torch.nn.functional.silu(gu[:, :inter]).bfloat16().float() * gu[:, inter:]).bfloat16()
    _close(full, ref, 1e-2)
    for n in (1, 16, 64, 160, 320):
        assert torch.equal(swiglu(x[:n].contiguous()), full[:n]), n
    lib.call("eesd_set_option", lib.OPT_PAIR, 0)
    try:
        _close(swiglu(x), ref, 1e-2)
    finally:
        lib.call("eesd_set_option", lib.OPT_PAIR, 1)


@pytest.mark.parametrize("n_tok", [1, 70, 300])
def test_gemm_f32(cuda_dev, n_tok):
    g = torch.Generator(device=cuda_dev).manual_seed(1)
    x = torch.randn(n_tok, 512, device=cuda_dev, generator=g)
    w = torch.randn(384, 512, device=cuda_dev, generator=g) * 0.02
    r = torch.randn(n_tok, 384, device=cuda_dev, generator=g)
    _close(_gemm(x, w), x @ w.T, 1e-5)
    _close(_gemm(x, w, lib.EPI_RESIDUAL, residual=r), r + x @ w.T, 1e-5)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_rmsnorm(cuda_dev, dtype):
    g = torch.Generator(device=cuda_dev).manual_seed(2)
    x = torch.randn(37, 4096, device=cuda_dev, generator=g).to(dtype)
    w = (1 + 0.1 * torch.randn(4096, device=cuda_dev, generator=g)).to(dtype)
    rows = torch.tensor([5, 0, 36, 5], dtype=torch.int32, device=cuda_dev)
    y = torch.empty(4, 4096, dtype=dtype, device=cuda_dev)
    lib.call("eesd_rmsnorm", lib.BF16 if dtype == torch.bfloat16 else lib.F32, x.data_ptr(), rows.data_ptr(),
             w.data_ptr(), y.data_ptr(), 4, 4096, 1e-5, lib.stream_ptr())
    xf = x[rows.long()].float()
    ref = w * (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-5)).to(dtype)
    _close(y, ref, 1e-2 if dtype == torch.bfloat16 else 1e-5)


def test_greedy_accept(cuda_dev):
    cols = 5
    seq = torch.tensor([[9, 1, 2, 3, 4], [9, 5, 6, 7, 8], [9, 1, 1, 1, 1]], dtype=torch.int32, device=cuda_dev)
    y = torch.tensor([1, 2, 0, 3, 4,    5, 6, 7, 8, 11,    2, 1, 1, 1, 1], dtype=torch.int32, device=cuda_dev)
    vinfo = torch.tensor([[0, 5, 0], [5, 5, 1], [10, 5, 2]], dtype=torch.int32, device=cuda_dev)
    acc = torch.empty(3, dtype=torch.int32, device=cuda_dev)
    lib.call("eesd_greedy_accept", y.data_ptr(), vinfo.data_ptr(), 3, seq.data_ptr(), cols, acc.data_ptr(),
             lib.stream_ptr())
    assert acc.tolist() == [2, 4, 0]
    assert seq[:, 0].tolist() == [0, 11, 2]


@pytest.mark.parametrize("rows,k", [(300, 512), (6144, 4096)])
def test_pack_weight_layout(cuda_dev, rows, k):
    """Tile-packed weights: tile (m, j) = rows 128m.. x cols 64j.., contiguous, zero-padded."""
    w = torch.randn(rows, k, device=cuda_dev).bfloat16()
    n = lib.load().eesd_packed_weight_bytes(rows, k)
    out = torch.empty(n // 2, dtype=torch.bfloat16, device=cuda_dev)
    lib.call("eesd_pack_weight", w.data_ptr(), rows, k, out.data_ptr(), lib.stream_ptr())
    mt, kb = -(-rows // 128), k // 64
    wp = torch.zeros(mt * 128, k, dtype=torch.bfloat16, device=cuda_dev)
    wp[:rows] = w
    ref = wp.view(mt, 128, kb, 64).permute(0, 2, 1, 3).reshape(-1)
    assert torch.equal(out, ref)


def _one_layer_model(cuda_dev, head_dim, max_seq=1088):
    from thesis_b200.config import ModelConfig
    from thesis_b200.model import DeviceModel, ModelWeights

    cfg = ModelConfig(vocab_size=512, dim=8 * head_dim, n_layers=1, n_heads=8, n_kv_heads=2, head_dim=head_dim,
                      intermediate_size=1024)
    w = ModelWeights.synthetic(cfg, seed=0, dtype=torch.bfloat16, device=cuda_dev)
    dm = DeviceModel(w, max_batch=4, max_seq=max_seq, max_tokens=64)
    g = torch.Generator(device=cuda_dev).manual_seed(1)
    dm.k_cache.copy_(torch.randn(dm.k_cache.shape, generator=g, device=cuda_dev))   # stands in for a prefill
    dm.v_cache.copy_(torch.randn(dm.v_cache.shape, generator=g, device=cuda_dev))
    x = torch.randn(64, cfg.dim, generator=g, device=cuda_dev).bfloat16()
    return dm, x


@pytest.mark.parametrize("pos0", [3, 254, 1000])
def test_layer_is_batch_invariant_across_step_shapes(cuda_dev, pos0):
    """A token's layer output does not depend on the call it runs in: token j of a 5-token
    verify-shaped block equals the same token run alone in a draft-shaped call (4-warp attention
    variant instead of the 8-warp one, other GEMM token tiles), bit for bit.  This is what makes
    speculative output identical to autoregressive output."""
    dm, x = _one_layer_model(cuda_dev, 128)
    xv = x[:10].clone()
    dm.forward_layers(xv, dm.upload(dm.pack([(0, pos0, 5), (1, 700, 5)])), 0, 1)
    for j in range(5):
        xd = x[j:j + 1].clone()
        dm.forward_layers(xd, dm.upload(dm.pack([(0, pos0 + j, 1)])), 0, 1)
        assert torch.equal(xd[0], xv[j]), j
    dm.check()


@pytest.mark.parametrize("gamma,item_tokens", [(4, 8), (6, 4), (0, 8)])
def test_round_metadata_matches_host_packing(cuda_dev, gamma, item_tokens):
    """The device-built round metadata (eesd_round_meta) equals what the host packing builds for
    the same blocks, and eesd_round_advance moves each row by its accepted drafts + 1."""
    from thesis_b200.packing import pack

    cols = gamma + 1
    act = np.array([5, 0, 3, 7], dtype=np.int32)
    pos = np.arange(8, dtype=np.int32) * 37 + 100
    n = len(act)
    L = lib.load()
    ints = L.eesd_round_meta_ints(n, gamma, item_tokens)
    out = torch.zeros(ints, dtype=torch.int32, device=cuda_dev)
    act_d = torch.from_numpy(act).to(cuda_dev)
    pos_d = torch.from_numpy(pos).to(cuda_dev)
    lib.call("eesd_round_meta", act_d.data_ptr(), n, pos_d.data_ptr(), 8, gamma, item_tokens, out.data_ptr(),
             lib.stream_ptr())
    o = out.cpu().numpy()
    for j in range(cols):
        st = o[j * 10 * n:(j + 1) * 10 * n]
        ph = pack([(int(r), int(pos[r]) + j, 1) for r in act], item_tokens)
        assert np.array_equal(st[:n], ph.tok_pos) and np.array_equal(st[n:2 * n], ph.tok_row)
        assert np.array_equal(st[2 * n:6 * n].reshape(n, 4), ph.blk)
        assert sorted(map(tuple, st[6 * n:8 * n].reshape(n, 2))) == sorted(map(tuple, ph.items))
        assert np.array_equal(st[8 * n:9 * n], act * cols + j) and np.array_equal(st[9 * n:], act * cols + j + 1)
    v = o[cols * 10 * n:]
    N, ni = n * cols, -(-cols // item_tokens)
    ph = pack([(int(r), int(pos[r]), cols) for r in act], item_tokens)
    assert np.array_equal(v[:N], ph.tok_pos) and np.array_equal(v[N:2 * N], ph.tok_row)
    assert np.array_equal(v[2 * N:2 * N + 4 * n].reshape(n, 4), ph.blk)
    items = v[2 * N + 4 * n:2 * N + 4 * n + 2 * n * ni].reshape(-1, 2)
    assert sorted(map(tuple, items)) == sorted(map(tuple, ph.items))
    rows = v[2 * N + 4 * n + 2 * n * ni:3 * N + 4 * n + 2 * n * ni]
    assert np.array_equal(rows, (act[:, None] * cols + np.arange(cols)[None, :]).reshape(-1))
    vinfo = v[3 * N + 4 * n + 2 * n * ni:].reshape(n, 3)
    assert np.array_equal(vinfo, np.stack([np.arange(n) * cols, np.full(n, cols), act], axis=1))
    acc = torch.tensor([0, 3, 1, 2], dtype=torch.int32, device=cuda_dev)
    lib.call("eesd_round_advance", act_d.data_ptr(), n, acc.data_ptr(), pos_d.data_ptr(), 8, lib.stream_ptr())
    want = pos.copy()
    want[act] += acc.cpu().numpy() + 1
    assert np.array_equal(pos_d.cpu().numpy(), want)


@pytest.mark.parametrize("n", [1, 37, 256, 300])
def test_head_two_row_tiles_per_cta(cuda_dev, n):
    """Head launches of up to 256 tokens take two 128-row tiles per CTA (two accumulators); a
    vocabulary of 11 tiles leaves the last CTA half past the end.  The token ids equal the
    one-tile kernel's and the argmax of the stored logits, through the model head (tile-packed
    weights) and, up to its 128 rows, the allocation-free head (row-major weights)."""
    from dataclasses import replace

    from thesis_b200.config import preset
    from thesis_b200.model import DeviceModel, ModelWeights

    cfg = replace(preset("c1s"), vocab_size=1300, n_layers=1)
    w = ModelWeights.synthetic(cfg, seed=4, dtype=torch.bfloat16, device=cuda_dev)
    dm = DeviceModel(w, max_batch=1, max_seq=64, max_tokens=320)
    g = torch.Generator(device=cuda_dev).manual_seed(n)
    x = torch.randn(n, cfg.dim, device=cuda_dev, generator=g).bfloat16()

    def static_head():   # its fixed scratch holds up to 128 rows
        ids = torch.full((n,), -1, dtype=torch.int32, device=cuda_dev)
        if n > 128:
            return None
        lib.call("eesd_head_argmax_static", x.data_ptr(), n, None, n, cfg.dim, cfg.vocab_size, w.t["norm"].data_ptr(),
                 w.t["lm_head"].data_ptr(), cfg.norm_eps, ids.data_ptr(), None, lib.stream_ptr())
        return ids

    two, two_static = dm.head_argmax(x), static_head()
    lib.call("eesd_set_option", lib.OPT_HEAD_TWO_TILES, 0)
    try:
        one, one_static = dm.head_argmax(x), static_head()
    finally:
        lib.call("eesd_set_option", lib.OPT_HEAD_TWO_TILES, 1)
    ids, lg = dm.head_argmax(x, logits=True)
    dm.check()
    assert torch.equal(two, one)
    if n <= 128:
        assert torch.equal(two_static, one_static) and torch.equal(two, two_static)
    assert torch.equal(two.long(), lg.float().argmax(-1))
