"""Varlen GQA attention and the RoPE / KV append, through the exported C-ABI primitives
(``eesd_attn_varlen_gqa``, ``eesd_rope_kv_append``), against plain PyTorch fp32 attention.

The reference op is ``_attend`` (solutions/packed.py:142-166): per bucket, SDPA of the GQA-folded
queries ``[b, Hkv, G T, D]`` over the first L cached positions with a causal bool mask, after
``apply_rope`` on q and k and the in-place cache write (solutions/packed.py:170-181).  Here the
expected output is that computation in fp32 from the same bf16 (or fp32) inputs.

Covered: contexts 1 .. 2048, including both sides of every 64-key tile edge (63 / 64 / 65,
1087); decode (T = 1), verify (T = 5, 9) and prefill-chunk blocks (T up to 512, several work
items per block); GQA group 4 and MHA; head_dim 64 and 128; the in-kernel RoPE / append variant
against the separate RoPE / KV kernel (bit-identical outputs and caches).

Tolerances: bf16 outputs within 2e-2 of the fp32 attention (relative = max |a - b| / max |b|),
fp32 within 1e-5; the rotated keys in the cache are bit-identical to PyTorch's bf16 ``apply_rope``.
"""

import numpy as np
import pytest
import torch

from thesis_b200 import lib
from thesis_b200.config import ModelConfig
from thesis_b200.model import build_rope_cache
from thesis_b200.packing import pack

pytestmark = pytest.mark.gpu

MAX_BATCH, MAX_SEQ = 8, 2112
BAD_INDEX, TIMEOUT_BITS = 1 << 3, 0b111

SCENARIOS = {
    # name: [(row, pos0, T)]; contexts pos0 + T span 1 .. 2048 and sit on both sides of tile edges
    "decode": [(0, 0, 1), (1, 62, 1), (2, 63, 1), (3, 64, 1), (4, 126, 1), (5, 1086, 1), (6, 2047, 1),
               (7, 500, 1)],
    "verify5": [(0, 0, 5), (1, 58, 5), (2, 59, 5), (3, 60, 5), (4, 123, 5), (5, 1082, 5), (6, 2043, 5)],
    "verify9": [(0, 0, 9), (1, 54, 9), (2, 55, 9), (3, 1078, 9), (4, 2039, 9)],
    "prefill": [(0, 0, 512), (1, 512, 300), (2, 1500, 37), (3, 63, 2)],
    # several blocks of one row in one call: later blocks read the keys earlier blocks write
    # (a prefill chunk followed by the row's next tokens)
    "same_row": [(0, 0, 9), (0, 9, 1), (1, 100, 5), (1, 105, 5), (2, 60, 3), (2, 63, 2)],
}


def _cfg(n_heads, n_kv_heads, head_dim):
    return ModelConfig(vocab_size=8, dim=n_heads * head_dim, n_layers=1, n_heads=n_heads, n_kv_heads=n_kv_heads,
                       head_dim=head_dim, intermediate_size=64, rope_theta=500000.0)


def _upload(ph, dev):
    parts = [torch.from_numpy(np.ascontiguousarray(a, dtype=np.int32).reshape(-1)).to(dev)
             for a in (ph.tok_pos, ph.tok_row, ph.blk, ph.items)]
    b = lib.Batch(ph.n_tokens, ph.n_blocks, len(ph.items), ph.max_ctx, *(p.data_ptr() for p in parts))
    return b, parts


def _rope_ref(x, pos, cos, sin):
    """common/model.py:143-150 in x's dtype: cos/sin cast to the model dtype, every product and the
    sum rounded as PyTorch rounds them."""
    c = cos[pos].to(x.dtype)[:, None, :]
    s = sin[pos].to(x.dtype)[:, None, :]
    x1, x2 = x.chunk(2, dim=-1)
    return x * c + torch.cat((-x2, x1), dim=-1) * s


def _attend_ref(q, kc, vc, blocks, offsets, n_heads, n_kv_heads, head_dim):
    """fp32 SDPA per block: query t of block (row, pos0, T) reads keys 0 .. pos0 + t of its row."""
    G = n_heads // n_kv_heads
    qf, kf, vf = q.float(), kc.float(), vc.float()
    out = torch.zeros(q.shape[0], n_heads * head_dim, dtype=torch.float32, device=q.device)
    for i, (row, pos0, T) in enumerate(blocks):
        s = int(offsets[i])
        L = pos0 + T
        qb = qf[s:s + T].view(T, n_kv_heads, G, head_dim).permute(1, 2, 0, 3).reshape(n_kv_heads, G * T, head_dim)
        K, V = kf[row, :, :L], vf[row, :, :L]
        sc = (qb @ K.transpose(-1, -2)) / head_dim ** 0.5
        qpos = pos0 + torch.arange(T, device=q.device).repeat(G)
        sc = sc.masked_fill(torch.arange(L, device=q.device)[None, :] > qpos[:, None], float("-inf"))
        o = torch.softmax(sc, dim=-1) @ V
        out[s:s + T] = o.view(n_kv_heads, G, T, head_dim).permute(2, 0, 1, 3).reshape(T, n_heads * head_dim)
    return out


def _rel(a, b):
    a, b = a.float(), b.float()
    return (a - b).abs().max().item() / max(b.abs().max().item(), 1e-30)


class Case:
    def __init__(self, dev, dtype, n_heads, n_kv_heads, head_dim, blocks, seed=0):
        self.dev, self.dtype = dev, dtype
        self.H, self.Hkv, self.D = n_heads, n_kv_heads, head_dim
        self.blocks = blocks
        self.item_tokens = lib.load().eesd_attn_item_tokens(n_heads, n_kv_heads)
        self.ph = pack(blocks, self.item_tokens)
        g = torch.Generator(device=dev).manual_seed(seed)
        shape = (MAX_BATCH, n_kv_heads, MAX_SEQ, head_dim)
        self.kc0 = torch.randn(shape, device=dev, generator=g).to(dtype)      # stands in for earlier calls
        self.vc0 = torch.randn(shape, device=dev, generator=g).to(dtype)
        qkv_dim = (n_heads + 2 * n_kv_heads) * head_dim
        self.qkv0 = (torch.randn(self.ph.n_tokens, qkv_dim, device=dev, generator=g) * 2).to(dtype)
        cos, sin = build_rope_cache(_cfg(n_heads, n_kv_heads, head_dim), MAX_SEQ)
        self.cos, self.sin = cos.to(dev).contiguous(), sin.to(dev).contiguous()
        self.dt = lib.BF16 if dtype == torch.bfloat16 else lib.F32

    def expected(self):
        """(output fp32, K cache, V cache) of the reference ops."""
        N, H, Hkv, D = self.ph.n_tokens, self.H, self.Hkv, self.D
        pos = torch.from_numpy(self.ph.tok_pos.astype(np.int64)).to(self.dev)
        row = torch.from_numpy(self.ph.tok_row.astype(np.int64)).to(self.dev)
        q, k, v = self.qkv0.split([H * D, Hkv * D, Hkv * D], dim=-1)
        q = _rope_ref(q.reshape(N, H, D), pos, self.cos, self.sin)
        k = _rope_ref(k.reshape(N, Hkv, D), pos, self.cos, self.sin)
        kc, vc = self.kc0.clone(), self.vc0.clone()
        kc[row, :, pos] = k
        vc[row, :, pos] = v.reshape(N, Hkv, D)
        return _attend_ref(q.reshape(N, H, D), kc, vc, self.blocks, self.ph.offsets, H, Hkv, D), kc, vc

    def run(self, append: bool, spin=None):
        """The primitives: RoPE/KV kernel then attention, or attention with the in-kernel append."""
        qkv, kc, vc = self.qkv0.clone(), self.kc0.clone(), self.vc0.clone()
        out = torch.zeros(self.ph.n_tokens, self.H * self.D, dtype=self.dtype, device=self.dev)
        status = torch.zeros(1, dtype=torch.int32, device=self.dev)
        b, keep = _upload(self.ph, self.dev)
        s = lib.stream_ptr()
        if not append:
            lib.call("eesd_rope_kv_append", self.dt, qkv.data_ptr(), keep[0].data_ptr(), keep[1].data_ptr(),
                     self.ph.n_tokens, self.H, self.Hkv, self.D, self.cos.data_ptr(), self.sin.data_ptr(),
                     kc.data_ptr(), vc.data_ptr(), MAX_BATCH, MAX_SEQ, status.data_ptr(), s)
        if spin is not None:
            lib.call("eesd_set_option", lib.OPT_SPIN_LIMIT, spin)
        try:
            lib.call("eesd_attn_varlen_gqa", self.dt, qkv.data_ptr(), self.H, self.Hkv, self.D, kc.data_ptr(),
                     vc.data_ptr(), MAX_BATCH, MAX_SEQ, b, int(append), self.cos.data_ptr(), self.sin.data_ptr(),
                     out.data_ptr(), status.data_ptr(), s)
            torch.cuda.synchronize()
        finally:
            if spin is not None:
                lib.call("eesd_set_option", lib.OPT_SPIN_LIMIT, -1)
        return out, kc, vc, int(status)


@pytest.mark.parametrize("head_dim", [64, 128])
@pytest.mark.parametrize("heads", [(32, 8), (8, 8)], ids=["gqa4", "mha"])
@pytest.mark.parametrize("scenario", list(SCENARIOS))
def test_attention_bf16_matches_fp32_attention(cuda_dev, scenario, heads, head_dim):
    c = Case(cuda_dev, torch.bfloat16, *heads, head_dim, SCENARIOS[scenario], seed=head_dim + heads[1])
    want, kc_w, vc_w = c.expected()
    out, kc, vc, st = c.run(append=False)
    assert st == 0
    assert torch.equal(kc, kc_w) and torch.equal(vc, vc_w)
    assert _rel(out, want) < 2e-2
    rows = [r for (r, _, _) in c.blocks]
    if len(c.ph.items) == c.ph.n_blocks and len(set(rows)) == len(rows):
        # every block one work item of its own row: the in-kernel RoPE / append
        out2, kc2, vc2, st2 = c.run(append=True)
        assert st2 == 0
        assert torch.equal(kc2, kc) and torch.equal(vc2, vc)
        assert torch.equal(out2, out)


@pytest.mark.parametrize("head_dim", [64, 128])
@pytest.mark.parametrize("scenario", ["decode", "verify5", "verify9"])
def test_attention_fp32_matches_fp32_attention(cuda_dev, scenario, head_dim):
    c = Case(cuda_dev, torch.float32, 16, 4, head_dim, SCENARIOS[scenario], seed=3)
    want, kc_w, vc_w = c.expected()
    out, kc, vc, st = c.run(append=False)
    assert st == 0
    assert _rel(kc, kc_w) < 1e-6 and torch.equal(vc, vc_w)
    assert _rel(out, want) < 1e-5


def test_attention_result_does_not_depend_on_the_other_blocks(cuda_dev):
    """A block's output is bit-identical whether it runs alone or with other blocks of other
    lengths in the same launch (what keeps speculative output equal to autoregressive output)."""
    blocks = SCENARIOS["verify5"]
    full = Case(cuda_dev, torch.bfloat16, 32, 8, 128, blocks, seed=9)
    out, _, _, _ = full.run(append=True)
    for i, blk in enumerate(blocks):
        one = Case(cuda_dev, torch.bfloat16, 32, 8, 128, [blk], seed=9)
        one.kc0, one.vc0 = full.kc0, full.vc0
        one.qkv0 = full.qkv0[full.ph.block_slice(i)].contiguous()
        o1, _, _, _ = one.run(append=True)
        assert torch.equal(o1, out[full.ph.block_slice(i)]), blk


def test_attention_reports_bad_blocks_and_timeouts(cuda_dev):
    c = Case(cuda_dev, torch.bfloat16, 32, 8, 128, SCENARIOS["decode"], seed=4)
    # a block whose row is outside the cache: skipped, bad-index bit set
    c.ph.blk[1, 2] = MAX_BATCH
    _, _, _, st = c.run(append=False)
    assert st & BAD_INDEX
    c.ph.blk[1, 2] = 1
    # every key-tile wait gives up at once: the call returns with a timeout bit, copies drain
    _, _, _, st = c.run(append=True, spin=0)
    assert st & TIMEOUT_BITS
    # the context is still usable
    want, _, _ = c.expected()
    out, _, _, st = c.run(append=True)
    assert st == 0 and _rel(out, want) < 2e-2
