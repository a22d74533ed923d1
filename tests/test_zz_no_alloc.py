"""The allocation-free exit head, checked through the C ABI.

``eesd_head_argmax_static`` exists for callers that cannot allocate device memory: a serving
runtime whose allocator is locked on its decode path, code running inside a foreign stream
capture, or a plug-in that is only handed raw input and output pointers.  Its scratch is a fixed
array inside the library instead of a caller workspace.  Checked here:

* it returns exactly the token ids that ``eesd_head_argmax`` returns for the same rows (integer
  outputs: exact equality), on two calls in a row, since the shared array keeps the previous
  call's contents;
* its ids are the argmax of a plain PyTorch fp32 ``norm(x) @ W^T`` at the Llama3-8B head shape,
  except where two logits are closer than the bf16 rounding of the logits;
* a call allocates no device memory;
* a row index outside ``x`` and a bounded wait that gives up are reported (every id -1, status
  bits in ``status_out``), and the next call is correct again;
* sizes beyond the fixed scratch are rejected.

This file is collected last so that a run stopping at the first failure has run every other test.
"""

from dataclasses import replace

import pytest
import torch

from thesis_b200 import lib
from thesis_b200.config import preset
from thesis_b200.model import DeviceModel, ModelWeights
from thesis_b200.synthetic import synthetic_weights

pytestmark = pytest.mark.gpu

BAD_INDEX, TIMEOUT_BITS = 1 << 3, 0b111


def _static_head(dm: DeviceModel, x: torch.Tensor, rows, n: int):
    """(ids, status bits) of one call of the allocation-free head."""
    cfg = dm.cfg
    ids = torch.full((n,), -7, dtype=torch.int32, device=x.device)
    status = torch.full((1,), -1, dtype=torch.int32, device=x.device)
    lib.call("eesd_head_argmax_static", x.data_ptr(), x.shape[0], lib.ptr(rows), n, cfg.dim, cfg.vocab_size,
             dm.w.t["norm"].data_ptr(), dm.w.t["lm_head"].data_ptr(), cfg.norm_eps, ids.data_ptr(),
             status.data_ptr(), lib.stream_ptr())
    return ids, status


def _model(name: str) -> DeviceModel:
    if name == "c1s":
        cfg = preset("c1s")
        w = ModelWeights.from_numpy(cfg, synthetic_weights(cfg, seed=2, norm_jitter=0.1), torch.bfloat16, "cuda")
    else:   # the Llama3-8B head shapes (dim 4096, vocab 128256) on a one-layer model
        cfg = replace(preset("llama3-8b"), n_layers=1)
        w = ModelWeights.synthetic(cfg, seed=3, dtype=torch.bfloat16, device="cuda")
    return DeviceModel(w, max_batch=1, max_seq=64, max_tokens=256)


@pytest.mark.parametrize("name,n", [("c1s", 37), ("llama3-8b", 128)])
def test_static_head_matches_model_head_on_two_calls(cuda_dev, name, n):
    dm = _model(name)
    g = torch.Generator(device=cuda_dev).manual_seed(n)
    for call in range(2):
        x = torch.randn(2 * n, dm.cfg.dim, device=cuda_dev, generator=g).bfloat16()
        rows = torch.randperm(2 * n, device=cuda_dev, generator=g)[:n].to(torch.int32)
        want = dm.head_argmax(x, rows)
        got, st = _static_head(dm, x, rows, n)
        got_dense, st_dense = _static_head(dm, x[:n].contiguous(), None, n)
        want_dense = dm.head_argmax(x[:n].contiguous())
        torch.cuda.synchronize()
        assert int(st) == 0 and int(st_dense) == 0
        assert torch.equal(got, want), (call, (got != want).sum().item())
        assert torch.equal(got_dense, want_dense), call
        assert int(got.min()) >= 0 and int(got.max()) < dm.cfg.vocab_size
    dm.check()


def test_static_head_is_the_argmax_of_fp32_logits(cuda_dev):
    """Against plain PyTorch at the Llama3-8B head shape: RMSNorm as the reference computes it
    (common/model.py:153-156, bf16 roundings), then fp32 logits.  The kernel takes the argmax of the
    logits rounded to bf16 (lowest id among equal rounded values), so where it picks another id,
    that id's fp32 logit must lie within one bf16 step (ulp) of the row's maximum."""
    import math

    dm = _model("llama3-8b")
    cfg, n = dm.cfg, 128
    g = torch.Generator(device=cuda_dev).manual_seed(5)
    x = torch.randn(n, cfg.dim, device=cuda_dev, generator=g).bfloat16()
    ids, st = _static_head(dm, x, None, n)
    xf = x.float()
    xn = dm.w.t["norm"] * (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + cfg.norm_eps)).bfloat16()
    logits = xn.float() @ dm.w.t["lm_head"].float().T
    want = logits.argmax(-1)
    torch.cuda.synchronize()
    assert int(st) == 0
    got = ids.long()
    diff = (got != want).nonzero().flatten().tolist()
    assert len(diff) <= n // 16, diff
    for r in diff:
        step = 2.0 ** (math.floor(math.log2(logits[r].abs().max().item())) - 7)   # bf16 ulp at the max
        assert logits[r, want[r]].item() - logits[r, got[r]].item() <= step, r


def test_static_head_allocates_nothing(cuda_dev):
    dm = _model("c1s")
    x = torch.randn(64, dm.cfg.dim, device=cuda_dev).bfloat16()
    _static_head(dm, x, None, 64)            # first call: module load, symbol address
    ids = torch.empty(64, dtype=torch.int32, device=cuda_dev)
    status = torch.empty(1, dtype=torch.int32, device=cuda_dev)
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        lib.call("eesd_head_argmax_static", x.data_ptr(), 64, None, 64, dm.cfg.dim, dm.cfg.vocab_size,
                 dm.w.t["norm"].data_ptr(), dm.w.t["lm_head"].data_ptr(), dm.cfg.norm_eps, ids.data_ptr(),
                 status.data_ptr(), lib.stream_ptr())
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0 and int(status) == 0


def test_static_head_reports_a_bad_row_and_a_timeout(cuda_dev):
    dm = _model("c1s")
    x = torch.randn(40, dm.cfg.dim, device=cuda_dev).bfloat16()
    want = dm.head_argmax(x[:8].contiguous())
    # a row index outside x: every id -1 and the bad-index bit
    rows = torch.tensor([0, 1, 40, 3], dtype=torch.int32, device=cuda_dev)
    ids, st = _static_head(dm, x, rows, 4)
    assert ids.tolist() == [-1] * 4 and int(st) & BAD_INDEX
    # every pipeline wait gives up at once: the call returns, copies in flight drain, bits are set
    lib.call("eesd_set_option", lib.OPT_SPIN_LIMIT, 0)
    try:
        ids, st = _static_head(dm, x, None, 8)
        torch.cuda.synchronize()
    finally:
        lib.call("eesd_set_option", lib.OPT_SPIN_LIMIT, -1)
    assert ids.tolist() == [-1] * 8 and int(st) & TIMEOUT_BITS, int(st)
    # the context is still usable and the array's stale contents do not leak into the next call
    ids, st = _static_head(dm, x[:8].contiguous(), None, 8)
    torch.cuda.synchronize()
    assert int(st) == 0 and torch.equal(ids, want)


def test_static_head_rejects_sizes_beyond_its_scratch(cuda_dev):
    L = lib.load()
    x = torch.zeros(129, 64, dtype=torch.bfloat16, device=cuda_dev)
    w = torch.ones(64, dtype=torch.bfloat16, device=cuda_dev)
    head = torch.zeros(32, 64, dtype=torch.bfloat16, device=cuda_dev)
    ids = torch.empty(129, dtype=torch.int32, device=cuda_dev)
    rc = L.eesd_head_argmax_static(x.data_ptr(), 129, None, 129, 64, 32, w.data_ptr(), head.data_ptr(), 1e-5,
                                   ids.data_ptr(), None, lib.stream_ptr())
    assert rc == lib.ERR_ARG and b"128" in L.eesd_last_error()
    rc = L.eesd_head_argmax_static(x.data_ptr(), 129, None, 4, 8256, 32, w.data_ptr(), head.data_ptr(), 1e-5,
                                   ids.data_ptr(), None, lib.stream_ptr())
    assert rc == lib.ERR_ARG and b"8192" in L.eesd_last_error()
    rc = L.eesd_head_argmax_static(x.data_ptr(), 2, None, 4, 64, 32, w.data_ptr(), head.data_ptr(), 1e-5,
                                   ids.data_ptr(), None, lib.stream_ptr())
    assert rc == lib.ERR_ARG
