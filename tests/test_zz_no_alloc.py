"""The allocation-free exit head, checked against the model-handle exit head through the C ABI.

``eesd_head_argmax_static`` exists for callers that cannot allocate device memory: a serving
runtime whose allocator is locked on its decode path, code running inside a foreign stream
capture, or a plug-in that is only handed raw input and output pointers.  Its scratch is a fixed
array inside the library instead of a caller workspace.  It must return exactly the token ids
that ``eesd_head_argmax`` returns for the same rows (integer outputs: exact equality), on two
calls in a row, since the shared array keeps the previous call's contents.

This file is collected last so that a run stopping at the first failure has run every other test.
"""

import ctypes as C
from dataclasses import replace

import pytest
import torch

from thesis_b200 import lib
from thesis_b200.config import preset
from thesis_b200.model import DeviceModel, ModelWeights
from thesis_b200.synthetic import synthetic_weights

pytestmark = pytest.mark.gpu


def _static_head(dm: DeviceModel, x: torch.Tensor, rows, n: int) -> torch.Tensor:
    cfg = dm.cfg
    ids = torch.full((n,), -1, dtype=torch.int32, device=x.device)
    lib.call("eesd_head_argmax_static", x.data_ptr(), lib.ptr(rows), n, cfg.dim, cfg.vocab_size,
             dm.w.t["norm"].data_ptr(), dm.w.t["lm_head"].data_ptr(), cfg.norm_eps, ids.data_ptr(), lib.stream_ptr())
    return ids


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
        got = _static_head(dm, x, rows, n)
        got_dense = _static_head(dm, x[:n].contiguous(), None, n)
        want_dense = dm.head_argmax(x[:n].contiguous())
        torch.cuda.synchronize()
        assert torch.equal(got, want), (call, (got != want).sum().item())
        assert torch.equal(got_dense, want_dense), call
        assert int(got.min()) >= 0 and int(got.max()) < dm.cfg.vocab_size
    dm.check()


def test_static_head_rejects_sizes_beyond_its_scratch(cuda_dev):
    L = lib.load()
    x = torch.zeros(129, 64, dtype=torch.bfloat16, device=cuda_dev)
    w = torch.ones(64, dtype=torch.bfloat16, device=cuda_dev)
    head = torch.zeros(32, 64, dtype=torch.bfloat16, device=cuda_dev)
    ids = torch.empty(129, dtype=torch.int32, device=cuda_dev)
    rc = L.eesd_head_argmax_static(x.data_ptr(), None, 129, 64, 32, w.data_ptr(), head.data_ptr(), 1e-5,
                                   ids.data_ptr(), lib.stream_ptr())
    assert rc == lib.ERR_ARG and b"128" in L.eesd_last_error()
    rc = L.eesd_head_argmax_static(x.data_ptr(), None, 4, 8256, 32, w.data_ptr(), head.data_ptr(), 1e-5,
                                   ids.data_ptr(), lib.stream_ptr())
    assert rc == lib.ERR_ARG and b"8192" in L.eesd_last_error()
