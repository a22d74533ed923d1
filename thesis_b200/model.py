"""LayerSkip-Llama on one B200: device weights, static KV cache and the native runtime.

``ModelWeights`` holds the weights in the reference layout (common/model.py:161-168, fused
``wqkv`` and ``w13``) on the device.  ``DeviceModel`` adds what one engine needs: the KV cache
``[n_layers, max_batch, n_kv_heads, max_seq, head_dim]`` (the reference keeps one
``[max_batch, n_kv_heads, max_seq, head_dim]`` tensor per layer, common/model.py:171-179), the
RoPE table, the runtime workspace, and the handle of the C-ABI runtime, whose calls implement
the reference's layer-range forward, exit head and embedding (common/model.py:325-389;
solutions/packed.py:169-196).  Every compute call goes to the sm_100a extension; there is no
other path.
"""

from __future__ import annotations

import ctypes as C
import json
import math
from pathlib import Path
from typing import Optional

import numpy as np
import torch

from . import lib
from .config import ModelConfig
from .packing import MetaUploader, PackedHost, pack

DTYPES = {torch.bfloat16: lib.BF16, torch.float32: lib.F32}


def round_up(x: int, m: int) -> int:
    return (x + m - 1) // m * m


def _llama3_inv_freq(inv_freq: torch.Tensor, s: dict) -> torch.Tensor:
    """llama3 RoPE frequency scaling (common/model.py:113-126, transformers' llama3 rule)."""
    factor, low, high = s["factor"], s["low_freq_factor"], s["high_freq_factor"]
    old = s["original_max_position_embeddings"]
    wavelen = 2 * math.pi / inv_freq
    out = torch.where(wavelen > old / low, inv_freq / factor, inv_freq)
    smooth = (old / wavelen - low) / (high - low)
    smoothed = (1 - smooth) * out / factor + smooth * out
    medium = ~(wavelen < old / high) & ~(wavelen > old / low)
    return torch.where(medium, smoothed, out)


def build_rope_cache(cfg: ModelConfig, max_seq: int) -> tuple[torch.Tensor, torch.Tensor]:
    """fp32 cos/sin tables [max_seq, head_dim] in the rotate-half layout, computed on the CPU with
    the same torch ops as the reference (common/model.py:129-140) so the tables are identical."""
    D = cfg.head_dim
    inv_freq = 1.0 / (cfg.rope_theta ** (torch.arange(0, D, 2, dtype=torch.int64).float() / D))
    sc = cfg.rope_scaling or {}
    kind = sc.get("rope_type", sc.get("type"))
    if kind == "llama3":
        inv_freq = _llama3_inv_freq(inv_freq, sc)
    elif kind not in (None, "default"):
        raise NotImplementedError(f"rope_scaling type {kind!r} is not supported")
    t = torch.arange(max_seq, dtype=torch.float32)
    freqs = torch.outer(t, inv_freq)
    emb = torch.cat([freqs, freqs], dim=-1)
    return emb.cos(), emb.sin()


class ModelWeights:
    """Device weights of a LayerSkip-Llama in the reference's fused layout."""

    def __init__(self, cfg: ModelConfig, tensors: dict, dtype: torch.dtype, device):
        if dtype not in DTYPES:
            raise ValueError(f"dtype {dtype} not supported (bf16 or fp32)")
        self.cfg, self.dtype, self.device = cfg, dtype, torch.device(device)
        self.t = {}
        for k, v in tensors.items():
            v = torch.as_tensor(v).to(device=self.device, dtype=dtype).contiguous()
            self.t[k] = v
        if cfg.tie_word_embeddings or "lm_head" not in self.t:
            self.t["lm_head"] = self.t["embed"]
        self._packed = {}
        for i in range(cfg.n_layers):
            for name in ("wqkv", "wo", "w13", "w2", "attn_norm", "ffn_norm"):
                if f"l{i}.{name}" not in self.t:
                    raise KeyError(f"missing weight l{i}.{name}")

    @property
    def n_layers(self) -> int:
        return self.cfg.n_layers

    def packs_gemm_weights(self) -> bool:
        """bf16 GEMM weights are streamed from a tile-packed copy (contiguous 16 KB tiles)."""
        return self.dtype == torch.bfloat16 and self.cfg.intermediate_size % 128 == 0

    def packed(self, key: str) -> torch.Tensor:
        """Tile-packed copy of a GEMM weight (``eesd_pack_weight``), built once and cached."""
        if key not in self._packed:
            w = self.t[key]
            rows, k = w.shape
            n = lib.load().eesd_packed_weight_bytes(rows, k)
            if n == 0:
                raise ValueError(f"{key}: cannot pack a [{rows}, {k}] weight (k must be a multiple of 64)")
            out = torch.empty(n // 2, dtype=torch.bfloat16, device=self.device)
            lib.call("eesd_pack_weight", w.data_ptr(), rows, k, out.data_ptr(), lib.stream_ptr())
            self._packed[key] = out
        return self._packed[key]

    def layer_bytes(self) -> int:
        return sum(self.t[f"l0.{n}"].numel() for n in ("wqkv", "wo", "w13", "w2", "attn_norm", "ffn_norm")) * \
            self.t["embed"].element_size()

    def head_bytes(self) -> int:
        return self.t["lm_head"].numel() * self.t["lm_head"].element_size()

    # ----------------------------------------------------------------- constructors
    @classmethod
    def from_numpy(cls, cfg: ModelConfig, W: dict, dtype=torch.bfloat16, device="cuda") -> "ModelWeights":
        return cls(cfg, {k: torch.from_numpy(v) for k, v in W.items()}, dtype, device)

    @classmethod
    def synthetic(cls, cfg: ModelConfig, seed: int = 0, dtype=torch.bfloat16, device="cuda",
                  residual_scale_from: Optional[int] = None, residual_scale: float = 1.0) -> "ModelWeights":
        from .synthetic import synthetic_weights_torch

        W = synthetic_weights_torch(cfg, seed, device, dtype, residual_scale_from=residual_scale_from,
                                    residual_scale=residual_scale)
        return cls(cfg, W, dtype, device)

    @classmethod
    def from_layerskip(cls, m) -> "ModelWeights":
        """Wrap the reference's ``LayerSkipLlama`` (common/model.py:218-278) without copying: its
        fused weights already have this layout."""
        rc = m.cfg
        cfg = ModelConfig(vocab_size=rc.vocab_size, dim=rc.dim, n_layers=rc.n_layers, n_heads=rc.n_heads,
                          n_kv_heads=rc.n_kv_heads, head_dim=rc.head_dim, intermediate_size=rc.intermediate_size,
                          norm_eps=rc.norm_eps, rope_theta=rc.rope_theta,
                          max_position_embeddings=rc.max_position_embeddings,
                          tie_word_embeddings=rc.tie_word_embeddings, rope_scaling=rc.rope_scaling,
                          bos_token_id=rc.bos_token_id, eos_token_ids=tuple(rc.eos_token_ids))
        T = {"embed": m.embed_w, "norm": m.norm_w, "lm_head": m.lm_head_w}
        for i, lw in enumerate(m.layers):
            T.update({f"l{i}.wqkv": lw.wqkv, f"l{i}.wo": lw.wo, f"l{i}.w13": lw.w13, f"l{i}.w2": lw.w2,
                      f"l{i}.attn_norm": lw.attn_norm, f"l{i}.ffn_norm": lw.ffn_norm})
        return cls(cfg, T, m.dtype, m.device)

    @classmethod
    def from_pretrained(cls, path, device="cuda", dtype=torch.bfloat16) -> "ModelWeights":
        """HF safetensors checkpoint -> fused layout (common/model.py:238-278)."""
        from safetensors import safe_open

        path = Path(path)
        cfg = ModelConfig.from_hf_dir(path)
        index = path / "model.safetensors.index.json"
        files = sorted(set(json.loads(index.read_text())["weight_map"].values())) if index.exists() else \
            ["model.safetensors"]
        raw = {}
        for f in files:
            with safe_open(str(path / f), framework="pt", device="cpu") as fh:
                for k in fh.keys():
                    raw[k] = fh.get_tensor(k)
        T = {"embed": raw.pop("model.embed_tokens.weight"), "norm": raw.pop("model.norm.weight")}
        if "lm_head.weight" in raw:
            T["lm_head"] = raw.pop("lm_head.weight")
        for i in range(cfg.n_layers):
            p = f"model.layers.{i}."
            T[f"l{i}.wqkv"] = torch.cat([raw.pop(p + "self_attn.q_proj.weight"), raw.pop(p + "self_attn.k_proj.weight"),
                                         raw.pop(p + "self_attn.v_proj.weight")])
            T[f"l{i}.w13"] = torch.cat([raw.pop(p + "mlp.gate_proj.weight"), raw.pop(p + "mlp.up_proj.weight")])
            T[f"l{i}.wo"] = raw.pop(p + "self_attn.o_proj.weight")
            T[f"l{i}.w2"] = raw.pop(p + "mlp.down_proj.weight")
            T[f"l{i}.attn_norm"] = raw.pop(p + "input_layernorm.weight")
            T[f"l{i}.ffn_norm"] = raw.pop(p + "post_attention_layernorm.weight")
        return cls(cfg, T, dtype, device)


class DeviceModel:
    """KV cache + runtime workspace + native handle for one engine on one GPU."""

    def __init__(self, weights: ModelWeights, max_batch: int, max_seq: int, max_tokens: int):
        if weights.device.type != "cuda":
            raise RuntimeError("DeviceModel needs CUDA weights: the compute path is the sm_100a extension only")
        L = lib.load()
        self.w, self.cfg, self.dtype, self.device = weights, weights.cfg, weights.dtype, weights.device
        cfg = self.cfg
        self.max_batch, self.max_tokens = int(max_batch), int(max_tokens)
        self.max_seq = round_up(int(max_seq), 64)                           # common/model.py:286
        self.item_tokens = L.eesd_attn_item_tokens(cfg.n_heads, cfg.n_kv_heads)
        if self.item_tokens <= 0:
            raise ValueError("n_heads must be a multiple of n_kv_heads")
        cos, sin = build_rope_cache(cfg, self.max_seq)
        self.rope_cos = cos.to(self.device).contiguous()
        self.rope_sin = sin.to(self.device).contiguous()
        shape = (cfg.n_layers, self.max_batch, cfg.n_kv_heads, self.max_seq, cfg.head_dim)
        self.k_cache = torch.zeros(shape, dtype=self.dtype, device=self.device)
        self.v_cache = torch.zeros(shape, dtype=self.dtype, device=self.device)
        t = weights.t
        packed = weights.packs_gemm_weights()
        self._ptr_arrays = {}

        def gemm_w(key):
            return (weights.packed(key) if packed else t[key]).data_ptr()

        def arr(name):
            ptrs = [gemm_w(f"l{i}.{name}") if name in ("wqkv", "wo", "w13", "w2") else t[f"l{i}.{name}"].data_ptr()
                    for i in range(cfg.n_layers)]
            a = (C.c_void_p * cfg.n_layers)(*ptrs)
            self._ptr_arrays[name] = a
            return C.cast(a, C.POINTER(C.c_void_p))

        d = lib.ModelDesc()
        d.dtype = DTYPES[self.dtype]
        d.n_layers, d.dim, d.n_heads, d.n_kv_heads = cfg.n_layers, cfg.dim, cfg.n_heads, cfg.n_kv_heads
        d.head_dim, d.intermediate, d.vocab = cfg.head_dim, cfg.intermediate_size, cfg.vocab_size
        d.norm_eps = cfg.norm_eps
        d.max_batch, d.max_seq, d.max_tokens = self.max_batch, self.max_seq, self.max_tokens
        d.weights_packed = int(packed)
        d.wqkv, d.wo, d.w13, d.w2 = arr("wqkv"), arr("wo"), arr("w13"), arr("w2")
        d.attn_norm, d.ffn_norm = arr("attn_norm"), arr("ffn_norm")
        d.final_norm, d.lm_head, d.embed = t["norm"].data_ptr(), gemm_w("lm_head"), t["embed"].data_ptr()
        d.rope_cos, d.rope_sin = self.rope_cos.data_ptr(), self.rope_sin.data_ptr()
        d.k_cache, d.v_cache = self.k_cache.data_ptr(), self.v_cache.data_ptr()
        ws = L.eesd_model_workspace_bytes(C.byref(d))
        self.workspace = torch.empty(ws + 256, dtype=torch.uint8, device=self.device)
        base = (self.workspace.data_ptr() + 255) // 256 * 256
        d.workspace, d.workspace_bytes = base, ws
        self.desc = d
        h = C.c_void_p()
        lib.check(L.eesd_model_create(C.byref(d), C.byref(h)), "eesd_model_create")
        self.handle = h
        max_blocks = self.max_tokens
        max_items = self.max_tokens + self.max_batch
        self.meta = MetaUploader(self.max_tokens, max_blocks, max_items, self.device,
                                 max_extra=4 * self.max_tokens + 4 * self.max_batch)
        self._ids = torch.empty(self.max_tokens, dtype=torch.int32, device=self.device)

    def close(self) -> None:
        if getattr(self, "handle", None) is not None and self.handle.value:
            lib.load().eesd_model_destroy(self.handle)
            self.handle = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ----------------------------------------------------------------- runtime calls
    def pack(self, blocks) -> PackedHost:
        return pack(blocks, self.item_tokens)

    def upload(self, ph: PackedHost, extra=()):
        """One pinned host-to-device copy of the packed metadata (+ extra int32 arrays)."""
        return self.meta.upload(ph, extra)

    def forward_layers(self, x: torch.Tensor, batch, start: int, end: int) -> torch.Tensor:
        """Layers [start, end) over packed hidden states x [N, dim] (in place)."""
        b = batch[0] if isinstance(batch, tuple) else batch
        if x.shape[0] != b.n_tokens or x.dtype != self.dtype or not x.is_contiguous():
            raise ValueError("x must be a contiguous [n_tokens, dim] tensor in the model dtype")
        lib.call("eesd_forward_layers", self.handle, x.data_ptr(), C.byref(b), start, end, lib.stream_ptr())
        return x

    def head_argmax(self, x: torch.Tensor, rows: Optional[torch.Tensor] = None, n: Optional[int] = None,
                    out: Optional[torch.Tensor] = None, logits: bool = False):
        """Final norm + LM head + argmax of rows ``rows`` (int32 device tensor) of x."""
        n = (rows.numel() if rows is not None else x.shape[0]) if n is None else n
        ids = out if out is not None else torch.empty(n, dtype=torch.int32, device=self.device)
        lg = torch.empty(n, self.cfg.vocab_size, dtype=self.dtype, device=self.device) if logits else None
        lib.call("eesd_head_argmax", self.handle, x.data_ptr(), lib.ptr(rows), n, ids.data_ptr(), lib.ptr(lg),
                 lib.stream_ptr())
        return (ids, lg) if logits else ids

    def embed(self, ids: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        n = ids.numel()
        x = out if out is not None else torch.empty(n, self.cfg.dim, dtype=self.dtype, device=self.device)
        lib.call("eesd_embed", self.handle, ids.data_ptr(), n, x.data_ptr(), lib.stream_ptr())
        return x

    def check(self) -> None:
        """Raise if a kernel recorded an error (bad index, bounded-wait timeout); synchronises."""
        bits = C.c_int(0)
        rc = lib.load().eesd_model_check(self.handle, C.byref(bits), lib.stream_ptr())
        lib.check(rc, f"device status (bits 0x{bits.value:x})")

    def launch_count(self) -> int:
        return int(lib.load().eesd_model_launch_count(self.handle))

    def profile(self, enable: bool) -> None:
        lib.call("eesd_model_profile", self.handle, int(enable))

    def profile_records(self, cap: int = 1 << 20):
        """[(kind name, packed tokens, ms)] of every launch recorded since profile(True)."""
        import numpy as np

        k = np.empty(cap, dtype=np.int32)
        n = np.empty(cap, dtype=np.int32)
        t = np.empty(cap, dtype=np.float32)
        cnt = lib.load().eesd_model_profile_records(self.handle, k.ctypes.data, n.ctypes.data, t.ctypes.data, cap)
        if cnt < 0:
            raise lib.EesdError("profile records")
        return [(lib.PROF_NAMES[k[i]], int(n[i]), float(t[i])) for i in range(cnt)]

    def profile_read(self) -> dict:
        ms = (C.c_double * lib.PROF_KINDS)()
        n = (C.c_int64 * lib.PROF_KINDS)()
        lib.call("eesd_model_profile_read", self.handle, ms, n)
        return {lib.PROF_NAMES[k]: (float(ms[k]), int(n[k])) for k in range(lib.PROF_KINDS)}

    # ----------------------------------------------------------------- convenience
    def prefill(self, prompts: dict, chunk: int = 512, budget: Optional[int] = None) -> dict:
        """Chunked causal prefill of several requests {row: tokens} through the packed path
        (solutions/engine.py:217-234 one request at a time; here chunk r of every request goes in
        the same call).  Returns {row: first generated token id} (argmax of the shared head on the
        last prompt position)."""
        budget = budget or self.max_tokens
        rows = list(prompts)
        done = {}
        last_h = []          # (rows, device ids): read back once, after every call is enqueued
        r = 0
        while True:
            chunks = [(row, r * chunk, min(chunk, len(prompts[row]) - r * chunk)) for row in rows
                      if len(prompts[row]) > r * chunk]
            if not chunks:
                break
            call, used = [], 0
            for c in chunks + [None]:
                if c is None or (call and used + c[2] > budget):
                    self._prefill_call(call, prompts, last_h)
                    call, used = [], 0
                if c is not None:
                    call.append(c)
                    used += c[2]
            r += 1
        for fin, y in last_h:
            for row, v in zip(fin, y.tolist()):
                done[row] = v
        return {row: done[row] for row in rows}

    def _prefill_call(self, call, prompts, last_h) -> None:
        if not call:
            return
        ph = self.pack(call)
        ids_h = np.array([t for (row, s, c) in call for t in prompts[row][s:s + c]], dtype=np.int32)
        b, (ids,) = self.upload(ph, (ids_h,))
        x = self.embed(ids)
        self.forward_layers(x, b, 0, self.cfg.n_layers)
        ends = [int(ph.offsets[i + 1]) - 1 for i, (row, s, c) in enumerate(call) if s + c == len(prompts[row])]
        if ends:
            rows_t = torch.tensor(ends, dtype=torch.int32).pin_memory().to(self.device, non_blocking=True)
            y = self.head_argmax(x, rows_t)
            last_h.append(([row for (row, s, c) in call if s + c == len(prompts[row])], y))
