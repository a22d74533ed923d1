"""B200 decoding engines over the sm_100a runtime: autoregressive and LayerSkip draft/verify.

Both engines implement the ``DecodeEngine`` contract (``thesis_b200/engine.py``) and run every
step as packed ragged calls of ``DeviceModel``:

* ``B200ARBatchEngine``  one token per request per step through all layers + head
                         (common/engine.py:302-331; solutions/engine.py:244-267).  This is the
                         in-engine lossless reference.
* ``B200SpecEngine``     synchronous self-speculation with a fixed exit layer E and draft length
                         gamma (common/engine.py:336-436, the EESD ``fixed`` schedule of
                         solutions/schedulers.py:77-89): gamma shallow steps draft one token each
                         through layers [0, E) + the shared head; the verify step runs the last
                         draft through [0, E), then all gamma+1 tokens of every request - inputs
                         are the cached exit-layer hidden states - through [E, L) + head, and the
                         acceptance kernel emits accepted lengths and corrected tokens in one pass.

Device state per engine: the token buffer ``seq_buf [B, gamma+1]`` (column 0 = last committed
token, columns 1.. = drafts, solutions/engine.py:17-19), the exit hidden states
``exit_h [B, gamma+1, dim]`` and the KV cache.  Rollback after a rejected draft moves nothing:
the host advances a request's position by accepted+1 and stale KV beyond it is never read
(solutions/engine.py:12-14).  The host reads the device once per verify step (accepted counts and
verified tokens) and never during draft steps.

Every kernel is batch-invariant (a token's result does not depend on which other tokens share a
launch), so speculative output is bit-identical to this engine's autoregressive output in bf16 as
well as fp32.
"""

from __future__ import annotations

from typing import Optional

import numpy as np
import torch

from . import lib
from .engine import DecodeEngine, Interval, StepRecord
from .model import DeviceModel, ModelWeights


def as_weights(model) -> ModelWeights:
    """Accept our ``ModelWeights``, a ``DeviceModel``, or the reference's ``LayerSkipLlama``."""
    if isinstance(model, ModelWeights):
        return model
    if isinstance(model, DeviceModel):
        return model.w
    if hasattr(model, "layers") and hasattr(model, "embed_w"):
        return ModelWeights.from_layerskip(model)
    raise TypeError(f"cannot build a B200 engine from {type(model).__name__}")


class _B200Engine(DecodeEngine):
    cols = 1
    pos_dev = None                 # device positions, for engines that run overlapped steps

    def __init__(self, model, batch_size, max_prompt_len, max_new_tokens, eos_ids, *, step_tokens: int = 1,
                 prefill_budget: int = 2048, prefill_chunk: int = 512, extra_tokens: int = 0, **kw):
        super().__init__(model, batch_size, max_prompt_len, max_new_tokens, eos_ids, **kw)
        self.weights = as_weights(model)
        self.prefill_chunk = prefill_chunk
        max_tokens = max(self.B * step_tokens + extra_tokens, min(prefill_budget, max(prefill_chunk, 1) * self.B))
        self.dm = DeviceModel(self.weights, self.B, self.max_seq, max_tokens)
        self.device = self.dm.device
        self.cfg = self.weights.cfg
        self.seq_buf = torch.zeros(self.B, self.cols, dtype=torch.int32, device=self.device)
        self.h2d_bytes = 0
        self.d2h_bytes = 0

    def max_seq_alloc(self) -> int:
        return self.dm.max_seq

    # ---------------------------------------------------------------- step-level API
    def start(self, prompts) -> None:
        """Put ``prompts`` (at most B) into slots 0.. with one batched prefill (EESDEngine.assign,
        solutions/engine.py:180-204, for a whole batch)."""
        if len(prompts) > self.B:
            raise ValueError(f"{len(prompts)} prompts for {self.B} slots")
        self._assign_many([(i, i, p) for i, p in enumerate(prompts)])

    def step(self, measured: bool = True) -> int:
        """One scheduling iteration over the occupied slots; returns committed tokens
        (EESDEngine.step, solutions/engine.py:237-242)."""
        return self._iteration(measured)

    def _prefill_slots(self, prompts: dict) -> dict:
        first = self.dm.prefill(prompts, chunk=self.prefill_chunk)
        slots = sorted(first)
        ids = np.array([first[s] for s in slots], dtype=np.int32)
        idx = np.array([s * self.cols for s in slots], dtype=np.int32)
        lens = np.array([len(prompts[s]) for s in slots], dtype=np.int32)
        ph = self.dm.pack([(0, 0, 1)])          # metadata slot carrying the index arrays
        _, (ids_d, idx_d, len_d, row_d) = self.dm.upload(ph, (ids, idx, lens, np.array(slots, dtype=np.int32)))
        sp = lib.stream_ptr()
        lib.call("eesd_scatter_ids", ids_d.data_ptr(), idx_d.data_ptr(), self.seq_buf.data_ptr(), len(slots), sp)
        if self.pos_dev is not None:
            # device-resident positions of the overlapped steps (the prompt length is the first decode position)
            lib.call("eesd_scatter_ids", len_d.data_ptr(), row_d.data_ptr(), self.pos_dev.data_ptr(), len(slots), sp)
        return first

    # ---------------------------------------------------------------- overlapped steps
    # Step k+1 is enqueued before step k is read back: positions live on the device
    # (eesd_round_meta builds the packed metadata from them, eesd_round_advance moves them), the
    # host keeps two pinned read-back buffers and commits a step one iteration later.  A request
    # that finished in step k runs one more (discarded) step, inside the engine's spec slack; a
    # slot reassigned meanwhile is recognised by its assignment count.
    def _init_overlap(self, overlap: bool, gamma: int) -> None:
        self.overlap = bool(overlap)
        self.pos_dev = torch.zeros(self.B, dtype=torch.int32, device=self.device)
        self.meta_ints = int(lib.load().eesd_round_meta_ints(self.B, gamma, self.dm.item_tokens))
        self.meta_dev = torch.empty(self.meta_ints, dtype=torch.int32, device=self.device)
        self.gen = [0] * self.B            # assignment count per slot: stale in-flight results are dropped
        self.inflight: list = []
        self.round_seq = 0

    def _on_assigned(self, slot: int) -> None:
        self.gen[slot] += 1

    def _overlapped(self, measured: bool) -> int:
        """Enqueue this step, then commit the previous one."""
        act = [s for s in self._active() if self.slots[s].finish_reason is None]
        if act:
            self.inflight.append(self._enqueue_round(act, measured))
        committed = 0
        while len(self.inflight) > (1 if act else 0):
            committed += self._commit_round(self.inflight.pop(0))
        return committed

    def _live(self, r: dict) -> list:
        return [self.gen[s] == gn and not self.slots[s].idle and self.slots[s].finish_reason is None
                for s, gn in zip(r["act"], r["gens"])]

    def free(self) -> None:
        if hasattr(self, "inflight"):
            self.inflight.clear()
        self.dm.close()


class B200ARBatchEngine(_B200Engine):
    name = "b200_autoregressive"

    def __init__(self, model, batch_size, max_prompt_len, max_new_tokens, eos_ids, *, overlap: bool = True, **kw):
        kw.setdefault("spec_slack", 32)
        super().__init__(model, batch_size, max_prompt_len, max_new_tokens, eos_ids, **kw)
        self._init_overlap(overlap, 0)
        self.zeros_dev = torch.zeros(self.B, dtype=torch.int32, device=self.device)
        self.y_dev = torch.empty(self.B, dtype=torch.int32, device=self.device)
        self.y_hosts = [torch.empty(self.B, dtype=torch.int32).pin_memory() for _ in range(2)]

    @torch.inference_mode()
    def _iteration(self, measured: bool) -> int:
        return self._overlapped(measured) if self.overlap else self._iteration_sync(measured)

    def _enqueue_round(self, act: list, measured: bool) -> dict:
        """One token per request through all layers + head; the token is the next step's input."""
        dm, n = self.dm, len(act)
        sp = lib.stream_ptr()
        _, (act_d,) = dm.upload(dm.pack([(0, 0, 1)]), (np.array(act, dtype=np.int32),))
        self.h2d_bytes += 4 * (n + 7)
        base = self.meta_dev.data_ptr()
        iv = Interval(self.device).start()
        lib.call("eesd_round_meta", act_d.data_ptr(), n, self.pos_dev.data_ptr(), self.B, 0, dm.item_tokens, base, sp)
        max_ctx = min(max(self.slots[s].pos for s in act) + 2, dm.max_seq)
        b = lib.Batch(n, n, n, max_ctx, base, base + 4 * n, base + 8 * n, base + 24 * n)
        src = base + 32 * n
        ids = torch.empty(n, dtype=torch.int32, device=self.device)
        lib.call("eesd_gather_ids", self.seq_buf.data_ptr(), src, ids.data_ptr(), n, sp)
        x = dm.embed(ids)
        dm.forward_layers(x, b, 0, self.cfg.n_layers)
        y = self.y_dev[:n]
        dm.head_argmax(x, out=y)
        lib.call("eesd_scatter_ids", y.data_ptr(), src, self.seq_buf.data_ptr(), n, sp)
        lib.call("eesd_round_advance", act_d.data_ptr(), n, self.zeros_dev.data_ptr(), self.pos_dev.data_ptr(), self.B,
                 sp)
        iv.stop()
        host = self.y_hosts[self.round_seq % 2]
        self.round_seq += 1
        host[:n].copy_(y, non_blocking=True)
        done = torch.cuda.Event()
        done.record()
        self.d2h_bytes += 4 * n
        kv = int(sum(self.slots[s].pos for s in act)) + n
        return {"act": act, "gens": [self.gen[s] for s in act], "host": host, "event": done, "iv": iv,
                "measured": measured, "n": n, "kv": kv}

    def _commit_round(self, r: dict) -> int:
        r["event"].synchronize()
        live = self._live(r)
        if not any(live):
            return 0
        n = r["n"]
        self.records.append(StepRecord("ar", r["iv"].ms, n, n, n, r["kv"], r["measured"]))
        y_h = r["host"][:n].tolist()
        committed = 0
        for v, (s, t) in enumerate(zip(r["act"], y_h)):
            if not live[v]:
                continue
            st = self.slots[s]
            st.pos += 1
            st.last_token = t
            committed += self._commit(s, [t])
        return committed

    def _iteration_sync(self, measured: bool) -> int:
        dm = self.dm
        act = self._active()
        n = len(act)
        ph = dm.pack([(s, self.slots[s].pos, 1) for s in act])
        idx = np.array(act, dtype=np.int32) * self.cols
        iv = Interval(self.device).start()
        b, (idx_d,) = dm.upload(ph, (idx,))
        ids = torch.empty(n, dtype=torch.int32, device=self.device)
        lib.call("eesd_gather_ids", self.seq_buf.data_ptr(), idx_d.data_ptr(), ids.data_ptr(), n, lib.stream_ptr())
        x = dm.embed(ids)
        dm.forward_layers(x, b, 0, self.cfg.n_layers)
        y = dm.head_argmax(x)
        lib.call("eesd_scatter_ids", y.data_ptr(), idx_d.data_ptr(), self.seq_buf.data_ptr(), n, lib.stream_ptr())
        iv.stop()
        y_h = y.cpu().tolist()
        self.h2d_bytes += 4 * (2 * n + 4 * ph.n_blocks + 2 * len(ph.items) + n)
        self.d2h_bytes += 4 * n
        self.records.append(StepRecord("ar", iv.ms, n, n, n, ph.kv_read, measured))
        committed = 0
        for s, t in zip(act, y_h):
            st = self.slots[s]
            st.pos += 1
            st.last_token = t
            committed += self._commit(s, [t])
        return committed


class B200SpecEngine(_B200Engine):
    """Synchronous batched LayerSkip self-speculation on the packed B200 path."""

    name = "b200_layerskip"

    def __init__(self, model, batch_size, max_prompt_len, max_new_tokens, eos_ids, *, exit_layer: int, gamma: int,
                 overlap: bool = True, **kw):
        w = as_weights(model)
        if not 1 <= exit_layer < w.cfg.n_layers:
            raise ValueError(f"exit_layer must be in [1, {w.cfg.n_layers - 1}]")
        if gamma < 0:
            raise ValueError("gamma must be >= 0")
        self.k, self.gamma = int(exit_layer), int(gamma)
        self.cols = self.gamma + 1
        kw.setdefault("spec_slack", gamma + 32)
        super().__init__(w, batch_size, max_prompt_len, max_new_tokens, eos_ids, step_tokens=self.cols, **kw)
        self.exit_h = torch.zeros(self.B * self.cols, self.cfg.dim, dtype=self.weights.dtype, device=self.device)
        self.xbuf = torch.empty(self.B * self.cols, self.cfg.dim, dtype=self.weights.dtype, device=self.device)
        self.out = torch.empty(self.B + self.B * self.cols, dtype=torch.int32, device=self.device)
        self.out_host = torch.empty_like(self.out, device="cpu").pin_memory()
        self.stats = {"rounds": 0, "request_rounds": 0, "drafted": 0, "accepted": 0, "rejected": 0,
                      "overdraft_steps": 0, "full_accept_rounds": 0}
        self.accept_hist = np.zeros(self.gamma + 1, dtype=np.int64)
        # overlapped rounds: round r+1 is enqueued before round r's acceptance is read back; its
        # metadata and positions are built on the device (eesd_round_meta / eesd_round_advance)
        self._init_overlap(overlap and type(self)._iteration is B200SpecEngine._iteration, self.gamma)
        self.out_hosts = [self.out_host, torch.empty_like(self.out_host).pin_memory()]

    # ---------------------------------------------------------------- one round
    def _shallow(self, act: list, pos: np.ndarray, j: int, draft: bool):
        """Token j of every active request through [0, E): exit_h[s, j] = h; drafts into seq_buf[s, j+1]."""
        dm = self.dm
        n = len(act)
        ph = dm.pack([(s, int(p) + j, 1) for s, p in zip(act, pos)])
        src = np.array(act, dtype=np.int32) * self.cols + j
        b, (src_d, dst_d) = dm.upload(ph, (src, src + 1))
        ids = torch.empty(n, dtype=torch.int32, device=self.device)
        sp = lib.stream_ptr()
        lib.call("eesd_gather_ids", self.seq_buf.data_ptr(), src_d.data_ptr(), ids.data_ptr(), n, sp)
        x = dm.embed(ids, out=self.xbuf[:n])
        dm.forward_layers(x, b, 0, self.k)
        lib.call("eesd_copy_rows", lib.BF16 if self.weights.dtype == torch.bfloat16 else lib.F32, x.data_ptr(), None,
                 self.exit_h.data_ptr(), src_d.data_ptr(), n, self.cfg.dim, sp)
        if draft:
            d = dm.head_argmax(x)
            lib.call("eesd_scatter_ids", d.data_ptr(), dst_d.data_ptr(), self.seq_buf.data_ptr(), n, sp)
        self.h2d_bytes += 4 * (2 * n + 4 * n + 2 * len(ph.items) + 2 * n)
        return ph

    @torch.inference_mode()
    def _iteration(self, measured: bool) -> int:
        return self._overlapped(measured) if self.overlap else self._iteration_sync(measured)

    def _iteration_sync(self, measured: bool) -> int:
        dm, g, cols = self.dm, self.gamma, self.cols
        act = self._active()
        n = len(act)
        pos = np.array([self.slots[s].pos for s in act], dtype=np.int64)
        recs = []
        for j in range(g):
            iv = Interval(self.device).start()
            ph = self._shallow(act, pos, j, draft=True)
            iv.stop()
            recs.append(("draft", iv, n, n, 0, ph.kv_read))
        # ---- verify: the last draft through [0, E), then gamma+1 tokens per request through [E, L)
        iv = Interval(self.device).start()
        self._shallow(act, pos, g, draft=False)
        ph = dm.pack([(s, int(p), cols) for s, p in zip(act, pos)])
        rows = (np.array(act, dtype=np.int32)[:, None] * cols + np.arange(cols, dtype=np.int32)[None, :]).reshape(-1)
        vinfo = np.stack([np.arange(n, dtype=np.int32) * cols, np.full(n, cols, dtype=np.int32),
                          np.array(act, dtype=np.int32)], axis=1)
        b, (rows_d, vinfo_d) = dm.upload(ph, (rows, vinfo))
        sp = lib.stream_ptr()
        N = n * cols
        x = self.xbuf[:N]
        lib.call("eesd_copy_rows", lib.BF16 if self.weights.dtype == torch.bfloat16 else lib.F32,
                 self.exit_h.data_ptr(), rows_d.data_ptr(), x.data_ptr(), None, N, self.cfg.dim, sp)
        dm.forward_layers(x, b, self.k, self.cfg.n_layers)
        acc = self.out[:n]
        y = self.out[n:n + N]
        dm.head_argmax(x, out=y)
        lib.call("eesd_greedy_accept", y.data_ptr(), vinfo_d.data_ptr(), n, self.seq_buf.data_ptr(), cols,
                 acc.data_ptr(), sp)
        iv.stop()
        host = self.out_host[:n + N]
        host.copy_(self.out[:n + N], non_blocking=True)
        torch.cuda.current_stream().synchronize()           # the one device->host read per round
        self.h2d_bytes += 4 * (2 * N + 4 * n + 2 * len(ph.items) + N + 3 * n)
        self.d2h_bytes += 4 * (n + N)
        recs.append(("verify", iv, n, n, N, ph.kv_read))
        for kind, t, bb, st, dt, kv in recs:
            self.records.append(StepRecord(kind, t.ms, bb, st, dt, kv, measured))
        out = host.numpy()
        acc_h, y_h = out[:n], out[n:n + N].reshape(n, cols)
        committed = 0
        self.stats["rounds"] += 1
        for v, s in enumerate(act):
            a = int(acc_h[v])
            st = self.slots[s]
            st.pos = int(pos[v]) + a + 1
            st.last_token = int(y_h[v, a])
            committed += self._commit(s, y_h[v, :a + 1].tolist())
            if measured and st.finish_reason is None:
                S = self.stats
                S["request_rounds"] += 1
                S["drafted"] += g
                S["accepted"] += a
                S["rejected"] += g - a
                S["overdraft_steps"] += max(g - a - 1, 0)
                S["full_accept_rounds"] += int(a == g)
                self.accept_hist[a] += 1
        return committed

    # ---------------------------------------------------------------- overlapped rounds
    def _enqueue_round(self, act: list, measured: bool) -> dict:
        dm, g, cols, L = self.dm, self.gamma, self.cols, self.cfg.n_layers
        n, it = len(act), dm.item_tokens
        ni = -(-cols // it)
        sp = lib.stream_ptr()
        act_np = np.array(act, dtype=np.int32)
        _, (act_d,) = dm.upload(dm.pack([(0, 0, 1)]), (act_np,))
        self.h2d_bytes += 4 * (n + 7)
        base = self.meta_dev.data_ptr()
        lib.call("eesd_round_meta", act_d.data_ptr(), n, self.pos_dev.data_ptr(), self.B, g, it, base, sp)
        # host bound on this round's keys: positions lag at most one round (cols) behind the device
        max_ctx = min(max(self.slots[s].pos for s in act) + 2 * cols, dm.max_seq)
        dt = lib.BF16 if self.weights.dtype == torch.bfloat16 else lib.F32
        ivs = []
        for j in range(cols):
            o = base + 4 * j * 10 * n
            b = lib.Batch(n, n, n, max_ctx, o, o + 4 * n, o + 8 * n, o + 24 * n)
            src, dst = o + 32 * n, o + 36 * n
            iv = Interval(self.device).start() if j < g else None
            if j == g:
                iv_v = Interval(self.device).start()
            ids = torch.empty(n, dtype=torch.int32, device=self.device)
            lib.call("eesd_gather_ids", self.seq_buf.data_ptr(), src, ids.data_ptr(), n, sp)
            x = dm.embed(ids, out=self.xbuf[:n])
            dm.forward_layers(x, b, 0, self.k)
            lib.call("eesd_copy_rows", dt, x.data_ptr(), None, self.exit_h.data_ptr(), src, n, self.cfg.dim, sp)
            if j < g:
                d = dm.head_argmax(x)
                lib.call("eesd_scatter_ids", d.data_ptr(), dst, self.seq_buf.data_ptr(), n, sp)
                iv.stop()
                ivs.append(("draft", iv, n, n, 0))
        # verify: gamma + 1 tokens per request from their exit-layer states through [E, L)
        N = n * cols
        v = base + 4 * cols * 10 * n
        vblk = v + 4 * 2 * N
        vitems = vblk + 4 * 4 * n
        vrows = vitems + 4 * 2 * n * ni
        vinfo = vrows + 4 * N
        b = lib.Batch(N, n, n * ni, max_ctx, v, v + 4 * N, vblk, vitems)
        x = self.xbuf[:N]
        lib.call("eesd_copy_rows", dt, self.exit_h.data_ptr(), vrows, x.data_ptr(), None, N, self.cfg.dim, sp)
        dm.forward_layers(x, b, self.k, L)
        acc = self.out[:n]
        y = self.out[n:n + N]
        dm.head_argmax(x, out=y)
        lib.call("eesd_greedy_accept", y.data_ptr(), vinfo, n, self.seq_buf.data_ptr(), cols, acc.data_ptr(), sp)
        lib.call("eesd_round_advance", act_d.data_ptr(), n, acc.data_ptr(), self.pos_dev.data_ptr(), self.B, sp)
        iv_v.stop()
        ivs.append(("verify", iv_v, n, n, N))
        host = self.out_hosts[self.round_seq % 2]     # two pinned buffers: one round read, one in flight
        self.round_seq += 1
        host[:n + N].copy_(self.out[:n + N], non_blocking=True)
        done = torch.cuda.Event()
        done.record()
        self.d2h_bytes += 4 * (n + N)
        kv = int(sum(self.slots[s].pos for s in act)) + n * cols
        return {"act": act, "gens": [self.gen[s] for s in act], "host": host, "event": done, "ivs": ivs,
                "measured": measured, "n": n, "N": N, "kv": kv}

    def _commit_round(self, r: dict) -> int:
        r["event"].synchronize()          # this round's read-back (the next round is already queued)
        g, cols, n, N = self.gamma, self.cols, r["n"], r["N"]
        out = r["host"].numpy()
        acc_h, y_h = out[:n], out[n:n + N].reshape(n, cols)
        live = self._live(r)
        if not any(live):
            return 0                          # every request of this round had finished before it was read
        self.stats["rounds"] += 1
        for kind, iv, bb, st_, dt in r["ivs"]:
            self.records.append(StepRecord(kind, iv.ms, bb, st_, dt, r["kv"], r["measured"]))
        committed = 0
        for v, s in enumerate(r["act"]):
            st = self.slots[s]
            if not live[v]:
                continue                      # finished (or reassigned) before this round was read
            a = int(acc_h[v])
            st.pos = st.pos + a + 1
            st.last_token = int(y_h[v, a])
            committed += self._commit(s, y_h[v, :a + 1].tolist())
            if r["measured"] and st.finish_reason is None:
                S = self.stats
                S["request_rounds"] += 1
                S["drafted"] += g
                S["accepted"] += a
                S["rejected"] += g - a
                S["overdraft_steps"] += max(g - a - 1, 0)
                S["full_accept_rounds"] += int(a == g)
                self.accept_hist[a] += 1
        return committed

    def extra_metrics(self) -> dict:
        st = dict(self.stats)
        rr = max(st["request_rounds"], 1)
        st.update(exit_layer=self.k, gamma=self.gamma,
                  acceptance_rate=st["accepted"] / max(st["drafted"], 1),
                  rejected_draft_ratio=st["rejected"] / max(st["drafted"], 1),
                  overdraft_step_ratio=st["overdraft_steps"] / max(st["drafted"], 1),
                  full_accept_round_ratio=st["full_accept_rounds"] / rr,
                  tokens_per_verify=(st["accepted"] + st["request_rounds"]) / rr,
                  accept_hist=self.accept_hist.tolist())
        return {"spec": st}
