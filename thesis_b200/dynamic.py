"""Per-request exit layer and per-request draft length, with coalesced ragged verification.

BASELINE config 4 (Llama2-7B shape: per-request exit in {4, 8, 12}, per-request draft length
drawn from 2..8 every round).  This goes beyond the reference, whose M2 controller switches ONE
batch-wide exit layer (solutions/exit_select.py:26-72, solutions/engine.py:522-527); the step
structure is the reference's synchronous draft/verify round (solutions/engine.py:269-489) with
two changes, both expressed as packed ragged calls of the same kernels:

* Draft step j runs every request whose draft length k_s is larger than j.  The requests are
  packed in DESCENDING exit-layer order, so the requests that still run at layer l (exit > l)
  are a prefix of the packed tokens: layers [0, e1) run on all of them, [e1, e2) on the prefix
  with exit >= e2, and so on.  A request's rows stop changing after its exit layer, so after the
  last segment the packed hidden states are every request's exit-layer state, and one head +
  argmax call drafts for all of them.
* The verify step runs the last draft through the shallow segments, then every request's k_s + 1
  tokens (ragged blocks) from the cached exit-layer states in ASCENDING exit order: layers
  [e1, e2) run on the prefix with exit e1, [e2, e3) on the prefix with exit <= e2, ..., [em, L)
  on all.  One head + argmax call and one acceptance launch cover every request, each with its
  own block length.

Exit layers are drawn per request (deterministic in the prompt index and ``policy_seed``), draft
lengths per request and round (a seeded generator).  Every kernel is batch-invariant, so the
output is bit-identical to the autoregressive engine's whatever the draws.

``schedule="unified"`` runs the reference's unified EESD step instead (solutions/engine.py:269-413
with the fixed rule V = requests whose drafts reached their own length): every step is one shallow
pass over all decoding requests - the drafting ones draft their next token, the ready ones run
their last draft - followed, when some request is ready, by one deep pass over the ready requests
only.  Requests verify out of phase, so a round no longer waits for the largest draw; instead most
steps carry a deep pass over a few requests.
"""

from __future__ import annotations

import numpy as np
import torch

from . import lib
from .eesd import _B200Engine, as_weights
from .engine import Interval, StepRecord


class B200DynamicSpecEngine(_B200Engine):
    """Synchronous self-speculation with a per-request exit layer and draft length."""

    name = "b200_layerskip_dynamic"

    def __init__(self, model, batch_size, max_prompt_len, max_new_tokens, eos_ids, *, exit_layers=(4, 8, 12),
                 gamma_range=(2, 8), policy_seed: int = 0, schedule: str = "lockstep", **kw):
        if schedule not in ("lockstep", "unified"):
            raise ValueError(f"schedule {schedule!r}: lockstep or unified")
        self.schedule = schedule
        w = as_weights(model)
        exits = sorted({int(e) for e in exit_layers})
        if not exits or exits[0] < 1 or exits[-1] >= w.cfg.n_layers:
            raise ValueError(f"exit layers must lie in [1, {w.cfg.n_layers - 1}]")
        g_lo, g_hi = int(gamma_range[0]), int(gamma_range[1])
        if not 0 <= g_lo <= g_hi:
            raise ValueError("gamma_range must be (lo, hi) with 0 <= lo <= hi")
        self.exits, self.g_lo, self.g_hi, self.policy_seed = exits, g_lo, g_hi, int(policy_seed)
        self.cols = g_hi + 1
        kw.setdefault("spec_slack", g_hi + 32)
        super().__init__(w, batch_size, max_prompt_len, max_new_tokens, eos_ids, step_tokens=self.cols, **kw)
        dt = self.weights.dtype
        self.exit_h = torch.zeros(self.B * self.cols, self.cfg.dim, dtype=dt, device=self.device)
        self.xbuf = torch.empty(self.B * self.cols, self.cfg.dim, dtype=dt, device=self.device)
        self.out = torch.empty(self.B + self.B * self.cols, dtype=torch.int32, device=self.device)
        self.out_host = torch.empty_like(self.out, device="cpu").pin_memory()
        self.exit_of = np.full(self.B, exits[-1], dtype=np.int64)
        self.rng = np.random.default_rng(self.policy_seed)
        self.dt_code = lib.BF16 if dt == torch.bfloat16 else lib.F32
        self.stats = {"rounds": 0, "request_rounds": 0, "drafted": 0, "accepted": 0, "rejected": 0,
                      "draft_steps": 0, "draft_rows": 0, "deep_tokens": 0}
        self.exit_hist = {e: 0 for e in exits}
        self.d = np.zeros(self.B, dtype=np.int64)       # unified: drafts of the current round so far
        self.k_target = np.zeros(self.B, dtype=np.int64)  # unified: this round's draft length

    # ---------------------------------------------------------------- policy
    def _on_assigned(self, slot: int) -> None:
        idx = self.slots[slot].prompt_idx
        g = np.random.default_rng([self.policy_seed, int(idx)])
        self.exit_of[slot] = self.exits[int(g.integers(len(self.exits)))]
        if self.schedule == "unified":
            self.d[slot] = 0
            self.k_target[slot] = int(self.draw_gammas(1)[0])

    def draw_gammas(self, n: int) -> np.ndarray:
        return self.rng.integers(self.g_lo, self.g_hi + 1, size=n)

    # ---------------------------------------------------------------- passes
    def _shallow(self, sel: list, jj: list, pos: dict, draft):
        """Token jj[i] of request sel[i] through [0, exit): exit_h[s, j] = h, and for the requests
        that draft (``draft``: True = all, or a set of slots) the head's argmax into
        seq_buf[s, j + 1].  Returns the KV positions read."""
        dm, cols = self.dm, self.cols
        order = sorted(range(len(sel)), key=lambda i: -int(self.exit_of[sel[i]]))
        sel = [sel[i] for i in order]
        jj = [int(jj[i]) for i in order]
        drafting = sel if draft is True else [s for s in sel if draft and s in draft]
        n = len(sel)
        ex = np.array([self.exit_of[s] for s in sel], dtype=np.int64)
        blocks = [(s, pos[s] + j, 1) for s, j in zip(sel, jj)]
        src = np.array([s * cols + j for s, j in zip(sel, jj)], dtype=np.int32)
        sp = lib.stream_ptr()
        prev, kv = 0, 0
        x = self.xbuf[:n]
        first = True
        for e in sorted(set(ex.tolist())):
            m = int((ex >= e).sum())                 # requests still running below layer e: a prefix
            ph = dm.pack(blocks[:m])
            if first:
                b, (src_d, dst_d) = dm.upload(ph, (src, src + 1))
                ids = torch.empty(n, dtype=torch.int32, device=self.device)
                lib.call("eesd_gather_ids", self.seq_buf.data_ptr(), src_d.data_ptr(), ids.data_ptr(), n, sp)
                dm.embed(ids, out=x)
                first = False
            else:
                b, _ = dm.upload(ph)
            dm.forward_layers(x[:m], b, prev, e)
            kv += ph.kv_read * (e - prev)
            self.h2d_bytes += 4 * (2 * m + 4 * m + 2 * len(ph.items))
            prev = e
        self.h2d_bytes += 4 * 2 * n
        lib.call("eesd_copy_rows", self.dt_code, x.data_ptr(), None, self.exit_h.data_ptr(), src_d.data_ptr(), n,
                 self.cfg.dim, sp)
        if len(drafting) == n:
            d = dm.head_argmax(x)
            lib.call("eesd_scatter_ids", d.data_ptr(), dst_d.data_ptr(), self.seq_buf.data_ptr(), n, sp)
        elif drafting:
            # the drafting requests' rows of x and their seq_buf cells, in one small upload
            who = set(drafting)
            rows = np.array([i for i, s in enumerate(sel) if s in who], dtype=np.int32)
            _, (rows_d, dsti_d) = dm.upload(dm.pack([(0, 0, 1)]), (rows, (src + 1)[rows]))
            self.h2d_bytes += 4 * (2 * len(rows) + 7)
            d = dm.head_argmax(x, rows_d)
            lib.call("eesd_scatter_ids", d.data_ptr(), dsti_d.data_ptr(), self.seq_buf.data_ptr(), len(rows), sp)
        return kv

    def _deep(self, act: list, K: dict, pos: dict):
        """Every request's K[s] + 1 tokens from their exit-layer states through [exit, L) + head,
        then greedy acceptance.  Returns (n, N, order, offsets, kv positions read)."""
        dm, cols, L = self.dm, self.cols, self.cfg.n_layers
        order = sorted(act, key=lambda s: int(self.exit_of[s]))
        n = len(order)
        ex = np.array([self.exit_of[s] for s in order], dtype=np.int64)
        T = np.array([K[s] + 1 for s in order], dtype=np.int64)
        offs = np.concatenate([[0], np.cumsum(T)]).astype(np.int64)
        N = int(offs[-1])
        blocks = [(s, pos[s], int(t)) for s, t in zip(order, T)]
        rows = np.concatenate([s * cols + np.arange(t, dtype=np.int32) for s, t in zip(order, T)]).astype(np.int32)
        vinfo = np.stack([offs[:-1].astype(np.int32), T.astype(np.int32), np.array(order, dtype=np.int32)], axis=1)
        sp = lib.stream_ptr()
        x = self.xbuf[:N]
        kv = 0
        uniq = sorted(set(ex.tolist()))
        for t, e in enumerate(uniq):
            e_next = uniq[t + 1] if t + 1 < len(uniq) else L
            m = int((ex <= e).sum())                 # requests whose deep part has started: a prefix
            ph = dm.pack(blocks[:m])
            if t == 0:
                b, (rows_d, vinfo_d) = dm.upload(ph, (rows, vinfo))
                lib.call("eesd_copy_rows", self.dt_code, self.exit_h.data_ptr(), rows_d.data_ptr(), x.data_ptr(),
                         None, N, self.cfg.dim, sp)
            else:
                b, _ = dm.upload(ph)
            dm.forward_layers(x[:int(offs[m])], b, e, e_next)
            kv += ph.kv_read * (e_next - e)
            self.h2d_bytes += 4 * (2 * int(offs[m]) + 4 * m + 2 * len(ph.items))
        self.h2d_bytes += 4 * (N + 3 * n)
        acc = self.out[:n]
        y = self.out[n:n + N]
        dm.head_argmax(x, out=y)
        lib.call("eesd_greedy_accept", y.data_ptr(), vinfo_d.data_ptr(), n, self.seq_buf.data_ptr(), cols,
                 acc.data_ptr(), sp)
        return n, N, order, offs, kv

    # ---------------------------------------------------------------- one round
    @torch.inference_mode()
    def _iteration(self, measured: bool) -> int:
        return self._unified_step(measured) if self.schedule == "unified" else self._lockstep_round(measured)

    def _unified_step(self, measured: bool) -> int:
        """One step of the unified schedule: the shallow pass of every decoding request, then the
        deep pass of the requests whose drafts reached this round's length (solutions/engine.py:269-413
        with V = {d >= k})."""
        act = self._active()
        pos = {s: int(self.slots[s].pos) for s in act}
        ready = [s for s in act if self.d[s] >= self.k_target[s]]
        drafting = {s for s in act if self.d[s] < self.k_target[s]}
        iv = Interval(self.device).start()
        kv = self._shallow(act, [int(self.d[s]) for s in act], pos, draft=drafting)
        if not ready:
            iv.stop()
            self.records.append(StepRecord("draft", iv.ms, len(act), len(act), 0, kv, measured))
            for s in drafting:
                self.d[s] += 1
            if measured:
                self.stats["draft_steps"] += 1
                self.stats["draft_rows"] += len(drafting)
            return 0
        K = {s: int(self.d[s]) for s in ready}
        n, N, order, offs, kv_deep = self._deep(ready, K, pos)
        iv.stop()
        host = self.out_host[:n + N]
        host.copy_(self.out[:n + N], non_blocking=True)
        torch.cuda.current_stream().synchronize()           # the deep step's one device->host read
        self.d2h_bytes += 4 * (n + N)
        self.records.append(StepRecord("verify", iv.ms, len(act), len(act), N, kv + kv_deep, measured))
        for s in drafting:
            self.d[s] += 1
        out = host.numpy()
        acc_h, y_h = out[:n], out[n:n + N]
        committed = 0
        self.stats["rounds"] += 1
        if measured and drafting:
            self.stats["draft_rows"] += len(drafting)
        for v, s in enumerate(order):
            a = int(acc_h[v])
            st = self.slots[s]
            st.pos = pos[s] + a + 1
            st.last_token = int(y_h[offs[v] + a])
            committed += self._commit(s, y_h[offs[v]:offs[v] + a + 1].tolist())
            if measured and st.finish_reason is None:
                S = self.stats
                S["request_rounds"] += 1
                S["drafted"] += K[s]
                S["accepted"] += a
                S["rejected"] += K[s] - a
                S["deep_tokens"] += K[s] + 1
                self.exit_hist[int(self.exit_of[s])] += 1
            self.d[s] = 0
            self.k_target[s] = int(self.draw_gammas(1)[0])
        return committed

    def _lockstep_round(self, measured: bool) -> int:
        act = self._active()
        pos = {s: int(self.slots[s].pos) for s in act}
        ks = self.draw_gammas(len(act))
        K = {s: int(k) for s, k in zip(act, ks)}
        recs = []
        for j in range(max(K.values(), default=0)):
            sel = [s for s in act if K[s] > j]
            iv = Interval(self.device).start()
            kv = self._shallow(sel, [j] * len(sel), pos, draft=True)
            iv.stop()
            recs.append(("draft", iv, len(sel), len(sel), 0, kv))
            if measured:
                self.stats["draft_steps"] += 1
                self.stats["draft_rows"] += len(sel)
        iv = Interval(self.device).start()
        kv = self._shallow(act, [K[s] for s in act], pos, draft=False)
        n, N, order, offs, kv_deep = self._deep(act, K, pos)
        iv.stop()
        host = self.out_host[:n + N]
        host.copy_(self.out[:n + N], non_blocking=True)
        torch.cuda.current_stream().synchronize()           # the one device->host read per round
        self.d2h_bytes += 4 * (n + N)
        recs.append(("verify", iv, n, n, N, kv + kv_deep))
        for kind, t, bb, st, dt, kvr in recs:
            self.records.append(StepRecord(kind, t.ms, bb, st, dt, kvr, measured))
        out = host.numpy()
        acc_h, y_h = out[:n], out[n:n + N]
        committed = 0
        self.stats["rounds"] += 1
        for v, s in enumerate(order):
            a = int(acc_h[v])
            st = self.slots[s]
            st.pos = pos[s] + a + 1
            st.last_token = int(y_h[offs[v] + a])
            committed += self._commit(s, y_h[offs[v]:offs[v] + a + 1].tolist())
            if measured and st.finish_reason is None:
                S = self.stats
                S["request_rounds"] += 1
                S["drafted"] += K[s]
                S["accepted"] += a
                S["rejected"] += K[s] - a
                S["deep_tokens"] += K[s] + 1
                self.exit_hist[int(self.exit_of[s])] += 1
        return committed

    def extra_metrics(self) -> dict:
        st = dict(self.stats)
        rr = max(st["request_rounds"], 1)
        st.update(exit_layers=self.exits, gamma_range=[self.g_lo, self.g_hi], schedule=self.schedule,
                  acceptance_rate=st["accepted"] / max(st["drafted"], 1),
                  tokens_per_verify=(st["accepted"] + st["request_rounds"]) / rr,
                  exit_hist={str(k): v for k, v in self.exit_hist.items()})
        return {"spec": st}
