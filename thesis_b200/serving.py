"""Open-loop serving: Poisson arrivals with new-request prefill piggybacked on draft/verify steps.

BASELINE config 5 (Llama3-8B shape, B=256 per GPU, Poisson arrivals, E=8, gamma=4, prefill
piggybacked on verify steps).  Counterparts in the reference:

* ``run_poisson`` (solutions/engine.py:625-673): requests arrive by a Poisson process in wall-clock
  time, free slots take them first-in first-out, warm-up requests are not measured.
* Mechanism 3, depth-split piggybacking (solutions/prefill.py:1-20, solutions/engine.py:269-305,
  415-489): a chunk of a pending prompt rides on the shallow segment of a step (layers [0, E), its
  layer-E hidden state is kept), and on the deep segment of the next verify step (layers [E, L)).
  KV is written to every layer as the chunk passes through it, later chunks attend to earlier
  ones, and the deep pass of the final chunk yields the request's first token.

Here every shallow step (the gamma draft steps and the shallow part of the verify step) carries
up to ``piggyback_budget`` prompt tokens (prompts in arrival order) in the same packed call as the
draft tokens; the verify step's deep call carries every chunk that went through the shallow
layers this round, merged into one block per request.  The chunk size is a fixed token budget per
step where the reference asks its calibrated cost model for the knee; with no decoding request
left, pending prompts are prefilled through all layers in one call (the reference's ``flush``).
"""

from __future__ import annotations

import time
from dataclasses import dataclass, field

import numpy as np
import torch

from . import lib
from .eesd import B200SpecEngine
from .engine import Interval, StepRecord


@dataclass
class _Prefill:
    tokens: list
    sh: int = 0                                   # prompt positions through the shallow layers
    pending: list = field(default_factory=list)   # [(p0, c, row in pend_h)] awaiting the deep layers


class B200ServingEngine(B200SpecEngine):
    """Fixed-exit speculation whose new requests are prefilled inside the draft/verify steps."""

    name = "b200_layerskip_serving"

    def __init__(self, model, batch_size, max_prompt_len, max_new_tokens, eos_ids, *, exit_layer: int, gamma: int,
                 piggyback_budget: int = 256, **kw):
        self.budget = int(piggyback_budget)
        if self.budget < 1:
            raise ValueError("piggyback_budget must be >= 1")
        # shallow calls: B drafts + budget; verify deep call: B (gamma + 1) + every pending chunk
        super().__init__(model, batch_size, max_prompt_len, max_new_tokens, eos_ids, exit_layer=exit_layer,
                         gamma=gamma, extra_tokens=(gamma + 1) * self.budget, **kw)
        self.pend_cap = (self.gamma + 1) * self.budget
        self.pend_h = torch.empty(self.pend_cap, self.cfg.dim, dtype=self.weights.dtype, device=self.device)
        self.xbuf = torch.empty(self.B * self.cols + self.pend_cap, self.cfg.dim, dtype=self.weights.dtype,
                                device=self.device)
        self.out = torch.empty(self.B + self.B * self.cols + self.B, dtype=torch.int32, device=self.device)
        self.out_host = torch.empty_like(self.out, device="cpu").pin_memory()
        self.dt_code = lib.BF16 if self.weights.dtype == torch.bfloat16 else lib.F32
        self.pf: dict = {}                 # slot -> _Prefill while its prompt is being prefilled
        self.pf_order: list = []           # prefilling slots in assignment order
        self.stats.update(piggyback_tokens=0, flush_tokens=0, flush_steps=0)
        self.first_token_wall: dict = {}

    # ---------------------------------------------------------------- admission (prefill deferred)
    def _assign_many(self, items) -> None:
        now = time.perf_counter()
        for slot, idx, prompt in items:
            if len(prompt.tokens) + self.max_new + 2 > self.max_seq_alloc():
                raise ValueError(f"prompt of {len(prompt.tokens)} tokens does not fit max_seq={self.max_seq_alloc()}")
            if not prompt.tokens:
                raise ValueError("empty prompt")
            s = self.slots[slot]
            s.prompt_idx, s.pid, s.prompt_len = idx, prompt.pid, len(prompt.tokens)
            s.pos, s.last_token = 0, 0
            s.output, s.finish_reason, s.idle = [], None, False
            s.t_assigned, s.decode_ms = now, 0.0
            s.max_new = min(int(prompt.max_new), self.max_new) if getattr(prompt, "max_new", None) else None
            self.pf[slot] = _Prefill(list(prompt.tokens))
            self.pf_order.append(slot)

    def _decoding(self) -> list:
        return [s for s in self._active() if s not in self.pf]

    def _plan_chunks(self, budget: int, pend_used: int) -> list:
        """[(slot, p0, c, pend row)] for one shallow call, prompts in assignment order."""
        out = []
        for s in self.pf_order:
            p = self.pf[s]
            rem = len(p.tokens) - p.sh
            c = min(rem, budget, self.pend_cap - pend_used)
            if c <= 0:
                continue
            out.append((s, p.sh, c, pend_used))
            p.pending.append((p.sh, c, pend_used))
            p.sh += c
            budget -= c
            pend_used += c
            if budget <= 0 or pend_used >= self.pend_cap:
                break
        return out

    # ---------------------------------------------------------------- passes
    def _shallow_pb(self, act: list, pos: np.ndarray, j: int, draft: bool, chunks: list):
        """Token j of every decoding request, plus prompt chunks, through [0, E)."""
        dm, cols = self.dm, self.cols
        n = len(act)
        nc = sum(c for (_, _, c, _) in chunks)
        blocks = [(s, int(p) + j, 1) for s, p in zip(act, pos)] + [(s, p0, c) for (s, p0, c, _) in chunks]
        ph = dm.pack(blocks)
        src = np.array(act, dtype=np.int32) * cols + j
        cid = np.array([t for (s, p0, c, _) in chunks for t in self.pf[s].tokens[p0:p0 + c]], dtype=np.int32)
        b, (src_d, dst_d, cid_d) = dm.upload(ph, (src, src + 1, cid))
        sp = lib.stream_ptr()
        x = self.xbuf[:n + nc]
        if n:
            ids = torch.empty(n, dtype=torch.int32, device=self.device)
            lib.call("eesd_gather_ids", self.seq_buf.data_ptr(), src_d.data_ptr(), ids.data_ptr(), n, sp)
            dm.embed(ids, out=x[:n])
        if nc:
            dm.embed(cid_d, out=x[n:])
        dm.forward_layers(x, b, 0, self.k)
        if n:
            lib.call("eesd_copy_rows", self.dt_code, x.data_ptr(), None, self.exit_h.data_ptr(), src_d.data_ptr(), n,
                     self.cfg.dim, sp)
        if nc:
            row0 = chunks[0][3]
            lib.call("eesd_copy_rows", self.dt_code, x[n:].data_ptr(), None, self.pend_h[row0:].data_ptr(), None, nc,
                     self.cfg.dim, sp)
        if draft and n:
            d = dm.head_argmax(x[:n])
            lib.call("eesd_scatter_ids", d.data_ptr(), dst_d.data_ptr(), self.seq_buf.data_ptr(), n, sp)
        self.h2d_bytes += 4 * (2 * (n + nc) + 4 * len(blocks) + 2 * len(ph.items) + 2 * n + nc)
        if nc and self._measuring:
            self.stats["piggyback_tokens"] += nc
        return ph

    def _finish_prefills(self, done: list, first: np.ndarray) -> int:
        """Slots whose prompt went through every layer: first token committed, decoding starts."""
        committed = 0
        now = time.perf_counter()
        for s, t in zip(done, first):
            st = self.slots[s]
            st.pos, st.last_token = st.prompt_len, int(t)
            del self.pf[s]
            self.pf_order.remove(s)
            self.first_token_wall[s] = now
            committed += self._commit(s, [int(t)])
        return committed

    @torch.inference_mode()
    def _flush(self, measured: bool) -> int:
        """No decoding request: prefill pending prompts through all layers in one call."""
        dm, L = self.dm, self.cfg.n_layers
        chunks = self._plan_chunks(self.pend_cap, 0)
        for s, _, _, _ in chunks:
            self.pf[s].pending.clear()
        blocks = [(s, p0, c) for (s, p0, c, _) in chunks]
        ph = dm.pack(blocks)
        cid = np.array([t for (s, p0, c, _) in chunks for t in self.pf[s].tokens[p0:p0 + c]], dtype=np.int32)
        ends = [int(ph.offsets[i + 1]) - 1 for i, (s, p0, c, _) in enumerate(chunks) if p0 + c == len(self.pf[s].tokens)]
        done = [s for (s, p0, c, _) in chunks if p0 + c == len(self.pf[s].tokens)]
        idx = np.array([s * self.cols for s in done], dtype=np.int32)
        iv = Interval(self.device).start()
        b, (cid_d, ends_d, idx_d) = dm.upload(ph, (cid, np.array(ends, dtype=np.int32), idx))
        x = dm.embed(cid_d)
        dm.forward_layers(x, b, 0, L)
        first = None
        if done:
            y = self.out[:len(done)]
            dm.head_argmax(x, ends_d, out=y)
            lib.call("eesd_scatter_ids", y.data_ptr(), idx_d.data_ptr(), self.seq_buf.data_ptr(), len(done),
                     lib.stream_ptr())
        iv.stop()
        if done:
            first = y.cpu().numpy()
        self.records.append(StepRecord("prefill", iv.ms, len(chunks), ph.n_tokens, ph.n_tokens, ph.kv_read, measured))
        if measured:
            self.stats["flush_tokens"] += ph.n_tokens
            self.stats["flush_steps"] += 1
        return self._finish_prefills(done, first) if done else 0

    @torch.inference_mode()
    def _iteration(self, measured: bool) -> int:
        self._measuring = measured
        act = self._decoding()
        if not act:
            return self._flush(measured) if self.pf else 0
        dm, g, cols, L = self.dm, self.gamma, self.cols, self.cfg.n_layers
        n = len(act)
        pos = np.array([self.slots[s].pos for s in act], dtype=np.int64)
        pend_used = 0
        recs = []
        for j in range(g + 1):
            chunks = self._plan_chunks(self.budget, pend_used)
            pend_used += sum(c for (_, _, c, _) in chunks)
            iv = Interval(self.device).start()
            ph = self._shallow_pb(act, pos, j, draft=j < g, chunks=chunks)
            if j < g:
                iv.stop()
                recs.append(("draft", iv, n, ph.n_tokens, 0, ph.kv_read))
        # ---- verify: every decoding request's gamma+1 tokens + every chunk that passed [0, E) this round
        pend = [(s, self.pf[s]) for s in self.pf_order if self.pf[s].pending]
        vblocks = [(s, int(p), cols) for s, p in zip(act, pos)]
        cblocks = [(s, p.pending[0][0], sum(c for (_, c, _) in p.pending)) for s, p in pend]
        ph = dm.pack(vblocks + cblocks)
        N_v = n * cols
        vrows = (np.array(act, dtype=np.int32)[:, None] * cols + np.arange(cols, dtype=np.int32)[None, :]).reshape(-1)
        prow = np.array([r0 + i for _, p in pend for (_, c, r0) in p.pending for i in range(c)], dtype=np.int32)
        done = [s for s, p in pend if p.sh == len(p.tokens)]
        ends, off = [], N_v
        for s, p in pend:
            off += sum(c for (_, c, _) in p.pending)
            if p.sh == len(p.tokens):
                ends.append(off - 1)
        hrows = np.concatenate([np.arange(N_v, dtype=np.int32), np.array(ends, dtype=np.int32)])
        vinfo = np.stack([np.arange(n, dtype=np.int32) * cols, np.full(n, cols, dtype=np.int32),
                          np.array(act, dtype=np.int32)], axis=1)
        fidx = np.array([s * cols for s in done], dtype=np.int32)
        b, (vrows_d, prow_d, hrows_d, vinfo_d, fidx_d) = dm.upload(ph, (vrows, prow, hrows, vinfo, fidx))
        sp = lib.stream_ptr()
        N = ph.n_tokens
        x = self.xbuf[:N]
        lib.call("eesd_copy_rows", self.dt_code, self.exit_h.data_ptr(), vrows_d.data_ptr(), x.data_ptr(), None, N_v,
                 self.cfg.dim, sp)
        if len(prow):
            lib.call("eesd_copy_rows", self.dt_code, self.pend_h.data_ptr(), prow_d.data_ptr(), x[N_v:].data_ptr(),
                     None, len(prow), self.cfg.dim, sp)
        dm.forward_layers(x, b, self.k, L)
        nh = len(hrows)
        acc = self.out[:n]
        y = self.out[n:n + nh]
        dm.head_argmax(x, hrows_d, out=y)
        lib.call("eesd_greedy_accept", y.data_ptr(), vinfo_d.data_ptr(), n, self.seq_buf.data_ptr(), cols,
                 acc.data_ptr(), sp)
        if done:
            lib.call("eesd_scatter_ids", y[N_v:].data_ptr(), fidx_d.data_ptr(), self.seq_buf.data_ptr(), len(done), sp)
        iv.stop()
        host = self.out_host[:n + nh]
        host.copy_(self.out[:n + nh], non_blocking=True)
        torch.cuda.current_stream().synchronize()           # the one device->host read per round
        self.h2d_bytes += 4 * (2 * N + 4 * len(vblocks + cblocks) + 2 * len(ph.items) + N_v + len(prow) + nh + 3 * n)
        self.d2h_bytes += 4 * (n + nh)
        recs.append(("verify", iv, n, n, N, ph.kv_read))
        for kind, t, bb, st_, dt, kv in recs:
            self.records.append(StepRecord(kind, t.ms, bb, st_, dt, kv, measured))
        for _, p in pend:
            p.pending.clear()
        out = host.numpy()
        acc_h, y_h = out[:n], out[n:n + N_v].reshape(n, cols)
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
                S["full_accept_rounds"] += int(a == g)
                self.accept_hist[a] += 1
        if done:
            committed += self._finish_prefills(done, out[n + N_v:n + nh])
        return committed

    _measuring = False

    # ---------------------------------------------------------------- open-loop driver
    @torch.inference_mode()
    def run_poisson(self, prompts: list, rate_per_s: float, n_requests: int, warm_requests: int = 8, seed: int = 0,
                    keep_outputs: bool = False) -> dict:
        """Requests arrive by a Poisson process in wall-clock time; free slots take them first in,
        first out (solutions/engine.py:625-673).  Completions of the first ``warm_requests`` are
        not measured; the run ends after ``n_requests`` measured completions."""
        rng = np.random.default_rng(seed)
        self.records = []
        queue, completions = [], []
        cursor = total_done = 0
        t0 = time.perf_counter()
        next_arr = t0 + rng.exponential(1 / rate_per_s)
        arrival, measured_req = {}, {}
        measuring = warm_requests == 0
        t_meas = t0 if measuring else None
        tok_measured = 0
        while total_done < n_requests + warm_requests:
            now = time.perf_counter()
            while next_arr <= now:
                queue.append((cursor, prompts[cursor % len(prompts)], next_arr))
                cursor += 1
                next_arr += rng.exponential(1 / rate_per_s)
            free = [s for s, st in enumerate(self.slots) if st.idle]
            take = []
            while free and queue:
                idx, p, t_arr = queue.pop(0)
                s = free.pop(0)
                take.append((s, idx, p))
                arrival[s] = t_arr
                measured_req[s] = measuring
            self._assign_many(take)
            if not self._active():
                time.sleep(max(0.0, min(next_arr - time.perf_counter(), 0.01)))
                continue
            committed = self._iteration(measured=measuring)
            if measuring:
                tok_measured += committed
            for s, st in enumerate(self.slots):
                if st.idle or st.finish_reason is None:
                    continue
                t_end = time.perf_counter()
                t_first = self.first_token_wall.pop(s, t_end)
                c = {"pid": st.pid, "prompt_idx": st.prompt_idx, "prompt_len": st.prompt_len,
                     "generated": len(st.output), "finish_reason": st.finish_reason, "measured": measured_req[s],
                     "ttft_s": t_first - arrival[s],
                     "tpot_s": (t_end - t_first) / max(len(st.output) - 1, 1)}
                if keep_outputs:
                    c["tokens"] = list(st.output)
                completions.append(c)
                total_done += 1
                st.idle = True
                if not measuring and total_done >= warm_requests:
                    measuring = True
                    torch.cuda.synchronize()
                    t_meas = time.perf_counter()
        torch.cuda.synchronize()
        wall = time.perf_counter() - t_meas if t_meas is not None else 0.0
        rec = [r for r in self.records if r.measured]
        decode_ms = sum(r.forward_ms for r in rec if r.kind != "prefill")
        prefill_ms = sum(r.forward_ms for r in rec if r.kind == "prefill")
        meas = [c for c in completions if c["measured"]]
        ttft = [1000 * c["ttft_s"] for c in meas]
        tpot = [1000 * c["tpot_s"] for c in meas if c["generated"] > 1]
        per_kind = {}
        for kind in sorted({r.kind for r in rec}):
            ms = [r.forward_ms for r in rec if r.kind == kind]
            per_kind[kind] = {"steps": len(ms), "mean_ms": float(np.mean(ms)), "p50_ms": float(np.median(ms))}
        S = self.stats
        metrics = {
            "stop_reason": "n_requests", "poisson_rate_per_s": rate_per_s, "queue_left": len(queue),
            "evaluated_completions": len(meas), "measured_tokens": tok_measured,
            "decode_ms": decode_ms, "prefill_ms": prefill_ms,
            "throughput_tok_s": tok_measured / (decode_ms / 1000) if decode_ms else None,
            "e2e_throughput_tok_s": tok_measured / ((decode_ms + prefill_ms) / 1000) if decode_ms + prefill_ms else None,
            "wall_s": wall, "wall_throughput_tok_s": tok_measured / wall if wall else None,
            "ttft_ms_mean": float(np.mean(ttft)) if ttft else None,
            "ttft_ms_p99": float(np.percentile(ttft, 99)) if ttft else None,
            "tpot_ms_mean": float(np.mean(tpot)) if tpot else None,
            "tpot_ms_p99": float(np.percentile(tpot, 99)) if tpot else None,
            "prefill_tokens_piggyback": S["piggyback_tokens"], "prefill_tokens_flush": S["flush_tokens"],
            "piggyback_share_of_prefill_tokens": S["piggyback_tokens"] / max(S["piggyback_tokens"] + S["flush_tokens"], 1),
            "acceptance_rate": S["accepted"] / max(S["drafted"], 1),
            "steps": per_kind,
        }
        return {"metrics": metrics, "completions": completions, "steps": []}
