"""Rollout engine for hybrid models (linear-recurrence layers interleaved with attention:
models.hybrid): the attention layers use the engine's paged KV, mounts and cursors as for a
dense decoder; each linear layer carries per-sequence state instead of KV.

State.  A linear layer's state is its recurrent state [heads, d, d] (fp32) plus its causal
conv's last W - 1 inputs [W - 1, 3C].  A request starts from zeros, or from the snapshot kept
with the cursor it continues; mounted rows reach the attention layers only (a recurrent
layer keeps the reader's own state, as in training).  Prefill runs each linear layer as
one varlen call over the batch's requests (initial states and conv contexts per request);
decode advances every row by one token per step.  A row's state stops changing after the
last token it keeps (a stop token or its max_new_tokens), so the snapshot stored with its
cursor is the state after exactly the cursor's rows with KV, and a continuation from the
cursor gives what one pass over the whole sequence would.

Prefix reuse.  The radix cache is off: a prefix match would give KV without the linear
layers' state at the match point.  A cursor whose snapshot is gone (released, evicted, or
reset) answers 404 (CursorNotFound), as an evicted cursor does.

CUDA graphs are not used (the varlen recurrence call takes host segment tables).

Reference parity (behaviour): SGLang's hybrid-model state pool used by the reference's
rollout for Qwen3.5 / Qwen3-Next (`octopus/serving/kv_mount.py:553-562` copies recurrent
state with mounts, which stay attention-only); models.hybrid for the layer.
"""
from __future__ import annotations

import numpy as np
import torch

from .. import ops
from ..models.hybrid import HybridWeights, _rmsnorm_heads
from ..ops import serve as sv
from ..ops.recurrence import causal_conv, recurrence
from .engine import CursorNotFound, Engine, GenInput, _Req

__all__ = ["HybridEngine"]


class HybridEngine(Engine):
    def __init__(self, hw: HybridWeights, **kw):
        kw["use_graphs"] = False
        super().__init__(hw.hc.base, hw.dense, **kw)
        self.hw = hw
        self.hc = hw.hc
        self._use_radix = False
        self.lin_layers = [i for i in range(self.cfg.layers) if self.hc.is_linear(i)]
        hc, B = self.hc, self.max_batch
        self._sdt = torch.float64 if hw.dense.flat.dtype == torch.float64 else torch.float32
        self.snap: dict[str, dict] = {}   # cursor id -> {layer: (state, conv)}
        self.live: dict[int, dict] = {}   # request id -> {layer: (state, conv)} between prefill and decode
        W, C = hc.conv_width, hc.lin_width
        dev = self.device
        # decode-time state of the batch rows
        self.s_state = {i: torch.zeros(B, hc.lin_heads, hc.lin_dim, hc.lin_dim, dtype=self._sdt, device=dev)
                        for i in self.lin_layers}
        self.s_conv = {i: torch.zeros(B, W - 1, 3 * C, dtype=self._sdt, device=dev) for i in self.lin_layers}
        self.s_done = torch.zeros(B, dtype=torch.bool, device=dev)
        self.s_limit = torch.zeros(B, dtype=torch.int64, device=dev)
        self.s_stop = torch.full((B, 1), -1, dtype=torch.int64, device=dev)
        self._done_now = None
        self._group = None

    # ------------------------------------------------------------------ state bookkeeping
    def _zero_state(self):
        hc, dev = self.hc, self.device
        W, C = hc.conv_width, hc.lin_width
        return {i: (torch.zeros(hc.lin_heads, hc.lin_dim, hc.lin_dim, dtype=self._sdt, device=dev),
                    torch.zeros(W - 1, 3 * C, dtype=self._sdt, device=dev)) for i in self.lin_layers}

    def _start_state(self, r: _Req):
        if r.inp.cursor is None:
            return self._zero_state()
        st = self.snap.get(r.inp.cursor)
        if st is None:
            raise CursorNotFound(r.inp.cursor)
        return st

    def _resolve(self, inp: GenInput) -> _Req:
        if inp.cursor is not None and inp.cursor not in self.snap:
            raise CursorNotFound(inp.cursor)
        return super()._resolve(inp)

    def release_cursor(self, cid: str):
        super().release_cursor(cid)
        self.snap.pop(cid, None)

    def reset(self):
        super().reset()
        self.snap.clear()
        self.live.clear()

    def _sweep(self):
        """Drop snapshots of cursors the store no longer holds (evicted)."""
        for cid in [c for c in self.snap if self.cursors.get(c) is None]:
            del self.snap[cid]

    # ------------------------------------------------------------------ prefill
    def _prefill_group(self, reqs, g, cu_q):
        starts = [self._start_state(reqs[j]) for j in g]
        segs = [(int(cu_q[k]), int(cu_q[k + 1] - cu_q[k])) for k in range(len(g))]
        self._group = {"reqs": [reqs[j] for j in g], "segs": segs, "starts": starts, "fin": {}}

    def _prefill_group_done(self, reqs, g):
        grp = self._group
        for k, r in enumerate(grp["reqs"]):
            self.live[r.rid] = {i: (grp["fin"][i][0][k], grp["fin"][i][1][k]) for i in self.lin_layers}
        self._group = None

    def _layer(self, x, i, pos, write_slots, attn):
        if not self.hc.is_linear(i):
            return super()._layer(x, i, pos, write_slots, attn)
        grp = self._group
        T = x.shape[0]
        segs = list(grp["segs"])
        n = len(segs)
        end = segs[-1][0] + segs[-1][1]
        if end < T:  # padding rows: a segment of their own from zeros
            segs.append((end, T - end))
        init = torch.stack([st[i][0] for st in grp["starts"]])
        ctx = torch.stack([st[i][1] for st in grp["starts"]])
        idx = list(range(n)) + ([-1] if len(segs) > n else [])
        y, fin, qkv = self._lin_forward(x, i, segs, init, idx, ctx, idx)
        # conv state after the request: the last W - 1 conv inputs of [context || its rows]
        W = self.hc.conv_width
        convs = []
        for k, (a, ln) in enumerate(segs[:n]):
            full = torch.cat([ctx[k].to(qkv.dtype), qkv[a:a + ln]])
            convs.append(full[-(W - 1):].to(self._sdt))
        grp["fin"][i] = (fin[:n].to(self._sdt), torch.stack(convs))
        return y

    def _lin_forward(self, x, i, segs, init, init_idx, ctx, ctx_idx):
        """models.hybrid.linear_layer_forward over request segments with given initial states
        and conv contexts; returns (layer output, final states, pre-conv rows)."""
        hw, hc, cfg = self.hw, self.hc, self.cfg
        t = hw.t
        h = ops.rmsnorm(x, t[f"layers.{i}.ln1"], cfg.rms_eps, cfg.norm_plus_one)
        qkv = ops.linear(h, t[f"layers.{i}.lin_qkv"])
        z = ops.linear(h, t[f"layers.{i}.lin_z"])
        ba = ops.linear(h, t[f"layers.{i}.lin_ba"])
        bb, aa = ba[:, :hc.lin_heads], ba[:, hc.lin_heads:2 * hc.lin_heads]
        cdt = torch.float64 if x.dtype == torch.float64 else torch.float32
        qc = causal_conv(qkv, hw.fp32[f"layers.{i}.conv_w"].to(cdt), None, segs, ctx=ctx.to(cdt), ctx_idx=ctx_idx)
        y, fin = self._lin_tail(x, qc, z, bb, aa, i, segs, init, init_idx)
        return y, fin, qkv

    def _lin_tail(self, x, qc, z, bb, aa, i, segs, init, init_idx):
        hw, hc, cfg = self.hw, self.hc, self.cfg
        t = hw.t
        C, Hh, d = hc.lin_width, hc.lin_heads, hc.lin_dim
        T = x.shape[0]
        q = torch.nn.functional.normalize(qc[:, :C].float().view(T, Hh, d), dim=-1).to(x.dtype).reshape(T, C)
        k = torch.nn.functional.normalize(qc[:, C:2 * C].float().view(T, Hh, d), dim=-1).to(x.dtype).reshape(T, C)
        v = qc[:, 2 * C:].to(x.dtype).contiguous()
        gd = torch.float64 if x.dtype == torch.float64 else torch.float32
        beta = torch.sigmoid(bb.to(gd))
        g = -torch.exp(hw.fp32[f"layers.{i}.A_log"].to(gd)) * torch.nn.functional.softplus(
            aa.to(gd) + hw.fp32[f"layers.{i}.dt_bias"].to(gd))
        o, fin = recurrence(q.contiguous(), k.contiguous(), v, g.contiguous(), beta.contiguous(), segs, d ** -0.5,
                            hc.kind == "gdn", init_state=init.to(torch.float64 if gd == torch.float64 else
                                                                  torch.float32), init_idx=init_idx)
        o = _rmsnorm_heads(o.view(T, Hh, d), t[f"layers.{i}.lin_norm"], cfg.rms_eps).reshape(T, C)
        o = (o.float() * torch.nn.functional.silu(z.float())).to(x.dtype)
        x = ops.linear(o, t[f"layers.{i}.lin_out"], None, residual=x)
        h2 = ops.rmsnorm(x, t[f"layers.{i}.ln2"], cfg.rms_eps, cfg.norm_plus_one)
        act = ops.swiglu(ops.linear(h2, t[f"layers.{i}.gu_w"]))
        return ops.linear(act, t[f"layers.{i}.down_w"], None, residual=x), fin

    # ------------------------------------------------------------------ decode
    def _decode_begin(self, reqs, chunk, B, steps):
        self._B = B
        stops = [list(reqs[j].inp.stop_ids or ()) for j in chunk]
        S = max([1] + [len(x) for x in stops])
        stop = np.full((B, S), -1, np.int64)
        limit = np.full(B, -1, np.int64)  # padding rows: done from the start
        for k, j in enumerate(chunk):
            r = reqs[j]
            stop[k, :len(stops[k])] = stops[k]
            limit[k] = (0 if r.inp.prefill_only else r.inp.max_new_tokens) - 1
            live = self.live[r.rid]
            for i in self.lin_layers:
                self.s_state[i][k].copy_(live[i][0])
                self.s_conv[i][k].copy_(live[i][1])
        self.s_stop = torch.as_tensor(stop, device=self.device)
        self.s_limit[:B].copy_(torch.as_tensor(limit, device=self.device))
        self.s_done[:B].zero_()

    def _decode_end(self, reqs, chunk):
        for k, j in enumerate(chunk):
            r = reqs[j]
            self.live[r.rid] = {i: (self.s_state[i][k].clone(), self.s_conv[i][k].clone()) for i in self.lin_layers}

    def _decode_forward(self, tok, pos, slot, attn, B: int, temperature: float):
        # a row whose input token is the last it keeps (a stop token, or its last allowed)
        # does not advance its state: the state stays at the cursor's last row with KV
        st = self.s_step.expand(B)
        self._done_now = self.s_done[:B] | (tok[:, None] == self.s_stop[:B]).any(-1) | (st >= self.s_limit[:B])
        cfg = self.cfg
        x = sv.embed(tok, self.w["embed"])
        for i in range(cfg.layers):
            if self.hc.is_linear(i):
                x = self._lin_decode(x, i, B)
            else:
                h = sv.rms(x, self.w.layer(i)[0], cfg.rms_eps, cfg.norm_plus_one)
                x, _ = self._layer_decode(x, h, i, pos, slot, attn)
        self.s_done[:B].copy_(self._done_now)
        h = self._final(x)
        tp_, tk_ = self._filter
        return ops.sample(h, self.w.head, temperature, self.seed, self.s_stream[:B], cfg.vocab_size, tp_, tk_)

    def _lin_decode(self, x, i, B):
        hw, hc, cfg = self.hw, self.hc, self.cfg
        t = hw.t
        h = ops.rmsnorm(x, t[f"layers.{i}.ln1"], cfg.rms_eps, cfg.norm_plus_one)
        qkv = ops.linear(h, t[f"layers.{i}.lin_qkv"])
        z = ops.linear(h, t[f"layers.{i}.lin_z"])
        ba = ops.linear(h, t[f"layers.{i}.lin_ba"])
        bb, aa = ba[:, :hc.lin_heads], ba[:, hc.lin_heads:2 * hc.lin_heads]
        # causal conv of one step: taps over [the row's last W - 1 inputs || this input]
        cdt = torch.float64 if x.dtype == torch.float64 else torch.float32
        xs = torch.cat([self.s_conv[i][:B].to(cdt), qkv.to(cdt)[:, None, :]], 1)  # [B, W, 3C]
        acc = (xs * hw.fp32[f"layers.{i}.conv_w"].to(cdt).t()[None]).sum(1)
        qc = (acc * torch.sigmoid(acc)).to(qkv.dtype)
        segs = [(k, 1) for k in range(B)]
        y, fin = self._lin_tail(x, qc, z, bb, aa, i, segs, self.s_state[i][:B], list(range(B)))
        keep = self._done_now[:, None, None, None]
        self.s_state[i][:B] = torch.where(keep, self.s_state[i][:B], fin.to(self._sdt))
        self.s_conv[i][:B] = torch.where(keep[:, :, :, 0], self.s_conv[i][:B], xs[:, 1:].to(self._sdt))
        return y

    # ------------------------------------------------------------------ cursors
    supports_continuous = False  # recurrent states follow the static batch layout of generate
    _spillable = False  # a cursor's recurrent-state snapshots are not rebuilt from its recipe

    def generate(self, inputs):
        self._sweep()
        try:
            return super().generate(inputs)
        finally:
            self.live.clear()

    def _on_cursor(self, r, cid: str):
        live = self.live.get(r.rid)
        if live is not None:
            self.snap[cid] = live
