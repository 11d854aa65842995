"""Rollout engine: paged (page size 1) KV with zero-copy sharing, cursors, mounts and
CUDA-graph decode on the sm_100a kernels.

Request model (the wire format of ``/generate``):
  * ``input_ids``   new tokens to prefill (the delta after ``cursor``, or a full prompt)
  * ``cursor``      continue from a server-resident reply (its KV is reused zero-copy)
  * ``mount``       ``[(cursor, start, end), ...]`` splice rows [start, end) of other
                    cursors into this request's context (zero-copy; rule K2 positions)
Every request owns the KV slots of its new tokens and of its generated tokens; all
other rows it attends to are slots shared by reference (radix prefix hits, cursor
rows, mounted rows).  Refcounts in the native SlotPool free a slot exactly once.

Prefill runs all requests of a batch through one ragged forward: the gathered-key
attention kernel reads each request's key list (context slots + its own new slots)
straight from the KV cache.  Decode runs one captured CUDA graph per batch bucket:
embedding -> 28x(norm, QKV GEMM + bias, RoPE, KV write, split-K paged attention,
O GEMM + residual, norm, gate/up GEMM, SwiGLU, down GEMM + residual) -> fused
sampling head (GEMM + Gumbel-max + logprob epilogue), with positions, KV lengths and
RNG streams advanced on the device, so a decode step needs no host work.

Reference parity: `octopus/serving/kv_mount.py:87-296` (prepare: tokens(B) +
placeholders + delta, K2 offsets, rebuild/abort semantics), `kv_mount.py:347-383`
(resolve: append mounted segment pages after B's prefix), `kv_mount.py:585-634`
(layer-subset views, position offsets), SGLang's scheduler/radix cache (prefix reuse).
"""
from __future__ import annotations

import itertools
import os
import time
from dataclasses import dataclass, field

import numpy as np
import torch

from .. import ops
from ..ops import serve as sv
from ..models.config import ModelConfig
from ..models.decoder import Weights
from ..utils.iostats import d2h, h2d
from .cursor_store import PLACEHOLDER, Cursor, CursorStore

try:
    from .. import _native
except ImportError:  # pragma: no cover - native module not built
    _native = None

NULL_SLOT = 0  # reserved scratch slot for padding rows


class CursorNotFound(KeyError):
    pass


class OutOfKV(RuntimeError):
    pass


def mount_layers_from_env(n_layers: int):
    v = os.environ.get("OCTOPUS_MOUNT_LAYERS", "").strip()
    if not v:
        return None
    return sorted({int(x) for x in v.replace(" ", "").split(",") if x != ""} & set(range(n_layers)))


@dataclass
class GenInput:
    input_ids: list
    cursor: str | None = None
    mount: list = field(default_factory=list)  # [(cursor_id, start, end)]
    max_new_tokens: int = 128
    temperature: float = 1.0
    stop_ids: tuple = ()
    rid: int | None = None
    keep_cursor: bool = True
    cursor_id: str | None = None  # id to store the reply under (default: generated)
    prefill_only: bool = False
    # positions of mounted keys: K2 (default) keeps their positions and continues at
    # max(own next, last mounted + 1); K1 keeps their positions and continues at its own
    # next; K3 relocates them to the request's next positions (copies whose keys are
    # re-rotated by the offset) and continues after them
    mount_rule: str = "K2"
    # nucleus / top-k filtering (1.0 / 0: off; top_k >= vocab: off); shared by the batch like
    # the temperature
    top_p: float = 1.0
    top_k: int = 0


@dataclass
class GenOutput:
    output_ids: list
    output_logprobs: list
    cursor: str | None
    prompt_tokens: int          # rows prefilled by this request (placeholders excluded)
    cached_tokens: int          # rows reused from cache/cursor
    first_pos: int
    finish_reason: str = "length"


@dataclass
class _Req:
    inp: GenInput
    rid: int
    ctx_tokens: np.ndarray
    ctx_slots: np.ndarray
    ctx_pos: np.ndarray
    ctx_mounted: np.ndarray
    new_tokens: np.ndarray
    first_pos: int
    own_slots: np.ndarray = None
    cached: int = 0
    radix_handle: int = -1
    out_tok: list = field(default_factory=list)
    out_lp: list = field(default_factory=list)
    mount_at: list = field(default_factory=list)
    extra_slots: list = field(default_factory=list)  # K3 relocated copies this request allocated
    pinned: bool = False  # holds one reference on ctx_slots while it runs (spills cannot free them)


class Engine:
    def __init__(self, cfg: ModelConfig, weights: Weights, *, kv_slots: int | None = None,
                 kv_bytes: int | None = None, max_batch: int = 256, device="cuda", use_graphs: bool = True,
                 seed: int = 1234, prefill_chunk: int = 16384, num_splits: int | None = None,
                 mount_layers=None, kv_index_capacity: int = 1 << 25):
        if _native is None:
            raise RuntimeError("octopus_b200._native (KV manager) is not built")
        self.cfg, self.w = cfg, weights
        self.device = torch.device(device)
        hq_loc, hkv_loc = self._local_heads()
        kvw = hkv_loc * cfg.head_dim
        if kv_slots is None:
            per = 2 * cfg.layers * kvw * 2
            kv_slots = max(4096, int((kv_bytes or (8 << 30)) // per))
        self.kv_slots = kv_slots
        kv_dtype = weights.flat.dtype
        self.kc = torch.zeros(cfg.layers, kv_slots, kvw, dtype=kv_dtype, device=self.device)
        self.vc = torch.zeros(cfg.layers, kv_slots, kvw, dtype=kv_dtype, device=self.device)
        self.pool = _native.SlotPool(kv_slots)
        self.null_slot = int(self.pool.alloc(1)[0])  # never freed: padding rows read/write it
        self.radix = _native.RadixCache(self.pool)
        self.cursors = CursorStore(self.pool)
        self.max_batch = max_batch
        self.seed = seed
        self.use_graphs = use_graphs and self.device.type == "cuda"
        self.prefill_chunk = prefill_chunk
        self.mount_layers = mount_layers if mount_layers is not None else mount_layers_from_env(cfg.layers)
        self.version = 0
        self._rid = itertools.count(1)
        self._cid = itertools.count(1)
        self._uid = os.urandom(3).hex()
        splits = num_splits or 8
        self.dec_attn = ops.DecodeAttention(hq_loc, hkv_loc, cfg.head_dim, max_batch, splits, self.device)
        # shared-prefix decode: rows that share context keys (mounted task prefix, forked parent)
        # gather them once per group; re-planned per decode call (graph-safe tables)
        self.shared_decode = None
        self._shared_active = False
        self._filter = (1.0, 0)  # the batch's (top_p, top_k)
        self._use_radix = True   # prefix reuse across requests (hybrid models: off, their states are per cursor)
        if (self.device.type == "cuda" and cfg.head_dim == 128 and self.mount_layers is None
                and os.environ.get("OCTO_SHARED_DECODE", "1") != "0"):
            self.shared_decode = ops.SharedDecode(hq_loc, hkv_loc, cfg.head_dim, max_batch, self.device)
        # static decode buffers (graph inputs)
        B = max_batch
        dev = self.device
        self.s_tok = torch.zeros(B, dtype=torch.int64, device=dev)
        self.s_pos = torch.zeros(B, dtype=torch.int32, device=dev)
        self.s_start = torch.zeros(B, dtype=torch.int32, device=dev)
        self.s_len = torch.zeros(B, dtype=torch.int32, device=dev)
        self.s_start_own = torch.zeros(B, dtype=torch.int32, device=dev)
        self.s_len_own = torch.zeros(B, dtype=torch.int32, device=dev)
        self.s_stream = torch.zeros(B, dtype=torch.int64, device=dev)
        self.s_step = torch.zeros(1, dtype=torch.int64, device=dev)
        self.kv_index_capacity = kv_index_capacity
        self.kv_indices = torch.zeros(kv_index_capacity, dtype=torch.int32, device=dev)
        self.kv_indices_own = torch.zeros(kv_index_capacity if self.mount_layers is not None else 1,
                                          dtype=torch.int32, device=dev)
        self.max_steps = 0
        self.s_out_tok = None
        self.s_out_lp = None
        self._graphs: dict[int, torch.cuda.CUDAGraph] = {}
        self._graph_kernels: dict = {}
        self._graph_pool = None
        self._graph_steps = 0
        self.stats = {"prefill_tokens": 0, "cached_tokens": 0, "decode_steps": 0, "requests": 0,
                      "prefill_s": 0.0, "decode_s": 0.0}
        # interaction records for training (reply id -> tokens, completion range, behaviour
        # logprobs, mounts, weight version); enabled by `record_interactions = True`
        self.record_interactions = False
        self.records: dict[str, dict] = {}

    # ------------------------------------------------------------------ helpers
    def _mount_rows(self, inp, ctx_t, ctx_s, ctx_p, ctx_m, mount_at, extra, next_pos: int) -> int:
        """Append the rows of inp.mount to the context lists under inp.mount_rule; returns
        the request's next position."""
        for (src, a, b) in inp.mount:
            mount_at.append(sum(len(x) for x in ctx_t))
            sc = self.cursors.get(src)
            if sc is None:
                raise CursorNotFound(src)
            if sc.meta.get("spilled"):
                self._rebuild(src)
            a, b = int(a), int(b)
            if not (0 <= a < b <= sc.length) or (sc.slots[a:b] < 0).any():
                raise ValueError(f"mount range [{a}, {b}) invalid for cursor {src} of length {sc.length}")
            rule = inp.mount_rule
            if rule not in ("K1", "K2", "K3"):
                raise ValueError(f"unknown mount rule {rule!r} (K1, K2, K3)")
            ctx_t.append(np.full(b - a, PLACEHOLDER, np.int32))
            ctx_m.append(np.ones(b - a, dtype=bool))
            if rule == "K3":
                pos = next_pos + np.arange(b - a, dtype=np.int64)
                ctx_s.append(self._relocated(sc.slots[a:b], pos - sc.positions[a:b], extra))
                ctx_p.append(pos)
                next_pos += b - a
                continue
            ctx_s.append(sc.slots[a:b])
            ctx_p.append(sc.positions[a:b])
            if rule == "K2":
                next_pos = max(next_pos, int(sc.positions[b - 1]) + 1)
        return next_pos

    def _relocated(self, src: np.ndarray, delta: np.ndarray, owned: list) -> np.ndarray:
        """Copies of KV slots `src` in every layer with the keys re-rotated by `delta`
        positions (rotary angles add: R(p + d) = R(d) R(p)); the new slots are appended to
        `owned` (the request holds one reference until it ends)."""
        new = self._alloc(len(src))
        owned.append(new)
        cfg = self.cfg
        _, hkv = self._local_heads()
        dev = self.kc.device
        si = torch.as_tensor(np.asarray(src, np.int64), device=dev)
        ni = torch.as_tensor(np.asarray(new, np.int64), device=dev)
        d = torch.as_tensor(np.asarray(delta, np.int32), device=dev)
        for layer in range(cfg.layers):
            k = self.kc[layer].index_select(0, si)
            sv.rope_(k, d, 0, hkv, cfg.head_dim, cfg.rope_theta)
            self.kc[layer].index_copy_(0, ni, k)
            self.vc[layer].index_copy_(0, ni, self.vc[layer].index_select(0, si))
        return new

    def _local_heads(self) -> tuple[int, int]:
        """(query heads, KV heads) this process computes and caches."""
        return self.cfg.heads, self.cfg.kv_heads

    def _pad_rows(self, T: int) -> int:
        """Rows a prefill forward of T tokens is padded to."""
        return (T + 7) // 8 * 8

    def new_cursor_id(self) -> str:
        # unique across engines (clients route by cursor id over a pool of servers)
        return f"c{self._uid}-{next(self._cid)}"

    def _alloc(self, n: int) -> np.ndarray:
        if n == 0:
            return np.empty(0, np.int64)
        s = self.pool.alloc(n)
        if len(s) < n:
            self.radix.evict(n - self.pool.free_count() + 1024)
            s = self.pool.alloc(n)
            if len(s) < n:
                self._spill(n)
                s = self.pool.alloc(n)
                if len(s) < n:
                    raise OutOfKV(f"KV pool exhausted: need {n}, free {self.pool.free_count()}")
        return np.asarray(s, dtype=np.int64)

    # ------------------------------------------------------------------ KV pressure: spill / rebuild
    _spillable = True  # (the hybrid engine's cursors also carry recurrent states: not spilled)

    def _spill(self, need: int) -> int:
        """Drop the KV of least-recently-used cursors until `need` slots are free.  A spilled
        cursor keeps its tokens, positions and recipe (the requests that built it); the
        next request that continues or mounts it rebuilds its KV first (_rebuild).  Slots a
        running request or another holder still references are not freed by a spill.
        Returns the number of cursors spilled."""
        if not self._spillable:
            return 0
        spilled = 0
        for cid in self.cursors.oldest_first():
            if self.pool.free_count() >= need:
                break
            cur = self.cursors.peek(cid)
            if cur is None or cur.meta.get("spilled") or cur.meta.get("recipe") is None:
                continue
            held = cur.held_slots()
            if not len(held):
                continue
            cur.meta["spilled"] = True
            cur.meta["kv_rows"] = int(np.argmin(cur.slots >= 0)) if not (cur.slots >= 0).all() else cur.length
            cur.slots = np.full(cur.length, -1, np.int64)
            self.pool.decref(held)
            spilled += 1
        self.stats["spills"] = self.stats.get("spills", 0) + spilled
        return spilled

    def _rebuild(self, cid: str, depth: int = 0) -> None:
        """Recompute a spilled cursor's KV by replaying its recipe as prefill-only requests
        with the same tokens, mounts and mount rules (hence the same K2 positions); mount
        sources that are spilled themselves are rebuilt first."""
        cur = self.cursors.peek(cid)
        if cur is None:
            raise CursorNotFound(cid)
        if not cur.meta.get("spilled"):
            return
        if depth > 64:
            raise RuntimeError(f"cursor {cid}: rebuild recursion too deep")
        recording, self.record_interactions = self.record_interactions, False
        tmp_ids, prev, mounts = [], None, []
        try:
            for seg in cur.meta["recipe"]:
                if seg[0] == "mount":
                    self._rebuild(seg[1], depth + 1)
                    mounts.append(seg)
                    continue
                tid = f"{cid}#rebuild{len(tmp_ids)}"
                rule = mounts[0][4] if mounts else "K2"
                self.generate([GenInput(list(seg[1]), cursor=prev, mount=[m[1:4] for m in mounts], mount_rule=rule,
                                        max_new_tokens=0, prefill_only=True, cursor_id=tid)])
                tmp_ids.append(tid)
                prev, mounts = tid, []
            built = self.cursors.peek(prev) if prev is not None else None
            n = cur.meta.get("kv_rows", cur.length)
            if built is None or built.length != n or not np.array_equal(built.tokens, cur.tokens[:n]) or \
                    not np.array_equal(built.positions, cur.positions[:n]):
                raise RuntimeError(f"cursor {cid}: its recipe does not rebuild its rows")
            slots = built.slots.copy()
            self.pool.incref(slots[slots >= 0])
            cur.slots = np.concatenate([slots, np.full(cur.length - n, -1, np.int64)])
            cur.meta["spilled"] = False
            self.stats["rebuilds"] = self.stats.get("rebuilds", 0) + 1
        finally:
            self.record_interactions = recording
            for tid in tmp_ids:
                self.cursors.pop(tid)

    def bump_version(self) -> int:
        """New weight version: cached KV of older versions is no longer matched."""
        self.version += 1
        return self.version

    # ------------------------------------------------------------------ request setup
    def _resolve(self, inp: GenInput) -> _Req:
        rid = inp.rid if inp.rid is not None else next(self._rid)
        new = np.asarray(inp.input_ids, dtype=np.int32)
        ctx_t, ctx_s, ctx_p, ctx_m = [], [], [], []
        next_pos = 0
        cached = 0
        handle = -1
        if inp.cursor is not None:
            cur = self.cursors.get(inp.cursor)
            if cur is None:
                raise CursorNotFound(inp.cursor)
            if cur.meta.get("spilled"):
                self._rebuild(inp.cursor)
            # rows without KV (a template terminator appended at put) are re-prefilled
            has_kv = cur.slots >= 0
            ok = int(np.argmin(has_kv)) if not has_kv.all() else cur.length
            ctx_t.append(cur.tokens[:ok])
            ctx_s.append(cur.slots[:ok])
            ctx_p.append(cur.positions[:ok])
            ctx_m.append(cur.mounted[:ok])
            if ok < cur.length:
                new = np.concatenate([cur.tokens[ok:], new])
            next_pos = int(cur.positions[ok - 1]) + 1 if ok else 0
            cached = ok
        elif len(new) > 1 and self._use_radix and not inp.mount:
            # (a request that mounts puts the mounted rows before its prompt, so its prompt
            # is not a prefix of the cached sequences)
            ln, slots, handle = self.radix.match(self.version, new[:-1])
            ln = int(ln)
            if ln > 0:
                ctx_t.append(new[:ln])
                ctx_s.append(np.asarray(slots, np.int64))
                ctx_p.append(np.arange(ln, dtype=np.int64))
                ctx_m.append(np.zeros(ln, dtype=bool))
                new = new[ln:]
                next_pos = ln
                cached = ln
                self.radix.lock(handle)
            else:
                self.radix.release_handle(handle)
                handle = -1
        # mounts: splice rows of other cursors (K2: next = max(own next, last mounted + 1))
        mount_at, extra = [], []
        try:
            next_pos = self._mount_rows(inp, ctx_t, ctx_s, ctx_p, ctx_m, mount_at, extra, next_pos)
        except Exception:
            for ex in extra:  # K3 copies made before the failing mount
                self.pool.decref(ex)
            if handle >= 0:
                self.radix.unlock(handle)
                self.radix.release_handle(handle)
            raise
        cat = (lambda xs, dt: np.concatenate(xs).astype(dt) if xs else np.empty(0, dt))
        r = _Req(inp, rid, cat(ctx_t, np.int32), cat(ctx_s, np.int64), cat(ctx_p, np.int64), cat(ctx_m, bool), new,
                 next_pos, cached=cached, radix_handle=handle)
        r.mount_at = mount_at
        r.extra_slots = extra
        if len(new) == 0:
            self._abandon(r)
            raise ValueError("request has no new tokens to prefill")
        if len(r.ctx_slots):  # pin the context: spills during this request cannot free it
            self.pool.incref(r.ctx_slots)
            r.pinned = True
        return r

    # ------------------------------------------------------------------ model-family hooks
    def _prefill_group(self, reqs, g, cu_q):
        """Before one prefill forward of requests g (rows cu_q, padding after the last)."""

    def _prefill_group_done(self, reqs, g):
        """After that forward."""

    def _decode_begin(self, reqs, chunk, B: int, steps: int):
        """Before the decode steps of requests `chunk` (rows 0..len-1 of a B-row batch)."""

    def _decode_end(self, reqs, chunk):
        """After them."""

    def _on_cursor(self, r, cid: str):
        """A request's reply was stored as cursor `cid`."""

    # ------------------------------------------------------------------ forward pieces
    def _layer(self, x, i, pos, write_slots, attn):
        cfg, w = self.cfg, self.w
        ln1, qkv_w, qkv_b, o_w, ln2, gu_w, down_w = w.layer(i)
        h = sv.rms(x, ln1, cfg.rms_eps, cfg.norm_plus_one)
        qkv = ops.gemm(h, qkv_w, bias=qkv_b).to(x.dtype)
        sv.rope_(qkv, pos, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.rope_theta)
        sv.kv_write(qkv, cfg.heads, cfg.kv_heads, cfg.head_dim, write_slots, self.kc[i], self.vc[i])
        o = attn(qkv[:, : cfg.q_width], i)
        x = ops.gemm(o, o_w, residual=x).to(x.dtype)
        h2 = sv.rms(x, ln2, cfg.rms_eps, cfg.norm_plus_one)
        act = ops.gemm_swiglu(h2, gu_w)
        return ops.gemm(act, down_w, residual=x).to(x.dtype)

    def _layer_decode(self, x, h, i, pos, slots, attn):
        """One decode layer on (x, h = RMSNorm_ln1(x)); returns (x, the next layer's normed
        input) with the projections fused into their neighbours (rotary + KV write into the
        qkv finish, residual + next norm into the o / down finishes)."""
        cfg, w = self.cfg, self.w
        _, qkv_w, qkv_b, o_w, ln2, gu_w, down_w = w.layer(i)
        nxt = w.layer(i + 1)[0] if i + 1 < cfg.layers else w["norm"]
        q = sv.qkv_rope_kv(h, qkv_w, qkv_b, pos, cfg.rope_theta, cfg.heads, cfg.kv_heads, cfg.head_dim, slots,
                           self.kc[i], self.vc[i])
        o = attn(q, i)
        x, h2 = sv.gemm_res_norm(o, o_w, x, ln2, cfg.rms_eps, cfg.norm_plus_one)
        act = ops.gemm_swiglu(h2, gu_w)  # gate / up GEMM with the activation in its epilogue
        return sv.gemm_res_norm(act, down_w, x, nxt, cfg.rms_eps, cfg.norm_plus_one)

    def _final(self, x):
        return sv.rms(x, self.w["norm"], self.cfg.rms_eps, self.cfg.norm_plus_one)

    # ------------------------------------------------------------------ prefill
    def _prefill(self, reqs: list[_Req], temperature: float):
        """Ragged forward of all new tokens; returns first sampled (tokens, logprobs)."""
        cfg = self.cfg
        dev = self.device
        first_tok = np.zeros(len(reqs), np.int64)
        first_lp = np.zeros(len(reqs), np.float32)
        # chunk requests so one forward holds <= prefill_chunk tokens
        groups, cur, cur_n = [], [], 0
        for j, r in enumerate(reqs):
            n = len(r.new_tokens)
            if cur and cur_n + n > self.prefill_chunk:
                groups.append(cur)
                cur, cur_n = [], 0
            cur.append(j)
            cur_n += n
        if cur:
            groups.append(cur)
        for g in groups:
            ids, pos, slots, cu_q, cu_k, keys, cu_k_own, keys_own, last = [], [], [], [0], [0], [], [0], [], []
            for j in g:
                r = reqs[j]
                n = len(r.new_tokens)
                ids.append(r.new_tokens)
                pos.append(np.arange(r.first_pos, r.first_pos + n))
                own = r.own_slots[:n]
                slots.append(own)
                kk = np.concatenate([r.ctx_slots, own])
                keys.append(kk)
                cu_q.append(cu_q[-1] + n)
                cu_k.append(cu_k[-1] + len(kk))
                if self.mount_layers is not None:
                    ko = np.concatenate([r.ctx_slots[~r.ctx_mounted], own])
                    keys_own.append(ko)
                    cu_k_own.append(cu_k_own[-1] + len(ko))
                last.append(cu_q[-1] - 1)
            T = cu_q[-1]
            pad = self._pad_rows(T) - T
            if pad:
                ids.append(np.zeros(pad, np.int32))
                pos.append(np.zeros(pad, np.int64))
                slots.append(np.full(pad, self.null_slot, np.int64))
                keys.append(np.full(pad, self.null_slot, np.int64))
                cu_q.append(cu_q[-1] + pad)
                cu_k.append(cu_k[-1] + pad)
                if self.mount_layers is not None:
                    keys_own.append(np.full(pad, self.null_slot, np.int64))
                    cu_k_own.append(cu_k_own[-1] + pad)
            t_ids = h2d(np.concatenate(ids).astype(np.int64), dev)
            t_pos = h2d(np.concatenate(pos).astype(np.int32), dev)
            t_slots = h2d(np.concatenate(slots).astype(np.int64), dev)
            plan = ops.AttnPlan.build(cu_q, cu_k, np.concatenate(keys).astype(np.int32), dev)
            plan_own = plan if self.mount_layers is None else ops.AttnPlan.build(
                cu_q, cu_k_own, np.concatenate(keys_own).astype(np.int32), dev)
            mset = set(self.mount_layers or [])
            scale = cfg.head_dim ** -0.5
            hq, hkv = self._local_heads()

            def attn(q, i):
                p = plan if (self.mount_layers is None or i in mset) else plan_own
                return sv.prefill_attn(q, self.kc[i], self.vc[i], p, hq, hkv, cfg.head_dim, scale)

            streams = np.asarray([(reqs[j].rid << 32) | (reqs[j].first_pos + len(reqs[j].new_tokens)) for j in g],
                                 np.int64)
            self._prefill_group(reqs, g, cu_q)
            tok, lp = self._prefill_forward(t_ids, t_pos, t_slots, attn, np.asarray(last, np.int64), streams,
                                            temperature)
            self._prefill_group_done(reqs, g)
            for k, j in enumerate(g):
                first_tok[j] = tok[k]
                first_lp[j] = lp[k]
            self.stats["prefill_tokens"] += T
        return first_tok, first_lp

    def _prefill_forward(self, t_ids, t_pos, t_slots, attn, last: np.ndarray, streams: np.ndarray,
                         temperature: float):
        """Forward of a padded prefill batch; samples the rows `last`; host (tokens, logprobs)."""
        cfg, dev = self.cfg, self.device
        x = sv.embed(t_ids, self.w["embed"])
        for i in range(cfg.layers):
            x = self._layer(x, i, t_pos, t_slots, attn)
        h = self._final(x.index_select(0, h2d(last, dev)))
        tp_, tk_ = self._filter
        tok, lp = ops.sample(h, self.w.head, temperature, self.seed, h2d(streams, dev), cfg.vocab_size, tp_, tk_)
        return d2h(tok).numpy(), d2h(lp).numpy()

    def _decode_forward(self, tok, pos, slot, attn, B: int, temperature: float):
        """One decode forward of B rows; returns device (tokens, logprobs)."""
        cfg = self.cfg
        x = sv.embed(tok, self.w["embed"])
        h = sv.rms(x, self.w.layer(0)[0], cfg.rms_eps, cfg.norm_plus_one)
        for i in range(cfg.layers):
            x, h = self._layer_decode(x, h, i, pos, slot, attn)
        # (h is the final norm's output)
        tp_, tk_ = self._filter
        return ops.sample(h, self.w.head, temperature, self.seed, self.s_stream[:B], cfg.vocab_size, tp_, tk_)

    # ------------------------------------------------------------------ decode
    def _decode_step(self, B: int, temperature: float):
        cfg = self.cfg
        tok = self.s_tok[:B]
        pos = self.s_pos[:B]
        start = self.s_start[:B]
        ln = self.s_len[:B]
        slot = self.kv_indices.index_select(0, (start + ln).long()).long()
        att_len = ln + 1
        mset = set(self.mount_layers or [])
        if self.mount_layers is not None:
            start_o = self.s_start_own[:B]
            len_o = self.s_len_own[:B] + 1

        def attn(q, i):
            if self._shared_active:
                return self.shared_decode(q, self.kc[i], self.vc[i], self.kv_indices, att_len)
            if self.mount_layers is None or i in mset:
                return self.dec_attn(q, self.kc[i], self.vc[i], start, self.kv_indices, kv_len=att_len)
            return self.dec_attn(q, self.kc[i], self.vc[i], start_o, self.kv_indices_own, kv_len=len_o)

        if self.device.type == "cuda":
            with ops.pdl_launches():
                new_tok, lp = self._decode_forward(tok, pos, slot, attn, B, temperature)
        else:
            new_tok, lp = self._decode_forward(tok, pos, slot, attn, B, temperature)
        step = self.s_step.expand(B)[:, None]
        self.s_out_tok[:B].scatter_(1, step, new_tok[:, None])
        self.s_out_lp[:B].scatter_(1, step, lp[:, None])
        self.s_tok[:B].copy_(new_tok)
        self.s_pos[:B].add_(1)
        self.s_len[:B].add_(1)
        if self.mount_layers is not None:
            self.s_len_own[:B].add_(1)
        self.s_stream[:B].add_(1)
        self.s_step.add_(1)

    def _bucket(self, n: int) -> int:
        b = self._min_bucket()
        while b < n:
            b *= 2
        return min(b, self.max_batch)

    def _min_bucket(self) -> int:
        return 8

    def _ensure_out(self, steps: int):
        if self.s_out_tok is None or self.s_out_tok.shape[1] < steps:
            # (re)allocating invalidates captured graphs
            self.s_out_tok = torch.zeros(self.max_batch, steps, dtype=torch.int64, device=self.device)
            self.s_out_lp = torch.zeros(self.max_batch, steps, dtype=torch.float32, device=self.device)
            self._graphs.clear()

    def _graph_key(self, B: int, temperature: float):
        return (B, float(temperature), self._shared_active, self._filter)

    def _graph(self, B: int, temperature: float):
        key = self._graph_key(B, temperature)
        g = self._graphs.get(key)
        if g is not None:
            return g
        # warm up on a side stream, then capture
        saved = [t.clone() for t in (self.s_tok, self.s_pos, self.s_len, self.s_len_own, self.s_stream,
                                     self.s_step)]
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            for _ in range(2):
                self._decode_step(B, temperature)
        torch.cuda.current_stream(self.device).wait_stream(s)
        for t, v in zip((self.s_tok, self.s_pos, self.s_len, self.s_len_own, self.s_stream, self.s_step), saved):
            t.copy_(v)
        if self._graph_pool is None:
            self._graph_pool = torch.cuda.graph_pool_handle()
        g = torch.cuda.CUDAGraph()
        n0 = ops.launches()
        with torch.cuda.graph(g, pool=self._graph_pool):
            self._decode_step(B, temperature)
        self._graph_kernels[key] = ops.launches() - n0
        for t, v in zip((self.s_tok, self.s_pos, self.s_len, self.s_len_own, self.s_stream, self.s_step), saved):
            t.copy_(v)
        self._graphs[key] = g
        return g

    def _decode(self, reqs: list[_Req], first_tok, steps: int, temperature: float):
        """Run `steps` decode steps for all requests (batched in buckets of max_batch)."""
        if steps <= 0:
            return np.zeros((len(reqs), 0), np.int64), np.zeros((len(reqs), 0), np.float32)
        out_t = np.zeros((len(reqs), steps), np.int64)
        out_l = np.zeros((len(reqs), steps), np.float32)
        self._ensure_out(steps)
        for b0 in range(0, len(reqs), self.max_batch):
            chunk = list(range(b0, min(len(reqs), b0 + self.max_batch)))
            n = len(chunk)
            B = self._bucket(n)
            # lay out kv index regions: [ctx slots | own slots (new + generated)]
            regions, off = [], 0
            starts = np.zeros(B, np.int32)
            lens = np.zeros(B, np.int32)
            starts_o = np.zeros(B, np.int32)
            lens_o = np.zeros(B, np.int32)
            regions_o, off_o = [], 0
            for k, j in enumerate(chunk):
                r = reqs[j]
                full = np.concatenate([r.ctx_slots, r.own_slots])
                regions.append(full)
                starts[k] = off
                lens[k] = len(r.ctx_slots) + len(r.new_tokens)
                off += len(full)
                if self.mount_layers is not None:
                    fo = np.concatenate([r.ctx_slots[~r.ctx_mounted], r.own_slots])
                    regions_o.append(fo)
                    starts_o[k] = off_o
                    lens_o[k] = int((~r.ctx_mounted).sum()) + len(r.new_tokens)
                    off_o += len(fo)
            # padding rows: a region of one null slot each
            for k in range(n, B):
                regions.append(np.full(1 + steps, self.null_slot, np.int64))
                starts[k] = off
                lens[k] = 0
                off += 1 + steps
                if self.mount_layers is not None:
                    regions_o.append(np.full(1 + steps, self.null_slot, np.int64))
                    starts_o[k] = off_o
                    off_o += 1 + steps
            if off > self.kv_index_capacity:
                raise OutOfKV("kv index capacity exceeded; lower the batch or raise kv_index_capacity")
            dev = self.device
            self.kv_indices[:off].copy_(h2d(np.concatenate(regions).astype(np.int32), dev))
            if self.mount_layers is not None:
                self.kv_indices_own[:off_o].copy_(h2d(np.concatenate(regions_o).astype(np.int32), dev))
                self.s_start_own[:B].copy_(h2d(starts_o, dev))
                self.s_len_own[:B].copy_(h2d(lens_o, dev))
            tok = np.zeros(B, np.int64)
            pos = np.zeros(B, np.int32)
            stream = np.zeros(B, np.int64)
            for k, j in enumerate(chunk):
                r = reqs[j]
                tok[k] = first_tok[j]
                p = r.first_pos + len(r.new_tokens)
                pos[k] = p
                stream[k] = (r.rid << 32) | (p + 1)
            self.s_tok[:B].copy_(h2d(tok, dev))
            self.s_pos[:B].copy_(h2d(pos, dev))
            self.s_start[:B].copy_(h2d(starts, dev))
            self.s_len[:B].copy_(h2d(lens, dev))
            self.s_stream[:B].copy_(h2d(stream, dev))
            self.s_step.zero_()
            if self.shared_decode is not None:
                ctx = np.asarray([len(reqs[j].ctx_slots) for j in chunk], np.int64)
                self._shared_active = self.shared_decode.plan(regions[:n], starts, ctx, lens[:n] + steps + 1, B)
            self._decode_begin(reqs, chunk, B, steps)
            if self.use_graphs:
                g = self._graph(B, temperature)
                for _ in range(steps):
                    g.replay()
                ops.add_launches(self._graph_kernels[self._graph_key(B, temperature)] * steps)
            else:
                for _ in range(steps):
                    self._decode_step(B, temperature)
            self._decode_end(reqs, chunk)
            ot = d2h(self.s_out_tok[:n, :steps]).numpy()
            ol = d2h(self.s_out_lp[:n, :steps]).numpy()
            out_t[b0:b0 + n] = ot
            out_l[b0:b0 + n] = ol
            self.stats["decode_steps"] += steps
        return out_t, out_l

    # ------------------------------------------------------------------ continuous batching
    # (serving.scheduler drives these: requests join after a prefill, decode in chunks of a
    # few steps together with every live request, and leave when they stop)
    @property
    def supports_continuous(self) -> bool:
        return self.mount_layers is None  # layer-subset mounts keep a second key list per row

    @torch.no_grad()
    def admit(self, inputs: list[GenInput]) -> list:
        """Resolve, allocate and prefill `inputs` (one sampling setting); per input either a
        live request (its first sampled token in out_tok / out_lp) or the exception that
        failed it alone (unknown cursor, bad mount, no KV room)."""
        live, out = [], []
        for inp in inputs:
            try:
                r = self._resolve(inp)
            except Exception as e:  # noqa: BLE001  (this request fails, the others go on)
                out.append(e)
                continue
            try:
                r.own_slots = self._alloc(len(r.new_tokens) + (0 if inp.prefill_only else inp.max_new_tokens))
            except OutOfKV as e:
                self._abandon(r)
                out.append(e)
                continue
            live.append(r)
            out.append(r)
        if live:
            self._filter = (float(live[0].inp.top_p), int(live[0].inp.top_k))
            t0 = time.perf_counter()
            tok, lp = self._prefill(live, live[0].inp.temperature)
            self.stats["prefill_s"] += time.perf_counter() - t0
            for r, a, b in zip(live, tok, lp):
                r.out_tok, r.out_lp = [int(a)], [float(b)]
        return out

    def _abandon(self, r: _Req):
        """Release what a resolved request holds when it does not run to the end."""
        if r.pinned:
            self.pool.decref(r.ctx_slots)
            r.pinned = False
        if r.own_slots is not None and len(r.own_slots):
            self.pool.decref(r.own_slots)
            r.own_slots = None
        for ex in r.extra_slots:
            self.pool.decref(ex)
        r.extra_slots = []
        if r.radix_handle >= 0:
            self.radix.unlock(r.radix_handle)
            self.radix.release_handle(r.radix_handle)
            r.radix_handle = -1

    def layout_rows(self, rows: list[_Req], tail: int) -> int:
        """Place live requests in decode rows 0..n-1 of a batch bucket for the next decode
        chunks of at most `tail` steps: each row's key list is [context | own slots | tail
        null slots] (steps past a request's end write the null slot) and its state continues
        from its last sampled token.  Returns the bucket size B."""
        n = len(rows)
        B = self._bucket(n)
        regions, off = [], 0
        starts, lens = np.zeros(B, np.int32), np.zeros(B, np.int32)
        tok, pos, stream = np.zeros(B, np.int64), np.zeros(B, np.int32), np.zeros(B, np.int64)
        final = np.zeros(n, np.int64)
        for k, r in enumerate(rows):
            g = len(r.out_tok)
            region = np.concatenate([r.ctx_slots, r.own_slots, np.full(tail, self.null_slot, np.int64)])
            regions.append(region)
            starts[k] = off
            lens[k] = len(r.ctx_slots) + len(r.new_tokens) + g - 1
            off += len(region)
            tok[k] = r.out_tok[-1]
            pos[k] = r.first_pos + len(r.new_tokens) + g - 1
            stream[k] = (r.rid << 32) | (int(pos[k]) + 1)
            final[k] = len(r.ctx_slots) + len(r.new_tokens) + r.inp.max_new_tokens + 1  # (steps past it: discarded)
        for k in range(n, B):
            regions.append(np.full(1 + tail, self.null_slot, np.int64))
            starts[k] = off
            off += 1 + tail
        if off > self.kv_index_capacity:
            raise OutOfKV("kv index capacity exceeded; lower the batch or raise kv_index_capacity")
        dev = self.device
        self.kv_indices[:off].copy_(h2d(np.concatenate(regions).astype(np.int32), dev))
        for dst, src in ((self.s_start, starts), (self.s_len, lens), (self.s_tok, tok), (self.s_pos, pos),
                         (self.s_stream, stream)):
            dst[:B].copy_(h2d(src, dev))
        self._shared_active = False
        if self.shared_decode is not None:
            ctx = np.asarray([len(r.ctx_slots) for r in rows], np.int64)
            self._shared_active = self.shared_decode.plan(regions[:n], starts, ctx, final, B)
        return B

    @torch.no_grad()
    def decode_chunk(self, n: int, B: int, steps: int, temperature: float) -> tuple[np.ndarray, np.ndarray]:
        """`steps` decode steps of the laid-out batch; host (tokens, logprobs) [n, steps]."""
        self._ensure_out(steps)
        self.s_step.zero_()
        # padding rows restart at their null region each chunk (their key count would
        # otherwise grow past it when a layout is reused for several chunks)
        self.s_len[n:B].zero_()
        t0 = time.perf_counter()
        if self.use_graphs:
            g = self._graph(B, temperature)
            for _ in range(steps):
                g.replay()
            ops.add_launches(self._graph_kernels[self._graph_key(B, temperature)] * steps)
        else:
            for _ in range(steps):
                self._decode_step(B, temperature)
        out_t = d2h(self.s_out_tok[:n, :steps]).numpy()
        out_l = d2h(self.s_out_lp[:n, :steps]).numpy()
        self.stats["decode_s"] += time.perf_counter() - t0
        self.stats["decode_steps"] += steps
        return out_t, out_l

    def finish(self, r: _Req) -> GenOutput:
        """Close a live request with what it generated (at most max_new_tokens)."""
        mx = 0 if r.inp.prefill_only else r.inp.max_new_tokens
        return self._finish(r, r.out_tok[:mx], r.out_lp[:mx])

    # ------------------------------------------------------------------ public API
    @torch.no_grad()
    def generate(self, inputs: list[GenInput]) -> list[GenOutput]:
        """Prefill + decode a batch of requests (all share the batch temperature)."""
        if not inputs:
            return []
        temperature = inputs[0].temperature
        self._filter = (float(inputs[0].top_p), int(inputs[0].top_k))
        reqs = [self._resolve(inp) for inp in inputs]
        for r in reqs:
            r.own_slots = self._alloc(len(r.new_tokens) + (0 if r.inp.prefill_only else r.inp.max_new_tokens))
        t0 = time.perf_counter()
        first_tok, first_lp = self._prefill(reqs, temperature)
        t1 = time.perf_counter()
        self.stats["prefill_s"] += t1 - t0
        max_new = max((0 if r.inp.prefill_only else r.inp.max_new_tokens) for r in reqs)
        out_t, out_l = self._decode(reqs, first_tok, max_new - 1, temperature)
        self.stats["decode_s"] += time.perf_counter() - t1
        outs = []
        for j, r in enumerate(reqs):
            mx = 0 if r.inp.prefill_only else r.inp.max_new_tokens
            toks = ([int(first_tok[j])] + [int(x) for x in out_t[j]])[:mx]
            lps = ([float(first_lp[j])] + [float(x) for x in out_l[j]])[:mx]
            outs.append(self._finish(r, toks, lps))
        return outs

    @staticmethod
    def _cut_at_stop(inp: GenInput, toks: list, lps: list) -> tuple[list, list, str]:
        """Tokens through the first stop token (finish reason "stop"), else all ("length")."""
        if inp.stop_ids:
            for k, t in enumerate(toks):
                if t in inp.stop_ids:
                    return toks[:k + 1], lps[:k + 1], "stop"
        return toks, lps, "length"

    def _recipe(self, r: _Req, gen_kv: list):
        """How to recompute this request's cursor rows with KV: its parent's recipe (a cursor
        continuation) or its radix prefix, its mounts, then its prompt and generated tokens.
        None when the parent cannot be rebuilt."""
        inp = r.inp
        if inp.cursor is not None:
            parent = self.cursors.peek(inp.cursor)
            base = None if parent is None else parent.meta.get("recipe")
            if base is None:
                return None
            steps = list(base)
        elif r.cached:
            steps = [("tokens", np.asarray(r.ctx_tokens[:r.cached], np.int32))]
        else:
            steps = []
        steps += [("mount", src, int(a), int(b), inp.mount_rule) for src, a, b in inp.mount]
        steps.append(("tokens", np.concatenate([r.new_tokens, np.asarray(gen_kv, np.int32)]).astype(np.int32)))
        return steps

    def _finish(self, r: _Req, toks: list, lps: list) -> GenOutput:
        """Close one request: cut at its stop token, keep its reply as a cursor (or release
        its slots), insert its prompt into the radix cache, record the interaction."""
        toks, lps, reason = self._cut_at_stop(r.inp, toks, lps)
        n_new = len(r.new_tokens)
        # generated rows with KV: all but the last sampled token (its KV is not written)
        n_kv_gen = max(0, len(toks) - 1)
        used = n_new + n_kv_gen
        cid = None
        if r.inp.keep_cursor:
            cid = r.inp.cursor_id or self.new_cursor_id()
            gen_pos = np.arange(r.first_pos + n_new, r.first_pos + n_new + len(toks))
            slots = np.concatenate([r.ctx_slots, r.own_slots[:used], np.full(len(toks) - n_kv_gen, -1, np.int64)])
            cur = Cursor(cid, np.concatenate([r.ctx_tokens, r.new_tokens, np.asarray(toks, np.int32)]), slots,
                         np.concatenate([r.ctx_pos, np.arange(r.first_pos, r.first_pos + n_new), gen_pos]),
                         prompt_len=len(r.ctx_tokens) + n_new,
                         mounted=np.concatenate([r.ctx_mounted, np.zeros(n_new + len(toks), bool)]),
                         version=self.version)
            cur.meta["recipe"] = self._recipe(r, toks[:n_kv_gen])
            # the store's reference: the request's pin on the ctx slots and its used own slots
            # move to the cursor
            self.cursors.put(cur, take_ref=False)
            self._on_cursor(r, cid)
            if len(r.ctx_slots) and not r.pinned:
                self.pool.incref(r.ctx_slots)
            r.pinned = False
        elif r.pinned:
            self.pool.decref(r.ctx_slots)
            r.pinned = False
        if r.inp.cursor is None and not r.inp.mount and len(r.new_tokens) and self._use_radix:
            full = np.concatenate([r.ctx_tokens, r.new_tokens]).astype(np.int32)
            sl = np.concatenate([r.ctx_slots, r.own_slots[:n_new]]).astype(np.int64)
            self.radix.insert(self.version, full, sl)
        # release what this request owns and did not hand to a cursor
        if not r.inp.keep_cursor:
            self.pool.decref(r.own_slots)
        elif len(r.own_slots) > used:
            self.pool.decref(r.own_slots[used:])
        for ex in r.extra_slots:  # K3 copies: a kept cursor holds its own reference
            self.pool.decref(ex)
        if r.radix_handle >= 0:
            self.radix.unlock(r.radix_handle)
            self.radix.release_handle(r.radix_handle)
        if self.record_interactions and cid is not None:
            prompt = np.concatenate([r.ctx_tokens, r.new_tokens]).astype(np.int32)
            self.records[cid] = {"tokens": np.concatenate([prompt, np.asarray(toks, np.int32)]),
                                 "prompt_len": len(prompt), "completion": len(toks),
                                 "logprobs": np.asarray(lps, np.float32), "parent": r.inp.cursor,
                                 "mounts": [(at, m[0], int(m[1]), int(m[2]))
                                            for at, m in zip(r.mount_at, r.inp.mount)],
                                 "version": self.version}
        self.stats["cached_tokens"] += r.cached
        self.stats["requests"] += 1
        return GenOutput(toks, lps, cid, n_new, r.cached, r.first_pos, reason)

    def release_cursor(self, cid: str):
        self.cursors.pop(cid)

    def extend_cursor(self, cid: str, tokens, drop_trailing=()) -> None:
        """Append tokens without KV yet (e.g. the template's turn terminator) to a cursor,
        after dropping trailing stop tokens that have no KV; the next continuation
        prefills them."""
        cur = self.cursors.get(cid)
        if cur is None:
            raise CursorNotFound(cid)
        n = cur.length
        drop = set(int(t) for t in drop_trailing)
        while n > 0 and int(cur.tokens[n - 1]) in drop and cur.slots[n - 1] < 0:
            n -= 1
        add = np.asarray(list(tokens), dtype=np.int32)
        last = int(cur.positions[n - 1]) if n else -1
        cur.tokens = np.concatenate([cur.tokens[:n], add])
        cur.slots = np.concatenate([cur.slots[:n], np.full(len(add), -1, np.int64)])
        cur.positions = np.concatenate([cur.positions[:n], np.arange(last + 1, last + 1 + len(add))])
        cur.mounted = np.concatenate([cur.mounted[:n], np.zeros(len(add), bool)])

    def reset(self):
        """Drop every cursor and cached prefix (KV memory returns to the pool)."""
        self.cursors.clear()
        self.radix.evict(1 << 62)

    def load_stats(self) -> dict:
        used = self.pool.used_count()
        return {"token_usage": used / self.kv_slots, "num_used_slots": used, "free_slots": self.pool.free_count(),
                "cursors": len(self.cursors), "cached_tokens": self.radix.cached_tokens(), **self.stats}
