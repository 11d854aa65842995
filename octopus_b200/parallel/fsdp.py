"""Sharded (FSDP / ZeRO) actor: optimizer state and fp32 master weights sharded over
ranks, bf16 compute weights replicated.

Each rank owns 1/W of the flat parameter buffer (contiguous shard; the layout pads
every unit so all shards are equal).  A training step:

1. forward/backward of the rank's micro-batches; wgrad GEMMs accumulate into the
   rank's full fp32 gradient buffer;
2. **fused reduce-scatter + grad-norm** (`rs_sum_sq`): the kernel reads the owned shard
   of every rank's gradient buffer over NVLink (peer loads), sums, writes the reduced
   fp32 shard and accumulates its squared norm; one scalar all-reduce gives the
   global norm (clip factor);
3. **fused AdamW + all-gather** (`adamw_bcast`): AdamW on the owned fp32 master/m/v
   shard, and each new bf16 weight is stored straight into the compute buffer of every
   rank (peer stores).  That compute buffer is also the colocated rollout engine's
   weight buffer, so this one kernel is the trainer -> rollout weight sync;
4. a bounded peer flag barrier so every rank sees all shards before the next use.

Buffers the kernels touch on peers (gradients, compute weights, barrier flags) are
cudaMalloc'd IPC buffers mapped into every rank.  Without peer memory (CPU / gloo, or
`fused=False`) the same step runs on NCCL/gloo collectives: reduce_scatter_tensor +
all_reduce(norm) + AdamW on the shard + all_gather_into_tensor — the baseline path.
Every rank issues the same collectives in the same order whatever its micro-batch
count (one scalar all-reduce for the loss denominator, then the step's collectives).

Reference parity: `octopus/rl/chunk_major.py:421-482` (FSDP2 gather/reduce once per
call), `octopus/rl/actor.py:332-341` (optimizer step), AReaL's clip + adam step.
"""
from __future__ import annotations

import functools
import math

import torch
import torch.distributed as dist

from .. import ops
from .peer import PeerBuffers  # noqa: F401  (re-exported: the sharded actors' IPC buffers)
from ..models.decoder import FlatLayout, Weights, init_flat
from ..rl.actor import Actor, OptimConfig
from ..rl.loss import PPOConfig, ppo_loss


class ShardedActor(Actor):
    def __init__(self, cfg, device="cuda", *, optim: OptimConfig | None = None, ppo: PPOConfig | None = None,
                 seed: int = 0, dtype=torch.bfloat16, ckpt: bool = True, temperature: float = 1.0, group=None,
                 fused: bool | None = None):
        self.cfg = cfg
        self.device = torch.device(device)
        self.optim = optim or OptimConfig()
        self.ppo = ppo or PPOConfig()
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.layout = FlatLayout(cfg, pad_multiple=self.world)
        total = self.layout.total
        assert total % (self.world * 8) == 0
        self.shard = total // self.world
        self.off = self.rank * self.shard
        self.fused = (self.device.type == "cuda") if fused is None else fused
        gdt = torch.float32 if dtype != torch.float64 else torch.float64
        if self.fused:
            self._grad_peers = PeerBuffers(total * 4, self.device, group)
            self._w_peers = PeerBuffers(total * 2, self.device, group)
            self._flags = PeerBuffers(64, self.device, group)
            self.grad = self._grad_peers.local.view(torch.float32)
            self.flat16 = self._w_peers.local.view(torch.bfloat16)
            self.flat16.copy_(init_flat(cfg, self.layout, self.device, dtype=dtype, seed=seed))
            self._barrier_seq = 0
        else:
            self.grad = torch.zeros(total, dtype=gdt, device=self.device)
            self.flat16 = init_flat(cfg, self.layout, self.device, dtype=dtype, seed=seed)
        self.master = self.flat16[self.off: self.off + self.shard].to(gdt).clone()
        self.exp_avg = torch.zeros_like(self.master)
        self.exp_avg_sq = torch.zeros_like(self.master)
        self.grad_shard = torch.zeros_like(self.master)
        self.weights = Weights(cfg, self.flat16, self.layout, self.grad)
        self.step_count = 0
        self.ckpt = ckpt
        self.temperature = temperature
        self.version = 0

    def forward_backward(self, mbs, denom=None):
        local = float(sum(mb.pair_w.sum() for mb in mbs))
        t = torch.tensor([local], dtype=torch.float64, device=self.device if self.device.type == "cuda" else "cpu")
        dist.all_reduce(t, group=self.group)
        return super().forward_backward(mbs, float(t))

    def _peer_barrier(self):
        self._barrier_seq += 1
        ops.ext().peer_barrier(self._flags.ptrs, self.rank, self._barrier_seq, self.device.index)

    def optimizer_step(self) -> torch.Tensor:
        self.step_count += 1
        o = self.optim
        sq = torch.zeros(1, dtype=torch.float32, device=self.device)
        if self.fused:
            C = ops.ext()
            self._peer_barrier()  # every rank's gradients are complete
            C.rs_sum_sq(self._grad_peers.ptrs, self.off, self.grad_shard, sq)
            dist.all_reduce(sq, group=self.group)
            self._peer_barrier()  # every rank finished reading peers' gradients (buffers may be reused)
            C.adamw_bcast(self.master, self.grad_shard, self.exp_avg, self.exp_avg_sq, self._w_peers.ptrs, self.off,
                          o.lr, o.betas[0], o.betas[1], o.eps, o.weight_decay, self.step_count, sq,
                          o.max_grad_norm, 1.0)
            self._peer_barrier()  # every rank's compute weights hold every new shard
        else:
            if self.grad.dtype == torch.float64 or self.device.type == "cpu":
                dist.reduce_scatter_tensor(self.grad_shard, self.grad, group=self.group)
            else:
                dist.reduce_scatter_tensor(self.grad_shard, self.grad, group=self.group)
            ops.sqnorm_(self.grad_shard, sq)
            dist.all_reduce(sq, group=self.group)
            shard16 = torch.empty(self.shard, dtype=self.flat16.dtype, device=self.device)
            ops.adamw_(self.master, self.grad_shard, self.exp_avg, self.exp_avg_sq, shard16, lr=o.lr,
                       betas=o.betas, eps=o.eps, weight_decay=o.weight_decay, step=self.step_count, sqnorm=sq,
                       max_norm=o.max_grad_norm)
            dist.all_gather_into_tensor(self.flat16, shard16, group=self.group)
        self.version += 1
        return sq

    def close(self):
        if self.fused:
            torch.cuda.synchronize(self.device)
            for b in (self._grad_peers, self._w_peers, self._flags):
                b.close()


# ============================================================================ full shard
class UnitShards:
    """Per-unit sharding of the flat layout over `world` ranks: rank r owns the r-th of
    `world` equal slices of every unit (units are padded to a multiple of world * 256
    elements), so each layer's parameters, gradients and optimizer state are split over
    all ranks and a layer is whole only while it is gathered."""

    def __init__(self, layout: FlatLayout, world: int, rank: int):
        self.layout, self.world, self.rank = layout, world, rank
        self.units = list(layout.units)
        self.size = [e - s for s, e in self.units]
        assert all(n % (world * 8) == 0 for n in self.size)
        self.su = [n // world for n in self.size]
        self.shard_off = [0]
        for n in self.su:
            self.shard_off.append(self.shard_off[-1] + n)
        self.total = self.shard_off[-1]

    def owned(self, u: int) -> slice:
        """This rank's slice of unit u in flat coordinates."""
        s = self.units[u][0] + self.rank * self.su[u]
        return slice(s, s + self.su[u])

    def local(self, u: int) -> slice:
        """Unit u's slice in the rank-local shard buffers."""
        return slice(self.shard_off[u], self.shard_off[u + 1])


class _StagedWeights(Weights):
    """Parameter views of the full-shard actor: a layer's views point into one of two
    rotating staging slots (layer i uses slot i % 2), the embedding and the final unit
    (norm + head) into staging of their own; every view's main_grad points into the
    matching gradient staging."""

    def __init__(self, cfg, layout: FlatLayout, wslots, gslots, edge_w: dict, edge_g: dict, full=None):
        # full: the complete bf16 flat buffer (the serving copy); when given, weight views point
        # into it and only the gradient views are staged
        self.cfg, self.layout, self.flat = cfg, layout, None
        self.t = {}
        last = len(layout.units) - 1
        for s in layout.specs:
            u0, _ = layout.units[s.unit]
            o = layout.offsets[s.name] - u0
            n = math.prod(s.shape)
            if 0 < s.unit < last:
                wb, gb = (None if full is not None else wslots[(s.unit - 1) % 2]), gslots[(s.unit - 1) % 2]
            else:
                wb, gb = (None if full is not None else edge_w[s.unit]), edge_g[s.unit]
            if wb is None:
                wb = full[u0:]
            v = wb[o: o + n].view(s.shape)
            v.main_grad = gb[o: o + n].view(s.shape)
            self.t[s.name] = v


class FSDPActor(Actor):
    """Full-shard (FSDP) actor over the flat layout.

    Each rank holds 1/W of every unit: bf16 weights (`shard16`), fp32 master, AdamW
    moments and the reduced fp32 gradient (`grad_shard`).  The colocated engine keeps the
    full bf16 serving copy (`serve16`) resident, and it equals the gathered shards for the
    whole of a training step (it is re-gathered right after each optimizer step), so by
    default the layers read their weights from it and only gradients are staged per layer;
    with `gather_weights=True` (a deployment whose serving copy lives elsewhere) every
    layer's weights are gathered from the shards as below.  A training micro-batch:

    * forward (gather_weights): before layer i the layer's unit is all-gathered into staging slot i % 2
      (peer loads of every rank's bf16 slice on a gather stream, the next layer prefetched
      while this one computes); the embedding and the norm + head unit are gathered once
      per step into staging of their own;
    * backward (activation-checkpointed): before layer i's recompute its unit is gathered
      again unless its slot still holds it, and its gradient slot is zeroed; once layer
      i's backward has run, a reduce-scatter on a second stream waits (bounded peer-flag
      barrier) until every rank has finished that layer, adds this rank's slice of every
      rank's gradient slot into `grad_shard` (peer loads, rank order), and a second
      barrier releases the slots, so the reduce-scatter of layer i overlaps the backward
      of the layers below it;
    * the embedding and head gradients are reduce-scattered once per step, before the
      optimizer.
    The optimizer step: squared norm of `grad_shard`, one scalar all-reduce, AdamW on the
    shard writing the new bf16 slice in place; then the serving copy (`weights`, the
    colocated engine's full bf16 buffer) is re-gathered unit by unit over peer memory -
    the trainer -> rollout weight sync.  Every rank runs the same number of micro-batches
    (a rank with fewer runs empty ones) so the per-layer collectives pair up.

    Without CUDA peer memory (CPU / gloo tests) the same steps run on torch.distributed
    collectives: all_gather per unit and an all_reduce of the gradient slot whose own
    slice is added to `grad_shard`.

    Reference parity: FSDP2 `fully_shard` per decoder layer in the reference's AReaL actor
    (`octopus/rl/actor.py`, `grpo.yaml` actor.backend fsdp), with the gather/reduce once
    per layer call (`octopus/rl/chunk_major.py:421-482`)."""

    def __init__(self, cfg, device="cuda", *, optim: OptimConfig | None = None, ppo: PPOConfig | None = None,
                 seed: int = 0, dtype=torch.bfloat16, temperature: float = 1.0, group=None,
                 fused: bool | None = None, wait_budget_us: int = 60_000_000, gather_weights: bool = False):
        self.cfg = cfg
        self.device = torch.device(device)
        self.optim = optim or OptimConfig()
        self.ppo = ppo or PPOConfig()
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.layout = FlatLayout(cfg, pad_multiple=self.world)
        self.us = UnitShards(self.layout, self.world, self.rank)
        self.fused = (self.device.type == "cuda") if fused is None else fused
        self.gather_weights = bool(gather_weights)
        self.ckpt, self.ckpt_block, self.chunk_tokens, self.host_acts, self.seq_tile = True, 1, 0, None, 0
        self.temperature, self.version, self.step_count = temperature, 0, 0
        gdt = torch.float64 if dtype == torch.float64 else torch.float32
        us, dev = self.us, self.device
        n_units = len(us.units)
        self.last_unit = n_units - 1
        full = init_flat(cfg, self.layout, dev, dtype=dtype, seed=seed)  # same on every rank
        layer_n = max(us.size[1:self.last_unit]) if n_units > 2 else 8
        if self.fused:
            self._shard_peers = PeerBuffers(us.total * 2, dev, group)
            self.shard16 = self._shard_peers.local.view(torch.bfloat16)
            self._gslot_peers = PeerBuffers(2 * layer_n * 4, dev, group)
            gsl = self._gslot_peers.local.view(torch.float32)
            self._edge_g_peers = {u: PeerBuffers(us.size[u] * 4, dev, group) for u in (0, self.last_unit)}
            edge_g = {u: b.local.view(torch.float32) for u, b in self._edge_g_peers.items()}
            self._flags = PeerBuffers(64, dev, group)
            self._seq = 0
            self._g_stream = torch.cuda.Stream(dev)
            self._r_stream = torch.cuda.Stream(dev)
            self._budget_us = int(wait_budget_us)  # the per-layer barriers may wait out a slower rank's layer
        else:
            self.shard16 = torch.empty(us.total, dtype=dtype, device=dev)
            gsl = torch.zeros(2 * layer_n, dtype=gdt, device=dev)
            edge_g = {u: torch.zeros(us.size[u], dtype=gdt, device=dev) for u in (0, self.last_unit)}
        for u in range(n_units):
            self.shard16[us.local(u)].copy_(full[us.owned(u)])
        self.gslots = [gsl[:layer_n], gsl[layer_n:]]
        if self.gather_weights:
            self.wslots = [torch.empty(layer_n, dtype=dtype, device=dev) for _ in range(2)]
            self.edge_w = {u: torch.empty(us.size[u], dtype=dtype, device=dev) for u in (0, self.last_unit)}
        else:
            self.wslots, self.edge_w = [], {}
        self.edge_g = edge_g
        self.tw = _StagedWeights(cfg, self.layout, self.wslots, self.gslots, self.edge_w, self.edge_g,
                                 full=None if self.gather_weights else full)
        # the serving copy: full bf16 weights the colocated engine reads
        self.serve16 = full
        self.weights = Weights(cfg, self.serve16, self.layout)
        self.flat16 = self.serve16
        self.master = self.shard16.to(gdt).clone()
        self.exp_avg = torch.zeros_like(self.master)
        self.exp_avg_sq = torch.zeros_like(self.master)
        self.grad_shard = torch.zeros_like(self.master)
        self.grad = self.grad_shard
        self._slot_unit = [-1, -1]     # unit currently held by each weight slot
        self._gather_ev = {}           # unit -> event: gathered (fused path)
        self._slot_free_ev = [None, None]   # weight slot -> event: its last compute was enqueued before this
        self._gslot_rs_ev = [None, None]    # gradient slot -> event: its last reduce-scatter finished
        self._edges_ready = False
        self._bwd_prev = None          # unit whose backward completed last (awaiting its reduce-scatter)
        self._lf = [functools.partial(self._layer, i) for i in range(cfg.layers)]

    # ------------------------------------------------------------------ collectives
    def _barrier(self):
        self._seq += 1
        ops.ext().peer_barrier(self._flags.ptrs, self.rank, self._seq, self.device.index, self._budget_us)

    def _gather_into(self, u: int, dst: torch.Tensor):
        n = self.us.su[u]
        if self.fused:
            ops.ext().peer_gather_bf16(self._shard_peers.ptrs, self.us.shard_off[u], n, dst)
        else:
            parts = [torch.empty(n, dtype=dst.dtype, device=dst.device) for _ in range(self.world)]
            dist.all_gather(parts, self.shard16[self.us.local(u)].contiguous(), group=self.group)
            dst[: n * self.world].copy_(torch.cat(parts))

    def _rs_into(self, u: int, slot: torch.Tensor, peers=None):
        """grad_shard[unit u] += this rank's slice of the sum over ranks of `slot`."""
        n = self.us.su[u]
        acc = self.grad_shard[self.us.local(u)]
        if self.fused:
            base = (slot.data_ptr() - peers.local.data_ptr()) // 4  # slot offset inside the peer buffers
            ops.ext().peer_rs_acc(peers.ptrs, base + self.rank * n, acc)
        else:
            red = slot[: n * self.world].clone()
            dist.all_reduce(red, group=self.group)
            acc.add_(red[self.rank * n: (self.rank + 1) * n])

    # ------------------------------------------------------------------ staging
    def _gather_layer(self, u: int, prefetch: bool):
        """Unit u (a layer) into weight slot (u - 1) % 2 unless it is there already."""
        if not self.gather_weights:
            return
        s = (u - 1) % 2
        if self._slot_unit[s] == u:
            return
        self._slot_unit[s] = u
        if not self.fused:
            self._gather_into(u, self.wslots[s])
            return
        main = torch.cuda.current_stream(self.device)
        ev = torch.cuda.Event()
        ev.record(main)  # every compute that read this slot before has been enqueued
        with torch.cuda.stream(self._g_stream):
            self._g_stream.wait_event(ev)
            self._gather_into(u, self.wslots[s])
            done = torch.cuda.Event()
            done.record(self._g_stream)
        self._gather_ev[u] = done
        if not prefetch:
            main.wait_event(done)

    def _wait_layer(self, u: int):
        if self.fused and u in self._gather_ev:
            torch.cuda.current_stream(self.device).wait_event(self._gather_ev.pop(u))

    def _stage_edges(self):
        if self._edges_ready or not self.gather_weights:
            return
        for u in (0, self.last_unit):
            self._gather_into(u, self.edge_w[u])
        self._edges_ready = True

    def _reduce_layer(self, u: int):
        """Reduce-scatter of unit u's gradient slot (a layer whose backward has run)."""
        s = (u - 1) % 2
        if not self.fused:
            self._rs_into(u, self.gslots[s])
            return
        main = torch.cuda.current_stream(self.device)
        ev = torch.cuda.Event()
        ev.record(main)
        with torch.cuda.stream(self._r_stream):
            self._r_stream.wait_event(ev)
            self._barrier()      # every rank has finished this layer's backward
            self._rs_into(u, self.gslots[s], self._gslot_peers)
            self._barrier()      # every rank has read this rank's slot
            done = torch.cuda.Event()
            done.record(self._r_stream)
        self._gslot_rs_ev[s] = done

    def _zero_gslot(self, u: int):
        s = (u - 1) % 2
        if self.fused and self._gslot_rs_ev[s] is not None:
            torch.cuda.current_stream(self.device).wait_event(self._gslot_rs_ev[s])
        self.gslots[s].zero_()

    def _layer(self, i: int, x, w, cfg, pos, plan, lw):
        """Layer i's forward (no grad) or its recompute in backward, with its unit staged."""
        from ..models.decoder import layer_forward

        u = i + 1
        if torch.is_grad_enabled():  # backward: the recompute of layer i
            if self._bwd_prev is not None and self._bwd_prev != self.last_unit:
                self._reduce_layer(self._bwd_prev)
            self._bwd_prev = u
            self._zero_gslot(u)
            self._gather_layer(u, prefetch=False)
            self._wait_layer(u)
            if u > 1:
                self._gather_layer(u - 1, prefetch=True)
        else:
            self._gather_layer(u, prefetch=False)
            self._wait_layer(u)
            if u < cfg.layers:
                self._gather_layer(u + 1, prefetch=True)
        return layer_forward(x, w, cfg, pos, plan, lw)

    # ------------------------------------------------------------------ training
    def _forward(self, batch):
        from ..models.decoder import _Ckpt

        cfg, tw = self.cfg, self.tw
        self._stage_edges()
        x = ops.embed(batch.ids, tw["embed"])
        if not x.requires_grad:
            x.requires_grad_(True)
        self._bwd_prev = self.last_unit
        for i in range(cfg.layers):
            x = _Ckpt.apply(x, self._lf[i], tw.layer(i), cfg, batch.pos, batch.plan, None)
        h = ops.rmsnorm(x, tw["norm"], cfg.rms_eps, cfg.norm_plus_one)
        hp = h.index_select(0, batch.pair_rows)
        return ops.logprob_head(hp, tw.head, batch.pair_labels, 1.0 / self.temperature, cfg.vocab_size)

    def _finish_backward(self):
        if self._bwd_prev is not None and self._bwd_prev != self.last_unit:
            self._reduce_layer(self._bwd_prev)
        self._bwd_prev = None

    def zero_grad(self):
        self.grad_shard.zero_()
        for g in self.edge_g.values():
            g.zero_()

    def forward_backward(self, mbs, denom=None):
        local = float(sum(mb.pair_w.sum() for mb in mbs))
        dev = self.device if self.device.type == "cuda" else "cpu"
        t = torch.tensor([local, float(len(mbs))], dtype=torch.float64, device=dev)
        dist.all_reduce(t[:1], group=self.group)
        cnt = t[1:].clone()
        dist.all_reduce(cnt, op=dist.ReduceOp.MAX, group=self.group)
        denom = float(t[0]) or 1.0
        mbs = list(mbs) + [_empty_microbatch(self.cfg)] * (int(cnt.item()) - len(mbs))
        stats = {}
        for mb in mbs:
            d = mb.to_device(self.device)
            logp, ent = self._forward(d.batch)
            loss, st = ppo_loss(logp, ent, d.adv, d.w, d.behav, None, denom, self.ppo)
            loss.backward()
            self._finish_backward()
            for k, v in st.items():
                stats[k] = stats.get(k, 0.0) + v.detach() * (1.0 if k == "tokens" else float(mb.pair_w.sum()))
            stats["loss"] = stats.get("loss", 0.0) + loss.detach()
        stats.setdefault("loss", torch.zeros((), device=self.device))
        tok = local or 1.0
        return {k: (v if k in ("tokens", "loss") else v / tok) for k, v in stats.items()}

    def optimizer_step(self) -> torch.Tensor:
        self.step_count += 1
        o = self.optim
        if self.fused:
            main = torch.cuda.current_stream(self.device)
            main.wait_stream(self._r_stream)
            self._barrier()  # every rank's edge gradients are complete
            for u in (0, self.last_unit):
                self._rs_into(u, self.edge_g[u], self._edge_g_peers[u])
            self._barrier()  # read by everyone
        else:
            for u in (0, self.last_unit):
                self._rs_into(u, self.edge_g[u])
        sq = torch.zeros(1, dtype=torch.float32, device=self.device)
        ops.sqnorm_(self.grad_shard, sq)
        dist.all_reduce(sq, group=self.group)
        ops.adamw_(self.master, self.grad_shard, self.exp_avg, self.exp_avg_sq, self.shard16, lr=o.lr, betas=o.betas,
                   eps=o.eps, weight_decay=o.weight_decay, step=self.step_count, sqnorm=sq, max_norm=o.max_grad_norm)
        self.sync_serving()
        self.version += 1
        return sq

    def sync_serving(self):
        """Gather every unit's new bf16 slices into the serving copy (trainer -> rollout sync)."""
        if self.fused:
            self._barrier()  # every rank's shard16 holds its updated slices
        for u in range(len(self.us.units)):
            s, e = self.us.units[u]
            self._gather_into(u, self.serve16[s:e])
        if self.fused:
            self._barrier()  # nobody reads a shard that its owner is about to update again
        self._slot_unit = [-1, -1]
        self._edges_ready = False

    def after_load(self):
        """After a recover checkpoint filled the serving copy and the fp32 shards: this rank's
        bf16 weight shards from the serving copy."""
        for u in range(len(self.us.units)):
            self.shard16[self.us.local(u)].copy_(self.serve16[self.us.owned(u)])
        self._slot_unit = [-1, -1]
        self._edges_ready = False

    def reload_master(self):
        """After a checkpoint load into the serving copy: shards <- it, master <- shards."""
        for u in range(len(self.us.units)):
            self.shard16[self.us.local(u)].copy_(self.serve16[self.us.owned(u)])
        self.master.copy_(self.shard16.to(self.master.dtype))
        self._slot_unit = [-1, -1]
        self._edges_ready = False

    def close(self):
        if self.fused:
            torch.cuda.synchronize(self.device)
            bufs = [self._shard_peers, self._gslot_peers, self._flags, *self._edge_g_peers.values()]
            for b in bufs:
                b.close()


def _empty_microbatch(cfg):
    """A micro-batch with no trained pair (keeps the ranks' collective sequences aligned)."""
    import numpy as np

    from ..rl.actor import build_microbatch

    toks = np.ones(8, np.int64)
    return build_microbatch(toks, [0, 8], None, np.zeros(8), np.zeros(8), np.zeros(8), pad_to=8)
