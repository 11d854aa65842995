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

import torch
import torch.distributed as dist

from .. import ops
from ..models.decoder import FlatLayout, Weights, init_flat
from ..rl.actor import Actor, OptimConfig
from ..rl.loss import PPOConfig


class PeerBuffers:
    """One IPC-capable buffer per rank, mapped into every rank (device pointers)."""

    def __init__(self, nbytes: int, device: torch.device, group=None):
        C = ops.ext()
        self.local = C.symm_alloc(nbytes, device.index)
        handle = C.ipc_handle(self.local)
        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
        handles = [None] * world
        dist.all_gather_object(handles, handle, group=group)
        self.ptrs = []
        self._opened = []
        for r, h in enumerate(handles):
            if r == rank:
                self.ptrs.append(self.local.data_ptr())
            else:
                p = C.ipc_open(h, device.index)
                self.ptrs.append(p)
                self._opened.append(p)

    def close(self):
        C = ops.ext()
        for p in self._opened:
            C.ipc_close(p)
        self._opened = []


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
