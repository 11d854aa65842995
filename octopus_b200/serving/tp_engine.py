"""Tensor-parallel rollout engine: the Engine's scheduler, cursors, mounts, radix cache
and CUDA-graph decode, with the model forward split over a TP group on the fused
AG -> GEMM / GEMM -> RS kernels (`octopus_b200.parallel.tp`).

Every rank of the group runs the same host logic on the same requests (SPMD), so slot
allocation, radix matches and cursors are identical; the KV cache of a rank holds its
own KV heads.  Activations between the row- and column-parallel GEMMs are sharded by
sequence rows; a forward of M rows is padded to tp * rows_s with rows_s one of the
sizes the fused kernels take (8, 16, 32, 64, k * 128).  Sampling is vocab-parallel and
every rank ends with the same tokens.

`sync_weights()` is the trainer -> rollout weight sync: one reshard launch copying the
trainer's weights into this rank's TP shards.

Reference parity: SGLang tensor-parallel serving (`--tp`) that the reference drives
through `octopus/rl/grpo.yaml` and its mount patch (`sglang_patches/mount.py`).
"""
from __future__ import annotations

import numpy as np
import torch

from .. import ops
from ..ops import serve as sv
from ..parallel.tp import TPGroup, TPWeights, shard_dims, tp_rows
from ..utils.iostats import d2h, h2d
from .engine import Engine


class TPEngine(Engine):
    supports_continuous = False  # every rank must take the same batching decisions: static batches
    def __init__(self, cfg, weights, *, group, max_batch: int = 256, prefill_chunk: int = 16384, **kw):
        import torch.distributed as dist

        self.tp = dist.get_world_size(group)
        self.tp_rank = dist.get_rank(group)
        self.sd = shard_dims(cfg, self.tp, self.tp_rank)
        super().__init__(cfg, weights, max_batch=max_batch, prefill_chunk=prefill_chunk, **kw)
        if self.device.type != "cuda":
            raise RuntimeError("TPEngine needs CUDA peer memory")
        # every rank of the group must hand out the same cursor ids
        uid = [self._uid]
        dist.broadcast_object_list(uid, src=dist.get_global_rank(group, 0), group=group)
        self._uid = uid[0]
        self.tw = TPWeights(cfg, weights, self.sd, self.device)
        max_rows = max(self._pad_rows(prefill_chunk), max_batch)
        # both row-parallel GEMMs (o_proj, down) produce hidden-wide partials
        self.comm = TPGroup(group, self.device, max_rows=max_rows, hidden=cfg.hidden, max_n=cfg.hidden,
                            max_sample_rows=max(max_batch, 1024))

    # ------------------------------------------------------------------ hooks
    def _local_heads(self):
        return self.sd.hq, self.sd.hkv

    def _pad_rows(self, T: int) -> int:
        return self.tp * tp_rows((T + self.tp - 1) // self.tp)

    def _min_bucket(self) -> int:
        return 8 * self.tp

    def sync_weights(self):
        self.tw.refresh()

    # ------------------------------------------------------------------ forward
    def _tp_forward(self, ids_local, pos, slots, attn, rows_s: int):
        """Layers over M = tp * rows_s rows; leaves the final-normed shard in the AG buffer."""
        cfg, c, tw = self.cfg, self.comm, self.tw
        M = self.tp * rows_s
        x = c.x_local(rows_s)
        c.barrier()
        h = sv.embed(ids_local, self.w["embed"])
        x.copy_(sv.rms(h, self.w["layers.0.ln1"], cfg.rms_eps, cfg.norm_plus_one))
        sd = self.sd
        for i in range(cfg.layers):
            ln1, qkv_w, qkv_b, o_w, ln2, gu_w, down_w = tw.layer(i)
            qkv = torch.empty(M, sd.qkv_loc, dtype=h.dtype, device=h.device)
            c.ag_linear(rows_s, qkv_w, qkv, bias=qkv_b)
            sv.rope_(qkv, pos, sd.hq, sd.hkv, cfg.head_dim, cfg.rope_theta)
            sv.kv_write(qkv, sd.hq, sd.hkv, cfg.head_dim, slots, self.kc[i], self.vc[i])
            o = attn(qkv[:, : sd.q_loc], i)
            g = c.rs_linear(o, o_w)
            c.reduce(h, g, w=ln2, x=x, eps=cfg.rms_eps, plus_one=cfg.norm_plus_one)
            gu = torch.empty(M, 2 * sd.f, dtype=h.dtype, device=h.device)
            c.ag_linear(rows_s, gu_w, gu)
            a = sv.swiglu(gu)
            g = c.rs_linear(a, down_w)
            nw = self.w[f"layers.{i + 1}.ln1"] if i + 1 < cfg.layers else self.w["norm"]
            c.reduce(h, g, w=nw, x=x, eps=cfg.rms_eps, plus_one=cfg.norm_plus_one)
        return x

    def _no_filter(self):
        tp_, tk_ = self._filter
        if tp_ < 1.0 or 0 < tk_ < self.cfg.vocab_size:
            raise ValueError("top_p / top_k sampling runs on single-GPU engines; the tensor-parallel engine "
                             "samples from the full tempered distribution (vocab-parallel fused head)")

    def _prefill_forward(self, t_ids, t_pos, t_slots, attn, last, streams, temperature):
        self._no_filter()
        M = t_ids.shape[0]
        rows_s = M // self.tp
        r0 = self.tp_rank * rows_s
        x = self._tp_forward(t_ids[r0:r0 + rows_s], t_pos, t_slots, attn, rows_s)
        # the sampled rows of each rank, compacted into its selection buffer
        owner = last // rows_s
        counts = np.bincount(owner, minlength=self.tp)
        rs = tp_rows(int(counts.max()))
        if rs > self.comm.max_sel:
            raise ValueError("too many sampled rows in one prefill forward")
        mine = last[owner == self.tp_rank] - r0
        sel = self.comm.sel_local(rs)
        if len(mine):
            sel[: len(mine)].copy_(x.index_select(0, h2d(mine, self.device)))
        # global sampling row of each request: rank-major, order of appearance
        rank_pos = np.zeros(len(last), np.int64)
        seen = np.zeros(self.tp, np.int64)
        for k, o in enumerate(owner):
            rank_pos[k] = o * rs + seen[o]
            seen[o] += 1
        st = np.zeros(self.tp * rs, np.int64)
        st[rank_pos] = streams
        tok, lp = self.comm.sample(rs, self.tw.head, temperature, self.seed, h2d(st, self.device), self.sd, sel=True)
        tok, lp = d2h(tok).numpy(), d2h(lp).numpy()
        return tok[rank_pos], lp[rank_pos]

    def _decode_forward(self, tok, pos, slot, attn, B: int, temperature: float):
        self._no_filter()
        rows_s = B // self.tp
        r0 = self.tp_rank * rows_s
        self._tp_forward(tok[r0:r0 + rows_s], pos, slot, attn, rows_s)
        return self.comm.sample(rows_s, self.tw.head, temperature, self.seed, self.s_stream[:B], self.sd)

    def close(self):
        self.comm.close()
