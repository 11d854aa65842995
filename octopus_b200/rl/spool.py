"""Rollout spool: finished groups survive a trainer restart.

Lifecycle of a group file ``<head version>~<task>~<id>.pt`` under the spool directory:

  save      rollout finished a group with reward variance      -> ready/
  recover   trainer start at the resumed version: ready/, taken/ and trained/ of the
            previous process -> resume/, keeping ONE group per task (the newest head
            version at most the resumed version, then the newest file); the others
            of that task are deleted
  take      a new group call reuses its own task's resume/ group, else the oldest one
            whose head version is within max_head_offpolicyness of the current
            version (atomic rename -> taken/); stale or too-new groups are dropped;
            with none left, a task whose group is already out (taken/ or trained/) is
            rejected ({}) instead of rolled out twice
  consume   a train step used these groups                       -> trained/
  commit    a recover checkpoint covers the step                 trained/ deleted

A group is gone only once a checkpoint covers the step that trained on it; reuse is
sound because the decoupled PPO loss weighs each token by its stored behaviour logprob.

Reference parity (behaviour): `octopus/rl/spool.py:66-144`.
"""
from __future__ import annotations

import glob
import os
import time
import uuid

import torch

KEY = "octopus_spool"


def head_version(traj: dict) -> int:
    """Oldest policy version among trained tokens."""
    v = traj["versions"]
    m = traj["loss_mask"].bool()
    sel = v[m]
    return int(sel.min()) if sel.numel() else -1


class Spool:
    def __init__(self, root: str, log=print):
        self.root = root
        self.log = log

    def _d(self, sub):
        p = os.path.join(self.root, sub)
        os.makedirs(p, exist_ok=True)
        return p

    @staticmethod
    def _head(path):
        return int(os.path.basename(path).split("~", 1)[0])

    @staticmethod
    def _task(path):
        return os.path.basename(path).split("~", 1)[1].rsplit("~", 1)[0]

    def save(self, traj: dict, task: str) -> str:
        path = os.path.join(self._d("ready"), f"{head_version(traj):06d}~{task}~{uuid.uuid4().hex[:8]}.pt")
        torch.save({k: v for k, v in traj.items() if k != KEY}, path + ".tmp")
        os.replace(path + ".tmp", path)
        return path

    def recover(self, version: int) -> int:
        res = self._d("resume")
        for sub in ("ready", "taken", "trained"):
            for p in glob.glob(os.path.join(self.root, sub, "*.pt")):
                os.replace(p, os.path.join(res, os.path.basename(p)))
        kept: dict[str, tuple] = {}
        files = [(os.path.getmtime(p), p) for p in glob.glob(os.path.join(res, "*.pt"))]
        for mt, p in sorted(files, key=lambda x: (self._head(x[1]) <= version, self._head(x[1]), x[0])):
            old = kept.get(self._task(p))
            if old:
                os.remove(old[1])
                self.log(f"[octopus] spool: deleted {os.path.basename(old[1])}, kept {os.path.basename(p)}")
            kept[self._task(p)] = (mt, p)
        return len(kept)

    def take(self, version: int, max_offpolicy: int, task: str):
        taken = self._d("taken")
        res = self._d("resume")
        for p in sorted(glob.glob(os.path.join(res, "*.pt")), key=lambda x: (self._task(x) != task, x)):
            name = os.path.basename(p)
            if not 0 <= version - self._head(p) <= max_offpolicy:
                try:
                    os.remove(p)
                except FileNotFoundError:
                    pass
                continue
            try:
                os.replace(p, os.path.join(taken, name))
            except FileNotFoundError:
                continue
            traj = torch.load(os.path.join(taken, name), weights_only=False)
            traj[KEY] = os.path.join(taken, name)
            self.log(f"[octopus] spool: reused {name} at version {version}")
            return traj
        out = [p for p in glob.glob(os.path.join(self.root, "taken", "*.pt")) +
               glob.glob(os.path.join(self.root, "trained", "*.pt")) if self._task(p) == task]
        if out:
            self.log(f"[octopus] spool: rejected a call of {task}: its group is already out")
            return {}
        return None

    def consume(self, batch: list[dict]) -> None:
        tr = self._d("trained")
        for d in batch:
            p = d.pop(KEY, None)
            if p:
                try:
                    os.replace(p, os.path.join(tr, os.path.basename(p)))
                except FileNotFoundError:
                    pass

    def commit(self) -> None:
        for p in glob.glob(os.path.join(self.root, "trained", "*.pt")):
            os.remove(p)

    def counts(self) -> dict:
        return {s: len(glob.glob(os.path.join(self.root, s, "*.pt"))) for s in ("ready", "resume", "taken",
                                                                                "trained")}
