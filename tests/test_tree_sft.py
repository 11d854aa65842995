"""Tree SFT on CPU: a scripted SWE episode (fork into a fixing branch and an aborting one)
is logged by the SWE eval; its fork tree is collected and encoded (labels on assistant
spans only, root shared by every child, root labels in the join row only); the tree loss
(root computed once in a prefix-tree micro-batch) equals the sum of the flat losses in
value and adapter gradients; tree and flat training run and save adapters, two gloo ranks
give the one-rank update; a saved adapter merges into an HF checkpoint as W + s B A; the
branch metrics of the logged run."""
import json
import os
import platform
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from octopus_b200.envs.swe.containers import LocalExec
from octopus_b200.envs.swe.taskset import TaskSpec, write_task_tree
from octopus_b200.eval.swe_eval import evaluate
from octopus_b200.models.config import get_config
from octopus_b200.serving.chat import ChatTokenizer
from octopus_b200.tools.tree_sft import build as tbuild
from octopus_b200.tools.tree_sft.check_equivalence import compare, make_actor, synthetic_tree
from octopus_b200.tools.tree_sft.encode import IGNORE, encode_tree, flat_rows
from octopus_b200.tools.tree_sft.eval_metrics import run_metrics
from octopus_b200.tools.tree_sft.merge_lora import merge as merge_lora
from octopus_b200.tools.tree_sft.train import train
from octopus_b200.tools.tree_sft.trees import collect
from test_runtime import Scripted, call
from test_swe_taskset import HIDDEN, _repo

x86 = pytest.mark.skipif(platform.machine() != "x86_64", reason="x86_64 guard")
FIX = "--- a/calc.py\n+++ b/calc.py\n@@ -1,2 +1,2 @@\n def add(a, b):\n-    return a - b\n+    return a + b\n"


class _Routed(Scripted):
    def __call__(self, body):
        sid = body["session_id"]
        return super().__call__({**body, "session_id": sid.rsplit("/", 1)[-1] if "/" in sid else "main"})


def _logged_run(tmp_path):
    repo = _repo(tmp_path)
    spec = TaskSpec("org__calc-1", repo, "HEAD", "add() subtracts; make it add.", "",
                    f"{sys.executable} test_hidden.py", {"test_hidden.py": HIDDEN}, fix_patch=FIX)
    chat = _Routed({
        "main": [("I will split the work.", [call("fork", tasks=["fix add", "look at mul"])]),
                 ("All merged.", [call("done", answer="fixed")])],
        "branch-0": [("Fixing.", [call("edit", path="calc.py", old="a - b", new="a + b")]),
                     ("Done.", [call("commit", branch_id="branch-0", summary="add fixed")])],
        "branch-1": [("Not needed.", [call("abort", branch_id="branch-1", reason="out of scope")])],
    })

    class Svc:
        pass

    svc = Svc()
    svc.chat = chat
    logs = tmp_path / "logs"
    out = evaluate(svc, [spec], samples=1, executor=LocalExec(sandbox=True), timeout=30, log_dir=str(logs))
    assert out["summary"]["resolved"] == 1.0
    return spec, logs


@x86
def test_collect_encode_build(tmp_path):
    _, logs = _logged_run(tmp_path)
    trees = collect([str(logs)])
    assert len(trees) == 1
    t = trees[0]
    assert t["train_root"] and [c["kind"] for c in t["children"]] == ["join", "branch", "branch"]
    assert t["children"][1]["messages"][0]["role"] == "user"  # the branch's task message opens its child
    assert collect([str(logs)], min_reward=2.0) == []
    tok = ChatTokenizer.tiny()
    enc = encode_tree(t, tok, max_len=1 << 16, min_child_tokens=1)
    assert enc is not None and len(enc["children"]) == 3
    text = tok.decode(enc["root_ids"])
    assert text.count("<|im_start|>assistant") == 1  # the forking reply is the root's only assistant turn
    for c in enc["children"]:
        assert len(c["ids"]) == len(c["labels"]) and any(x != IGNORE for x in c["labels"])
        lab = tok.decode([x for x in c["labels"] if x != IGNORE])
        assert "<|im_start|>" not in lab and "<tool_response>" not in lab
    assert any(x != IGNORE for x in enc["root_labels"])
    rows = flat_rows(enc)
    nroot = len(enc["root_ids"])
    assert [r["kind"] for r in rows] == ["join", "branch", "branch"]
    assert rows[0]["labels"][:nroot] == enc["root_labels"]
    assert all(x == IGNORE for r in rows[1:] for x in r["labels"][:nroot])
    stats = tbuild.build([str(logs)], tok, tmp_path / "enc.jsonl", max_len=1 << 16, max_tree_tokens=None)
    assert stats["kept"] == 1 and stats["children"] == 3
    assert tbuild.build([str(logs)], tok, tmp_path / "e2.jsonl", max_len=8)["dropped"] == 1  # dropped whole


@pytest.mark.parametrize("dtype,tol", [(torch.float64, 1e-10), (torch.float32, 2e-4)])
def test_tree_equals_flat(dtype, tol):
    cfg = get_config("tiny", layers=2)
    actor = make_actor(cfg, "cpu", dtype)
    r = compare(actor, synthetic_tree(cfg.vocab_size, root=60, child=24))
    assert r["tokens_tree"] == r["tokens_flat"] == 30 + 3 * 16
    assert r["loss_rel_diff"] < tol and r["grad_rel_diff"] < tol * 10 and r["grad_norm"] > 0


def _trees(n=3, seed=0):
    return [synthetic_tree(4096, root=40, child=16, seed=seed + i) for i in range(n)]


def test_train_tree_and_flat(tmp_path):
    cfg = get_config("tiny", layers=1)
    for method in ("tree", "flat"):
        actor = make_actor(cfg, "cpu", torch.float32)
        recs = train(actor, _trees(), tmp_path / method, method=method, epochs=3, per_step=3 if method == "tree" else 9,
                     lr=3e-3, warmup=0.0, log=lambda *_: None)
        assert len(recs) == 3 and all(np.isfinite(r["loss"]) for r in recs)
        assert recs[-1]["loss"] < recs[0]["loss"]
        assert (tmp_path / method / "final" / "adapter_model.safetensors").exists()
        assert (tmp_path / method / "epoch3" / "adapter_config.json").exists()


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, out_dir, q):
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    from datetime import timedelta

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    try:
        actor = make_actor(get_config("tiny", layers=1), "cpu", torch.float64)
        train(actor, _trees(4), out_dir, method="tree", epochs=1, per_step=4, lr=1e-3, warmup=0.0, rank=rank,
              world=world, log=lambda *_: None)
        q.put((rank, actor.lora.master.clone().numpy()))
    finally:
        dist.destroy_process_group()


def test_two_ranks_match_one(tmp_path):
    actor = make_actor(get_config("tiny", layers=1), "cpu", torch.float64)
    train(actor, _trees(4), tmp_path / "one", method="tree", epochs=1, per_step=4, lr=1e-3, warmup=0.0,
          log=lambda *_: None)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, str(tmp_path / "two"), q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    want = actor.lora.master.numpy()
    for r in (0, 1):
        assert np.allclose(got[r], want, rtol=1e-9, atol=1e-12)


def test_merge_lora_into_checkpoint(tmp_path):
    from octopus_b200.models.decoder import FlatLayout, Weights, init_flat, load_hf, save_hf

    cfg = get_config("tiny", layers=1)
    actor = make_actor(cfg, "cpu", torch.float32)
    with torch.no_grad():
        for name, t in actor.lora.t.items():
            t.mul_(50.0)  # a visible delta
    actor.reload_master()
    actor.optimizer_merge()
    save_hf(actor.base, str(tmp_path / "base"))
    actor.lora.save_peft(str(tmp_path / "ad"))
    n = merge_lora(tmp_path / "ad", tmp_path / "base", tmp_path / "merged")
    assert n == 7  # q, k, v, o, gate, up, down of the one layer
    lay = FlatLayout(cfg)
    w = Weights(cfg, init_flat(cfg, lay, "cpu", dtype=torch.float32, seed=5), lay)
    load_hf(w, str(tmp_path / "merged"))
    assert torch.allclose(w.flat, actor.serving.flat, atol=1e-5)
    assert (tmp_path / "merged" / "MERGED_FROM.json").exists() and (tmp_path / "merged" / "config.json").exists()


@x86
def test_branch_metrics(tmp_path):
    spec, logs = _logged_run(tmp_path)
    tasks = tmp_path / "tasks"
    write_task_tree(tasks, spec)
    m = run_metrics(logs, tasks)
    assert m["episodes"] == 1 and m["success"] == 1.0 and m["fork_rate"] == 1.0 and m["forks"] == 1
    assert m["branch_close"] == 1.0 and m["merge_ok"] == 1.0 and m["merges"] == 1
    assert m["branch_hit"] == 0.5 and m["branch_fix"] == 1.0
    assert m["select_ok"] == 1.0 and m["select_branch"] == 1.0 and m["bug_coverage"] == 1.0
