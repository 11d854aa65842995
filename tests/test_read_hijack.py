"""Read-hijack measures on CPU: scripted episodes whose branch reads a sibling (mounted) or
itself (refused) are logged; measure 1 extracts units with their arms, relations and mounted
steps, a fake judge labels them (resumably), the report and the export run.  Measure 2
rebuilds a mount point's token sequences from the logged tree and samples the three
conditions on a tiny CPU engine; its report gives a decision."""
import json

import numpy as np

from octopus_b200.runtime.tree import WorkspaceProvider, run_episode
from octopus_b200.serving.chat import ChatTokenizer
from octopus_b200.tools import read_hijack as rh
from octopus_b200.tools import read_hijack_probe as rhp
from test_engine_cpu import tiny_engine
from test_runtime import Scripted, call


def _episodes(root, monkeypatch, n=3):
    monkeypatch.setenv("OCTOPUS_READ_TOOL", "1")
    for q in range(n):
        chat = Scripted({
            "ep": [("plan", [call("fork", tasks=["find a", "find b"])]), ("end", [call("done", answer=f"a{q}")])],
            "branch-0": [("found a", [call("commit", branch_id="branch-0", summary=f"a is {q}")])],
            "branch-1": [("", [call("read_thread", thread="branch-0")]),
                         ("reading done", [call("commit", branch_id="branch-1", summary="b from a")])] if q % 2 == 0
            else [("", [call("read_thread", thread="branch-1")]),
                  ("own work", [call("commit", branch_id="branch-1", summary="b alone")])],
        })
        run_episode(WorkspaceProvider(), chat, f"question {q}", log_dir=str(root / f"ep{q}"))


def test_measure1_extract_judge_report(tmp_path, monkeypatch):
    run = tmp_path / "run1"
    _episodes(run, monkeypatch)
    units, stats = rh.extract_units([str(run)])
    arms = sorted((u["arm"], u["refusal"], u["relation"]) for u in units)
    assert arms == [("mounted", None, "sibling"), ("mounted", None, "sibling"), ("refused", "self", "self")]
    m = next(u for u in units if u["arm"] == "mounted")
    assert m["S"].endswith("branch-0") and m["R"].endswith("branch-1") and m["steps"][:2] == [0, 0]
    assert m["steps"][2] > 0 and "commit" in m["action"] and m["S_task"] == "find a"
    assert len({u["cluster"] for u in units}) == 3
    up, lp = tmp_path / "units.jsonl", tmp_path / "labels.jsonl"
    up.write_text("".join(json.dumps(u) + "\n" for u in units))
    calls = {"n": 0}

    def post(body):
        calls["n"] += 1
        text = body["messages"][0]["content"]
        assert "Answer with the label only." in text
        if calls["n"] == 1:
            raise OSError("judge down")  # retried
        return "S_TASK" if "b from a" in text else "own"

    assert rh.judge(up, lp, post, workers=1) == 0
    n_calls = calls["n"]
    assert rh.judge(up, lp, post, workers=1) == 0 and calls["n"] == n_calls  # resumes: nothing left
    lab = rh.labels(lp)
    assert sorted(lab.values()) == ["OWN", "S_TASK", "S_TASK"]
    lines = []
    assert rh.report(up, lp, out=lines.append) == 0
    assert any(line.startswith("| run1 | all | 2 / 1 |") for line in lines)
    cp = tmp_path / "cases.jsonl"
    assert rh.export(up, cp, n=4) == 3
    cases = [json.loads(x) for x in cp.read_text().splitlines()]
    assert all("arm" not in c and c["label"] == "" for c in cases)
    for c in cases:
        c["label"], c["annotator"] = lab[c["id"]], "a"
    cp.write_text("".join(json.dumps(c) + "\n" for c in cases))
    res = rh.precision(rh.load(up, lp), cp, out=lambda *_: None)
    assert res["hijack_precision"] == 1.0 and res["hijack_recall"] == 1.0
    lp.write_text(lp.read_text() + json.dumps({"id": units[0]["id"], "label": "UNPARSED"}) + "\n")
    assert rh.report(up, lp, out=lambda *_: None) == 1  # an invalid label left: no result


def test_boot_and_diff():
    groups = [[1.0, 0.0], [1.0], [0.0, 0.0, 1.0]]
    m, lo, hi = rh.boot(groups)
    assert abs(m - 3 / 6) < 1e-12 and lo <= m <= hi
    rows = [{"cluster": c, "a": a, "y": y} for c, a, y in [(0, 1, 1), (0, 0, 0), (1, 1, 1), (1, 0, 1), (2, 1, 0),
                                                           (2, 0, 0)]]
    d = rh.boot_diff(rows, lambda u: u["y"], lambda u: u["a"])
    assert abs(d[0] - (2 / 3 - 1 / 3)) < 1e-12 and d[1] <= d[0] <= d[2]


def test_measure2_probe_on_engine(tmp_path, monkeypatch):
    run = tmp_path / "run1"
    _episodes(run, monkeypatch)
    units, _ = rh.extract_units([str(run)])
    tok = ChatTokenizer.tiny()
    points, skipped = rhp.select_points(units, tok, n=10)
    assert len(points) == 2 and not skipped
    u, p = points[0]
    assert 0 < p["s"] < p["e"] == len(p["a"]) and p["delta"]["text"] != p["delta"]["none"]
    assert p["jump"] == max(0, p["e"] - len(p["b"]))
    _, w, eng = tiny_engine()
    free = eng.pool.free_count()
    items = tmp_path / "items.jsonl"
    res = rhp.run(eng, tok, units, items, "base", n=10, samples=2, temperature=1.0, max_tokens=4)
    assert res["written"] == 2 and res["failed"] == 0
    rows = [json.loads(x) for x in items.read_text().splitlines()]
    assert len(rows) == 2 * 3 * 2 and {r["cond"] for r in rows} == set(rhp.CONDITIONS)
    res2 = rhp.run(eng, tok, units, items, "base", n=10, samples=2, max_tokens=4)
    assert res2["written"] == 0 and res2["before"] == 2  # resumed
    eng.reset()
    assert eng.pool.free_count() == free  # no slot leaked
    rng = np.random.default_rng(0)
    lp = tmp_path / "labels.jsonl"
    lp.write_text("".join(json.dumps({"id": r["id"], "label": "S_TASK" if r["cond"] == "mount" and rng.random() < 0.9
                                      else "OWN"}) + "\n" for r in rows))
    lines = []
    assert rhp.report(items, lp, out=lines.append) == 0
    assert any("mount - none" in line and "->" in line for line in lines)
