"""BrowseComp-Plus judge and evaluation on CPU: the three verdict forms parse, a reply without
a verdict gets one follow-up, verdicts are cached and reused, grading falls back to the
environment's judge and counts unparsed verdicts; the BCP evaluation computes judged
accuracy and the three recalls from run lines and from a logged search episode, with judge
failures counted and empty responses never judged."""
import json

from octopus_b200.envs.search import judge as J
from octopus_b200.envs.search.reward import grade
from octopus_b200.eval.bcp import episode_run, evaluate


def test_parse_forms():
    assert J.parse_judge("**correct:** yes\n**confidence:** 90") == (True, 90.0)
    assert J.parse_judge("**correct**: No\nconfidence: 250") == (False, 100.0)
    assert J.parse_judge("reasoning...\ncorrect: yes") == (True, None)
    assert J.parse_judge("confidence: 80") == (None, 80.0)


def test_follow_up_and_cache(tmp_path, monkeypatch):
    monkeypatch.setattr(J, "judge_identity", lambda url, model, key=None: "judge-model-path")
    calls = []

    def post(url, body, headers, timeout):
        calls.append(body["messages"])
        text = "long reasoning, no verdict" if len(calls) == 1 else "correct: yes\nconfidence: 70"
        return {"choices": [{"message": {"content": text}}]}

    cache = str(tmp_path / "verdicts.jsonl")
    assert J.judge("q?", "resp", "gold", "http://x/v1", cache=cache, post=post) == (True, 70.0)
    assert len(calls) == 2 and calls[1][-1]["content"] == J.FOLLOW_UP and "[correct_answer]: gold" in calls[0][0]["content"]
    assert J.judge("q?", "resp", "gold", "http://x/v1", cache=cache, post=post) == (True, 70.0)
    assert len(calls) == 2  # served from the cache

    def silent(url, body, headers, timeout):
        return {"choices": [{"message": {"content": "no verdict"}}]}

    assert J.judge("q2", "r", "g", "http://x/v1", cache=cache, post=silent) == (None, None)
    assert sum(1 for _ in open(cache)) == 1  # only verdicts are cached


def test_grade_uses_env_judge(monkeypatch):
    assert grade("q", "Paris", "paris") == {"correct": True, "by": "exact"}
    assert grade("q", "Lyon", "Paris") == {"correct": False, "by": "exact"}
    monkeypatch.setattr(J, "env_judge", lambda: (lambda q, r, g: None))
    assert grade("q", "Lyon", "Paris") == {"correct": False, "by": "judge_unparsed"}
    monkeypatch.setattr(J, "env_judge", lambda: (lambda q, r, g: True))
    assert grade("q", "the capital of France", "Paris") == {"correct": True, "by": "judge"}


def test_evaluate_recalls_and_failures():
    truth = {"1": {"query": "q1", "answer": "a1", "evidence_docids": ["d1", "d2"], "gold_docids": ["d1"]},
             "2": {"query": "q2", "answer": "a2", "evidence_docids": ["d3"], "gold_docids": ["d3"]},
             "3": {"query": "q3", "answer": "a3", "evidence_docids": [], "gold_docids": []}}
    run = [{"query_id": 1, "response": "a1", "retrieved_docids": ["d1", "d9"], "opened_docids": ["d2"]},
           {"query_id": 2, "response": "", "retrieved_docids": ["d3"], "opened_docids": ["d3"]},
           {"query_id": 3, "response": "boom", "retrieved_docids": [], "opened_docids": []}]
    asked = []

    def judge(q, r, g):
        asked.append(q)
        if q == "q3":
            raise OSError("endpoint down")
        return r == g, 100.0

    s, rows = evaluate(run, truth, judge, workers=2)
    assert "q2" not in asked  # empty response: no judge call
    assert s["n"] == 3 and abs(s["accuracy"] - 1 / 3) < 1e-12 and s["judge_failures"] == 1
    assert abs(s["recall"] - (0.5 + 1.0) / 2) < 1e-12 and abs(s["open_recall"] - (0.5 + 1.0) / 2) < 1e-12
    assert abs(s["open_gold_recall"] - (0.0 + 1.0) / 2) < 1e-12
    assert all(set(r) == {"query_id", "correct", "confidence", "recall", "open_recall", "open_gold_recall"}
               for r in rows)


def test_episode_run_from_logs(tmp_path, monkeypatch):
    from octopus_b200.envs.search.agent import SearchWorkspace
    from octopus_b200.envs.search.service import Retrieval
    from octopus_b200.runtime.tree import run_episode
    from test_runtime import Scripted, call

    docs = [{"docid": f"d{i}", "title": f"t{i}", "text": f"alpha beta {i} gamma"} for i in range(5)]
    ws = SearchWorkspace(Retrieval(docs), "q")
    chat = Scripted({"ep": [("", [call("search", query="alpha", k=3)]), ("", [call("open", docid="d2")]),
                            ("", [call("done", answer="42")])]})
    run_episode(ws, chat, "q", log_dir=str(tmp_path / "ep"))
    line = episode_run(tmp_path / "ep", "7")
    assert line["query_id"] == "7" and line["response"] == "42"
    assert len(line["retrieved_docids"]) == 3 and line["opened_docids"] == ["d2"]
