"""Evaluation harnesses on CPU: search episodes graded with recall; DAG rollout-only eval."""
import json

import torch

from octopus_b200.envs.search.service import Retrieval
from octopus_b200.eval import dag_eval
from octopus_b200.eval.search_eval import evaluate
from octopus_b200.models.config import get_config
from octopus_b200.models.decoder import FlatLayout, Weights, init_flat
from octopus_b200.serving.chat import ChatTokenizer
from octopus_b200.serving.engine import Engine
from octopus_b200.serving.local import ChatService

CORPUS = [{"docid": "d1", "title": "Octopus", "text": "An octopus has three hearts."},
          {"docid": "d2", "title": "Squid", "text": "Squids have ten limbs."}]


def test_search_eval_cpu(monkeypatch):
    monkeypatch.setenv("OCTOPUS_MAX_TOKENS", "8")
    tok = ChatTokenizer.tiny()
    cfg = get_config("tiny", vocab_size=(tok.vocab_size + 127) // 128 * 128, layers=2)
    lay = FlatLayout(cfg)
    w = Weights(cfg, init_flat(cfg, lay, "cpu", dtype=torch.float32, seed=0, std=0.05), lay)
    eng = Engine(cfg, w, kv_slots=40000, max_batch=8, device="cpu")
    svc = ChatService(eng, tok, window=0.001)
    qs = [{"qid": "q1", "question": "How many hearts?", "answer": "3", "evidence": ["d1"]},
          {"qid": "q2", "question": "How many limbs?", "answer": "10"}]
    res = evaluate(svc, Retrieval(CORPUS), qs, samples=2, max_main_calls=2, engine=eng)
    s = res["summary"]
    assert s["questions"] == 2 and s["episodes"] == 4
    assert 0.0 <= s["accuracy"] <= 1.0 and s["recall"] in (0.0, 0.5, 1.0)
    assert all(r["requests"] >= 1 for r in res["rows"])
    assert eng.load_stats()["cursors"] == 0


def test_dag_eval_cpu(capsys, monkeypatch):
    assert dag_eval.main(["--preset", "tiny", "--instances", "2", "--samples", "2", "--prefix", "16", "--turn", "4",
                          "--steps", "1", "--cpu"]) == 0
    row = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert row["generated_tokens"] == 2 * 2 * 4 * 4 and row["cache_reuse"] > 0
