"""Search environment: BM25 ranking, retrieval service, grading rules, CPU dry-run episode."""
from octopus_b200.envs.search import dry_run
from octopus_b200.envs.search.bm25 import BM25Index
from octopus_b200.envs.search.reward import exact_match, grade, normalize
from octopus_b200.envs.search.service import Retrieval, create_app


def test_bm25_ranks_relevant_first():
    idx = BM25Index(dry_run.CORPUS)
    top = idx.search("octopus three hearts", k=3)
    assert dry_run.CORPUS[top[0][0]]["docid"] in ("d1", "d3")
    assert all(s > 0 for _, s in top)
    assert idx.search("zzzz unknown") == []


def test_service_endpoints():
    from fastapi.testclient import TestClient

    c = TestClient(create_app(Retrieval(dry_run.CORPUS)))
    assert c.get("/health").json()["docs"] == 3
    res = c.post("/search", json={"query": "squid beak", "k": 2}).json()["results"]
    assert res[0]["docid"] == "d2" and res[0]["snippet"]
    page = c.post("/open", json={"docid": "d3", "page": 0}).json()
    assert page["pages"] >= 1 and "hearts" in page["text"]
    assert "error" in c.post("/open", json={"docid": "nope"}).json()


def test_grading_rules():
    assert normalize("The \\boxed{Answer}!") == "answer"
    assert exact_match("3.5", "3.5") and not exact_match("35", "3.5")
    assert not exact_match("-4", "4")
    assert grade("q", "", "x")["by"] == "empty"
    assert grade("q", "Paris", "paris")["correct"]
    assert grade("q", "the city of Paris", "Paris", judge=lambda q, r, g: "paris" in r.lower())["by"] == "judge"


def test_dry_run_episode_forks_and_answers():
    out, g = dry_run.main()
    assert out["tree"]["main_end"] == "done" and out["tree"]["answer"] == "three"
    assert len(out["tree"]["forks"][0]["branches"]) == 2
    assert all(b["ended_with"] == "done" for b in out["tree"]["forks"][0]["branches"])
    assert grade("q", out["tree"]["answer"], "three")["correct"]
