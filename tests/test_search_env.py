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


def test_dense_backend_ranks_by_inner_product(tmp_path):
    """Dense retrieval: document vectors from (reps, docids) pickles, normalised fp16,
    exact top-k by inner product with the encoded query; same result contract as BM25."""
    import pickle

    import numpy as np

    from octopus_b200.envs.search.dense import DenseIndex, load_embeddings
    from octopus_b200.envs.search.service import Retrieval

    docs = [{"docid": f"d{i}", "title": f"t{i}", "text": f"document number {i} " * 5} for i in range(50)]
    rng = np.random.default_rng(0)
    reps = rng.normal(size=(50, 16)).astype(np.float32)
    for k, part in enumerate((slice(0, 30), slice(30, 50))):
        with open(tmp_path / f"emb{k}.pkl", "wb") as f:
            pickle.dump((reps[part], [f"d{i}" for i in range(50)][part]), f)
    r, ids = load_embeddings(str(tmp_path / "emb*.pkl"))
    assert r.shape == (50, 16) and ids[31] == "d31"
    idx = DenseIndex(r, ids, block=7)  # host search in row blocks with a running top-k
    q = reps[17] + 0.01 * rng.normal(size=16)
    enc = {"find seventeen": q}
    ret = Retrieval(docs, backend="dense", dense=idx, encode=lambda s: enc[s])
    hits = ret.search("find seventeen", k=3)
    assert hits[0]["docid"] == "d17" and len(hits) == 3
    norm = reps / np.linalg.norm(reps, axis=1, keepdims=True)
    want = np.argsort(-(norm @ (q / np.linalg.norm(q))))[:3]
    assert [h["docid"] for h in hits] == [f"d{i}" for i in want]
    assert ret.open("d17")["docid"] == "d17"
