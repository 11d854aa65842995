"""Retrieval service (HTTP): ``/search``, ``/open``, ``/health``.

  POST /search {"query": str, "k": int}  -> {"results": [{docid, title, snippet, score}]}
  POST /open   {"docid": str, "page": int} -> {"docid", "title", "page", "pages", "text"}
  GET  /health -> {"ok": true, "docs": n}

Snippets are the first `snippet_words` words of a document (the reference uses 512
tokens of the policy tokenizer); `/open` pages a document in `page_words` chunks.

Reference parity (behaviour): `octopus/envs/search/service.py:100-230`.
"""
from __future__ import annotations

from .bm25 import BM25Index


class Retrieval:
    """In-process retrieval with the same contract as the HTTP service.  backend "bm25"
    (default) ranks with the in-process BM25 index; "dense" ranks by inner product of the
    query embedding (`encode(query) -> vector`) with document embeddings (`dense`: a
    DenseIndex whose docids name documents of `docs`)."""

    def __init__(self, docs: list[dict], snippet_words: int = 64, page_words: int = 512, backend: str = "bm25",
                 dense=None, encode=None):
        self.index = BM25Index(docs)
        self.snippet_words = snippet_words
        self.page_words = page_words
        self.backend = backend
        if backend == "dense":
            if dense is None or encode is None:
                raise ValueError("the dense backend needs a DenseIndex and a query encoder")
            self.dense, self.encode = dense, encode
            self._dense_rows = [self.index.by_id.get(d) for d in dense.docids]
        elif backend != "bm25":
            raise ValueError(f"backend {backend!r}: bm25 or dense")

    def _ranked(self, query: str, k: int):
        if self.backend == "bm25":
            return self.index.search(query, k)
        hits = self.dense.search(self.encode(query), k)
        return [(self._dense_rows[r], s) for r, s in hits if self._dense_rows[r] is not None]

    def search(self, query: str, k: int = 10) -> list[dict]:
        out = []
        for i, s in self._ranked(query, k):
            d = self.index.docs[i]
            words = d.get("text", "").split()
            out.append({"docid": d["docid"], "title": d.get("title", ""),
                        "snippet": " ".join(words[: self.snippet_words]), "score": round(s, 4)})
        return out

    def open(self, docid: str, page: int = 0) -> dict:
        i = self.index.by_id.get(docid)
        if i is None:
            return {"error": f"no document {docid}"}
        d = self.index.docs[i]
        words = d.get("text", "").split()
        pages = max(1, (len(words) + self.page_words - 1) // self.page_words)
        page = max(0, min(int(page), pages - 1))
        return {"docid": docid, "title": d.get("title", ""), "page": page, "pages": pages,
                "text": " ".join(words[page * self.page_words:(page + 1) * self.page_words])}


def create_app(retrieval: Retrieval):
    from fastapi import FastAPI

    app = FastAPI()

    @app.get("/health")
    async def health():
        return {"ok": True, "docs": len(retrieval.index.docs), "backend": retrieval.backend}

    @app.post("/search")
    async def search(body: dict):
        return {"results": retrieval.search(str(body.get("query", "")), int(body.get("k", 10)))}

    @app.post("/open")
    async def open_(body: dict):
        return retrieval.open(str(body.get("docid", "")), int(body.get("page", 0)))

    return app


class HTTPRetrieval:
    """Client of the service with the Retrieval interface."""

    def __init__(self, url: str, timeout: float = 30.0):
        self.url = url.rstrip("/")
        self.timeout = timeout

    def _post(self, path, body):
        import json
        import urllib.request

        req = urllib.request.Request(self.url + path, data=json.dumps(body).encode(),
                                     headers={"Content-Type": "application/json"})
        with urllib.request.urlopen(req, timeout=self.timeout) as r:
            return json.load(r)

    def search(self, query: str, k: int = 10):
        return self._post("/search", {"query": query, "k": k})["results"]

    def open(self, docid: str, page: int = 0):
        return self._post("/open", {"docid": docid, "page": page})


def make_retrieval(docs: list[dict], backend: str = "bm25", embeddings: str = "", encoder: str = "",
                   device: str = "cpu") -> Retrieval:
    """A Retrieval over `docs`: BM25, or dense with document embeddings from `embeddings`
    (a glob of (reps, docids) pickles) and the query encoder at local path `encoder`."""
    if backend != "dense":
        return Retrieval(docs)
    from .dense import DenseIndex, QueryEncoder, load_embeddings

    reps, ids = load_embeddings(embeddings)
    return Retrieval(docs, backend="dense", dense=DenseIndex(reps, ids, device), encode=QueryEncoder(encoder, device))


def main(argv=None) -> int:
    import argparse
    import json

    ap = argparse.ArgumentParser(prog="python -m octopus_b200.envs.search.service")
    ap.add_argument("--docs", required=True, help="JSONL corpus: one {docid, title, text} per line")
    ap.add_argument("--backend", default="bm25", choices=["bm25", "dense"])
    ap.add_argument("--embeddings", default="", help="dense: glob of (reps, docids) pickles")
    ap.add_argument("--encoder", default="", help="dense: local path of the query embedding model")
    ap.add_argument("--device", default="cpu")
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8000)
    args = ap.parse_args(argv)
    with open(args.docs) as f:
        docs = [json.loads(line) for line in f if line.strip()]
    import uvicorn

    uvicorn.run(create_app(make_retrieval(docs, args.backend, args.embeddings, args.encoder, args.device)),
                host=args.host, port=args.port)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
