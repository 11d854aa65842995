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
    """In-process retrieval with the same contract as the HTTP service."""

    def __init__(self, docs: list[dict], snippet_words: int = 64, page_words: int = 512):
        self.index = BM25Index(docs)
        self.snippet_words = snippet_words
        self.page_words = page_words

    def search(self, query: str, k: int = 10) -> list[dict]:
        out = []
        for i, s in self.index.search(query, k):
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
        return {"ok": True, "docs": len(retrieval.index.docs)}

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
