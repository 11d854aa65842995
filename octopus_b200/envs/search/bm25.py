"""BM25 retrieval over an in-memory corpus (numpy inverted index, Okapi BM25).

Documents are tokenised into lower-case word tokens; the index is a CSR posting list
(term -> doc ids, term frequencies).  `search` scores only the documents that contain
a query term (vectorised accumulation per query term) and returns the top k.
Parameters k1 = 0.9, b = 0.4 (the Pyserini / Anserini defaults for BM25).

Reference parity (behaviour): the BM25 side of `octopus/envs/search/service.py:100-230`
(tantivy there); the service contract is `/search`, `/open`, `/health`.
"""
from __future__ import annotations

import re
from collections import Counter

import numpy as np

WORD = re.compile(r"[A-Za-z0-9]+")


def tokenize(text: str) -> list[str]:
    return [w.lower() for w in WORD.findall(text)]


class BM25Index:
    def __init__(self, docs: list[dict], k1: float = 0.9, b: float = 0.4):
        """docs: [{"docid", "title", "text"}]."""
        self.docs = docs
        self.k1, self.b = k1, b
        self.vocab: dict[str, int] = {}
        postings: dict[int, list] = {}
        lens = np.zeros(len(docs), dtype=np.float32)
        for d, doc in enumerate(docs):
            toks = tokenize(doc.get("title", "") + " " + doc.get("text", ""))
            lens[d] = len(toks)
            for w, c in Counter(toks).items():
                t = self.vocab.setdefault(w, len(self.vocab))
                postings.setdefault(t, []).append((d, c))
        self.doc_len = lens
        self.avg_len = float(lens.mean()) if len(lens) else 1.0
        ptr = np.zeros(len(self.vocab) + 1, dtype=np.int64)
        ids, tfs = [], []
        for t in range(len(self.vocab)):
            lst = postings.get(t, [])
            ptr[t + 1] = ptr[t] + len(lst)
            ids.extend(x[0] for x in lst)
            tfs.extend(x[1] for x in lst)
        self.ptr = ptr
        self.ids = np.asarray(ids, dtype=np.int64)
        self.tfs = np.asarray(tfs, dtype=np.float32)
        n = len(docs)
        df = np.diff(ptr).astype(np.float32)
        self.idf = np.log(1.0 + (n - df + 0.5) / (df + 0.5))
        self.by_id = {doc["docid"]: i for i, doc in enumerate(docs)}

    def search(self, query: str, k: int = 10) -> list[tuple[int, float]]:
        scores = np.zeros(len(self.docs), dtype=np.float32)
        for w in set(tokenize(query)):
            t = self.vocab.get(w)
            if t is None:
                continue
            a, b = self.ptr[t], self.ptr[t + 1]
            d = self.ids[a:b]
            tf = self.tfs[a:b]
            norm = self.k1 * (1 - self.b + self.b * self.doc_len[d] / self.avg_len)
            scores[d] += self.idf[t] * tf * (self.k1 + 1) / (tf + norm)
        if not scores.any():
            return []
        k = min(k, int((scores > 0).sum()))
        top = np.argpartition(-scores, k - 1)[:k]
        top = top[np.argsort(-scores[top])]
        return [(int(i), float(scores[i])) for i in top]
