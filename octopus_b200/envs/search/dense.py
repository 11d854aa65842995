"""Dense retrieval: exact maximum inner product over L2-normalised document embeddings.

Document vectors come from precomputed embedding files (pickles of ``(reps [n, d],
docids [n])``, the layout BrowseComp-Plus / OpenResearcher ship their indexes in); they
are L2-normalised and stored as fp16, on the GPU when one is given (a query is one
[d] x [d, n] product and a top-k), else on the host in row blocks.  Queries are encoded
by an embedding model the BrowseComp-Plus way: an instruction prefix, the last token's
final hidden state, L2 normalisation.

Reference parity (behaviour): `octopus/envs/search/service.py:83-125` (the query encoder
with its instruction prefix and last-token pooling; inner-product search over fp16
vectors normalised at load).
"""
from __future__ import annotations

import glob
import pickle

import numpy as np
import torch

QUERY_PREFIX = "Instruct: Given a web search query, retrieve relevant passages that answer the query\nQuery:"


class QueryEncoder:
    """An embedding model from a local Hugging Face checkpoint (no network): the query with
    the instruction prefix, left-padded, last-token hidden state, L2-normalised."""

    def __init__(self, path: str, device: str = "cpu", max_length: int = 512):
        import transformers

        self.device = torch.device(device)
        self.max_length = max_length
        self.tok = transformers.AutoTokenizer.from_pretrained(path, padding_side="left")
        dtype = torch.float32 if self.device.type == "cpu" else torch.float16
        self.model = transformers.AutoModel.from_pretrained(path, dtype=dtype).to(self.device).eval()

    @torch.no_grad()
    def __call__(self, query: str) -> np.ndarray:
        batch = self.tok([QUERY_PREFIX + query], truncation=True, max_length=self.max_length, return_tensors="pt")
        h = self.model(**batch.to(self.device)).last_hidden_state[:, -1].float()
        return torch.nn.functional.normalize(h, dim=-1).cpu().numpy()[0]


def load_embeddings(pattern: str) -> tuple[np.ndarray, list[str]]:
    """All (reps, docids) pickles matching `pattern`, concatenated in sorted file order."""
    reps, ids = [], []
    for f in sorted(glob.glob(pattern)):
        with open(f, "rb") as fh:
            r, d = pickle.load(fh)
        reps.append(np.asarray(r, dtype=np.float32))
        ids += [str(x) for x in d]
    if not reps:
        raise FileNotFoundError(f"no embedding files match {pattern}")
    return np.concatenate(reps), ids


class DenseIndex:
    """Exact inner-product search over normalised fp16 vectors."""

    def __init__(self, reps: np.ndarray, docids: list[str], device: str = "cpu", block: int = 1 << 18):
        self.docids = list(docids)
        self.device = torch.device(device)
        self.block = block
        x = torch.as_tensor(np.asarray(reps, dtype=np.float32))
        x = torch.nn.functional.normalize(x, dim=-1)
        self.vecs = x.to(self.device, torch.float16)

    def search(self, q: np.ndarray, k: int) -> list[tuple[int, float]]:
        """Top-k (row, score) for one query vector (normalised here)."""
        qv = torch.nn.functional.normalize(torch.as_tensor(np.asarray(q, np.float32)), dim=-1)
        k = max(1, min(int(k), len(self.docids)))
        if self.device.type == "cuda":
            s = (self.vecs @ qv.to(self.device, torch.float16)).float()
            val, idx = torch.topk(s, k)
            return list(zip(idx.cpu().tolist(), val.cpu().tolist()))
        best_v = torch.empty(0)
        best_i = torch.empty(0, dtype=torch.int64)
        for r0 in range(0, len(self.docids), self.block):  # host: row blocks, running top-k
            s = self.vecs[r0:r0 + self.block].float() @ qv
            v, i = torch.topk(s, min(k, len(s)))
            best_v = torch.cat([best_v, v])
            best_i = torch.cat([best_i, i + r0])
            keep = torch.topk(best_v, min(k, len(best_v)))
            best_v, best_i = keep.values, best_i[keep.indices]
        return list(zip(best_i.tolist(), best_v.tolist()))
