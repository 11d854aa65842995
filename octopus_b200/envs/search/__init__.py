"""Offline deep-search environment: BM25 retrieval service, search agent workspace,
answer grading, and a CPU dry run with fake retrieval and a stub policy."""
