"""Evaluation harnesses (no training): agent-runtime episodes and the synthetic DAG."""
