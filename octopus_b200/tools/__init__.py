"""Command-line tools: kernel benchmarks, probes and replays."""
