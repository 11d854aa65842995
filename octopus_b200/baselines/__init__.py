"""Reproductions of external baselines the reference compares against (route_a: ways of
letting one branch read a sibling's context)."""
