"""Evaluation helpers (instruction-following checks) used by the root ``eval_ifeval.py``."""
