"""Test helpers (re-exported from the oracle's block adapters)."""

from oracle.blocks import gptq_oracle_weights, oracle_weights  # noqa: F401
