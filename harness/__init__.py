"""Model-level harness (measurement and parity infrastructure; see harness/model.py)."""
