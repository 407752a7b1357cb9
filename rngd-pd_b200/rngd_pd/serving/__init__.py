"""Serving-side callers of the engines (the reference's rngd_pd.serving): continuous batching
(scheduler.py) and the in-process gateway over the pairings (gateway.py)."""
