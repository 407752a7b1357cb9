"""Serving-side callers of the engines (the reference's rngd_pd.serving): continuous batching."""
