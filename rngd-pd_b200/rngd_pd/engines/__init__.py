"""Weights on the device, KV placement, a step API (the reference's rngd_pd.engines)."""
