"""KV handoff over the vLLM KVConnector interface (the reference's rngd_pd.connector)."""
