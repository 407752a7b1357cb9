"""rngd-pd hot path on B200: batched decode, prefill_full and the KV handoff.

Same module layout and entry points as the reference package (rngd_pd.kernels,
rngd_pd.engines, rngd_pd.connector, rngd_pd.airm) plus rngd_pd.nvlink, the
NVLink peer-to-peer KV transport.  Host code is Python/PyTorch (device memory,
streams, torch.distributed plumbing); every hot op is a hand-written sm_100a
kernel in _rngd_b200.so reached through the C ABI of include/rngd_b200.h.
"""
