"""rngd-pd hot path on B200: batched decode, prefill_full and the KV handoff.

The reference package's module layout and entry points for that path:
  rngd_pd.kernels     DecodeModel / rot_batch, PrefillModel, ChunkModel / rot_matrices
                      (the reference's graph inputs, run by the B200 kernels)
  rngd_pd.engines     BatchDecodeEngine, FullPrefillEngine, ChunkPrefillEngine, TieredDecode
  rngd_pd.connector   RngdKVConnector, the transports and their wire formats
  rngd_pd.airm        the rm-core KV transports and the serving metrics
  rngd_pd.serving     continuous batching, the gateway, the PD box, the worker glue
plus rngd_pd.nvlink, the NVLink peer-to-peer KV transport.  Host code is Python/PyTorch
(device memory, streams, torch.distributed plumbing); every hot op is a hand-written sm_100a
kernel in _rngd_b200.so reached through the C ABI of include/rngd_b200.h.
"""
