"""CPU restatement of rngd-pd's hot path (decode step, prefill_full, KV wire).

TEST INFRASTRUCTURE ONLY.  This package is the checker, never the thing
measured or shipped: only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import it.
The product package (``rngd_pd``) never imports anything from here and fails
loudly when its CUDA library is missing.

Parity is pinned: ``tests/golden/make_golden.py`` runs the reference's own
CPU functions (``cpu_layer`` from src/rngd_pd/kernels/decode_batch.py:126-161,
``cpu_layer_p`` from src/rngd_pd/kernels/prefill_full.py:97-128, ``cpu_layer``
from src/rngd_pd/kernels/prefill_chunk.py:198-232, ``rot_batch``,
``GenericRuntime`` from src/rngd_pd/engines/model.py, ``ser``/``deser`` from
src/rngd_pd/connector/transport.py:29-43) on seeded inputs and commits their
outputs as fixtures; ``tests/test_oracle_pin.py`` checks this restatement
against them.

Modules
  synth_np   seeded synthetic tensors (bit-exact spec shared with the CUDA
             generator and the C oracle)
  ref_np     numpy fp32 restatement of the reference's layer functions
  corc       ctypes binding of the C restatement (oracle/c/oracle.c), used at
             full Llama-3.1-8B size where numpy would need 32 GB of fp32
             weights
"""
