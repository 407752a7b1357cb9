"""The reference's kernel modules (src/rngd_pd/kernels/): DecodeModel / rot_batch
(decode_batch), PrefillModel (prefill_full) and ChunkModel / rot_matrices (prefill_chunk), as
torch modules over the B200 C ABI that take the reference's graph inputs.  The reference's CPU
fp32 functions of these modules (cpu_layer, cpu_layer_p) are its numeric check, restated in
this repository's test oracle, not part of the product."""
