"""Model-level kernel entry points (the reference's rngd_pd.kernels)."""
