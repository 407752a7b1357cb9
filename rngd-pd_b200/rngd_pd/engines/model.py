"""Model configuration (same fields and RoPE rule as src/rngd_pd/engines/model.py:15-50).

The reference module also carries a numpy runtime (GenericRuntime); that is a
CPU implementation and lives with the test oracle (oracle/ref_np.py), not in
the product.
"""
import math
from types import SimpleNamespace

import numpy as np


class ModelConfig:
    """Dims, eps, theta and llama3 rope scaling from an HF config (engines/model.py:15-30)."""

    def __init__(self, hf):
        self.n_layers = hf.num_hidden_layers
        self.hidden = hf.hidden_size
        self.n_heads = hf.num_attention_heads
        self.n_kv = getattr(hf, "num_key_value_heads", self.n_heads)
        self.head_dim = getattr(hf, "head_dim", None) or self.hidden // self.n_heads
        self.inter = hf.intermediate_size
        self.eps = getattr(hf, "rms_norm_eps", 1e-6)
        self.vocab = hf.vocab_size
        self.tie = getattr(hf, "tie_word_embeddings", False)
        rs = getattr(hf, "rope_scaling", None) or {}
        self.theta = getattr(hf, "rope_theta", None) or rs.get("rope_theta") or 10000.0
        self.rope_scaling = rs if rs.get("rope_type") == "llama3" else None
        self.gqa = self.n_heads // self.n_kv

    def inv_freq(self):
        """fp32 inverse frequencies, float64 power cast once (engines/model.py:32-50)."""
        d = self.head_dim
        inv = 1.0 / (self.theta ** (np.arange(0, d, 2, dtype=np.float64) / d))
        rs = self.rope_scaling
        if rs:
            factor, lo, hi, orig = (rs["factor"], rs["low_freq_factor"], rs["high_freq_factor"],
                                    rs["original_max_position_embeddings"])
            low_wl, high_wl = orig / lo, orig / hi
            wl = 2 * math.pi / inv
            out = inv.copy()
            for i, w in enumerate(wl):
                if w > low_wl:
                    out[i] = inv[i] / factor
                elif w < high_wl:
                    out[i] = inv[i]
                else:
                    s = (orig / w - lo) / (hi - lo)
                    out[i] = (1 - s) * inv[i] / factor + s * inv[i]
            inv = out
        return inv.astype(np.float32)

    @classmethod
    def from_dims(cls, H=4096, M=14336, NH=32, NKV=8, HD=128, L=32, V=128256, eps=1e-5, theta=500000.0):
        return cls(SimpleNamespace(num_hidden_layers=L, hidden_size=H, num_attention_heads=NH,
                                   num_key_value_heads=NKV, head_dim=HD, intermediate_size=M,
                                   rms_norm_eps=eps, vocab_size=V, tie_word_embeddings=False,
                                   rope_theta=theta, rope_scaling=None))

    @classmethod
    def llama31_8b(cls):
        """Llama-3.1-8B shape as BASELINE.json states it (RoPE theta 5e5, no llama3 scaling)."""
        return cls.from_dims()
