"""Weights in the HBM layout the B200 kernels stream.

One contiguous bf16 block per kind over all layers, rows K-major (the HF
[out, in] layout), so a GEMV/GEMM tile is a run of whole rows:

  wqkv [L][(NH+2*NKV)*HD][H]   q, k, v projections concatenated (one fused GEMV)
  wo   [L][H][NH*HD]
  wgu  [L][2*M][H]             gate/up interleaved in 64-row blocks, so a 128-row
                               tile holds the gate and up rows of the same 64
                               features (SwiGLU fuses into its epilogue)
  wd   [L][H][M]
  n1, n2 [L][H], norm [H] fp32; embed, lm [V][H] bf16; inv_freq [HD/2] fp32

Unlike the reference (src/rngd_pd/engines/decode_batch.py:194-219), q is not
pre-scaled by 1/sqrt(HD) nor the norms by sqrt(H): both are applied in fp32
inside the kernels, so the bf16 weights are exactly the checkpoint's.
"""
import numpy as np
import torch

from rngd_pd import synth

BF = torch.bfloat16

_HF = {synth.T_Q: "self_attn.q_proj", synth.T_K: "self_attn.k_proj", synth.T_V: "self_attn.v_proj",
       synth.T_O: "self_attn.o_proj", synth.T_GATE: "mlp.gate_proj", synth.T_UP: "mlp.up_proj",
       synth.T_DOWN: "mlp.down_proj"}


def _dev_bf16(a, device):
    if torch.is_tensor(a):
        return a.to(device=device, dtype=BF)
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(device).to(BF)


def _dev_f32(a, device):
    if torch.is_tensor(a):
        return a.to(device=device, dtype=torch.float32)
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(device)


class DeviceWeights:
    """All weights of one model on one device; shared by every engine width on that card."""

    def __init__(self, cfg, sd, device):
        self.cfg, self.device = cfg, torch.device(device)
        c = cfg
        L, H, M, V = c.n_layers, c.hidden, c.inter, c.vocab
        QN, KN = c.n_heads * c.head_dim, c.n_kv * c.head_dim
        self.NQKV = QN + 2 * KN
        dev = self.device
        self.wqkv = torch.empty((L, self.NQKV, H), dtype=BF, device=dev)
        self.wo = torch.empty((L, H, QN), dtype=BF, device=dev)
        self.wgu = torch.empty((L, 2 * M, H), dtype=BF, device=dev)
        self.wd = torch.empty((L, H, M), dtype=BF, device=dev)
        self.n1 = torch.empty((L, H), dtype=torch.float32, device=dev)
        self.n2 = torch.empty((L, H), dtype=torch.float32, device=dev)
        self.inv_freq = torch.from_numpy(cfg.inv_freq()).to(dev)
        if isinstance(sd, synth.SyntheticState):
            self._fill_synthetic(sd)
        else:
            self._fill_from_state_dict(sd)
        torch.cuda.synchronize(dev)

    # -- sources -----------------------------------------------------------
    def _fill_synthetic(self, st):
        c, dev = self.cfg, self.device
        L, H, M, V = c.n_layers, c.hidden, c.inter, c.vocab
        QN, KN = c.n_heads * c.head_dim, c.n_kv * c.head_dim
        s, sg = st.seed, st.sigma
        tmp = torch.empty((M, H), dtype=BF, device=dev)
        with torch.cuda.device(dev):
            for l in range(L):
                t = lambda k: l * 16 + k
                synth.fill_gauss(self.wqkv[l, :QN], s, t(synth.T_Q), sg)
                synth.fill_gauss(self.wqkv[l, QN:QN + KN], s, t(synth.T_K), sg)
                synth.fill_gauss(self.wqkv[l, QN + KN:], s, t(synth.T_V), sg)
                synth.fill_gauss(self.wo[l], s, t(synth.T_O), sg)
                gu = self.wgu[l].view(M // 64, 2, 64, H)
                synth.fill_gauss(tmp, s, t(synth.T_GATE), sg)
                gu[:, 0].copy_(tmp.view(M // 64, 64, H))
                synth.fill_gauss(tmp, s, t(synth.T_UP), sg)
                gu[:, 1].copy_(tmp.view(M // 64, 64, H))
                synth.fill_gauss(self.wd[l], s, t(synth.T_DOWN), sg)
            self.n1.fill_(1.0)
            self.n2.fill_(1.0)
            self.norm = torch.ones(H, dtype=torch.float32, device=dev)
            self.embed = synth.fill_gauss(torch.empty((V, H), dtype=BF, device=dev), s, synth.T_EMBED, sg)
            self.lm = synth.fill_gauss(torch.empty((V, H), dtype=BF, device=dev), s, synth.T_LMHEAD, sg)
        del tmp

    def _fill_from_state_dict(self, sd):
        c, dev = self.cfg, self.device
        L, H, M = c.n_layers, c.hidden, c.inter
        QN, KN = c.n_heads * c.head_dim, c.n_kv * c.head_dim
        for l in range(L):
            p = lambda k: sd[f"model.layers.{l}.{_HF[k]}.weight"]
            self.wqkv[l, :QN] = _dev_bf16(p(synth.T_Q), dev)
            self.wqkv[l, QN:QN + KN] = _dev_bf16(p(synth.T_K), dev)
            self.wqkv[l, QN + KN:] = _dev_bf16(p(synth.T_V), dev)
            self.wo[l] = _dev_bf16(p(synth.T_O), dev)
            gu = self.wgu[l].view(M // 64, 2, 64, H)
            gu[:, 0] = _dev_bf16(p(synth.T_GATE), dev).view(M // 64, 64, H)
            gu[:, 1] = _dev_bf16(p(synth.T_UP), dev).view(M // 64, 64, H)
            self.wd[l] = _dev_bf16(p(synth.T_DOWN), dev)
            self.n1[l] = _dev_f32(sd[f"model.layers.{l}.input_layernorm.weight"], dev)
            self.n2[l] = _dev_f32(sd[f"model.layers.{l}.post_attention_layernorm.weight"], dev)
        self.norm = _dev_f32(sd["model.norm.weight"], dev)
        self.embed = _dev_bf16(sd["model.embed_tokens.weight"], dev)
        self.lm = self.embed if c.tie else _dev_bf16(sd["lm_head.weight"], dev)

    # -- C ABI view ----------------------------------------------------------
    def model_struct(self):
        from rngd_pd import _lib
        c = self.cfg
        p = lambda t: t.data_ptr()
        return _lib.Model(H=c.hidden, M=c.inter, NH=c.n_heads, NKV=c.n_kv, HD=c.head_dim, L=c.n_layers,
                          V=c.vocab, eps=c.eps, wqkv=p(self.wqkv), wo=p(self.wo), wgu=p(self.wgu),
                          wd=p(self.wd), n1=p(self.n1), n2=p(self.n2), norm=p(self.norm),
                          embed=p(self.embed), lm=p(self.lm), inv_freq=p(self.inv_freq))

    def nbytes_per_step(self):
        """Algorithmic weight bytes a decode step streams: 32 layers + lm_head."""
        t = [self.wqkv, self.wo, self.wgu, self.wd, self.lm]
        return sum(x.numel() * x.element_size() for x in t)
