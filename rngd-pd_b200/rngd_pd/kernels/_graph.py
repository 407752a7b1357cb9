"""What the three kernel modules share: the reference's compiled-graph calling convention
(src/rngd_pd/kernels/decode_batch.py:56-109, prefill_full.py:36-94, prefill_chunk.py:117-180)
mapped onto this library's layer calls.

The reference feeds its NPU graph the weights of a layer group as inputs, prepared by its
engines (src/rngd_pd/engines/decode_batch.py:194-233):
  * projections transposed to [in, out] (wqT, wkT, ...), q pre-scaled by 1/sqrt(HD);
  * RMSNorm weights tiled to one row per stream and pre-scaled by sqrt(H), with eps passed
    as eps*H and the exponent as nh = -0.5 (so rms = x * n / sqrt(sum x^2 + eps*H));
  * RoPE as a rotation matrix per stream, the new K/V column as a one-hot row and the
    causal limit as an additive mask.
The B200 kernels stream K-major weight rows ([out, in], gate/up interleaved in 64-row
blocks), apply 1/sqrt(HD) and the norm in fp32 themselves, compute RoPE from the position
and keep both caches as [L][lane][NKV][S][HD].  `PackedGroup` converts a group's weights
once (packed copies are cached by the identity and version of the input tensors, so a
caller that passes the same resident weights every step pays the conversion once) and
`check_*` turn the one-hot / mask / rotation inputs back into positions, failing loudly
when they are not the decode contract's (one position per stream, causal up to it, the
rotation for that position, an empty cache slot there).
"""
import collections
import math

import numpy as np
import torch

from rngd_pd import _lib

BF = torch.bfloat16
H, M, NH, NKV, HD = 4096, 14336, 32, 8, 128      # Llama-3.1-8B, as the reference modules fix them
G = NH // NKV
# NPU compiler knobs of the reference modules: importable for its callers, unused here (the
# kernels are compiled ahead of time; there is no tactic search or shape cap)
HINT = "ForLlmModelDecode"
MAX_SHAPES = {}

_ROT_TOL = 2e-2          # rotation entries arrive as bf16 (8 bits of mantissa)


def default_inv(theta=500000.0, head_dim=HD):
    """RoPE inverse frequencies 1 / theta^(2i/HD), float64 power cast to fp32."""
    return (1.0 / (theta ** (np.arange(0, head_dim, 2, dtype=np.float64) / head_dim))).astype(np.float32)


def rotation_tables(inv, positions):
    """[n, HD, HD] fp32 block rotations, one per position: the matrix R with x @ R equal to the
    rotate-half RoPE of x at that position (the layout the reference's graphs multiply by).
    The angle is positions * inv in numpy's promotion of the two: integer positions give float64
    angles (as the reference's decode and prefill tables), float32 positions float32 angles (as
    its chunk table); cos and sin are rounded to fp32 afterwards."""
    inv = np.asarray(inv, np.float32)
    half = inv.shape[0]
    ang = np.asarray(positions)[:, None] * inv[None, :]
    cos, sin = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    out = np.zeros((len(ang), 2 * half, 2 * half), np.float32)
    idx = np.arange(half)
    out[:, idx, idx] = cos
    out[:, idx + half, idx + half] = cos
    out[:, idx, idx + half] = sin
    out[:, idx + half, idx] = -sin
    return out


def _rotations_device(inv_t, pos_t):
    """rotation_tables on the device, for checking a caller's rotation input."""
    ang = pos_t.to(torch.float32)[:, None] * inv_t[None, :]
    cos, sin = torch.cos(ang), torch.sin(ang)
    half = inv_t.shape[0]
    out = torch.zeros((pos_t.shape[0], 2 * half, 2 * half), dtype=torch.float32, device=inv_t.device)
    idx = torch.arange(half, device=inv_t.device)
    out[:, idx, idx] = cos
    out[:, idx + half, idx + half] = cos
    out[:, idx, idx + half] = sin
    out[:, idx + half, idx] = -sin
    return out


def stacked(t):
    """A group input given as one stacked tensor or as a list of per-layer tensors."""
    return t if torch.is_tensor(t) else torch.stack(list(t))


class Dims:
    """Model dimensions read off a group's inputs (H from x, heads from the projections)."""

    def __init__(self, x, aq, ak, awg, head_dim):
        self.H = int(x.shape[-1])
        self.HD = int(head_dim)
        self.QN, self.KN = int(aq.shape[-1]), int(ak.shape[-1])
        self.NH, self.NKV = self.QN // self.HD, self.KN // self.HD
        self.M = int(awg.shape[-1])
        if self.HD != 128 or self.NH != 4 * self.NKV or self.H % 128 or self.M % 64:
            raise ValueError(f"the B200 kernels take HD=128, NH=4*NKV, H % 128 == 0, M % 64 == 0; got "
                             f"H={self.H} HD={self.HD} NH={self.NH} NKV={self.NKV} M={self.M}")


class PackedGroup:
    """One layer group's weights in the kernels' HBM layout, built from the reference's graph
    inputs, plus the rngd_model_t that describes them (L = the group's layer count)."""

    def __init__(self, dims, an1, aq, ak, av, ao, an2, awg, awu, awd, eps, inv, device):
        d, dev = dims, device
        nl = aq.shape[0]
        self.nl, self.dims = nl, d
        sqrt_h, sqrt_hd = math.sqrt(d.H), math.sqrt(d.HD)
        self.wqkv = torch.empty((nl, d.QN + 2 * d.KN, d.H), dtype=BF, device=dev)
        self.wo = torch.empty((nl, d.H, d.QN), dtype=BF, device=dev)
        self.wgu = torch.empty((nl, 2 * d.M, d.H), dtype=BF, device=dev)
        self.wd = torch.empty((nl, d.H, d.M), dtype=BF, device=dev)
        self.n1 = torch.empty((nl, d.H), dtype=torch.float32, device=dev)
        self.n2 = torch.empty((nl, d.H), dtype=torch.float32, device=dev)
        for l in range(nl):
            # q: the reference folded 1/sqrt(HD) into the weight; the kernels apply it in fp32
            self.wqkv[l, :d.QN] = (aq[l].to(dev, torch.float32) * sqrt_hd).t().to(BF)
            self.wqkv[l, d.QN:d.QN + d.KN] = ak[l].to(dev).t()
            self.wqkv[l, d.QN + d.KN:] = av[l].to(dev).t()
            self.wo[l] = ao[l].to(dev).t()
            gu = self.wgu[l].view(d.M // 64, 2, 64, d.H)
            gu[:, 0] = awg[l].to(dev).t().reshape(d.M // 64, 64, d.H)
            gu[:, 1] = awu[l].to(dev).t().reshape(d.M // 64, 64, d.H)
            self.wd[l] = awd[l].to(dev).t()
            # norms arrive tiled per row and scaled by sqrt(H); every row must be the same
            for src, dst in ((an1[l], self.n1[l]), (an2[l], self.n2[l])):
                rows = src.to(dev, torch.float32).reshape(-1, d.H)
                if not torch.equal(rows, rows[:1].expand_as(rows)):
                    raise ValueError("norm inputs must tile one weight row per stream")
                dst.copy_(rows[0] / sqrt_h)
        self.norm = torch.ones(d.H, dtype=torch.float32, device=dev)     # unused after the last layer
        self.vocab = 128                                                  # no lm_head in a layer group
        self.lm = torch.zeros((self.vocab, d.H), dtype=BF, device=dev)
        self.inv = torch.as_tensor(np.asarray(inv, np.float32)).to(dev)
        self.eps = float(eps)
        p = lambda t: t.data_ptr()
        self.model = _lib.Model(H=d.H, M=d.M, NH=d.NH, NKV=d.NKV, HD=d.HD, L=nl, V=self.vocab, eps=self.eps,
                                wqkv=p(self.wqkv), wo=p(self.wo), wgu=p(self.wgu), wd=p(self.wd), n1=p(self.n1),
                                n2=p(self.n2), norm=p(self.norm), embed=p(self.lm), lm=p(self.lm),
                                inv_freq=p(self.inv))


class PackCache:
    """Packed groups keyed by the identity, version and shape of their input tensors, least
    recently used first out.  Capacity in groups (a 32-layer model in groups of 8 is 4)."""

    def __init__(self, capacity=8):
        self.capacity = int(capacity)
        self._groups = collections.OrderedDict()

    @staticmethod
    def _key(tensors, eps, inv, device):
        ident = tuple((t.data_ptr(), t._version, tuple(t.shape), t.dtype) for t in tensors)
        return ident + (float(eps), np.asarray(inv, np.float32).tobytes(), str(device))

    def get(self, dims, weights, eps, inv, device):
        key = self._key(weights, eps, inv, device)
        group = self._groups.get(key)
        if group is None:
            group = PackedGroup(dims, *weights, eps, inv, device)
            self._groups[key] = group
            while len(self._groups) > self.capacity:
                self._groups.popitem(last=False)
        else:
            self._groups.move_to_end(key)
        return group


def scalar_eps(eps_t, nh_t, H_):
    """eps from the reference's eps*H tensor, after checking it and nh (= -0.5) are uniform."""
    e = eps_t.to(torch.float32)
    n = nh_t.to(torch.float32)
    lo, hi = torch.aminmax(e)
    nlo, nhi = torch.aminmax(n)
    vals = torch.stack([lo, hi, nlo, nhi]).cpu().tolist()
    if vals[0] != vals[1] or vals[2] != -0.5 or vals[3] != -0.5:
        raise ValueError("eps must be eps*H tiled and nh must be -0.5 everywhere (the reference's rms inputs)")
    return vals[0] / H_


def check_rows(pos, onehot, mask_rows, rot, inv_t, cache_k, cache_v, S):
    """Device-side checks of the decode contract; one host sync.

    pos [R] int64 positions read off `onehot` [R, S]; mask_rows [R, S] must be 0 up to and
    including pos and <= -1e3 after it; rot [R, HD, HD] the rotation of pos (within bf16
    rounding); cache_k / cache_v (optional) must be zero at pos (the slot the step writes)."""
    R = pos.shape[0]
    ar = torch.arange(S, device=pos.device)
    oh = onehot.to(torch.float32)
    ok = [(oh.sum(-1) == 1).all(), (oh.gather(1, pos[:, None]) == 1).all()]
    m = mask_rows.to(torch.float32)
    upto = ar[None, :] <= pos[:, None]
    ok += [(m[upto] == 0).all(), (m[~upto] <= -1e3).all()]
    want = _rotations_device(inv_t, pos)
    ok.append(((rot.to(torch.float32) - want).abs().max() <= _ROT_TOL) if R else torch.tensor(True))
    if cache_k is not None:
        ok += [(cache_k == 0).all(), (cache_v == 0).all()]
    flags = torch.stack([t.to(torch.bool).reshape(()) for t in ok]).cpu().tolist()
    names = ["one-hot rows", "one-hot at the position", "mask zero up to the position",
             "mask negative after the position", "rotation of the position", "empty K slot", "empty V slot"]
    bad = [n for n, f in zip(names, flags) if not f]
    if bad:
        raise ValueError("inputs outside the decode contract the B200 kernels implement: " + ", ".join(bad))
