"""Seeded synthetic tensors, numpy restatement (test infrastructure only).

The reference measures on a real Llama-3.1-8B checkpoint that is absent here;
BASELINE.json asks for random-init bf16 weights ~N(0, 0.02), seeded bf16 KV
~N(0, 1) and uniform token ids.  Every generator in this build (the CUDA one in
rngd-pd_b200/csrc/synth.cu, the C one in oracle/c/oracle.c and this one) follows
ONE integer-only recipe so the three agree bit for bit:

  mix(x)        splitmix64 finaliser: z = x + 0x9E3779B97F4A7C15;
                z = (z ^ z>>30) * 0xBF58476D1CE4E5B9; z = (z ^ z>>27) *
                0x94D049BB133111EB; z ^ z>>31          (all mod 2**64)
  key(seed,tid) mix(mix(seed) ^ tid)
  h(i)          mix(key + i)                          i = flat element index
  gaussian      s = sum of the four 16-bit fields of h(i)  (Irwin-Hall, n=4)
                f = float32(s - 131070) * float32(sigma / sqrt(4*(65536**2-1)/12))
                bf16 = round-to-nearest-even of f's upper 16 bits
  uniform int   (h(i) >> 32) % n

No transcendental function is involved, so host and device results are equal
by construction (the fp32 product of an exact integer and an fp32 constant is
correctly rounded on both).
"""
import math

import numpy as np

_C1 = np.uint64(0x9E3779B97F4A7C15)
_C2 = np.uint64(0xBF58476D1CE4E5B9)
_C3 = np.uint64(0x94D049BB133111EB)

# tensor ids of the synthetic Llama state dict (also in csrc/synth.cu and oracle/c/oracle.c)
T_Q, T_K, T_V, T_O, T_GATE, T_UP, T_DOWN = range(7)
T_EMBED = 0x7000
T_LMHEAD = 0x7001
T_KCACHE = 0x8000
T_VCACHE = 0x8001
T_TOKENS = 0x9000
T_CTXLEN = 0x9001


def layer_tid(layer, kind):
    return layer * 16 + kind


def mix(x):
    with np.errstate(over="ignore"):
        z = np.asarray(x, dtype=np.uint64) + _C1
        z = (z ^ (z >> np.uint64(30))) * _C2
        z = (z ^ (z >> np.uint64(27))) * _C3
        return z ^ (z >> np.uint64(31))


def stream_key(seed, tid):
    return mix(mix(np.uint64(seed)) ^ np.uint64(tid))


def hashes(seed, tid, start, n):
    with np.errstate(over="ignore"):
        return mix(stream_key(seed, tid) + np.arange(start, start + n, dtype=np.uint64))


def gauss_scale(sigma):
    """fp32 multiplier that gives the Irwin-Hall(4) sum a standard deviation of sigma."""
    return np.float32(sigma / math.sqrt(4.0 * (65536.0 ** 2 - 1.0) / 12.0))


def f32_to_bf16_bits(f):
    """Round-to-nearest-even fp32 -> bf16, as uint16 bits (finite inputs)."""
    u = np.ascontiguousarray(f, dtype=np.float32).view(np.uint32)
    with np.errstate(over="ignore"):
        r = (u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)
    return r.astype(np.uint16)


def bf16_bits_to_f32(b):
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def bf16_round(f):
    """fp32 array rounded to the nearest bf16 value, returned as fp32."""
    return bf16_bits_to_f32(f32_to_bf16_bits(f))


def gauss_bf16_bits(seed, tid, n, sigma, start=0):
    h = hashes(seed, tid, start, n)
    m = np.uint64(0xFFFF)
    s = ((h & m) + ((h >> np.uint64(16)) & m) + ((h >> np.uint64(32)) & m)
         + (h >> np.uint64(48))).astype(np.int64) - 131070
    f = s.astype(np.float32) * gauss_scale(sigma)
    return f32_to_bf16_bits(f)


def gauss_bf16(seed, tid, shape, sigma, start=0):
    """bf16-valued fp32 array of the given shape (flat index = C order)."""
    n = int(np.prod(shape))
    return bf16_bits_to_f32(gauss_bf16_bits(seed, tid, n, sigma, start)).reshape(shape)


def uniform_ints(seed, tid, n, hi, start=0):
    h = hashes(seed, tid, start, n)
    return ((h >> np.uint64(32)) % np.uint64(hi)).astype(np.int64)
