"""ctypes binding of the C restatement oracle/c/oracle.c (test infrastructure only)."""
import ctypes
import os
import subprocess

import numpy as np

from oracle import synth_np as sy
from oracle.ref_np import Dims, LLAMA8B, inv_freq

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "_build", "liboracle.so")
_lib = None

_u16p = ctypes.POINTER(ctypes.c_uint16)
_i64p = ctypes.POINTER(ctypes.c_int64)
_f32p = ctypes.POINTER(ctypes.c_float)


def build():
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            build()
        L = ctypes.CDLL(LIB)
        L.orc_gauss_bf16.argtypes = [_u16p, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64,
                                     ctypes.c_uint64, ctypes.c_float]
        L.orc_uniform.argtypes = [_i64p, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64,
                                  ctypes.c_uint64, ctypes.c_uint64]
        L.orc_set_threads.argtypes = [ctypes.c_int]
        L.orc_get_threads.restype = ctypes.c_int
        L.orc_model_create.restype = ctypes.c_void_p
        L.orc_model_create.argtypes = [ctypes.c_int] * 7 + [ctypes.c_float, _f32p, ctypes.c_uint64,
                                                             ctypes.c_float]
        L.orc_model_free.argtypes = [ctypes.c_void_p]
        L.orc_decode_step.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, _i64p, _i64p,
                                      _u16p, _u16p, _f32p, _i64p, _f32p]
        L.orc_decode_step_rows.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, _i64p, _i64p,
                                           _u16p, _u16p, _f32p, _i64p, _f32p, ctypes.c_int, _u16p, _u16p]
        L.orc_prefill.argtypes = [ctypes.c_void_p, ctypes.c_int, _i64p, ctypes.c_int, _u16p, _u16p,
                                  _f32p, _i64p, _f32p]
        L.orc_kv_fill_lane.argtypes = [_u16p, _u16p] + [ctypes.c_int] * 6 + [ctypes.c_uint64,
                                                                             ctypes.c_int, ctypes.c_float]
        _lib = L
    return _lib


def _p(a, t):
    return a.ctypes.data_as(t)


def set_threads(n):
    lib().orc_set_threads(int(n))


def threads():
    return lib().orc_get_threads()


def gauss_bf16_bits(seed, tid, n, sigma, start=0):
    out = np.empty(n, np.uint16)
    lib().orc_gauss_bf16(_p(out, _u16p), seed, tid, start, n, float(sy.gauss_scale(sigma)))
    return out


class CModel:
    """Full synthetic model held by the C oracle (weights as bf16, ~16 GB at Llama-3.1-8B)."""

    def __init__(self, d: Dims = LLAMA8B, seed=0, sigma=0.02):
        self.d = d
        inv = inv_freq(d)
        self._inv = np.ascontiguousarray(inv)
        self.h = lib().orc_model_create(d.H, d.M, d.NH, d.NKV, d.HD, d.L, d.V, d.eps,
                                        _p(self._inv, _f32p), seed, float(sy.gauss_scale(sigma)))

    def close(self):
        if self.h:
            lib().orc_model_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:        # interpreter shutdown: the library may already be gone
            pass

    def new_cache(self, B, S):
        d = self.d
        shape = (d.L, B, d.NKV, S, d.HD)
        return np.zeros(shape, np.uint16), np.zeros(shape, np.uint16)

    def fill_lane(self, Kc, Vc, b, seed, length, sigma=1.0):
        d = self.d
        L, B, NKV, S, HD = Kc.shape
        lib().orc_kv_fill_lane(_p(Kc, _u16p), _p(Vc, _u16p), L, B, NKV, S, HD, b, seed, length,
                               float(sy.gauss_scale(sigma)))

    def decode_step(self, toks, pos, Kc, Vc, want_logits=True, want_hidden=False):
        d = self.d
        B, S = Kc.shape[1], Kc.shape[3]
        t = np.ascontiguousarray(toks, np.int64)
        p = np.ascontiguousarray(pos, np.int64)
        lg = np.empty((B, d.V), np.float32) if want_logits else None
        hid = np.empty((B, d.H), np.float32) if want_hidden else None
        nxt = np.empty(B, np.int64)
        lib().orc_decode_step(self.h, B, S, _p(t, _i64p), _p(p, _i64p), _p(Kc, _u16p), _p(Vc, _u16p),
                              _p(lg, _f32p) if lg is not None else None, _p(nxt, _i64p),
                              _p(hid, _f32p) if hid is not None else None)
        return nxt, lg, hid

    def decode_step_given_rows(self, toks, pos, Kc, Vc):
        """decode_step over a cache whose rows at pos[b] the caller has already written (kept as
        given); returns (next, logits, own_k, own_v), own_* = the bf16 rows this oracle computes
        for those positions, [L][B][NKV][HD] bits."""
        d = self.d
        B, S = Kc.shape[1], Kc.shape[3]
        t = np.ascontiguousarray(toks, np.int64)
        p = np.ascontiguousarray(pos, np.int64)
        lg = np.empty((B, d.V), np.float32)
        nxt = np.empty(B, np.int64)
        own_k = np.empty((d.L, B, d.NKV, d.HD), np.uint16)
        own_v = np.empty_like(own_k)
        lib().orc_decode_step_rows(self.h, B, S, _p(t, _i64p), _p(p, _i64p), _p(Kc, _u16p), _p(Vc, _u16p),
                                   _p(lg, _f32p), _p(nxt, _i64p), None, 1, _p(own_k, _u16p), _p(own_v, _u16p))
        return nxt, lg, own_k, own_v

    def prefill(self, toks, S, want_hidden=False):
        d = self.d
        t = np.ascontiguousarray(toks, np.int64)
        P = len(t)
        K = np.empty((d.L, d.NKV, d.HD, S), np.uint16)
        V = np.empty((d.L, d.NKV, S, d.HD), np.uint16)
        lg = np.empty(d.V, np.float32)
        nxt = np.empty(1, np.int64)
        hid = np.empty((P, d.H), np.float32) if want_hidden else None
        lib().orc_prefill(self.h, P, _p(t, _i64p), S, _p(K, _u16p), _p(V, _u16p), _p(lg, _f32p),
                          _p(nxt, _i64p), _p(hid, _f32p) if hid is not None else None)
        return K, V, lg, int(nxt[0]), hid
