"""ctypes binding of the C ABI in include/rngd_b200.h (the B200 kernels).

The product has no CPU or library fallback: importing this module without the
built ``_rngd_b200.so`` raises, and every call that returns a negative status
raises ``RngdError`` with the library's own message.
"""
import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_rngd_b200.so")

RNGD_OK = 0
RNGD_ERR_ARG = -1
RNGD_ERR_CUDA = -2
RNGD_ERR_TIMEOUT = -3
RNGD_ERR_UNSUPPORTED = -4


class RngdError(RuntimeError):
    def __init__(self, status, msg):
        super().__init__(f"rngd status {status}: {msg}")
        self.status = status


class RngdTimeout(RngdError, TimeoutError):
    pass


if not os.path.exists(LIB_PATH):
    raise ImportError(f"{LIB_PATH} is missing: build it with `make -C rngd-pd_b200/csrc` "
                      "(or __graft_entry__.build()); there is no fallback path")

lib = ctypes.CDLL(LIB_PATH)

_vp = ctypes.c_void_p
_i32 = ctypes.c_int32
_f32p = ctypes.POINTER(ctypes.c_float)


class Model(ctypes.Structure):
    """rngd_model_t"""
    _fields_ = [("H", _i32), ("M", _i32), ("NH", _i32), ("NKV", _i32), ("HD", _i32), ("L", _i32),
                ("V", _i32), ("eps", ctypes.c_float), ("wqkv", _vp), ("wo", _vp), ("wgu", _vp),
                ("wd", _vp), ("n1", _vp), ("n2", _vp), ("norm", _vp), ("embed", _vp), ("lm", _vp),
                ("inv_freq", _vp)]


class DecodeIO(ctypes.Structure):
    """rngd_decode_io_t"""
    _fields_ = [("B", _i32), ("Bcap", _i32), ("S", _i32), ("kv_layers", _i32), ("kcache", _vp), ("vcache", _vp),
                ("toks", _vp), ("pos", _vp), ("x", _vp), ("q", _vp), ("act", _vp), ("act_o", _vp),
                ("act2", _vp), ("ss", _vp), ("logits", _vp), ("attn_part", _vp), ("partial", _vp),
                ("counters", _vp), ("best", _vp), ("next", _vp), ("lanes", _vp)]


class PrefillIO(ctypes.Structure):
    """rngd_prefill_io_t"""
    _fields_ = [("C", _i32), ("P", _i32), ("S", _i32), ("kv_layers", _i32), ("kv", _vp), ("toks", _vp),
                ("x", _vp), ("q", _vp), ("act", _vp), ("act_o", _vp), ("act2", _vp), ("ss", _vp),
                ("partial", _vp), ("counters", _vp), ("operand_lo", _i32)]


def _sig(name, *args):
    f = getattr(lib, name)
    f.argtypes = list(args)
    f.restype = ctypes.c_int
    return f


_sig("rngd_last_error", ctypes.c_char_p, ctypes.c_size_t)
_sig("rngd_abi_version")
_sig("rngd_synth_gauss_bf16", _vp, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64,
     ctypes.c_float, _vp)
_sig("rngd_synth_uniform_i32", _vp, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64,
     ctypes.c_uint32, _vp)
_MP = ctypes.POINTER(Model)
_IOP = ctypes.POINTER(DecodeIO)
_sig("rngd_decode_embed", _MP, _IOP, _vp)
_sig("rngd_decode_layers", _MP, _IOP, ctypes.c_int, ctypes.c_int, _vp)
_sig("rngd_decode_begin", _MP, _IOP, ctypes.c_int, _vp)
_sig("rngd_decode_lmhead", _MP, _IOP, _vp)
_sig("rngd_decode_advance", _IOP, _vp)
_szp = ctypes.POINTER(ctypes.c_size_t)
_sig("rngd_decode_workspace", _MP, ctypes.c_int, _szp, _szp, _szp, _szp)
_sig("rngd_decode_attn_workspace", _MP, ctypes.c_int, ctypes.c_int, _szp)
_sig("rngd_tc_gemv", _vp, ctypes.c_int, ctypes.c_int, _vp, ctypes.c_int, ctypes.c_int, _vp, ctypes.c_int, _vp,
     _vp, _vp, ctypes.c_int, _vp)
_sig("rngd_tc_gemv_workspace", ctypes.c_int, ctypes.c_int, _szp, _szp)
_sig("rngd_tc_gemv_trace", _vp)
_sig("rngd_trace_decode_gemms", _vp, ctypes.c_int)
_PIOP = ctypes.POINTER(PrefillIO)
_sig("rngd_prefill_workspace", _MP, ctypes.c_int, _szp, _szp)
_sig("rngd_prefill_embed", _MP, _PIOP, _vp)
_sig("rngd_prefill_layers", _MP, _PIOP, ctypes.c_int, ctypes.c_int, _vp)
_sig("rngd_prefill_begin", _MP, _PIOP, ctypes.c_int, _vp)
_sig("rngd_lmhead_rows", _MP, _vp, ctypes.c_int, ctypes.c_int, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp)
_sig("rngd_lmhead_workspace", _MP, _szp, _szp)
_sig("rngd_tc_gemm_tokens", _vp, ctypes.c_int, ctypes.c_int, _vp, ctypes.c_int, _vp, _vp, _vp, _vp, ctypes.c_int,
     _vp)
_sig("rngd_tc_gemm_tokens_workspace", ctypes.c_int, ctypes.c_int, ctypes.c_int, _szp, _szp)
_sig("rngd_ipc_alloc", ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p), _vp)
_sig("rngd_ipc_free", _vp)
_sig("rngd_ipc_open", _vp, ctypes.POINTER(ctypes.c_void_p))
_sig("rngd_ipc_close", _vp)
_sig("rngd_ipc_handle_size")
_sig("rngd_peer_enable", ctypes.c_int, ctypes.c_int)
_sig("rngd_host_alloc_mapped", ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_void_p))
_sig("rngd_host_free", _vp)
_sig("rngd_kv_handoff", _vp, _vp, ctypes.c_size_t, _vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
     ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, _vp, _vp, ctypes.c_int64, _vp)
class KvItem(ctypes.Structure):
    _fields_ = [("src_k", ctypes.c_void_p), ("src_v", ctypes.c_void_p), ("lane", ctypes.c_int),
                ("tokens", ctypes.c_int), ("seq", ctypes.c_int64)]


KV_MAX_BATCH = 16
_sig("rngd_kv_handoff_batch", ctypes.POINTER(KvItem), ctypes.c_int, ctypes.c_size_t, _vp, _vp, ctypes.c_int,
     ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, _vp, _vp, _vp)
_sig("rngd_kv_wait", _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int64, ctypes.c_int64, _vp, _vp)
_sig("rngd_kv_read_flags", _vp, _vp, ctypes.c_size_t, _vp)
_sig("rngd_peer_copy", _vp, ctypes.c_int, _vp, ctypes.c_int, ctypes.c_size_t, _vp)
_sig("rngd_device_status", ctypes.POINTER(ctypes.c_int), ctypes.c_int)
_sig("rngd_gemv_bf16", _vp, ctypes.c_int, ctypes.c_int, _vp, ctypes.c_int, ctypes.c_int, _vp, ctypes.c_int,
     ctypes.c_int, _vp)
_sig("rngd_rmsnorm_f32", _vp, ctypes.c_int, ctypes.c_int, _vp, ctypes.c_float, _vp, _vp)
_sig("rngd_attn_decode", _vp, _vp, _vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
     ctypes.c_int, ctypes.c_int, _vp, _vp, _vp)
_sig("rngd_attn_decode_noalloc", _vp, _vp, _vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
     ctypes.c_int, ctypes.c_int, _vp, _vp)


def last_error():
    buf = ctypes.create_string_buffer(512)
    lib.rngd_last_error(buf, 512)
    return buf.value.decode(errors="replace")


def check(status):
    if status != RNGD_OK:
        msg = last_error()
        if status == RNGD_ERR_TIMEOUT:
            raise RngdTimeout(status, msg)
        raise RngdError(status, msg)
    return status


def call(name, *args):
    return check(getattr(lib, name)(*args))


def stream_handle(stream=None):
    """Raw cudaStream_t of a torch stream (the current one by default)."""
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


def ptr(t):
    """Device pointer of a torch tensor (None -> NULL)."""
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def device_status(reset=True):
    """Status word of the kernels' bounded waits: 0, or the code of the first wait that timed out."""
    st = ctypes.c_int(0)
    call("rngd_device_status", ctypes.byref(st), 1 if reset else 0)
    return st.value


def decode_workspace(model, S):
    out = [ctypes.c_size_t(0) for _ in range(4)]
    call("rngd_decode_workspace", ctypes.byref(model), S, *[ctypes.byref(o) for o in out])
    return [o.value for o in out]


def decode_attn_workspace(model, Bcap, S):
    out = ctypes.c_size_t(0)
    call("rngd_decode_attn_workspace", ctypes.byref(model), Bcap, S, ctypes.byref(out))
    return out.value


def exported_symbols():
    """Names declared in include/rngd_b200.h, for the ABI completeness test."""
    return [n for n in dir(lib) if n.startswith("rngd_")]


def on_device(fn):
    """Run an engine method with the engine's GPU current (`self.dev`, or `self.e.dev` for a
    helper object holding its engine as `e`), so streams, launches and the library's per-device
    state all agree when one process drives several GPUs."""
    import functools

    @functools.wraps(fn)
    def wrapped(self, *a, **k):
        import torch
        dev = getattr(self, "dev", None)
        if dev is None:
            dev = self.e.dev
        with torch.cuda.device(dev):
            return fn(self, *a, **k)
    return wrapped
