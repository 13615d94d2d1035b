"""ctypes wrapper of liboracle.so — TEST INFRASTRUCTURE ONLY.

The CPU F32 restatement of the reference's CPU path (oracle.cpp). Imported by
tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg, as the checker
or as the timed CPU baseline; the product never imports it.
"""
import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"

_f32p = ctypes.POINTER(ctypes.c_float)
_i32p = ctypes.POINTER(ctypes.c_int32)
_i64p = ctypes.POINTER(ctypes.c_int64)
_lib = None


def build() -> Path:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB


def lib():
    global _lib
    if _lib is None:
        if not LIB.exists():
            build()
        L = ctypes.CDLL(str(LIB))
        L.oracle_last_error.restype = ctypes.c_char_p
        L.oracle_model_create.restype = ctypes.c_void_p
        L.oracle_model_create.argtypes = [ctypes.c_void_p]
        L.oracle_model_destroy.argtypes = [ctypes.c_void_p]
        L.oracle_model_set_weight.argtypes = [ctypes.c_void_p, ctypes.c_char_p, _f32p, ctypes.c_int64]
        L.oracle_model_weight_count.argtypes = [ctypes.c_void_p, ctypes.c_char_p]
        L.oracle_model_weight_count.restype = ctypes.c_int64
        L.oracle_model_num_weights.argtypes = [ctypes.c_void_p]
        L.oracle_model_weight_name.argtypes = [ctypes.c_void_p, ctypes.c_int]
        L.oracle_model_weight_name.restype = ctypes.c_char_p
        L.oracle_model_check.argtypes = [ctypes.c_void_p]
        L.oracle_model_prefill.argtypes = [ctypes.c_void_p, _i32p, ctypes.c_int64, ctypes.c_void_p,
                                           ctypes.c_int64, _f32p, ctypes.POINTER(ctypes.c_void_p)]
        L.oracle_prefix_tokens.argtypes = [ctypes.c_void_p]
        L.oracle_prefix_tokens.restype = ctypes.c_int64
        L.oracle_prefix_bytes.argtypes = [ctypes.c_void_p]
        L.oracle_prefix_bytes.restype = ctypes.c_int64
        L.oracle_prefix_destroy.argtypes = [ctypes.c_void_p]
        L.oracle_linear.argtypes = [_f32p, ctypes.c_int64, _f32p, ctypes.c_int64, ctypes.c_int64, _f32p]
        L.oracle_rms.argtypes = [_f32p, _f32p, ctypes.c_int64, ctypes.c_int64, ctypes.c_float, _f32p]
        L.oracle_conv4.argtypes = [_f32p, ctypes.c_int64, ctypes.c_int64, _f32p, _f32p]
        L.oracle_delta_recurrence.argtypes = [_f32p, _f32p, _f32p, _f32p, _f32p, ctypes.c_int64,
                                              ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                              _f32p, ctypes.c_int64, _f32p, _f32p]
        L.oracle_attention.argtypes = [_f32p, _f32p, _f32p, ctypes.c_int, ctypes.c_int,
                                       ctypes.c_int64, ctypes.c_int64, ctypes.c_int, ctypes.c_int, _f32p]
        L.oracle_rotary.argtypes = [_f32p, ctypes.c_int64, ctypes.c_int, ctypes.c_int, _i64p,
                                    ctypes.c_int, ctypes.c_double]
        L.oracle_head.argtypes = [_f32p, _f32p, ctypes.c_int, ctypes.c_int, _f32p]
        L.oracle_set_threads.argtypes = [ctypes.c_int]
        L.oracle_max_threads.restype = ctypes.c_int
        L.oracle_set_rounding.argtypes = [ctypes.c_int]
        _lib = L
    return _lib


def _p(a: np.ndarray, t=_f32p):
    assert a.flags.c_contiguous
    return a.ctypes.data_as(t)


def f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def set_threads(n: int) -> None:
    lib().oracle_set_threads(int(n))


def max_threads() -> int:
    return int(lib().oracle_max_threads())


# BF16 rounding points of oracle.cpp (kRound*): 0 is the reference's F32 path.
ROUND_OPERAND, ROUND_PROJ, ROUND_ATTN_QKV, ROUND_P, ROUND_FLOW = 1, 2, 4, 8, 16
# Finer sites (each also inside ROUND_OPERAND or ROUND_PROJ): the operand of
# a mixer's projections, of gate/up, of down, of DeltaNet out_proj, of o_proj;
# the outputs of DeltaNet in_proj_qkv, the attention projections, in_proj_z and
# in_proj_a/b.
(ROUND_OP_MIX_IN, ROUND_OP_MLP_IN, ROUND_OP_DOWN, ROUND_OP_DELTA_OUT, ROUND_OP_ATTN_OUT,
 ROUND_PROJ_DELTA_QKV, ROUND_PROJ_ATTN, ROUND_PROJ_DELTA_Z, ROUND_PROJ_DELTA_AB) = (
    32, 64, 128, 256, 512, 1024, 2048, 4096, 8192)


def set_rounding(mask: int) -> None:
    """Rounds the chosen intermediates to BF16 in every later prefill (a
    measuring aid for BF16 device profiles; 0 restores the F32 path)."""
    lib().oracle_set_rounding(int(mask))


def linear(x, w):
    x, w = f32(x), f32(w)
    out = np.empty((x.shape[0], w.shape[0]), np.float32)
    lib().oracle_linear(_p(x), x.shape[0], _p(w), w.shape[0], w.shape[1], _p(out))
    return out


def rms(x, w, eps=1e-6):
    x, w = f32(x), f32(w)
    out = np.empty_like(x)
    lib().oracle_rms(_p(x), _p(w), x.size // x.shape[-1], x.shape[-1], eps, _p(out))
    return out


def conv4(x, w):
    """x [T, width] (history rows already prepended), w [width, 4]."""
    x, w = f32(x), f32(w)
    out = np.empty_like(x)
    lib().oracle_conv4(_p(x), x.shape[0], x.shape[1], _p(w), _p(out))
    return out


def delta_recurrence(q, k, v, g, beta, state=None, capture=0):
    """The reference's public recurrence (qwen.rs:826-882): q, k [T, Hk, dk]
    normalised inside, v [T, Hv, dv], g, beta [T, Hv]. Returns (o, final
    state, captured state or None)."""
    q, k, v, g, beta = map(f32, (q, k, v, g, beta))
    t, hk, kd = q.shape
    hv, vd = v.shape[1], v.shape[2]
    st = np.zeros((hv, kd, vd), np.float32) if state is None else f32(state).copy()
    cap = np.zeros((hv, kd, vd), np.float32) if capture else None
    out = np.empty((t, hv, vd), np.float32)
    lib().oracle_delta_recurrence(_p(q), _p(k), _p(v), _p(g), _p(beta), t, hk, hv, kd, vd,
                                  _p(st), int(capture), _p(cap) if cap is not None else None,
                                  _p(out))
    return out, st, cap


def attention(q, k, v, causal=True):
    """ops::attention (ops.rs:62-143): q [H, Tq, d], k, v [Hkv, Tk, d]."""
    q, k, v = map(f32, (q, k, v))
    out = np.empty_like(q)
    lib().oracle_attention(_p(q), _p(k), _p(v), q.shape[0], k.shape[0], q.shape[1], k.shape[1],
                           q.shape[2], int(causal), _p(out))
    return out


def rotary(x, positions, dim, theta):
    """x [T, H, width] rotated in place on a copy."""
    x = f32(x).copy()
    pos = np.ascontiguousarray(positions, dtype=np.int64)
    lib().oracle_rotary(_p(x), x.shape[0], x.shape[1], x.shape[2], _p(pos, _i64p), dim, theta)
    return x


def head(h_last, w):
    h_last, w = f32(h_last), f32(w)
    out = np.empty(w.shape[0], np.float32)
    lib().oracle_head(_p(h_last), _p(w), w.shape[0], w.shape[1], _p(out))
    return out


class Prefix:
    def __init__(self, handle):
        self.handle = handle

    @property
    def tokens(self) -> int:
        return int(lib().oracle_prefix_tokens(self.handle))

    def bytes(self) -> int:
        return int(lib().oracle_prefix_bytes(self.handle))

    def __del__(self):
        if self.handle and _lib is not None:
            _lib.oracle_prefix_destroy(self.handle)
            self.handle = None


class Model:
    """Backbone (qwen.rs:145-426) on the CPU in F32."""

    def __init__(self, cfg):
        self.cfg = cfg
        self.handle = lib().oracle_model_create(ctypes.byref(cfg))

    def names(self):
        L = lib()
        return [L.oracle_model_weight_name(self.handle, i).decode()
                for i in range(L.oracle_model_num_weights(self.handle))]

    def count(self, name: str) -> int:
        return int(lib().oracle_model_weight_count(self.handle, name.encode()))

    def set_weight(self, name: str, data) -> None:
        a = f32(data).reshape(-1)
        if lib().oracle_model_set_weight(self.handle, name.encode(), _p(a), a.size):
            raise ValueError(lib().oracle_last_error().decode())

    def check(self) -> None:
        if lib().oracle_model_check(self.handle):
            raise ValueError(lib().oracle_last_error().decode())

    def prefill(self, ids, initial: "Prefix" = None, capture: int = 0):
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        pre = initial.tokens if initial is not None else 0
        hidden = np.empty((pre + ids.size, self.cfg.hidden_size), np.float32)
        cap = ctypes.c_void_p()
        rc = lib().oracle_model_prefill(self.handle, _p(ids, _i32p), ids.size,
                                        initial.handle if initial is not None else None,
                                        int(capture), _p(hidden), ctypes.byref(cap))
        if rc:
            raise ValueError(lib().oracle_last_error().decode())
        return hidden, (Prefix(cap.value) if cap.value else None)

    def __del__(self):
        if getattr(self, "handle", None) and _lib is not None:
            _lib.oracle_model_destroy(self.handle)
            self.handle = None
