"""Python host mirror of the clef-rs prefill backend's C ABI (libclef_b200.so).

Every compute call goes through the shared library built from csrc/ for
sm_100a; there is no CPU or framework fallback. The library is mapped on first
use (not at import, so that host-only modules such as clef_b200.config and
clef_b200.workloads can be used without it); if it is missing or cannot be
loaded, that first use raises ImportError.

The operator functions take torch CUDA tensors (torch is only the device
allocator and stream provider here) and mirror the reference engine's Candle
custom ops (crates/core/src/models/{metal,pointwise,neural}.rs): each validates
shapes before launch and raises ClefError carrying the library's message.
"""
import ctypes
from pathlib import Path

import numpy as np

from .config import ClefConfig, benchmark_config, from_text_config, weight_shapes  # noqa: F401

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE.parent / "libclef_b200.so"

F32, BF16 = 0, 1
PRECISION_BF16, PRECISION_SPLIT = 0, 1
EPI_BF16, EPI_F32, EPI_ADD_F32 = 0, 1, 2
STATUS = {0: "OK", 1: "INVALID", 2: "CUDA", 3: "UNSUPPORTED", 4: "NOMEM", 5: "CANCELLED",
          6: "DEVICE_TIMEOUT"}
STAGES = ["embed", "norm", "gemm", "delta_prologue", "delta_scan", "delta_epilogue",
          "attention_prologue", "attention", "head"]

# Every symbol include/clef_b200.h declares.
EXPORTS = [
    "clef_last_error", "clef_version", "clef_config_validate", "clef_rmsnorm", "clef_conv4",
    "clef_delta_prologue", "clef_delta_scan_workspace_size", "clef_delta_scan",
    "clef_delta_scan_noalloc", "clef_delta_packed", "clef_delta_prepare_packed", "clef_gemm_bf16", "clef_gemm_bf16_split",
    "clef_gemm_swiglu", "clef_attention_gqa_workspace_size", "clef_attention_gqa", "clef_attention_gqa_vt", "clef_compact_copy",
    "clef_engine_create",
    "clef_engine_set_weight", "clef_engine_init_random", "clef_engine_get_weight",
    "clef_engine_weight_count", "clef_engine_finalize", "clef_engine_prefill",
    "clef_engine_prefill_device", "clef_engine_set_precision", "clef_engine_precision",
    "clef_engine_set_sm_limit",
    "clef_engine_launches", "clef_engine_cancel",
    "clef_engine_stage_times", "clef_engine_set_profiling", "clef_engine_destroy",
    "clef_prefix_tokens", "clef_prefix_bytes", "clef_prefix_destroy", "clef_prefix_span_bytes",
    "clef_prefix_create", "clef_prefix_export", "clef_prefix_import", "clef_head_create",
    "clef_head_set_weight", "clef_head_finalize", "clef_head_forward", "clef_head_destroy",
    "clef_selftest_wait_timeout", "clef_decide",
]


class ClefError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{STATUS.get(code, code)}: {msg}")
        self.code = code


class HeadConfig(ctypes.Structure):
    """clef_head_config (HeadConfig, head.rs:26-33)."""
    _fields_ = [("hidden_size", ctypes.c_int32), ("width", ctypes.c_int32),
                ("routing_layers", ctypes.c_int32), ("layers", ctypes.c_int32),
                ("heads", ctypes.c_int32), ("feedforward", ctypes.c_int32)]


class HeadQuestion(ctypes.Structure):
    _fields_ = [("kind", ctypes.c_int32), ("instruction_start", ctypes.c_int32),
                ("instruction_end", ctypes.c_int32), ("option_offset", ctypes.c_int32),
                ("option_count", ctypes.c_int32)]


class Decision(ctypes.Structure):
    _fields_ = [("noul", ctypes.c_float), ("choice", ctypes.c_int32),
                ("confidence", ctypes.c_float), ("score", ctypes.c_float)]


_vp, _i32, _i64, _f32, _sz = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_float, ctypes.c_size_t


def _load():
    if not LIB_PATH.exists():
        raise ImportError(f"{LIB_PATH} is missing: build it with `python clef-rs_b200/build.py`")
    L = ctypes.CDLL(str(LIB_PATH))
    sig = {
        "clef_last_error": (ctypes.c_char_p, []),
        "clef_version": (ctypes.c_char_p, []),
        "clef_config_validate": (ctypes.c_int, [_vp]),
        "clef_rmsnorm": (ctypes.c_int, [_vp, _vp, _i64, _i32, _f32, _i32, _vp, _vp]),
        "clef_conv4": (ctypes.c_int, [_vp, _i64, _vp, _i32, _vp, _i64, _i32, _vp, _vp]),
        "clef_delta_prologue": (ctypes.c_int, [_vp, _i64, _i32, _i32, _vp, _i32, _vp, _vp, _vp, _i64,
                                               _i32, _i32, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp]),
        "clef_delta_scan_workspace_size": (_sz, [_i64, _i32, _i32, _i32, _i32, _i32]),
        "clef_delta_scan": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _i64, _i32, _i32, _i32, _i32, _vp,
                                           _i32, _vp, _i32, _i64, _vp, _vp, _vp, _vp, _sz, _vp]),
        "clef_delta_scan_noalloc": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _i64, _i32, _i32, _i32, _i32,
                                                   _vp, _i32, _vp, _i32, _i64, _vp, _vp, _vp, _vp]),
        "clef_delta_packed": (ctypes.c_int, [_vp, _i64, _i32, _i32, _i32, _vp, _i64, _vp, _vp]),
        "clef_delta_prepare_packed": (ctypes.c_int, [_vp, _i64, _vp, _vp, _i64, _i32, _i32, _vp, _vp]),
        "clef_gemm_bf16": (ctypes.c_int, [_vp, _vp, _i64, _i32, _i32, _i32, _vp, _i64, _vp]),
        "clef_gemm_bf16_split": (ctypes.c_int, [_vp, _vp, _i64, _i32, _i32, _i32, _vp, _i64, _vp]),
        "clef_gemm_swiglu": (ctypes.c_int, [_vp, _vp, _vp, _i64, _i32, _i32, _vp, _vp]),
        "clef_attention_gqa_workspace_size": (_sz, [_i32, _i32, _i64, _i64]),
        "clef_attention_gqa": (ctypes.c_int, [_vp, _vp, _vp, _i32, _i32, _i64, _i64, _i32, _vp, _vp, _sz,
                                              _vp]),
        "clef_attention_gqa_vt": (ctypes.c_int, [_vp, _vp, _vp, _i32, _i32, _i64, _i64, _i32, _i64, _vp,
                                                 _vp]),
        "clef_compact_copy": (ctypes.c_int, [_vp, _i32, _vp, _vp, _i32, _vp, _vp]),
        "clef_engine_create": (ctypes.c_int, [_vp, _i32, ctypes.POINTER(_vp)]),
        "clef_engine_set_weight": (ctypes.c_int, [_vp, ctypes.c_char_p, _vp, _sz]),
        "clef_engine_init_random": (ctypes.c_int, [_vp, ctypes.c_uint64, _f32]),
        "clef_engine_get_weight": (ctypes.c_int, [_vp, ctypes.c_char_p, _vp, _sz]),
        "clef_engine_weight_count": (_sz, [_vp, ctypes.c_char_p]),
        "clef_engine_finalize": (ctypes.c_int, [_vp]),
        "clef_engine_prefill": (ctypes.c_int, [_vp, _vp, _vp, _i32, _vp, _i64, ctypes.POINTER(_vp),
                                               _vp, _vp]),
        "clef_engine_prefill_device": (ctypes.c_int, [_vp, _vp, _vp, _i32, _vp, _vp, _vp]),
        "clef_engine_launches": (_i64, [_vp]),
        "clef_engine_set_precision": (ctypes.c_int, [_vp, _i32]),
        "clef_engine_precision": (_i32, [_vp]),
        "clef_engine_set_sm_limit": (ctypes.c_int, [_vp, _i32]),
        "clef_engine_cancel": (ctypes.c_int, [_vp, _i32]),
        "clef_engine_stage_times": (ctypes.c_int, [_vp, _vp, _i32]),
        "clef_engine_set_profiling": (ctypes.c_int, [_vp, _i32]),
        "clef_engine_destroy": (ctypes.c_int, [_vp]),
        "clef_prefix_tokens": (_i64, [_vp]),
        "clef_prefix_bytes": (ctypes.c_uint64, [_vp]),
        "clef_prefix_destroy": (ctypes.c_int, [_vp]),
        "clef_prefix_span_bytes": (ctypes.c_uint64, [_vp]),
        "clef_prefix_create": (ctypes.c_int, [_vp, _i64, ctypes.POINTER(_vp)]),
        "clef_prefix_export": (ctypes.c_int, [_vp, _vp, ctypes.c_uint64, _vp]),
        "clef_prefix_import": (ctypes.c_int, [_vp, _vp, ctypes.c_uint64, _vp]),
        "clef_head_create": (ctypes.c_int, [_vp, _i32, ctypes.POINTER(_vp)]),
        "clef_head_set_weight": (ctypes.c_int, [_vp, ctypes.c_char_p, _vp, _i64]),
        "clef_head_finalize": (ctypes.c_int, [_vp]),
        "clef_head_forward": (ctypes.c_int, [_vp, _vp, _i64, _vp, _i64, _vp, _vp, _i32, _vp, _vp]),
        "clef_head_destroy": (ctypes.c_int, [_vp]),
        "clef_selftest_wait_timeout": (ctypes.c_int, [_i32, _vp]),
        "clef_decide": (ctypes.c_int, [_vp, _i32, _i32, _vp]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    return L


class _LazyLib:
    """The ctypes handle of libclef_b200.so, loaded on first attribute access."""

    _handle = None

    def __getattr__(self, name):
        if _LazyLib._handle is None:
            _LazyLib._handle = _load()
        return getattr(_LazyLib._handle, name)

    @staticmethod
    def loaded() -> bool:
        return _LazyLib._handle is not None


lib = _LazyLib()


def load():
    """Maps the library now (raises ImportError if it is missing)."""
    lib.clef_version
    return lib


def version() -> str:
    return lib.clef_version().decode()


def _check(rc: int) -> None:
    if rc != 0:
        raise ClefError(rc, lib.clef_last_error().decode())


def _ptr(t) -> int:
    if t is None:
        return None
    return t.data_ptr()


def _stream(stream=None):
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


# ---------------------------------------------------------------------------
# Operators (torch CUDA tensors in, caller-allocated outputs).
# ---------------------------------------------------------------------------
def rmsnorm(x, weight, eps=1e-6, out_dtype=F32, out=None, stream=None):
    """RmsKernel / ops::rms_inner: x F32 [rows, width], weight F32 (1+w for
    offset norms)."""
    import torch
    width = x.shape[-1]
    rows = x.numel() // width
    if out is None:
        out = torch.empty(x.shape, dtype=torch.float32 if out_dtype == F32 else torch.bfloat16,
                          device=x.device)
    _check(lib.clef_rmsnorm(_ptr(x), _ptr(weight), rows, width, eps, out_dtype, _ptr(out), _stream(stream)))
    return out


def conv4(x, weight, history=None, out=None, stream=None):
    """ConvKernel / causal_convolution: x F32 [T, width], weight F32 [width, 4]."""
    import torch
    T, width = x.shape
    if out is None:
        out = torch.empty_like(x)
    hr = 0 if history is None else history.shape[0]
    _check(lib.clef_conv4(_ptr(x), x.stride(0), _ptr(history), hr, _ptr(weight), T, width, _ptr(out),
                          _stream(stream)))
    return out


def delta_prologue(proj, a_col, b_col, conv_weight, dt_bias, a_log, Hk, Hv, dk=128, dv=128,
                   history=None, stream=None):
    """ConvKernel + DeltaPrepareKernel + gates: returns q, k, v, g, beta."""
    import torch
    T = proj.shape[0]
    dev = proj.device
    q = torch.empty((T, Hk, dk), dtype=torch.float32, device=dev)
    k = torch.empty_like(q)
    v = torch.empty((T, Hv, dv), dtype=torch.float32, device=dev)
    g = torch.empty((T, Hv), dtype=torch.float32, device=dev)
    beta = torch.empty_like(g)
    hr = 0 if history is None else history.shape[0]
    _check(lib.clef_delta_prologue(_ptr(proj), proj.stride(0), a_col, b_col, _ptr(history), hr,
                                   _ptr(conv_weight), _ptr(dt_bias), _ptr(a_log), T, Hk, Hv, dk, dv,
                                   _ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(beta), _stream(stream)))
    return q, k, v, g, beta


def delta_scan_workspace_size(total_tokens, nseq, Hk, Hv, dk=128, dv=128) -> int:
    return int(lib.clef_delta_scan_workspace_size(total_tokens, nseq, Hk, Hv, dk, dv))


def delta_scan(q, k, v, g, beta, cu_seqlens=None, init_state=None, init_shared=False, capture=0,
               final_state=False, workspace=None, stream=None):
    """DeltaKernel / CachedDelta: chunked scan. q, k [T, Hk, 128] normalised
    (q scaled), v [T, Hv, 128], g (log decay), beta [T, Hv]. Returns
    (out [T, Hv, 128], captured state or None, final states or None)."""
    import torch
    T, Hk, dk = q.shape
    Hv, dv = v.shape[1], v.shape[2]
    dev = q.device
    if cu_seqlens is None:
        nseq, cu_arr = 1, None
    else:
        cu_np = np.ascontiguousarray(cu_seqlens, dtype=np.int64)
        nseq = cu_np.size - 1
        cu_arr = cu_np
    out = torch.empty((T, Hv, dv), dtype=torch.float32, device=dev)
    cap = torch.empty((Hv, dk, dv), dtype=torch.float32, device=dev) if capture else None
    fin = torch.empty((nseq, Hv, dk, dv), dtype=torch.float32, device=dev) if final_state else None
    if workspace is None:
        size = delta_scan_workspace_size(T, nseq, Hk, Hv, dk, dv)
        workspace = torch.empty(size, dtype=torch.uint8, device=dev)
    _check(lib.clef_delta_scan(_ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(beta), T, Hk, Hv, dk, dv,
                               cu_arr.ctypes.data if cu_arr is not None else None, nseq,
                               _ptr(init_state), int(bool(init_shared)), int(capture), _ptr(cap),
                               _ptr(fin), _ptr(out), _ptr(workspace), workspace.numel(),
                               _stream(stream)))
    return out, cap, fin


def delta_packed(packed, dk, dv, initial=None, capture=0, stream=None):
    """DeltaKernel / CachedDelta on the reference's packed input: packed F32
    [T, H, 2 dk + dv + 2] (q | k | v | e^g | beta). Returns (o [T, H, dv],
    captured state [H, dk, dv] or None)."""
    import torch
    T, H, width = packed.shape
    if width != 2 * dk + dv + 2:
        raise ClefError(1, "delta_packed: packed width must be 2 dk + dv + 2")
    n = T * H * dv + (H * dk * dv if capture else 0)
    out = torch.empty(n, dtype=torch.float32, device=packed.device)
    _check(lib.clef_delta_packed(_ptr(packed), T, H, dk, dv, _ptr(initial), int(capture), _ptr(out),
                                 _stream(stream)))
    o = out[:T * H * dv].view(T, H, dv)
    state = out[T * H * dv:].view(H, dk, dv) if capture else None
    return o, state


def delta_prepare_packed(mixed, g, beta, Hk, Hv, stream=None):
    """DeltaPrepareKernel: mixed F32 [T, >= (2 Hk + Hv) 128], g, beta F32
    [T, Hv] -> packed [T, Hv, 386]."""
    import torch
    T = mixed.shape[0]
    out = torch.empty((T, Hv, 386), dtype=torch.float32, device=mixed.device)
    _check(lib.clef_delta_prepare_packed(_ptr(mixed), mixed.stride(0), _ptr(g), _ptr(beta), T, Hk, Hv, _ptr(out),
                                         _stream(stream)))
    return out


def gemm(x, w, epilogue=EPI_BF16, out=None, stream=None):
    """GemmKernel / Projection::forward: x BF16 [M, K], w BF16 [N, K]."""
    import torch
    M, K = x.shape
    N = w.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16 if epilogue == EPI_BF16 else torch.float32,
                          device=x.device)
    _check(lib.clef_gemm_bf16(_ptr(x), _ptr(w), M, N, K, epilogue, _ptr(out), out.stride(0),
                              _stream(stream)))
    return out


def split_bf16(x):
    """(hi | lo) BF16 pair of an F32 tensor [M, K] as one [M, 2K] tensor:
    hi = bf16(x), lo = bf16(x - hi)."""
    import torch
    hi = x.float().bfloat16()
    lo = (x.float() - hi.float()).bfloat16()
    return torch.cat([hi, lo], dim=1).contiguous()


def gemm_split(x2, w, epilogue=EPI_F32, out=None, stream=None):
    """x2 BF16 [M, 2K] split pair (split_bf16), w BF16 [N, K]: (hi + lo) w^T."""
    import torch
    M, K2 = x2.shape
    N = w.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16 if epilogue == EPI_BF16 else torch.float32,
                          device=x2.device)
    _check(lib.clef_gemm_bf16_split(_ptr(x2), _ptr(w), M, N, K2 // 2, epilogue, _ptr(out), out.stride(0),
                                    _stream(stream)))
    return out


def gemm_swiglu(x, wg, wu, out=None, stream=None):
    """gated TileKernel / Projection::gated_forward: silu(x wg^T) * (x wu^T)."""
    import torch
    M, K = x.shape
    N = wg.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=x.device)
    _check(lib.clef_gemm_swiglu(_ptr(x), _ptr(wg), _ptr(wu), M, N, K, _ptr(out), _stream(stream)))
    return out


def attention_gqa(q, k, v, out=None, workspace=None, stream=None):
    """AttentionKernel / ops::attention on the tcgen05 tensor cores: q BF16
    [Hq, Tq, 256], k, v BF16 [Hkv, Tk, 256], causal lower-right; returns F32
    [Hq, Tq, 256]."""
    import torch
    Hq, Tq, d = q.shape
    Hkv, Tk = k.shape[0], k.shape[1]
    if out is None:
        out = torch.empty((Hq, Tq, d), dtype=torch.float32, device=q.device)
    if workspace is None:
        size = int(lib.clef_attention_gqa_workspace_size(Hq, Hkv, Tq, Tk))
        workspace = torch.empty(size, dtype=torch.uint8, device=q.device)
    _check(lib.clef_attention_gqa(_ptr(q), _ptr(k), _ptr(v), Hq, Hkv, Tq, Tk, d, _ptr(out), _ptr(workspace),
                                  workspace.numel(), _stream(stream)))
    return out


def attention_gqa_tc(q, k, v, out=None, stream=None):
    """tcgen05 attention: q BF16 [Hq, Tq, 256], k, v BF16 [Hkv, Tk, 256]
    (head-major like attention_gqa; converted to the kernel's token-major
    q/k and transposed V here); returns F32 [Hq, Tq, 256]."""
    import torch
    Hq, Tq, d = q.shape
    Hkv, Tk = k.shape[0], k.shape[1]
    qt = q.transpose(0, 1).contiguous()
    kt = k.transpose(0, 1).contiguous()
    pitch = (Tk + 63) // 64 * 64
    vt = torch.zeros((Hkv * d, pitch), dtype=torch.bfloat16, device=q.device)
    vt[:, :Tk] = v.permute(0, 2, 1).reshape(Hkv * d, Tk)
    o = torch.empty((Tq, Hq, d), dtype=torch.float32, device=q.device)
    _check(lib.clef_attention_gqa_vt(_ptr(qt), _ptr(kt), _ptr(vt), Hq, Hkv, Tq, Tk, d, pitch, _ptr(o),
                                     _stream(stream)))
    res = o.transpose(0, 1).contiguous()
    if out is not None:
        out.copy_(res)
        return out
    return res


def compact_copy(src, out=None, stream=None):
    """CompactCopy: contiguous copy of a strided view (<= 4 dims)."""
    import torch
    if out is None:
        out = torch.empty(src.shape, dtype=src.dtype, device=src.device)
    nd = src.dim()
    dims = (ctypes.c_int64 * nd)(*src.shape)
    strides = (ctypes.c_int64 * nd)(*src.stride())
    _check(lib.clef_compact_copy(_ptr(src), nd, dims, strides, src.element_size(), _ptr(out),
                                 _stream(stream)))
    return out


def decide(logits: np.ndarray):
    """answers (types.rs:728-802) over [n, 7] logits -> list of Decision."""
    lg = np.ascontiguousarray(logits, dtype=np.float32).reshape(-1, 7)
    out = (Decision * lg.shape[0])()
    _check(lib.clef_decide(lg.ctypes.data, lg.shape[0], 7, out))
    return list(out)


# ---------------------------------------------------------------------------
# Engine (Backbone::load / forward / prefill).
# ---------------------------------------------------------------------------
class Prefix:
    """Captured prefix state (PrefixState) owned by the library."""

    def __init__(self, handle):
        self.handle = handle

    @property
    def tokens(self) -> int:
        return int(lib.clef_prefix_tokens(self.handle))

    def bytes(self) -> int:
        return int(lib.clef_prefix_bytes(self.handle))

    def span_bytes(self) -> int:
        """Bytes of the prefix's single device allocation."""
        return int(lib.clef_prefix_span_bytes(self.handle))

    def export_to(self, dst, stream=None) -> None:
        """Copies the prefix's device allocation into `dst`, a CUDA tensor of
        span_bytes() bytes on the prefix's device (stream-ordered)."""
        _check(lib.clef_prefix_export(self.handle, _ptr(dst), dst.numel() * dst.element_size(),
                                      _stream(stream)))

    def import_from(self, src, stream=None) -> None:
        """Fills the prefix from a copy made by export_to (stream-ordered)."""
        _check(lib.clef_prefix_import(self.handle, _ptr(src), src.numel() * src.element_size(),
                                      _stream(stream)))

    def close(self):
        if self.handle and lib is not None:
            lib.clef_prefix_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Engine:
    def __init__(self, cfg: ClefConfig, device: int = 0):
        self.cfg = cfg
        h = ctypes.c_void_p()
        _check(lib.clef_engine_create(ctypes.byref(cfg), device, ctypes.byref(h)))
        self.handle = h

    def count(self, name: str) -> int:
        return int(lib.clef_engine_weight_count(self.handle, name.encode()))

    def set_weight(self, name: str, data) -> None:
        a = np.ascontiguousarray(data, dtype=np.float32).reshape(-1)
        _check(lib.clef_engine_set_weight(self.handle, name.encode(), a.ctypes.data, a.size))

    def get_weight(self, name: str) -> np.ndarray:
        n = self.count(name)
        out = np.empty(n, np.float32)
        _check(lib.clef_engine_get_weight(self.handle, name.encode(), out.ctypes.data, n))
        return out

    def init_random(self, seed: int, std: float = 0.02) -> None:
        _check(lib.clef_engine_init_random(self.handle, seed, std))

    def finalize(self) -> None:
        _check(lib.clef_engine_finalize(self.handle))

    def set_precision(self, precision: int) -> None:
        """PRECISION_BF16 (default) or PRECISION_SPLIT (split-BF16 operands and
        F32 projection outputs: F32-class projections at twice the tensor work)."""
        _check(lib.clef_engine_set_precision(self.handle, int(precision)))

    def set_sm_limit(self, sms: int) -> None:
        """SMs the engine's persistent kernels may occupy (0 = all)."""
        _check(lib.clef_engine_set_sm_limit(self.handle, int(sms)))

    @property
    def precision(self) -> int:
        return int(lib.clef_engine_precision(self.handle))

    def set_profiling(self, on: bool) -> None:
        _check(lib.clef_engine_set_profiling(self.handle, int(on)))

    def stage_times(self) -> dict:
        buf = (ctypes.c_float * len(STAGES))()
        n = lib.clef_engine_stage_times(self.handle, buf, len(STAGES))
        return {STAGES[i]: float(buf[i]) for i in range(n)}

    def cancel(self, on: bool = True) -> None:
        _check(lib.clef_engine_cancel(self.handle, int(on)))

    def prefill(self, seqs, initial: Prefix = None, capture: int = 0, logits: bool = True,
                hidden: bool = False):
        """seqs: list of int arrays (token ids). Returns (logits [n, outputs]
        or None, hidden or None, captured Prefix or None)."""
        lens = [len(s) for s in seqs]
        offsets = np.zeros(len(seqs) + 1, np.int64)
        offsets[1:] = np.cumsum(lens)
        ids = np.ascontiguousarray(np.concatenate([np.asarray(s, dtype=np.int32) for s in seqs]))
        return self.prefill_packed(ids, offsets, initial, capture, logits, hidden)

    def prefill_packed(self, ids: np.ndarray, offsets: np.ndarray, initial: Prefix = None,
                       capture: int = 0, logits: bool = True, hidden: bool = False,
                       logits_out: np.ndarray = None):
        nseq = offsets.size - 1
        lg = None
        if logits and self.cfg.head_outputs:
            lg = logits_out if logits_out is not None else np.empty((nseq, self.cfg.head_outputs), np.float32)
        hid = None
        if hidden:
            pre = initial.tokens if (initial is not None and nseq == 1) else 0
            hid = np.empty((pre + int(offsets[-1]), self.cfg.hidden_size), np.float32)
        cap = ctypes.c_void_p()
        _check(lib.clef_engine_prefill(self.handle, ids.ctypes.data, offsets.ctypes.data, nseq,
                                       initial.handle if initial is not None else None, int(capture),
                                       ctypes.byref(cap) if capture else None,
                                       lg.ctypes.data if lg is not None else None,
                                       hid.ctypes.data if hid is not None else None))
        return lg, hid, (Prefix(cap.value) if cap.value else None)

    def prefill_device(self, ids_dev, offsets: np.ndarray, logits_dev, initial: Prefix = None,
                       stream=None) -> None:
        """Stream-ordered prefill: ids_dev int32 CUDA tensor, logits_dev F32
        CUDA tensor [nseq, outputs]; returns without synchronising."""
        offsets = np.ascontiguousarray(offsets, dtype=np.int64)
        _check(lib.clef_engine_prefill_device(self.handle, _ptr(ids_dev), offsets.ctypes.data,
                                              offsets.size - 1,
                                              initial.handle if initial is not None else None,
                                              _ptr(logits_dev), _stream(stream)))

    def launches(self) -> int:
        return int(lib.clef_engine_launches(self.handle))

    def create_prefix(self, tokens: int) -> Prefix:
        """An empty prefix of `tokens` tokens with this engine's layout, to be
        filled by Prefix.import_from."""
        h = ctypes.c_void_p()
        _check(lib.clef_prefix_create(self.handle, int(tokens), ctypes.byref(h)))
        return Prefix(h.value)

    def close(self):
        if getattr(self, "handle", None) and lib is not None:
            lib.clef_engine_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Head:
    """The learned joint schema head (Head::load / Head::forward,
    head.rs:91-274) on one GPU, F32.

    Usage: h = Head(dict(hidden_size=.., width=.., routing_layers=.., layers=..,
    heads=.., feedforward=..)); h.set_weight(name, array) for every tensor of
    joint_head.safetensors; h.finalize(); h.forward(hidden, output_embeddings,
    ids, questions) with `questions` a list of (kind, (start, end),
    [(start, end), ...]) and torch CUDA F32 tensors for hidden [T, hidden] and
    output_embeddings [vocab, hidden]. Returns one numpy array per question.
    """

    def __init__(self, config, device=0):
        self.cfg = HeadConfig(**{k: int(config[k]) for k, _ in HeadConfig._fields_})
        h = _vp()
        _check(lib.clef_head_create(ctypes.byref(self.cfg), device, ctypes.byref(h)))
        self.h = h

    def set_weight(self, name, array):
        a = np.ascontiguousarray(np.asarray(array, dtype=np.float32)).reshape(-1)
        _check(lib.clef_head_set_weight(self.h, name.encode(), a.ctypes.data, a.size))

    def finalize(self):
        _check(lib.clef_head_finalize(self.h))

    def forward(self, hidden, output_embeddings, ids, questions):
        ids = np.ascontiguousarray(np.asarray(ids, dtype=np.int32))
        qs = (HeadQuestion * len(questions))()
        spans, off = [], 0
        for i, (kind, (s, e), options) in enumerate(questions):
            qs[i] = HeadQuestion(kind, s, e, off, len(options))
            for (a, b) in options:
                spans += [a, b]
            off += len(options)
        spans = np.ascontiguousarray(np.asarray(spans, dtype=np.int32))
        out = np.zeros(off, np.float32)
        _check(lib.clef_head_forward(self.h, _ptr(hidden), int(hidden.shape[0]), _ptr(output_embeddings),
                                     int(output_embeddings.shape[0]), ids.ctypes.data, qs, len(questions),
                                     spans.ctypes.data, out.ctypes.data))
        res, o = [], 0
        for (_, _, options) in questions:
            res.append(out[o:o + len(options)].copy())
            o += len(options)
        return res

    def close(self):
        if getattr(self, "h", None):
            lib.clef_head_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
