"""ctypes binding of libscope_b200.so (the C ABI declared in include/scope_b200.h).

The library is the only compute path: when it is missing this module raises
instead of falling back to anything else.
"""
from __future__ import annotations

import contextlib
import ctypes
import os
import threading

import torch

PKG = os.path.dirname(os.path.abspath(__file__))
# SCOPE_B200_LIB selects another build of the same library (e.g. a tuned variant).
LIB_PATH = os.environ.get("SCOPE_B200_LIB") or os.path.join(PKG, "libscope_b200.so")

WS_OK = 0
WS_ERR_INVALID_ARG = 1
WS_ERR_UNSUPPORTED = 2
WS_ERR_CUDA = 3
WS_ERR_WORKSPACE = 4
WS_ERR_DEVICE = 5

WS_DTYPE_BF16 = 0
WS_DTYPE_F32 = 1
WS_DTYPE_I8 = 2

WS_OUT_NORM_BF16 = 0
WS_OUT_UNNORM_F32 = 1
WS_OUT_NORM_F32 = 2

WS_CSA_IDX_ALL = 0
WS_CSA_IDX_SORTED_SHARD = 1
WS_CSA_IDX_SHARD = 2

WS_TOPK_BY_SCORE = 0
WS_TOPK_BY_ID = 1

_V = ctypes.c_void_p
_i = ctypes.c_int
_i64 = ctypes.c_int64
_f = ctypes.c_float
_sz = ctypes.c_size_t


class KvShare(ctypes.Structure):
    """Mirror of `ws_kv_share` (include/scope_b200.h)."""
    _fields_ = [("k", _V), ("v", _V), ("cu_seqlens", _V), ("seqlens", _V), ("n_tok", _i64),
                ("k_stride_t", _i64), ("k_stride_h", _i64), ("v_stride_t", _i64), ("v_stride_h", _i64)]


# exported symbol -> (restype, argtypes); the CPU tests check that every
# declaration of include/scope_b200.h is here and exported by the library.
SIGNATURES = {
    "ws_last_error": (ctypes.c_char_p, []),
    "ws_version": (_i, []),
    "ws_status_take": (_i, [_V]),
    "ws_gqa_decode": (_i, [_V, _V, _V, _i64, _i64, _i64, _i64, _i, _i, _i, _i, _i, _f, _i, _i,
                           _V, _V, _V, _V, _V, _sz, _V]),
    "ws_gqa_decode_workspace_size": (_sz, [_i, _i, _i, _i]),
    "ws_gqa_decode_shares": (_i, [_V, _i, _i, _i, _i, _i, _f, ctypes.POINTER(KvShare), _i, _V, _V, _V, _sz, _V]),
    "ws_gqa_decode_shares_workspace_size": (_sz, [_i, _i, _i, _i, _i]),
    "ws_lse_merge": (_i, [_V, _V, _i, _i64, _i, _V, _i, _V, _V]),
    "ws_lse_merge_strided": (_i, [_V, _i64, _V, _i64, _i, _i64, _i, _V, _i, _V, _V]),
    "ws_gqa_decode_noalloc": (_i, [_V, _V, _V, _i64, _i64, _i64, _i64, _i, _i, _i, _i, _i, _f, _i,
                                   _V, _V, _V, _V, _V]),
    "ws_gqa_decode_noalloc_max_scratch": (_sz, []),
    "ws_mla_decode": (_i, [_V, _V, _V, _V, _i, _i, _i, _f, _i, _V, _V, _V, _V, _V, _sz, _V]),
    "ws_mla_decode_workspace_size": (_sz, [_i, _i, _i]),
    "ws_mla_decode_strided": (_i, [_V, _V, _V, _i64, _V, _i64, _i, _i, _i, _f, _i, _V, _V, _V, _V, _V, _sz, _V]),
    "ws_mla_decode_absorbed": (_i, [_V, _V, _i64, _V, _V, _V, _V, _i64, _i, _i, _i, _i, _i, _f, _V, _V, _V, _sz,
                                    _V]),
    "ws_mla_decode_absorbed_workspace_size": (_sz, [_i, _i, _i]),
    "ws_mla_decode_absorbed_strided": (_i, [_V, _V, _i64, _V, _V, _i64, _V, _i64, _V, _i64, _i, _i, _i, _i, _i, _f, _V,
                                            _V, _V, _sz, _V]),
    "ws_csa_kv_quantize_s8": (_i, [_V, _i64, _i, _V, _V, _V, _V]),
    "ws_csa_q_quantize_u8": (_i, [_V, _i64, _i, _V, _V, _V]),
    "ws_csa_decode": (_i, [_V, _i, _i, _i, _i, _V, _i, _V, _i64, _i64, _V, _i, _i, _i64, _i64, _f, _V, _i, _V,
                           _V, _sz, _V]),
    "ws_csa_decode_workspace_size": (_sz, [_i, _i, _i]),
    "ws_csa_decode_qcodes": (_i, [_V, _V, _i, _i, _i, _V, _V, _V, _V, _i64, _i64, _V, _i, _i, _i64, _i64, _f, _V, _i,
                                  _V, _V, _sz, _V]),
    "ws_indexer_topk": (_i, [_V, _V, _i, _V, _i, _i, _i, _i64, _i, _i, _V, _V, _V, _sz, _V]),
    "ws_indexer_topk_workspace_size": (_sz, [_i, _i64]),
    "ws_kv_append": (_i, [_V, _i64, _i64, _i64, _V, _i64, _i64, _i64, _i64, _i, _i, _i64, _V]),
    "ws_peer_exchange_bytes": (_sz, [_i, _i64, _i]),
    "ws_peer_slot_offset": (_sz, [_i, _i64, _i, _i]),
    "ws_peer_buffer_create": (_i, [_sz, ctypes.POINTER(_V), _V]),
    "ws_peer_buffer_open": (_i, [_V, ctypes.POINTER(_V)]),
    "ws_peer_buffer_close": (_i, [_V]),
    "ws_peer_buffer_free": (_i, [_V]),
    "ws_peer_push": (_i, [_V, _V, _i, _i64, _i, _i, _V, _V]),
    "ws_peer_merge": (_i, [_V, _i, _i64, _i, _V, _i, _V, _V]),
    "ws_peer_rs_bytes": (_sz, [_i, _i64, _i]),
    "ws_peer_rs_scatter": (_i, [_V, _V, _i, _i64, _i, _i, _V, _V]),
    "ws_peer_rs_merge": (_i, [_V, _V, _i, _i64, _i, _i, _V, _V, _i, _V, _V]),
}

_lib = None
_lock = threading.Lock()


class ScopeError(RuntimeError):
    """Raised when an entry point returns a non-zero status."""


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise ImportError(
                        f"{LIB_PATH} is missing; build it with `python -m scope_b200.compile_lib` "
                        "(there is no CPU fallback)")
                L = ctypes.CDLL(LIB_PATH)
                for name, (res, args) in SIGNATURES.items():
                    fn = getattr(L, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = L
    return _lib


def check(rc: int, what: str) -> None:
    if rc != WS_OK:
        msg = lib().ws_last_error().decode(errors="replace")
        raise ScopeError(f"{what} failed (status {rc}): {msg}")


# The current stream's raw handle without building a Stream object (2 us per call on the host otherwise, and
# every launch asks for it).
_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_ptr(device: torch.device) -> int:
    if _raw_stream is not None:
        return _raw_stream(device.index if device.index is not None else torch.cuda.current_device())
    return torch.cuda.current_stream(device).cuda_stream


def on_device(device: torch.device):
    """Context that makes `device` current for a launch: nothing to do (and no device switch paid for) when
    it already is."""
    if device.index is None or device.index == torch.cuda.current_device():
        return contextlib.nullcontext()
    return torch.cuda.device(device)


def ptr(t: torch.Tensor | None):
    return None if t is None else t.data_ptr()


class _WorkspacePool:
    """Zeroed device workspaces, one per (device, stream), grown on demand.

    The kernels reset their counters after every launch, so a workspace is
    zeroed only when it is (re)allocated.  Keyed by stream because launches on
    different streams may overlap and must not share counters.
    """

    def __init__(self):
        self._bufs: dict[tuple[int, int], torch.Tensor] = {}

    def get(self, nbytes: int, device: torch.device) -> torch.Tensor:
        key = (device.index if device.index is not None else torch.cuda.current_device(), stream_ptr(device))
        buf = self._bufs.get(key)
        if buf is None or buf.numel() < nbytes:
            size = max(nbytes, 1 << 20, 0 if buf is None else 2 * buf.numel())
            buf = torch.zeros(size, dtype=torch.uint8, device=device)
            self._bufs[key] = buf
        return buf

    def clear(self) -> None:
        self._bufs.clear()

    def drop_device(self, index: int) -> None:
        """Forget every workspace of device ``index``; the next launch there
        allocates a freshly zeroed one.  Called after a kernel reported a
        device-side failure: a launch that gave up may leave a merge counter
        of its workspace non-zero."""
        for key in [k for k in self._bufs if k[0] == index]:
            del self._bufs[key]


workspaces = _WorkspacePool()
