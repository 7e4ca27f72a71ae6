"""ctypes binding of librfsn_b200.so (declared in include/rfsn_b200.h).

The library is the product's only compute path: there is no CPU or PyTorch
fallback.  ``lib()`` raises ``RuntimeError`` when the shared object is missing
(build it with ``python apple_b200/csrc/build.py``) and every call raises
``RFSNError`` on a non-zero status.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIB_PATH = Path(os.environ.get("RFSN_B200_LIB", _PKG / "librfsn_b200.so"))

RFSN_ERR_WORKSPACE_TOO_SMALL = -4  # rfsn_status in include/rfsn_b200.h
RFSN_MAX_SEGMENTS = 256
RFSN_MAX_ROWS_PER_KV = 8

STATUS = {
    0: "ok", -1: "invalid argument", -2: "unsupported configuration", -3: "CUDA error",
    -4: "workspace too small", -5: "device-side bounded wait timed out", -6: "alignment",
}


class RFSNError(RuntimeError):
    def __init__(self, fn: str, status: int, detail: str = ""):
        self.status = status
        msg = f"{fn} failed: {STATUS.get(status, status)} ({status})"
        if detail:
            msg += f": {detail}"
        super().__init__(msg)


class Quantizer(C.Structure):
    _fields_ = [("pq_codebooks", C.c_void_p), ("rvq_codebooks", C.c_void_p), ("head_dim", C.c_int32),
                ("num_subspaces", C.c_int32), ("subspace_dim", C.c_int32), ("pq_codebook_size", C.c_int32),
                ("rvq_layers", C.c_int32), ("rvq_codebook_size", C.c_int32), ("rvq_threshold", C.c_float),
                ("sparse_topk", C.c_int32)]


class CodeStore(C.Structure):
    _fields_ = [("data", C.c_void_p), ("cap", C.c_int64), ("rows", C.c_int64), ("slots", C.c_int64)]


class DenseStore(C.Structure):
    _fields_ = [("k", C.c_void_p), ("v", C.c_void_p), ("cap", C.c_int64), ("rows", C.c_int64)]


class Segment(C.Structure):
    _fields_ = [("store", C.c_int32), ("slot", C.c_int32), ("first", C.c_int32), ("count", C.c_int32),
                ("pos0", C.c_int32), ("reserved", C.c_int32 * 3)]


RFSN_MAX_PEERS = 8


class PeerGather(C.Structure):
    _fields_ = [("num_ranks", C.c_int32), ("rank", C.c_int32), ("seq_offset", C.c_int64), ("total_seqs", C.c_int64),
                ("buffers", C.c_void_p * RFSN_MAX_PEERS), ("flags", C.c_void_p * RFSN_MAX_PEERS),
                ("step", C.c_void_p), ("out_full", C.c_void_p)]


class AttnArgs(C.Structure):
    _fields_ = [("q", C.c_void_p), ("qpos", C.c_void_p), ("out", C.c_void_p), ("batch", C.c_int32),
                ("queries", C.c_int32), ("q_heads", C.c_int32), ("kv_heads", C.c_int32), ("head_dim", C.c_int32),
                ("causal", C.c_int32), ("scale", C.c_float), ("hot", DenseStore), ("warm", CodeStore),
                ("cold", CodeStore),
                ("segments", C.POINTER(Segment)), ("num_segments", C.c_int32), ("num_ctas", C.c_int32),
                ("workspace", C.c_void_p), ("workspace_bytes", C.c_size_t), ("device_status", C.c_void_p),
                ("q_batch_stride", C.c_int64), ("gather", C.POINTER(PeerGather))]


# exported symbol -> (restype, argtypes); must match include/rfsn_b200.h
SIGNATURES = {
    "rfsn_version": (C.c_int, []),
    "rfsn_status_string": (C.c_char_p, [C.c_int]),
    "rfsn_last_cuda_error": (C.c_char_p, []),
    "rfsn_code_block_bytes": (C.c_int64, [C.POINTER(Quantizer)]),
    "rfsn_encode": (C.c_int, [C.POINTER(Quantizer), C.c_void_p, C.c_int64, C.c_int64, C.c_int64, C.c_int64,
                              C.c_int64, C.c_int64, C.POINTER(CodeStore), C.c_int32, C.c_int64, C.c_int64,
                              C.c_void_p, C.c_void_p]),
    "rfsn_encode_kv": (C.c_int, [C.POINTER(Quantizer), C.c_void_p, C.c_void_p, C.c_int64, C.c_int64, C.c_int64,
                                 C.c_int64, C.c_int64, C.c_int64, C.POINTER(CodeStore), C.c_int64, C.c_int64,
                                 C.c_void_p]),
    "rfsn_decode_codes": (C.c_int, [C.POINTER(Quantizer), C.POINTER(CodeStore), C.c_int32, C.c_int64, C.c_int64,
                                    C.c_int64, C.c_int64, C.c_int64, C.c_void_p, C.c_int64, C.c_int64,
                                    C.c_int64, C.c_void_p]),
    "rfsn_attention_workspace_size": (C.c_int, [C.POINTER(AttnArgs), C.POINTER(Quantizer),
                                                C.POINTER(C.c_size_t)]),
    "rfsn_decode_attention": (C.c_int, [C.POINTER(AttnArgs), C.POINTER(Quantizer), C.c_void_p]),
    "rfsn_decode_attention_noalloc": (C.c_int, [C.POINTER(AttnArgs), C.POINTER(Quantizer), C.c_void_p]),
    "rfsn_decode_attention_host": (C.c_int, [C.POINTER(AttnArgs), C.POINTER(Quantizer), C.c_void_p, C.c_void_p,
                                             C.c_int, C.c_void_p]),
    "rfsn_route_topk": (C.c_int, [C.c_void_p, C.c_int64, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32,
                                  C.c_void_p, C.c_int32, C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "rfsn_peer_alloc": (C.c_int, [C.c_size_t, C.POINTER(C.c_void_p), C.c_void_p]),
    "rfsn_peer_open": (C.c_int, [C.c_void_p, C.POINTER(C.c_void_p)]),
    "rfsn_peer_close": (C.c_int, [C.c_void_p]),
    "rfsn_peer_free": (C.c_int, [C.c_void_p]),
    "rfsn_cold_prefetch": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p, C.c_void_p]),
    "rfsn_cold_evict": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p]),
    "rfsn_rmsnorm_f16": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_int, C.c_float, C.c_void_p]),
    "rfsn_gelu_tanh_f16": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int64, C.c_void_p]),
    "rfsn_add_rmsnorm_f16": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64,
                                       C.c_int, C.c_float, C.c_void_p]),
    "rfsn_llama_rmsnorm_f16": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64,
                                         C.c_int, C.c_float, C.c_void_p]),
    "rfsn_rope_f16": (C.c_int, [C.c_void_p, C.c_int64, C.c_int64, C.c_int64, C.c_void_p, C.c_int64, C.c_int64,
                                C.c_int64, C.c_void_p, C.c_void_p, C.c_int64, C.c_int, C.c_int, C.c_int, C.c_void_p]),
    "rfsn_silu_mul_f16": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_void_p]),
    "rfsn_linear_workspace_size": (C.c_int, [C.c_int, C.c_int, C.c_int, C.POINTER(C.c_size_t)]),
    "rfsn_linear_f16": (C.c_int, [C.c_void_p, C.c_int64, C.c_void_p, C.c_int64, C.c_void_p, C.c_int64, C.c_void_p,
                                  C.c_int64, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_size_t, C.c_void_p,
                                  C.c_void_p]),
    "rfsn_affine_quantize_f32": (C.c_int, [C.c_void_p, C.c_int64, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p,
                                           C.c_void_p, C.c_void_p, C.c_void_p]),
}

_LIB = None


def lib() -> C.CDLL:
    """Load (once) and return the CUDA library; raise if it is not built."""
    global _LIB
    if _LIB is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} not found: build it with `python apple_b200/csrc/build.py` "
                               "(the RFSN B200 path has no CPU fallback)")
        handle = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = handle
    return _LIB


def check(fn_name: str, status: int) -> None:
    if status != 0:
        detail = ""
        if status == -3:
            detail = lib().rfsn_last_cuda_error().decode(errors="replace")
        raise RFSNError(fn_name, status, detail)


def call(fn_name: str, *args) -> None:
    check(fn_name, getattr(lib(), fn_name)(*args))
