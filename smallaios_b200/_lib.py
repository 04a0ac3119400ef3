"""ctypes binding of libsa_b200.so (include/sa_b200.h).

The compute path of this package is the CUDA library and nothing else: if the
library is missing or fails to load, importing this module raises -- there is
no CPU or PyTorch fallback.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIB_PATH = Path(os.environ.get("SA_B200_LIB", _PKG / "libsa_b200.so"))

SA_OK = 0
SA_ERR_INVALID_ATTRIBUTE = 1
SA_ERR_SHAPE_MISMATCH = 2
SA_ERR_UNSUPPORTED = 3
SA_ERR_CAPACITY = 4
SA_ERR_OUT_OF_MEMORY = 5
SA_ERR_CUDA = 6
SA_ERR_DEVICE_CHECK = 7
SA_ERR_TIMEOUT = 8
SA_ERR_INVALID_ARGUMENT = 9

SA_DTYPE_FLOAT = 1
SA_DTYPE_FLOAT16 = 10
SA_DTYPE_BFLOAT16 = 16

# Every symbol include/sa_b200.h declares (checked by tests/test_lib_exports.py).
EXPORTED = [
    "sa_last_error_string", "sa_status_string", "sa_version", "sa_kernel_launches",
    "sa_kv_cache_create", "sa_kv_cache_destroy", "sa_kv_cache_reset", "sa_kv_cache_position",
    "sa_kv_cache_set_position", "sa_kv_cache_advance", "sa_kv_cache_layer_view", "sa_kv_cache_get_config", "sa_kv_cache_memory_bytes",
    "sa_kv_cache_device_status", "sa_kv_cache_set_gather",
    "sa_kv_append", "sa_gqa_attend", "sa_group_query_attention", "sa_matmul_nbits", "sa_gqa_attend_no_alloc",
    "sa_matmul_nbits_packed_bytes", "sa_matmul_nbits_prepack", "sa_matmul_nbits_packed",
    "sa_qkv_project_append", "sa_rms_norm", "sa_silu_mul", "sa_rotary_embedding",
]
SA_STATIC_SCRATCH_BYTES = 8 << 20


class KvCacheConfig(ctypes.Structure):
    _fields_ = [
        ("num_layers", ctypes.c_int32),
        ("batch", ctypes.c_int32),
        ("num_heads", ctypes.c_int32),
        ("num_kv_heads", ctypes.c_int32),
        ("kv_head_begin", ctypes.c_int32),
        ("kv_head_count", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("max_seq_len", ctypes.c_int32),
        ("bits", ctypes.c_int32),
        ("seed", ctypes.c_uint64),
        ("qjl_residual", ctypes.c_int32),
        ("lowrank_k", ctypes.c_int32),
    ]


class KvLayerView(ctypes.Structure):
    _fields_ = [
        ("k_codes", ctypes.c_void_p),
        ("v_codes", ctypes.c_void_p),
        ("k_meta", ctypes.c_void_p),
        ("v_meta", ctypes.c_void_p),
        ("signs", ctypes.c_void_p),
        ("batch", ctypes.c_int32),
        ("kv_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("bits", ctypes.c_int32),
        ("code_bytes", ctypes.c_int32),
        ("capacity", ctypes.c_int32),
        ("wht_scale", ctypes.c_float),
        ("k_qjl_bits", ctypes.c_void_p),
        ("v_qjl_bits", ctypes.c_void_p),
        ("k_qjl_mag", ctypes.c_void_p),
        ("v_qjl_mag", ctypes.c_void_p),
        ("lr_vt", ctypes.c_void_p),
        ("lr_us", ctypes.c_void_p),
        ("lr_kmeta", ctypes.c_void_p),
        ("lr_vtr", ctypes.c_void_p),
    ]


_P = ctypes.c_void_p
_I32 = ctypes.c_int32
_I64 = ctypes.c_int64
_F = ctypes.c_float


def _declare(l: ctypes.CDLL) -> None:
    l.sa_last_error_string.restype = ctypes.c_char_p
    l.sa_last_error_string.argtypes = []
    l.sa_status_string.restype = ctypes.c_char_p
    l.sa_status_string.argtypes = [ctypes.c_int]
    l.sa_version.restype = ctypes.c_int
    l.sa_version.argtypes = []
    l.sa_kernel_launches.restype = ctypes.c_uint64
    l.sa_kernel_launches.argtypes = []
    l.sa_kv_cache_create.restype = ctypes.c_int
    l.sa_kv_cache_create.argtypes = [ctypes.POINTER(KvCacheConfig), ctypes.POINTER(_P)]
    l.sa_kv_cache_destroy.restype = ctypes.c_int
    l.sa_kv_cache_destroy.argtypes = [_P]
    l.sa_kv_cache_reset.restype = ctypes.c_int
    l.sa_kv_cache_reset.argtypes = [_P]
    l.sa_kv_cache_position.restype = ctypes.c_int
    l.sa_kv_cache_position.argtypes = [_P, ctypes.POINTER(_I64)]
    l.sa_kv_cache_set_position.restype = ctypes.c_int
    l.sa_kv_cache_set_position.argtypes = [_P, _I64]
    l.sa_kv_cache_advance.restype = ctypes.c_int
    l.sa_kv_cache_advance.argtypes = [_P, _I64]
    l.sa_kv_cache_layer_view.restype = ctypes.c_int
    l.sa_kv_cache_layer_view.argtypes = [_P, _I32, ctypes.POINTER(KvLayerView)]
    l.sa_kv_cache_get_config.restype = ctypes.c_int
    l.sa_kv_cache_get_config.argtypes = [_P, ctypes.POINTER(KvCacheConfig)]
    l.sa_kv_cache_memory_bytes.restype = ctypes.c_int
    l.sa_kv_cache_memory_bytes.argtypes = [_P, ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_uint64)]
    l.sa_kv_cache_device_status.restype = ctypes.c_int
    l.sa_kv_cache_device_status.argtypes = [_P, ctypes.POINTER(_I32), _I32]
    l.sa_kv_cache_set_gather.restype = ctypes.c_int
    l.sa_kv_cache_set_gather.argtypes = [_P, ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_void_p), _I32,
                                         _I32, _I32, _I32, _I64]
    l.sa_kv_append.restype = ctypes.c_int
    l.sa_kv_append.argtypes = [_P, _I32, _P, _P, _I32, _I32, _I32, _P, _P, _I32, _I32, _I32, _P]
    l.sa_gqa_attend.restype = ctypes.c_int
    l.sa_gqa_attend.argtypes = [_P, _I32, _P, _P, _I32, _I32, _I32, _I64, _I32, _F, _P, _P, _I32, _I32, _I32, _P]
    l.sa_group_query_attention.restype = ctypes.c_int
    l.sa_group_query_attention.argtypes = [_P, _I32, _P, _P, _P, _P, _I32, _I32, _I32, _I64, _I64, _I32, _F, _I64,
                                           _I32, _I32, _P, _P, _I32, _P]
    l.sa_gqa_attend_no_alloc.restype = ctypes.c_int
    l.sa_gqa_attend_no_alloc.argtypes = [ctypes.POINTER(KvLayerView), _I64, _P, _P, _I32, _I32, _I32, _I32, _I32, _F,
                                         _P, _P, _I32, _I32, _I32, _P]
    l.sa_matmul_nbits.restype = ctypes.c_int
    l.sa_matmul_nbits.argtypes = [_P, _P, _P, _P, _P, _P, _I32, _I64, _I64, _I64, _I32, _I32, _P]
    l.sa_matmul_nbits_packed_bytes.restype = _I64
    l.sa_matmul_nbits_packed_bytes.argtypes = [_I64, _I64, _I32, _I32, _I32]
    l.sa_matmul_nbits_prepack.restype = ctypes.c_int
    l.sa_matmul_nbits_prepack.argtypes = [_P, _P, _P, _I32, _I64, _I64, _I32, _I32, _P]
    l.sa_matmul_nbits_packed.restype = ctypes.c_int
    l.sa_matmul_nbits_packed.argtypes = [_P, _P, _P, _P, _I32, _I64, _I64, _I64, _I32, _I32, _P]
    l.sa_rms_norm.restype = ctypes.c_int
    l.sa_rms_norm.argtypes = [_P, _P, _P, _P, _P, _P, _I32, _I64, _I64, _F, _P]
    l.sa_silu_mul.restype = ctypes.c_int
    l.sa_silu_mul.argtypes = [_P, _P, _I64, _P, _I32, _I64, _I64, _P]
    l.sa_rotary_embedding.restype = ctypes.c_int
    l.sa_rotary_embedding.argtypes = [_P, _P, _I32, _I32, _I64, _I64, _I64, _I32, _P, _P, _I32, _I64, _I32, _P, _I32,
                                      _I64, _I64, _I32, _I32, _P, _P]
    l.sa_qkv_project_append.restype = ctypes.c_int
    l.sa_qkv_project_append.argtypes = [_P, _I32, _P, _P, _P, _I32, _I32, _I64, _P, _P, _I32, _I32, _I32, _P, _P,
                                        _P, _P]


def _load() -> ctypes.CDLL:
    if not LIB_PATH.exists():
        raise ImportError(
            f"smallaios_b200: {LIB_PATH} is missing; build it with `python smallaios_b200/build.py` "
            "(there is no CPU fallback)")
    l = ctypes.CDLL(str(LIB_PATH))
    _declare(l)
    return l


lib = _load()


class SaError(RuntimeError):
    """A non-zero sa_status from the library (message from sa_last_error_string)."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{lib.sa_status_string(status).decode()}: {message}")
        self.status = status


def check(status: int) -> None:
    if status != SA_OK:
        raise SaError(status, lib.sa_last_error_string().decode(errors="replace"))
