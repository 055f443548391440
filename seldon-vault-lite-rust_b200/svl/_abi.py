"""ctypes mirror of include/svl_gpu.h (structs and prototypes).

The same struct definitions describe the CPU oracle's model input, so the
test-side oracle wrapper imports them from here.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

from . import errors

c_u32 = ctypes.c_uint32
c_u64 = ctypes.c_uint64
c_f32 = ctypes.c_float
c_ptr = ctypes.c_void_p
c_char_p = ctypes.c_char_p
c_size = ctypes.c_size_t


class SvlLayerConfig(ctypes.Structure):
    _fields_ = [("layer_type", c_u32), ("head_dim", c_u32), ("num_key_value_heads", c_u32)]


class SvlTextConfig(ctypes.Structure):
    _fields_ = [
        ("vocab_size", c_u32),
        ("hidden_size", c_u32),
        ("intermediate_size", c_u32),
        ("num_hidden_layers", c_u32),
        ("num_attention_heads", c_u32),
        ("hidden_size_per_layer_input", c_u32),
        ("embedding_dim", c_u32),
        ("max_position_embeddings", c_u32),
        ("sliding_window", c_u32),
        ("pad_token_id", ctypes.c_int64),
        ("rms_norm_eps", c_f32),
        ("embedding_scale", c_f32),
        ("ple_scale", c_f32),
        ("full_rope_theta", c_f32),
        ("sliding_rope_theta", c_f32),
        ("layers", ctypes.POINTER(SvlLayerConfig)),
    ]


class SvlTensorView(ctypes.Structure):
    _fields_ = [
        ("name", c_char_p),
        ("data", c_ptr),
        ("dtype", c_u32),
        ("ndim", c_u32),
        ("shape", c_u64 * 4),
    ]


class SvlModelOptions(ctypes.Structure):
    _fields_ = [("precision", ctypes.c_uint32), ("reserved", ctypes.c_uint32 * 7)]


PRECISION_FAST = 0
PRECISION_SPLIT = 1


class SvlFeatureSpan(ctypes.Structure):
    _fields_ = [
        ("sequence", c_u32),
        ("start", c_u32),
        ("count", c_u32),
        ("reserved", c_u32),
        ("feature_offset", c_u64),
    ]


DTYPE_F32 = 0
DTYPE_BF16 = 1

# name -> (restype, argtypes); every int-returning call returns svl_status
PROTOTYPES = {
    "svl_abi_version": (c_u32, []),
    "svl_device_count": (ctypes.c_int, []),
    "svl_model_create": (ctypes.c_int, [ctypes.POINTER(SvlTextConfig), ctypes.POINTER(SvlTensorView), c_size, ctypes.c_int, ctypes.POINTER(c_ptr), c_char_p, c_size]),
    "svl_model_create_ex": (ctypes.c_int, [ctypes.POINTER(SvlTextConfig), ctypes.POINTER(SvlTensorView), c_size, ctypes.c_int, ctypes.POINTER(SvlModelOptions), ctypes.POINTER(c_ptr), c_char_p, c_size]),
    "svl_model_precision": (ctypes.c_int, [c_ptr, ctypes.POINTER(ctypes.c_uint32)]),
    "svl_model_destroy": (None, [c_ptr]),
    "svl_model_parameters": (ctypes.c_int, [c_ptr, ctypes.POINTER(c_u64)]),
    "svl_forward_batch": (ctypes.c_int, [c_ptr, c_ptr, c_ptr, c_u32, c_ptr, c_ptr, c_u32, c_ptr, c_ptr, c_ptr, c_ptr, c_char_p, c_size]),
    "svl_embed_batch": (ctypes.c_int, [c_ptr, c_ptr, c_ptr, c_u32, c_u32, c_ptr, c_char_p, c_size]),
    "svl_embed_batch_device": (ctypes.c_int, [c_ptr, c_ptr, c_ptr, c_u32, c_u32, c_ptr, c_ptr, c_char_p, c_size]),
    "svl_model_check": (ctypes.c_int, [c_ptr, c_char_p, c_size]),
    "svl_index_create": (ctypes.c_int, [ctypes.c_int, c_u32, c_u64, ctypes.POINTER(c_ptr), c_char_p, c_size]),
    "svl_index_destroy": (None, [c_ptr]),
    "svl_index_len": (c_u64, [c_ptr]),
    "svl_index_dim": (c_u32, [c_ptr]),
    "svl_index_append": (ctypes.c_int, [c_ptr, c_ptr, c_ptr, c_u64, c_char_p, c_size]),
    "svl_index_append_device": (ctypes.c_int, [c_ptr, c_ptr, c_ptr, c_u64, c_ptr, c_char_p, c_size]),
    "svl_ingest_batch": (ctypes.c_int, [c_ptr, c_ptr, c_ptr, c_ptr, c_u32, c_ptr, c_char_p, c_size]),
    "svl_index_search": (ctypes.c_int, [c_ptr, c_ptr, c_u32, c_u32, c_ptr, c_u32, c_ptr, c_ptr, c_ptr, c_ptr, c_char_p, c_size]),
    "svl_index_search_device": (ctypes.c_int, [c_ptr, c_ptr, c_u32, c_ptr, c_u32, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_char_p, c_size]),
    "svl_index_check": (ctypes.c_int, [c_ptr, c_char_p, c_size]),
    "svl_merge_topk_device": (ctypes.c_int, [ctypes.c_int, c_ptr, c_ptr, c_ptr, c_ptr, c_u32, c_u32, c_u32, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_char_p, c_size]),
    "svl_nccl_unique_id": (ctypes.c_int, [c_ptr, c_char_p, c_size]),
    "svl_nccl_comm_create": (ctypes.c_int, [ctypes.c_int, ctypes.c_int, ctypes.c_int, c_ptr, ctypes.POINTER(c_ptr), c_char_p, c_size]),
    "svl_nccl_comm_destroy": (ctypes.c_int, [c_ptr, ctypes.c_int]),
    "svl_allgather_rows": (ctypes.c_int, [c_ptr, c_ptr, c_u64, c_u32, c_ptr, c_ptr, c_char_p, c_size]),
    "svl_sharded_search": (ctypes.c_int, [c_ptr, c_ptr, c_u64, c_ptr, c_u32, c_u32, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_char_p, c_size]),
    "svl_search_noalloc": (ctypes.c_int, [c_ptr, c_ptr, c_u64, c_u32, c_ptr, c_u32, c_ptr, c_u32, c_ptr, c_ptr, c_ptr, c_ptr, c_ptr, c_char_p, c_size]),
}

PACKAGE_ROOT = Path(__file__).resolve().parent.parent
LIBRARY_PATH = PACKAGE_ROOT / "build" / "libsvl_gpu.so"

_lib = None


def load_library(path: str | os.PathLike | None = None) -> ctypes.CDLL:
    """Loads libsvl_gpu.so (built in-tree by `make -C seldon-vault-lite-rust_b200`).

    There is no fallback: a missing library is an error, never a CPU path."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path else LIBRARY_PATH
    if not p.exists():
        raise errors.InternalError(
            f"{p} is missing: build the CUDA library first (make -C seldon-vault-lite-rust_b200)"
        )
    lib = ctypes.CDLL(str(p))
    for name, (res, args) in PROTOTYPES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if lib.svl_abi_version() != 1:
        raise errors.InternalError("libsvl_gpu.so ABI version mismatch")
    if path is None:
        _lib = lib
    return lib


class ErrBuf:
    """A message buffer for the (err, err_len) pair of every call."""

    def __init__(self, size: int = 512):
        self.buf = ctypes.create_string_buffer(size)

    @property
    def args(self):
        return self.buf, len(self.buf)

    def check(self, status: int) -> None:
        errors.raise_for_status(status, self.buf.value.decode(errors="replace"))


def tensor_views(tensors: dict):
    """Builds an svl_tensor_view array from {name: TensorEntry | ndarray}."""
    import numpy as np

    views = (SvlTensorView * len(tensors))()
    keep = []
    for i, (name, t) in enumerate(tensors.items()):
        if hasattr(t, "raw"):
            arr, dtype, shape = t.raw, (DTYPE_BF16 if t.dtype == "BF16" else DTYPE_F32), t.shape
        else:
            arr = np.ascontiguousarray(t, dtype=np.float32)
            dtype, shape = DTYPE_F32, arr.shape
        arr = np.ascontiguousarray(arr)
        keep.append(arr)
        nb = name.encode()
        keep.append(nb)
        views[i].name = nb
        views[i].data = arr.ctypes.data
        views[i].dtype = dtype
        views[i].ndim = len(shape)
        for d, s in enumerate(shape):
            views[i].shape[d] = s
    return views, keep
