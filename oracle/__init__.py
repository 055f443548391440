"""ctypes wrapper of the CPU parity oracle (oracle/_build/libsvl_oracle.so).

TEST INFRASTRUCTURE ONLY.  Imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg, and nowhere else.  It restates the reference's
scalar FP32 path (src/tensor/kernels.rs, src/model/text.rs:182-538) and its
f64 vector rank (src/index/vector.rs:17-97); see svl_oracle.cpp.

Parity pin: tests/test_oracle_golden.py checks this oracle against the
reference's own tiny_text golden fixture and kernel known-answer tests.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "libsvl_oracle.so"

_lib = None


def build() -> Path:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = ctypes.CDLL(str(LIB_PATH))
        P, S, F, I = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_float, ctypes.c_int
        for name, args in {
            "orc_linear": [P, P, S, S, S, P],
            "orc_matmul": [P, P, S, S, S, P],
            "orc_rms_norm_rows": [P, P, S, S, F, P],
            "orc_geglu": [P, P, S, P],
            "orc_softmax": [P, S, P],
            "orc_l2_normalize": [P, S, P],
            "orc_mean_pool": [P, S, S, P],
            "orc_truncate_and_normalize": [P, S, S, P],
            "orc_rope_inv_freq": [S, F, P],
            "orc_rope_with_inv_freq": [P, S, S, S, P, S, S],
            "orc_bidirectional_attention": [P, P, P, S, S, S, S, ctypes.c_int64, F, P],
            "orc_model_create": [P, P, S, ctypes.POINTER(P), ctypes.c_char_p, S],
            "orc_forward": [P, P, S, P, S, S, P, P, P, P, ctypes.c_char_p, S],
            "orc_vector_rank": [P, S, P, S, P, P, P, P, ctypes.POINTER(S), I],
            "orc_vector_topk": [P, S, S, P, S, P, S, P, P, I],
            "orc_normalize_embedding": [P, S],
            "orc_embed_many": [P, P, P, S, S, P, I],
        }.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = I
        L.orc_gelu_tanh_value.argtypes = [F]
        L.orc_gelu_tanh_value.restype = F
        L.orc_model_destroy.argtypes = [P]
        L.orc_model_destroy.restype = None
        _lib = L
    return _lib


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _p(a):
    return a.ctypes.data if a is not None else None


class OracleError(Exception):
    def __init__(self, code, msg=""):
        super().__init__(f"oracle status {code}: {msg}")
        self.code = code


def _check(code, msg=""):
    if code:
        raise OracleError(code, msg)


# ---------------------------------------------------------------- kernels --
def linear(x, w):
    x, w = _f32(x), _f32(w)
    rows, inf = x.shape
    outf = w.shape[0]
    out = np.empty((rows, outf), np.float32)
    _check(lib().orc_linear(_p(x), _p(w), rows, inf, outf, _p(out)))
    return out


def matmul(a, b):
    a, b = _f32(a), _f32(b)
    out = np.empty((a.shape[0], b.shape[1]), np.float32)
    _check(lib().orc_matmul(_p(a), _p(b), a.shape[0], a.shape[1], b.shape[1], _p(out)))
    return out


def rms_norm_rows(x, w, width, eps):
    x = _f32(x)
    w = None if w is None else _f32(w)
    out = np.empty_like(x)
    _check(lib().orc_rms_norm_rows(_p(x), _p(w), x.size // width, width, eps, _p(out)))
    return out


def gelu_tanh_value(v):
    return lib().orc_gelu_tanh_value(float(v))


def geglu(g, u):
    g, u = _f32(g), _f32(u)
    out = np.empty_like(g)
    _check(lib().orc_geglu(_p(g), _p(u), g.size, _p(out)))
    return out


def softmax(v):
    v = _f32(v)
    out = np.empty_like(v)
    _check(lib().orc_softmax(_p(v), v.size, _p(out)))
    return out


def l2_normalize(v):
    v = _f32(v)
    out = np.empty_like(v)
    _check(lib().orc_l2_normalize(_p(v), v.size, _p(out)))
    return out


def mean_pool(v, rows, width):
    v = _f32(v)
    out = np.empty(width, np.float32)
    _check(lib().orc_mean_pool(_p(v), rows, width, _p(out)))
    return out


def truncate_and_normalize(v, dim):
    v = _f32(v)
    out = np.empty(dim, np.float32)
    _check(lib().orc_truncate_and_normalize(_p(v), v.size, dim, _p(out)))
    return out


def rope_inv_freq(head_dim, base):
    out = np.empty(head_dim // 2, np.float32)
    _check(lib().orc_rope_inv_freq(head_dim, base, _p(out)))
    return out


def rope(values, seq, heads, head_dim, inv, offset=0):
    v = _f32(values).copy()
    inv = _f32(inv)
    _check(lib().orc_rope_with_inv_freq(_p(v), seq, heads, head_dim, _p(inv), inv.size, offset))
    return v


def attention(q, k, v, seq, nh, nkv, hd, window=None, scale=1.0):
    q, k, v = _f32(q), _f32(k), _f32(v)
    out = np.empty(seq * nh * hd, np.float32)
    _check(lib().orc_bidirectional_attention(_p(q), _p(k), _p(v), seq, nh, nkv, hd,
                                             -1 if window is None else window, scale, _p(out)))
    return out


# ------------------------------------------------------------------ model --
class OracleModel:
    """The reference's TextModel on the CPU: forward / embed over host weights."""

    def __init__(self, config, tensors: dict):
        from svl._abi import tensor_views

        self.config = config
        self._cfg, self._keep_cfg = config.to_c()
        views, self._keep = tensor_views(tensors)
        handle = ctypes.c_void_p()
        err = ctypes.create_string_buffer(512)
        _check(lib().orc_model_create(ctypes.addressof(self._cfg), ctypes.addressof(views), len(tensors),
                                      ctypes.byref(handle), err, 512), err.value.decode())
        self._h = handle

    def close(self):
        if self._h:
            lib().orc_model_destroy(self._h)
            self._h = None

    __del__ = close

    def forward(self, ids, capture_hidden=False, features=None, feature_start=0):
        c = self.config
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        seq = ids.size
        projected = np.empty((seq, c.embedding_dim), np.float32)
        pooled = np.empty(c.embedding_dim, np.float32)
        normalized = np.empty(c.embedding_dim, np.float32)
        hidden = np.empty((c.num_hidden_layers + 1, seq, c.hidden_size), np.float32) if capture_hidden else None
        feats = None if features is None else _f32(features)
        count = 0 if feats is None else feats.size // c.hidden_size
        err = ctypes.create_string_buffer(512)
        _check(lib().orc_forward(self._h, _p(ids), seq, _p(feats), feature_start, count, _p(projected),
                                 _p(pooled), _p(normalized), _p(hidden), err, 512), err.value.decode())
        return {"projected": projected, "pooled": pooled, "normalized": normalized, "hidden_states": hidden}

    def embed_many(self, ids, cu_seqlens, dimension, threads=None):
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        cu = np.ascontiguousarray(cu_seqlens, dtype=np.uint64)
        batch = cu.size - 1
        out = np.empty((batch, dimension), np.float32)
        threads = threads or os.cpu_count() or 1
        _check(lib().orc_embed_many(self._h, _p(ids), _p(cu), batch, dimension, _p(out), threads))
        return out


# ----------------------------------------------------------------- search --
def normalize_embedding(v):
    v = _f32(v).copy()
    _check(lib().orc_normalize_embedding(_p(v), v.size))
    return v


def vector_rank(query, corpus, chunk_ids=None, row_mask=None):
    q, c = _f32(query), _f32(corpus)
    n, d = c.shape
    ids = np.ascontiguousarray(np.arange(n, dtype=np.uint64) if chunk_ids is None else chunk_ids, dtype=np.uint64)
    mask = None if row_mask is None else np.ascontiguousarray(row_mask, dtype=np.uint8)
    rows = np.empty(n, np.uint64)
    scores = np.empty(n, np.float64)
    count = ctypes.c_size_t()
    _check(lib().orc_vector_rank(_p(q), q.size, _p(c), n, _p(ids), _p(mask), _p(rows), _p(scores),
                                 ctypes.byref(count), 1))
    return rows[: count.value], scores[: count.value]


def vector_topk(queries, corpus, k, chunk_ids=None, threads=None):
    q, c = _f32(queries), _f32(corpus)
    nq, d = q.shape
    n = c.shape[0]
    ids = np.ascontiguousarray(np.arange(n, dtype=np.uint64) if chunk_ids is None else chunk_ids, dtype=np.uint64)
    rows = np.empty((nq, k), np.uint64)
    scores = np.empty((nq, k), np.float64)
    _check(lib().orc_vector_topk(_p(q), nq, d, _p(c), n, _p(ids), k, _p(rows), _p(scores),
                                 threads or os.cpu_count() or 1))
    return rows, scores
