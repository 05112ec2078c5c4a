"""ORACLE (test infrastructure only): ctypes wrapper over ``oracle/liboracle.so``.

``ref_cpu.cpp`` restates glypr's CPU text-embedding path (see its header for the file:line
map).  Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
reference arm may import this package, and only as the checker or the timed CPU baseline;
the product (``glypr_b200`` and ``libglypr_cuda.so``) never does.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading
from typing import Optional

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lock = threading.Lock()
_lib: Optional[ctypes.CDLL] = None

M1_CANDLE = 1  # activations quantised to Q8_0, int8 block dots (candle QMatMul on CPU)
M2_EXACT = 2   # exact f32 dequantisation, f64 accumulation


def build(force: bool = False) -> str:
    src = os.path.join(_HERE, "ref_cpu.cpp")
    if force or not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", _HERE, "liboracle.so"], check=True)
    return _LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    with _lock:
        if _lib is None:
            build()
            L = ctypes.CDLL(_LIB_PATH)
            P, I, I64, F, D = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_double
            L.oracle_open.restype = P
            L.oracle_open.argtypes = [ctypes.c_char_p]
            L.oracle_close.argtypes = [P]
            L.oracle_last_error.restype = ctypes.c_char_p
            L.oracle_info.argtypes = [P, P]
            L.oracle_set_threads.argtypes = [I]
            L.oracle_set_simd.argtypes = [I]
            L.oracle_max_threads.restype = I
            L.oracle_embed.argtypes = [P, P, P, I, I, I, I, P]
            L.oracle_hidden.argtypes = [P, P, I, I, I, P]
            L.oracle_tokens.argtypes = [P, P, I, I, P]
            L.oracle_q8_0_dequant.argtypes = [P, I64, P]
            L.oracle_q8_0_quantize.argtypes = [P, I64, P]
            L.oracle_q8_0_matmul.argtypes = [P, I, I, P, I, I, P]
            L.oracle_rmsnorm.argtypes = [P, P, I64, I64, F, P]
            L.oracle_geglu.argtypes = [P, P, I64, P]
            L.oracle_rope_tables.argtypes = [I, D, I64, P, P]
            L.oracle_attention.argtypes = [P, P, P, I64, I, I, I, I, I, P]
            L.oracle_pool_normalize.argtypes = [P, I64, I64, I, P]
            _lib = L
        return _lib


def _p(a: Optional[np.ndarray]):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def set_threads(n: int) -> None:
    lib().oracle_set_threads(int(n))


def set_simd(on: bool) -> None:
    """AVX2 block dots and attention (default) or the scalar loops: identical results."""
    lib().oracle_set_simd(int(bool(on)))


def max_threads() -> int:
    return int(lib().oracle_max_threads())


class OracleModel:
    """The reference CPU forward on a GGUF file (per-sequence, valid tokens only)."""

    def __init__(self, path: str):
        self._h = lib().oracle_open(path.encode())
        if not self._h:
            raise RuntimeError(lib().oracle_last_error().decode())
        info = np.zeros(10, dtype=np.int32)
        lib().oracle_info(self._h, _p(info))
        (self.n_layers, self.hidden, self.ffn, self.n_heads, self.vocab, self.emb_out,
         self.max_pos, self.head_dim, self.n_kv, self.window) = (int(v) for v in info)

    def close(self) -> None:
        if self._h:
            lib().oracle_close(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def embed(self, ids: np.ndarray, lengths: np.ndarray, mode: int = M1_CANDLE,
              out_dim: Optional[int] = None) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        lengths = np.ascontiguousarray(lengths, dtype=np.int32)
        n, s = ids.shape
        od = out_dim or self.emb_out
        out = np.zeros((n, od), dtype=np.float32)
        rc = lib().oracle_embed(self._h, _p(ids), _p(lengths), n, s, mode, od, _p(out))
        if rc:
            raise RuntimeError(lib().oracle_last_error().decode())
        return out

    def hidden_after(self, ids: np.ndarray, layer: int, mode: int = M1_CANDLE) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        out = np.zeros((ids.size, self.hidden), dtype=np.float32)
        rc = lib().oracle_hidden(self._h, _p(ids), ids.size, layer, mode, _p(out))
        if rc:
            raise RuntimeError(lib().oracle_last_error().decode())
        return out

    def tokens(self, ids: np.ndarray, mode: int = M1_CANDLE) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        out = np.zeros((ids.size, self.emb_out), dtype=np.float32)
        lib().oracle_tokens(self._h, _p(ids), ids.size, mode, _p(out))
        return out


# ---- kernel-level restatements --------------------------------------------------------

def q8_0_dequant(blocks: np.ndarray) -> np.ndarray:
    raw = np.ascontiguousarray(blocks).view(np.uint8).reshape(-1)
    nb = raw.size // 34
    out = np.empty(nb * 32, dtype=np.float32)
    lib().oracle_q8_0_dequant(_p(raw), nb, _p(out))
    return out


def q8_0_quantize(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    out = np.empty(x.size // 32 * 34, dtype=np.uint8)
    lib().oracle_q8_0_quantize(_p(x), x.size, _p(out))
    return out


def q8_0_matmul(w_blocks: np.ndarray, n: int, k: int, x: np.ndarray, mode: int) -> np.ndarray:
    raw = np.ascontiguousarray(w_blocks).view(np.uint8).reshape(-1)
    x = np.ascontiguousarray(x, dtype=np.float32)
    m = x.shape[0]
    y = np.empty((m, n), dtype=np.float32)
    rc = lib().oracle_q8_0_matmul(_p(raw), n, k, _p(x), m, mode, _p(y))
    if rc:
        raise RuntimeError(lib().oracle_last_error().decode())
    return y


def rmsnorm(x: np.ndarray, w: Optional[np.ndarray], eps: float = 1e-6) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    d = x.shape[-1]
    out = np.empty_like(x)
    wv = None if w is None else np.ascontiguousarray(w, dtype=np.float32)
    lib().oracle_rmsnorm(_p(x), _p(wv), x.size // d, d, eps, _p(out))
    return out


def geglu(g: np.ndarray, u: np.ndarray) -> np.ndarray:
    g = np.ascontiguousarray(g, dtype=np.float32)
    u = np.ascontiguousarray(u, dtype=np.float32)
    out = np.empty_like(g)
    lib().oracle_geglu(_p(g), _p(u), g.size, _p(out))
    return out


def rope_tables(d: int, theta: float, s: int):
    c = np.empty((s, d), dtype=np.float32)
    sn = np.empty((s, d), dtype=np.float32)
    lib().oracle_rope_tables(d, theta, s, _p(c), _p(sn))
    return c, sn


def attention(q, k, v, n_heads: int, n_kv: int, d: int, window: int, sliding: bool) -> np.ndarray:
    q = np.ascontiguousarray(q, dtype=np.float32)
    k = np.ascontiguousarray(k, dtype=np.float32)
    v = np.ascontiguousarray(v, dtype=np.float32)
    t = q.shape[0]
    out = np.empty((t, n_heads * d), dtype=np.float32)
    lib().oracle_attention(_p(q), _p(k), _p(v), t, n_heads, n_kv, d, window, int(sliding), _p(out))
    return out


def pool_normalize(tok: np.ndarray, out_dim: Optional[int] = None) -> np.ndarray:
    tok = np.ascontiguousarray(tok, dtype=np.float32)
    t, e = tok.shape
    od = out_dim or e
    out = np.empty(od, dtype=np.float32)
    lib().oracle_pool_normalize(_p(tok), t, e, od, _p(out))
    return out
