"""ctypes front end of the CPU oracle (oracle.cpp).

TEST INFRASTRUCTURE ONLY: tests/, __graft_entry__.smoke() and bench.py's CPU
baseline legs use this module as the checker.  The shipped engine never imports
it.  Every function mirrors a reference function; oracle.cpp cites file:line for
each one.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(dtype=np.uint8, flags="C_CONTIGUOUS")
_szp = np.ctypeslib.ndpointer(dtype=np.uintp, flags="C_CONTIGUOUS")


def build() -> str:
    """Compile liboracle.so with the oracle's Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(
        os.path.join(_HERE, "oracle.cpp")
    ):
        build()
    L = C.CDLL(_LIB_PATH)
    sz, f32, i32 = C.c_size_t, C.c_float, C.c_int
    L.or_set_threads.argtypes = [i32]
    L.or_max_threads.restype = i32
    L.or_quantize_q4_0.argtypes = [_f32p, sz, _u8p]
    L.or_quantize_q8_0.argtypes = [_f32p, sz, _u8p]
    L.or_q4_0_dequant.argtypes = [_u8p, sz, i32, _f32p]
    for n in ("or_q4_0_dot_avx2", "or_q4_0_dot_scalar", "or_q8_0_dot_avx2"):
        getattr(L, n).argtypes = [_u8p, _f32p, sz]
        getattr(L, n).restype = f32
    L.or_lut4_dot.argtypes = [_u8p, _f32p, _f32p, sz, sz]
    L.or_lut4_dot.restype = f32
    L.or_dot_f32.argtypes = [_f32p, _f32p, sz]
    L.or_dot_f32.restype = f32
    L.or_rms_norm.argtypes = [_f32p, _f32p, f32, sz, _f32p]
    L.or_swiglu_balanced.argtypes = [_f32p, _f32p, _f32p, sz]
    L.or_kwta.argtypes = [_f32p, sz, sz]
    L.or_rope.argtypes = [_f32p, sz, sz, sz, f32, i32]
    L.or_q4_0_gemv.argtypes = [_u8p, _f32p, C.c_void_p, sz, sz, _f32p]
    L.or_f32_gemv.argtypes = [_f32p, _f32p, sz, sz, _f32p]
    L.or_load.argtypes = [C.c_char_p, C.c_char_p, sz]
    L.or_load.restype = C.c_void_p
    L.or_free.argtypes = [C.c_void_p]
    L.or_info.argtypes = [C.c_void_p, sz]
    L.or_info.restype = sz
    L.or_info_f.argtypes = [C.c_void_p, sz]
    L.or_info_f.restype = f32
    L.or_last_error.argtypes = [C.c_void_p]
    L.or_last_error.restype = C.c_char_p
    L.or_set_k_wta_ratio.argtypes = [C.c_void_p, f32]
    L.or_clear_cache.argtypes = [C.c_void_p]
    L.or_forward.argtypes = [C.c_void_p, sz, i32, C.c_void_p]
    L.or_forward.restype = i32
    L.or_forward_hidden.argtypes = [C.c_void_p, sz, i32, _f32p]
    L.or_forward_hidden.restype = i32
    L.or_linear.argtypes = [C.c_void_p, i32, i32, _f32p, sz, _f32p]
    L.or_linear.restype = i32
    L.or_get_row.argtypes = [C.c_void_p, i32, i32, sz, _f32p]
    L.or_get_row.restype = i32
    L.or_generate.argtypes = [C.c_void_p, _szp, sz, sz, f32, f32, _szp, sz, C.c_uint64, _szp,
                              C.POINTER(C.c_size_t)]
    L.or_generate.restype = i32
    L.or_fill_normal.argtypes = [_f32p, sz, C.c_uint64, C.c_char_p, f32]
    L.or_genomize_4bit.argtypes = [_f32p, sz, _u8p, _f32p]
    L.or_sample_top_p.argtypes = [_f32p, sz, f32, f32, f32, C.POINTER(C.c_size_t)]
    L.or_sample_top_p.restype = sz
    _lib = L
    return L


def set_threads(n: int) -> None:
    lib().or_set_threads(int(n))


def max_threads() -> int:
    return int(lib().or_max_threads())


# ------------------------------------------------------------------ kernels
def quantize_q4_0(w: np.ndarray) -> np.ndarray:
    """quantize_q4_0_native (src/compute/quantize/python.rs:152-232): 20-byte blocks."""
    w = np.ascontiguousarray(w, dtype=np.float32).ravel()
    out = np.zeros(w.size // 32 * 20, dtype=np.uint8)
    if lib().or_quantize_q4_0(w, w.size, out) != 0:
        raise ValueError("Weights length must be divisible by 32")
    return out


def quantize_q8_0(w: np.ndarray) -> np.ndarray:
    w = np.ascontiguousarray(w, dtype=np.float32).ravel()
    out = np.zeros(w.size // 32 * 34, dtype=np.uint8)
    if lib().or_quantize_q8_0(w, w.size, out) != 0:
        raise ValueError("Weights length must be divisible by 32")
    return out


def sample_top_p(logits, temperature: float, top_p: float, r: float):
    """sample_top_p_core (src/compute/sampling.rs:14-55) with the uniform r
    given: (token, number of tokens kept in the nucleus)."""
    lg = np.ascontiguousarray(logits, np.float32)
    kept = C.c_size_t(0)
    tok = lib().or_sample_top_p(lg, lg.size, float(temperature), float(top_p), float(r), C.byref(kept))
    return int(tok), int(kept.value)


def genomize_4bit(w: np.ndarray):
    """genomize_4bit_core (src/compute/quantize/genomize.rs:286-382), no
    anchors: (nibbles [n/2] high nibble first, centroids [n/32 * 16])."""
    w = np.ascontiguousarray(w, dtype=np.float32).ravel()
    if w.size % 32:
        raise ValueError("length must be divisible by 32")
    nib = np.zeros(w.size // 2, dtype=np.uint8)
    cen = np.zeros(w.size // 32 * 16, dtype=np.float32)
    lib().or_genomize_4bit(w, w.size, nib, cen)
    return nib, cen


def lut4_dot(nibbles, x, centroids, n_blocks: int) -> float:
    """genomic_dot_product_4bit (genomic.rs:149-204) over one row."""
    return float(lib().or_lut4_dot(np.ascontiguousarray(nibbles, np.uint8), np.ascontiguousarray(x, np.float32),
                                   np.ascontiguousarray(centroids, np.float32), 16, int(n_blocks)))


def q4_0_dequant(blocks: np.ndarray, fused: bool = True) -> np.ndarray:
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    nb = blocks.size // 20
    out = np.zeros(nb * 32, dtype=np.float32)
    lib().or_q4_0_dequant(blocks, nb, 1 if fused else 0, out)
    return out


def q4_0_dot(blocks, x, scalar: bool = False) -> float:
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    f = lib().or_q4_0_dot_scalar if scalar else lib().or_q4_0_dot_avx2
    return float(f(blocks, x, blocks.size // 20))


def q8_0_dot(blocks, x) -> float:
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    return float(lib().or_q8_0_dot_avx2(blocks, np.ascontiguousarray(x, np.float32), blocks.size // 34))


def dot_f32(a, b) -> float:
    a = np.ascontiguousarray(a, np.float32)
    return float(lib().or_dot_f32(a, np.ascontiguousarray(b, np.float32), a.size))


def rms_norm(x, w, eps) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    out = np.zeros_like(x)
    lib().or_rms_norm(x, np.ascontiguousarray(w, np.float32), float(eps), x.size, out)
    return out


def swiglu_balanced(g, u) -> np.ndarray:
    g = np.ascontiguousarray(g, np.float32)
    out = np.zeros_like(g)
    lib().or_swiglu_balanced(g, np.ascontiguousarray(u, np.float32), out, g.size)
    return out


def kwta(s, k) -> np.ndarray:
    s = np.array(s, dtype=np.float32, copy=True)
    lib().or_kwta(s, s.size, int(k))
    return s


def rope(vec, heads, head_dim, pos, base, split=True) -> np.ndarray:
    v = np.array(vec, dtype=np.float32, copy=True)
    lib().or_rope(v, heads, head_dim, pos, float(base), 1 if split else 0)
    return v


def q4_0_gemv(blocks, x, N, K, bias=None) -> np.ndarray:
    blocks = np.ascontiguousarray(blocks, np.uint8)
    x = np.ascontiguousarray(x, np.float32)
    y = np.zeros(N, dtype=np.float32)
    b = None
    if bias is not None:
        bias = np.ascontiguousarray(bias, np.float32)
        b = bias.ctypes.data
    lib().or_q4_0_gemv(blocks, x, b, N, K, y)
    return y


def f32_gemv(W, x) -> np.ndarray:
    W = np.ascontiguousarray(W, np.float32)
    y = np.zeros(W.shape[0], dtype=np.float32)
    lib().or_f32_gemv(W, np.ascontiguousarray(x, np.float32), W.shape[0], W.shape[1], y)
    return y


def synthetic_normal(n: int, seed: int, name: str, std: float = 0.02) -> np.ndarray:
    """The synthetic N(0, std) weights of tensor `name` (or `name.bias`) of a
    benchmark / test model, as the product's synthetic writer draws them."""
    v = np.empty(int(n), dtype=np.float32)
    lib().or_fill_normal(v, v.size, int(seed) & 0xFFFFFFFFFFFFFFFF, name.encode(), float(std))
    return v


# -------------------------------------------------------------------- model
class OracleModel:
    """The reference GenomicLLM as loaded by load_genomic_auto from a .flat file."""

    def __init__(self, path: str):
        err = C.create_string_buffer(512)
        self._h = lib().or_load(path.encode(), err, 512)
        if not self._h:
            raise IOError(err.value.decode())
        L = lib()
        self.vocab_size = L.or_info(self._h, 0)
        self.n_embd = L.or_info(self._h, 1)
        self.n_head = L.or_info(self._h, 2)
        self.n_head_kv = L.or_info(self._h, 3)
        self.n_blocks = L.or_info(self._h, 4)
        self.head_dim = L.or_info(self._h, 5)
        self.ffn_dim = L.or_info(self._h, 6)
        self.eps = L.or_info_f(self._h, 0)
        self.rope_base = L.or_info_f(self._h, 1)

    def __del__(self):
        if getattr(self, "_h", None):
            lib().or_free(self._h)
            self._h = None

    @property
    def cache_len(self) -> int:
        return int(lib().or_info(self._h, 7))

    @property
    def k_wta_ratio(self) -> float:
        return float(lib().or_info_f(self._h, 2))

    def set_k_wta_ratio(self, r: float) -> None:
        lib().or_set_k_wta_ratio(self._h, float(r))

    def clear_cache(self) -> None:
        lib().or_clear_cache(self._h)

    def forward(self, token_id: int, clear_cache: bool = False) -> np.ndarray:
        out = np.zeros(self.vocab_size, dtype=np.float32)
        if lib().or_forward(self._h, int(token_id), 1 if clear_cache else 0, out.ctypes.data) != 0:
            raise ValueError(lib().or_last_error(self._h).decode())
        return out

    def forward_hidden(self, token_id: int, clear_cache: bool = False) -> np.ndarray:
        out = np.zeros(self.n_embd, dtype=np.float32)
        if lib().or_forward_hidden(self._h, int(token_id), 1 if clear_cache else 0, out) != 0:
            raise ValueError(lib().or_last_error(self._h).decode())
        return out

    def linear(self, layer: int, which: int, x: np.ndarray, n_out: int) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        y = np.zeros(n_out, dtype=np.float32)
        if lib().or_linear(self._h, layer, which, x, x.size, y) != 0:
            raise ValueError("bad layer")
        return y

    def get_row(self, layer: int, which: int, idx: int, n_in: int) -> np.ndarray:
        out = np.zeros(n_in, dtype=np.float32)
        if lib().or_get_row(self._h, layer, which, idx, out) != 0:
            raise ValueError("bad layer")
        return out

    def generate(self, prompt, max_new_tokens=30, temperature=0.7, repetition_penalty=1.0,
                 eos_token_ids=(2, 151643, 151645), seed=0):
        p = np.ascontiguousarray(prompt, dtype=np.uintp)
        e = np.ascontiguousarray(list(eos_token_ids), dtype=np.uintp)
        if e.size == 0:
            e = np.zeros(1, dtype=np.uintp)
            ne = 0
        else:
            ne = e.size
        out = np.zeros(max(1, max_new_tokens), dtype=np.uintp)
        n = C.c_size_t(0)
        if lib().or_generate(self._h, p, p.size, max_new_tokens, float(temperature),
                             float(repetition_penalty), e, ne, int(seed), out, C.byref(n)) != 0:
            raise ValueError(lib().or_last_error(self._h).decode())
        return [int(t) for t in out[: n.value]]
