"""Python mirror of the reference's PyO3 surface for `.gaje.flat` decode, over the
C ABI of include/gaje_cuda.h (libgaje_cuda.so, built in-tree).

Reference interface mirrored (paths inside the reference project):
  load_genomic_auto(path)                 src/io/flat_reader.rs:240-251 (PyO3 src/io/ffi.rs:66-70)
  RustGenomicLLM.forward(token, clear)    src/nn/llm/python.rs:75-78
  RustGenomicLLM.generate_native_py(...)  src/nn/llm/python.rs:102-119
  RustGenomicLLM.set_k_wta_ratio(r)       src/nn/llm/python.rs:53-59
  RustGenomicLLM.clear_cache_py()         src/nn/llm/python.rs:97-100
  RustGenomicLLM.vocab_size / n_embd      src/nn/llm/python.rs:30-38
  quantize_q4_0_native / _q8_0_native     src/compute/quantize/python.rs:152-303
Errors map as PyO3 maps them: load failures (io::Error) raise IOError, step
failures (Result<_, String>) raise ValueError.

There is no CPU fallback: importing this module without the built library, or
calling the engine without a CUDA device, raises.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass
from typing import Iterable, Optional, Sequence

import numpy as np

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libgaje_cuda.so")

GAJE_OK = 0
STATUS_NAMES = {
    0: "GAJE_OK", 1: "GAJE_ERR_INVALID", 2: "GAJE_ERR_IO", 3: "GAJE_ERR_NOT_FOUND",
    4: "GAJE_ERR_SHAPE", 5: "GAJE_ERR_UNSUPPORTED", 6: "GAJE_ERR_CUDA", 7: "GAJE_ERR_NAN",
    8: "GAJE_ERR_CONTEXT", 9: "GAJE_ERR_TIMEOUT",
}


class GajeError(RuntimeError):
    """A non-zero gaje_status with its message."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status
        self.message = message


class GajeIOError(GajeError, IOError):
    pass


class GajeValueError(GajeError, ValueError):
    pass


class FlatHeader(C.Structure):
    _fields_ = [("version", C.c_uint32), ("flags", C.c_uint32), ("num_tensors", C.c_uint32),
                ("meta_len", C.c_uint64), ("dir_len", C.c_uint64), ("weights_offset", C.c_uint64),
                ("weights_len", C.c_uint64), ("group_size", C.c_uint32), ("quant_format", C.c_uint32),
                ("arch_family", C.c_uint32), ("arch_n_embd", C.c_uint32), ("arch_n_head", C.c_uint32),
                ("arch_n_head_kv", C.c_uint32), ("arch_n_blocks", C.c_uint32),
                ("arch_qk_permute", C.c_uint32)]


class FlatInfo(C.Structure):
    _fields_ = [("header", FlatHeader), ("n_embd", C.c_uint32), ("n_head", C.c_uint32),
                ("n_head_kv", C.c_uint32), ("n_blocks", C.c_uint32), ("head_dim", C.c_uint32),
                ("ffn_dim", C.c_uint32), ("vocab_size", C.c_uint32), ("eps", C.c_float),
                ("rope_base", C.c_float), ("rope_split", C.c_int), ("use_genomic_norm", C.c_int),
                ("fused_qkv", C.c_int), ("fused_gate_up", C.c_int), ("embd_bit_depth", C.c_int),
                ("lm_head_bit_depth", C.c_int), ("body_bit_depth", C.c_int), ("n_entries", C.c_uint32)]


class FlatMeta(C.Structure):
    _fields_ = [("name", C.c_char_p), ("tokenizer_id", C.c_char_p), ("tokenizer", C.c_char_p),
                ("arch_family", C.c_uint32), ("qk_permute", C.c_uint32), ("n_embd", C.c_uint32),
                ("n_head", C.c_uint32), ("n_head_kv", C.c_uint32), ("n_blocks", C.c_uint32),
                ("vocab_size", C.c_uint32), ("eps", C.c_float), ("rope_base", C.c_double)]


class SynthSpec(C.Structure):
    _fields_ = [("arch_family", C.c_uint32), ("n_embd", C.c_uint32), ("n_head", C.c_uint32),
                ("n_head_kv", C.c_uint32), ("n_blocks", C.c_uint32), ("ffn_dim", C.c_uint32),
                ("vocab_size", C.c_uint32), ("eps", C.c_float), ("rope_base", C.c_double),
                ("qkv_bias", C.c_int), ("embd_bit_depth", C.c_int), ("std", C.c_float),
                ("seed", C.c_uint64)]


class LoadOpts(C.Structure):
    _fields_ = [("device", C.c_int), ("max_ctx", C.c_uint32), ("seed", C.c_uint64),
                ("use_graph", C.c_int), ("use_megakernel", C.c_int), ("max_streams", C.c_uint32),
                ("max_prefill", C.c_uint32)]


class ModelInfo(C.Structure):
    _fields_ = [("vocab_size", C.c_uint32), ("n_embd", C.c_uint32), ("n_head", C.c_uint32),
                ("n_head_kv", C.c_uint32), ("n_blocks", C.c_uint32), ("head_dim", C.c_uint32),
                ("ffn_dim", C.c_uint32), ("max_ctx", C.c_uint32), ("cache_len", C.c_uint32),
                ("eps", C.c_float), ("rope_base", C.c_float), ("k_wta_ratio", C.c_float),
                ("device_bytes", C.c_size_t), ("grid", C.c_uint32), ("megakernel", C.c_uint32),
                ("nranks", C.c_uint32), ("rank", C.c_uint32), ("vocab_row0", C.c_uint32),
                ("vocab_rows", C.c_uint32)]

NCCL_ID_BYTES = 128


_lib = None


def lib() -> C.CDLL:
    """The loaded libgaje_cuda.so (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: build it with __graft_entry__.build() "
                          "(the engine has no CPU fallback)")
    L = C.CDLL(LIB_PATH)
    vp, sz, u32, u64, i32, f32 = C.c_void_p, C.c_size_t, C.c_uint32, C.c_uint64, C.c_int, C.c_float
    sig = {
        "gaje_cuda_last_error": ([], C.c_char_p),
        "gaje_flat_header_decode": ([C.c_char_p, sz, C.POINTER(FlatHeader)], i32),
        "gaje_flat_inspect": ([C.c_char_p, C.POINTER(FlatInfo)], i32),
        "gaje_quantize_q4_0": ([vp, sz, vp], i32),
        "gaje_quantize_q8_0": ([vp, sz, vp], i32),
        "gaje_flat_writer_open": ([C.c_char_p, C.POINTER(FlatMeta)], vp),
        "gaje_flat_writer_add_linear": ([vp, C.c_char_p, i32, sz, sz, vp, vp], i32),
        "gaje_flat_writer_add_norm": ([vp, C.c_char_p, vp, sz], i32),
        "gaje_flat_writer_close": ([vp], i32),
        "gaje_flat_write_synthetic": ([C.c_char_p, C.POINTER(SynthSpec)], i32),
        "gaje_load_opts_init": ([C.POINTER(LoadOpts)], None),
        "gaje_cuda_load": ([C.c_char_p, C.POINTER(LoadOpts)], vp),
        "gaje_cuda_free": ([vp], None),
        "gaje_cuda_model_info": ([vp, C.POINTER(ModelInfo)], i32),
        "gaje_cuda_forward": ([vp, u32, i32, vp, C.POINTER(u32)], i32),
        "gaje_cuda_generate": ([vp, vp, sz, sz, f32, f32, vp, sz, vp, C.POINTER(sz)], i32),
        "gaje_cuda_clear_cache": ([vp], i32),
        "gaje_cuda_set_k_wta_ratio": ([vp, f32], i32),
        "gaje_cuda_set_seed": ([vp, u64], i32),
        "gaje_cuda_decode_greedy": ([vp, u32, sz, vp], i32),
        "gaje_cuda_stream": ([vp], vp),
        "gaje_cuda_profile_steps": ([vp, u32, sz, vp, vp], i32),
        "gaje_cuda_profile_phases": ([vp, u32, sz, vp, vp, vp], i32),
        "gaje_cuda_trace_steps": ([vp, u32, sz, vp, sz, vp], i32),
        "gaje_cuda_trace_fused": ([vp, u32, sz, vp, sz, vp], i32),
        "gaje_cuda_set_wait_limit": ([i32, u64], i32),
        "gaje_cuda_debug_withhold_flag": ([vp, i32], i32),
        "gaje_cuda_profile_batch": ([vp, vp, vp, sz, vp, vp], i32),
        "gaje_cuda_attention_decode_static": ([vp, vp, vp, sz, sz, sz, sz, sz, vp, vp], i32),
        "gaje_cuda_forward_batch": ([vp, vp, vp, sz, vp, vp], i32),
        "gaje_cuda_prefill": ([vp, u32, vp, sz, vp, vp], i32),
        "gaje_cuda_clear_stream": ([vp, u32], i32),
        "gaje_cuda_stream_len": ([vp, u32, vp], i32),
        "gaje_cuda_q4_0_upload": ([vp, sz, sz, vp, i32], vp),
        "gaje_cuda_q4_0_release": ([vp], None),
        "gaje_cuda_lut4_upload": ([vp, vp, sz, sz, sz, vp, i32], vp),
        "gaje_cuda_q4_0_gemv": ([vp, vp, vp, sz, vp], i32),
        "gaje_cuda_q4_0_dequant": ([vp, vp, vp], i32),
        "gaje_cuda_f32_gemv_argmax": ([vp, vp, sz, sz, vp, vp, vp], i32),
        "gaje_cuda_rms_norm": ([vp, vp, f32, sz, vp, vp], i32),
        "gaje_cuda_attention_decode": ([vp, vp, vp, sz, sz, sz, sz, sz, vp, vp], i32),
        "gaje_cuda_kwta": ([vp, sz, sz, vp], i32),
        "gaje_cuda_sample_top_p": ([vp, sz, f32, f32, f32, vp, vp, vp], i32),
        "gaje_cuda_quantize_q4_0": ([vp, sz, vp, vp], i32),
        "gaje_cuda_quantize_q8_0": ([vp, sz, vp, vp], i32),
        "gaje_cuda_nccl_unique_id": ([vp], i32),
        "gaje_cuda_load_sharded": ([C.c_char_p, C.POINTER(LoadOpts), i32, i32, vp], vp),
        "gaje_vocab_shard": ([u32, i32, i32, C.POINTER(u32), C.POINTER(u32)], i32),
        "gaje_cuda_batch_timings": ([vp, vp, C.POINTER(u32), i32], i32),
        "gaje_argmax_key": ([f32, u32], u64),
        "gaje_argmax_key_index": ([u64], u32),
    }
    for name, (args, res) in sig.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = res
    _lib = L
    return L


def last_error() -> str:
    return lib().gaje_cuda_last_error().decode("utf-8", "replace")


def _check(status: int, exc=GajeValueError) -> None:
    if status != GAJE_OK:
        raise exc(status, last_error())


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


# ------------------------------------------------------------------ format
QUANT_FORMATS = {0: "LegacyCentroids", 1: "Q4_0", 2: "Q8_0"}


def decode_header(buf: bytes) -> dict:
    """FlatHeaderV2::from_bytes on a byte buffer, plus quantization_type() and
    effective_group_size() (src/io/header/flat.rs:47-79)."""
    h = FlatHeader()
    _check(lib().gaje_flat_header_decode(buf, len(buf), C.byref(h)), GajeIOError)
    out = {f: getattr(h, f) for f, _ in FlatHeader._fields_}
    out["quantization_type"] = QUANT_FORMATS.get(h.quant_format, "Unknown")
    out["effective_group_size"] = 16 if h.group_size == 0 else h.group_size
    return out


def inspect_flat(path: str) -> dict:
    """Parse-only open of a `.gaje.flat` file (header, config, directory)."""
    info = FlatInfo()
    _check(lib().gaje_flat_inspect(path.encode(), C.byref(info)), GajeIOError)
    out = {f: getattr(info, f) for f, _ in FlatInfo._fields_ if f != "header"}
    out["header"] = {f: getattr(info.header, f) for f, _ in FlatHeader._fields_}
    out["rope_style"] = "split" if info.rope_split else "interleaved"
    return out


def quantize_q4_0_native(data_u8: bytes) -> bytes:
    """quantize_q4_0_native: f32 bytes -> packed 20-byte Q4_0 Variant B blocks."""
    w = np.frombuffer(data_u8, dtype=np.float32)
    if w.size % 32:
        raise TypeError("Weights length must be divisible by 32")
    out = np.empty(w.size // 32 * 20, dtype=np.uint8)
    w = np.ascontiguousarray(w)
    _check(lib().gaje_quantize_q4_0(_ptr(w), w.size, _ptr(out)))
    return out.tobytes()


def quantize_q8_0_native(data_u8: bytes) -> bytes:
    w = np.frombuffer(data_u8, dtype=np.float32)
    if w.size % 32:
        raise TypeError("Weights length must be divisible by 32")
    out = np.empty(w.size // 32 * 34, dtype=np.uint8)
    w = np.ascontiguousarray(w)
    _check(lib().gaje_quantize_q8_0(_ptr(w), w.size, _ptr(out)))
    return out.tobytes()


class FlatWriter:
    """`.gaje.flat` v2 writer with the exporter's layout (scripts/export_gaje_flat.py)."""

    def __init__(self, path: str, *, name: str, arch_family: int, n_embd: int, n_head: int,
                 n_head_kv: int, n_blocks: int, vocab_size: int, eps: float, rope_base: float,
                 qk_permute: int = 0, tokenizer_id: str = "", tokenizer: str = ""):
        self._keep = [name.encode(), tokenizer_id.encode(), tokenizer.encode()]
        meta = FlatMeta(self._keep[0], self._keep[1], self._keep[2], arch_family, qk_permute,
                        n_embd, n_head, n_head_kv, n_blocks, vocab_size, eps, rope_base)
        self._w = lib().gaje_flat_writer_open(path.encode(), C.byref(meta))
        if not self._w:
            raise GajeIOError(2, last_error())

    def add_linear(self, name: str, bit_depth: int, weights: np.ndarray,
                   bias: Optional[np.ndarray] = None) -> None:
        w = np.ascontiguousarray(weights, dtype=np.float32)
        b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
        _check(lib().gaje_flat_writer_add_linear(self._w, name.encode(), bit_depth, w.shape[0],
                                                 w.shape[1], _ptr(w), None if b is None else _ptr(b)))

    def add_norm(self, name: str, v: np.ndarray) -> None:
        v = np.ascontiguousarray(v, dtype=np.float32)
        _check(lib().gaje_flat_writer_add_norm(self._w, name.encode(), _ptr(v), v.size))

    def close(self) -> None:
        if self._w:
            w, self._w = self._w, None
            _check(lib().gaje_flat_writer_close(w), GajeIOError)


def write_synthetic(path: str, *, arch_family: int, n_embd: int, n_head: int, n_head_kv: int,
                    n_blocks: int, ffn_dim: int, vocab_size: int, eps: float, rope_base: float,
                    qkv_bias: bool = False, embd_bit_depth: int = 32, std: float = 0.02,
                    seed: int = 0) -> str:
    """Seeded random-init model in `.gaje.flat` v2 (N(0, std) weights, norms 1.0,
    tied embedding/lm_head written twice, Q4_0 body)."""
    spec = SynthSpec(arch_family, n_embd, n_head, n_head_kv, n_blocks, ffn_dim, vocab_size, eps,
                     rope_base, 1 if qkv_bias else 0, embd_bit_depth, std, seed)
    _check(lib().gaje_flat_write_synthetic(path.encode(), C.byref(spec)), GajeIOError)
    return path


# ------------------------------------------------------------------- model
class GenomicLLM:
    """A `.gaje.flat` model resident on one GPU (the reference's RustGenomicLLM)."""

    def __init__(self, path: str, device: int = 0, max_ctx: int = 4096, seed: int = 0,
                 use_graph: bool = True, use_megakernel: bool = True, max_streams: int = 0,
                 max_prefill: int = 0, shard: Optional[tuple] = None):
        opts = LoadOpts()
        lib().gaje_load_opts_init(C.byref(opts))
        opts.device, opts.max_ctx, opts.seed, opts.use_graph = device, max_ctx, seed, int(use_graph)
        opts.use_megakernel = int(use_megakernel)
        opts.max_streams = int(max_streams)
        opts.max_prefill = int(max_prefill)
        if shard is None:
            self._m = lib().gaje_cuda_load(path.encode(), C.byref(opts))
        else:  # (nranks, rank, nccl_id): one rank of a vocab-sharded group (collective)
            nranks, rank, nid = shard
            idb = C.create_string_buffer(bytes(nid), NCCL_ID_BYTES)
            self._m = lib().gaje_cuda_load_sharded(path.encode(), C.byref(opts), int(nranks), int(rank), idb)
        if not self._m:
            raise GajeIOError(2, last_error())
        info = self.info()
        self.vocab_size = int(info.vocab_size)
        self.n_embd = int(info.n_embd)
        self.n_head = int(info.n_head)
        self.n_head_kv = int(info.n_head_kv)
        self.n_blocks = int(info.n_blocks)
        self.head_dim = int(info.head_dim)
        self.ffn_dim = int(info.ffn_dim)
        self.max_ctx = int(info.max_ctx)
        self._logits = np.empty(self.vocab_size, dtype=np.float32)

    def close(self) -> None:
        if getattr(self, "_m", None):
            lib().gaje_cuda_free(self._m)
            self._m = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def info(self) -> ModelInfo:
        mi = ModelInfo()
        _check(lib().gaje_cuda_model_info(self._m, C.byref(mi)))
        return mi

    @property
    def cache_len(self) -> int:
        return int(self.info().cache_len)

    @property
    def k_wta_ratio(self) -> float:
        return float(self.info().k_wta_ratio)

    @property
    def stream(self) -> int:
        """The model's cudaStream_t as an integer handle."""
        return int(lib().gaje_cuda_stream(self._m) or 0)

    def set_k_wta_ratio(self, ratio: float) -> None:
        _check(lib().gaje_cuda_set_k_wta_ratio(self._m, float(ratio)))

    def set_seed(self, seed: int) -> None:
        _check(lib().gaje_cuda_set_seed(self._m, int(seed)))

    def clear_cache_py(self) -> None:
        _check(lib().gaje_cuda_clear_cache(self._m))

    clear_cache = clear_cache_py

    def forward(self, token_id: int, clear_cache: bool = False) -> np.ndarray:
        """One decode step; returns the logits (a fresh float32 array)."""
        out = np.empty(self.vocab_size, dtype=np.float32)
        am = C.c_uint32(0)
        _check(lib().gaje_cuda_forward(self._m, int(token_id), 1 if clear_cache else 0, _ptr(out),
                                       C.byref(am)))
        return out

    def forward_argmax(self, token_id: int, clear_cache: bool = False) -> int:
        """One decode step returning only the greedy token (no logits copy)."""
        am = C.c_uint32(0)
        _check(lib().gaje_cuda_forward(self._m, int(token_id), 1 if clear_cache else 0, None,
                                       C.byref(am)))
        return int(am.value)

    def decode_greedy(self, first_token: int, n_steps: int) -> list:
        """n_steps greedy steps kept on the device; returns each step's argmax."""
        out = np.zeros(max(1, n_steps), dtype=np.uint32)
        _check(lib().gaje_cuda_decode_greedy(self._m, int(first_token), int(n_steps), _ptr(out)))
        return [int(t) for t in out[:n_steps]]

    KERNEL_CLASSES = ("qkv", "attn", "oproj", "gateup", "down", "lmhead", "kwta")

    def profile_steps(self, first_token: int, n_steps: int) -> dict:
        """Greedy steps with every kernel bracketed by CUDA events: mean ms per
        step and launches per step for each kernel class."""
        ms = np.zeros(len(self.KERNEL_CLASSES), dtype=np.float32)
        n = np.zeros(len(self.KERNEL_CLASSES), dtype=np.uint32)
        _check(lib().gaje_cuda_profile_steps(self._m, int(first_token), int(n_steps), _ptr(ms), _ptr(n)))
        return {k: (float(ms[i]), int(n[i])) for i, k in enumerate(self.KERNEL_CLASSES)}

    PHASES = ("qkv", "attn", "oproj", "gateup", "down", "lmhead")

    DETAIL = ("to_entry", "to_flags", "to_staged", "to_rows", "to_published")

    def profile_phases(self, first_token: int, n_steps: int, detail: bool = False) -> dict:
        """Greedy steps in the persistent kernel with a timer stamp at every grid
        barrier: mean microseconds per step in each phase, plus "step"; with
        detail, the in-phase intervals of CTA 0 under "detail"."""
        us = np.zeros(len(self.PHASES), dtype=np.float32)
        det = np.zeros(len(self.PHASES) * 5, dtype=np.float32)
        step = C.c_float(0)
        _check(lib().gaje_cuda_profile_phases(self._m, int(first_token), int(n_steps), _ptr(us), C.byref(step),
                                              _ptr(det) if detail else None))
        out = {k: float(us[i]) for i, k in enumerate(self.PHASES)}
        out["step"] = float(step.value)
        if detail:
            out["detail"] = {self.PHASES[p]: {self.DETAIL[j]: round(float(det[p * 5 + j]), 3) for j in range(5)}
                             for p in range(len(self.PHASES))}
        return out

    def forward_batch(self, stream_ids: Sequence[int], tokens: Sequence[int], logits: bool = False):
        """One decode step for each listed stream (its own KV cache and
        position): the greedy argmax per stream, and the logits [B, vocab]
        when asked for."""
        sids = np.ascontiguousarray(list(stream_ids), dtype=np.uint32)
        toks = np.ascontiguousarray(list(tokens), dtype=np.uint32)
        if sids.size != toks.size:
            raise ValueError("stream_ids and tokens differ in length")
        am = np.zeros(sids.size, dtype=np.uint32)
        lg = np.empty((sids.size, self.vocab_size), dtype=np.float32) if logits else None
        _check(lib().gaje_cuda_forward_batch(self._m, _ptr(sids), _ptr(toks), sids.size, _ptr(am),
                                             _ptr(lg) if logits else None))
        return (am, lg) if logits else am

    def prefill(self, stream_id: int, tokens: Sequence[int], logits: bool = False):
        """The prompt of one batched stream in one pass (whole-prompt GEMMs and
        a causal attention pass), as len(tokens) consecutive steps would leave
        its cache: the last token's greedy argmax, and its logits when asked."""
        toks = np.ascontiguousarray(list(tokens), dtype=np.uint32)
        am = np.zeros(1, dtype=np.uint32)
        lg = np.empty(self.vocab_size, dtype=np.float32) if logits else None
        _check(lib().gaje_cuda_prefill(self._m, int(stream_id), _ptr(toks), toks.size, _ptr(am),
                                       _ptr(lg) if logits else None))
        return (int(am[0]), lg) if logits else int(am[0])

    def profile_batch(self, stream_ids: Sequence[int], tokens: Sequence[int]) -> dict:
        """One batched step launched kernel by kernel: milliseconds per kernel
        class (all blocks together)."""
        sids = np.ascontiguousarray(list(stream_ids), dtype=np.uint32)
        toks = np.ascontiguousarray(list(tokens), dtype=np.uint32)
        ms = np.zeros(7, dtype=np.float32)
        n = np.zeros(7, dtype=np.uint32)
        _check(lib().gaje_cuda_profile_batch(self._m, _ptr(sids), _ptr(toks), sids.size, _ptr(ms), _ptr(n)))
        names = ["qkv", "attn", "oproj", "gateup", "down", "lmhead", "kwta"]
        return {names[k]: float(ms[k]) for k in range(6)}

    BATCH_SEGMENTS = ("body", "gather_rows", "lm_head", "gather_keys")

    def batch_timings(self, reset: bool = False) -> dict:
        """Device time of the batched steps per segment (ms, summed over the
        forward_batch calls since the last reset) and the number of calls; on
        one GPU "body" is the whole step."""
        ms = np.zeros(4, dtype=np.float32)
        n = C.c_uint32(0)
        _check(lib().gaje_cuda_batch_timings(self._m, _ptr(ms), C.byref(n), 1 if reset else 0))
        out = {k: float(ms[i]) for i, k in enumerate(self.BATCH_SEGMENTS)}
        out["steps"] = int(n.value)
        return out

    def clear_stream(self, stream_id: int) -> None:
        _check(lib().gaje_cuda_clear_stream(self._m, int(stream_id)))

    def stream_len(self, stream_id: int) -> int:
        n = C.c_uint32(0)
        _check(lib().gaje_cuda_stream_len(self._m, int(stream_id), C.byref(n)))
        return int(n.value)

    def trace_steps(self, first_token: int, n_steps: int) -> np.ndarray:
        """Every CTA's trace stamps (ns) of n_steps greedy steps in one launch:
        shape [grid, n_steps, 5*n_blocks+1, 6] (points: entry, input flags
        seen, staged, rows done, published, first weight slot ready; 0 where a
        CTA had no work in that phase)."""
        inf = self.info()
        per = 5 * inf.n_blocks + 1
        out = np.zeros((inf.grid, int(n_steps), per, 6), dtype=np.uint64)
        n = C.c_size_t(0)
        _check(lib().gaje_cuda_trace_steps(self._m, int(first_token), int(n_steps), _ptr(out), C.c_size_t(out.size),
                                           C.byref(n)))
        return out

    def debug_withhold_flag(self, cta: int) -> None:
        """Failure-path diagnostic (gaje_cuda_debug_withhold_flag): attention CTA
        `cta` raises no flag in the next launch of the two-exchange kernel, so
        that call returns GAJE_ERR_TIMEOUT once the bounded waits run out."""
        _check(lib().gaje_cuda_debug_withhold_flag(self._m, int(cta)))

    def trace_fused(self, first_token: int, n_steps: int) -> np.ndarray:
        """The two-exchange kernel's trace stamps of n_steps greedy steps in one
        launch, in nanoseconds of the global timer from the first CTA's start
        (float64, 0 where a CTA had no such point): shape [grid, n_steps, n_blocks+1, 24] (see
        gaje_cuda_trace_fused for the points).  The kernel stamps SM cycles;
        each CTA's (globaltimer, cycle) anchors at its start and end map them
        onto the global clock.  The CTAs' SM ids are left in self.trace_smid."""
        inf = self.info()
        L = inf.n_blocks
        raw = np.zeros((inf.grid, int(n_steps), L + 1, 24), dtype=np.uint64)
        n = C.c_size_t(0)
        _check(lib().gaje_cuda_trace_fused(self._m, int(first_token), int(n_steps), _ptr(raw), C.c_size_t(raw.size),
                                           C.byref(n)))
        self.trace_smid = raw[:, 0, 0, 22].astype(np.int64)  # each CTA's SM
        raw[:, 0, 0, 22] = 0
        # differences in integers first: float64 cannot resolve single
        # nanoseconds (or cycles) at the timers' absolute magnitudes
        g0i, c0i = raw[:, 0, L, 22].copy(), raw[:, 0, L, 23].copy()
        g1i, c1i = raw[:, -1, L, 20].copy(), raw[:, -1, L, 21].copy()
        base = int(g0i.min())
        g0 = (g0i - np.uint64(base)).astype(np.float64)
        rate = (g1i - g0i).astype(np.float64) / np.maximum((c1i - c0i).astype(np.float64), 1.0)  # ns per cycle
        raw[:, 0, L, 22:24] = 0
        raw[:, -1, L, 20:22] = 0
        shape = (-1,) + (1,) * 3
        rel = (raw.astype(np.int64) - c0i.astype(np.int64).reshape(shape)).astype(np.float64)
        ns = 1.0 + g0.reshape(shape) + rel * rate.reshape(shape)  # > 0 for every stamp
        return np.where(raw > 0, ns, 0.0)

    def generate_native_py(self, prompt_tokens: Sequence[int], max_new_tokens: int = 30,
                           temperature: float = 0.7, repetition_penalty: float = 1.0,
                           eos_token_ids: Iterable[int] = (2, 151643, 151645)) -> list:
        p = np.ascontiguousarray(list(prompt_tokens), dtype=np.uint32)
        e = np.ascontiguousarray(list(eos_token_ids), dtype=np.uint32)
        out = np.zeros(max(1, max_new_tokens), dtype=np.uint32)
        n = C.c_size_t(0)
        _check(lib().gaje_cuda_generate(self._m, _ptr(p) if p.size else None, p.size, max_new_tokens,
                                        float(temperature), float(repetition_penalty),
                                        _ptr(e) if e.size else None, e.size, _ptr(out), C.byref(n)))
        return [int(t) for t in out[: n.value]]

    generate = generate_native_py


def set_wait_limit(device: int, ns: int) -> None:
    """The limit of every bounded device-side wait of the library's kernels on
    `device` (gaje_cuda_set_wait_limit); 0 restores the default of 2 s."""
    _check(lib().gaje_cuda_set_wait_limit(int(device), int(ns)))


def nccl_unique_id() -> bytes:
    """A fresh NCCL unique id (GAJE_NCCL_ID_BYTES bytes) for load_genomic_sharded."""
    buf = C.create_string_buffer(NCCL_ID_BYTES)
    _check(lib().gaje_cuda_nccl_unique_id(buf))
    return buf.raw


def vocab_shard(vocab_size: int, nranks: int, rank: int) -> tuple:
    """(row0, rows): the lm_head rows rank `rank` of `nranks` holds."""
    r0, n = C.c_uint32(0), C.c_uint32(0)
    _check(lib().gaje_vocab_shard(int(vocab_size), int(nranks), int(rank), C.byref(r0), C.byref(n)))
    return int(r0.value), int(n.value)


def argmax_key(value: float, index: int) -> int:
    """The orderable (value, first index) key the sharded ranks exchange."""
    return int(lib().gaje_argmax_key(float(value), int(index)))


def argmax_key_index(key: int) -> int:
    return int(lib().gaje_argmax_key_index(int(key)))


def load_genomic_sharded(path: str, nranks: int, rank: int, nccl_id: bytes, **kw) -> GenomicLLM:
    """One rank of a request-parallel group with the f32 lm_head split by
    vocabulary over `nranks` GPUs (every rank calls it together with the same
    nccl_id).  Batched calls only (forward_batch / prefill, collective: the
    same sequence with the same batch size on every rank)."""
    if kw.get("max_streams", 0) <= 0:
        raise ValueError("a vocab-sharded model serves batched streams: pass max_streams > 0")
    return GenomicLLM(path, shard=(nranks, rank, nccl_id), **kw)


def load_genomic_auto(path: str, **kw) -> GenomicLLM:
    """load_genomic_auto for `.gaje.flat` files (magic "GAJE")."""
    with open(path, "rb") as f:
        magic = f.read(4)
    if magic != b"GAJE":
        raise GajeIOError(5, "not a .gaje.flat file; the redb .gaje container is not supported")
    return GenomicLLM(path, **kw)


# ---------------------------------------------------------------- op level
class Q4Matrix:
    """A Q4_0 matrix uploaded to the device (op-level entry points)."""

    def __init__(self, blocks: np.ndarray, N: int, K: int, bias: Optional[np.ndarray] = None,
                 device: int = 0):
        b = np.ascontiguousarray(blocks, dtype=np.uint8)
        if b.size != N * (K // 32) * 20:
            raise ValueError("blocks size does not match N x K")
        bias_a = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
        self.N, self.K = N, K
        self._h = lib().gaje_cuda_q4_0_upload(_ptr(b), N, K, None if bias_a is None else _ptr(bias_a),
                                               device)
        if not self._h:
            raise GajeValueError(1, last_error())

    @classmethod
    def from_lut4(cls, nibbles: np.ndarray, centroids: np.ndarray, N: int, K: int,
                  bias: Optional[np.ndarray] = None, device: int = 0) -> "Q4Matrix":
        """A Genomic4Bit matrix: nibbles [N*K/2] (high nibble first) and a
        centroid table of 16, K/32*16 or N*K/32*16 floats."""
        nib = np.ascontiguousarray(nibbles, dtype=np.uint8)
        cen = np.ascontiguousarray(centroids, dtype=np.float32)
        if nib.size != N * K // 2:
            raise ValueError("nibbles size does not match N x K")
        bias_a = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
        self = cls.__new__(cls)
        self.N, self.K = N, K
        self._h = lib().gaje_cuda_lut4_upload(_ptr(nib), _ptr(cen), cen.size, N, K,
                                              None if bias_a is None else _ptr(bias_a), device)
        if not self._h:
            raise GajeValueError(1, last_error())
        return self

    def __del__(self):
        if getattr(self, "_h", None):
            lib().gaje_cuda_q4_0_release(self._h)
            self._h = None

    def gemv(self, x_ptr: int, y_ptr: int, M: int = 1, stream: int = 0) -> None:
        _check(lib().gaje_cuda_q4_0_gemv(self._h, x_ptr, y_ptr, M, stream or None))

    def dequant(self, w_ptr: int, stream: int = 0) -> None:
        _check(lib().gaje_cuda_q4_0_dequant(self._h, w_ptr, stream or None))


def f32_gemv_argmax(W_ptr: int, x_ptr: int, N: int, K: int, logits_ptr: Optional[int],
                    argmax_ptr: int, stream: int = 0) -> None:
    _check(lib().gaje_cuda_f32_gemv_argmax(W_ptr, x_ptr, N, K, logits_ptr, argmax_ptr, stream or None))


def rms_norm(x_ptr: int, w_ptr: int, eps: float, n: int, out_ptr: int, stream: int = 0) -> None:
    _check(lib().gaje_cuda_rms_norm(x_ptr, w_ptr, eps, n, out_ptr, stream or None))


def attention_decode(q_ptr: int, k_ptr: int, v_ptr: int, ctx: int, cache_stride: int, n_head: int,
                     n_head_kv: int, head_dim: int, out_ptr: int, stream: int = 0) -> None:
    _check(lib().gaje_cuda_attention_decode(q_ptr, k_ptr, v_ptr, ctx, cache_stride, n_head, n_head_kv,
                                            head_dim, out_ptr, stream or None))


def kwta(scores_ptr: int, n: int, k: int, stream: int = 0) -> None:
    _check(lib().gaje_cuda_kwta(scores_ptr, n, k, stream or None))


def quantize_q4_0_device(w_ptr: int, n: int, out_ptr: int, stream: int = 0) -> None:
    """quantize_q4_0_native on the device: n f32 at w_ptr -> n/32 20-byte blocks at out_ptr."""
    _check(lib().gaje_cuda_quantize_q4_0(w_ptr, n, out_ptr, stream or None))


def quantize_q8_0_device(w_ptr: int, n: int, out_ptr: int, stream: int = 0) -> None:
    """The Q8_0 quantiser on the device: n f32 at w_ptr -> n/32 34-byte blocks at out_ptr."""
    _check(lib().gaje_cuda_quantize_q8_0(w_ptr, n, out_ptr, stream or None))


def sample_top_p(logits_ptr: int, n: int, temperature: float, top_p: float, r: float, token_ptr: int,
                 kept_ptr: Optional[int] = None, stream: int = 0) -> None:
    """sample_top_p (src/compute/sampling.rs:14-55) on the device with the
    uniform draw r in [0, 1) given: the token into token_ptr (device u32)."""
    _check(lib().gaje_cuda_sample_top_p(logits_ptr, n, float(temperature), float(top_p), float(r), token_ptr,
                                        kept_ptr, stream or None))
