"""B200 decode engine for GAJE `.gaje.flat` v2 models.

The product is libgaje_cuda.so (include/gaje_cuda.h): hand-written sm_100a
kernels plus a C++ host engine.  This package is its Python face, mirroring the
reference's PyO3 API (load_genomic_auto, RustGenomicLLM.forward /
generate_native_py / set_k_wta_ratio / clear_cache_py, quantize_q4_0_native).
"""
from .runtime import (  # noqa: F401
    FlatWriter,
    GajeError,
    GajeIOError,
    GajeValueError,
    GenomicLLM,
    Q4Matrix,
    argmax_key,
    argmax_key_index,
    attention_decode,
    decode_header,
    f32_gemv_argmax,
    inspect_flat,
    kwta,
    last_error,
    lib,
    load_genomic_auto,
    load_genomic_sharded,
    nccl_unique_id,
    quantize_q4_0_device,
    quantize_q4_0_native,
    quantize_q8_0_device,
    quantize_q8_0_native,
    rms_norm,
    sample_top_p,
    set_wait_limit,
    vocab_shard,
    write_synthetic,
)
from . import configs  # noqa: F401

RustGenomicLLM = GenomicLLM
