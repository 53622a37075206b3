"""Independent numpy/struct restatement of the `.gaje.flat` v2 packing of
scripts/export_gaje_flat.py:184-483 (metadata dict, directory list, 64-byte
aligned blobs, 4 KiB aligned weights, "<4sIIIQQQQIIIIIIII" header), used to
check the product writer byte for byte.  Quantisation goes through the CPU
oracle's restatement of quantize_q4_0_native / quantize_q8_0_native.
"""
from __future__ import annotations

import json
import struct

import numpy as np

import oracle


def write_flat(path, *, name, arch_family, n_embd, n_head, n_head_kv, n_blocks, vocab_size, eps,
               rope_base, qk_permute, tensors, config_extra=None):
    """tensors: list of ("linear", name, bit_depth, W[out][in], bias|None) or
    ("norm", name, v) in file order.  config_extra updates metadata["config"]."""
    metadata_dict = {
        "config": {
            "name": name,
            "version": "0.9.8",
            "tokenizer_id": "",
            "rope_base": float(np.float32(rope_base)),
            "ffn_act": "swiglu" if arch_family != 5 else "geglu",
            "use_genomic_norm": False,
        },
        "n_embd": n_embd,
        "n_head": n_head,
        "n_head_kv": n_head_kv,
        "n_blocks": n_blocks,
        "vocab_size": vocab_size,
        "eps": float(np.float32(eps)),
        "tokenizer": "",
    }
    if config_extra:
        metadata_dict["config"].update(config_extra)
    metadata_json_bytes = json.dumps(metadata_dict).encode("utf-8")
    tensor_directory = []
    blob_bytes = bytearray()

    def add_blob_data(raw):
        offset = len(blob_bytes)
        blob_bytes.extend(raw)
        padding = (64 - (len(blob_bytes) % 64)) % 64
        blob_bytes.extend(b"\x00" * padding)
        return offset, len(raw)

    for t in tensors:
        if t[0] == "norm":
            _, nm, v = t
            off, ln = add_blob_data(np.asarray(v, np.float32).tobytes())
            tensor_directory.append({"name": nm, "bit_depth": 32, "out_features": n_embd,
                                     "in_features": 1, "dna_off": off, "dna_len": ln, "c_off": 0,
                                     "c_len": 0, "anc_off": 0, "anc_len": 0, "bias_off": 0,
                                     "bias_len": 0})
            continue
        if t[0] == "lut4":  # Genomic4Bit: nibbles + a centroid table of 16, nb*16 or out*nb*16 floats
            _, nm, out_f, in_f, nibbles, cents, bias = t
            dna_off, dna_len = add_blob_data(np.asarray(nibbles, np.uint8).tobytes())
            c_off, c_len = add_blob_data(np.asarray(cents, np.float32).tobytes())
            anc_off, anc_len = add_blob_data(b"")
            bias_off, bias_len = 0, 0
            if bias is not None and len(bias) > 0:
                bias_off, bias_len = add_blob_data(np.asarray(bias, np.float32).tobytes())
            tensor_directory.append({"name": nm, "bit_depth": 4, "out_features": int(out_f),
                                     "in_features": int(in_f), "dna_off": int(dna_off), "dna_len": int(dna_len),
                                     "c_off": int(c_off), "c_len": int(c_len), "anc_off": int(anc_off),
                                     "anc_len": int(anc_len), "bias_off": int(bias_off),
                                     "bias_len": int(bias_len)})
            continue
        _, nm, bits, W, bias = t
        W = np.ascontiguousarray(W, np.float32)
        if bits == 4:
            dna = oracle.quantize_q4_0(W).tobytes()
        elif bits == 8:
            dna = oracle.quantize_q8_0(W).tobytes()
        else:
            dna = W.tobytes()
        dna_off, dna_len = add_blob_data(dna)
        c_off, c_len = add_blob_data(b"")
        anc_off, anc_len = add_blob_data(b"")
        bias_off, bias_len = 0, 0
        if bias is not None and len(bias) > 0:
            bias_off, bias_len = add_blob_data(np.asarray(bias, np.float32).tobytes())
        tensor_directory.append({"name": nm, "bit_depth": int(bits), "out_features": int(W.shape[0]),
                                 "in_features": int(W.shape[1]), "dna_off": int(dna_off),
                                 "dna_len": int(dna_len), "c_off": int(c_off), "c_len": int(c_len),
                                 "anc_off": int(anc_off), "anc_len": int(anc_len),
                                 "bias_off": int(bias_off), "bias_len": int(bias_len)})
    dir_json_bytes = json.dumps(tensor_directory).encode("utf-8")
    meta_len, dir_len = len(metadata_json_bytes), len(dir_json_bytes)
    weights_offset = 4096 + meta_len + dir_len
    if weights_offset % 4096 != 0:
        weights_offset = ((weights_offset // 4096) + 1) * 4096
    header_bin = bytearray(4096)
    struct.pack_into("<4sIIIQQQQIIIIIIII", header_bin, 0, b"GAJE", 0x000908, 0x0003,
                     len(tensor_directory), meta_len, dir_len, weights_offset, len(blob_bytes), 32, 1,
                     arch_family, n_embd, n_head, n_head_kv, n_blocks, 1 if qk_permute else 0)
    with open(path, "wb") as f:
        f.write(header_bin)
        f.write(metadata_json_bytes)
        f.write(dir_json_bytes)
        pad = weights_offset - (4096 + meta_len + dir_len)
        if pad > 0:
            f.write(b"\x00" * pad)
        f.write(blob_bytes)
    return path


def write_synthetic(path, *, seed, arch_family, n_embd, n_head, n_head_kv, n_blocks, ffn_dim, vocab_size, eps,
                    rope_base, qkv_bias, embd_bit_depth=32, std=0.02):
    """The benchmark / test model files without the product: the oracle's
    restatement of the synthetic N(0, std) generator, the oracle's quantisers
    and write_flat, in the synthetic writer's tensor order (tied token_embd /
    lm_head written twice, unit norms).  Byte-identical to the product's
    gaje_flat_write_synthetic (tests/test_format.py)."""
    d, hd = n_embd, n_embd // n_head
    qd, kvd, ff, V = n_head * hd, n_head_kv * hd, ffn_dim, vocab_size

    def normal(rows, cols, name):
        return oracle.synthetic_normal(rows * cols, seed, name, std).reshape(rows, cols)

    ones = np.ones(d, np.float32)
    emb = normal(V, d, "token_embd")
    tensors = [("linear", "token_embd", embd_bit_depth, emb, None), ("norm", "output_norm", ones),
               ("linear", "lm_head", embd_bit_depth, emb, None)]
    for i in range(n_blocks):
        p = f"blk.{i}."
        bias = oracle.synthetic_normal(qd + 2 * kvd, seed, p + "attn_qkv.bias", std) if qkv_bias else None
        tensors += [("norm", p + "attn_norm", ones), ("norm", p + "ffn_norm", ones),
                    ("linear", p + "attn_qkv", 4, normal(qd + 2 * kvd, d, p + "attn_qkv"), bias),
                    ("linear", p + "attn_output", 4, normal(d, qd, p + "attn_output"), None),
                    ("linear", p + "ffn_gate_up", 4, normal(2 * ff, d, p + "ffn_gate_up"), None),
                    ("linear", p + "ffn_down", 4, normal(d, ff, p + "ffn_down"), None)]
    return write_flat(path, name=f"synthetic-family{arch_family}", arch_family=arch_family, n_embd=n_embd,
                      n_head=n_head, n_head_kv=n_head_kv, n_blocks=n_blocks, vocab_size=vocab_size, eps=eps,
                      rope_base=rope_base, qk_permute=1 if arch_family in (1, 2) else 0, tensors=tensors)


def write_synthetic_lut4(path, *, seed, arch_family, n_embd, n_head, n_head_kv, n_blocks, ffn_dim, vocab_size, eps,
                         rope_base, qkv_bias, std=0.02, lut_tensors=("attn_qkv", "attn_output", "ffn_gate_up",
                                                                      "ffn_down"), centroid_layout="full"):
    """A synthetic model whose listed body matrices are Genomic4Bit tables
    (genomize_4bit_core of the same N(0, std) weights as write_synthetic) and
    the rest Q4_0.  centroid_layout: "full" (out*nb*16 floats, the quantiser's
    output), "column" (nb*16: the first row's tables shared by every row) or
    "shared" (16: block 0's table for the whole matrix), the three layouts
    GenomicLinear::new expands (src/nn/linear/init.rs:109-124); the nibbles are
    re-chosen against the shared tables."""
    d, hd = n_embd, n_embd // n_head
    qd, kvd, ff, V = n_head * hd, n_head_kv * hd, ffn_dim, vocab_size

    def normal(rows, cols, name):
        return oracle.synthetic_normal(rows * cols, seed, name, std).reshape(rows, cols)

    def lut(name, W, bias):
        out_f, in_f = W.shape
        nib, cen = oracle.genomize_4bit(W)
        nb = in_f // 32
        if centroid_layout != "full":
            cen3 = cen.reshape(out_f, nb, 16)
            table = cen3[0] if centroid_layout == "column" else cen3[0, 0]  # [nb, 16] or [16]
            full = np.broadcast_to(table, (out_f, nb, 16))
            wb = W.reshape(out_f, nb, 32)
            idx = np.argmin(np.abs(wb[..., None] - full[:, :, None, :]), axis=-1).astype(np.uint8)
            nib = ((idx[..., 0::2] << 4) | idx[..., 1::2]).reshape(-1)
            cen = np.ascontiguousarray(table, np.float32).reshape(-1)
        return ("lut4", name, out_f, in_f, nib, cen, bias)

    def mat(name, W, bias=None):
        short = name.split(".")[-1]
        return lut(name, W, bias) if short in lut_tensors else ("linear", name, 4, W, bias)

    ones = np.ones(d, np.float32)
    emb = normal(V, d, "token_embd")
    tensors = [("linear", "token_embd", 32, emb, None), ("norm", "output_norm", ones),
               ("linear", "lm_head", 32, emb, None)]
    for i in range(n_blocks):
        p = f"blk.{i}."
        bias = oracle.synthetic_normal(qd + 2 * kvd, seed, p + "attn_qkv.bias", std) if qkv_bias else None
        tensors += [("norm", p + "attn_norm", ones), ("norm", p + "ffn_norm", ones),
                    mat(p + "attn_qkv", normal(qd + 2 * kvd, d, p + "attn_qkv"), bias),
                    mat(p + "attn_output", normal(d, qd, p + "attn_output")),
                    mat(p + "ffn_gate_up", normal(2 * ff, d, p + "ffn_gate_up")),
                    mat(p + "ffn_down", normal(d, ff, p + "ffn_down"))]
    return write_flat(path, name=f"synthetic-family{arch_family}", arch_family=arch_family, n_embd=n_embd,
                      n_head=n_head, n_head_kv=n_head_kv, n_blocks=n_blocks, vocab_size=vocab_size, eps=eps,
                      rope_base=rope_base, qk_permute=1 if arch_family in (1, 2) else 0, tensors=tensors)
