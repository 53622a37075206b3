"""The reference's own known-answer tests for this path, restated against the CPU
oracle and the product's host code (no GPU).

  src/io/header/tests.rs:7-49    header v1 compatibility, v2 Q4_0, invalid magic
  src/io/header/tests.rs:51-89   Q4_0 block round trip, |err| <= 0.11
  src/io/header/tests.rs:120-165 Q8_0 round trip, |err| <= scale/2 + 1e-5
  src/nn/linear/tests.rs:8-100   Q4_0 GenomicLinear forward == sum of dequant, 1e-4
  tests/unit/test_rope_logic.py  split RoPE formula
"""
import struct

import numpy as np
import pytest


def _header(**fields):
    b = bytearray(4096)
    b[0:4] = fields.get("magic", b"GAJE")
    for off, key in ((4, "version"), (8, "flags"), (12, "num_tensors"), (48, "group_size"),
                     (52, "quant_format")):
        if key in fields:
            struct.pack_into("<I", b, off, fields[key])
    return bytes(b)


def test_header_v1_backward_compatibility(g):
    h = g.decode_header(_header(version=0x000907, flags=1, num_tensors=12))
    assert h["quantization_type"] == "LegacyCentroids"
    assert h["effective_group_size"] == 16
    assert h["num_tensors"] == 12
    assert h["version"] == 0x000907


def test_header_v2_q4_0(g):
    h = g.decode_header(_header(version=0x000908, group_size=32, quant_format=1))
    assert h["quantization_type"] == "Q4_0"
    assert h["effective_group_size"] == 32
    assert h["version"] == 0x000908


def test_invalid_magic_bytes(g):
    with pytest.raises(IOError) as e:
        g.decode_header(_header(magic=b"XGAJ"))
    assert "magic" in str(e.value)
    with pytest.raises(IOError):
        g.decode_header(b"GAJE" + bytes(100))  # shorter than 4096


def _dequant_numpy(blocks):
    """blocks.rs:18-31 in float64 numpy: q*scale + min from the f16 fields.
    Exact for Q4_0: q (4 bits) times an f16 scale and an f16 min fit in f64."""
    b = np.asarray(blocks, np.uint8).reshape(-1, 20)
    scale = b[:, 0:2].copy().view(np.float16).astype(np.float64)
    mn = b[:, 2:4].copy().view(np.float16).astype(np.float64)
    qs = b[:, 4:20]
    q = np.empty((b.shape[0], 32), np.float64)
    q[:, 0::2] = qs & 0x0F
    q[:, 1::2] = qs >> 4
    return q * scale + mn


@pytest.mark.parametrize("which", ["oracle", "product"])
def test_q4_0_block_roundtrip(g, O, which):
    w = (np.arange(32, dtype=np.float32) * np.float32(0.1))
    blocks = O.quantize_q4_0(w) if which == "oracle" else np.frombuffer(g.quantize_q4_0_native(w.tobytes()), np.uint8)
    deq = O.q4_0_dequant(blocks, fused=False)
    assert np.all(np.abs(w - deq) <= 0.11)
    # the oracle's unfused dequant (blocks.rs:29) rounds q*scale then +min
    ref = _dequant_numpy(blocks).ravel()
    assert np.all(np.abs(deq - ref) <= np.abs(ref) * 2.0 ** -23 + 1e-12)


def test_q8_0_block_roundtrip(g, O):
    w = np.arange(32, dtype=np.float32) * np.float32(0.1) - np.float32(1.6)
    blocks = np.frombuffer(g.quantize_q8_0_native(w.tobytes()), np.uint8)
    assert np.array_equal(blocks, O.quantize_q8_0(w))
    scale = float(blocks[0:2].copy().view(np.float16)[0])
    q = blocks[2:34].view(np.int8).astype(np.float32)
    deq = q * np.float32(scale)
    assert np.all(np.abs(w - deq) <= scale / 2 + 1e-5)


def test_q4_0_linear_forward_roundtrip(O):
    """src/nn/linear/tests.rs:8-100: rows i*0.1 and -i*0.1, input all ones."""
    row0 = np.arange(32, dtype=np.float32) * np.float32(0.1)
    row1 = np.arange(32, dtype=np.float32) * np.float32(-0.1)
    blocks = np.concatenate([O.quantize_q4_0(row0), O.quantize_q4_0(row1)])
    x = np.ones(32, np.float32)
    y = O.q4_0_gemv(blocks, x, 2, 32)
    for r in range(2):
        expected = float(np.sum(O.q4_0_dequant(blocks[r * 20:(r + 1) * 20], fused=False)))
        assert abs(y[r] - expected) < 1e-4


def _rope_split_numpy(x, pos, base=10000.0):
    """tests/unit/test_rope_logic.py:22-31 (split halves)."""
    dim = x.shape[-1]
    res = np.zeros_like(x)
    inv_freq = 1.0 / (base ** (np.arange(0, dim, 2, dtype=np.float32) / dim))
    theta = pos * inv_freq
    cos, sin = np.cos(theta), np.sin(theta)
    v0, v1 = x[..., : dim // 2], x[..., dim // 2:]
    res[..., : dim // 2] = v0 * cos - v1 * sin
    res[..., dim // 2:] = v0 * sin + v1 * cos
    return res


def _rope_interleaved_numpy(x, pos, base=10000.0):
    dim = x.shape[-1]
    res = np.zeros_like(x)
    inv_freq = 1.0 / (base ** (np.arange(0, dim, 2, dtype=np.float32) / dim))
    theta = pos * inv_freq
    cos, sin = np.cos(theta), np.sin(theta)
    v0, v1 = x[..., 0::2], x[..., 1::2]
    res[..., 0::2] = v0 * cos - v1 * sin
    res[..., 1::2] = v0 * sin + v1 * cos
    return res


@pytest.mark.parametrize("pos", [1, 7, 300])
def test_rope_split_matches_reference_formula(O, pos):
    rng = np.random.default_rng(pos)
    x = rng.standard_normal(64).astype(np.float32)
    got = O.rope(x, 1, 64, pos, 10000.0, split=True)
    np.testing.assert_allclose(got, _rope_split_numpy(x, pos), rtol=2e-5, atol=2e-5)
    inter = O.rope(x, 1, 64, pos, 10000.0, split=False)
    np.testing.assert_allclose(inter, _rope_interleaved_numpy(x, pos), rtol=2e-5, atol=2e-5)
    assert not np.allclose(got, inter)
