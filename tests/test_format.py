"""Host-side format work with no GPU: quantisers, the `.gaje.flat` writer and
reader, and the loader's error mapping (every malformed input is a status code,
where the reference would panic or read out of bounds)."""
import json
import os
import struct

import numpy as np
import pytest

import flat_numpy


def _edge_blocks():
    rng = np.random.default_rng(3)
    blocks = [
        np.full(32, 1.0, np.float32),                        # zero range -> scale 0
        np.full(32, -3.5, np.float32),
        np.linspace(0, 3.1, 32, dtype=np.float32),           # the reference KAT row
        np.linspace(-1e-8, 1e-8, 32, dtype=np.float32),      # range below 1e-7
        np.linspace(-70000, 70000, 32, dtype=np.float32),    # f16 overflow of min
        (rng.standard_normal(32) * 1e-6).astype(np.float32),  # subnormal f16 scale
        np.where(np.arange(32) % 2 == 0, 0.5, -0.5).astype(np.float32),
        (np.arange(32) * 15.0 / 31).astype(np.float32),      # ties at .5 steps
    ]
    return np.concatenate(blocks)


@pytest.mark.parametrize("kind", ["random", "edges"])
def test_quantizers_match_oracle(g, O, kind):
    if kind == "random":
        w = (np.random.default_rng(0).standard_normal(32 * 4096) * 0.02).astype(np.float32)
    else:
        w = _edge_blocks()
    q4 = np.frombuffer(g.quantize_q4_0_native(w.tobytes()), np.uint8)
    assert np.array_equal(q4, O.quantize_q4_0(w))
    q8 = np.frombuffer(g.quantize_q8_0_native(w.tobytes()), np.uint8)
    assert np.array_equal(q8, O.quantize_q8_0(w))


def test_quantizer_rejects_ragged(g):
    with pytest.raises(TypeError):
        g.quantize_q4_0_native(np.zeros(33, np.float32).tobytes())


def test_q4_scale_min_are_rne_f16(g):
    """half::f16::from_f32 rounds to nearest even; numpy float16 does too."""
    rng = np.random.default_rng(1)
    w = np.concatenate([(rng.standard_normal(32 * 2048) * s).astype(np.float32)
                        for s in (1e-6, 1e-3, 0.02, 3.0, 3e4)])
    b = np.frombuffer(g.quantize_q4_0_native(w.tobytes()), np.uint8).reshape(-1, 20)
    blocks = w.reshape(-1, 32)
    mn = blocks.min(axis=1)
    scale = (blocks.max(axis=1) - mn) / np.float32(15.0)
    assert np.array_equal(b[:, 0:2].copy().view(np.uint16).ravel(), scale.astype(np.float16).view(np.uint16))
    with np.errstate(over="ignore"):
        assert np.array_equal(b[:, 2:4].copy().view(np.uint16).ravel(), mn.astype(np.float16).view(np.uint16))


def test_oracle_avx2_dot_vs_float64(O):
    rng = np.random.default_rng(5)
    for nb in (1, 18, 28, 152):
        w = (rng.standard_normal(32 * nb) * 0.02).astype(np.float32)
        x = rng.standard_normal(32 * nb).astype(np.float32)
        blk = O.quantize_q4_0(w)
        deq = O.q4_0_dequant(blk, fused=True).astype(np.float64)
        exact = float(deq @ x.astype(np.float64))
        got = O.q4_0_dot(blk, x)
        scalar = O.q4_0_dot(blk, x, scalar=True)
        tol = 1e-6 * np.sum(np.abs(deq * x)) + 1e-6
        assert abs(got - exact) <= tol
        assert abs(scalar - exact) <= 4 * tol


def test_fused_dequant_within_one_ulp_of_unfused(O):
    w = (np.random.default_rng(9).standard_normal(32 * 512) * 0.02).astype(np.float32)
    blk = O.quantize_q4_0(w)
    a, b = O.q4_0_dequant(blk, True), O.q4_0_dequant(blk, False)
    assert np.all(np.abs(a - b) <= np.spacing(np.maximum(np.abs(a), np.abs(b))))


def _tiny_tensors(seed=0, bits_embd=32, n_embd=64, n_head=4, n_kv=2, ff=128, V=96, L=2, bias=True):
    rng = np.random.default_rng(seed)
    hd = n_embd // n_head
    qkv = (n_head + 2 * n_kv) * hd
    N = lambda *s: (rng.standard_normal(s) * 0.02).astype(np.float32)  # noqa: E731
    embd = N(V, n_embd)
    t = [("linear", "token_embd", bits_embd, embd, None), ("norm", "output_norm", np.ones(n_embd)),
         ("linear", "lm_head", bits_embd, embd, None)]
    for i in range(L):
        p = f"blk.{i}."
        t += [("norm", p + "attn_norm", np.ones(n_embd)), ("norm", p + "ffn_norm", np.ones(n_embd)),
              ("linear", p + "attn_qkv", 4, N(qkv, n_embd), N(qkv) if bias else None),
              ("linear", p + "attn_output", 4, N(n_embd, n_head * hd), None),
              ("linear", p + "ffn_gate_up", 4, N(2 * ff, n_embd), None),
              ("linear", p + "ffn_down", 4, N(n_embd, ff), None)]
    meta = dict(name="tiny", arch_family=3, n_embd=n_embd, n_head=n_head, n_head_kv=n_kv, n_blocks=L,
                vocab_size=V, eps=1e-6, rope_base=1e6, qk_permute=0)
    return meta, t


@pytest.mark.parametrize("bits_embd", [32, 8])
def test_writer_matches_numpy_exporter_bytes(g, tmp_path, bits_embd):
    meta, tensors = _tiny_tensors(bits_embd=bits_embd)
    a, b = str(tmp_path / "numpy.flat"), str(tmp_path / "product.flat")
    flat_numpy.write_flat(a, tensors=tensors, **meta)
    w = g.FlatWriter(b, **meta)
    for t in tensors:
        if t[0] == "norm":
            w.add_norm(t[1], t[2])
        else:
            w.add_linear(t[1], t[2], t[3], t[4])
    w.close()
    assert open(a, "rb").read() == open(b, "rb").read()


@pytest.mark.parametrize("name,over", [("tiny", {}), ("small", {}), ("tiny", {"embd_bit_depth": 8}),
                                       ("small", {"n_embd": 384, "n_head": 6, "n_head_kv": 3})])
def test_synthetic_model_without_the_product_is_byte_identical(g, tmp_path, name, over):
    """bench.py's CPU arm writes its model with the oracle and the numpy writer
    only; the file must be the product's synthetic model byte for byte."""
    cfg = dict(g.configs.CONFIGS[name])
    cfg.update(over)
    a, b = str(tmp_path / "numpy.flat"), str(tmp_path / "product.flat")
    flat_numpy.write_synthetic(a, seed=77, **cfg)
    g.write_synthetic(b, seed=77, **cfg)
    assert open(a, "rb").read() == open(b, "rb").read()


def test_inspect_reads_config_and_descriptor(g, make_model):
    info = g.inspect_flat(make_model("small"))
    assert info["n_embd"] == 256 and info["n_head"] == 8 and info["n_head_kv"] == 2
    assert info["head_dim"] == 32 and info["ffn_dim"] == 768 and info["vocab_size"] == 4096
    assert info["rope_base"] == 100000.0  # arch_family 2 (SmolLM)
    assert info["rope_style"] == "split"
    assert info["header"]["weights_offset"] % 4096 == 0
    assert abs(info["eps"] - 1e-5) < 1e-12


def test_descriptor_overrides_metadata_and_forces_split(g, O, tmp_path):
    meta, tensors = _tiny_tensors()
    p = str(tmp_path / "m.flat")
    # family 0: the metadata decides; "interleaved" survives, base from JSON
    flat_numpy.write_flat(p, tensors=tensors, **dict(meta, arch_family=0),
                          config_extra={"rope_style": "interleaved", "rope_base": 5000.0})
    info = g.inspect_flat(p)
    assert info["rope_style"] == "interleaved" and info["rope_base"] == 5000.0
    assert O.OracleModel(p).rope_base == 5000.0
    # family 3: the header descriptor forces split and 1e6
    raw = bytearray(open(p, "rb").read())
    struct.pack_into("<I", raw, 56, 3)
    open(p, "wb").write(bytes(raw))
    info = g.inspect_flat(p)
    assert info["rope_style"] == "split" and info["rope_base"] == 1e6
    assert O.OracleModel(p).rope_base == 1e6


def _corrupt(tmp_path, make, edit):
    meta, tensors = _tiny_tensors()
    p = str(tmp_path / f"{make}.flat")
    flat_numpy.write_flat(p, tensors=tensors, **meta)
    raw = bytearray(open(p, "rb").read())
    raw = edit(raw)
    open(p, "wb").write(bytes(raw))
    return p


def _edit_dir(raw, fn):
    mlen = struct.unpack_from("<Q", raw, 16)[0]
    dlen = struct.unpack_from("<Q", raw, 24)[0]
    woff = struct.unpack_from("<Q", raw, 32)[0]
    d = json.loads(bytes(raw[4096 + mlen:4096 + mlen + dlen]))
    d = fn(d)
    new = json.dumps(d).encode()
    assert 4096 + mlen + len(new) <= woff
    raw[4096 + mlen:woff] = new + b"\0" * (woff - 4096 - mlen - len(new))
    struct.pack_into("<Q", raw, 24, len(new))
    return raw


def _drop(name):
    return lambda d: [e for e in d if e["name"] != name]


def _set(name, key, val):
    def f(d):
        for e in d:
            if e["name"] == name:
                e[key] = val
        return d
    return f


@pytest.mark.parametrize("case,status", [
    ("truncated", "GAJE_ERR_IO"),
    ("bad_magic", "GAJE_ERR_IO"),
    ("bad_json", "GAJE_ERR_IO"),
    ("missing_eps", "GAJE_ERR_IO"),
    ("missing_tensor", "GAJE_ERR_NOT_FOUND"),
    ("dna_len", "GAJE_ERR_SHAPE"),
    ("in_features", "GAJE_ERR_SHAPE"),
    ("past_eof", "GAJE_ERR_IO"),
    ("anchors", "GAJE_ERR_UNSUPPORTED"),
    ("centroids", "GAJE_ERR_SHAPE"),  # a Q4_0 block buffer is not Genomic4Bit nibbles
])
def test_loader_errors_are_status_codes(g, tmp_path, case, status):
    def edit(raw):
        if case == "truncated":
            return raw[:3000]
        if case == "bad_magic":
            raw[0:4] = b"GAJF"
            return raw
        if case == "bad_json":
            raw[4096] = ord("[")
            return raw
        if case == "missing_eps":
            mlen = struct.unpack_from("<Q", raw, 16)[0]
            md = json.loads(bytes(raw[4096:4096 + mlen]))
            del md["eps"]
            new = json.dumps(md).encode()
            raw[4096:4096 + mlen] = new + b" " * (mlen - len(new))
            return raw
        if case == "missing_tensor":
            return _edit_dir(raw, _drop("blk.1.ffn_down"))
        if case == "dna_len":
            return _edit_dir(raw, _set("blk.0.attn_output", "dna_len", 100))
        if case == "in_features":
            return _edit_dir(raw, _set("blk.0.ffn_down", "in_features", 100))
        if case == "past_eof":
            return _edit_dir(raw, _set("lm_head", "dna_off", 10 ** 9))
        if case == "anchors":
            return _edit_dir(raw, _set("blk.0.attn_qkv", "anc_len", 16))
        if case == "centroids":
            return _edit_dir(raw, _set("blk.0.ffn_gate_up", "c_len", 64))
        raise AssertionError(case)

    p = _corrupt(tmp_path, case, edit)
    with pytest.raises(IOError) as e:
        g.inspect_flat(p)
    assert e.value.status == {"GAJE_ERR_IO": 2, "GAJE_ERR_NOT_FOUND": 3, "GAJE_ERR_SHAPE": 4,
                              "GAJE_ERR_UNSUPPORTED": 5}[status]


def test_missing_tensor_message_matches_reference(g, tmp_path):
    p = _corrupt(tmp_path, "mt", lambda raw: _edit_dir(raw, _drop("lm_head")))
    with pytest.raises(IOError) as e:
        g.inspect_flat(p)
    assert "Flat tensor entry 'lm_head' not found" in str(e.value)


def test_unfused_tensors_load(g, O, tmp_path):
    """attn_q/k/v and ffn_gate/ffn_up (no fused entries) resolve to the same
    model as the fused file (forward_fused_3/_2 concatenate rows)."""
    meta, tensors = _tiny_tensors(seed=4)
    fused = str(tmp_path / "fused.flat")
    flat_numpy.write_flat(fused, tensors=tensors, **meta)
    hd = meta["n_embd"] // meta["n_head"]
    qd, kvd = meta["n_head"] * hd, meta["n_head_kv"] * hd
    split = []
    for t in tensors:
        if t[0] == "linear" and t[1].endswith("attn_qkv"):
            p = t[1][: -len("attn_qkv")]
            W, b = t[3], t[4]
            split += [("linear", p + "attn_q", 4, W[:qd], b[:qd]),
                      ("linear", p + "attn_k", 4, W[qd:qd + kvd], b[qd:qd + kvd]),
                      ("linear", p + "attn_v", 4, W[qd + kvd:], b[qd + kvd:])]
        elif t[0] == "linear" and t[1].endswith("ffn_gate_up"):
            p = t[1][: -len("ffn_gate_up")]
            ff = t[3].shape[0] // 2
            split += [("linear", p + "ffn_gate", 4, t[3][:ff], None),
                      ("linear", p + "ffn_up", 4, t[3][ff:], None)]
        else:
            split.append(t)
    unf = str(tmp_path / "unfused.flat")
    flat_numpy.write_flat(unf, tensors=split, **meta)
    info = g.inspect_flat(unf)
    assert info["fused_qkv"] == 0 and info["fused_gate_up"] == 0 and info["ffn_dim"] == 128
    a, b = O.OracleModel(fused), O.OracleModel(unf)
    for tok in (3, 17, 5):
        assert np.array_equal(a.forward(tok), b.forward(tok))


def test_lut4_files_resolve_and_engine_limits(g, tmp_path):
    """Genomic4Bit body tensors (bit_depth 4 with a centroid blob) resolve; the
    engine takes them on the single-stream path only, and a matrix kind must
    be a table in every block or in none (checked before any CUDA call)."""
    cfg = dict(g.configs.CONFIGS["tiny"])
    path = str(tmp_path / "lut.flat")
    flat_numpy.write_synthetic_lut4(path, seed=2, **cfg)
    info = g.inspect_flat(path)
    assert info["n_blocks"] == cfg["n_blocks"]
    with pytest.raises(IOError) as e:  # load_genomic_auto failures are io::Error (flat_reader.rs:240)
        g.load_genomic_auto(path, max_ctx=16, max_streams=2)
    assert "single-stream" in str(e.value)

    mixed = str(tmp_path / "mixed.flat")
    flat_numpy.write_synthetic_lut4(mixed, seed=2, **cfg)
    raw = bytearray(open(mixed, "rb").read())
    q4 = str(tmp_path / "q4.flat")
    g.write_synthetic(q4, seed=2, **cfg)
    # block 1's ffn_down back to a Q4_0 entry: a kind that mixes formats
    meta, dlen = struct.unpack_from("<Q", raw, 16)[0], struct.unpack_from("<Q", raw, 24)[0]
    d = json.loads(bytes(raw[4096 + meta:4096 + meta + dlen]))
    e1 = next(x for x in d if x["name"] == "blk.1.ffn_down")
    e1["c_len"] = 0
    e1["dna_len"] = e1["out_features"] * e1["in_features"] // 32 * 20
    new = json.dumps(d).encode()
    assert len(new) <= dlen
    raw[4096 + meta:4096 + meta + dlen] = new + b" " * (dlen - len(new))
    weights_len = struct.unpack_from("<Q", raw, 40)[0]
    raw.extend(b"\0" * (e1["dna_len"]))  # room for the reinterpreted blob
    struct.pack_into("<Q", raw, 40, weights_len + e1["dna_len"])
    open(mixed, "wb").write(raw)
    with pytest.raises(IOError) as e:
        g.load_genomic_auto(mixed, max_ctx=16)
    assert "mixes Genomic4Bit tables and Q4_0 blocks" in str(e.value)
