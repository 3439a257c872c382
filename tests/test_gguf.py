"""GGUF reading (rq_gguf_*), on the CPU: files written the way the
reference's shards are (candle's writer: version 3, no metadata) and by
gguf-py's GGUFWriter (metadata, custom alignment) parse to the same names,
types, shapes and bytes as written; F16 / BF16 / F32 norms read as f32;
truncated and malformed files are errors, never crashes."""
import numpy as np
import pytest

from gguf_util import BF16, F16, F32, Q3_K, Q4_0, Q4_K, write_gguf


def _tensors(oracle):
    rng = np.random.default_rng(3)
    out = []
    for name, t, (o, i) in (("blk.q4k", Q4_K, (48, 512)), ("blk.q40", Q4_0, (40, 256)),
                            ("blk.q3k", Q3_K, (24, 768))):
        w = (rng.standard_normal((o, i)) * 0.02).astype(np.float32)
        out.append((name, t, (o, i), oracle.quantize(t, w).tobytes()))
    v = rng.standard_normal(512).astype(np.float32)
    out.append(("norm.f16", F16, (512,), np.float16(v).tobytes()))
    out.append(("norm.f32", F32, (512,), v.tobytes()))
    bf = (v.view(np.uint32) >> 16).astype(np.uint16)
    out.append(("norm.bf16", BF16, (512,), bf.tobytes()))
    out.append(("odd.i8", 24, (3, 5), bytes(range(15))))
    return out, v, bf


def test_candle_style_file_roundtrip(oracle, tmp_path):
    from rustyllm_b200.gguf import GGUFFile
    ts, v, bf = _tensors(oracle)
    path = tmp_path / "model.layers.0.gguf"
    write_gguf(path, ts)
    f = GGUFFile(path)
    assert len(f) == len(ts)
    assert f.names() == [t[0] for t in ts]
    for k, (name, t, shape, raw) in enumerate(ts):
        info = f.info(k)
        assert (info["type"], info["shape"], info["nbytes"]) == (t, shape, len(raw))
        assert f.raw(name).tobytes() == raw
        assert info["offset"] % 32 == 0
    np.testing.assert_array_equal(f.read_f32("norm.f32"), v)
    np.testing.assert_array_equal(f.read_f32("norm.f16"), np.float16(v).astype(np.float32))
    np.testing.assert_array_equal(f.read_f32("norm.bf16"), (bf.astype(np.uint32) << 16).view(np.float32))
    # the same bytes through the in-memory entry point
    g = GGUFFile(open(path, "rb").read())
    assert g.names() == f.names() and g.raw("blk.q3k").tobytes() == ts[2][3]


def test_gguf_py_written_file(oracle, tmp_path):
    """gguf-py writes metadata (architecture string, custom alignment 64) and
    a Q4_K tensor given as raw bytes; our offsets agree with its reader."""
    import gguf
    from rustyllm_b200.gguf import GGUFFile
    rng = np.random.default_rng(5)
    w = (rng.standard_normal((32, 512)) * 0.02).astype(np.float32)
    blocks = oracle.quantize(Q4_K, w)
    norm = rng.standard_normal(512).astype(np.float16)
    path = str(tmp_path / "gp.gguf")
    wr = gguf.GGUFWriter(path, "llama")
    wr.add_custom_alignment(64)
    wr.add_uint32("test.count", 7)
    wr.add_array("test.list", [1, 2, 3])
    wr.add_tensor("model.layers.0.mlp.up_proj.weight", blocks.reshape(32, -1),
                  raw_dtype=gguf.GGMLQuantizationType.Q4_K)
    wr.add_tensor("model.layers.0.input_layernorm.weight", norm)
    wr.write_header_to_file()
    wr.write_kv_data_to_file()
    wr.write_tensors_to_file()
    wr.close()
    f = GGUFFile(path)
    rd = gguf.GGUFReader(path)
    assert f.names() == [t.name for t in rd.tensors]
    for k, t in enumerate(rd.tensors):
        info = f.info(k)
        assert info["offset"] == t.data_offset and info["offset"] % 64 == 0
        assert info["nbytes"] == t.n_bytes
    assert f.raw("model.layers.0.mlp.up_proj.weight").tobytes() == blocks.tobytes()
    assert f.info(0)["shape"] == (32, 512) and f.info(0)["type"] == Q4_K
    np.testing.assert_array_equal(f.read_f32("model.layers.0.input_layernorm.weight"), norm.astype(np.float32))


def test_malformed_files_are_errors(oracle, tmp_path):
    from rustyllm_b200._lib import RqError
    from rustyllm_b200.gguf import GGUFFile
    ts, _, _ = _tensors(oracle)
    path = tmp_path / "m.gguf"
    write_gguf(path, ts)
    data = open(path, "rb").read()
    # (the last tensor has 15 bytes + 17 of padding: cutting 20 bytes cuts its data)
    for cut in (0, 3, 8, 23, 40, 100, len(data) // 2, len(data) - 20):
        with pytest.raises(RqError):
            GGUFFile(data[:cut])
    bad = bytearray(data)
    bad[:4] = b"GGUX"
    with pytest.raises(RqError, match="magic"):
        GGUFFile(bytes(bad))
    bad = bytearray(data)
    bad[4:8] = (1).to_bytes(4, "little")
    with pytest.raises(RqError, match="version"):
        GGUFFile(bytes(bad))
    with pytest.raises(RqError):
        GGUFFile(tmp_path / "missing.gguf")
    f = GGUFFile(data)
    with pytest.raises(RqError, match="no tensor"):
        f.index("nope")
    with pytest.raises(RqError, match="not F32/F16/BF16"):
        f.read_f32("blk.q4k")
