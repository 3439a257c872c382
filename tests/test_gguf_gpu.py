"""GGUF shards straight to the GPU: a Llama model loaded from a shard
directory in the reference's layout (rq_llama_load_gguf_dir) decodes the
oracle's greedy tokens for the same weights (F16 norms as the shards store
them), and row / column slices of a GGUF matrix (tensor-parallel shards)
give the oracle's products of the same sliced blocks."""
import numpy as np
import pytest

from gguf_util import Q4_K, write_gguf, write_shard_dir

pytestmark = pytest.mark.gpu

CFG = dict(hidden=512, intermediate=1024, n_heads=8, n_kv_heads=2, head_dim=64, n_layers=2,
           vocab=1000, max_seq=64, max_batch_tokens=32, rms_eps=1e-5, rope_theta=10000.0)


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


@pytest.mark.parametrize("qtype", [12, 11])
def test_llama_from_gguf_dir_matches_oracle(oracle, rq_ctx, tmp_path, qtype):
    from rustyllm_b200.llama import StreamingLlamaQuantized, random_model
    src, host = random_model(CFG, qtype, seed=31 + qtype, host_blocks=True)
    src.close()
    layers, lnf = write_shard_dir(tmp_path / "shards", CFG, qtype, host)
    model = StreamingLlamaQuantized.from_gguf_dir(CFG, tmp_path / "shards")
    ref = oracle.OracleLlama(CFG, qtype)
    for l, (blocks, r1, r2) in enumerate(layers):
        ref.set_layer(l, blocks, r1, r2)
    ref.set_embedding(host["embed"])
    ref.set_head(lnf, host["lm_head"])
    prompt = np.random.default_rng(7).integers(0, CFG["vocab"], size=14).astype(np.int32)
    lg, nxt = model.forward(prompt, 0)
    lr, nr = ref.forward(prompt, 0)
    assert rel_l2(lg, lr) <= 1e-4 and nxt == nr
    model.close()
    model = StreamingLlamaQuantized.from_gguf_dir(CFG, tmp_path / "shards")
    assert model.generate(prompt, 10) == ref.generate(prompt, 10)
    model.close()


def test_gguf_matrix_slices(oracle, rq_ctx, tmp_path):
    """Rows (column-parallel shard) and block-aligned columns (row-parallel
    shard) of a Q4_K matrix uploaded from a GGUF file."""
    from rustyllm_b200.gguf import GGUFFile
    from rustyllm_b200.linear import _linear
    out, n_in = 96, 1024
    rng = np.random.default_rng(2)
    w = (rng.standard_normal((out, n_in)) * 0.02).astype(np.float32)
    blocks = oracle.quantize(Q4_K, w).reshape(out, -1)          # [out][4 * 144]
    write_gguf(tmp_path / "w.gguf", [("m.weight", Q4_K, (out, n_in), blocks.tobytes())])
    f = GGUFFile(tmp_path / "w.gguf")
    x = rng.standard_normal((3, n_in)).astype(np.float32)
    full = f.upload(rq_ctx, "m.weight")
    ref = oracle.matmul_ref(Q4_K, blocks, out, n_in, x, acc64=True)
    assert rel_l2(_linear(full, x), ref) <= 1e-4
    rows = f.upload(rq_ctx, "m.weight", rows=(32, 80))
    ref_r = oracle.matmul_ref(Q4_K, blocks[32:80], 48, n_in, x, acc64=True)
    assert rel_l2(_linear(rows, x), ref_r) <= 1e-4
    cols = f.upload(rq_ctx, "m.weight", cols=(512, 1024))       # super-blocks 2, 3
    sub = np.ascontiguousarray(blocks[:, 2 * 144:4 * 144])
    ref_c = oracle.matmul_ref(Q4_K, sub, out, 512, x[:, 512:], acc64=True)
    assert rel_l2(_linear(cols, x[:, 512:]), ref_c) <= 1e-4
    from rustyllm_b200._lib import RqError
    with pytest.raises(RqError):
        f.upload(rq_ctx, "m.weight", cols=(100, 1024))            # not on a block boundary


@pytest.mark.parametrize("qtype", [8, 14, 13, 10])
def test_gguf_other_formats(oracle, rq_ctx, tmp_path, qtype):
    """Q8_0 / Q6_K / Q5_K / Q2_K tensors read from a GGUF file: the bytes the
    file holds reach the device unchanged and the matvec matches the oracle,
    whole and as a row slice."""
    from rustyllm_b200.gguf import GGUFFile
    from rustyllm_b200.linear import _linear
    out, n_in = 80, 2048
    rng = np.random.default_rng(qtype)
    w = (rng.standard_normal((out, n_in)) * 0.02).astype(np.float32)
    blocks = oracle.quantize(qtype, w).reshape(out, -1)
    write_gguf(tmp_path / "w.gguf", [("m.weight", qtype, (out, n_in), blocks.tobytes())])
    f = GGUFFile(tmp_path / "w.gguf")
    full = f.upload(rq_ctx, "m.weight")
    assert np.array_equal(full.download(), blocks)
    x = rng.standard_normal((2, n_in)).astype(np.float32)
    assert rel_l2(_linear(full, x), oracle.matmul_ref(qtype, blocks, out, n_in, x, acc64=True)) <= 1e-4
    rows = f.upload(rq_ctx, "m.weight", rows=(16, 64))
    ref_r = oracle.matmul_ref(qtype, np.ascontiguousarray(blocks[16:64]), 48, n_in, x, acc64=True)
    assert rel_l2(_linear(rows, x), ref_r) <= 1e-4
