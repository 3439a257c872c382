"""GPU parity of the resident quantized Llama loop (QBlock stack + greedy
generate) against the CPU oracle's restatement of
src/streaming_quantized.rs:193-317,539-633 on identical weights:
logits of the last position, and identical greedy token ids (north-star
test c).  Also the device-side decode step under CUDA-graph replay and
KV-cache truncation (truncate_caches, :603-609)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CFG = dict(hidden=512, intermediate=1024, n_heads=8, n_kv_heads=2, head_dim=64, n_layers=2,
           vocab=1000, max_seq=64, max_batch_tokens=32, rms_eps=1e-5, rope_theta=10000.0)
LOGIT_TOL = 1e-4  # relative L2 of the last-position logits


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


def build(oracle, qtype, seed, cfg=CFG):
    from rustyllm_b200.llama import random_model
    model, host = random_model(cfg, qtype, seed, host_blocks=True)
    ref = oracle.OracleLlama(cfg, qtype)
    for l, (blocks, r1, r2) in enumerate(host["layers"]):
        ref.set_layer(l, blocks, r1, r2)
    ref.set_embedding(host["embed"])
    ref.set_head(host["ln_f"], host["lm_head"])
    return model, ref


@pytest.mark.parametrize("qtype,n_prompt", [(12, 20), (12, 28), (11, 20), (12, 3), (12, 13)])
def test_prompt_logits_and_greedy_tokens_match_oracle(oracle, rq_ctx, qtype, n_prompt):
    """Q4_K prompts of 4..23 tokens run their linears on the mma.sync
    kernel, 24 and more on tcgen05; 3 tokens and Q3_K run M=1 jobs."""
    model, ref = build(oracle, qtype, seed=qtype + n_prompt)
    rng = np.random.default_rng(20)
    prompt = rng.integers(0, CFG["vocab"], size=n_prompt).astype(np.int32)
    lg, nxt = model.forward(prompt, 0)
    lr, nr = ref.forward(prompt, 0)
    assert rel_l2(lg, lr) <= LOGIT_TOL
    assert nxt == nr
    gen = model.generate(prompt, 16)
    want = ref.generate(prompt, 16)
    assert gen == want


@pytest.mark.parametrize("n_prompt", [2, 3, 7, 30])
def test_q3k_prompt_one_weight_pass_matches_oracle(oracle, rq_ctx, n_prompt):
    """Q3_K layers whose every K is a multiple of 2048 run two- and
    three-token forwards (speculative verify) on the int8 tensor-core
    kernel and prompts of 6 or more tokens on the tcgen05 kernel, one weight
    pass each; the logits and the greedy tokens still equal the oracle's."""
    cfg = dict(CFG, hidden=2048, intermediate=4096, n_heads=16, n_kv_heads=4, head_dim=128)
    model, ref = build(oracle, 11, seed=77 + n_prompt, cfg=cfg)
    rng = np.random.default_rng(21)
    prompt = rng.integers(0, cfg["vocab"], size=n_prompt).astype(np.int32)
    lg, nxt = model.forward(prompt, 0)
    lr, nr = ref.forward(prompt, 0)
    assert rel_l2(lg, lr) <= LOGIT_TOL
    assert nxt == nr
    assert model.generate(prompt, 8) == ref.generate(prompt, 8)


def test_chunked_prompt_matches_one_pass(oracle, rq_ctx):
    """A prompt fed as chunks of 6 and 25 tokens (the second at position 6,
    attention over the cached keys) gives the one-pass logits and tokens."""
    model, ref = build(oracle, 12, seed=44)
    prompt = np.random.default_rng(9).integers(0, CFG["vocab"], size=31).astype(np.int32)
    model.forward(prompt[:6], 0)
    lg, nxt = model.forward(prompt[6:], 6)
    lr, nr = ref.forward(prompt, 0)
    assert rel_l2(lg, lr) <= LOGIT_TOL
    assert nxt == nr


def test_decode_step_graph_and_truncate(oracle, rq_ctx):
    import torch
    model, ref = build(oracle, 12, seed=5)
    prompt = np.random.default_rng(3).integers(0, CFG["vocab"], size=12).astype(np.int32)
    want = ref.generate(prompt, 10)
    # graph-captured device step
    from rustyllm_b200._lib import check, lib
    check(lib().rq_llama_reset_tokens(model.handle))
    model.forward(prompt, 0)
    model.decode_step()  # warm-up outside capture
    s = torch.cuda.Stream()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        model.decode_step(torch.cuda.current_stream().cuda_stream)
    for _ in range(8):
        g.replay()
    torch.cuda.synchronize()
    toks, pos = model.tokens()
    assert toks[:10] == want
    assert pos == len(prompt) + 9
    # roll back three positions and decode again from there
    keep = len(prompt) + 4          # prompt + 4 accepted tokens in the cache
    model.truncate_caches(keep)
    _, nxt = model.forward([want[4]], keep)
    assert nxt == want[5]
    del g


@pytest.mark.parametrize("qtype", [12, 11, 2])
def test_one_launch_step_matches_launch_chain(oracle, rq_ctx, qtype):
    """The persistent one-launch decode step computes the same tokens as the
    per-layer launch chain and the oracle, for every weight type."""
    cfg = dict(CFG, n_layers=3)
    model, ref = build(oracle, qtype, seed=30 + qtype, cfg=cfg)
    prompt = np.random.default_rng(8).integers(0, cfg["vocab"], size=9).astype(np.int32)
    model.set_fused(True)
    fused = model.generate(prompt, 12)
    model.set_fused(False)
    chain = model.generate(prompt, 12)
    assert fused == chain
    assert fused == ref.generate(prompt, 12)


def test_llama_rejects_bad_config(rq_ctx):
    from rustyllm_b200 import RqError
    from rustyllm_b200.llama import StreamingLlamaQuantized
    bad = dict(CFG, hidden=500)
    with pytest.raises(RqError, match="multiples of 256"):
        StreamingLlamaQuantized(bad)
