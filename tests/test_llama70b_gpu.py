"""GPU parity of the resident Llama loop at the full Llama-2-70B layer
geometry (Platypus2-70B: hidden 8192, 64 query / 8 KV heads, head_dim 128,
intermediate 28672, vocab 32000, RMSNorm eps 1e-5, RoPE theta 10000) with
two Q4_K layers, against the oracle's restatement of
src/streaming_quantized.rs:193-317,539-633 on identical block bytes:

  - the prompt's last-position logits within relative L2 1e-4;
  - 16 greedy tokens identical (north-star test c): the oracle runs the
    prompt plus the GPU's tokens teacher-forced, and its argmax at every
    position must be the token the GPU emitted there;
  - the speculative-verify forward (forward_all) logits of every position
    within relative L2 1e-4.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CFG = dict(hidden=8192, intermediate=28672, n_heads=64, n_kv_heads=8, head_dim=128, n_layers=2,
           vocab=32000, max_seq=64, max_batch_tokens=40, rms_eps=1e-5, rope_theta=10000.0)
LOGIT_TOL = 1e-4  # relative L2 of a position's logits
PROMPT, NEW = 20, 16


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


@pytest.fixture(scope="module")
def pair(oracle, rq_ctx):
    from rustyllm_b200.llama import random_model
    model, host = random_model(CFG, 12, seed=7070, host_blocks=True)
    ref = oracle.OracleLlama(CFG, 12)
    for l, (blocks, r1, r2) in enumerate(host["layers"]):
        ref.set_layer(l, blocks, r1, r2)
    ref.set_embedding(host["embed"])
    ref.set_head(host["ln_f"], host["lm_head"])
    yield model, ref, host
    model.close()


def margins(logits):
    top2 = np.sort(logits, axis=1)[:, -2:]
    return top2[:, 1] - top2[:, 0]


def test_70b_geometry_prompt_logits_and_greedy_tokens(pair):
    model, ref, _ = pair
    prompt = np.random.default_rng(20).integers(0, CFG["vocab"], size=PROMPT).astype(np.int32)
    lg, nxt = model.forward(prompt, 0)
    gen = model.generate(prompt, NEW)
    seq = np.concatenate([prompt, np.array(gen[:-1], np.int32)])
    ref_logits, ref_amax = ref.forward_all(seq, 0)
    assert rel_l2(lg, ref_logits[PROMPT - 1]) <= LOGIT_TOL
    want = ref_amax[PROMPT - 1:].tolist()
    m = margins(ref_logits[PROMPT - 1:])
    assert nxt == want[0]
    assert gen == want, f"GPU {gen} oracle {want}; top-1/top-2 margins {np.round(m, 5).tolist()}"


def test_70b_geometry_verify_forward_logits(pair):
    """forward_all over K+1 = 9 tokens after a 12-token prompt (the
    speculative-verify batch, M = 9 on the split-K tcgen05 kernel): every
    position's logits and argmax against the oracle."""
    model, ref, _ = pair
    rng = np.random.default_rng(21)
    prompt = rng.integers(0, CFG["vocab"], size=12).astype(np.int32)
    draft = rng.integers(0, CFG["vocab"], size=9).astype(np.int32)
    model.forward(prompt, 0, want_logits=False)
    logits, amax = model.forward_all(draft, 12, want_logits=True)
    ref_logits, ref_amax = ref.forward_all(np.concatenate([prompt, draft]), 0)
    for t in range(9):
        assert rel_l2(logits[t], ref_logits[12 + t]) <= LOGIT_TOL, t
    assert amax == ref_amax[12:].tolist()


@pytest.mark.parametrize("T", [2, 3, 4, 6, 8])
def test_70b_geometry_small_verify(pair, T):
    """forward_all over 2..8 tokens (the verify of a one- to seven-token
    draft): all seven linears on the int8 tensor-core kernels in one weight
    pass (two tokens: B fragments in registers; three and four: the
    twelve-column form; five to eight: the 24-column form; down_proj,
    in = 28672, with K split over four CTAs per row group); every position
    within 1e-4 of the oracle, argmax equal."""
    model, ref, _ = pair
    rng = np.random.default_rng(20 + T)
    prompt = rng.integers(0, CFG["vocab"], size=12).astype(np.int32)
    draft = rng.integers(0, CFG["vocab"], size=T).astype(np.int32)
    model.forward(prompt, 0, want_logits=False)
    logits, amax = model.forward_all(draft, 12, want_logits=True)
    ref_logits, ref_amax = ref.forward_all(np.concatenate([prompt, draft]), 0)
    for t in range(T):
        assert rel_l2(logits[t], ref_logits[12 + t]) <= LOGIT_TOL, t
    assert amax == ref_amax[12:].tolist()
