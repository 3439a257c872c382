"""Speculative decoding on the GPU (examples/spec_decode_70b.rs:213-336,
forward_all and truncate_caches of src/streaming_quantized.rs:603-620): the
verify forward's per-position logits and greedy tokens match the oracle
decoding the same tokens one at a time, and the draft/verify loop emits the
target's greedy tokens whatever the draft proposes (verify widths M = K+1 of
2, 5 and 25 run the M=1 pipeline, the mma.sync and the tcgen05 kernels)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CFG = dict(hidden=512, intermediate=1024, n_heads=8, n_kv_heads=2, head_dim=64, n_layers=2,
           vocab=1000, max_seq=128, max_batch_tokens=32, rms_eps=1e-5, rope_theta=10000.0)


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


def _oracle(oracle, host, qtype=12):
    ref = oracle.OracleLlama(CFG, qtype)
    for l, (blocks, r1, r2) in enumerate(host["layers"]):
        ref.set_layer(l, blocks, r1, r2)
    ref.set_embedding(host["embed"])
    ref.set_head(host["ln_f"], host["lm_head"])
    return ref


@pytest.mark.parametrize("T", [2, 4, 5, 12, 25])
def test_forward_all_matches_oracle_per_position(oracle, rq_ctx, T):
    from rustyllm_b200.llama import random_model
    model, host = random_model(CFG, 12, seed=61, host_blocks=True)
    ref = _oracle(oracle, host)
    rng = np.random.default_rng(T)
    prompt = rng.integers(0, CFG["vocab"], size=12).astype(np.int32)
    verify = rng.integers(0, CFG["vocab"], size=T).astype(np.int32)
    model.forward(prompt, 0, want_logits=False)
    ref.forward(prompt, 0)
    logits, amax = model.forward_all(verify, len(prompt), want_logits=True)
    for i in range(T):
        lr, nr = ref.forward([verify[i]], len(prompt) + i)
        assert rel_l2(logits[i], lr) <= 1e-4
        assert amax[i] == nr
    model.close()


@pytest.mark.parametrize("k,adaptive", [(1, False), (4, False), (4, True), (24, False)])
def test_spec_decode_emits_the_target_greedy_tokens(rq_ctx, k, adaptive):
    from rustyllm_b200.llama import random_model
    from rustyllm_b200.spec import SpecDecoder
    target, _ = random_model(CFG, 12, seed=71)
    draft, _ = random_model(CFG, 12, seed=72)
    prompt = np.random.default_rng(3).integers(0, CFG["vocab"], size=10).astype(np.int32)
    want = target.generate(prompt, 30)
    sd = SpecDecoder(target, draft, k=k, adaptive=adaptive)
    assert sd.generate(prompt, 30) == want
    target.close()
    draft.close()


def test_self_draft_is_accepted(rq_ctx):
    """The target's own weights as the draft: the draft proposes the target's
    greedy tokens, so (numerical near-ties aside) every draft is accepted."""
    from rustyllm_b200.llama import random_model
    from rustyllm_b200.spec import SpecDecoder
    target, _ = random_model(CFG, 12, seed=81)
    draft, _ = random_model(CFG, 12, seed=81)
    prompt = np.random.default_rng(4).integers(0, CFG["vocab"], size=10).astype(np.int32)
    want = target.generate(prompt, 25)
    sd = SpecDecoder(target, draft, k=4)
    assert sd.generate(prompt, 25) == want
    assert sd.stats["accepted"] >= 0.9 * sd.stats["proposed"]
    assert sd.stats["target_forwards"] <= 1 + (25 + 4) // 5 + 1
    target.close()
    draft.close()
