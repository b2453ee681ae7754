"""Block-causal sessions with retained K/V on the GPU: block forwards against
the oracle's block-causal whole-sequence forward, recompute against cached
generation (exact), and the two-turn report."""

import numpy as np
import pytest

from diffusionhard_b200 import _lib
from diffusionhard_b200.model import MDLMConfig, build_quantized
from diffusionhard_b200.session import BlockCausalSession, evaluate_two_turn_mdlm_session
from oracle import model_oracle

pytestmark = pytest.mark.gpu

SMALL = MDLMConfig(vocab_size=1000, mask_token_id=999, blocks=2)


@pytest.fixture(scope="module")
def small_model():
    return build_quantized(SMALL, seed=0)


def _device_error():
    err = np.zeros(1, np.uint32)
    _lib.call("dh_device_error", err.ctypes.data, 1)
    return int(err[0])


def test_block_forwards_match_block_causal_oracle(cuda, small_model):
    torch = cuda
    qm = small_model
    B, sizes = 2, [64, 32, 32, 64]
    total = sum(sizes)
    ids = torch.randint(0, 999, (B, total), generator=torch.Generator().manual_seed(6))
    sess = BlockCausalSession(qm, B, total)
    starts = np.cumsum([0] + sizes)
    engines = [sess.append(ids[:, starts[i]:starts[i + 1]]) for i in range(3)]
    active = sess.engine(int(starts[3]), sizes[3])
    active.tokens.copy_(ids[:, starts[3]:].reshape(-1).to(torch.int32))
    active.forward()
    torch.cuda.synchronize()
    rec = {}
    model_oracle.forward(qm, ids.numpy(), block_ends=[int(e) for e in starts[1:4]], record=rec)
    ref = rec[f"x{SMALL.blocks - 1}"]
    for i, e in enumerate(engines + [active]):
        got = e.x.cpu().view(B, sizes[i], 768)
        want = ref[:, starts[i]:starts[i + 1]]
        assert ((got - want).norm() / want.norm()).item() < 1e-2, i
    # the completed blocks' K/V are those of the block-causal forward: re-running
    # block 1 after block 3 was written leaves its output unchanged
    x1 = engines[1].x.clone()
    engines[1].forward()
    assert torch.equal(engines[1].x, x1)
    assert sess.kv_bytes() == 2 * SMALL.blocks * B * 128 * 768 * 2
    assert _device_error() == 0


def test_recompute_equals_cached_generation(cuda, small_model):
    torch = cuda
    sess = BlockCausalSession(small_model, 1, 192)
    prompt = torch.randint(0, 999, (1, 64), generator=torch.Generator().manual_seed(1))
    sess.append(prompt)
    a, meta_a, _, ev_a = sess.generate(64, steps=24, seed=5, recompute=True)
    b, meta_b, _, ev_b = sess.generate(64, steps=24, seed=5)
    assert torch.equal(a, b)
    assert meta_a["transition_active_tokens"] == meta_b["transition_active_tokens"]
    assert not (b == SMALL.mask_token_id).any()
    sess.append(b)
    c, _, _, _ = sess.generate(64, steps=24, seed=6, recompute=True)
    d, _, _, _ = sess.generate(64, steps=24, seed=6)
    assert torch.equal(c, d)
    assert sess.length == 128
    sess.truncate(64)
    assert sess.block_ends() == [64]
    with pytest.raises(ValueError, match="block boundary"):
        sess.truncate(40)
    with pytest.raises(ValueError, match="multiples of 32"):
        sess.engine(64, 48)
    assert _device_error() == 0


def test_two_turn_report(cuda, small_model):
    r = evaluate_two_turn_mdlm_session(quantized=small_model, samples=2, steps=16)
    agg = r["aggregate"]
    assert agg["exact_turn_1_sequences"] == 2 and agg["exact_turn_2_sequences"] == 2
    assert agg["identical_turn_2_transition_schedules"] == 2
    assert agg["minimum_turn_2_token_agreement"] == 1.0
    s = r["sample_results"][0]
    assert s["turn_2"]["final_cache_tokens"] == 160
    assert s["turn_2"]["recompute"]["model_forward_latency_ms"] > 0
    assert r["session_shape"]["final_session_tokens"] == 160
