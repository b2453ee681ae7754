"""Block-causal attention bias of the oracle against the reference's own
block_isolation attention (tests/golden/make_block_golden.py), and the
session's argument checks.  No GPU."""

import sys

import numpy as np
import pytest
import torch

from conftest import GOLDEN

sys.path.insert(0, str(GOLDEN))
from make_block_golden import CASES, qkv_case  # noqa: E402

from oracle.model_oracle import block_causal_bias  # noqa: E402

G = np.load(GOLDEN / "block_golden.npz")


@pytest.mark.parametrize("case", range(len(CASES)))
def test_block_causal_bias_matches_reference(case):
    qkv = qkv_case(torch)
    S = qkv.shape[0]
    q, k, v = (t.transpose(0, 1).unsqueeze(0) for t in qkv.unbind(dim=1))
    bias = block_causal_bias(S, CASES[case]) if CASES[case] else None
    out = torch.nn.functional.scaled_dot_product_attention(q, k, v, attn_mask=bias)
    got = out.squeeze(0).transpose(0, 1).numpy()
    np.testing.assert_allclose(got, G[f"case{case}"], rtol=0, atol=1e-6)


def test_session_argument_errors():
    from diffusionhard_b200.session import evaluate_two_turn_mdlm_session

    with pytest.raises(ValueError, match="positive"):
        evaluate_two_turn_mdlm_session(samples=0)
    with pytest.raises(ValueError, match="multiples of 32"):
        evaluate_two_turn_mdlm_session(first_answer_tokens=16)
