"""The numpy restatement of the packed INT8 attention candidates
(oracle/attention_int8_oracle.py) pinned to the reference's own outputs
(tests/golden/make_attention_int8_golden.py), and the argument checks of the
drop-ins, which run before any device work."""

import hashlib
import json
import sys

import numpy as np
import pytest

from conftest import GOLDEN, ROOT

sys.path.insert(0, str(GOLDEN))
sys.path.insert(0, str(ROOT))
from make_attention_int8_golden import EVALUATE_OPTIONS  # noqa: E402
from make_fixed_point_golden import fixed_point_cases  # noqa: E402
from oracle import attention_int8_oracle as oracle  # noqa: E402

GJ = json.loads((GOLDEN / "attention_int8_golden.json").read_text())


def _digest(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(np.asarray(a).astype("<i8")).tobytes()).hexdigest()


@pytest.fixture(scope="module")
def cases():
    import torch

    _, qkvs, cos, sin, _, _, _ = fixed_point_cases(torch)
    return {k: v.numpy() for k, v in qkvs.items()}, cos.numpy(), sin.numpy()


@pytest.mark.parametrize("name", ["unit", "hot", "saturating"])
def test_oracle_dynamic_matches_reference(cases, name):
    qkvs, cos, sin = cases
    r = oracle.packed_attention(qkvs[name], cos, sin, qk_mode="dynamic", qk_levels=127, qk_frac=17)
    g = GJ["dynamic"][name]
    assert _digest(r["attention"]) == g["attention"]
    assert _digest(r["attention"].reshape(-1, 12, 64)) == g["attention_q12"]
    for key in ("scores_q10", "probabilities_q16", "query_maxima_q12", "key_maxima_q12"):
        assert _digest(r[key]) == g[key], key


def test_oracle_calibration_matches_reference(cases):
    qkvs, cos, sin = cases
    assert oracle.head_maxima(qkvs["unit"], cos, sin) == GJ["calibration"]


@pytest.mark.parametrize("opt", sorted(EVALUATE_OPTIONS))
@pytest.mark.parametrize("name", ["unit", "hot"])
def test_oracle_evaluate_matches_reference(cases, name, opt):
    qkvs, cos, sin = cases
    r = oracle.packed_attention(qkvs[name], cos, sin, calibration=GJ["calibration"],
                                **oracle.evaluate_options(EVALUATE_OPTIONS[opt]))
    g = GJ["evaluate"]["%s_%s" % (name, opt)]
    assert _digest(r["attention"]) == g["candidate"]
    assert _digest(r["baseline"]) == g["baseline"]
    agree = (r["scores_q10"].argmax(-1) == r["baseline_scores"].argmax(-1)).mean(-1)
    assert [h["score_argmax_agreement_vs_fixed18"] for h in g["heads"]] == agree.tolist()


def test_argument_errors():
    import torch

    from diffusionhard_b200 import attention_int8 as ai
    from diffusionhard_b200.fixed_point import sweep_qkv_weight_precision

    qkv, cs = torch.zeros(64, 2304), torch.zeros(64, 32)
    cal = GJ["calibration"]
    lut = torch.zeros(1025, dtype=torch.int64)
    with pytest.raises(ValueError, match="Q17 multipliers"):
        ai.dynamic_qk_fixed_pv_attention_q12(qkv, cs, cs, qk_multiplier_fraction_bits=24)
    for kw, msg in (({"qk_bits": 7}, "qk_bits"), ({"qk_scale_mode": "x"}, "qk_scale_mode"),
                    ({"qk_multiplier_fraction_bits": 20}, "fraction_bits"),
                    ({"pv_probability_levels": 63}, "pv_probability_levels"), ({"pv_value_bits": 10}, "pv_value_bits")):
        with pytest.raises(ValueError, match=msg):
            ai._evaluate_with_fixed_maxima(qkv, cs, cs, cal, lut, **kw)
    with pytest.raises(ValueError, match="held-out seed"):
        ai.screen_packed_int8_attention_heldout("unused", seeds=[])
    with pytest.raises(ValueError, match="logit-screen seed"):
        ai.screen_packed_int8_attention_logits("unused", seeds=[])
    with pytest.raises(ValueError, match="at least one attention matrix phase"):
        ai.screen_packed_int8_attention_logits("unused", quantize_qk=False, quantize_pv=False)
    with pytest.raises(ValueError, match="weight_bits"):
        sweep_qkv_weight_precision("unused", weight_bits=(4,))
    with pytest.raises(ValueError, match="smoothquant_alphas"):
        sweep_qkv_weight_precision("unused", smoothquant_alphas=(1.5,))
