"""Host side of the RTL integer MLP arithmetic against the reference's own
outputs (fixtures from tests/golden/make_fixed_golden.py): the factorised
multipliers and the Q5.10 GELU table.  No GPU."""

import json
import sys

import numpy as np
import pytest

from conftest import GOLDEN

sys.path.insert(0, str(GOLDEN))
from make_fixed_golden import fixed_case  # noqa: E402

from diffusionhard_b200.fixed_mlp import (_quantize_symmetric, _quantize_weight_per_output,  # noqa: E402
                                          factorize_up_requant_scales, gelu_q10_table)

G = np.load(GOLDEN / "fixed_golden.npz")
GJ = json.loads((GOLDEN / "fixed_golden.json").read_text())


def _up_scales():
    import torch

    act, w_up, _, _, _ = fixed_case(torch)
    s = (act.abs().amax(dim=0).clamp_min(1e-8).pow(0.75) / w_up.abs().amax(dim=0).clamp_min(1e-8).pow(0.25)
         ).clamp_min(1e-8)
    _, a_scale = _quantize_symmetric(act / s[None, :], 8, "token")
    _, w_scale = _quantize_weight_per_output(w_up * s[None, :], 8)
    return a_scale, w_scale


def test_factorized_multipliers_match_reference():
    a_scale, w_scale = _up_scales()
    mult, tensors, metrics = factorize_up_requant_scales(a_scale, w_scale)
    assert np.array_equal(tensors["token_factor"].numpy(), G["token_factor"])
    assert np.array_equal(tensors["output_factor"].numpy(), G["output_factor"])
    assert int(mult.sum().item()) == GJ["factorized_multiplier_sum"]
    for k, v in GJ["factorize"].items():
        assert metrics[k] == pytest.approx(v, rel=1e-12), k


def test_factorization_width_errors():
    import torch

    with pytest.raises(ValueError, match="token factor"):
        factorize_up_requant_scales(torch.tensor([1.0]), torch.tensor([0.001]))
    with pytest.raises(ValueError, match="exceed combined"):
        factorize_up_requant_scales(torch.tensor([0.01]), torch.tensor([0.01]), token_fraction_bits=10,
                                    output_fraction_bits=10)


def test_gelu_table_matches_reference_lookup():
    table = gelu_q10_table()
    assert len(table) == 1024
    xs = np.arange(-9000, 9001)
    ref = G["gelu_lut_q"].astype(np.int64)
    for a in range(1024):
        x = -8192 + 16 * a
        assert table[a] == ref[x + 9000], a


def test_host_quantisation_matches_reference_scales():
    a_scale, w_scale = _up_scales()
    assert float(a_scale.min()) == pytest.approx(GJ["up"]["activation_scale_min"], rel=1e-7)
    assert float(a_scale.max()) == pytest.approx(GJ["up"]["activation_scale_max"], rel=1e-7)
    assert float(w_scale.min()) == pytest.approx(GJ["up"]["weight_scale_min"], rel=1e-7)
