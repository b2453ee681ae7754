"""RTL integer MLP arithmetic on the GPU, bit-exact against the reference's
own outputs (tests/golden/make_fixed_golden.py): the integer requantisation
of W8A8 MACs (hardware_requantized_linear, fixed_mlp.py:139-224) on the
reference's unit cases and an MLP-sized up -> GELU -> down chain, the
factorised-multiplier form (fixed_mlp.py:327-392) and the Q5.10 GELU lookup
(fixed_mlp.py:227-247)."""

import json
import sys

import numpy as np
import pytest

from conftest import GOLDEN

sys.path.insert(0, str(GOLDEN))
from make_fixed_golden import fixed_case  # noqa: E402

pytestmark = pytest.mark.gpu

G = np.load(GOLDEN / "fixed_golden.npz")
GJ = json.loads((GOLDEN / "fixed_golden.json").read_text())


def _check_metrics(got, ref):
    for k, v in ref.items():
        if isinstance(v, str):
            assert got[k] == v, k
        elif isinstance(v, int):
            assert got[k] == v, k
        else:
            assert got[k] == pytest.approx(v, rel=1e-6, abs=1e-12), k


def test_reference_unit_cases(cuda):
    torch = cuda
    from diffusionhard_b200.fixed_mlp import hardware_requantized_linear

    a = torch.tensor([[0.25, -0.5, 0.75]])
    w = torch.tensor([[0.5, -0.25, 0.75], [-0.5, 0.5, 0.25]])
    b = torch.tensor([0.125, -0.25])
    out, q, m = hardware_requantized_linear(a, w, b, activation_granularity="token", smoothquant_alpha=0.5,
                                            output_width=16)
    assert q.dtype == torch.int64 and np.array_equal(q.numpy(), G["small_q"])
    _check_metrics(m, GJ["small"])
    torch.testing.assert_close(out, torch.nn.functional.linear(a, w, b), rtol=0.02, atol=0.02)
    ga = torch.tensor([[0.01, -0.02], [10.0, -20.0]])
    gw = torch.tensor([[0.5, -0.25]])
    gb = torch.tensor([0.0])
    for name, gran, width in (("token", "token", 16), ("tensor", "tensor", 24)):
        _, q, m = hardware_requantized_linear(ga, gw, gb, activation_granularity=gran, smoothquant_alpha=0.5,
                                              output_width=width)
        assert np.array_equal(q.numpy(), G[f"gran_{name}_q"]), name
        _check_metrics(m, GJ[f"gran_{name}"])


def test_mlp_chain_bit_exact(cuda):
    torch = cuda
    from diffusionhard_b200.fixed_mlp import hardware_gelu_q10, hardware_requantized_linear

    act, w_up, b_up, w_down, b_down = fixed_case(torch)
    _, up_q, up_m = hardware_requantized_linear(act, w_up, b_up, activation_granularity="token",
                                                smoothquant_alpha=0.75, output_width=16)
    assert np.array_equal(up_q.numpy(), G["up_q"].astype(np.int64))
    _check_metrics(up_m, GJ["up"])
    gelu, gelu_q = hardware_gelu_q10(up_q)
    assert np.array_equal(gelu_q.numpy(), G["gelu_q"].astype(np.int64))
    _, down_q, down_m = hardware_requantized_linear(gelu, w_down, b_down, activation_granularity="token",
                                                    smoothquant_alpha=0.75, output_width=24)
    assert np.array_equal(down_q.numpy(), G["down_q"].astype(np.int64))
    _check_metrics(down_m, GJ["down"])


def test_factorized_requantisation_bit_exact(cuda):
    torch = cuda
    from diffusionhard_b200.fixed_mlp import (_quantize_symmetric, _quantize_weight_per_output,
                                              factorize_up_requant_scales, requantized_linear_factorized)

    act, w_up, b_up, _, _ = fixed_case(torch)
    s = (act.abs().amax(dim=0).clamp_min(1e-8).pow(0.75) / w_up.abs().amax(dim=0).clamp_min(1e-8).pow(0.25)
         ).clamp_min(1e-8)
    aq, a_scale = _quantize_symmetric(act / s[None, :], 8, "token")
    wq, w_scale = _quantize_weight_per_output(w_up * s[None, :], 8)
    _, tensors, metrics = factorize_up_requant_scales(a_scale, w_scale)
    bias_q = torch.round(b_up.double() * 1024).to(torch.int64)
    q, stats = requantized_linear_factorized(aq, wq, tensors["token_factor"], tensors["output_factor"],
                                             metrics["factor_shift"], bias_q, output_width=16)
    assert np.array_equal(q.numpy(), G["factorized_q"].astype(np.int64))
    # same int8 operands as the up projection: same accumulator range
    assert stats[0] == GJ["up"]["accumulator_min"] and stats[1] == GJ["up"]["accumulator_max"]
    tf = tensors["token_factor"].long()
    of = tensors["output_factor"].long()
    shift = metrics["factor_shift"]
    assert stats[3] == int(((tf[:, None] * of[None, :] + (1 << (shift - 1))) >> shift).max())


def test_gelu_lookup_all_inputs(cuda):
    torch = cuda
    from diffusionhard_b200.fixed_mlp import hardware_gelu_q10

    xs = torch.arange(-9000, 9001, dtype=torch.int64)
    f, q = hardware_gelu_q10(xs)
    assert np.array_equal(q.numpy(), G["gelu_lut_q"].astype(np.int64))
    assert torch.equal(f, q.float() / 1024.0)


def test_requant_argument_errors(cuda):
    torch = cuda
    from diffusionhard_b200 import _lib
    from diffusionhard_b200.fixed_mlp import hardware_requantized_linear

    with pytest.raises(ValueError, match="output width"):
        hardware_requantized_linear(torch.ones(1, 4), torch.ones(2, 4), torch.zeros(2),
                                    activation_granularity="token", smoothquant_alpha=0.5, output_width=10)
    with pytest.raises(ValueError, match="multiplier exceeds"):
        hardware_requantized_linear(torch.ones(1, 4) * 1e6, torch.ones(2, 4) * 1e6, torch.zeros(2),
                                    activation_granularity="token", smoothquant_alpha=0.5, output_width=16,
                                    multiplier_bits=4)
    assert _lib.raw("dh_gemm_i8_requant", None, None, 1, 1, 16, 0, None, 1, None, None, None, 0, None, 20, 10, 16,
                    None, None, None) == 100
