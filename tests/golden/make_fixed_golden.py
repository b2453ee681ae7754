#!/usr/bin/env python3
"""Golden fixtures for the RTL integer MLP arithmetic, produced by the
reference's own Python (src/diffusion_accel/fixed_mlp.py, imported in place):

  * hardware_requantized_linear on the reference's own unit cases
    (tests/test_fixed_mlp.py:91-146) and on an MLP-sized case: 64 tokens of
    seeded N(0, 1) activations through a 768 -> 3072 up projection (token
    granularity, alpha 0.75, 16-bit Q5.10 output), the Q5.10 GELU lookup, and a
    3072 -> 768 down projection (24-bit output) -- the chain of
    validate_hardware_fixed_mlp (fixed_mlp.py:918-1030) with seeded weights;
  * factorize_up_requant_scales on that case's token / output scales, and the
    factorised requantisation of its up projection;
  * hardware_gelu_q10 on every input in [-9000, 9000].
Inputs are regenerated from the seeds by tests/test_fixed_mlp_*.py (fixed_case
below); only outputs are stored.  Writes tests/golden/fixed_golden.npz (+ .json).

    python tests/golden/make_fixed_golden.py --reference <reference root>
"""

from __future__ import annotations

import argparse
import os
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def fixed_case(torch):
    """The MLP-sized case's inputs (seed 5): activations [64, 768] ~ N(0, 1),
    up W [3072, 768] and down W [768, 3072] ~ N(0, 0.02), biases ~ N(0, 0.02)."""
    g = torch.Generator().manual_seed(5)
    act = torch.randn((64, 768), generator=g)
    w_up = torch.randn((3072, 768), generator=g) * 0.02
    b_up = torch.randn(3072, generator=g) * 0.02
    w_down = torch.randn((768, 3072), generator=g) * 0.02
    b_down = torch.randn(768, generator=g) * 0.02
    return act, w_up, b_up, w_down, b_down


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--reference", default=os.environ.get("DH_REFERENCE_ROOT"),
                    required="DH_REFERENCE_ROOT" not in os.environ,
                    help="reference tree (default: $DH_REFERENCE_ROOT)")
    args = ap.parse_args()
    sys.path.insert(0, str(Path(args.reference) / "src"))
    import torch

    from diffusion_accel import fixed_mlp  # reference, in place

    out: dict = {}
    meta: dict = {}
    # unit cases (tests/test_fixed_mlp.py:91-146)
    small_a = torch.tensor([[0.25, -0.5, 0.75]])
    small_w = torch.tensor([[0.5, -0.25, 0.75], [-0.5, 0.5, 0.25]])
    small_b = torch.tensor([0.125, -0.25])
    _, q, m = fixed_mlp.hardware_requantized_linear(small_a, small_w, small_b, activation_granularity="token",
                                                    smoothquant_alpha=0.5, output_width=16)
    out["small_q"] = q.numpy().astype(np.int64)
    meta["small"] = m
    gran_a = torch.tensor([[0.01, -0.02], [10.0, -20.0]])
    gran_w = torch.tensor([[0.5, -0.25]])
    gran_b = torch.tensor([0.0])
    for name, gran, width in (("token", "token", 16), ("tensor", "tensor", 24)):
        _, q, m = fixed_mlp.hardware_requantized_linear(gran_a, gran_w, gran_b, activation_granularity=gran,
                                                        smoothquant_alpha=0.5, output_width=width)
        out[f"gran_{name}_q"] = q.numpy().astype(np.int64)
        meta[f"gran_{name}"] = m

    # MLP-sized chain
    act, w_up, b_up, w_down, b_down = fixed_case(torch)
    _, up_q, up_m = fixed_mlp.hardware_requantized_linear(act, w_up, b_up, activation_granularity="token",
                                                          smoothquant_alpha=0.75, output_width=16)
    gelu, gelu_q = fixed_mlp.hardware_gelu_q10(up_q)
    _, down_q, down_m = fixed_mlp.hardware_requantized_linear(gelu, w_down, b_down, activation_granularity="token",
                                                              smoothquant_alpha=0.75, output_width=24)
    out["up_q"] = up_q.numpy().astype(np.int16)
    out["gelu_q"] = gelu_q.numpy().astype(np.int16)
    out["down_q"] = down_q.numpy().astype(np.int32)
    meta["up"] = up_m
    meta["down"] = down_m

    # factorised multipliers from the up projection's token / output scales
    amax = act.abs().amax(dim=0).clamp_min(1e-8)
    wmax = w_up.abs().amax(dim=0).clamp_min(1e-8)
    s = (amax.pow(0.75) / wmax.pow(0.25)).clamp_min(1e-8)
    aq, a_scale = fixed_mlp._quantize_symmetric(act / s[None, :], 8, "token")
    wq, w_scale = fixed_mlp._quantize_weight_per_output(w_up * s[None, :], 8)
    mult, tensors, fm = fixed_mlp.factorize_up_requant_scales(a_scale, w_scale)
    acc = torch._int_mm(aq.contiguous(), wq.t().contiguous()).to(torch.int64)
    prod = acc * mult
    rounded = torch.sign(prod) * ((prod.abs() + (1 << 19)) >> 20)
    bias_q = torch.round(b_up.double() * 1024).to(torch.int64)
    fact_q = (rounded + bias_q[None, :]).clamp(-(1 << 15), (1 << 15) - 1)
    out["token_factor"] = tensors["token_factor"].numpy()
    out["output_factor"] = tensors["output_factor"].numpy()
    out["factorized_q"] = fact_q.numpy().astype(np.int16)
    meta["factorize"] = fm
    meta["factorized_multiplier_sum"] = int(mult.sum().item())

    # Q5.10 GELU lookup on every input in [-9000, 9000]
    xs = torch.arange(-9000, 9001, dtype=torch.int64)
    _, lut_q = fixed_mlp.hardware_gelu_q10(xs)
    out["gelu_lut_q"] = lut_q.numpy().astype(np.int16)

    np.savez_compressed(HERE / "fixed_golden.npz", **out)
    (HERE / "fixed_golden.json").write_text(json.dumps(meta, indent=1, sort_keys=True) + "\n")
    print({k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main()
