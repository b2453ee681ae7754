#!/usr/bin/env python3
"""Golden fixtures for the model path, produced by the reference's own Python.

Runs, in place from the reference tree (its src/ directory):
  * hardware_package.folded_mdlm_forward on the seeded stand-in DDiT built by
    diffusionhard_b200.model.build_standin (HF attribute names; 2 blocks,
    vocabulary 1000) -> fp32 logits;
  * fixed_mlp.quantized_linear (bits 8, per-token activations, SmoothQuant
    alpha 0.5) on a seeded activation / weight pair -> output and metrics;
  * prefix_drift._apply_rotary on seeded vectors;
  * prefix_drift.tensor_drift_metrics on a seeded pair.
Writes tests/golden/model_golden.npz (+ .json for the scalar metrics).

    python tests/golden/make_model_golden.py --reference <reference root>
"""

from __future__ import annotations

import argparse
import os
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

SMALL = dict(vocab_size=1000, mask_token_id=999, blocks=2)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--reference", default=os.environ.get("DH_REFERENCE_ROOT"),
                    required="DH_REFERENCE_ROOT" not in os.environ,
                    help="reference tree (default: $DH_REFERENCE_ROOT)")
    args = ap.parse_args()
    sys.path.insert(0, str(Path(args.reference) / "src"))
    import torch

    from diffusion_accel import fixed_mlp, hardware_package, prefix_drift  # reference, in place
    from diffusionhard_b200.model import MDLMConfig, build_standin

    torch.manual_seed(0)
    cfg = MDLMConfig(**SMALL)
    model = build_standin(cfg, seed=0)
    g = torch.Generator().manual_seed(5)
    ids = torch.randint(0, cfg.mask_token_id + 1, (1, 32), generator=g)
    ids[0, ::4] = cfg.mask_token_id
    with torch.no_grad():
        logits = hardware_package.folded_mdlm_forward(model, ids, "cpu")

    act = torch.randn((64, 768), generator=g) * 0.7
    act[:, 5] *= 20  # an outlier channel, the SmoothQuant case
    weight = torch.randn((256, 768), generator=g) * 0.02
    bias = torch.randn(256, generator=g) * 0.01
    out, metrics = fixed_mlp.quantized_linear(act, weight, bias, 8, "token", smoothquant_alpha=0.5)

    vec = torch.randn((2, 16, 12, 64), generator=g)
    positions = torch.arange(100, 116)
    inv_freq = model.backbone.rotary_emb.inv_freq
    rotated = prefix_drift._apply_rotary(vec, positions, inv_freq)

    a = torch.randn((4, 33), generator=g)
    b = a + 1e-3 * torch.randn((4, 33), generator=g)
    drift = prefix_drift.tensor_drift_metrics(a, b)

    np.savez_compressed(HERE / "model_golden.npz", ids=ids.numpy(), logits=logits.numpy(),
                        act=act.numpy(), weight=weight.numpy(), bias=bias.numpy(), ql_out=out.numpy(),
                        vec=vec.numpy(), positions=positions.numpy(), rotated=rotated.numpy(),
                        drift_a=a.numpy(), drift_b=b.numpy())
    (HERE / "model_golden.json").write_text(json.dumps({
        "config": SMALL,
        "quantized_linear_metrics": {k: v for k, v in metrics.items() if not isinstance(v, str)},
        "drift_metrics": drift,
    }, indent=1, default=float))
    print("logits", tuple(logits.shape), "ql", tuple(out.shape))


if __name__ == "__main__":
    main()
