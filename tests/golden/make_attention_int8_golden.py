#!/usr/bin/env python3
"""Golden outputs of the reference's packed INT8 attention screens
(src/diffusion_accel/attention_int8.py and
fixed_attention.sweep_qkv_weight_precision, imported in place):

  * dynamic_qk_fixed_pv_attention_q12 on the seeded qkv canvases of
    make_fixed_point_golden.fixed_point_cases (unit, hot, saturating);
  * _evaluate_with_fixed_maxima over EVALUATE_OPTIONS on the unit and hot
    canvases, calibrated on the unit canvas (so the hot one saturates);
  * screen_packed_int8_attention and sweep_qkv_weight_precision on the
    synthetic 12-block package of make_fixed_point_golden.sweep_package;
  * screen_packed_int8_attention_heldout and
    screen_packed_int8_attention_logits (LOGIT_OPTIONS) on that package with
    the full-size DDiT stand-in of diffusionhard_b200.model.build_standin
    (seed STANDIN_SEED) in place of the Hugging Face checkpoint, which the
    reference loads from its local cache (its loader is replaced for this
    run), on the HELDOUT_SEEDS canvases.
Integer outputs are stored as SHA-256 digests of their int64 arrays, metrics
as JSON.  Writes tests/golden/attention_int8_golden.json.

    python tests/golden/make_attention_int8_golden.py --reference <reference root>
"""

from __future__ import annotations

import argparse
import os
import json
import math
import sys
import tempfile
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent

EVALUATE_OPTIONS = {
    "default": {},
    "wide": {"qk_bits": 9, "pv_probability_levels": 255, "pv_value_bits": 9},
    "calibrated_q17": {"qk_multiplier_fraction_bits": 17},
    "dynamic_q17": {"qk_scale_mode": "dynamic-vector", "qk_multiplier_fraction_bits": 17},
    "dynamic_9bit": {"qk_scale_mode": "dynamic-vector", "qk_bits": 9},
    "sum_correction": {"pv_probability_sum_correction": True, "pv_probability_levels": 255},
    "fixed18_qk": {"quantize_qk": False},
    "fixed18_pv": {"quantize_pv": False, "qk_scale_mode": "dynamic-vector"},
}
LOGIT_OPTIONS = {
    "default": {},
    "dynamic_corrected": {"qk_scale_mode": "dynamic-vector", "qk_multiplier_fraction_bits": 17,
                          "pv_probability_sum_correction": True},
}
HELDOUT_SEEDS = [101, 202]
STANDIN_SEED = 5


def calibration_of(fa, qkv, cos, sin):
    """Per-head maxima of one canvas, as the reference's screens take them
    (attention_int8.py:564-583)."""
    import torch

    _, _, q12, k12, _ = fa.fixed_rotary_q12(qkv, cos, sin)
    v12 = torch.round(qkv.view(qkv.shape[0], 3, 12, 64)[:, 2].double() * 4096.0).to(torch.int64).clamp(
        -(1 << 17), (1 << 17) - 1)
    return [{"query_q12": max(1, int(q12[:, h].abs().max())), "key_q12": max(1, int(k12[:, h].abs().max())),
             "value_q12": max(1, int(v12[:, h].abs().max()))} for h in range(12)]


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--reference", default=os.environ.get("DH_REFERENCE_ROOT"),
                    required="DH_REFERENCE_ROOT" not in os.environ,
                    help="reference tree (default: $DH_REFERENCE_ROOT)")
    args = ap.parse_args()
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(HERE))
    sys.path.insert(0, str(Path(args.reference) / "src"))
    import torch
    from make_fixed_point_golden import digest, fixed_point_cases, strip, sweep_package

    from diffusion_accel import attention_int8 as ai  # reference, in place
    from diffusion_accel import fixed_attention as fa
    from diffusion_accel import mdlm
    from diffusionhard_b200.model import MDLMConfig, build_standin

    _, qkvs, cos, sin, _, _, _ = fixed_point_cases(torch)
    lut = torch.tensor([min(65535, round(math.exp(-i / 64.0) * 65536)) for i in range(1025)], dtype=torch.int64)
    out = {"dynamic": {}, "evaluate": {}}
    for name, qkv in qkvs.items():
        att, d = ai.dynamic_qk_fixed_pv_attention_q12(qkv, cos, sin)
        t = d["tensors"]
        out["dynamic"][name] = {k: digest(t[k]) for k in ("attention_q12", "scores_q10", "probabilities_q16",
                                                          "query_maxima_q12", "key_maxima_q12")}
        out["dynamic"][name]["attention"] = digest(att)
    calibration = calibration_of(fa, qkvs["unit"], cos, sin)
    out["calibration"] = calibration
    for name in ("unit", "hot"):
        for opt, kw in EVALUATE_OPTIONS.items():
            cand, base, heads = ai._evaluate_with_fixed_maxima(qkvs[name], cos, sin, calibration, lut, **kw)
            out["evaluate"]["%s_%s" % (name, opt)] = {"candidate": digest(cand), "baseline": digest(base),
                                                      "heads": heads}
    standin = build_standin(MDLMConfig(), seed=STANDIN_SEED)
    mdlm._load_mdlm_model = lambda **kwargs: standin  # no checkpoint in the cache: the stand-in instead
    with tempfile.TemporaryDirectory() as tmp:
        pkg = Path(tmp) / "pkg"
        out["sweep_package_files"] = sweep_package(pkg)
        out["screen"] = strip(ai.screen_packed_int8_attention(pkg))
        out["qkv_weight_precision"] = strip(fa.sweep_qkv_weight_precision(pkg, smoothquant_alphas=(None, 0.5)))
        out["heldout"] = ai.screen_packed_int8_attention_heldout(pkg, seeds=HELDOUT_SEEDS, device="cpu")
        out["logits"] = {k: ai.screen_packed_int8_attention_logits(pkg, seeds=HELDOUT_SEEDS, device="cpu", **kw)
                         for k, kw in LOGIT_OPTIONS.items()}
    (HERE / "attention_int8_golden.json").write_text(json.dumps(out, sort_keys=True) + "\n")
    print({k: (len(v) if isinstance(v, (dict, list)) else v) for k, v in out.items()})


if __name__ == "__main__":
    main()
