#!/usr/bin/env python3
"""Golden hardware package written by the reference's own package code
(src/diffusion_accel/hardware_package.py, imported in place) for a tiny
seeded DDiT stand-in with the HF attribute names (package_standin below:
d=64, 2 heads x 32, MLP 256, 2 blocks, vocabulary 101, adaLN biases ~
N(0, 0.3) so that the fold matters):

  * folded_fp16_weights.safetensors from _export_folded_weights,
  * folded_fp16_weights.bin from _write_aligned_weight_binary,
  * golden_tensors.safetensors with the input ids, the reference's
    folded_mdlm_forward logits and top-1 ids, and its captured per-block
    tensors that the fixed-point MLP validation reads (norm2_unaffine,
    mlp_up, gelu, mlp_down, after_attention, output),
  * manifest.json in the layout of export_mdlm_hardware_package, whose
    constant-fold validation compares folded_mdlm_forward with the
    stand-in's unfolded forward (diffusionhard_b200.model.ddit_forward),
and package_golden.json with validate_mdlm_hardware_package's verdicts on
that package, on a copy with one flipped weight byte, and on the package
that diffusionhard_b200.checkpoint.export_hardware_package writes for the
same stand-in, plus the reference's validate_hardware_fixed_mlp reports on
the package's two blocks (FIXED_MLP_CASES).  Writes tests/golden/package/ and tests/golden/package_golden.json.

    python tests/golden/make_package_golden.py --reference <reference root>
"""

from __future__ import annotations

import argparse
import os
import json
import shutil
import sys
import tempfile
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
MLP_GOLDENS = (".norm2_unaffine", ".mlp_up", ".gelu", ".mlp_down", ".after_attention", ".output")
FIXED_MLP_CASES = [(0, "token", None, 0.75), (1, "token", None, 0.5), (0, "tensor", "token", 0.5),
                   (1, "tensor", None, 0.75)]


def package_config():
    from diffusionhard_b200.model import MDLMConfig

    return MDLMConfig(vocab_size=101, mask_token_id=100, hidden=64, heads=2, head_dim=32, mlp=256, blocks=2,
                      max_positions=128)


def package_standin():
    """The tiny stand-in (seed 3) with adaLN biases ~ N(0, 0.3) and LayerNorm
    weights 1 + N(0, 0.1) (generator seed 9)."""
    import torch

    from diffusionhard_b200.model import build_standin

    m = build_standin(package_config(), seed=3)
    g = torch.Generator().manual_seed(9)
    with torch.no_grad():
        for blk in m.backbone.blocks:
            blk.adaLN_modulation.bias.copy_(torch.randn(blk.adaLN_modulation.bias.shape, generator=g) * 0.3)
            blk.norm1.weight.copy_(1 + torch.randn(blk.norm1.weight.shape, generator=g) * 0.1)
            blk.norm2.weight.copy_(1 + torch.randn(blk.norm2.weight.shape, generator=g) * 0.1)
        ol = m.backbone.output_layer
        ol.adaLN_modulation.bias.copy_(torch.randn(ol.adaLN_modulation.bias.shape, generator=g) * 0.3)
        ol.norm_final.weight.copy_(1 + torch.randn(ol.norm_final.weight.shape, generator=g) * 0.1)
    return m


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--reference", default=os.environ.get("DH_REFERENCE_ROOT"),
                    required="DH_REFERENCE_ROOT" not in os.environ,
                    help="reference tree (default: $DH_REFERENCE_ROOT)")
    args = ap.parse_args()
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(Path(args.reference) / "src"))
    import torch
    from safetensors.torch import save_file

    from diffusion_accel import hardware_package as hp  # reference, in place
    from diffusionhard_b200 import checkpoint
    from diffusionhard_b200.model import ddit_forward, fold

    model = package_standin()
    cfg = package_config()
    mask = cfg.mask_token_id
    ids = hp.deterministic_hardware_input(64, cfg.vocab_size, mask)
    input_ids = torch.tensor([ids], dtype=torch.long)
    captured = {}
    with torch.no_grad():
        folded_logits = hp.folded_mdlm_forward(model, input_ids, "cpu", captured)
        unfolded = ddit_forward(model, input_ids.numpy())
        weights = hp._export_folded_weights(model, hp._constant_condition(model, "cpu"))
    diff = (unfolded - folded_logits).abs()
    fs, us = folded_logits.clone(), unfolded.clone()
    fs[..., mask] = -torch.inf
    us[..., mask] = -torch.inf
    f_top1, u_top1 = fs.argmax(-1), us.argmax(-1)
    goldens = {"input.ids": input_ids.to(torch.int32), "folded.final.logits": folded_logits.contiguous(),
               "folded.top1": f_top1.to(torch.int32), "reference.top1": u_top1.to(torch.int32)}
    for b in range(cfg.blocks):
        for suffix in MLP_GOLDENS:
            name = "folded.block_%02d%s" % (b, suffix)
            goldens[name] = captured[name]
    out = HERE / "package"
    if out.exists():
        shutil.rmtree(out)
    out.mkdir()
    gp, wp, bp = out / "golden_tensors.safetensors", out / "folded_fp16_weights.safetensors", \
        out / "folded_fp16_weights.bin"
    save_file(goldens, gp)
    save_file(weights, wp)
    layout = hp._write_aligned_weight_binary(weights, bp)
    agreement = float(u_top1.eq(f_top1).float().mean().item())
    manifest = {
        "schema_version": hp.PACKAGE_SCHEMA_VERSION,
        "source_checkpoint": {"model_id": "tiny seeded stand-in (tests/golden/make_package_golden.py)"},
        "fixed_graph": {"canvas_tokens": 64, "batch_size": 1, "hidden_size": cfg.hidden, "blocks": cfg.blocks,
                        "heads": cfg.heads, "vocabulary_size": cfg.vocab_size, "mask_token_id": mask,
                        "time_conditioning": False},
        "input": {"construction": "position*7919+17 modulo mask ID; positions not divisible by three are masked",
                  "visible_tokens": sum(v != mask for v in ids), "masked_tokens": sum(v == mask for v in ids),
                  "reference_top1_token_ids": u_top1[0].tolist(), "reference_top1_decoded_text": None},
        "constant_fold_validation": {
            "folded_vs_reference_max_abs_error": float(diff.max().item()),
            "folded_vs_reference_mean_abs_error": float(diff.mean().item()),
            "top1_agreement": agreement, "acceptance_max_abs_error": 1e-4,
            "passed": float(diff.max().item()) <= 1e-4 and agreement == 1.0},
        "goldens": hp._tensor_manifest(goldens),
        "weights": hp._tensor_manifest(weights),
        "weight_binary_layout": layout,
        "files": {p.name: {"bytes": p.stat().st_size, "sha256": hp._sha256(p)} for p in (gp, wp, bp)},
        "device_used_for_reference": "cpu",
    }
    (out / "manifest.json").write_text(json.dumps(manifest, indent=2, sort_keys=True) + "\n", encoding="utf-8")

    verdicts = {"reference_package": hp.validate_mdlm_hardware_package(out)}
    with tempfile.TemporaryDirectory() as tmp:
        bad = Path(tmp) / "bad"
        shutil.copytree(out, bad)
        raw = bytearray((bad / "folded_fp16_weights.bin").read_bytes())
        raw[4096 + 10] ^= 0x40
        (bad / "folded_fp16_weights.bin").write_bytes(bytes(raw))
        verdicts["flipped_byte"] = hp.validate_mdlm_hardware_package(bad)
        ours = Path(tmp) / "ours"
        folded = fold(model)
        folded.config = cfg
        checkpoint.export_hardware_package(folded, ours, unfolded_logits=unfolded)
        verdicts["our_export"] = hp.validate_mdlm_hardware_package(ours)
        ours_manifest = json.loads((ours / "manifest.json").read_text())
        verdicts["our_export_weights_sha256"] = ours_manifest["files"]["folded_fp16_weights.bin"]["sha256"]
    from diffusion_accel import fixed_mlp  # reference, in place

    verdicts["fixed_mlp"] = []
    for block, gran, down_gran, alpha in FIXED_MLP_CASES:
        r = fixed_mlp.validate_hardware_fixed_mlp(out, block=block, activation_granularity=gran,
                                                  down_activation_granularity=down_gran, smoothquant_alpha=alpha)
        r.pop("package_dir")
        verdicts["fixed_mlp"].append(r)
    for v in verdicts.values():
        if isinstance(v, dict):
            v.pop("package_dir", None)
    (HERE / "package_golden.json").write_text(json.dumps(verdicts, indent=1, sort_keys=True) + "\n")
    print({k: (v["passed"] if isinstance(v, dict) else len(v) if isinstance(v, list) else v)
           for k, v in verdicts.items()})


if __name__ == "__main__":
    main()
