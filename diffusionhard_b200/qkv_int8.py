"""Error-propagating screen of a SmoothQuant INT8 QKV projection, with the
integer stages on the GPU.

Drop-in for ``screen_qkv_int8_logits`` (src/diffusion_accel/qkv_int8.py:
14-257): every block's fixed LayerNorm output (Q5.12) goes through the fixed
QKV projection -- INT16 weights for the baseline, INT8 weights with
SmoothQuant scales calibrated on the package's captured canvas for the
candidate -- and the retained dynamic-INT8-QK / fixed18-PV attention, inside
an otherwise floating-point folded forward, and the masked positions' logits
are compared.  Same arguments, errors and report.  The integer stages are
``fixed_point.fixed_layer_norm_q12`` / ``fixed_qkv_projection_q12``
(dh_fixed_layer_norm_q12, dh_fixed_wide_linear) and
``attention_int8.dynamic_qk_fixed_pv_attention_q12``
(dh_fixed_rotary_q12, dh_packed_int8_attention_q12); the float model runs
in ``model.fp32_forward`` on the host, given as ``model`` where the
reference loads its checkpoint from the local Hugging Face cache.
"""

from __future__ import annotations

import statistics
from pathlib import Path
from typing import Any, Dict, Optional, Sequence

from .attention_int8 import _folded, _half_masked_canvas, dynamic_qk_fixed_pv_attention_q12
from .fixed_mlp import _package_tensors
from .fixed_point import fixed_layer_norm_q12, fixed_qkv_projection_q12

DEFAULT_MODEL_ID = "kuleshov-group/mdlm-owt"
DEFAULT_REVISION = "d0958fa851335ece6c15260ce0025f030673c0fb"


def screen_qkv_int8_logits(package_dir: Any, *, seeds: Optional[Sequence[int]] = None, device: str = "auto",
                           smoothquant_alpha: float = 0.25, model: Any = None) -> Dict[str, object]:
    """Calibrated INT8 QKV against INT16 QKV through all twelve blocks
    (qkv_int8.py:14-257)."""
    import torch
    import torch.nn.functional as F

    from .model import fp32_forward

    if not 0.0 <= smoothquant_alpha <= 1.0:
        raise ValueError("smoothquant_alpha must be between zero and one")
    selected = [101, 202, 303, 404, 505] if seeds is None else list(seeds)
    if not selected:
        raise ValueError("at least one logit-screen seed is required")
    package_dir = Path(package_dir)
    golden_names = ["folded.embedding"] + ["folded.block_%02d.output" % b for b in range(12)]
    weight_names = []
    for b in range(12):
        weight_names += ["block_%02d.qkv.weight" % b, "block_%02d.qkv.bias" % b]
    goldens = _package_tensors(package_dir / "golden_tensors.safetensors", golden_names)
    tables = _package_tensors(package_dir / "folded_fp16_weights.safetensors",
                              ["rotary.cos", "rotary.sin", *weight_names])
    cosine, sine = tables["rotary.cos"].float(), tables["rotary.sin"].float()
    dev = "cuda" if device == "auto" else device

    # SmoothQuant scales of each block from the package's captured canvas
    # (qkv_int8.py:64-92)
    scales, calibration_metrics = [], []
    for b in range(12):
        residual = goldens["folded.embedding"][0] if b == 0 else goldens["folded.block_%02d.output" % (b - 1)][0]
        _, normalized_q12, _ = fixed_layer_norm_q12(residual, device=dev)
        _, _, details = fixed_qkv_projection_q12(normalized_q12, tables["block_%02d.qkv.weight" % b],
                                                 tables["block_%02d.qkv.bias" % b], weight_bits=8,
                                                 smoothquant_alpha=smoothquant_alpha, device=dev)
        scales.append(details["tensors"]["smoothquant_input_scales"])
        calibration_metrics.append({
            "block": b,
            "minimum_scale": float(scales[-1].min().item()),
            "maximum_scale": float(scales[-1].max().item()),
            "activation_saturation_fraction": details["metrics"]["smoothed_activation_saturation_fraction"],
        })

    folded = _folded(model)
    mask = int(folded.config.vocab_size) - 1
    head_w = torch.from_numpy(folded.head.weight)
    head_b = torch.from_numpy(folded.head.bias)

    def fixed_qkv_attention(weight_bits: int):
        def attention(block: int, normalized: Any, qkv: Any) -> Any:
            normalized_q12 = torch.round(normalized.detach().cpu().double() * 4096.0).to(torch.int64).clamp(
                -(1 << 17), (1 << 17) - 1)
            _, qkv_q12, _ = fixed_qkv_projection_q12(
                normalized_q12[0], tables["block_%02d.qkv.weight" % block], tables["block_%02d.qkv.bias" % block],
                weight_bits=weight_bits, smoothquant_scales=scales[block] if weight_bits == 8 else None, device=dev)
            attention_q12, _ = dynamic_qk_fixed_pv_attention_q12(qkv_q12.float() / 4096.0, cosine, sine, device=dev)
            return attention_q12.to(torch.float32)[None] / 4096.0

        return attention

    samples = []
    with torch.inference_mode():
        for seed in selected:
            ids = _half_masked_canvas(seed, mask).numpy()
            base_h = torch.from_numpy(fp32_forward(folded, ids, attention=fixed_qkv_attention(16)))
            cand_h = torch.from_numpy(fp32_forward(folded, ids, attention=fixed_qkv_attention(8)))
            baseline = F.linear(base_h, head_w, head_b)[0, 1::2].float()
            candidate = F.linear(cand_h, head_w, head_b)[0, 1::2].float()
            baseline[:, mask] = -torch.inf
            candidate[:, mask] = -torch.inf
            fb = torch.where(torch.isfinite(baseline), baseline, torch.zeros_like(baseline))
            fc = torch.where(torch.isfinite(candidate), candidate, torch.zeros_like(candidate))
            diff = fc - fb
            bp = torch.log_softmax(baseline, dim=-1).exp()
            cp = torch.log_softmax(candidate, dim=-1).exp()
            tv = 0.5 * (bp - cp).abs().sum(dim=-1)
            top1 = baseline.argmax(dim=-1).eq(candidate.argmax(dim=-1))
            samples.append({
                "seed": seed,
                "masked_positions": 32,
                "top1_matches": int(top1.sum().item()),
                "top1_agreement": float(top1.float().mean().item()),
                "logit_cosine_similarity": float(F.cosine_similarity(fb.flatten(), fc.flatten(), dim=0).item()),
                "normalized_logit_rmse": float((diff.square().mean().sqrt() / fb.square().mean().sqrt()).item()),
                "mean_total_variation": float(tv.mean().item()),
                "maximum_total_variation": float(tv.max().item()),
            })
    total = sum(s["masked_positions"] for s in samples)
    matches = sum(s["top1_matches"] for s in samples)
    return {
        "artifact": "error-propagating SmoothQuant INT8 QKV logit screen",
        "model": DEFAULT_MODEL_ID,
        "revision": DEFAULT_REVISION,
        "device": dev,
        "reference": "INT16 QKV with retained dynamic-INT8-QK fixed18-PV path",
        "candidate": {
            "qkv_weight_bits": 8,
            "smoothquant_alpha": smoothquant_alpha,
            "calibration": "deterministic hardware-package H0 trace",
        },
        "calibration_blocks": calibration_metrics,
        "samples": samples,
        "summary": {
            "sample_count": len(samples),
            "masked_positions": total,
            "top1_matches": matches,
            "mean_top1_agreement": matches / total,
            "minimum_top1_agreement": min(s["top1_agreement"] for s in samples),
            "mean_logit_cosine_similarity": statistics.mean(s["logit_cosine_similarity"] for s in samples),
            "maximum_normalized_logit_rmse": max(s["normalized_logit_rmse"] for s in samples),
            "mean_total_variation": statistics.mean(s["mean_total_variation"] for s in samples),
            "maximum_total_variation": max(s["maximum_total_variation"] for s in samples),
        },
        "scope": (f"{len(samples)} fresh deterministic half-masked canvases with "
                  "QKV projection error propagated through all twelve blocks"),
        "limitation": "one forward evaluation per canvas, not an eight-evaluation generation-quality result",
    }
