"""RTL fixed-point DDiT stages on the GPU, bit-exact with the reference.

Drop-ins for the reference's fixed-point block validation
(src/diffusion_accel/fixed_norm.py, fixed_attention.py):

* ``fixed_layer_norm_q12`` (fixed_norm.py:13-104);
* ``fixed_rotary_q12`` (fixed_attention.py:24-113);
* ``fixed_attention_q12`` (:174-298);
* ``fixed_attention_projection_q10`` (:301-364);
* ``fixed_qkv_projection_q12`` (:367-494);
* the package sweeps ``sweep_fixed_layer_norm`` (fixed_norm.py:107-183),
  ``sweep_fixed_rotary`` (fixed_attention.py:116-171),
  ``sweep_qkv_weight_precision`` (:497-655) and ``sweep_fixed_attention``
  (:658-841).

They take the same arguments, raise the same errors, and return the same
outputs, tensors and metrics.  The integer stages run in
csrc/fixed_point.cu:
  * dh_fixed_layer_norm_q12, dh_fixed_rotary_q12, dh_fixed_attention_q12;
  * dh_fixed_wide_linear: int64 accumulators of 18-bit activations x 8/16-bit
    weights.
The host does three things:
  * the weight quantisation, O(outputs x inputs) and the same torch
    operations as the reference;
  * the exponential table;
  * the float comparisons the metrics report.
"""

from __future__ import annotations

import math
import statistics
from pathlib import Path
from typing import Any, Dict, List, Optional, Tuple

from . import _lib
from .fixed_mlp import _error_metrics, _package_tensors, _quantize_weight_per_output

INT64_MAX = (1 << 63) - 1
INT64_MIN = -(1 << 63)
Q12_MIN, Q12_MAX = -(1 << 17), (1 << 17) - 1
Q10_MIN, Q10_MAX = -(1 << 23), (1 << 23) - 1


def _dev(device: Any) -> Any:
    import torch

    return torch.device(device)


def fixed_layer_norm_q12(activation: Any, *, input_fraction_bits: int = 10, output_fraction_bits: int = 12,
                         inverse_fraction_bits: int = 18, sqrt_extra_fraction_bits: int = 6,
                         epsilon: float = 1e-5, device: Any = "cuda") -> Tuple[Any, Any, Dict[str, object]]:
    """Unaffine LayerNorm of 768-channel Q13.10 rows into signed 18-bit Q5.12
    (fixed_norm.py:13-104); outputs on the activation's device."""
    import torch

    if activation.ndim != 2 or activation.shape[1] != 768:
        raise ValueError("fixed LayerNorm expects a token by 768 matrix")
    dev = _dev(device)
    rows = activation.shape[0]
    x = activation.to(device=dev, dtype=torch.float32).contiguous()
    out = torch.empty((rows, 768), dtype=torch.int32, device=dev)
    st = torch.empty((rows, 5), dtype=torch.int64, device=dev)
    eps_q = round(epsilon * (1 << (2 * input_fraction_bits)))
    _lib.call("dh_fixed_layer_norm_q12", _lib.ptr(x), rows, 768, input_fraction_bits, output_fraction_bits,
              inverse_fraction_bits, sqrt_extra_fraction_bits, eps_q, _lib.ptr(out), _lib.ptr(st),
              _lib.stream_handle())
    output_q = out.to(torch.int64).to(activation.device)
    s = st.cpu()
    output = output_q.float() / float(1 << output_fraction_bits)
    reference = torch.nn.functional.layer_norm(activation.float(), [768])
    metrics: Dict[str, object] = {
        "input_format": "signed-q13.10-24-bit",
        "output_format": "signed-q5.12-18-bit",
        "mean_format": "signed-q13.10",
        "variance_format": "unsigned-q12.20-32-bit",
        "inverse_std_format": "unsigned-q18",
        "sqrt_extra_fraction_bits": sqrt_extra_fraction_bits,
        "epsilon_q20": eps_q,
        "input_saturation_fraction": float(s[:, 4].sum().item()) / float(rows * 768),
        "variance_bits_required": max(1, int(s[:, 1].max().item()).bit_length()),
        "sqrt_radicand_bits_required": max(1, int(s[:, 3].max().item()).bit_length()),
        "inverse_std_bits_required": max(1, int(s[:, 2].max().item()).bit_length()),
        "mean_q10_min": int(s[:, 0].min().item()),
        "mean_q10_max": int(s[:, 0].max().item()),
        "variance_q20_min": int(s[:, 1].min().item()),
        "variance_q20_max": int(s[:, 1].max().item()),
        "inverse_q18_min": int(s[:, 2].min().item()),
        "inverse_q18_max": int(s[:, 2].max().item()),
        "accuracy": _error_metrics(output, reference),
    }
    return output, output_q, metrics


def _rotary_device(qkv: Any, cosine: Any, sine: Any, dev: Any) -> Tuple[Any, Any, Any, List[int]]:
    import torch

    T = qkv.shape[0]
    x = qkv.to(device=dev, dtype=torch.float32).contiguous()
    c = cosine.to(device=dev, dtype=torch.float32).contiguous()
    s = sine.to(device=dev, dtype=torch.float32).contiguous()
    qkv_q = torch.empty((T, 3, 12, 64), dtype=torch.int32, device=dev)
    q = torch.empty((T, 12, 64), dtype=torch.int32, device=dev)
    k = torch.empty((T, 12, 64), dtype=torch.int32, device=dev)
    stats = torch.tensor([0, 0, INT64_MAX, INT64_MIN, INT64_MAX, INT64_MIN], dtype=torch.int64, device=dev)
    _lib.call("dh_fixed_rotary_q12", _lib.ptr(x), _lib.ptr(c), _lib.ptr(s), T, 12, _lib.ptr(qkv_q), _lib.ptr(q),
              _lib.ptr(k), _lib.ptr(stats), _lib.stream_handle())
    return qkv_q, q, k, stats.cpu().tolist()


def _check_qkv(qkv: Any, cosine: Any, sine: Any) -> Any:
    if qkv.ndim == 2 and qkv.shape[1] == 2304:
        qkv = qkv.view(qkv.shape[0], 3, 12, 64)
    if qkv.ndim != 4 or tuple(qkv.shape[1:]) != (3, 12, 64):
        raise ValueError("qkv must have shape tokens by 3 by 12 by 64")
    if cosine.shape != (qkv.shape[0], 32) or sine.shape != cosine.shape:
        raise ValueError("rotary tables must have shape tokens by 32")
    return qkv


def _rotate_float(values: Any, cosine: Any, sine: Any) -> Any:
    import torch

    cos, sin = cosine.float()[:, None, :], sine.float()[:, None, :]
    first, second = values[..., :32], values[..., 32:]
    return torch.cat((first * cos - second * sin, second * cos + first * sin), dim=-1)


def fixed_rotary_q12(qkv: Any, cosine: Any, sine: Any, *, device: Any = "cuda") -> Tuple[Any, Any, Any, Any, Dict]:
    """Rotate Q and K as Q5.12 vectors with signed Q1.15 constants
    (fixed_attention.py:24-113); outputs on the input's device."""
    qkv = _check_qkv(qkv, cosine, sine)
    return _rotary_report(qkv, cosine, sine, *_rotary_device(qkv, cosine, sine, _dev(device)))


def _rotary_report(qkv: Any, cosine: Any, sine: Any, qkv_q: Any, q: Any, k: Any, st: List[int]) -> Tuple:
    import torch

    home = qkv.device
    q12, k12 = q.to(torch.int64).to(home), k.to(torch.int64).to(home)
    cos_q15 = torch.round(cosine.double() * 32768.0).to(torch.int64).clamp(-(1 << 15), (1 << 15) - 1)
    sin_q15 = torch.round(sine.double() * 32768.0).to(torch.int64).clamp(-(1 << 15), (1 << 15) - 1)
    query_rotated, key_rotated = q12.float() / 4096.0, k12.float() / 4096.0
    metrics: Dict[str, object] = {
        "input_and_output_format": "signed-q5.12-18-bit",
        "rotary_constant_format": "signed-q1.15-16-bit",
        "product_format": "signed-q6.27",
        "combined_numerator_bits": 35,
        "input_saturation_fraction": st[0] / float(qkv.shape[0] * 2 * 12 * 64),
        "query_accuracy": _error_metrics(query_rotated, _rotate_float(qkv[:, 0].float(), cosine, sine)),
        "key_accuracy": _error_metrics(key_rotated, _rotate_float(qkv[:, 1].float(), cosine, sine)),
        "query_output_q12_min": st[2],
        "query_output_q12_max": st[3],
        "key_output_q12_min": st[4],
        "key_output_q12_max": st[5],
    }
    tensors = {"qkv_q12": qkv_q.to(torch.int64).to(home), "cosine_q15": cos_q15, "sine_q15": sin_q15}
    return query_rotated, key_rotated, q12, k12, {"metrics": metrics, "tensors": tensors}


def exponential_lut_q16(exponential_step_bits: int = 6, exponential_cutoff: float = 16.0) -> List[int]:
    """Q0.16 exponential table: entry i = min(65535, round(exp(-i / 2^step) *
    65536)) for i <= cutoff * 2^step (fixed_attention.py:213-224)."""
    entries = int(exponential_cutoff * (1 << exponential_step_bits)) + 1
    return [min(65535, round(math.exp(-i / (1 << exponential_step_bits)) * 65536)) for i in range(entries)]


def fixed_attention_q12(qkv: Any, cosine: Any, sine: Any, *, exponential_step_bits: int = 6,
                        exponential_cutoff: float = 16.0, device: Any = "cuda") -> Tuple[Any, Any, Dict]:
    """Fixed QK scores, LUT softmax and probability-times-V attention
    (fixed_attention.py:174-298); outputs on the input's device."""
    import torch

    if exponential_step_bits < 1 or exponential_step_bits > 9:
        raise ValueError("exponential_step_bits must be between 1 and 9")
    if exponential_cutoff <= 0:
        raise ValueError("exponential_cutoff must be positive")
    qkv = _check_qkv(qkv, cosine, sine)
    dev = _dev(device)
    T = qkv.shape[0]
    home = qkv.device
    qkv_q, q, k, rst = _rotary_device(qkv, cosine, sine, dev)
    query_rotated, key_rotated, _, _, rotary = _rotary_report(qkv, cosine, sine, qkv_q, q, k, rst)
    lut = exponential_lut_q16(exponential_step_bits, exponential_cutoff)
    lut_dev = torch.tensor(lut, dtype=torch.int32, device=dev)
    out = torch.empty((T, 768), dtype=torch.int32, device=dev)
    scores = torch.empty((12, T, T), dtype=torch.int32, device=dev)
    probs = torch.empty((12, T, T), dtype=torch.int32, device=dev)
    stats = torch.tensor([0, INT64_MAX, INT64_MIN, 0, 0], dtype=torch.int64, device=dev)
    _lib.call("dh_fixed_attention_q12", _lib.ptr(q), _lib.ptr(k), _lib.ptr(qkv_q), T, 12, exponential_step_bits,
              round(exponential_cutoff * 1024.0), _lib.ptr(lut_dev), len(lut), _lib.ptr(out), _lib.ptr(scores),
              _lib.ptr(probs), _lib.ptr(stats), _lib.stream_handle())
    st = stats.cpu().tolist()
    attention_q12 = out.to(torch.int64).to(home)
    attention = attention_q12.float() / 4096.0
    probabilities_q16 = probs.to(torch.int64).to(home)
    value_q12 = qkv_q[:, 2].to(torch.int64).to(home)
    value_sat = rst[1] / float(T * 12 * 64)
    float_scores = torch.einsum("thd,shd->hts", query_rotated, key_rotated) / 8.0
    float_probabilities = torch.softmax(float_scores, dim=-1)
    float_attention = torch.einsum("hts,shd->thd", float_probabilities, qkv[:, 2].float()).reshape(T, 768)
    probabilities = probabilities_q16.float() / 65536.0
    metrics: Dict[str, object] = {
        "score_format": "signed-q7.10-18-bit",
        "exponential_format": "unsigned-q0.16-16-bit-saturating",
        "probability_format": "unsigned-q0.16-16-bit-saturating",
        "value_and_output_format": "signed-q5.12-18-bit",
        "exponential_step_bits": exponential_step_bits,
        "exponential_lut_entries": len(lut),
        "exponential_cutoff": exponential_cutoff,
        "reciprocal_format": "unsigned-q14-derived-from-2^30-over-sum",
        "score_saturation_fraction": st[0] / float(12 * T * T),
        "value_saturation_fraction": float(value_sat),
        "score_q10_min": st[1],
        "score_q10_max": st[2],
        "minimum_delta_q10": st[3],
        "maximum_probability_row_sum_error_q16": st[4],
        "probability_accuracy": _error_metrics(probabilities, float_probabilities),
        "attention_accuracy": _error_metrics(attention, float_attention),
        "score_argmax_agreement": float(
            probabilities_q16.argmax(dim=-1).eq(float_probabilities.argmax(dim=-1)).float().mean().item()),
        "rotary": rotary["metrics"],
    }
    tensors = {"scores_q10": scores.to(torch.int64).to(home), "probabilities_q16": probabilities_q16,
               "value_q12": value_q12, "exponential_lut_q16": torch.tensor(lut, dtype=torch.int64)}
    return attention, attention_q12, {"metrics": metrics, "tensors": tensors}


def _wide_linear(act_q: Any, weight_q: Any, multipliers: Any, bias_q: Any, shift: int, lo: int, hi: int,
                 dev: Any) -> Tuple[Any, Any, List[int]]:
    import torch

    rows, k = act_q.shape
    n = weight_q.shape[0]
    a = act_q.to(device=dev, dtype=torch.int32).contiguous()
    w = weight_q.to(device=dev, dtype=torch.int16).contiguous()
    m = multipliers.to(device=dev, dtype=torch.int64).contiguous()
    b = None if bias_q is None else bias_q.to(device=dev, dtype=torch.int32).contiguous()
    out = torch.empty((rows, n), dtype=torch.int32, device=dev)
    acc = torch.empty((rows, n), dtype=torch.int64, device=dev)
    stats = torch.tensor([INT64_MAX, INT64_MIN, 0, 0], dtype=torch.int64, device=dev)
    _lib.call("dh_fixed_wide_linear", _lib.ptr(a), _lib.ptr(w), _lib.ptr(m), _lib.ptr(b), rows, n, k, shift, lo, hi,
              _lib.ptr(out), _lib.ptr(acc), _lib.ptr(stats), _lib.stream_handle())
    return out, acc, stats.cpu().tolist()


def fixed_attention_projection_q10(attention_q12: Any, weight: Any, *, requant_shift: int = 24,
                                   device: Any = "cuda") -> Tuple[Any, Any, Dict]:
    """Q5.12 attention through per-output int8 folded weights into saturating
    Q13.10 (fixed_attention.py:301-364); outputs on the input's device."""
    import torch

    if attention_q12.ndim != 2 or attention_q12.shape[1] != 768:
        raise ValueError("attention_q12 must have shape tokens by 768")
    if tuple(weight.shape) != (768, 768):
        raise ValueError("attention projection weight must have shape 768 by 768")
    if requant_shift < 1:
        raise ValueError("requant_shift must be positive")
    weight_q, weight_scales = _quantize_weight_per_output(weight.float(), 8)
    multipliers = torch.round(weight_scales.double() * (1 << requant_shift) / 4.0).to(torch.int64)
    out, acc, st = _wide_linear(attention_q12, weight_q, multipliers, None, requant_shift, Q10_MIN, Q10_MAX,
                                _dev(device))
    home = attention_q12.device
    projection_q10 = out.to(torch.int64).to(home)
    projection = projection_q10.float() / 1024.0
    reference = (attention_q12.float() / 4096.0) @ weight.float().t()
    metrics: Dict[str, object] = {
        "activation_format": "signed-q5.12-18-bit",
        "weight_format": "signed-int8-per-output-scale",
        "output_format": "signed-q13.10-24-bit-saturating",
        "requant_shift": requant_shift,
        "requant_multiplier_min": int(multipliers.min().item()),
        "requant_multiplier_max": int(multipliers.max().item()),
        "required_unsigned_multiplier_bits": max(1, int(multipliers.max().item()).bit_length()),
        "accumulator_min": st[0],
        "accumulator_max": st[1],
        "required_signed_accumulator_bits": max(1, st[3].bit_length() + 1),
        "output_saturation_fraction": st[2] / float(out.numel()),
        "projection_accuracy_from_fixed_attention": _error_metrics(projection, reference),
    }
    tensors = {"weight_int8": weight_q, "requant_multiplier_q24": multipliers,
               "accumulators": acc.to(home)}
    return projection, projection_q10, {"metrics": metrics, "tensors": tensors}


def fixed_qkv_projection_q12(normalized_q12: Any, weight: Any, bias: Any, *, requant_shift: int = 28,
                             weight_bits: int = 16, smoothquant_alpha: Optional[float] = None,
                             smoothquant_scales: Optional[Any] = None, device: Any = "cuda") -> Tuple[Any, Any, Dict]:
    """Fixed LayerNorm output through per-output signed int8 / int16 QKV
    weights into saturating Q5.12, with optional SmoothQuant
    (fixed_attention.py:367-494); outputs on the input's device."""
    import torch

    if normalized_q12.ndim != 2 or normalized_q12.shape[1] != 768:
        raise ValueError("normalized_q12 must have shape tokens by 768")
    if tuple(weight.shape) != (2304, 768):
        raise ValueError("QKV weight must have shape 2304 by 768")
    if tuple(bias.shape) != (2304,):
        raise ValueError("QKV bias must have shape 2304")
    if requant_shift < 1:
        raise ValueError("requant_shift must be positive")
    if weight_bits not in (8, 16):
        raise ValueError("weight_bits must be 8 or 16")
    if smoothquant_alpha is not None and not 0.0 <= smoothquant_alpha <= 1.0:
        raise ValueError("smoothquant_alpha must be between zero and one")
    if smoothquant_alpha is not None and smoothquant_scales is not None:
        raise ValueError("smoothquant_alpha and smoothquant_scales are mutually exclusive")
    home = normalized_q12.device
    act = normalized_q12.to(torch.int64)
    projection_weight = weight.float()
    smoothing = None
    smoothing_sat = 0.0
    if smoothquant_alpha is not None:
        a_max = (normalized_q12.double().abs().amax(dim=0) / 4096.0).clamp_min(1e-8)
        w_max = weight.double().abs().amax(dim=0).clamp_min(1e-8)
        smoothing = a_max.pow(smoothquant_alpha) / w_max.pow(1.0 - smoothquant_alpha)
    elif smoothquant_scales is not None:
        smoothing = torch.as_tensor(smoothquant_scales, dtype=torch.float64)
        if tuple(smoothing.shape) != (768,):
            raise ValueError("smoothquant_scales must have shape 768")
        if not bool(torch.isfinite(smoothing).all()) or bool(smoothing.le(0).any()):
            raise ValueError("smoothquant_scales must be finite and positive")
    if smoothing is not None:
        scaled = torch.round(normalized_q12.double() / smoothing[None, :]).to(torch.int64)
        smoothing_sat = float(((scaled < Q12_MIN) | (scaled > Q12_MAX)).float().mean().item())
        act = scaled.clamp(Q12_MIN, Q12_MAX)
        projection_weight = (weight.double() * smoothing[None, :]).float()
    weight_q, weight_scales = _quantize_weight_per_output(projection_weight, weight_bits)
    multipliers = torch.round(weight_scales.double() * (1 << requant_shift)).to(torch.int64)
    bias_q12 = torch.round(bias.double() * 4096.0).to(torch.int64)
    if int(bias_q12.abs().max().item()) >= 1 << 31:
        raise ValueError("bias exceeds the int32 range in Q5.12")
    out, acc, st = _wide_linear(act, weight_q, multipliers, bias_q12, requant_shift, Q12_MIN, Q12_MAX, _dev(device))
    output_q12 = out.to(torch.int64).to(home)
    output = output_q12.float() / 4096.0
    reference = (normalized_q12.float() / 4096.0) @ weight.float().t() + bias.float()[None, :]
    metrics: Dict[str, object] = {
        "activation_format": "signed-q5.12-18-bit",
        "weight_format": "signed-int%d-per-output-scale" % weight_bits,
        "weight_bits": weight_bits,
        "smoothquant_alpha": smoothquant_alpha,
        "smoothed_activation_saturation_fraction": smoothing_sat,
        "bias_format": "signed-q5.12-18-bit",
        "output_format": "signed-q5.12-18-bit-saturating",
        "requant_shift": requant_shift,
        "requant_multiplier_min": int(multipliers.min().item()),
        "requant_multiplier_max": int(multipliers.max().item()),
        "required_unsigned_multiplier_bits": max(1, int(multipliers.max().item()).bit_length()),
        "required_signed_accumulator_bits": max(1, st[3].bit_length() + 1),
        "output_saturation_fraction": st[2] / float(out.numel()),
        "projection_accuracy_from_fixed_norm": _error_metrics(output, reference),
    }
    tensors = {"weight_int%d" % weight_bits: weight_q, "requant_multiplier_q28": multipliers, "bias_q12": bias_q12,
               "accumulators": acc.to(home)}
    if smoothing is not None:
        tensors["smoothquant_input_scales"] = smoothing
        tensors["smoothed_activation_q12"] = act
    return output, output_q12, {"metrics": metrics, "tensors": tensors}


def _package_blocks(package_dir: Path) -> int:
    import json

    manifest = json.loads((Path(package_dir) / "manifest.json").read_text(encoding="utf-8"))
    return int(manifest["fixed_graph"]["blocks"])


def sweep_fixed_layer_norm(package_dir: Any, *, device: Any = "cuda") -> Dict[str, object]:
    """Every norm1, norm2 and final LayerNorm boundary of a package
    (fixed_norm.py:107-183)."""
    package_dir = Path(package_dir)
    nb = _package_blocks(package_dir)
    names = ["folded.embedding", "folded.final.norm_unaffine"]
    for b in range(nb):
        p = "folded.block_%02d" % b
        names += [p + ".after_attention", p + ".output", p + ".norm1_unaffine", p + ".norm2_unaffine"]
    t = _package_tensors(package_dir / "golden_tensors.safetensors", names)
    boundaries = []
    for b in range(nb):
        p = "folded.block_%02d" % b
        norm1_in = t["folded.embedding"][0] if b == 0 else t["folded.block_%02d.output" % (b - 1)][0]
        for name, act, expected in (("block_%02d.norm1" % b, norm1_in, t[p + ".norm1_unaffine"][0]),
                                    ("block_%02d.norm2" % b, t[p + ".after_attention"][0],
                                     t[p + ".norm2_unaffine"][0])):
            out, _, m = fixed_layer_norm_q12(act, device=device)
            m["accuracy_vs_h0_golden"] = _error_metrics(out, expected)
            boundaries.append({"name": name, "metrics": m})
    out, _, m = fixed_layer_norm_q12(t["folded.block_%02d.output" % (nb - 1)][0], device=device)
    m["accuracy_vs_h0_golden"] = _error_metrics(out, t["folded.final.norm_unaffine"][0])
    boundaries.append({"name": "final.norm", "metrics": m})
    rel = [x["metrics"]["accuracy_vs_h0_golden"]["relative_rms_error"] for x in boundaries]
    return {
        "package_dir": str(package_dir),
        "boundary_count": len(boundaries),
        "boundaries": boundaries,
        "summary": {
            "minimum_relative_rms": min(rel),
            "mean_relative_rms": statistics.mean(rel),
            "median_relative_rms": statistics.median(rel),
            "maximum_relative_rms": max(rel),
            "maximum_input_saturation_fraction": max(x["metrics"]["input_saturation_fraction"] for x in boundaries),
            "maximum_variance_bits_required": max(x["metrics"]["variance_bits_required"] for x in boundaries),
            "maximum_sqrt_radicand_bits_required": max(x["metrics"]["sqrt_radicand_bits_required"]
                                                       for x in boundaries),
            "maximum_inverse_std_bits_required": max(x["metrics"]["inverse_std_bits_required"] for x in boundaries),
        },
        "scope": "all %d H0 unaffine LayerNorm boundaries on one frozen input" % len(boundaries),
    }


def sweep_fixed_rotary(package_dir: Any, *, device: Any = "cuda") -> Dict[str, object]:
    """Fixed rotary Q/K at every block of a package (fixed_attention.py:116-171)."""
    package_dir = Path(package_dir)
    nb = _package_blocks(package_dir)
    names = ["folded.block_%02d.qkv" % b for b in range(nb)]
    qkv = _package_tensors(package_dir / "golden_tensors.safetensors", names)
    tables = _package_tensors(package_dir / "folded_fp16_weights.safetensors", ["rotary.cos", "rotary.sin"])
    cos, sin = tables["rotary.cos"].float(), tables["rotary.sin"].float()
    blocks = []
    for b, name in enumerate(names):
        _, _, _, _, details = fixed_rotary_q12(qkv[name][0], cos, sin, device=device)
        blocks.append({"block": b, "metrics": details["metrics"]})
    qe = [x["metrics"]["query_accuracy"]["relative_rms_error"] for x in blocks]
    ke = [x["metrics"]["key_accuracy"]["relative_rms_error"] for x in blocks]
    return {
        "package_dir": str(package_dir),
        "block_count": len(blocks),
        "blocks": blocks,
        "summary": {
            "mean_query_relative_rms": statistics.mean(qe),
            "maximum_query_relative_rms": max(qe),
            "mean_key_relative_rms": statistics.mean(ke),
            "maximum_key_relative_rms": max(ke),
            "maximum_input_saturation_fraction": max(x["metrics"]["input_saturation_fraction"] for x in blocks),
            "minimum_output_q12": min(min(x["metrics"]["query_output_q12_min"], x["metrics"]["key_output_q12_min"])
                                      for x in blocks),
            "maximum_output_q12": max(max(x["metrics"]["query_output_q12_max"], x["metrics"]["key_output_q12_max"])
                                      for x in blocks),
        },
        "scope": "all twelve H0 Q/K rotary boundaries on one frozen input",
    }


def sweep_fixed_attention(package_dir: Any, *, device: Any = "cuda") -> Dict[str, object]:
    """Fixed LayerNorm -> QKV projection -> attention -> output projection ->
    residual at every block of a package (fixed_attention.py:658-841)."""
    import torch

    package_dir = Path(package_dir)
    nb = _package_blocks(package_dir)
    names = ["folded.embedding"]
    for b in range(nb):
        names += ["folded.block_%02d.%s" % (b, s) for s in ("qkv", "attention", "attention_projection",
                                                             "after_attention", "output")]
    g = _package_tensors(package_dir / "golden_tensors.safetensors", names)
    wn = ["block_%02d.attention_out.weight" % b for b in range(nb)]
    for b in range(nb):
        wn += ["block_%02d.qkv.weight" % b, "block_%02d.qkv.bias" % b]
    tables = _package_tensors(package_dir / "folded_fp16_weights.safetensors", ["rotary.cos", "rotary.sin", *wn])
    cos, sin = tables["rotary.cos"].float(), tables["rotary.sin"].float()
    blocks = []
    for b in range(nb):
        p = "folded.block_%02d" % b
        residual = g["folded.embedding"][0] if b == 0 else g["folded.block_%02d.output" % (b - 1)][0]
        _, normalized_q12, _ = fixed_layer_norm_q12(residual, device=device)
        fixed_qkv, _, qkv_details = fixed_qkv_projection_q12(normalized_q12, tables["block_%02d.qkv.weight" % b],
                                                              tables["block_%02d.qkv.bias" % b], device=device)
        qkv_details["metrics"]["accuracy_vs_h0_golden"] = _error_metrics(fixed_qkv, g[p + ".qkv"][0])
        cascade, cascade_q12, _ = fixed_attention_q12(fixed_qkv, cos, sin, device=device)
        qkv_details["metrics"]["attention_accuracy_vs_h0_golden"] = _error_metrics(cascade, g[p + ".attention"][0])
        attention, _, details = fixed_attention_q12(g[p + ".qkv"][0], cos, sin, device=device)
        m = details["metrics"]
        m["qkv_projection"] = qkv_details["metrics"]
        m["accuracy_vs_h0_golden"] = _error_metrics(attention, g[p + ".attention"][0])
        projection, projection_q10, pd = fixed_attention_projection_q10(
            cascade_q12, tables["block_%02d.attention_out.weight" % b], device=device)
        m["projection"] = pd["metrics"]
        m["projection"]["accuracy_vs_h0_golden"] = _error_metrics(projection, g[p + ".attention_projection"][0])
        residual_q10 = torch.round(residual.double() * 1024.0).to(torch.int64).clamp(Q10_MIN, Q10_MAX)
        after_unclipped = residual_q10 + projection_q10
        after = after_unclipped.clamp(Q10_MIN, Q10_MAX).float() / 1024.0
        m["residual"] = {
            "format": "signed-q13.10-24-bit-saturating",
            "output_saturation_fraction": float(((after_unclipped < Q10_MIN) | (after_unclipped > Q10_MAX))
                                                .float().mean().item()),
            "accuracy_vs_h0_golden": _error_metrics(after, g[p + ".after_attention"][0]),
        }
        blocks.append({"block": b, "metrics": m})

    def rel(path) -> List[float]:
        out = []
        for x in blocks:
            v = x["metrics"]
            for key in path:
                v = v[key]
            out.append(v["relative_rms_error"])
        return out

    e = rel(["accuracy_vs_h0_golden"])
    pe = rel(["projection", "accuracy_vs_h0_golden"])
    re_ = rel(["residual", "accuracy_vs_h0_golden"])
    qe = rel(["qkv_projection", "accuracy_vs_h0_golden"])
    ce = rel(["qkv_projection", "attention_accuracy_vs_h0_golden"])
    return {
        "package_dir": str(package_dir),
        "block_count": len(blocks),
        "blocks": blocks,
        "summary": {
            "mean_attention_relative_rms_vs_h0": statistics.mean(e),
            "maximum_attention_relative_rms_vs_h0": max(e),
            "maximum_score_saturation_fraction": max(x["metrics"]["score_saturation_fraction"] for x in blocks),
            "maximum_value_saturation_fraction": max(x["metrics"]["value_saturation_fraction"] for x in blocks),
            "minimum_score_argmax_agreement": min(x["metrics"]["score_argmax_agreement"] for x in blocks),
            "maximum_probability_row_sum_error_q16": max(x["metrics"]["maximum_probability_row_sum_error_q16"]
                                                         for x in blocks),
            "mean_projection_relative_rms_vs_h0": statistics.mean(pe),
            "maximum_projection_relative_rms_vs_h0": max(pe),
            "mean_after_attention_relative_rms_vs_h0": statistics.mean(re_),
            "maximum_after_attention_relative_rms_vs_h0": max(re_),
            "maximum_projection_output_saturation_fraction": max(
                x["metrics"]["projection"]["output_saturation_fraction"] for x in blocks),
            "maximum_residual_output_saturation_fraction": max(
                x["metrics"]["residual"]["output_saturation_fraction"] for x in blocks),
            "mean_qkv_projection_relative_rms_vs_h0": statistics.mean(qe),
            "maximum_qkv_projection_relative_rms_vs_h0": max(qe),
            "mean_attention_from_fixed_qkv_relative_rms_vs_h0": statistics.mean(ce),
            "maximum_attention_from_fixed_qkv_relative_rms_vs_h0": max(ce),
        },
        "scope": ("all twelve complete H0 attention, folded output projection, and "
                  "residual boundaries on one frozen input"),
    }


def sweep_qkv_weight_precision(package_dir: Any, *, weight_bits: Tuple[int, ...] = (8, 16),
                               smoothquant_alphas: Tuple[Optional[float], ...] = (None,),
                               device: Any = "cuda") -> Dict[str, object]:
    """QKV weight widths (and SmoothQuant equalisation of the 8-bit design)
    at every captured attention boundary of a package: fixed LayerNorm ->
    fixed QKV projection -> fixed attention, against the package's float
    goldens (fixed_attention.py:497-655)."""
    if not weight_bits or any(bits not in (8, 16) for bits in weight_bits):
        raise ValueError("weight_bits must contain only 8 or 16")
    if not smoothquant_alphas or any(alpha is not None and not 0.0 <= alpha <= 1.0 for alpha in smoothquant_alphas):
        raise ValueError("smoothquant_alphas must contain none or values from zero to one")
    package_dir = Path(package_dir)
    names = ["folded.embedding"]
    for b in range(12):
        names += ["folded.block_%02d.%s" % (b, s) for s in ("qkv", "attention", "output")]
    g = _package_tensors(package_dir / "golden_tensors.safetensors", names)
    wn = []
    for b in range(12):
        wn += ["block_%02d.qkv.weight" % b, "block_%02d.qkv.bias" % b]
    tables = _package_tensors(package_dir / "folded_fp16_weights.safetensors", ["rotary.cos", "rotary.sin", *wn])
    cos, sin = tables["rotary.cos"].float(), tables["rotary.sin"].float()
    # the fixed LayerNorm of each boundary does not depend on the design
    normalized = []
    for b in range(12):
        residual = g["folded.embedding"][0] if b == 0 else g["folded.block_%02d.output" % (b - 1)][0]
        normalized.append(fixed_layer_norm_q12(residual, device=device)[1])
    designs = []
    for bits in weight_bits:
        for alpha in (smoothquant_alphas if bits == 8 else (None,)):
            blocks = []
            for b in range(12):
                fixed_qkv, _, qd = fixed_qkv_projection_q12(normalized[b], tables["block_%02d.qkv.weight" % b],
                                                            tables["block_%02d.qkv.bias" % b], weight_bits=bits,
                                                            smoothquant_alpha=alpha, device=device)
                attention, _, ad = fixed_attention_q12(fixed_qkv, cos, sin, device=device)
                blocks.append({
                    "block": b,
                    "qkv_accuracy_vs_h0": _error_metrics(fixed_qkv, g["folded.block_%02d.qkv" % b][0]),
                    "attention_accuracy_vs_h0": _error_metrics(attention, g["folded.block_%02d.attention" % b][0]),
                    "qkv_projection": qd["metrics"],
                    "attention": ad["metrics"],
                })
            qe = [x["qkv_accuracy_vs_h0"]["relative_rms_error"] for x in blocks]
            ae = [x["attention_accuracy_vs_h0"]["relative_rms_error"] for x in blocks]
            designs.append({
                "weight_bits": bits,
                "smoothquant_alpha": alpha,
                "blocks": blocks,
                "summary": {
                    "mean_qkv_relative_rms_vs_h0": statistics.mean(qe),
                    "maximum_qkv_relative_rms_vs_h0": max(qe),
                    "mean_attention_relative_rms_vs_h0": statistics.mean(ae),
                    "maximum_attention_relative_rms_vs_h0": max(ae),
                    "maximum_qkv_output_saturation_fraction": max(
                        x["qkv_projection"]["output_saturation_fraction"] for x in blocks),
                    "maximum_smoothed_activation_saturation_fraction": max(
                        x["qkv_projection"]["smoothed_activation_saturation_fraction"] for x in blocks),
                    "minimum_score_argmax_agreement": min(x["attention"]["score_argmax_agreement"] for x in blocks),
                },
            })
    return {
        "package_dir": str(package_dir),
        "block_count": 12,
        "designs": designs,
        "scope": "all twelve H0 QKV projection and attention boundaries on one frozen input",
        "limitation": ("boundary fidelity screen only; fresh-canvas final-logit and "
                       "generation validation remains required before changing RTL"),
    }
