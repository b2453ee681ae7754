"""Packed INT8 attention candidates on the GPU, bit-exact with the reference.

Drop-ins for the reference's paired-token INT8 attention screens
(src/diffusion_accel/attention_int8.py):

* ``dynamic_qk_fixed_pv_attention_q12`` (:28-123), the packed M8 RTL
  contract: dynamic per-vector INT8 Q / K, fixed18 P . V;
* ``_evaluate_with_fixed_maxima`` (:126-315), the candidate space: QK in
  fixed18, calibrated-head or dynamic-vector INT8 / INT9, P . V in fixed18
  or with 7 / 8-bit probabilities (optionally sum-corrected) and 8 / 9-bit
  values;
* ``screen_packed_int8_attention`` (:318-519) over a package's captured
  attention boundaries, ``screen_packed_int8_attention_heldout`` (:522-686)
  on fresh half-masked canvases, and ``screen_packed_int8_attention_logits``
  (:689-936), which propagates the candidate through all twelve blocks to the
  logits.

Same arguments, errors, outputs and metrics.  The integer stages run in
csrc/fixed_point.cu: dh_fixed_rotary_q12 (K12), dh_fixed_attention_q12 (K13,
the fixed18 baseline) and dh_packed_int8_attention_q12 (K15: requantisation
of Q / K / V, Q28 score rescale, LUT softmax, probability requantisation and
the integer P . V).  The host computes the per-head multipliers (Python
integer arithmetic, as the reference does), the calibration maxima and the
metrics.

The reference's held-out and logit screens load the MDLM-OWT checkpoint from
the local Hugging Face cache; here the float model is passed as ``model``
(a module with the HF DDiT attribute names, e.g. ``model.build_standin`` or a
loaded checkpoint, or an already folded ``FoldedMDLM``) and run by
``model.fp32_forward`` (the folded forward of hardware_package.py:195-289)
on the host.
"""

from __future__ import annotations

import statistics
from pathlib import Path
from typing import Any, Dict, List, Optional, Sequence, Tuple

from . import _lib
from .fixed_mlp import _error_metrics, _package_tensors
from .fixed_point import _check_qkv, _dev, _rotary_device, exponential_lut_q16, fixed_attention_projection_q10

_QK_MODES = {"calibrated-head": 1, "dynamic-vector": 2}


def _exponential_table() -> Any:
    """The 1,025-entry Q0.16 table the screens build inline
    (attention_int8.py:49-56): exp(-i / 64), 16 nats."""
    import torch

    return torch.tensor(exponential_lut_q16(6, 16.0), dtype=torch.int64)


class _Device:
    """K12 rotary of one qkv canvas, kept on the device for K13 / K15."""

    def __init__(self, qkv: Any, cosine: Any, sine: Any, device: Any, lut: Any) -> None:
        import torch

        lut = torch.as_tensor(lut)
        if lut.ndim != 1 or lut.shape[0] < 1025:
            raise ValueError("exponential_lut_q16 must hold at least 1025 entries")
        self.dev = _dev(device)
        self.T = qkv.shape[0]
        self.qkv_q, self.q, self.k, _ = _rotary_device(qkv, cosine, sine, self.dev)
        self.lut = lut.to(device=self.dev, dtype=torch.int32).contiguous()

    def fixed18(self) -> Tuple[Any, Any]:
        """K13 with the screens' table: attention_q12 [T, 768] and scores_q10
        [12, T, T] (fixed_attention.py:174-298)."""
        import torch

        T, dev = self.T, self.dev
        out = torch.empty((T, 768), dtype=torch.int32, device=dev)
        scores = torch.empty((12, T, T), dtype=torch.int32, device=dev)
        _lib.call("dh_fixed_attention_q12", _lib.ptr(self.q), _lib.ptr(self.k), _lib.ptr(self.qkv_q), T, 12, 6,
                  16 * 1024, _lib.ptr(self.lut), self.lut.shape[0], _lib.ptr(out), _lib.ptr(scores), None, None,
                  _lib.stream_handle())
        return out, scores

    def packed(self, *, qk_mode: int, qk_scores: bool, qk_levels: int, qk_fraction_bits: int,
               probability_levels: int, sum_correction: bool, value_levels: int,
               head_params: List[List[int]]) -> Dict[str, Any]:
        """K15 (dh_packed_int8_attention_q12); device tensors."""
        import torch

        T, dev = self.T, self.dev
        params = torch.tensor(head_params, dtype=torch.int64).to(dev)
        out = torch.empty((T, 768), dtype=torch.int32, device=dev)
        scores = torch.empty((12, T, T), dtype=torch.int32, device=dev)
        probs = torch.empty((12, T, T), dtype=torch.int32, device=dev)
        probs_q = torch.zeros((12, T, T), dtype=torch.int32, device=dev)
        qmax = torch.zeros((T, 12), dtype=torch.int32, device=dev)
        kmax = torch.zeros((T, 12), dtype=torch.int32, device=dev)
        work = torch.empty(3 * T * 12 * 64, dtype=torch.int32, device=dev)
        stats = torch.zeros((12, 4), dtype=torch.int64, device=dev)
        _lib.call("dh_packed_int8_attention_q12", _lib.ptr(self.q), _lib.ptr(self.k), _lib.ptr(self.qkv_q), T, 12,
                  qk_mode, int(qk_scores), qk_levels, qk_fraction_bits, probability_levels, int(sum_correction),
                  value_levels, _lib.ptr(params), 6, 16 * 1024, _lib.ptr(self.lut), self.lut.shape[0],
                  _lib.ptr(work), _lib.ptr(out), _lib.ptr(scores), _lib.ptr(probs), _lib.ptr(probs_q),
                  _lib.ptr(qmax), _lib.ptr(kmax), _lib.ptr(stats), _lib.stream_handle())
        return {"out": out, "scores": scores, "probs": probs, "probs_q": probs_q, "qmax": qmax, "kmax": kmax,
                "stats": stats}


def _head_maxima(q12: Any, k12: Any, v12: Any) -> List[Dict[str, int]]:
    """Per-head calibration maxima max(1, max |x|) of the rotated query, key
    and value (attention_int8.py:567-583)."""
    qm = q12.abs().amax(dim=(0, 2)).clamp(min=1).tolist()
    km = k12.abs().amax(dim=(0, 2)).clamp(min=1).tolist()
    vm = v12.abs().amax(dim=(0, 2)).clamp(min=1).tolist()
    return [{"query_q12": int(qm[h]), "key_q12": int(km[h]), "value_q12": int(vm[h])} for h in range(12)]


def dynamic_qk_fixed_pv_attention_q12(qkv: Any, cosine: Any, sine: Any, *, qk_multiplier_fraction_bits: int = 17,
                                      device: Any = "cuda") -> Tuple[Any, Dict[str, Any]]:
    """The retained dynamic-INT8-QK and fixed18-PV attention of the packed M8
    RTL (attention_int8.py:28-123): per-vector Q17 multipliers, Q28 score
    rescale, the LUT softmax and Q16 x Q12 P . V.  Returns the attention
    [tokens, 768] int64 and its tensors, on the input's device."""
    import torch

    if qk_multiplier_fraction_bits != 17:
        raise ValueError("the retained packed RTL uses Q17 multipliers")
    qkv = _check_qkv(qkv, cosine, sine)
    home = qkv.device
    d = _Device(qkv, cosine, sine, device, _exponential_table())
    r = d.packed(qk_mode=2, qk_scores=True, qk_levels=127, qk_fraction_bits=17, probability_levels=0,
                 sum_correction=False, value_levels=0, head_params=[[0] * 8 for _ in range(12)])
    T = d.T

    def h64(t):
        return t.to(torch.int64).to(home)

    attention = h64(r["out"]).view(T, 12, 64)
    return attention.reshape(T, 768), {
        "tensors": {
            "query_q12": h64(d.q),
            "key_q12": h64(d.k),
            "value_q12": h64(d.qkv_q[:, 2]),
            "query_maxima_q12": h64(r["qmax"]).t().contiguous(),
            "key_maxima_q12": h64(r["kmax"]).t().contiguous(),
            "scores_q10": h64(r["scores"]),
            "probabilities_q16": h64(r["probs"]),
            "attention_q12": attention,
        }
    }


def _evaluate_with_fixed_maxima(qkv: Any, cosine: Any, sine: Any, calibration: Sequence[Dict[str, int]],
                                exponential_lut_q16: Any, *, quantize_qk: bool = True, quantize_pv: bool = True,
                                qk_bits: int = 8, qk_scale_mode: str = "calibrated-head",
                                qk_multiplier_fraction_bits: int = 24, pv_probability_levels: int = 127,
                                pv_probability_sum_correction: bool = False, pv_value_bits: int = 8,
                                device: Any = "cuda") -> Tuple[Any, Any, List[Dict[str, object]]]:
    """Packed INT8 attention with previously calibrated per-head maxima
    (attention_int8.py:126-315).  Returns the candidate and the fixed18
    baseline attention [tokens, 768] int64 (input's device) and per-head
    metrics."""
    if qk_bits not in {8, 9}:
        raise ValueError("qk_bits must be 8 or 9")
    if qk_scale_mode not in {"calibrated-head", "dynamic-vector"}:
        raise ValueError("qk_scale_mode must be calibrated-head or dynamic-vector")
    if qk_multiplier_fraction_bits not in {17, 24}:
        raise ValueError("qk_multiplier_fraction_bits must be 17 or 24")
    if pv_probability_levels not in {127, 255}:
        raise ValueError("pv_probability_levels must be 127 or 255")
    if pv_value_bits not in {8, 9}:
        raise ValueError("pv_value_bits must be 8 or 9")
    import torch

    value_levels = (1 << (pv_value_bits - 1)) - 1
    qk_levels = (1 << (qk_bits - 1)) - 1
    qkv = _check_qkv(qkv, cosine, sine)
    home = qkv.device
    d = _Device(qkv, cosine, sine, device, exponential_lut_q16)
    base_out, base_scores = d.fixed18()
    calibrated = qk_scale_mode == "calibrated-head"
    params = []
    for h in range(12):
        m = calibration[h]
        params.append([
            round(qk_levels * (1 << qk_multiplier_fraction_bits) / max(1, m["query_q12"])) if calibrated else 0,
            round(qk_levels * (1 << qk_multiplier_fraction_bits) / max(1, m["key_q12"])) if calibrated else 0,
            round(value_levels * (1 << 24) / max(1, m["value_q12"])),
            round(m["query_q12"] * m["key_q12"] * (1 << 28) / (qk_levels * qk_levels * (1 << 17))),
            round(m["value_q12"] * (1 << 24) / (value_levels * pv_probability_levels)),
            m["query_q12"], m["key_q12"], m["value_q12"],
        ])
    r = d.packed(qk_mode=_QK_MODES[qk_scale_mode], qk_scores=quantize_qk, qk_levels=qk_levels,
                 qk_fraction_bits=qk_multiplier_fraction_bits,
                 probability_levels=pv_probability_levels if quantize_pv else 0,
                 sum_correction=pv_probability_sum_correction, value_levels=value_levels, head_params=params)
    T = d.T
    stats = r["stats"].cpu().tolist()
    agree = r["scores"].argmax(dim=-1).eq(base_scores.argmax(dim=-1)).float().mean(dim=-1).cpu().tolist()
    head_metrics = []
    for h in range(12):
        head_metrics.append({
            "head": h,
            "query_saturation_fraction": stats[h][0] / float(T * 64) if calibrated else 0.0,
            "key_saturation_fraction": stats[h][1] / float(T * 64) if calibrated else 0.0,
            "value_saturation_fraction": stats[h][2] / float(T * 64),
            "score_argmax_agreement_vs_fixed18": float(agree[h]),
        })
    return r["out"].to(torch.int64).to(home), base_out.to(torch.int64).to(home), head_metrics


def _attention_boundary_inputs(package_dir: Path, extra: Sequence[str]) -> Tuple[Dict[str, Any], Dict[str, Any]]:
    qkv_names = ["folded.block_%02d.qkv" % b for b in range(12)]
    goldens = _package_tensors(package_dir / "golden_tensors.safetensors", qkv_names)
    tables = _package_tensors(package_dir / "folded_fp16_weights.safetensors", ["rotary.cos", "rotary.sin", *extra])
    return goldens, tables


def _package_calibrations(goldens: Dict[str, Any], cosine: Any, sine: Any, device: Any) -> List[List[Dict]]:
    """Per-block, per-head maxima of the package's captured canvas
    (attention_int8.py:564-583)."""
    import torch

    out = []
    for b in range(12):
        qkv = _check_qkv(goldens["folded.block_%02d.qkv" % b][0], cosine, sine)
        qkv_q, q, k, _ = _rotary_device(qkv, cosine, sine, _dev(device))
        out.append(_head_maxima(q.to(torch.int64), k.to(torch.int64), qkv_q[:, 2].to(torch.int64)))
    return out


def screen_packed_int8_attention(package_dir: Any, *, device: Any = "cuda") -> Dict[str, object]:
    """Integer-only paired-token attention on a package's captured boundaries
    (attention_int8.py:318-519): Q, K and V with one symmetric maximum per
    block and head taken from the same canvas, 7-bit probabilities."""
    import torch

    package_dir = Path(package_dir)
    projection_names = ["block_%02d.attention_out.weight" % b for b in range(12)]
    goldens, tables = _attention_boundary_inputs(package_dir, projection_names)
    cosine, sine = tables["rotary.cos"].float(), tables["rotary.sin"].float()
    lut = _exponential_table()
    blocks = []
    for b in range(12):
        qkv = _check_qkv(goldens["folded.block_%02d.qkv" % b][0], cosine, sine)
        d = _Device(qkv, cosine, sine, device, lut)
        base_out, base_scores = d.fixed18()
        maxima = _head_maxima(d.q.to(torch.int64), d.k.to(torch.int64), d.qkv_q[:, 2].to(torch.int64))
        params = []
        for m in maxima:
            qm, km, vm = m["query_q12"], m["key_q12"], m["value_q12"]
            params.append([round(127 * (1 << 24) / qm), round(127 * (1 << 24) / km), round(127 * (1 << 24) / vm),
                           round(qm * km * (1 << 28) / (127 * 127 * (1 << 17))), round(vm * (1 << 24) / (127 * 127)),
                           qm, km, vm])
        r = d.packed(qk_mode=1, qk_scores=True, qk_levels=127, qk_fraction_bits=24, probability_levels=127,
                     sum_correction=False, value_levels=127, head_params=params)
        T = d.T
        stats = r["stats"].cpu().tolist()
        agree = r["scores"].argmax(dim=-1).eq(base_scores.argmax(dim=-1)).float().mean(dim=-1).cpu().tolist()
        head_metrics = []
        for h in range(12):
            p = params[h]
            head_metrics.append({
                "head": h,
                "query_calibration_maximum_q12": p[5],
                "key_calibration_maximum_q12": p[6],
                "value_calibration_maximum_q12": p[7],
                "query_requant_multiplier_q24": p[0],
                "key_requant_multiplier_q24": p[1],
                "value_requant_multiplier_q24": p[2],
                "score_multiplier_q28": p[3],
                "output_multiplier_q24": p[4],
                "score_argmax_agreement_vs_fixed18": float(agree[h]),
                "zero_probability_fraction_int7": stats[h][3] / float(T * T),
            })
        cand = r["out"].to(torch.int64).cpu()
        base = base_out.to(torch.int64).cpu()
        w = tables[projection_names[b]]
        _, base_proj, _ = fixed_attention_projection_q10(base, w, device=device)
        _, cand_proj, _ = fixed_attention_projection_q10(cand, w, device=device)
        blocks.append({
            "block": b,
            "attention_accuracy_vs_fixed18": _error_metrics(cand.float() / 4096.0, base.float() / 4096.0),
            "projection_accuracy_vs_fixed18": _error_metrics(cand_proj.float() / 1024.0, base_proj.float() / 1024.0),
            "maximum_attention_absolute_error_q12": int((cand - base).abs().max().item()),
            "minimum_score_argmax_agreement_vs_fixed18": min(x["score_argmax_agreement_vs_fixed18"]
                                                             for x in head_metrics),
            "heads": head_metrics,
        })
    att = [x["attention_accuracy_vs_fixed18"]["relative_rms_error"] for x in blocks]
    cos_ = [x["attention_accuracy_vs_fixed18"]["cosine_similarity"] for x in blocks]
    proj = [x["projection_accuracy_vs_fixed18"]["relative_rms_error"] for x in blocks]
    return {
        "artifact": "paired-token INT8 attention captured-trace screen",
        "package_dir": str(package_dir),
        "blocks": blocks,
        "summary": {
            "mean_attention_relative_rms_vs_fixed18": statistics.mean(att),
            "maximum_attention_relative_rms_vs_fixed18": max(att),
            "mean_attention_cosine_similarity_vs_fixed18": statistics.mean(cos_),
            "minimum_attention_cosine_similarity_vs_fixed18": min(cos_),
            "maximum_attention_absolute_error_q12": max(x["maximum_attention_absolute_error_q12"] for x in blocks),
            "mean_projection_relative_rms_vs_fixed18": statistics.mean(proj),
            "maximum_projection_relative_rms_vs_fixed18": max(proj),
            "minimum_head_score_argmax_agreement_vs_fixed18": min(
                x["minimum_score_argmax_agreement_vs_fixed18"] for x in blocks),
        },
        "formats": {
            "query_key_value": "signed-int8-symmetric-per-block-per-head",
            "probability": "unsigned-magnitude-7-bit-in-signed-int8-lane",
            "score": "signed-q7.10-18-bit",
            "attention_output": "signed-q5.12-18-bit",
        },
        "scope": ("all twelve H0 blocks on the same captured input used to calibrate "
                  "each per-head maximum; this is not held-out quality evidence"),
    }


def _folded(model: Any) -> Any:
    from .model import FoldedMDLM, fold

    if model is None:
        raise ValueError("no local MDLM checkpoint: pass model= (a module with the HF DDiT attribute names "
                         "or a FoldedMDLM)")
    return model if isinstance(model, FoldedMDLM) else fold(model)


def _half_masked_canvas(seed: int, mask_token_id: int) -> Any:
    """64 ids from a CPU generator seeded with `seed`, odd positions masked
    (attention_int8.py:587-595)."""
    import torch

    g = torch.Generator(device="cpu").manual_seed(seed)
    ids = torch.randint(0, mask_token_id, (1, 64), generator=g, dtype=torch.long)
    ids[:, 1::2] = mask_token_id
    return ids


def screen_packed_int8_attention_heldout(package_dir: Any, *, seeds: Optional[Sequence[int]] = None,
                                         device: str = "auto", model: Any = None) -> Dict[str, object]:
    """The package's per-head calibration applied to fresh deterministic
    half-masked canvases (attention_int8.py:522-686); each block boundary is
    evaluated on the float model's own qkv, without error propagation."""
    from .model import fp32_forward

    selected = [101, 202, 303, 404, 505] if seeds is None else list(seeds)
    if not selected:
        raise ValueError("at least one held-out seed is required")
    package_dir = Path(package_dir)
    projection_names = ["block_%02d.attention_out.weight" % b for b in range(12)]
    goldens, tables = _attention_boundary_inputs(package_dir, projection_names)
    cosine, sine = tables["rotary.cos"].float(), tables["rotary.sin"].float()
    dev = "cuda" if device == "auto" else device
    lut = _exponential_table()
    calibrations = _package_calibrations(goldens, cosine, sine, dev)
    folded = _folded(model)
    mask = int(folded.config.vocab_size) - 1
    samples = []
    for seed in selected:
        ids = _half_masked_canvas(seed, mask)
        captured: Dict[str, Any] = {}
        fp32_forward(folded, ids.numpy(), captured=captured)
        block_results = []
        for b in range(12):
            cand, base, heads = _evaluate_with_fixed_maxima(captured["folded.block_%02d.qkv" % b][0], cosine, sine,
                                                            calibrations[b], lut, device=dev)
            w = tables[projection_names[b]]
            _, cand_proj, _ = fixed_attention_projection_q10(cand, w, device=dev)
            _, base_proj, _ = fixed_attention_projection_q10(base, w, device=dev)
            block_results.append({
                "block": b,
                "attention_accuracy_vs_fixed18": _error_metrics(cand.float() / 4096.0, base.float() / 4096.0),
                "projection_accuracy_vs_fixed18": _error_metrics(cand_proj.float() / 1024.0,
                                                                 base_proj.float() / 1024.0),
                "maximum_operand_saturation_fraction": max(
                    max(x["query_saturation_fraction"], x["key_saturation_fraction"], x["value_saturation_fraction"])
                    for x in heads),
                "minimum_score_argmax_agreement_vs_fixed18": min(x["score_argmax_agreement_vs_fixed18"]
                                                                 for x in heads),
            })
        samples.append({"seed": seed, "blocks": block_results})
    allb = [b for s in samples for b in s["blocks"]]
    return {
        "artifact": "held-out paired-token INT8 attention boundary screen",
        "device": dev,
        "calibration": "original deterministic hardware-package H0 trace",
        "samples": samples,
        "summary": {
            "sample_count": len(samples),
            "block_boundaries": len(allb),
            "mean_attention_relative_rms_vs_fixed18": statistics.mean(
                b["attention_accuracy_vs_fixed18"]["relative_rms_error"] for b in allb),
            "maximum_attention_relative_rms_vs_fixed18": max(
                b["attention_accuracy_vs_fixed18"]["relative_rms_error"] for b in allb),
            "mean_projection_relative_rms_vs_fixed18": statistics.mean(
                b["projection_accuracy_vs_fixed18"]["relative_rms_error"] for b in allb),
            "maximum_projection_relative_rms_vs_fixed18": max(
                b["projection_accuracy_vs_fixed18"]["relative_rms_error"] for b in allb),
            "maximum_operand_saturation_fraction": max(b["maximum_operand_saturation_fraction"] for b in allb),
            "minimum_head_score_argmax_agreement_vs_fixed18": min(
                b["minimum_score_argmax_agreement_vs_fixed18"] for b in allb),
        },
        "scope": ("fresh deterministic random half-masked canvases, fixed calibration, "
                  "independent attention boundaries without quantization-error propagation"),
    }


def screen_packed_int8_attention_logits(package_dir: Any, *, seeds: Optional[Sequence[int]] = None,
                                        device: str = "auto", quantize_qk: bool = True, quantize_pv: bool = True,
                                        qk_bits: int = 8, qk_scale_mode: str = "calibrated-head",
                                        qk_multiplier_fraction_bits: int = 24, pv_probability_levels: int = 127,
                                        pv_probability_sum_correction: bool = False, pv_value_bits: int = 8,
                                        model: Any = None) -> Dict[str, object]:
    """Fixed-calibration INT8 attention propagated through all twelve
    otherwise floating-point folded blocks to the masked positions' logits
    (attention_int8.py:689-936)."""
    import torch
    import torch.nn.functional as F

    from .model import fp32_forward

    selected = [101, 202, 303, 404, 505] if seeds is None else list(seeds)
    if not selected:
        raise ValueError("at least one logit-screen seed is required")
    if not quantize_qk and not quantize_pv:
        raise ValueError("at least one attention matrix phase must be quantized")
    package_dir = Path(package_dir)
    goldens, tables = _attention_boundary_inputs(package_dir, [])
    cosine, sine = tables["rotary.cos"].float(), tables["rotary.sin"].float()
    dev = "cuda" if device == "auto" else device
    lut = _exponential_table()
    calibrations = _package_calibrations(goldens, cosine, sine, dev)
    folded = _folded(model)
    mask = int(folded.config.vocab_size) - 1
    head_w = torch.from_numpy(folded.head.weight)
    head_b = torch.from_numpy(folded.head.bias)

    def candidate_attention(block: int, normalized: Any, qkv: Any) -> Any:
        cand, _, _ = _evaluate_with_fixed_maxima(
            qkv.detach().cpu()[0], cosine, sine, calibrations[block], lut, quantize_qk=quantize_qk,
            quantize_pv=quantize_pv, qk_bits=qk_bits, qk_scale_mode=qk_scale_mode,
            qk_multiplier_fraction_bits=qk_multiplier_fraction_bits, pv_probability_levels=pv_probability_levels,
            pv_probability_sum_correction=pv_probability_sum_correction, pv_value_bits=pv_value_bits, device=dev)
        return cand.to(torch.float32)[None] / 4096.0

    samples = []
    with torch.inference_mode():
        for seed in selected:
            ids = _half_masked_canvas(seed, mask).numpy()
            base_h = torch.from_numpy(fp32_forward(folded, ids))
            cand_h = torch.from_numpy(fp32_forward(folded, ids, attention=candidate_attention))
            baseline = F.linear(base_h, head_w, head_b)[0, 1::2].float()
            candidate = F.linear(cand_h, head_w, head_b)[0, 1::2].float()
            baseline[:, mask] = -torch.inf
            candidate[:, mask] = -torch.inf
            fb = torch.where(torch.isfinite(baseline), baseline, torch.zeros_like(baseline))
            fc = torch.where(torch.isfinite(candidate), candidate, torch.zeros_like(candidate))
            diff = fc - fb
            blp = torch.log_softmax(baseline, dim=-1)
            clp = torch.log_softmax(candidate, dim=-1)
            bp, cp = blp.exp(), clp.exp()
            tv = 0.5 * (bp - cp).abs().sum(dim=-1)
            delta = torch.where(bp > 0, blp - clp, torch.zeros_like(blp))
            kl = (bp * delta).sum(dim=-1)
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
                "mean_kl_divergence_nats": float(kl.mean().item()),
                "maximum_kl_divergence_nats": float(kl.max().item()),
            })
    total = sum(s["masked_positions"] for s in samples)
    matches = sum(s["top1_matches"] for s in samples)
    return {
        "artifact": "error-propagating packed INT8 attention logit screen",
        "quantized_phases": {
            "query_key": quantize_qk,
            "probability_value": quantize_pv,
            "query_key_bits": qk_bits if quantize_qk else 18,
            "query_key_scale_mode": qk_scale_mode if quantize_qk else "fixed18",
            "query_key_multiplier_fraction_bits": qk_multiplier_fraction_bits if quantize_qk else 0,
            "probability_levels": pv_probability_levels if quantize_pv else 65535,
            "probability_sum_correction": pv_probability_sum_correction if quantize_pv else False,
            "value_bits": pv_value_bits if quantize_pv else 18,
        },
        "device": dev,
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
                  "selected INT8 attention error propagated through all twelve "
                  "otherwise floating-point folded blocks"),
    }
