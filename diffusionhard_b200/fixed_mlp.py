"""RTL integer arithmetic of the MLP on the B200 tensor engine.

Drop-ins for the reference's fixed-point MLP functions
(src/diffusion_accel/fixed_mlp.py):

* ``hardware_requantized_linear`` (:139-224) -- W8A8 MACs with the RTL integer
  requantisation (24-bit per-(token, output) multipliers, rounding right
  shift, Q10 bias, saturating output width);
* ``factorize_up_requant_scales`` (:327-392) and
  ``requantized_linear_factorized`` -- the same requantisation with the
  multipliers built from two small integer factor vectors;
* ``hardware_gelu_q10`` (:227-247) -- the Q5.10 GELU lookup with its bypass
  rules.

The SmoothQuant / symmetric-quantisation preparation is O(rows x cols) host
torch arithmetic, the same operations as the reference so that the int8
operands are identical.  The O(m x n x k) part -- int8 tensor-core MACs and
the integer requantisation of every output -- runs on the GPU in one kernel
(``dh_gemm_i8_requant``), as does the GELU lookup (``dh_gelu_q10``).
"""

from __future__ import annotations

import math
from typing import Any, Dict, List, Tuple

from . import _lib

INT64_MAX = (1 << 63) - 1
INT64_MIN = -(1 << 63)


def _quantize_symmetric(tensor: Any, bits: int, granularity: str) -> Tuple[Any, Any]:
    """Symmetric per-tensor or per-row quantisation (fixed_mlp.py:11-35)."""
    import torch

    if bits not in {8, 16}:
        raise ValueError("fixed MLP validation supports 8 or 16 bits")
    limit = (1 << (bits - 1)) - 1
    if granularity == "tensor":
        maximum = tensor.abs().max()
    elif granularity == "token":
        if tensor.ndim != 2:
            raise ValueError("token activation quantization expects a matrix")
        maximum = tensor.abs().amax(dim=1)
    else:
        raise ValueError("activation granularity must be tensor or token")
    scale = torch.where(maximum > 0, maximum / float(limit), torch.ones_like(maximum))
    divisor = scale if scale.ndim == 0 else scale[:, None]
    quantized = torch.round(tensor / divisor).clamp(-limit, limit)
    return quantized.to(torch.int8 if bits == 8 else torch.int16), scale


def _quantize_weight_per_output(tensor: Any, bits: int) -> Tuple[Any, Any]:
    """Symmetric per-output-row weight quantisation (fixed_mlp.py:38-52)."""
    import torch

    if bits not in {8, 16}:
        raise ValueError("fixed MLP validation supports 8 or 16 bits")
    limit = (1 << (bits - 1)) - 1
    maximum = tensor.abs().amax(dim=1)
    scales = torch.where(maximum > 0, maximum / float(limit), torch.ones_like(maximum))
    quantized = torch.round(tensor / scales[:, None]).clamp(-limit, limit)
    return quantized.to(torch.int8 if bits == 8 else torch.int16), scales


def _padded_int8(q: Any, k16: int, device: Any) -> Any:
    """int8 [rows, k] -> contiguous device int8 [rows, k16] (zero columns
    add nothing to the products; the tensor engine wants k % 16 == 0)."""
    import torch

    out = torch.zeros((q.shape[0], k16), dtype=torch.int8, device=device)
    out[:, : q.shape[1]] = q.to(device)
    return out


def _run_requant(aq: Any, wq: Any, *, mode: int, a_scale: Any = None, a_stride: int = 1, w_scale: Any = None,
                 token_factor: Any = None, output_factor: Any = None, factor_shift: int = 0, bias_q: Any,
                 right_shift: int, frac_bits: int, output_width: int, device: Any) -> Tuple[Any, List[int]]:
    import torch

    m, k = aq.shape
    n = wq.shape[0]
    k16 = max(16, -(-k // 16) * 16)
    a_dev = _padded_int8(aq, k16, device)
    w_dev = _padded_int8(wq, k16, device)
    out = torch.empty((m, n), dtype=torch.int32, device=device)
    stats = torch.tensor([INT64_MAX, INT64_MIN, 0, 0], dtype=torch.int64, device=device)
    dev32 = lambda t, dt: None if t is None else t.to(device=device, dtype=dt).contiguous()  # noqa: E731
    a_s = dev32(a_scale, torch.float32)
    w_s = dev32(w_scale, torch.float32)
    tf = dev32(token_factor, torch.int32)
    of = dev32(output_factor, torch.int32)
    bq = dev32(bias_q, torch.int32)
    _lib.call("dh_gemm_i8_requant", _lib.ptr(a_dev), _lib.ptr(w_dev), m, n, k16, mode, _lib.ptr(a_s), a_stride,
              _lib.ptr(w_s), _lib.ptr(tf), _lib.ptr(of), factor_shift, _lib.ptr(bq), right_shift, frac_bits,
              output_width, _lib.ptr(out), _lib.ptr(stats), _lib.stream_handle())
    return out, stats.cpu().tolist()


def hardware_requantized_linear(
    activation: Any,
    weight: Any,
    bias: Any,
    *,
    activation_granularity: str,
    smoothquant_alpha: float,
    output_width: int,
    output_fraction_bits: int = 10,
    right_shift: int = 20,
    multiplier_bits: int = 24,
    device: Any = "cuda",
) -> Tuple[Any, Any, Dict[str, object]]:
    """W8A8 MACs and the RTL integer requantisation (fixed_mlp.py:139-224);
    same arguments, outputs (on the activation's device) and metrics."""
    import torch

    if not 0.0 <= smoothquant_alpha <= 1.0:
        raise ValueError("SmoothQuant alpha must be between zero and one")
    if output_width <= output_fraction_bits + 1:
        raise ValueError("output width must include sign and integer bits")
    if right_shift <= 0 or multiplier_bits <= 0:
        raise ValueError("right shift and multiplier bits must be positive")
    if output_width > 32:
        raise ValueError("the device output is int32: output_width must be at most 32")
    activation_max = activation.abs().amax(dim=0).clamp_min(1e-8)
    weight_max = weight.abs().amax(dim=0).clamp_min(1e-8)
    smoothing_scale = (activation_max.pow(smoothquant_alpha) /
                       weight_max.pow(1.0 - smoothquant_alpha)).clamp_min(1e-8)
    activation_q, activation_scale = _quantize_symmetric(activation / smoothing_scale[None, :], 8,
                                                         activation_granularity)
    weight_q, weight_scales = _quantize_weight_per_output(weight * smoothing_scale[None, :], 8)
    bias_q = torch.round(bias.double() * (1 << output_fraction_bits)).to(torch.int64)
    if int(bias_q.abs().max().item()) >= 1 << 31:
        raise ValueError("bias exceeds the int32 range in the output format")

    # the multipliers' range follows from the scale vectors: fp32 products of
    # positive scales and the rounding are monotonic in each factor
    scale_mult = float(1 << (right_shift + output_fraction_bits))
    a_vec = activation_scale.reshape(-1).float()

    def mult_of(a: Any, w: Any) -> int:
        return int(torch.round((a.float() * w.float()).double() * scale_mult).item())

    mult_min = mult_of(a_vec.min(), weight_scales.min())
    mult_max = mult_of(a_vec.max(), weight_scales.max())
    if mult_max > (1 << multiplier_bits) - 1:
        raise ValueError("requant multiplier exceeds configured unsigned width")

    out, stats = _run_requant(activation_q, weight_q, mode=0, a_scale=a_vec,
                              a_stride=0 if activation_scale.ndim == 0 else 1, w_scale=weight_scales,
                              bias_q=bias_q, right_shift=right_shift, frac_bits=output_fraction_bits,
                              output_width=output_width, device=device)
    output_q = out.to(torch.int64).to(activation.device)
    output = output_q.double() / float(1 << output_fraction_bits)
    return output.float(), output_q, {
        "activation_granularity": activation_granularity,
        "output_width": output_width,
        "output_fraction_bits": output_fraction_bits,
        "right_shift": right_shift,
        "multiplier_bits": multiplier_bits,
        "multiplier_min": mult_min,
        "multiplier_max": mult_max,
        "required_unsigned_multiplier_bits": max(1, mult_max.bit_length()),
        "output_saturation_fraction": stats[2] / float(out.numel()),
        "activation_scale_min": float(activation_scale.min().item()),
        "activation_scale_max": float(activation_scale.max().item()),
        "weight_scale_min": float(weight_scales.min().item()),
        "weight_scale_max": float(weight_scales.max().item()),
        "smoothquant_scale_min": float(smoothing_scale.min().item()),
        "smoothquant_scale_max": float(smoothing_scale.max().item()),
        "accumulator_min": stats[0],
        "accumulator_max": stats[1],
    }


def factorize_up_requant_scales(
    token_scales: Any,
    output_scales: Any,
    *,
    token_fraction_bits: int = 18,
    output_fraction_bits: int = 20,
    combined_fraction_bits: int = 30,
    token_factor_bits: int = 16,
    output_factor_bits: int = 18,
    multiplier_bits: int = 24,
) -> Tuple[Any, Dict[str, Any], Dict[str, object]]:
    """Token x output requant multipliers from two small integer factor
    vectors (fixed_mlp.py:327-392): mult = (tf * of + 2^(s-1)) >> s with
    s = token + output - combined fraction bits.  Integer tensor arithmetic on
    the scales' device; same outputs and metrics as the reference."""
    import torch

    factor_shift = token_fraction_bits + output_fraction_bits - combined_fraction_bits
    if factor_shift <= 0:
        raise ValueError("factor fractions must exceed combined fraction bits")
    token_factors = torch.round(token_scales.double() * (1 << token_fraction_bits)).to(torch.int64)
    output_factors = torch.round(output_scales.double() * (1 << output_fraction_bits)).to(torch.int64)
    if int(token_factors.max().item()) >= (1 << token_factor_bits):
        raise ValueError("token factor exceeds configured width")
    if int(output_factors.max().item()) >= (1 << output_factor_bits):
        raise ValueError("output factor exceeds configured width")
    multipliers = (token_factors[:, None] * output_factors[None, :] + (1 << (factor_shift - 1))) >> factor_shift
    if int(multipliers.max().item()) >= (1 << multiplier_bits):
        raise ValueError("factorized multiplier exceeds configured width")
    reference = torch.round(token_scales.double()[:, None] * output_scales.double()[None, :] *
                            (1 << combined_fraction_bits)).to(torch.int64)
    relative_error = (multipliers - reference).abs().double() / reference.clamp_min(1).double()
    tensors = {
        "token_factor": token_factors.to(torch.int32).contiguous(),
        "output_factor": output_factors.to(torch.int32).contiguous(),
    }
    metrics = {
        "token_fraction_bits": token_fraction_bits,
        "output_fraction_bits": output_fraction_bits,
        "combined_fraction_bits": combined_fraction_bits,
        "factor_shift": factor_shift,
        "token_factor_bits": token_factor_bits,
        "output_factor_bits": output_factor_bits,
        "token_factor_min": int(token_factors.min().item()),
        "token_factor_max": int(token_factors.max().item()),
        "output_factor_min": int(output_factors.min().item()),
        "output_factor_max": int(output_factors.max().item()),
        "maximum_multiplier_relative_error": float(relative_error.max().item()),
        "mean_multiplier_relative_error": float(relative_error.mean().item()),
        "exact_multiplier_fraction": float(multipliers.eq(reference).float().mean().item()),
    }
    return multipliers, tensors, metrics


def requantized_linear_factorized(activation_q: Any, weight_q: Any, token_factor: Any, output_factor: Any,
                                  factor_shift: int, bias_q: Any, *, output_width: int, right_shift: int = 20,
                                  output_fraction_bits: int = 10, device: Any = "cuda") -> Tuple[Any, List[int]]:
    """int8 activations x int8 weights requantised with the factorised
    multipliers (mode 1 of dh_gemm_i8_requant): out int64 [rows, outputs] on
    the activation's device, and the statistics [min acc, max acc, saturated
    outputs, max multiplier]."""
    import torch

    out, stats = _run_requant(activation_q, weight_q, mode=1, token_factor=token_factor,
                              output_factor=output_factor, factor_shift=factor_shift, bias_q=bias_q,
                              right_shift=right_shift, frac_bits=output_fraction_bits, output_width=output_width,
                              device=device)
    return out.to(torch.int64).to(activation_q.device), stats


def gelu_q10_table() -> List[int]:
    """The 1024-entry Q5.10 GELU lookup of the RTL (fixed_mlp.py:231-241):
    entry a holds round(1024 * gelu(x)) at x = (-8192 + 16 a) / 1024, with the
    tanh form of GELU evaluated in double precision."""
    c = math.sqrt(2.0 / math.pi)
    table = []
    for address in range(1024):
        x = (-8192 + (address << 4)) / 1024.0
        table.append(round(0.5 * x * (1.0 + math.tanh(c * (x + 0.044715 * x ** 3))) * 1024.0))
    return table


_GELU_TABLES: Dict[str, Any] = {}


def hardware_gelu_q10(input_q: Any, device: Any = "cuda") -> Tuple[Any, Any]:
    """The RTL Q5.10 GELU lookup and bypass rules (fixed_mlp.py:227-247) on
    the GPU; returns (float output, int64 output) on the input's device."""
    import torch

    dev = torch.device(device)
    key = str(dev)
    if key not in _GELU_TABLES:
        _GELU_TABLES[key] = torch.tensor(gelu_q10_table(), dtype=torch.int32, device=dev)
    flat = input_q.reshape(-1)
    if flat.numel() and (int(flat.min().item()) < -(1 << 31) or int(flat.max().item()) >= 1 << 31):
        raise ValueError("input exceeds the int32 range")
    src = flat.to(device=dev, dtype=torch.int32).contiguous()
    out = torch.empty_like(src)
    _lib.call("dh_gelu_q10", _lib.ptr(src), _lib.ptr(out), src.numel(), _lib.ptr(_GELU_TABLES[key]),
              _lib.stream_handle())
    output_q = out.to(torch.int64).reshape(input_q.shape).to(input_q.device)
    return output_q.float() / 1024.0, output_q


def _error_metrics(actual: Any, expected: Any) -> Dict[str, float]:
    """Max / mean / RMS / relative RMS error and cosine similarity
    (fixed_mlp.py:500-517)."""
    import torch
    import torch.nn.functional as F

    a, e = actual.float().cpu(), expected.float().cpu()
    d = a - e
    rms = torch.sqrt(torch.mean(d.square()))
    cosine = float(F.cosine_similarity(a.reshape(1, -1), e.reshape(1, -1)).item())
    return {
        "max_abs_error": float(d.abs().max().item()),
        "mean_abs_error": float(d.abs().mean().item()),
        "rms_error": float(rms.item()),
        "relative_rms_error": float((rms / torch.sqrt(torch.mean(e.square()))).item()),
        "cosine_similarity": max(-1.0, min(1.0, cosine)),
    }


def _package_tensors(path: Any, names: List[str]) -> Dict[str, Any]:
    from safetensors import safe_open

    with safe_open(str(path), framework="pt", device="cpu") as handle:
        return {n: handle.get_tensor(n).float() for n in names}


Q13_10_MIN, Q13_10_MAX = -(1 << 23), (1 << 23) - 1
SWEEP_ALPHAS = (0.75, 0.5, 0.5, 0.75, 0.5, 0.5, 0.75, 0.5, 0.5, 0.5, 0.5, 0.75)


def validate_hardware_fixed_mlp(package_dir: Any, *, block: int = 0, activation_granularity: str = "token",
                                down_activation_granularity: Any = None, smoothquant_alpha: float = 0.75,
                                device: Any = "cuda") -> Dict[str, object]:
    """One folded MLP of a hardware package through the RTL integer path
    (fixed_mlp.validate_hardware_fixed_mlp, fixed_mlp.py:918-1036): the
    package's norm2 golden -> 16-bit Q5.10 up requant -> Q5.10 GELU lookup ->
    24-bit Q13.10 down requant -> saturating Q13.10 residual add, compared
    with the fp32 goldens.  The MACs and requantisation run on the GPU
    (dh_gemm_i8_requant, dh_gelu_q10); same report as the reference."""
    import torch
    from pathlib import Path

    package_dir = Path(package_dir)
    if not 0 <= block < 12:
        raise ValueError("block must be between 0 and 11")
    pre, wpre = "folded.block_%02d" % block, "block_%02d" % block
    g = _package_tensors(package_dir / "golden_tensors.safetensors",
                         [pre + s for s in (".norm2_unaffine", ".mlp_up", ".gelu", ".mlp_down", ".after_attention",
                                            ".output")])
    w = _package_tensors(package_dir / "folded_fp16_weights.safetensors",
                         [wpre + s for s in (".mlp_up.weight", ".mlp_up.bias", ".mlp_down.weight", ".mlp_down.bias")])
    down_gran = activation_granularity if down_activation_granularity is None else down_activation_granularity
    up, up_q, up_m = hardware_requantized_linear(g[pre + ".norm2_unaffine"][0], w[wpre + ".mlp_up.weight"],
                                                 w[wpre + ".mlp_up.bias"],
                                                 activation_granularity=activation_granularity,
                                                 smoothquant_alpha=smoothquant_alpha, output_width=16, device=device)
    gelu, gelu_q = hardware_gelu_q10(up_q, device=device)
    down, down_q, down_m = hardware_requantized_linear(gelu, w[wpre + ".mlp_down.weight"], w[wpre + ".mlp_down.bias"],
                                                       activation_granularity=down_gran,
                                                       smoothquant_alpha=smoothquant_alpha, output_width=24,
                                                       device=device)
    residual_unclipped = torch.round(g[pre + ".after_attention"][0].double() * 1024.0).to(torch.int64)
    residual_q = residual_unclipped.clamp(Q13_10_MIN, Q13_10_MAX)
    block_unclipped = residual_q + down_q
    block_q = block_unclipped.clamp(Q13_10_MIN, Q13_10_MAX)
    block_out = block_q.float() / 1024.0

    def sat(t: Any) -> float:
        return float(((t < Q13_10_MIN) | (t > Q13_10_MAX)).float().mean().item())

    return {
        "package_dir": str(package_dir),
        "block": block,
        "activation_granularity": activation_granularity,
        "down_activation_granularity": down_gran,
        "smoothquant_alpha": smoothquant_alpha,
        "formats": {"mlp_up": "signed-q5.10-16-bit", "gelu": "signed-q5.10-1024-entry-lut",
                    "mlp_down": "signed-q13.10-24-bit",
                    "residual_and_block_output": "signed-q13.10-24-bit-saturating"},
        "integer": {
            "mlp_up": up_m, "mlp_down": down_m,
            "mlp_up_q_min": int(up_q.min().item()), "mlp_up_q_max": int(up_q.max().item()),
            "gelu_q_min": int(gelu_q.min().item()), "gelu_q_max": int(gelu_q.max().item()),
            "mlp_down_q_min": int(down_q.min().item()), "mlp_down_q_max": int(down_q.max().item()),
            "residual_q_min": int(residual_q.min().item()), "residual_q_max": int(residual_q.max().item()),
            "residual_saturation_fraction": sat(residual_unclipped),
            "block_output_saturation_fraction": sat(block_unclipped),
        },
        "accuracy": {
            "mlp_up": _error_metrics(up, g[pre + ".mlp_up"][0]),
            "gelu": _error_metrics(gelu, g[pre + ".gelu"][0]),
            "mlp_down": _error_metrics(down, g[pre + ".mlp_down"][0]),
            "block_output": _error_metrics(block_out, g[pre + ".output"][0]),
        },
        "scope": ("one frozen H0 input with RTL-equivalent integer requantization "
                  "and GELU; generation quality and vendor timing are not established"),
    }


def sweep_hardware_fixed_mlp(package_dir: Any, *, activation_granularity: str = "token",
                             down_activation_granularity: Any = None, blocks: int = 12,
                             device: Any = "cuda") -> Dict[str, object]:
    """validate_hardware_fixed_mlp over the package's blocks with the
    reference's per-block alphas and summary (fixed_mlp.py:1039-1110)."""
    import statistics

    results = [validate_hardware_fixed_mlp(package_dir, block=b, activation_granularity=activation_granularity,
                                           down_activation_granularity=down_activation_granularity,
                                           smoothquant_alpha=SWEEP_ALPHAS[b], device=device)
               for b in range(blocks)]
    rel = [r["accuracy"]["block_output"]["relative_rms_error"] for r in results]
    return {
        "package_dir": str(package_dir),
        "activation_granularity": activation_granularity,
        "down_activation_granularity": (activation_granularity if down_activation_granularity is None
                                        else down_activation_granularity),
        "blocks": results,
        "summary": {
            "minimum_block_output_relative_rms": min(rel),
            "median_block_output_relative_rms": statistics.median(rel),
            "maximum_block_output_relative_rms": max(rel),
            "mean_block_output_relative_rms": statistics.mean(rel),
            "maximum_up_q5_10_saturation_fraction": max(
                r["integer"]["mlp_up"]["output_saturation_fraction"] for r in results),
            "maximum_down_q13_10_saturation_fraction": max(
                r["integer"]["mlp_down"]["output_saturation_fraction"] for r in results),
            "maximum_residual_q13_10_saturation_fraction": max(
                r["integer"]["residual_saturation_fraction"] for r in results),
            "maximum_block_output_q13_10_saturation_fraction": max(
                r["integer"]["block_output_saturation_fraction"] for r in results),
            "maximum_required_unsigned_multiplier_bits": max(
                r["integer"][layer]["required_unsigned_multiplier_bits"] for r in results
                for layer in ("mlp_up", "mlp_down")),
        },
        "scope": ("all checkpoint blocks on one frozen H0 input; errors are local "
                  "block comparisons and not composed generation quality"),
    }
