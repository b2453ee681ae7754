"""Prefix-conditioned generation with prefix K/V reuse, and the drift report.

Generation follows conditioned._run_conditioned_ddpm_candidate_cache
(conditioned.py:132-242): the candidate-cache loop runs over the suffix only,
while every forward attends over [prefix ; suffix] keys.  The prefix K/V of all
blocks are computed once by an isolated prefix forward (prefix queries see the
prefix only: the prefix_isolation semantics, mdlm.py:45-58) and written into
per-block K / V buffers that the suffix forwards extend in place
(prefix_drift._cached_suffix_forward, prefix_drift.py:155-238), so clean
prefix positions are never recomputed.

Under full bidirectional attention the prefix K/V would drift once the suffix
changes; `drift_report` measures that drift against a full recompute with
tensor_drift_metrics (prefix_drift.py:26-55).
"""

from __future__ import annotations

import math
from typing import Any, Dict, List, Optional

import numpy as np

from .engine import MDLMEngine
from .model import QuantizedMDLM


def tensor_drift_metrics(reference: Any, changed: Any) -> Dict[str, object]:
    """Scalar drift metrics of two same-shaped tensors (prefix_drift.py:26-55)."""
    import torch

    if tuple(reference.shape) != tuple(changed.shape):
        raise ValueError("drift tensors must have the same shape")
    # computed where the tensors live (fp32), so large device tensors stay put
    reference = reference.detach().float()
    changed = changed.detach().float().to(reference.device)
    difference = changed - reference
    reference_rms = reference.square().mean().sqrt()
    rmse = difference.square().mean().sqrt()
    denominator = reference.flatten().norm() * changed.flatten().norm()
    cosine = torch.tensor(1.0, device=reference.device)
    if float(denominator.item()) > 0:
        cosine = (torch.dot(reference.flatten(), changed.flatten()) / denominator).clamp(-1.0, 1.0)
    return {
        "exact_equal": bool(torch.equal(reference, changed)),
        "cosine_similarity": float(cosine.item()),
        "mean_absolute_error": float(difference.abs().mean().item()),
        "max_absolute_error": float(difference.abs().max().item()),
        "normalized_rmse": float((rmse / reference_rms).item()) if float(reference_rms.item()) > 0 else math.inf,
        "fraction_changed_gt_1e_6": float(difference.abs().gt(1e-6).float().mean().item()),
    }


class PrefixConditionedGenerator:
    """B sequences of a clean prefix (P positions) and a generated suffix (S)."""

    def __init__(self, qm: QuantizedMDLM, batch: int, prefix_len: int, suffix_len: int,
                 device: Any = "cuda") -> None:
        self.qm = qm
        self.B, self.P, self.S = batch, prefix_len, suffix_len
        self.kv = MDLMEngine.kv_cache(qm, batch, prefix_len + suffix_len, device)
        self.prefix = MDLMEngine(qm, batch, prefix_len, device, kv_len=prefix_len, kv_buffers=self.kv)
        self.suffix = MDLMEngine(qm, batch, suffix_len, device, pos_offset=prefix_len,
                                 kv_len=prefix_len + suffix_len, kv_offset=prefix_len, kv_buffers=self.kv)
        self.prefix_forwards = 0

    def set_prefix(self, prefix_ids: Any) -> None:
        """Compute and keep the prefix K/V of every block (one forward)."""
        import torch

        self.prefix.tokens.copy_(prefix_ids.to(self.prefix.device, torch.int32).reshape(-1))
        self.prefix.forward()
        self.prefix_forwards += 1

    def generate(self, prefix_ids: Any, suffix_ids: Any, *, steps: int, seed: int = 0,
                 graph: bool = False) -> tuple[Any, dict]:
        self.set_prefix(prefix_ids)
        out, _ = self.suffix.generate(suffix_ids, steps=steps, seed=seed, graph=graph)
        meta = self.suffix.metadata(steps)
        mask = self.qm.config.mask_token_id
        meta.update({
            "prefix_forwards": self.prefix_forwards,
            "prefix_kv_reused_evaluations": meta["model_evaluations"],
            "all_tokens_committed": not bool((out == mask).any().item()),
        })
        return out, meta

    def drift_report(self, prefix_ids: Any, suffix_ids: Any) -> Dict[str, object]:
        """Per-block drift of the isolated prefix K/V against the K/V a full
        bidirectional forward over [prefix ; suffix] gives the prefix rows."""
        import torch

        qm, B, P, S = self.qm, self.B, self.P, self.S
        full = MDLMEngine(qm, B, P + S, self.prefix.device)
        full.tokens.copy_(torch.cat([prefix_ids, suffix_ids], dim=1).to(full.device, torch.int32).reshape(-1))
        layers = []
        k_full, vt_full = full.kv_buffers[0]

        def hook(i: int) -> None:
            k_iso, vt_iso = self.kv[i]
            layers.append({
                "layer": i,
                "key": tensor_drift_metrics(k_iso[:, :, :P], k_full[:, :, :P]),
                "value": tensor_drift_metrics(vt_iso[:, :, :, :P], vt_full[:, :, :, :P]),
            })

        full.forward(hook=hook)
        first = next((l["layer"] for l in layers if not (l["key"]["exact_equal"] and l["value"]["exact_equal"])),
                     None)
        return {"layers": layers, "first_drifting_layer": first,
                "all_prefix_kv_exact_equal": first is None}


def timed_ms(operation: Any, repeats: int) -> tuple:
    """(median ms, samples ms) of `operation` timed with CUDA events on the
    current stream, one sample per call."""
    import statistics

    import torch

    samples = []
    out = None
    for _ in range(repeats):
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        out = operation()
        end.record()
        end.synchronize()
        samples.append(float(start.elapsed_time(end)))
    return out, statistics.median(samples), samples


def top1_ids(logits: Any, mask_token_id: int) -> Any:
    """argmax over the vocabulary with the mask token excluded
    (prefix_drift._top1_ids, prefix_drift.py:125-128)."""
    logits = logits.detach().float().clone()
    logits[..., mask_token_id] = -math.inf
    return logits.argmax(dim=-1)


def analyze_mdlm_prefix_drift(*, quantized: Optional[QuantizedMDLM] = None, prefix_ids: Any = None,
                              prefix_tokens: int = 64, suffix_tokens: int = 32, changed_suffix_tokens: int = 1,
                              warmup: int = 1, timing_repeats: int = 5, seed: int = 0,
                              weights_seed: int = 0, device: Any = "cuda") -> Dict[str, object]:
    """Fixed-prefix K/V drift after a suffix edit, on the B200 engines
    (prefix_drift.analyze_mdlm_prefix_drift, prefix_drift.py:282-577).

    Baseline = [prefix ; masked suffix]; changed = the same with
    `changed_suffix_tokens` suffix positions replaced (the reference's draws:
    randint ids, then randperm positions, from Generator(seed)).  Under full
    bidirectional attention the per-block prefix K / V of both are compared
    with tensor_drift_metrics.  Under prefix isolation the prefix K / V come
    from the isolated prefix forward: the suffix cannot reach them, and the
    cached-suffix logits are compared with a recompute of prefix and suffix.
    Captured operands are the attention inputs as stored: post-rotary K and
    smoothing-scaled V^T, bf16.  Without a checkpoint the model is the
    random-init stand-in (seeded); without a tokenizer the prefix is
    `prefix_ids` or seeded uniform ids.  Lengths are multiples of 32."""
    import torch

    from .model import MDLMConfig, build_quantized

    if suffix_tokens <= 0:
        raise ValueError("suffix_tokens must be positive")
    if changed_suffix_tokens <= 0 or changed_suffix_tokens > suffix_tokens:
        raise ValueError("changed_suffix_tokens must be in [1, suffix_tokens]")
    if warmup < 0:
        raise ValueError("warmup must be non-negative")
    if timing_repeats <= 0:
        raise ValueError("timing_repeats must be positive")
    qm = quantized if quantized is not None else build_quantized(MDLMConfig(), seed=weights_seed)
    cfg = qm.config
    mask = cfg.mask_token_id
    if prefix_ids is None:
        g = torch.Generator().manual_seed(seed + 2)
        prefix_ids = torch.randint(0, mask, (prefix_tokens,), generator=g)
    prefix_ids = torch.as_tensor(prefix_ids, dtype=torch.long).reshape(-1).cpu()
    P, S = int(prefix_ids.numel()), suffix_tokens
    if P % 32 or S % 32:
        raise ValueError("prefix and suffix lengths must be multiples of 32")
    if P + S > cfg.max_positions:
        raise ValueError(f"prefix and suffix exceed the model length {cfg.max_positions}")

    baseline_ids = torch.cat([prefix_ids, torch.full((S,), mask, dtype=torch.long)]).unsqueeze(0)
    changed_ids = baseline_ids.clone()
    generator = torch.Generator(device="cpu").manual_seed(seed)
    replacement_ids = torch.randint(0, mask, (changed_suffix_tokens,), generator=generator, dtype=torch.long)
    changed_positions = torch.randperm(S, generator=generator)[:changed_suffix_tokens].sort().values
    changed_ids[0, P + changed_positions] = replacement_ids

    full = MDLMEngine(qm, 1, P + S, device)
    dev = full.device

    def run_full(ids: Any, capture: Optional[list] = None) -> None:
        full.tokens.copy_(ids.reshape(-1).to(dev, torch.int32))

        def hook(i: int) -> None:
            k, vt = full.kv_buffers[i]
            capture.append((k[:, :, :P].clone(), vt[:, :, :, :P].clone()))

        full.forward(hook=hook if capture is not None else None)

    # forwards are timed without the (debug) logits materialisation
    for _ in range(warmup):
        run_full(baseline_ids)
    torch.cuda.synchronize()
    _, baseline_ms, baseline_samples = timed_ms(lambda: run_full(baseline_ids), timing_repeats)
    _, changed_ms, changed_samples = timed_ms(lambda: run_full(changed_ids), timing_repeats)
    baseline_kv: list = []
    changed_kv: list = []
    run_full(baseline_ids, baseline_kv)
    baseline_logits = full.logits()
    run_full(changed_ids, changed_kv)
    changed_logits = full.logits()

    layers = []
    first_drifting_layer = None
    for i, ((kb, vb), (kc, vc)) in enumerate(zip(baseline_kv, changed_kv)):
        key_metrics = tensor_drift_metrics(kb, kc)
        value_metrics = tensor_drift_metrics(vb, vc)
        exact = bool(key_metrics["exact_equal"] and value_metrics["exact_equal"])
        if not exact and first_drifting_layer is None:
            first_drifting_layer = i
        layers.append({"layer": i, "prefix_kv_exact_equal": exact, "key": key_metrics, "value": value_metrics})

    # prefix isolation: isolated prefix forward once, suffix forwards reuse it
    gen = PrefixConditionedGenerator(qm, 1, P, S, device)
    suffix_changed = changed_ids[:, P:]
    suffix_baseline = baseline_ids[:, P:]

    def suffix_forward(ids: Any) -> None:
        gen.suffix.tokens.copy_(ids.reshape(-1).to(dev, torch.int32))
        gen.suffix.forward()

    def recompute(ids: Any) -> None:
        gen.set_prefix(prefix_ids.unsqueeze(0))
        suffix_forward(ids)

    recompute(suffix_changed)  # warm both engines
    torch.cuda.synchronize()
    _, isolated_ms, isolated_samples = timed_ms(lambda: recompute(suffix_changed), timing_repeats)
    isolated_logits = gen.suffix.logits()
    _, prefill_ms, prefill_samples = timed_ms(lambda: gen.set_prefix(prefix_ids.unsqueeze(0)), timing_repeats)
    iso_before = [(k[:, :, :P].clone(), vt[:, :, :, :P].clone()) for k, vt in gen.kv]
    suffix_forward(suffix_baseline)
    iso_baseline = [(k[:, :, :P].clone(), vt[:, :, :, :P].clone()) for k, vt in gen.kv]
    _, cached_ms, cached_samples = timed_ms(lambda: suffix_forward(suffix_changed), timing_repeats)
    cached_logits = gen.suffix.logits()
    isolated_prefix_exact = all(torch.equal(a[0], b[0]) and torch.equal(a[1], b[1]) and
                                torch.equal(a[0], k[:, :, :P]) and torch.equal(a[1], vt[:, :, :, :P])
                                for a, b, (k, vt) in zip(iso_before, iso_baseline, gen.kv))

    baseline_top1 = top1_ids(baseline_logits, mask)
    changed_top1 = top1_ids(changed_logits, mask)
    isolated_top1 = top1_ids(isolated_logits, mask)
    cached_top1 = top1_ids(cached_logits, mask)

    def agreement(a: Any, b: Any) -> float:
        return float(a.eq(b).float().mean().item())

    return {
        "model": "random-init MDLM-169.6M stand-in, W8A8" if quantized is None else "supplied",
        "weights_seed": weights_seed,
        "device": torch.cuda.get_device_name(dev),
        "attention_policy": "full-bidirectional",
        "capture_point": "post-rotary key and smoothing-scaled value, bf16 attention operands",
        "seed": seed,
        "prefix_tokens": P,
        "suffix_tokens": S,
        "changed_suffix_tokens": changed_suffix_tokens,
        "changed_absolute_positions": [P + int(p) for p in changed_positions.tolist()],
        "replacement_token_ids": replacement_ids.tolist(),
        "baseline_forward_latency_ms": baseline_ms,
        "baseline_forward_latency_samples_ms": baseline_samples,
        "changed_forward_latency_ms": changed_ms,
        "changed_forward_latency_samples_ms": changed_samples,
        "prefix_logits_top1_agreement": agreement(baseline_top1[0, :P], changed_top1[0, :P]),
        "suffix_logits_top1_agreement": agreement(baseline_top1[0, P:], changed_top1[0, P:]),
        "first_drifting_layer": first_drifting_layer,
        "all_prefix_kv_exact_equal": first_drifting_layer is None,
        "vanilla_prefix_kv_reuse_is_exact": first_drifting_layer is None,
        "layers": layers,
        "prefix_isolated_cache_experiment": {
            "latency_measurement": "CUDA events, median of timing_repeats after warm-up",
            "all_prefix_kv_exact_equal_after_suffix_edit": bool(isolated_prefix_exact),
            "full_recompute_latency_ms": isolated_ms,
            "full_recompute_latency_samples_ms": isolated_samples,
            "one_time_prefix_prefill_latency_ms": prefill_ms,
            "one_time_prefix_prefill_latency_samples_ms": prefill_samples,
            "cached_suffix_latency_ms": cached_ms,
            "cached_suffix_latency_samples_ms": cached_samples,
            "suffix_top1_agreement": agreement(isolated_top1, cached_top1),
            "suffix_logit_drift": tensor_drift_metrics(isolated_logits, cached_logits),
        },
    }
