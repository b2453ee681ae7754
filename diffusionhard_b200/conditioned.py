"""Prefix-conditioned generation compared across three attention paths, on
the B200 engines (conditioned.evaluate_conditioned_mdlm_ddpm,
src/diffusion_accel/conditioned.py:295-650).

Per sample, a window of prefix + target suffix tokens; the suffix starts
fully masked and the candidate-cache loop generates it with:

* ``original_full_attention``: one engine over the whole [prefix ; suffix]
  canvas, so the prefix attends to the suffix (prefix K / V drift);
* ``prefix_isolated_recompute``: the prefix forward (prefix attends to the
  prefix only) recomputed with every model evaluation, then the suffix
  forward over [prefix ; suffix] keys;
* ``prefix_isolated_cache``: the prefix K / V computed once and reused by
  every suffix forward (prefix_drift._cached_suffix_forward,
  prefix_drift.py:155-238).

Randomness is keyed by canvas position and sequence, so the three paths draw
the same noise and reveal words.  The reference reseeds torch's RNG per path
for the same purpose.  Recompute and cache must then agree token for token:
the prefix K / V are a deterministic function of the prefix.

Without the dataset and tokenizer, windows are seeded uniform token ids, and
the target agreement only measures chance.  Without a checkpoint, the model
is the random-init stand-in.
"""

from __future__ import annotations

import statistics
from typing import Any, Dict, Optional

from .engine import MDLMEngine
from .model import MDLMConfig, QuantizedMDLM, build_quantized
from .prefix import PrefixConditionedGenerator
from .sampler import reveal_thresholds_q32


def _terminal_kv_valid(meta: Dict[str, Any], counters: Any, steps: int) -> bool:
    """True when no token changed after the last model evaluation, so the
    K / V of that evaluation describe the final canvas
    (conditioned.py:226-229)."""
    n = meta["sampling_transitions"]
    rows = counters.view(steps, 3).cpu().tolist()[:n]
    remaining = rows[-1][0] - rows[-1][1] if n else 0
    if remaining > 0:
        return False  # the final greedy pass evaluates, then fills the rest
    last_eval = max((k for k in range(n) if rows[k][2]), default=-1)
    return last_eval >= 0 and all(rows[k][1] == 0 for k in range(last_eval, n))


def _path_result(generated: Any, target: Any, meta: Dict[str, Any], forward_ms: list,
                 wall_ms: float, terminal_kv_valid: bool) -> Dict[str, object]:
    return {
        **meta,
        "wall_latency_ms": wall_ms,
        "model_forward_latency_ms": float(sum(forward_ms)),
        "median_model_evaluation_latency_ms": statistics.median(forward_ms) if forward_ms else 0.0,
        "terminal_kv_valid": terminal_kv_valid,
        "target_token_agreement": float(generated.eq(target).float().mean().item()),
        "generated_token_ids": generated[0].detach().cpu().tolist(),
    }


def _gate(fwd_rows: Any, rows: int, out: Any) -> Any:
    """Device word `rows` when the suffix forward runs (*fwd_rows != 0), else 0."""
    import torch

    torch.mul(torch.clamp(fwd_rows.view(torch.int32), max=1), rows, out=out)
    return out


def _timed_transitions(engine: MDLMEngine, steps: int, seed: int) -> tuple:
    """Run one generation transition by transition, timing every model
    evaluation (CUDA events around the transition that ran a forward).
    Returns (wall ms, per-evaluation ms)."""
    import torch

    thresholds = reveal_thresholds_q32(steps)
    evals = []
    wall0, wall1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    wall0.record()
    for k in range(steps + 1):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        engine.enqueue_transition(k, steps, seed, thresholds[k] if k < steps else 0)
        b.record()
        evals.append((a, b))
    wall1.record()
    wall1.synchronize()
    counters = engine.counters.view(steps, 3).cpu().tolist()
    meta = engine.metadata(steps)
    n = meta["sampling_transitions"]
    per_eval = [evals[k][0].elapsed_time(evals[k][1]) for k in range(n) if counters[k][2]]
    remaining = counters[n - 1][0] - counters[n - 1][1] if n else 0
    if remaining > 0:
        per_eval.append(evals[steps][0].elapsed_time(evals[steps][1]))
    return float(wall0.elapsed_time(wall1)), [float(x) for x in per_eval]


def evaluate_conditioned_mdlm_ddpm(*, quantized: Optional[QuantizedMDLM] = None, prefix_tokens: int = 64,
                                   suffix_tokens: int = 32, samples: int = 3, steps: int = 64, seed: int = 0,
                                   weights_seed: int = 0, windows: Any = None,
                                   device: Any = "cuda") -> Dict[str, object]:
    """Original / isolated-recompute / isolated-cache conditioned generation
    (conditioned.py:295-650).  `windows` optionally supplies [samples,
    prefix + suffix] token ids; lengths are multiples of 32."""
    import torch

    if min(prefix_tokens, suffix_tokens, samples, steps) <= 0:
        raise ValueError("token counts, samples, and steps must be positive")
    if prefix_tokens % 32 or suffix_tokens % 32:
        raise ValueError("prefix_tokens and suffix_tokens must be multiples of 32")
    qm = quantized if quantized is not None else build_quantized(MDLMConfig(), seed=weights_seed)
    cfg = qm.config
    P, S = prefix_tokens, suffix_tokens
    if P + S > cfg.max_positions:
        raise ValueError("conditioned sequence exceeds the model length")
    mask = cfg.mask_token_id
    synthetic_windows = windows is None
    if windows is None:
        g = torch.Generator().manual_seed(seed + 2)
        windows = torch.randint(0, mask, (samples, P + S), generator=g)
    windows = torch.as_tensor(windows, dtype=torch.long)
    if tuple(windows.shape) != (samples, P + S):
        raise ValueError("windows must be [samples, prefix_tokens + suffix_tokens]")

    full = MDLMEngine(qm, 1, P + S, device)
    dev = full.device
    gen = PrefixConditionedGenerator(qm, 1, P, S, device)
    suffix = gen.suffix
    prefix_gate = torch.zeros(1, dtype=torch.int32, device=dev)

    sample_results = []
    for index in range(samples):
        sample_seed = seed + index
        prefix_ids = windows[index : index + 1, :P]
        target = windows[index : index + 1, P:].to(dev)
        masked_suffix = torch.full((1, S), mask, dtype=torch.long)

        # original: whole canvas, full bidirectional attention
        full.init_loop(torch.cat([prefix_ids, masked_suffix], dim=1).to(dev), steps)
        wall_o, evals_o = _timed_transitions(full, steps, sample_seed)
        original = full.tokens.view(1, P + S)[:, P:].to(torch.long).clone()
        meta_o = full.metadata(steps)
        term_o = _terminal_kv_valid(meta_o, full.counters, steps)

        # isolated recompute: the prefix forward runs with every suffix
        # forward (gated by the same device flag: B*P rows or none)
        gen.set_prefix(prefix_ids)
        suffix.pre_forward = lambda fwd_rows: gen.prefix.forward(run_rows=_gate(fwd_rows, P, prefix_gate))
        suffix.init_loop(masked_suffix.to(dev), steps)
        try:
            wall_i, evals_i = _timed_transitions(suffix, steps, sample_seed)
        finally:
            suffix.pre_forward = None
        isolated = suffix.tokens.view(1, S).to(torch.long).clone()
        meta_i = suffix.metadata(steps)
        term_i = _terminal_kv_valid(meta_i, suffix.counters, steps)

        # isolated cache: prefix once
        p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        p0.record()
        gen.set_prefix(prefix_ids)
        p1.record()
        suffix.init_loop(masked_suffix.to(dev), steps)
        wall_c, evals_c = _timed_transitions(suffix, steps, sample_seed)
        cached = suffix.tokens.view(1, S).to(torch.long).clone()
        meta_c = suffix.metadata(steps)
        term_c = _terminal_kv_valid(meta_c, suffix.counters, steps)

        cached_result = _path_result(cached, target, meta_c, evals_c, wall_c, term_c)
        cached_result["one_time_prefix_prefill_latency_ms"] = float(p0.elapsed_time(p1))
        sample_results.append({
            "sample": index,
            "seed": sample_seed,
            "prefix_token_ids": prefix_ids[0].tolist(),
            "target_suffix_token_ids": target[0].cpu().tolist(),
            "original_full_attention": _path_result(original, target, meta_o, evals_o, wall_o, term_o),
            "prefix_isolated_recompute": _path_result(isolated, target, meta_i, evals_i, wall_i, term_i),
            "prefix_isolated_cache": cached_result,
            "cached_vs_recompute_token_agreement": float(cached.eq(isolated).float().mean().item()),
            "cached_vs_recompute_exact_sequence": bool(cached.eq(isolated).all().item()),
            "cached_vs_recompute_transition_schedule_equal": bool(
                meta_c["transition_active_tokens"] == meta_i["transition_active_tokens"]
                and meta_c["transition_changed_tokens"] == meta_i["transition_changed_tokens"]),
            "original_vs_isolated_token_agreement": float(original.eq(isolated).float().mean().item()),
        })

    def med(path: str, key: str) -> float:
        return statistics.median(float(r[path][key]) for r in sample_results)

    median_isolated = med("prefix_isolated_recompute", "model_forward_latency_ms")
    median_cached = med("prefix_isolated_cache", "model_forward_latency_ms")
    median_isolated_wall = med("prefix_isolated_recompute", "wall_latency_ms")
    median_cached_wall = med("prefix_isolated_cache", "wall_latency_ms")
    prefix_kv_bytes = 2 * cfg.blocks * P * cfg.hidden * 2  # K and V, bf16
    return {
        "model": "random-init MDLM-169.6M stand-in, W8A8" if quantized is None else "supplied",
        "weights_seed": weights_seed,
        "device": torch.cuda.get_device_name(dev),
        "windows": "seeded uniform token ids" if synthetic_windows else "supplied",
        "prefix_tokens": P,
        "suffix_tokens": S,
        "steps": steps,
        "samples": samples,
        "sampler": "candidate-cache DDPM (device loop), canvas-position-keyed Philox",
        "aggregate": {
            "exact_cached_sequences": sum(bool(r["cached_vs_recompute_exact_sequence"]) for r in sample_results),
            "identical_cached_transition_schedules": sum(
                bool(r["cached_vs_recompute_transition_schedule_equal"]) for r in sample_results),
            "minimum_cached_token_agreement": min(float(r["cached_vs_recompute_token_agreement"])
                                                  for r in sample_results),
            "median_isolated_model_forward_latency_ms": median_isolated,
            "median_cached_model_forward_latency_ms": median_cached,
            "median_model_forward_latency_reduction_fraction": (
                (median_isolated - median_cached) / median_isolated if median_isolated else 0.0),
            "median_isolated_wall_latency_ms": median_isolated_wall,
            "median_cached_wall_latency_ms": median_cached_wall,
            "median_wall_latency_reduction_fraction": (
                (median_isolated_wall - median_cached_wall) / median_isolated_wall if median_isolated_wall else 0.0),
            "median_one_time_prefix_prefill_latency_ms": statistics.median(
                float(r["prefix_isolated_cache"]["one_time_prefix_prefill_latency_ms"]) for r in sample_results),
            "median_isolated_model_evaluations": statistics.median(
                int(r["prefix_isolated_recompute"]["model_evaluations"]) for r in sample_results),
            "median_probability_cache_hits": statistics.median(
                int(r["prefix_isolated_cache"]["probability_cache_hits"]) for r in sample_results),
            "terminal_kv_valid_sequences": sum(bool(r["prefix_isolated_cache"]["terminal_kv_valid"])
                                               for r in sample_results),
            "mean_original_vs_isolated_token_agreement": statistics.mean(
                float(r["original_vs_isolated_token_agreement"]) for r in sample_results),
            "mean_original_target_token_agreement": statistics.mean(
                float(r["original_full_attention"]["target_token_agreement"]) for r in sample_results),
            "mean_isolated_target_token_agreement": statistics.mean(
                float(r["prefix_isolated_recompute"]["target_token_agreement"]) for r in sample_results),
            "prefix_kv_bytes": prefix_kv_bytes,
            "prefix_kv_mib": prefix_kv_bytes / 1024 ** 2,
        },
        "sample_results": sample_results,
    }
