"""Public drop-in API behind the reference's sampler protocol.

``run_ddpm_candidate_cache_sampler`` and ``run_ddpm_cache_sampler`` take the
same arguments as the reference's ``_run_ddpm_candidate_cache_sampler`` /
``_run_ddpm_cache_sampler`` (src/diffusion_accel/mdlm.py:995-1218) -- a model,
``input_ids`` [B, L] (any device, int64), ``mask_token_id``, ``steps``,
``device``, ``sampling_epsilon`` -- plus ``seed`` for the counter-based RNG,
and return ``(ids, measurements, metadata)`` with the reference metadata keys.
The model is an :class:`~diffusionhard_b200.engine.MDLMEngine`; the whole loop
runs on the GPU and the ids come back on the input's device.

``run_conditioned_candidate_cache`` is the prefix-conditioned form
(conditioned._run_conditioned_ddpm_candidate_cache, conditioned.py:132-242,
with prefix K/V reuse under prefix isolation, prefix_drift.py:155-238).
"""

from __future__ import annotations

from typing import Any, Optional

from .engine import MDLMEngine
from .model import MDLMConfig, QuantizedMDLM, build_quantized


def load_mdlm(batch: int, seq_len: int = 1024, *, seed: int = 0, config: Optional[MDLMConfig] = None,
              device: str = "cuda", quantized: Optional[QuantizedMDLM] = None) -> MDLMEngine:
    """Random-init MDLM-169.6M (N(0, 0.02)), folded, W8A8-quantised, on `device`."""
    qm = quantized if quantized is not None else build_quantized(config or MDLMConfig(), seed=seed)
    return MDLMEngine(qm, batch, seq_len, device)


def run_ddpm_candidate_cache_sampler(model: MDLMEngine, input_ids: Any, *, mask_token_id: int, steps: int,
                                     device: Any = None, sampling_epsilon: float = 1e-5, seed: int = 0,
                                     graph: bool = True) -> tuple[Any, list, dict]:
    """Drop-in for mdlm._run_ddpm_candidate_cache_sampler (mdlm.py:1104-1218)."""
    import torch

    if mask_token_id != model.cfg.mask_token_id:
        raise ValueError("mask_token_id does not match the model")
    if tuple(input_ids.shape) != (model.B, model.L):
        raise ValueError(f"input_ids must be [{model.B}, {model.L}]")
    src_device = input_ids.device
    ids_dev = input_ids.to(model.device, non_blocking=True)
    out, _ = model.generate(ids_dev, steps=steps, seed=seed, sampling_epsilon=sampling_epsilon, graph=graph)
    ids = out.to(torch.int64).to(src_device)
    return ids, model.measurements(steps, sampling_epsilon), model.metadata(steps)


def run_ddpm_cache_sampler(model: MDLMEngine, input_ids: Any, *, mask_token_id: int, steps: int,
                           device: Any = None, sampling_epsilon: float = 1e-5, seed: int = 0,
                           graph: bool = True) -> tuple[Any, list, dict]:
    """ddpm_cache sampler (mdlm.py:995-1101).  For the non-time-conditioned
    model the probability-cache update and the candidate-cache reveal draw
    from the same transition distribution (candidate_cache.py:90-254), so the
    same device loop serves both; the metadata carries the ddpm_cache keys."""
    ids, meas, meta = run_ddpm_candidate_cache_sampler(model, input_ids, mask_token_id=mask_token_id,
                                                       steps=steps, device=device,
                                                       sampling_epsilon=sampling_epsilon, seed=seed,
                                                       graph=graph)
    keys = ("sampling_transitions", "model_evaluations", "probability_cache_hits",
            "transition_active_tokens", "transition_changed_tokens", "cache_hit_sampling_overhead_modeled")
    return ids, meas, {k: meta[k] for k in keys}
