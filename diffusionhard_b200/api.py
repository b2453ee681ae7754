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

from . import _lib
from .engine import MDLMEngine
from .model import MDLMConfig, QuantizedMDLM, build_quantized


def load_mdlm(batch: int, seq_len: int = 1024, *, seed: int = 0, config: Optional[MDLMConfig] = None,
              device: str = "cuda", quantized: Optional[QuantizedMDLM] = None, checkpoint: Any = None,
              package: Any = None, alpha: float = 0.5) -> MDLMEngine:
    """MDLM-169.6M on `device`, W8A8-quantised with SmoothQuant (alpha) from
    the seeded calibration batch.  Weights, in order of precedence:
    `quantized`; `checkpoint` (an HF-layout state dict or file,
    checkpoint.load_checkpoint); `package` (a hardware package directory,
    checkpoint.load_hardware_package); else the random-init N(0, 0.02)
    stand-in of `seed`."""
    if quantized is not None:
        qm = quantized
    elif checkpoint is not None or package is not None:
        from .checkpoint import load_checkpoint, load_hardware_package
        from .model import quantize

        cfg = config or MDLMConfig()
        folded = load_checkpoint(checkpoint, cfg) if checkpoint is not None else \
            load_hardware_package(package, config=cfg)
        qm = quantize(folded, alpha)
    else:
        qm = build_quantized(config or MDLMConfig(), seed=seed, alpha=alpha)
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
    with torch.cuda.device(model.device):
        _lib.check_device_error()  # the generation's kernels all completed their waits
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


def run_event_driven_candidate_sampler(model: MDLMEngine, input_ids: Any, *, mask_token_id: int, steps: int,
                                       device: Any = None, reveal_seed: int, sampling_epsilon: float = 1e-5,
                                       reveal_uniforms: Any = None, seed: int = 0,
                                       graph: bool = False) -> tuple[Any, dict]:
    """Drop-in for apple_mdlm._run_event_driven_candidate_sampler
    (apple_mdlm.py:62-156) with the engine as the selected-row model.

    Same schedule as the reference: one uniform per position, by default
    ``torch.rand`` from a CPU generator seeded with ``reveal_seed``, or the
    caller's ``reveal_uniforms``.  Transitions that reveal nothing are
    skipped, and candidates are drawn only for the revealed rows.  Unlike the
    reference, any batch size works: each sequence draws its own uniforms,
    and a transition runs when any sequence reveals.  Every canvas position
    takes its candidate at its reveal transition, as in the reference.
    Returns ``(ids, metadata)`` with the reference keys; ids come back on the
    input's device."""
    import torch

    from .event import EventSchedule, default_reveal_uniforms, reveal_steps_from_uniforms

    if mask_token_id != model.cfg.mask_token_id:
        raise ValueError("mask_token_id does not match the model")
    if input_ids.ndim != 2 or tuple(input_ids.shape) != (model.B, model.L):
        raise ValueError(f"input_ids must be [{model.B}, {model.L}]")
    if reveal_seed < 0:
        raise ValueError("reveal_seed must be non-negative")
    shape = (model.L,) if model.B == 1 else (model.B, model.L)
    if reveal_uniforms is None:
        reveal_uniforms = default_reveal_uniforms(reveal_seed, shape)
    elif reveal_uniforms.numel() != model.B * model.L:
        raise ValueError("reveal_uniforms must contain one value per position")
    rs = reveal_steps_from_uniforms(reveal_uniforms.reshape(model.B, model.L), steps=steps,
                                    sampling_epsilon=sampling_epsilon)
    sched = EventSchedule.build(rs, steps)
    src_device = input_ids.device
    out = model.generate_event_driven(input_ids.to(model.device), sched, seed=seed, graph=graph)
    ids = out.to(torch.int64).to(src_device)
    with torch.cuda.device(model.device):
        _lib.check_device_error()
    return ids, sched.metadata(model.generation_ms())


def run_event_sampler(model: MDLMEngine, *, canvas_tokens: int = 64, prefix_token_ids: Any = (), steps: int = 64,
                      seed: int = 0, graph: bool = False) -> tuple[Any, dict]:
    """The reference's MLX event sampler (mlx_mdlm.py:754-826) on the engine:
    a single sequence of ``prefix_token_ids`` followed by ``canvas_tokens``
    masks (model.L must equal their sum).  The reveal groups come from
    ``random.Random(seed)`` as in the reference, and the candidates from the
    Philox-Gumbel race keyed by ``seed``.  Returns (ids [1, L] int64 on the
    CPU, metadata with the reference keys)."""
    import torch

    from .event import NEVER, EventSchedule, reveal_groups

    prefix = [int(t) for t in prefix_token_ids]
    if model.B != 1 or model.L != len(prefix) + canvas_tokens:
        raise ValueError("the engine must hold one sequence of prefix + canvas tokens")
    groups = reveal_groups(positions=canvas_tokens, steps=steps, seed=seed)
    rs = torch.full((1, model.L), NEVER, dtype=torch.long)
    for k, g in enumerate(groups):
        for p in g:
            rs[0, len(prefix) + p] = k
    sched = EventSchedule.build(rs, steps)
    ids = torch.tensor([prefix + [model.cfg.mask_token_id] * canvas_tokens], dtype=torch.int64)
    out = model.generate_event_driven(ids.to(model.device), sched, seed=seed, graph=graph)
    wall_ms = model.generation_ms()
    meta = sched.metadata(wall_ms)
    return out.to(torch.int64).cpu(), {
        "wall_latency_ms": wall_ms,
        "output_tokens_per_second": meta["output_tokens_per_second"],
        "model_evaluations": meta["model_evaluations"],
        "selected_output_rows": canvas_tokens,
        "prefix_tokens": len(prefix),
    }
