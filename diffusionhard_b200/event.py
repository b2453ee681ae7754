"""Event-driven selected-row sampling: only transitions that reveal a token run.

Drop-ins for the reference's event-driven sampler
(src/diffusion_accel/apple_mdlm.py:20-156, mlx_mdlm.py:727-826).  Every
canvas position draws its reveal transition once, up front, from one uniform:

    step(u) = min(steps - 1, floor(u * steps / (1 - eps)))   if u < 1 - eps
              steps  (the final greedy pass)                 otherwise

For the non-time-conditioned MDLM this is distribution-equivalent to the
per-transition Bernoulli reveals of the ddpm_cache loop: under the linear
schedule a masked position's reveal time is uniform over the transitions.
Transitions that reveal nothing change nothing and are skipped.  Candidates
are drawn only for the rows that reveal.

The schedule is host data known before the first launch.  The whole
generation is therefore a fixed launch sequence over the non-empty
transitions, with no device-side planning.  Each non-empty transition runs:
  1. the forward over the canvas;
  2. the final LayerNorm + int8 quantisation of its selected rows;
  3. the head with the Philox-Gumbel race;
  4. the commit.
The selected rows of all transitions sit in one device array, and each
transition takes its slice.

Here the race is the reference's hardware Q10 Gumbel race, keyed by the
counter (vocabulary group, position, transition, 0) and (seed, sequence).
The reference's torch-RNG exponential race (apple_mdlm.py:43-59) is
distribution-equivalent to it.
"""

from __future__ import annotations

import random
from dataclasses import dataclass
from typing import Any, Callable, Dict, List, Optional

NEVER = -1  # positions outside the canvas (a conditioning prefix) never reveal


def reveal_steps_from_uniforms(uniforms: Any, *, steps: int, sampling_epsilon: float) -> Any:
    """Reveal transition of each uniform draw (apple_mdlm.py:20-40): int64 CPU
    tensor of the input's shape, `steps` for the final greedy pass.  The same
    float32 arithmetic as the reference, so the schedules are identical."""
    import torch

    if steps <= 0:
        raise ValueError("steps must be positive")
    if not 0.0 <= sampling_epsilon < 1.0:
        raise ValueError("sampling_epsilon must be in [0, 1)")
    uniforms = uniforms.detach().cpu()
    out = torch.full(uniforms.shape, steps, dtype=torch.long)
    reveal_mass = 1.0 - sampling_epsilon
    reveal = uniforms < reveal_mass
    out[reveal] = torch.floor(uniforms[reveal] * steps / reveal_mass).long().clamp(max=steps - 1)
    return out


def reveal_groups(*, positions: int, steps: int, seed: int, sampling_epsilon: float = 1e-5) -> List[List[int]]:
    """Positions revealing at each transition, [steps + 1] lists, drawn with
    Python's `random.Random(seed)` as the reference's MLX sampler does
    (mlx_mdlm.py:727-751)."""
    if positions <= 0 or steps <= 0:
        raise ValueError("positions and steps must be positive")
    if seed < 0:
        raise ValueError("seed must be non-negative")
    if not 0.0 <= sampling_epsilon < 1.0:
        raise ValueError("sampling_epsilon must be in [0, 1)")
    gen = random.Random(seed)
    groups: List[List[int]] = [[] for _ in range(steps + 1)]
    mass = 1.0 - sampling_epsilon
    for position in range(positions):
        draw = gen.random()
        groups[min(steps - 1, int(draw * steps / mass)) if draw < mass else steps].append(position)
    return groups


def steps_from_groups(groups: List[List[int]], positions: int) -> Any:
    """Inverse of reveal_groups: int64 [positions] reveal transitions."""
    import torch

    out = torch.full((positions,), NEVER, dtype=torch.long)
    for k, g in enumerate(groups):
        if g:
            out[torch.tensor(g, dtype=torch.long)] = k
    if bool((out == NEVER).any()):
        raise ValueError("every position needs a reveal transition")
    return out


def default_reveal_uniforms(reveal_seed: int, shape: tuple) -> Any:
    """The reference's default draws (apple_mdlm.py:87-89):
    torch.rand(positions) from a CPU generator seeded with reveal_seed; for B
    sequences, B * positions draws in row-major order (sequence 0 gets the
    single-sequence draws)."""
    import torch

    if reveal_seed < 0:
        raise ValueError("reveal_seed must be non-negative")
    g = torch.Generator(device="cpu").manual_seed(reveal_seed)
    return torch.rand(shape, generator=g)


@dataclass
class EventSchedule:
    """Host form of a reveal schedule over B sequences x L positions.

    rows[k] lists the flattened rows b * L + p that reveal at transition k
    (k == steps: final greedy pass), in ascending order, which is the
    position-major order of the ddpm_cache loop's row compaction."""

    steps: int
    sequences: int
    positions: int
    reveal_steps: Any            # int64 [B, L] (NEVER outside the canvas)
    order: Any                   # int64 [n]: rows sorted by (transition, row)
    offsets: List[int]           # [steps + 2] slice bounds of each transition in `order`

    @classmethod
    def build(cls, reveal_steps: Any, steps: int) -> "EventSchedule":
        import torch

        rs = reveal_steps.detach().cpu().to(torch.long)
        if rs.ndim == 1:
            rs = rs[None, :]
        if rs.ndim != 2:
            raise ValueError("reveal steps must be [positions] or [sequences, positions]")
        if bool(((rs < NEVER) | (rs > steps)).any()):
            raise ValueError("reveal steps must lie in [0, steps] (or -1 outside the canvas)")
        B, L = rs.shape
        flat = rs.reshape(-1)
        idx = torch.arange(flat.numel(), dtype=torch.long)
        live = flat >= 0
        key = flat[live] * flat.numel() + idx[live]
        order = idx[live][torch.argsort(key)]
        counts = torch.bincount(flat[live], minlength=steps + 1).tolist()
        offsets = [0]
        for c in counts:
            offsets.append(offsets[-1] + c)
        return cls(steps, B, L, rs, order, offsets)

    def count(self, k: int) -> int:
        return self.offsets[k + 1] - self.offsets[k]

    def rows(self, k: int) -> Any:
        return self.order[self.offsets[k]: self.offsets[k + 1]]

    def metadata(self, wall_ms: float) -> Dict[str, object]:
        """The reference's metadata (apple_mdlm.py:137-150), summed over the
        sequences.  The transition loop stops once nothing is left to reveal
        before the final pass."""
        canvas = self.offsets[-1]
        active = canvas
        active_tokens: List[int] = []
        changed_tokens: List[int] = []
        evaluations = 0
        projected = 0
        for k in range(self.steps):
            if active == 0:
                break
            active_tokens.append(active)
            c = self.count(k)
            changed_tokens.append(c)
            if c:
                evaluations += 1
                projected += c
                active -= c
        final = self.count(self.steps)
        if final:
            evaluations += 1
            projected += final
            active -= final
        full_rows = evaluations * canvas
        wall_s = wall_ms / 1e3
        return {
            "sampling_transitions": len(active_tokens),
            "model_evaluations": evaluations,
            "empty_transitions_elided": sum(c == 0 for c in changed_tokens),
            "transition_active_tokens": active_tokens,
            "transition_changed_tokens": changed_tokens,
            "selected_output_rows": projected,
            "full_output_rows_equivalent": full_rows,
            "output_row_reduction": (1.0 - projected / full_rows) if full_rows else 0.0,
            "wall_latency_ms": wall_ms,
            "output_tokens_per_second": canvas / wall_s if wall_s > 0 else float("inf"),
            "all_tokens_committed": active == 0,
            "correctness_class": "distribution-equivalent",
        }


def greedy_argmax_f32(logits: Any, mask_token_id: int) -> Any:
    """Greedy argmax of fp32 logit rows on the GPU (dh_greedy_argmax_f32),
    the mask token excluded, lowest id on ties: int32 ids [rows]."""
    import torch

    from . import _lib

    if logits.dim() != 2 or logits.dtype != torch.float32 or not logits.is_cuda:
        raise ValueError("logits must be a CUDA float32 [rows, vocab] tensor")
    logits = logits.contiguous()
    rows, vocab = logits.shape
    ids = torch.empty(rows, dtype=torch.int32, device=logits.device)
    chunk = 65535
    ws_bytes = int(_lib.lib().dh_noisy_argmax_workspace_size(min(rows, chunk), vocab))
    ws = torch.empty(max(ws_bytes, 256), dtype=torch.uint8, device=logits.device)
    for i in range(0, rows, chunk):
        j = min(rows, i + chunk)
        _lib.call("dh_greedy_argmax_f32", _lib.ptr(logits[i:j]), vocab, j - i, vocab, mask_token_id,
                  _lib.ptr(ids[i:j]), _lib.ptr(ws), ws.numel(), _lib.stream_handle())
    return ids


def run_event_driven_candidate_sampler_f32(
    logits_function: Callable[[Any, Any], Any],
    input_ids: Any,
    *,
    mask_token_id: int,
    steps: int,
    device: Any = "cuda",
    reveal_seed: int,
    sampling_epsilon: float = 1e-5,
    reveal_uniforms: Optional[Any] = None,
    seed: int = 0,
) -> tuple[Any, Dict[str, object]]:
    """Drop-in for apple_mdlm._run_event_driven_candidate_sampler
    (apple_mdlm.py:62-156) over a selected-row logits function.

    ``logits_function(input_ids, selected)`` returns logits [n, V] for the
    n selected positions of the single sequence, on the device.  Same
    arguments, errors, schedule and metadata as the reference, plus ``seed``
    (the race's Philox key).  The race runs on the GPU
    (dh_noisy_argmax_f32, final pass dh_greedy_argmax_f32).  ``input_ids`` is
    updated in place and returned."""
    import torch

    from .sampler import noisy_argmax_f32

    if input_ids.ndim != 2 or input_ids.shape[0] != 1:
        raise ValueError("event-driven sampler currently requires batch size one")
    if reveal_seed < 0:
        raise ValueError("reveal_seed must be non-negative")
    positions = input_ids.shape[1]
    if reveal_uniforms is None:
        reveal_uniforms = default_reveal_uniforms(reveal_seed, (positions,))
    elif reveal_uniforms.numel() != positions:
        raise ValueError("reveal_uniforms must contain one value per position")
    rs = reveal_steps_from_uniforms(reveal_uniforms.reshape(positions), steps=steps,
                                    sampling_epsilon=sampling_epsilon)
    sched = EventSchedule.build(rs, steps)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    start.record()
    for k in range(steps + 1):
        n = sched.count(k)
        if n == 0:
            continue
        sel_cpu = sched.rows(k)
        selected = sel_cpu.to(device)
        logits = logits_function(input_ids, selected).float().reshape(n, -1)
        if k < steps:
            ids = noisy_argmax_f32(logits, mask_token_id, row_position=sel_cpu, row_key_hi=[0] * n,
                                   row_eval=[k] * n, key_lo=seed)
        else:
            ids = greedy_argmax_f32(logits, mask_token_id)
        input_ids[0].index_copy_(0, selected.to(input_ids.device), ids.to(input_ids.dtype).to(input_ids.device))
    end.record()
    end.synchronize()
    return input_ids, sched.metadata(float(start.elapsed_time(end)))


def benchmark_event_sampler(*, canvas_tokens: int = 64, steps: int = 64, seeds: tuple = (0, 1, 2),
                            weights_seed: int = 0, device: str = "cuda", graph: bool = True) -> Dict[str, object]:
    """The B200 form of the reference's sampler comparison
    (apple_mdlm.benchmark_apple_mdlm, apple_mdlm.py:203-390): per seed, the
    candidate-cache loop (the baseline) and the event-driven sampler on one
    all-masked sequence of ``canvas_tokens``, each run once to warm up
    (graph capture) and once timed on the device.  The selected-row head is
    validated against the full-canvas logits on a half-revealed canvas."""
    import statistics

    import torch

    from .api import load_mdlm, run_ddpm_candidate_cache_sampler, run_event_driven_candidate_sampler
    from .model import MDLMConfig

    if canvas_tokens <= 0 or steps <= 0:
        raise ValueError("canvas_tokens and steps must be positive")
    if not seeds or any(s < 0 for s in seeds):
        raise ValueError("seeds must contain non-negative integers")
    cfg = MDLMConfig()
    if canvas_tokens > cfg.max_positions:
        raise ValueError("canvas_tokens exceeds the checkpoint context length")
    eng = load_mdlm(1, canvas_tokens, seed=weights_seed, device=device)
    mask = cfg.mask_token_id

    def blank() -> Any:
        return torch.full((1, canvas_tokens), mask, dtype=torch.long)

    # selected-row head against the full canvas: same int8 rows, same GEMM
    vids = blank()
    vids[:, ::2] = torch.arange((canvas_tokens + 1) // 2)
    eng.tokens.copy_(vids.view(-1).to(torch.int32))
    eng.forward()
    full = eng.logits()[0]
    sel = torch.nonzero(vids[0].eq(mask)).squeeze(1).to(device)
    selected = eng.selected_logits(vids, sel)
    full_sel = full.index_select(0, sel)
    max_err = float((full_sel - selected).abs().max().item())
    top1 = float(full_sel.argmax(-1).eq(selected.argmax(-1)).float().mean().item())

    samples = []
    for seed in seeds:
        for _ in range(2):
            base_ids, _, base_meta = run_ddpm_candidate_cache_sampler(eng, blank(), mask_token_id=mask,
                                                                      steps=steps, seed=seed, graph=graph)
            base_ms = eng.generation_ms()
        for _ in range(2):
            opt_ids, opt_meta = run_event_driven_candidate_sampler(eng, blank(), mask_token_id=mask, steps=steps,
                                                                   reveal_seed=seed, seed=seed, graph=graph)
        samples.append({
            "seed": seed,
            "candidate_cache": {**base_meta, "wall_latency_ms": base_ms,
                                "output_tokens_per_second": canvas_tokens / (base_ms / 1e3)},
            "optimized": opt_meta,
            "baseline_generated_token_ids": base_ids[0].tolist(),
            "optimized_generated_token_ids": opt_ids[0].tolist(),
        })
    base_med = statistics.median(s["candidate_cache"]["wall_latency_ms"] for s in samples)
    opt_med = statistics.median(s["optimized"]["wall_latency_ms"] for s in samples)
    return {
        "device": torch.cuda.get_device_name(eng.device),
        "torch_version": torch.__version__,
        "canvas_tokens": canvas_tokens,
        "steps": steps,
        "seeds": list(seeds),
        "optimization": "event-driven-reveal; selected-row-output-head; philox-gumbel-race; cuda-graph",
        "selected_head_validation": {"maximum_absolute_logit_error": max_err, "top1_agreement": top1},
        "samples": samples,
        "baseline_median_latency_ms": base_med,
        "optimized_median_latency_ms": opt_med,
        "speedup": base_med / opt_med if opt_med > 0 else None,
        "all_tokens_committed": all(s["optimized"]["all_tokens_committed"] for s in samples),
    }
