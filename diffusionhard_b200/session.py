"""Block-causal sessions with retained K/V (multi-turn generation).

A session is one canvas of consecutive blocks: a prompt, generated answers
and follow-up turns.  Attention is block-causal (mdlm.block_isolation,
mdlm.py:61-77).  A completed block attends to itself and to earlier blocks,
and the active block attends to everything before it and to itself.  So a
completed block's K/V never change once the block is final, and the session
keeps them in per-layer K/V buffers (prefix_drift._materialize_cached_block,
prefix_drift.py:241-264).

Each block runs on its own engine view of the shared buffers:
  * rotary positions start at the block's offset;
  * its K/V rows are written at that offset;
  * its keys are everything up to the block's end.
The session has three operations:
  * ``append`` runs one forward of given tokens, e.g. a prompt, a
    follow-up, or a finished answer (prefill / finalisation);
  * ``generate`` runs the candidate-cache loop on a masked active block
    over the retained K/V;
  * ``generate(recompute=True)`` re-runs every completed block's forward
    before each model evaluation.  That is the block-isolated full
    recompute of the reference (multiturn.py:146-642), done block by block.
The two generate paths run the same arithmetic and must agree token for
token.

Block lengths are multiples of 32, the kernels' row granule.
"""

from __future__ import annotations

import statistics
from typing import Any, Dict, List, Optional, Tuple

from .engine import MDLMEngine
from .model import QuantizedMDLM


class BlockCausalSession:
    """`batch` sequences sharing one block layout, up to `capacity` tokens."""

    def __init__(self, qm: QuantizedMDLM, batch: int, capacity: int, device: Any = "cuda") -> None:
        import torch

        if capacity % 32 or capacity <= 0:
            raise ValueError("capacity must be a positive multiple of 32")
        if capacity > qm.config.max_positions:
            raise ValueError("session exceeds the model length")
        self.qm, self.B, self.capacity = qm, batch, capacity
        self.kv = MDLMEngine.kv_cache(qm, batch, capacity, device)
        self.device = torch.device(device)
        self.blocks: List[Tuple[int, int, Any]] = []  # (start, end, device int32 ids [B * n])
        self._engines: Dict[Tuple[int, int], MDLMEngine] = {}
        self._gate = torch.zeros(1, dtype=torch.int32, device=self.device)

    @property
    def length(self) -> int:
        return self.blocks[-1][1] if self.blocks else 0

    def block_ends(self) -> List[int]:
        return [end for _, end, _ in self.blocks]

    def engine(self, start: int, n: int) -> MDLMEngine:
        """Engine for rows [start, start + n): rotary positions and K/V rows
        at `start`, keys [0, start + n)."""
        if start % 32 or n % 32 or n <= 0:
            raise ValueError("block offsets and lengths must be multiples of 32")
        if start + n > self.capacity:
            raise ValueError("block exceeds the session capacity")
        key = (start, n)
        e = self._engines.get(key)
        if e is None:
            e = MDLMEngine(self.qm, self.B, n, self.device, pos_offset=start, kv_len=start + n, kv_offset=start,
                           kv_buffers=self.kv)
            self._engines[key] = e
        return e

    def append(self, ids: Any) -> MDLMEngine:
        """Run one forward of `ids` [B, n] as the next completed block and
        keep its K/V (a prompt or follow-up prefill, or the finalisation of a
        generated answer).  Returns the engine that ran it."""
        import torch

        ids = ids.reshape(self.B, -1)
        n = ids.shape[1]
        e = self.engine(self.length, n)
        dev_ids = ids.to(device=self.device, dtype=torch.int32).reshape(-1).contiguous()
        e.tokens.copy_(dev_ids)
        e.forward()
        self.blocks.append((self.length, self.length + n, dev_ids.clone()))
        return e

    def truncate(self, length: int) -> None:
        """Drop completed blocks past `length` (a block boundary)."""
        if length not in [0] + self.block_ends():
            raise ValueError("truncate to a block boundary")
        self.blocks = [b for b in self.blocks if b[1] <= length]

    def _recompute_history(self, fwd_rows: Any) -> None:
        """Re-run every completed block's forward, gated by the active
        block's device flag (no forward on a cache hit)."""
        import torch

        for start, end, ids in self.blocks:
            e = self.engine(start, end - start)
            e.tokens.copy_(ids)
            torch.mul(torch.clamp(fwd_rows.view(torch.int32), max=1), e.M, out=self._gate)
            e.forward(run_rows=self._gate)

    def generate(self, n: int, *, steps: int, seed: int = 0, recompute: bool = False,
                 initial: Any = None) -> Tuple[Any, Dict[str, object], float, List[float]]:
        """Generate the next block of `n` tokens (initially masked, or
        `initial` [B, n]) with the candidate-cache loop over the retained
        K/V.  The block is not appended: call `append` with the result to
        finalise it.  Returns (ids [B, n] int64 on the device, metadata,
        wall ms, per-evaluation ms)."""
        import torch

        from .conditioned import _timed_transitions

        e = self.engine(self.length, n)
        mask = self.qm.config.mask_token_id
        ids = torch.full((self.B, n), mask, dtype=torch.long) if initial is None else initial
        e.init_loop(ids.to(self.device), steps)
        if recompute:
            e.pre_forward = self._recompute_history
        try:
            wall, evals = _timed_transitions(e, steps, seed)
        finally:
            e.pre_forward = None
        return e.tokens.view(self.B, n).to(torch.long).clone(), e.metadata(steps), wall, evals

    def kv_bytes(self, tokens: Optional[int] = None) -> int:
        """K (bf16) and V (f16) bytes held for `tokens` positions."""
        t = self.length if tokens is None else tokens
        cfg = self.qm.config
        return 2 * cfg.blocks * self.B * t * cfg.hidden * 2


def _timed(fn) -> Tuple[Any, float]:
    import torch

    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    out = fn()
    b.record()
    b.synchronize()
    return out, float(a.elapsed_time(b))


def _path(generated: Any, target: Any, meta: Dict[str, object], wall: float, evals: List[float]) -> Dict[str, object]:
    return {
        **meta,
        "wall_latency_ms": wall,
        "model_forward_latency_ms": float(sum(evals)),
        "median_model_evaluation_latency_ms": statistics.median(evals) if evals else 0.0,
        "target_token_agreement": float(generated.eq(target).float().mean().item()),
        "generated_token_ids": generated[0].cpu().tolist(),
        "generated_text": None,
    }


def evaluate_two_turn_mdlm_session(*, quantized: Optional[QuantizedMDLM] = None, prefix_tokens: int = 64,
                                   first_answer_tokens: int = 32, followup_tokens: int = 32,
                                   second_answer_tokens: int = 32, samples: int = 3, steps: int = 64,
                                   seed: int = 0, weights_seed: int = 0, windows: Any = None,
                                   device: Any = "cuda") -> Dict[str, object]:
    """Two answer blocks in a block-causal session, each generated by full
    block-isolated recompute and over retained K/V; the report of
    multiturn.evaluate_two_turn_mdlm_session (multiturn.py:146-642).

    Per sample (seeded windows of prefix + answer + follow-up + answer ids):
    turn 1 generates the first answer after the prompt both ways.  The cached
    answer is then finalised (one forward appends its K/V), the follow-up is
    prefilled, and turn 2 is generated both ways.  The noise is keyed by
    canvas position and sequence, so the recompute and cached paths must
    agree exactly."""
    import torch

    from .model import MDLMConfig, build_quantized

    lengths = (prefix_tokens, first_answer_tokens, followup_tokens, second_answer_tokens, samples, steps)
    if min(lengths) <= 0:
        raise ValueError("token counts, samples, and steps must be positive")
    if any(t % 32 for t in lengths[:4]):
        raise ValueError("block lengths must be multiples of 32")
    qm = quantized if quantized is not None else build_quantized(MDLMConfig(), seed=weights_seed)
    cfg = qm.config
    P, A1, F, A2 = prefix_tokens, first_answer_tokens, followup_tokens, second_answer_tokens
    total = P + A1 + F + A2
    if total > cfg.max_positions:
        raise ValueError("two-turn session exceeds checkpoint context length")
    mask = cfg.mask_token_id
    synthetic = windows is None
    if windows is None:
        windows = torch.randint(0, mask, (samples, total), generator=torch.Generator().manual_seed(seed + 3))
    windows = torch.as_tensor(windows, dtype=torch.long)
    if tuple(windows.shape) != (samples, total):
        raise ValueError("windows must be [samples, total session tokens]")
    sess = BlockCausalSession(qm, 1, total, device)
    dev = sess.device

    results = []
    for index in range(samples):
        w = windows[index: index + 1]
        prefix, first_target = w[:, :P], w[:, P:P + A1].to(dev)
        followup, second_target = w[:, P + A1:P + A1 + F], w[:, P + A1 + F:].to(dev)
        first_seed, second_seed = seed + 2 * index, seed + 2 * index + 1

        sess.truncate(0)
        _, prefill_ms = _timed(lambda: sess.append(prefix))
        first_rec, meta_fr, wall_fr, ev_fr = sess.generate(A1, steps=steps, seed=first_seed, recompute=True)
        first_cached, meta_fc, wall_fc, ev_fc = sess.generate(A1, steps=steps, seed=first_seed)
        _, fin1_ms = _timed(lambda: sess.append(first_cached))
        _, follow_ms = _timed(lambda: sess.append(followup))
        second_rec, meta_sr, wall_sr, ev_sr = sess.generate(A2, steps=steps, seed=second_seed, recompute=True)
        second_cached, meta_sc, wall_sc, ev_sc = sess.generate(A2, steps=steps, seed=second_seed)
        _, fin2_ms = _timed(lambda: sess.append(second_cached))

        def same_schedule(a: Dict[str, Any], b: Dict[str, Any]) -> bool:
            return (a["transition_active_tokens"] == b["transition_active_tokens"]
                    and a["transition_changed_tokens"] == b["transition_changed_tokens"])

        h1, h2 = P + A1, P + A1 + F
        results.append({
            "sample": index,
            "first_seed": first_seed,
            "second_seed": second_seed,
            "initial_prefix_token_ids": prefix[0].tolist(),
            "first_target_token_ids": first_target[0].cpu().tolist(),
            "followup_token_ids": followup[0].tolist(),
            "second_target_token_ids": second_target[0].cpu().tolist(),
            "turn_1": {
                "recompute": _path(first_rec, first_target, meta_fr, wall_fr, ev_fr),
                "cached": _path(first_cached, first_target, meta_fc, wall_fc, ev_fc),
                "exact_sequence": bool(first_rec.eq(first_cached).all().item()),
                "token_agreement": float(first_rec.eq(first_cached).float().mean().item()),
                "transition_schedule_equal": same_schedule(meta_fr, meta_fc),
                "initial_prefix_prefill_latency_ms": prefill_ms,
                "answer_finalization_latency_ms": fin1_ms,
                "session_kv_mib_after_answer": sess.kv_bytes(h1) / 1024 ** 2,
            },
            "followup_prefill": {
                "tokens": F,
                "latency_ms": follow_ms,
                "session_kv_mib_before_second_answer": sess.kv_bytes(h2) / 1024 ** 2,
            },
            "turn_2": {
                "recompute": _path(second_rec, second_target, meta_sr, wall_sr, ev_sr),
                "cached": _path(second_cached, second_target, meta_sc, wall_sc, ev_sc),
                "exact_sequence": bool(second_rec.eq(second_cached).all().item()),
                "token_agreement": float(second_rec.eq(second_cached).float().mean().item()),
                "transition_schedule_equal": same_schedule(meta_sr, meta_sc),
                "answer_finalization_latency_ms": fin2_ms,
                "final_session_kv_mib": sess.kv_bytes(total) / 1024 ** 2,
                "final_cache_tokens": sess.length,
            },
        })

    def med(values) -> float:
        return statistics.median(list(values))

    rec2 = med(r["turn_2"]["recompute"]["model_forward_latency_ms"] for r in results)
    cached2 = med(r["turn_2"]["cached"]["model_forward_latency_ms"] for r in results)
    follow_req = [r["followup_prefill"]["latency_ms"] + r["turn_2"]["cached"]["model_forward_latency_ms"]
                  for r in results]
    cross = [r["turn_1"]["answer_finalization_latency_ms"] + f for r, f in zip(results, follow_req)]
    ready = [c + r["turn_2"]["answer_finalization_latency_ms"] for r, c in zip(results, cross)]

    def frac(x: float) -> float:
        return (rec2 - x) / rec2 if rec2 else 0.0

    return {
        "model": "random-init MDLM-169.6M stand-in, W8A8" if quantized is None else "supplied",
        "weights_seed": weights_seed,
        "device": torch.cuda.get_device_name(dev),
        "windows": "seeded uniform token ids" if synthetic else "supplied",
        "session_shape": {"initial_prefix_tokens": P, "first_answer_tokens": A1, "followup_tokens": F,
                          "second_answer_tokens": A2, "final_session_tokens": total},
        "steps_per_answer": steps,
        "samples": samples,
        "aggregate": {
            "exact_turn_1_sequences": sum(r["turn_1"]["exact_sequence"] for r in results),
            "exact_turn_2_sequences": sum(r["turn_2"]["exact_sequence"] for r in results),
            "identical_turn_1_transition_schedules": sum(r["turn_1"]["transition_schedule_equal"] for r in results),
            "identical_turn_2_transition_schedules": sum(r["turn_2"]["transition_schedule_equal"] for r in results),
            "minimum_turn_2_token_agreement": min(r["turn_2"]["token_agreement"] for r in results),
            "median_turn_2_recompute_model_forward_latency_ms": rec2,
            "median_turn_2_cached_model_forward_latency_ms": cached2,
            "median_turn_2_model_forward_latency_reduction_fraction": frac(cached2),
            "median_cached_followup_request_latency_ms": med(follow_req),
            "median_cached_followup_request_reduction_fraction": frac(med(follow_req)),
            "median_cross_request_cost_including_first_finalization_ms": med(cross),
            "median_cross_request_reduction_including_first_finalization_fraction": frac(med(cross)),
            "median_cached_cost_ready_for_third_turn_ms": med(ready),
            "median_ready_for_third_turn_reduction_fraction": frac(med(ready)),
            "median_first_answer_finalization_latency_ms": med(
                r["turn_1"]["answer_finalization_latency_ms"] for r in results),
            "median_followup_prefill_latency_ms": med(r["followup_prefill"]["latency_ms"] for r in results),
            "median_second_answer_finalization_latency_ms": med(
                r["turn_2"]["answer_finalization_latency_ms"] for r in results),
            "final_session_kv_mib": sess.kv_bytes(total) / 1024 ** 2,
        },
        "sample_results": results,
    }
