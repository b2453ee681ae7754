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
    reference = reference.detach().float().cpu()
    changed = changed.detach().float().cpu()
    difference = changed - reference
    reference_rms = reference.square().mean().sqrt()
    rmse = difference.square().mean().sqrt()
    denominator = reference.flatten().norm() * changed.flatten().norm()
    cosine = torch.tensor(1.0)
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
