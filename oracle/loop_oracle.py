"""CPU oracle of the whole candidate-cache generation over the W8A8 model.
TEST INFRASTRUCTURE ONLY.

Restates mdlm._run_ddpm_candidate_cache_sampler (src/diffusion_accel/
mdlm.py:1104-1218) with the reference's hardware forms of its random draws,
sequence by sequence:
  * log-linear schedule t = linspace(1, eps, S + 1), move = (1 - 1e-3) t, and
    reveal probability p_k = (move_k - move_{k+1}) / move_k in float32
    (mdlm.py:1116-1117, 1151-1153), as a Q32 threshold
    min(2^32, floor(p_k 2^32));
  * a sequence evaluates the model when it has masked positions and its canvas
    changed at the previous transition (the cache is filled at the start,
    mdlm.py:1134-1147, and invalidated on any change, :1173-1174);
  * position p reveals at transition k when
    philox((p/4, 0, k, 1), (seed, b))[p%4] < threshold_k (the reveal
    comparison of candidate_sampler.cpp:5-79);
  * the candidate of a revealed position is the noisy argmax of the int8 head
    on the model's final hidden row: round_half_even(logit * 1024) +
    gumbel_q10(philox((v/4, p, e, 0), (seed, b))[v%4]), mask skipped, lowest
    id on ties, e = the transition of the sequence's last evaluation
    (output_head.cpp:23-157 with rng.py:262-263; pyoracle.head_i8 mode 1);
  * the final pass takes the greedy argmax of every position still masked
    (mdlm.py:1177-1200; pyoracle.head_i8 mode 2).
The model is model_oracle.forward (the reference W8A8 arithmetic).
"""

from __future__ import annotations

import math
from typing import Callable, Dict, List, Optional

import numpy as np

from oracle import model_oracle, pyoracle

NOISE_EPSILON = 1e-3


def thresholds_q32(steps: int, sampling_epsilon: float = 1e-5) -> List[int]:
    """Reveal thresholds of mdlm.py:1116-1117, 1151-1153 (float32 arithmetic)."""
    import torch

    t = torch.linspace(1.0, sampling_epsilon, steps + 1)
    move = (1 - NOISE_EPSILON) * t
    out = []
    for k in range(steps):
        p = float(((move[k:k + 1] - move[k + 1:k + 2]) / move[k:k + 1]).item())
        out.append(max(0, min(1 << 32, math.floor(p * 4294967296.0))))
    return out


def generate(qm, ids: np.ndarray, *, steps: int, seed: int, seq_offset: int = 0,
             sampling_epsilon: float = 1e-5, ln_fp64: bool = False,
             on_transition: Optional[Callable[[int, np.ndarray], None]] = None) -> Dict[str, object]:
    """Candidate-cache generation of ids [B, L] (int, mask = model mask id).
    Returns {"tokens": [B, L] int32, "evaluations": per-sequence counts,
    "changed": per-transition changed counts}.  on_transition(k, tokens) is
    called after each transition's commit.  ln_fp64: the forward's
    LayerNorms in float64 (model_oracle.forward), a second CPU evaluation of
    the same arithmetic."""
    mask = qm.config.mask_token_id
    tokens = np.array(ids, dtype=np.int32, copy=True)
    B, L = tokens.shape
    thr = thresholds_q32(steps, sampling_epsilon)
    need = np.ones(B, bool)
    eval_id = np.zeros(B, np.int64)
    hidden: Dict[int, tuple] = {}
    evaluations = np.zeros(B, np.int64)
    changed_per_step = []
    head = qm.head
    for k in range(steps + 1):
        final = k == steps
        active = tokens == mask
        changed = 0
        for b in range(B):
            if not active[b].any():
                continue
            if final or need[b]:
                rec: Dict[str, object] = {}
                model_oracle.forward(qm, tokens[b:b + 1], record=rec, ln_fp64=ln_fp64)
                hidden[b] = (rec["head_q"].numpy(), rec["head_scale"].numpy())
                evaluations[b] += 1
                if not final:
                    eval_id[b] = k
                    need[b] = False
            if final:
                rows = np.nonzero(active[b])[0]
            else:
                words = pyoracle.reveal_words(L, k, seed, seq_offset + b)
                rows = np.nonzero(active[b] & (words.astype(np.uint64) < thr[k]))[0]
            if rows.size == 0:
                continue
            hq, hs = hidden[b]
            cand, _ = pyoracle.head_i8(2 if final else 1, hq[rows], head.weight_q, mask, a_scale=hs[rows],
                                       w_scale=head.w_scale, bias=head.bias, row_position=rows,
                                       row_key_hi=np.full(rows.size, seq_offset + b),
                                       row_eval=np.full(rows.size, eval_id[b]), key_lo=seed)
            tokens[b, rows] = cand
            need[b] = True
            changed += rows.size
        if not final:
            changed_per_step.append(changed)
        if on_transition is not None:
            on_transition(k, tokens)
    return {"tokens": tokens, "evaluations": evaluations, "changed": changed_per_step}
