"""CPU baseline: the reference's path run on host cores.  TEST / BENCH
INFRASTRUCTURE ONLY (the checker side; never the product).

One candidate-cache transition with a model evaluation, as
mdlm._run_ddpm_candidate_cache_sampler does it on CPU (mdlm.py:1134-1174):
W8A8 forward (model_oracle, int8 products through torch._int_mm like
fixed_mlp._integer_matmul), full-vocabulary SUBS log-softmax, exponential-race
candidates for every position (mdlm.py:844-858), reveal with probability
(move_t - move_s) / move_t, commit.  torch uses all host threads it is given.
"""

from __future__ import annotations

import os
import time
from typing import Tuple

import numpy as np


def transition(qm, ids, k: int, steps: int, gen) -> Tuple[object, int]:
    import torch

    from oracle import model_oracle

    model_oracle.USE_INT_MM = True
    mask = qm.config.mask_token_id
    with torch.no_grad():
        h = model_oracle.forward(qm, ids.numpy())
        logits = model_oracle.logits(qm, h)
        logits[:, :, mask] = -torch.inf
        probs = torch.log_softmax(logits, dim=-1).exp()
        exponential = 1e-10 - torch.log(torch.rand(probs.shape, generator=gen) + 1e-10)
        cand = (probs / exponential).argmax(dim=-1)
        t = torch.linspace(1.0, 1e-5, steps + 1)
        move_t, move_s = (1 - 1e-3) * t[k], (1 - 1e-3) * t[k + 1]
        reveal = torch.rand(ids.shape, generator=gen) < (move_t - move_s) / move_t
        active = ids.eq(mask)
        nxt = torch.where(active, torch.where(reveal, cand, torch.full_like(cand, mask)), ids)
        changed = int(ids.ne(nxt).sum())
    return nxt, changed


def measure(qm, positions: int = 1024, transitions: int = 3, steps: int = 64, threads: int = 0) -> dict:
    """Time `transitions` evaluated transitions of one sequence; extrapolate
    generated tok/s for a full generation of `steps` transitions (every
    transition evaluates at L=1024: a change happens nearly every step) plus
    the final greedy pass."""
    import torch

    cores = threads or len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    gen = torch.Generator().manual_seed(0)
    ids = torch.full((1, positions), qm.config.mask_token_id, dtype=torch.int64)
    transition(qm, ids, 0, steps, gen)  # warm-up (allocations, transposed weights)
    t0 = time.perf_counter()
    for k in range(transitions):
        ids, _ = transition(qm, ids, k, steps, gen)
    dt = (time.perf_counter() - t0) / transitions
    evaluations = steps + 1
    return {"value": positions / (dt * evaluations), "unit": "tok/s", "cores": cores, "kind": "port",
            "seconds_per_evaluated_transition": dt,
            "sample": f"1 sequence x {positions} positions, {transitions} evaluated transitions timed "
                      f"(W8A8 forward via torch._int_mm + full-vocab SUBS softmax race), extrapolated to "
                      f"{evaluations} evaluations of a {steps}-step generation"}
