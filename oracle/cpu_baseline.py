"""CPU baseline: the reference's path run on host cores.  TEST / BENCH
INFRASTRUCTURE ONLY (the checker side; never the product).

`measure_reference_sampler` times the reference's own sampler function,
mdlm._run_ddpm_candidate_cache_sampler (src/diffusion_accel/mdlm.py:1104-1218),
imported unmodified from the reference package installed under
baseline/_ref, with `OracleModel` as its `model`: the W8A8 forward of
model_oracle (int8 products through torch._int_mm like
fixed_mlp._integer_matmul) and the W8A8 head, returning fp32 logits
[B, L, V].  The sampler itself does what the reference does on the CPU:
full-vocabulary SUBS log-softmax, exponential-race candidates for every
position (mdlm.py:844-858), reveal, commit, final greedy pass.  The
reference's own checkpoint (Hugging Face remote code) cannot run here, so the
model is the oracle restatement of the same architecture.

`measure` is the fallback when the reference package is absent: one
candidate-cache transition with a model evaluation restated in this file
(`transition`).  torch uses all host threads it is given.
"""

from __future__ import annotations

import os
import sys
import time
from pathlib import Path
from typing import Tuple

REF_INSTALL = Path(__file__).resolve().parents[1] / "baseline" / "_ref"


class OracleModel:
    """model(input_ids=LongTensor[B, L], timesteps=...) -> fp32 logits
    [B, L, V]: the call protocol of mdlm.py:1139-1142 over the oracle's W8A8
    forward and head (the model is not time-conditioned, so timesteps is
    unused, as for the reference checkpoint)."""

    def __init__(self, qm) -> None:
        self.qm = qm
        self.calls = 0

    def __call__(self, input_ids, timesteps=None):
        from oracle import model_oracle

        self.calls += 1
        h = model_oracle.forward(self.qm, input_ids.numpy())
        return model_oracle.logits(self.qm, h)


def reference_sampler():
    """The reference's mdlm module from baseline/_ref, or None."""
    if not (REF_INSTALL / "diffusion_accel").is_dir():
        return None
    if str(REF_INSTALL) not in sys.path:
        sys.path.insert(0, str(REF_INSTALL))
    try:
        from diffusion_accel import mdlm
    except Exception:  # pragma: no cover - depends on the install
        return None
    return mdlm


def measure_reference_sampler(qm, positions: int = 1024, sample_steps: int = 4, steps: int = 64,
                              threads: int = 0, seed: int = 0) -> dict:
    """Time one call of the reference's candidate-cache sampler over
    `sample_steps` transitions (+ its final greedy pass) of one all-masked
    sequence, and extrapolate generated tok/s to a `steps`-transition
    generation from the time per model evaluation (at L = 1024 every
    transition evaluates).  Returns None when the reference is absent."""
    import torch

    from oracle import model_oracle

    mdlm = reference_sampler()
    if mdlm is None:
        return None
    cores = threads or len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    torch.manual_seed(seed)
    model_oracle.USE_INT_MM = True
    model = OracleModel(qm)
    ids = torch.full((1, positions), qm.config.mask_token_id, dtype=torch.int64)
    with torch.no_grad():
        model(input_ids=ids[:, :64])  # warm-up (transposed weights)
        t0 = time.perf_counter()
        _, _, meta = mdlm._run_ddpm_candidate_cache_sampler(model, ids, mask_token_id=qm.config.mask_token_id,
                                                            steps=sample_steps, device="cpu")
        dt = time.perf_counter() - t0
    evaluations = max(1, int(meta["model_evaluations"]))
    per_eval = dt / evaluations
    value = positions / (per_eval * (steps + 1))
    return {"value": value, "unit": "tok/s", "cores": cores, "kind": "reference",
            "seconds_per_evaluated_transition": per_eval, "seconds": dt,
            "sample": f"mdlm._run_ddpm_candidate_cache_sampler (the reference's own function) on 1 x "
                      f"{positions} all-masked, steps={sample_steps} ({evaluations} model evaluations incl. "
                      f"the final pass) with the oracle W8A8 model (torch._int_mm) as `model`, "
                      f"extrapolated to the {steps + 1} evaluations of a {steps}-step generation"}


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
    """Fallback port: time `transitions` evaluated transitions of one
    sequence restated above; extrapolate generated tok/s for a full
    generation of `steps` transitions (every transition evaluates at
    L=1024: a change happens nearly every step) plus the final greedy pass."""
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


def measure_best(qm, **kw) -> dict:
    """The reference's own sampler when installed, else the port."""
    r = measure_reference_sampler(qm, steps=kw.get("steps", 64), threads=kw.get("threads", 0))
    return r if r is not None else measure(qm, **kw)

