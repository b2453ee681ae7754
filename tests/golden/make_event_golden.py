#!/usr/bin/env python3
"""Golden fixtures for the event-driven selected-row sampler, produced by the
reference's own Python (src/diffusion_accel/apple_mdlm.py, imported in place):

  * _reveal_steps_from_uniforms on seeded uniforms for several (steps,
    epsilon) pairs, plus uniforms at the bucket edges;
  * _run_event_driven_candidate_sampler on the CPU with the deterministic
    selected-row logits function below (one winning token per row with a
    1e4 margin, a function of the position and of the canvas state, so the
    order of the reveals matters): the final ids and the metadata minus
    wall-clock fields, for several (positions, steps, reveal_seed).
Inputs are regenerated from the seeds by tests/test_event_*.py; only outputs
are stored.  Writes tests/golden/event_golden.json.

    python tests/golden/make_event_golden.py --reference <reference root>
"""

from __future__ import annotations

import argparse
import os
import json
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
MASK = 50257
VOCAB = 50258
UNIFORM_CASES = [(64, 1e-5, 0, 256), (64, 1e-3, 1, 1000), (7, 0.0, 2, 100), (1, 0.5, 3, 50), (1000, 1e-5, 4, 4096)]
RUN_CASES = [(64, 64, 0), (64, 64, 7), (96, 16, 3), (32, 128, 11), (128, 8, 5)]
WALL_KEYS = ("wall_latency_ms", "output_tokens_per_second")


def edge_uniforms(torch, steps: int, eps: float):
    """Uniforms on and next to every bucket edge k * (1 - eps) / steps."""
    mass = 1.0 - eps
    vals = []
    for k in range(steps + 1):
        e = torch.tensor(k * mass / steps, dtype=torch.float32)
        vals += [e, torch.nextafter(e, torch.tensor(0.0)), torch.nextafter(e, torch.tensor(2.0))]
    return torch.stack(vals).clamp(0.0, 0.99999994)


def winner_logits(torch, input_ids, selected):
    """Deterministic selected-row logits [n, VOCAB]: 0 at the winning token,
    -1e4 elsewhere.  winner = (7 p + 13 revealed + sum(revealed ids)) mod MASK,
    over the canvas state, so every reveal changes later winners."""
    ids = input_ids[0]
    revealed = ids.ne(MASK)
    n_rev = int(revealed.sum().item())
    tok_sum = int(ids[revealed].sum().item()) if n_rev else 0
    win = (7 * selected.to(torch.int64) + 13 * n_rev + tok_sum) % MASK
    logits = torch.full((selected.numel(), VOCAB), -1e4, dtype=torch.float32, device=input_ids.device)
    logits[torch.arange(selected.numel(), device=input_ids.device), win.to(input_ids.device)] = 0.0
    return logits


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--reference", default=os.environ.get("DH_REFERENCE_ROOT"),
                    required="DH_REFERENCE_ROOT" not in os.environ,
                    help="reference tree (default: $DH_REFERENCE_ROOT)")
    args = ap.parse_args()
    sys.path.insert(0, str(Path(args.reference) / "src"))
    import torch

    from diffusion_accel import apple_mdlm  # reference, in place

    out = {"uniform_cases": [], "edge_cases": [], "run_cases": []}
    for n, eps, seed, steps in UNIFORM_CASES:
        u = torch.rand(n, generator=torch.Generator().manual_seed(seed))
        rs = apple_mdlm._reveal_steps_from_uniforms(u, steps=steps, sampling_epsilon=eps)
        out["uniform_cases"].append({"n": n, "eps": eps, "seed": seed, "steps": steps, "reveal_steps": rs.tolist()})
    for steps, eps in ((64, 1e-5), (10, 0.0), (3, 0.25)):
        u = edge_uniforms(torch, steps, eps)
        rs = apple_mdlm._reveal_steps_from_uniforms(u, steps=steps, sampling_epsilon=eps)
        out["edge_cases"].append({"steps": steps, "eps": eps, "reveal_steps": rs.tolist()})
    for positions, steps, reveal_seed in RUN_CASES:
        ids = torch.full((1, positions), MASK, dtype=torch.long)
        ids, meta = apple_mdlm._run_event_driven_candidate_sampler(
            lambda x, sel: winner_logits(torch, x, sel), ids, mask_token_id=MASK, steps=steps, device="cpu",
            reveal_seed=reveal_seed)
        out["run_cases"].append({"positions": positions, "steps": steps, "reveal_seed": reveal_seed,
                                 "ids": ids[0].tolist(),
                                 "metadata": {k: v for k, v in meta.items() if k not in WALL_KEYS}})
    (HERE / "event_golden.json").write_text(json.dumps(out, sort_keys=True) + "\n")
    print({k: len(v) for k, v in out.items()})


if __name__ == "__main__":
    main()
