"""Event-driven sampler host logic against the reference's own outputs
(tests/golden/make_event_golden.py): reveal schedules from uniforms, the
selected-row order and the metadata.  No GPU."""

import json
import random
import sys

import pytest

from conftest import GOLDEN

sys.path.insert(0, str(GOLDEN))
from make_event_golden import MASK, RUN_CASES, WALL_KEYS, edge_uniforms, winner_logits  # noqa: E402

from diffusionhard_b200.event import (NEVER, EventSchedule, default_reveal_uniforms, reveal_groups,  # noqa: E402
                                      reveal_steps_from_uniforms, steps_from_groups)

GJ = json.loads((GOLDEN / "event_golden.json").read_text())


def test_reveal_steps_match_reference():
    import torch

    for c in GJ["uniform_cases"]:
        u = torch.rand(c["n"], generator=torch.Generator().manual_seed(c["seed"]))
        rs = reveal_steps_from_uniforms(u, steps=c["steps"], sampling_epsilon=c["eps"])
        assert rs.tolist() == c["reveal_steps"], c["seed"]
    for c in GJ["edge_cases"]:
        rs = reveal_steps_from_uniforms(edge_uniforms(torch, c["steps"], c["eps"]), steps=c["steps"],
                                        sampling_epsilon=c["eps"])
        assert rs.tolist() == c["reveal_steps"], c["steps"]


def test_reveal_step_argument_errors():
    import torch

    with pytest.raises(ValueError, match="steps must be positive"):
        reveal_steps_from_uniforms(torch.zeros(3), steps=0, sampling_epsilon=0.0)
    with pytest.raises(ValueError, match="sampling_epsilon"):
        reveal_steps_from_uniforms(torch.zeros(3), steps=4, sampling_epsilon=1.0)
    with pytest.raises(ValueError, match="reveal_seed"):
        default_reveal_uniforms(-1, (4,))


def _host_run(positions, steps, reveal_seed):
    """The event loop on the host with the deterministic winner logits (the
    race is decided by the 1e4 margin), driven by EventSchedule."""
    import torch

    rs = reveal_steps_from_uniforms(default_reveal_uniforms(reveal_seed, (positions,)), steps=steps,
                                    sampling_epsilon=1e-5)
    sched = EventSchedule.build(rs, steps)
    ids = torch.full((1, positions), MASK, dtype=torch.long)
    for k in range(steps + 1):
        sel = sched.rows(k)
        if sel.numel():
            ids[0, sel] = winner_logits(torch, ids, sel).argmax(dim=-1)
    return ids, sched


@pytest.mark.parametrize("case", range(len(RUN_CASES)))
def test_schedule_order_and_metadata_match_reference(case):
    c = GJ["run_cases"][case]
    ids, sched = _host_run(c["positions"], c["steps"], c["reveal_seed"])
    assert ids[0].tolist() == c["ids"]
    meta = sched.metadata(1.0)
    for k in WALL_KEYS:
        assert k in meta
    assert {k: v for k, v in meta.items() if k not in WALL_KEYS} == c["metadata"]


def test_schedule_batched_and_prefix_rows():
    import torch

    rs = torch.tensor([[2, 0, NEVER, 1], [0, 3, 3, NEVER]])
    s = EventSchedule.build(rs, 3)
    assert [s.rows(k).tolist() for k in range(4)] == [[1, 4], [3], [0], [5, 6]]
    assert s.offsets == [0, 2, 3, 4, 6]
    meta = s.metadata(2.0)
    assert meta["transition_active_tokens"] == [6, 4, 3]
    assert meta["transition_changed_tokens"] == [2, 1, 1]
    assert meta["model_evaluations"] == 4 and meta["all_tokens_committed"]
    with pytest.raises(ValueError, match="reveal steps"):
        EventSchedule.build(torch.tensor([[5]]), 3)


def test_reveal_groups_restate_python_random():
    groups = reveal_groups(positions=200, steps=16, seed=4)
    assert sorted(p for g in groups for p in g) == list(range(200))
    gen = random.Random(4)
    for p in range(200):
        d = gen.random()
        k = min(15, int(d * 16 / (1 - 1e-5))) if d < 1 - 1e-5 else 16
        assert p in groups[k]
    rs = steps_from_groups(groups, 200)
    assert all(p in groups[int(rs[p])] for p in range(200))
