"""Event-driven selected-row sampler on the GPU.

* Over a logits function: with the deterministic winner logits of
  tests/golden/make_event_golden.py the ids and metadata equal the
  reference's own run; with random logits every revealed token is the
  oracle's Philox-Gumbel race on the logits it was drawn from.
* On the engine: only non-empty transitions run, and every revealed row's
  candidate equals the oracle head on the GPU's own int8 hidden row for the
  canvas of its transition (teacher forcing, bit-exact); graph replay equals
  eager; the MLX-style prefix sampler leaves the prefix alone.
"""

import json
import sys

import numpy as np
import pytest

from conftest import GOLDEN

sys.path.insert(0, str(GOLDEN))
from make_event_golden import MASK, RUN_CASES, WALL_KEYS, winner_logits  # noqa: E402

from diffusionhard_b200 import _lib  # noqa: E402
from diffusionhard_b200.engine import MDLMEngine  # noqa: E402
from diffusionhard_b200.model import MDLMConfig, build_quantized  # noqa: E402
from oracle import pyoracle  # noqa: E402

pytestmark = pytest.mark.gpu

GJ = json.loads((GOLDEN / "event_golden.json").read_text())
SMALL = MDLMConfig(vocab_size=1000, mask_token_id=999, blocks=2)


@pytest.fixture(scope="module")
def small_model():
    return build_quantized(SMALL, seed=0)


def _device_error():
    err = np.zeros(1, np.uint32)
    _lib.call("dh_device_error", err.ctypes.data, 1)
    return int(err[0])


@pytest.mark.parametrize("case", range(len(RUN_CASES)))
def test_logits_function_sampler_matches_reference(cuda, case):
    torch = cuda
    from diffusionhard_b200.event import run_event_driven_candidate_sampler_f32

    c = GJ["run_cases"][case]
    ids = torch.full((1, c["positions"]), MASK, dtype=torch.long, device="cuda")
    out, meta = run_event_driven_candidate_sampler_f32(lambda x, sel: winner_logits(torch, x, sel), ids,
                                                       mask_token_id=MASK, steps=c["steps"], device="cuda",
                                                       reveal_seed=c["reveal_seed"], seed=3)
    assert out is ids
    assert out[0].tolist() == c["ids"]
    assert {k: v for k, v in meta.items() if k not in WALL_KEYS} == c["metadata"]
    assert meta["wall_latency_ms"] > 0


def test_logits_function_sampler_race_is_oracle_race(cuda):
    torch = cuda
    from diffusionhard_b200.event import (EventSchedule, default_reveal_uniforms,
                                          run_event_driven_candidate_sampler_f32, reveal_steps_from_uniforms)

    V, mask, L, steps, seed = 777, 776, 96, 24, 12
    seen = {}

    def logits_fn(x, sel):
        g = torch.Generator(device="cuda").manual_seed(int(sel.sum().item()) + int(x.ne(mask).sum().item()))
        lg = torch.randn((sel.numel(), V), generator=g, device="cuda") * 3
        seen[tuple(sel.tolist())] = lg.cpu().numpy()
        return lg

    ids = torch.full((1, L), mask, dtype=torch.long, device="cuda")
    out, meta = run_event_driven_candidate_sampler_f32(logits_fn, ids, mask_token_id=mask, steps=steps,
                                                       reveal_seed=4, seed=seed)
    sched = EventSchedule.build(reveal_steps_from_uniforms(default_reveal_uniforms(4, (L,)), steps=steps,
                                                           sampling_epsilon=1e-5), steps)
    got = out[0].cpu().numpy()
    for k in range(steps + 1):
        sel = sched.rows(k).numpy()
        if sel.size == 0:
            continue
        lg = seen[tuple(sel.tolist())]
        if k < steps:
            exp, _ = pyoracle.noisy_argmax_f32(lg, mask, row_position=sel, row_key_hi=np.zeros_like(sel),
                                               row_eval=np.full_like(sel, k), key_lo=seed)
        else:
            exp = pyoracle.greedy_argmax_f32(lg, mask)
        assert np.array_equal(got[sel], exp), k
    assert meta["all_tokens_committed"] and not (got == mask).any()


def test_logits_function_sampler_argument_errors(cuda):
    torch = cuda
    from diffusionhard_b200.event import run_event_driven_candidate_sampler_f32

    f = lambda x, s: None  # noqa: E731
    with pytest.raises(ValueError, match="batch size one"):
        run_event_driven_candidate_sampler_f32(f, torch.zeros((2, 4), dtype=torch.long), mask_token_id=1,
                                               steps=4, reveal_seed=0)
    with pytest.raises(ValueError, match="reveal_seed"):
        run_event_driven_candidate_sampler_f32(f, torch.zeros((1, 4), dtype=torch.long), mask_token_id=1,
                                               steps=4, reveal_seed=-1)
    with pytest.raises(ValueError, match="one value per position"):
        run_event_driven_candidate_sampler_f32(f, torch.zeros((1, 4), dtype=torch.long), mask_token_id=1,
                                               steps=4, reveal_seed=0, reveal_uniforms=torch.zeros(3))


def _teacher_forced_check(torch, eng, qm, rs, final_ids, steps, seed, seq_offset=0):
    """Each non-empty transition k: canvas = final ids of rows revealed
    before k, mask elsewhere; the candidate of every row revealing at k is the
    oracle head on the GPU's hidden row of that canvas."""
    B, L = eng.B, eng.L
    mask = qm.config.mask_token_id
    ran = 0
    for k in range(steps + 1):
        sel = np.nonzero(rs.reshape(-1) == k)[0]
        if sel.size == 0:
            continue
        ran += 1
        canvas = np.where((rs.reshape(-1) >= 0) & (rs.reshape(-1) < k), final_ids.reshape(-1),
                          eng._ids_in.cpu().numpy())
        eng.tokens.copy_(torch.from_numpy(canvas.astype(np.int32)))
        eng.forward()
        rows = torch.from_numpy(sel.astype(np.int32)).cuda()
        cnt = torch.tensor([sel.size], dtype=torch.int32, device="cuda")
        eng.final_hidden_q(rows, cnt)
        torch.cuda.synchronize()
        hq = eng.head_q[: sel.size].cpu().numpy()
        hs = eng.head_scale[: sel.size].cpu().numpy()
        mode = 2 if k == steps else 1
        oids, _ = pyoracle.head_i8(mode, hq, qm.head.weight_q, mask, a_scale=hs, w_scale=qm.head.w_scale,
                                   bias=qm.head.bias, row_position=eng.pos_offset + sel % L,
                                   row_key_hi=seq_offset + sel // L, row_eval=np.full(sel.size, k), key_lo=seed)
        assert np.array_equal(final_ids.reshape(-1)[sel], oids), k
    return ran


@pytest.mark.parametrize("B,L,steps", [(1, 64, 64), (2, 96, 16)])
def test_engine_event_sampler_teacher_forced(cuda, small_model, B, L, steps):
    torch = cuda
    from diffusionhard_b200.api import run_event_driven_candidate_sampler
    from diffusionhard_b200.event import default_reveal_uniforms, reveal_steps_from_uniforms

    qm = small_model
    eng = MDLMEngine(qm, B, L)
    eng.seq_offset = 2
    mask = SMALL.mask_token_id
    ids = torch.full((B, L), mask, dtype=torch.int64)
    out, meta = run_event_driven_candidate_sampler(eng, ids, mask_token_id=mask, steps=steps, reveal_seed=6,
                                                   seed=9)
    assert out.device.type == "cpu" and out.shape == (B, L)
    final = out.numpy()
    assert not (final == mask).any() and meta["all_tokens_committed"]
    shape = (L,) if B == 1 else (B, L)
    rs = reveal_steps_from_uniforms(default_reveal_uniforms(6, shape).reshape(B, L), steps=steps,
                                    sampling_epsilon=1e-5).numpy()
    ran = _teacher_forced_check(torch, eng, qm, rs, final, steps, 9, seq_offset=2)
    assert meta["model_evaluations"] == ran
    assert meta["empty_transitions_elided"] == sum(
        1 for k in range(len(meta["transition_changed_tokens"])) if meta["transition_changed_tokens"][k] == 0)
    if B == 1 and steps == 64:
        assert meta["empty_transitions_elided"] > 0  # at L = 64 some transitions reveal nothing
    assert _device_error() == 0


def test_engine_event_sampler_graph_equals_eager(cuda, small_model):
    torch = cuda
    from diffusionhard_b200.api import run_event_driven_candidate_sampler

    eng = MDLMEngine(small_model, 2, 64)
    ids = torch.full((2, 64), SMALL.mask_token_id, dtype=torch.int64)
    a, ma = run_event_driven_candidate_sampler(eng, ids, mask_token_id=SMALL.mask_token_id, steps=32,
                                               reveal_seed=1, seed=4, graph=False)
    b, mb = run_event_driven_candidate_sampler(eng, ids, mask_token_id=SMALL.mask_token_id, steps=32,
                                               reveal_seed=1, seed=4, graph=True)
    c, _ = run_event_driven_candidate_sampler(eng, ids, mask_token_id=SMALL.mask_token_id, steps=32,
                                              reveal_seed=1, seed=4, graph=True)
    assert torch.equal(a, b) and torch.equal(a, c)
    assert {k: v for k, v in ma.items() if k not in WALL_KEYS} == {k: v for k, v in mb.items()
                                                                  if k not in WALL_KEYS}


def test_engine_prefix_event_sampler(cuda, small_model):
    torch = cuda
    from diffusionhard_b200.api import run_event_sampler
    from diffusionhard_b200.event import reveal_groups

    prefix = list(range(5, 5 + 32))
    eng = MDLMEngine(small_model, 1, 96)
    out, meta = run_event_sampler(eng, canvas_tokens=64, prefix_token_ids=prefix, steps=64, seed=3)
    assert out[0, :32].tolist() == prefix
    assert not (out[0, 32:] == SMALL.mask_token_id).any()
    groups = reveal_groups(positions=64, steps=64, seed=3)
    assert meta["model_evaluations"] == sum(1 for g in groups if g)
    assert meta["prefix_tokens"] == 32 and meta["selected_output_rows"] == 64
    rs = np.full((1, 96), -1, np.int64)
    for k, g in enumerate(groups):
        for p in g:
            rs[0, 32 + p] = k
    _teacher_forced_check(torch, eng, small_model, rs, out.numpy(), 64, 3)


def test_event_benchmark_cli_path(cuda):
    from diffusionhard_b200.event import benchmark_event_sampler

    r = benchmark_event_sampler(canvas_tokens=64, steps=16, seeds=(0,))
    assert r["selected_head_validation"]["maximum_absolute_logit_error"] == 0.0
    assert r["selected_head_validation"]["top1_agreement"] == 1.0
    assert r["all_tokens_committed"] and r["speedup"] > 0
    s = r["samples"][0]
    assert s["optimized"]["model_evaluations"] <= 17
    assert 50257 not in s["optimized_generated_token_ids"]


def test_engine_and_logits_function_samplers_agree(cuda, small_model):
    """The engine's fused selected-row head and the logits-function sampler
    over engine.selected_logits draw the same race on the same logits."""
    torch = cuda
    from diffusionhard_b200.api import run_event_driven_candidate_sampler
    from diffusionhard_b200.event import run_event_driven_candidate_sampler_f32

    mask = SMALL.mask_token_id
    eng = MDLMEngine(small_model, 1, 64)
    a, ma = run_event_driven_candidate_sampler(eng, torch.full((1, 64), mask, dtype=torch.int64),
                                               mask_token_id=mask, steps=32, reveal_seed=8, seed=21)
    ids = torch.full((1, 64), mask, dtype=torch.int64, device="cuda")
    b, mb = run_event_driven_candidate_sampler_f32(eng.selected_logits, ids, mask_token_id=mask, steps=32,
                                                   reveal_seed=8, seed=21)
    assert torch.equal(a, b.cpu())
    assert {k: v for k, v in ma.items() if k not in WALL_KEYS} == {k: v for k, v in mb.items()
                                                                  if k not in WALL_KEYS}
