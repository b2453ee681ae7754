"""GPU sampler distribution checks and the command line on the device.

* candidate-cache equivalence (candidate_cache.py:90-254) with the
  factorised samples drawn by the device race + reveal kernels: the
  reference's own small case and the 64-position, 50,258-token,
  64-transition, 500,000-trial variant;
* the RNG / Gumbel validation (rng.py:196-380) on the device race;
* trace-mdlm at the reference's default canvas (64 tokens), prefix drift and
  conditioned generation on a small model.
"""

import json

import numpy as np
import pytest

from diffusionhard_b200.model import MDLMConfig, build_quantized

pytestmark = pytest.mark.gpu

SMALL = MDLMConfig(vocab_size=1000, mask_token_id=999, blocks=2)


@pytest.fixture(scope="module")
def small_model():
    return build_quantized(SMALL, seed=0)


def test_candidate_cache_equivalence_reference_small_case(cuda):
    from diffusionhard_b200.validation import validate_candidate_cache_equivalence

    # tests/test_candidate_cache.py:9-30
    r = validate_candidate_cache_equivalence(positions=8, vocabulary_size=128, analytic_vocabulary_size=17,
                                             transitions=4, monte_carlo_trials=50_000,
                                             monte_carlo_vocabulary_size=4, maximum_total_variation=0.02, seed=3)
    assert r["analytic_factorization"]["passed"] is True
    assert r["analytic_factorization"]["maximum_absolute_probability_error"] < 1e-12
    assert r["monte_carlo"]["passed"] is True
    assert r["storage"]["candidate_cache_bytes"] == 10
    assert r["storage"]["candidate_id_bits"] == 7
    assert r["storage"]["full_probability_cache_bytes"] == 2048
    assert r["passed"] is True


def test_candidate_cache_equivalence_500k_trials(cuda):
    """validate-candidate-cache --positions 64 --vocabulary-size 50258
    --transitions 64 --monte-carlo-trials 500000, factorised samples from the
    device sampler."""
    from diffusionhard_b200.validation import validate_candidate_cache_equivalence

    r = validate_candidate_cache_equivalence(positions=64, vocabulary_size=50258, transitions=64,
                                             monte_carlo_trials=500_000)
    assert r["passed"] is True
    assert r["monte_carlo"]["total_variation_distance"] <= 0.01
    assert r["monte_carlo"]["total_variation_to_exact_distribution"] <= 0.01
    assert r["storage"]["candidate_cache_bytes"] == 144
    assert r["storage"]["candidate_id_bytes"] == 2


def test_rng_and_gumbel_reference_small_case(cuda):
    from diffusionhard_b200.validation import validate_rng_and_gumbel

    # tests/test_rng.py:29-44
    r = validate_rng_and_gumbel(distribution_trials=20_000, distribution_vocabulary_size=8, full_vocabulary_size=257,
                                full_vocabulary_batches=2, full_vocabulary_batch_size=8, mantissa_bits=[4, 8],
                                maximum_distribution_tv=0.03, minimum_full_vocabulary_agreement=0.9)
    assert r["philox4x32_10"]["passed"] is True
    assert r["distribution_validation"]["passed"] is True
    assert r["full_vocabulary_stress"]["selected_passed"] is True
    assert r["passed"] is True


def test_rng_and_gumbel_default_sizes(cuda):
    from diffusionhard_b200.validation import validate_rng_and_gumbel

    r = validate_rng_and_gumbel()
    assert r["passed"] is True
    fz = r["full_vocabulary_stress"]["factorized_design"]
    assert fz["samples"] == 1024 and fz["pathwise_agreement"] >= 0.995
    sweep = {s["mantissa_bits"]: s["pathwise_agreement"] for s in r["full_vocabulary_stress"]["sweep"]}
    assert sweep[4] <= sweep[8]  # the coarse table agrees less often


def test_race_words_match_the_oracle(cuda):
    """The words the validation feeds the exact Gumbel argmax are the race's
    own: philox((v/4, r, eval, 0), (seed, 0))."""
    from diffusionhard_b200.validation import _noise_words
    from oracle import pyoracle

    w = _noise_words(3, 37, 5, 11, "cuda").cpu().numpy()
    for r in range(3):
        for v in range(37):
            assert int(w[r, v]) == pyoracle.philox((v // 4, r, 5, 0), (11, 0))[v % 4]


def test_trace_mdlm_cli_default_canvas(cuda, tmp_path):
    from diffusionhard_b200.cli import main

    out = tmp_path / "trace.json"
    assert main(["trace-mdlm", "--out", str(out), "--steps", "16", "--warmup", "0",
                 "--sampler", "ddpm-candidate-cache"]) == 0
    trace = json.loads(out.read_text())
    meta = trace["metadata"]
    assert meta["all_tokens_committed"] is True
    assert len(meta["generated_token_ids"]) == 64
    assert len(trace["steps"]) == meta["model_evaluations"]
    assert meta["sampling_transitions"] == 16
    assert sum(meta["transition_changed_tokens"]) + (meta["transition_active_tokens"][-1] -
                                                     meta["transition_changed_tokens"][-1]) == 64
    assert all(s["sigma"] > 0 for s in trace["steps"])


def test_prefix_drift_analysis(cuda, small_model):
    from diffusionhard_b200.prefix import analyze_mdlm_prefix_drift

    r = analyze_mdlm_prefix_drift(quantized=small_model, prefix_tokens=64, suffix_tokens=32,
                                  changed_suffix_tokens=3, timing_repeats=2)
    assert len(r["layers"]) == SMALL.blocks
    # block 0's K / V come from the prefix embeddings alone; block 1 sees the edit
    assert r["layers"][0]["prefix_kv_exact_equal"] is True
    assert r["first_drifting_layer"] == 1
    iso = r["prefix_isolated_cache_experiment"]
    assert iso["all_prefix_kv_exact_equal_after_suffix_edit"] is True
    assert iso["suffix_logit_drift"]["exact_equal"] is True
    assert iso["suffix_top1_agreement"] == 1.0
    assert len(r["changed_absolute_positions"]) == 3
    assert all(64 <= p < 96 for p in r["changed_absolute_positions"])


def test_conditioned_generation_cache_equals_recompute(cuda, small_model):
    from diffusionhard_b200.conditioned import evaluate_conditioned_mdlm_ddpm

    r = evaluate_conditioned_mdlm_ddpm(quantized=small_model, prefix_tokens=64, suffix_tokens=32, samples=2,
                                       steps=8)
    agg = r["aggregate"]
    assert agg["exact_cached_sequences"] == 2
    assert agg["identical_cached_transition_schedules"] == 2
    for s in r["sample_results"]:
        for path in ("original_full_attention", "prefix_isolated_recompute", "prefix_isolated_cache"):
            assert SMALL.mask_token_id not in s[path]["generated_token_ids"]
        # the recompute path runs the prefix forward with every evaluation
        assert s["prefix_isolated_recompute"]["model_forward_latency_ms"] > 0
    assert agg["prefix_kv_bytes"] == 2 * SMALL.blocks * 64 * 768 * 2


def test_api_measurements_follow_the_reference_shape(cuda, small_model):
    import torch

    from diffusionhard_b200.api import run_ddpm_candidate_cache_sampler
    from diffusionhard_b200.engine import MDLMEngine

    eng = MDLMEngine(small_model, 2, 96)
    ids = torch.full((2, 96), SMALL.mask_token_id, dtype=torch.long)
    out, meas, meta = run_ddpm_candidate_cache_sampler(eng, ids, mask_token_id=SMALL.mask_token_id, steps=12,
                                                       seed=4)
    assert out.device == ids.device and out.shape == ids.shape
    assert len(meas) == meta["model_evaluations"]
    assert [m.step_id for m in meas] == sorted(m.step_id for m in meas)
    t = torch.linspace(1.0, 1e-5, 13)
    sig = (-torch.log1p(-(1 - 1e-3) * t)).tolist()
    for m in meas:
        if m.step_id < meta["sampling_transitions"]:
            assert m.sigma == pytest.approx(sig[m.step_id], rel=1e-6)
            assert m.active_tokens == meta["transition_active_tokens"][m.step_id]
    assert np.isfinite([m.elapsed_s for m in meas]).all()
