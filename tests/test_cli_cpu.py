"""Host-side checks of the command line and validation entry points (no GPU):
subcommand names and flags as the reference's cli.py declares them, and the
argument errors raised before any device work."""

import pytest
import torch

from diffusionhard_b200.cli import build_parser
from diffusionhard_b200.conditioned import _terminal_kv_valid
from diffusionhard_b200.prefix import analyze_mdlm_prefix_drift
from diffusionhard_b200.validation import validate_candidate_cache_equivalence, validate_rng_and_gumbel


def _flags(sub):
    parser = build_parser()
    action = next(a for a in parser._actions if a.dest == "command")
    return {o for a in action.choices[sub]._actions for o in a.option_strings if o.startswith("--")}


# flags of the reference subcommands (cli.py:155-213, 260-342, 375-409, 552-563, 666-682, 724-739, 769-807)
REFERENCE_FLAGS = {
    "trace-mdlm": {"--out", "--model-id", "--revision", "--device", "--canvas-tokens", "--steps", "--warmup",
                   "--seed", "--sampler", "--local-files-only"},
    "validate-candidate-cache": {"--positions", "--vocabulary-size", "--probability-bits",
                                 "--analytic-vocabulary-size", "--transitions", "--monte-carlo-trials",
                                 "--monte-carlo-vocabulary-size", "--seed", "--maximum-total-variation", "--out"},
    "validate-rng-gumbel": {"--distribution-trials", "--distribution-vocabulary-size", "--full-vocabulary-size",
                            "--full-vocabulary-batches", "--full-vocabulary-batch-size", "--mantissa-bits",
                            "--fraction-bits", "--seed", "--maximum-distribution-tv",
                            "--minimum-full-vocabulary-agreement", "--out"},
    "analyze-mdlm-prefix-drift": {"--out", "--model-id", "--revision", "--device", "--prefix-text",
                                  "--suffix-tokens", "--changed-suffix-tokens", "--warmup", "--timing-repeats",
                                  "--seed", "--local-files-only"},
    "generate-mdlm-conditioned": {"--out", "--model-id", "--revision", "--device", "--prefix-tokens",
                                  "--suffix-tokens", "--samples", "--steps", "--seed", "--local-files-only"},
    "run-mdlm-two-turn": {"--out", "--model-id", "--revision", "--device", "--dataset-id", "--dataset-config",
                          "--dataset-revision", "--split", "--prefix-tokens", "--first-answer-tokens",
                          "--followup-tokens", "--second-answer-tokens", "--samples", "--steps", "--seed",
                          "--local-files-only"},
    "export-mdlm-hardware-package": {"--out-dir", "--model-id", "--revision", "--device", "--local-files-only"},
    "validate-mdlm-hardware-package": {"--package-dir"},
    "validate-hardware-fixed-mlp": {"--package-dir", "--block", "--activation-granularity",
                                    "--down-activation-granularity", "--smoothquant-alpha", "--out"},
    "sweep-hardware-fixed-mlp": {"--package-dir", "--activation-granularity", "--down-activation-granularity",
                                 "--out"},
    "sweep-fixed-layernorm": {"--package-dir", "--out"},
    "sweep-fixed-rotary": {"--package-dir", "--out"},
    "sweep-fixed-attention": {"--package-dir", "--out"},
    "benchmark-mdlm-apple": {"--out", "--model-id", "--revision", "--device", "--canvas-tokens", "--steps",
                             "--seeds", "--local-files-only"},
    # cli.py:260-272, 286-342
    "sweep-qkv-weight-precision": {"--package-dir", "--weight-bits", "--smoothquant-alphas", "--out"},
    "screen-packed-int8-attention": {"--package-dir", "--out"},
    "screen-packed-int8-attention-heldout": {"--package-dir", "--device", "--seeds", "--out"},
    "screen-packed-int8-attention-logits": {"--package-dir", "--device", "--seeds", "--preserve-qk18",
                                            "--preserve-pv18", "--qk-bits", "--qk-scale-mode",
                                            "--qk-multiplier-fraction-bits", "--pv-probability-levels",
                                            "--pv-probability-sum-correction", "--pv-value-bits", "--out"},
}


@pytest.mark.parametrize("sub", sorted(REFERENCE_FLAGS))
def test_subcommands_accept_the_reference_flags(sub):
    assert REFERENCE_FLAGS[sub] <= _flags(sub)


def test_defaults_match_the_reference():
    p = build_parser()
    a = p.parse_args(["validate-candidate-cache"])
    assert (a.positions, a.vocabulary_size, a.transitions, a.monte_carlo_trials, a.maximum_total_variation) == \
        (64, 50258, 16, 200000, 0.01)
    a = p.parse_args(["validate-rng-gumbel"])
    assert a.mantissa_bits == [4, 6, 8] and a.full_vocabulary_batches == 16 and a.distribution_trials == 200000
    a = p.parse_args(["benchmark-mdlm-apple"])
    assert (a.canvas_tokens, a.steps, a.seeds) == (64, 64, [0, 1, 2])
    a = p.parse_args(["trace-mdlm", "--out", "x.json"])
    assert (a.canvas_tokens, a.steps, a.sampler) == (64, 64, "ddpm-cache")
    a = p.parse_args(["sweep-qkv-weight-precision", "--package-dir", "x"])
    assert (a.weight_bits, a.smoothquant_alphas) == ([8, 16], [])
    a = p.parse_args(["screen-packed-int8-attention-logits", "--package-dir", "x"])
    assert (a.qk_bits, a.qk_scale_mode, a.qk_multiplier_fraction_bits, a.pv_probability_levels, a.pv_value_bits,
            a.preserve_qk18, a.pv_probability_sum_correction) == (8, "calibrated-head", 24, 127, 8, False, False)


def test_validation_argument_errors_precede_device_work():
    with pytest.raises(ValueError, match="byte aligned"):
        validate_candidate_cache_equivalence(probability_bits=7)
    with pytest.raises(ValueError, match="positive"):
        validate_candidate_cache_equivalence(monte_carlo_trials=0)
    with pytest.raises(ValueError, match="between zero and one"):
        validate_candidate_cache_equivalence(maximum_total_variation=1.5)
    with pytest.raises(ValueError, match="8-bit-mantissa"):
        validate_rng_and_gumbel(mantissa_bits=[4, 6])
    with pytest.raises(ValueError, match=r"\(0, 1\]"):
        validate_rng_and_gumbel(minimum_full_vocabulary_agreement=0)
    with pytest.raises(ValueError, match="changed_suffix_tokens"):
        analyze_mdlm_prefix_drift(suffix_tokens=32, changed_suffix_tokens=33)


def _counters(rows):
    return torch.tensor(rows, dtype=torch.int32).view(-1)


def test_terminal_kv_valid_follows_the_last_evaluation():
    """Counters are (active, changed, evaluated) per transition.  An
    evaluation only runs while a position is masked, and every masked
    position is filled later (by a reveal or the final greedy pass), so the
    last evaluated canvas never equals the final one: terminal K / V are
    never valid for this loop (conditioned.py:226-229 gives the same)."""
    # reveals after the last evaluation
    assert not _terminal_kv_valid({"sampling_transitions": 2}, _counters([[4, 2, 1], [2, 2, 1]]), 2)
    # last evaluation revealed nothing, a later cache hit did
    assert not _terminal_kv_valid({"sampling_transitions": 3}, _counters([[4, 2, 1], [2, 0, 1], [2, 2, 0]]), 3)
    # masks left for the final greedy pass
    assert not _terminal_kv_valid({"sampling_transitions": 2}, _counters([[4, 1, 1], [3, 1, 1]]), 2)
    # no transition ran (nothing masked): no evaluation, nothing cached
    assert not _terminal_kv_valid({"sampling_transitions": 0}, _counters([[0, 0, 0]]), 1)
