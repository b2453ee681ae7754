"""Validation suites of the sampling path, run through the B200 kernels.

Two entry points keep the names, arguments, checks and report layout of the
reference's validation functions, but their sampled quantities come from the
device path this package ships instead of torch's RNG:

* ``validate_candidate_cache_equivalence`` (candidate_cache.py:90-254):
  - the analytic part is the same identity check: one DDPM transition over
    [tokens ; mask] factorises into a categorical draw and a Bernoulli reveal
    with p = (move_t - move_s) / move_t;
  - the Monte-Carlo part draws the factorised samples with the GPU sampler.
    The candidate is the Philox4x32-10 + factorized-Gumbel-Q10 race
    (dh_noisy_argmax_f32) over the log-probabilities. The reveal is the
    device reveal kernel (dh_candidate_reveal): word < floor(p * 2^32), with
    the loop's reveal words.
  - The histogram is compared with the reference's own torch.multinomial
    baseline and with the exact distribution.
* ``validate_rng_and_gumbel`` (rng.py:196-380):
  - Philox known answers computed on the GPU;
  - the distribution check and the full-vocabulary pathwise agreement run the
    GPU race on Philox words. The exact Gumbel argmax is computed over the
    same words, so agreement is path by path;
  - the mantissa sweep of the non-factorised table is a design-space study.
    It is restated in torch on the device (approximate_gumbel_q_from_words,
    rng.py:64-108).

Both report ``"sampler": "b200"`` and the device name.
"""

from __future__ import annotations

import math
from typing import Any, Dict, Sequence

from . import _lib
from .sampler import noisy_argmax_f32, philox4x32_10, reveal_words

# Random123 kat_vectors, Philox4x32 10-round entries (counter, key, output),
# the vectors rng.py:17-33 and philox_rng_test.cpp:24-39 check.
PHILOX4X32_10_KNOWN_ANSWERS = (
    ((0x00000000, 0x00000000, 0x00000000, 0x00000000), (0x00000000, 0x00000000),
     (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)),
    ((0xFFFFFFFF, 0xFFFFFFFF, 0xFFFFFFFF, 0xFFFFFFFF), (0xFFFFFFFF, 0xFFFFFFFF),
     (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)),
    ((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0),
     (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1)),
)

# Fixed shape of the device Gumbel tables (csrc/gen_gumbel_lut.py): Q5.10
# scores, 8-bit mantissa, exact tables for the three lowest exponents.
DEVICE_MANTISSA_BITS = 8
DEVICE_FRACTION_BITS = 10
DEVICE_CORRECTION_EXPONENTS = 3

# Positions per canvas when Monte-Carlo trials are laid out as sequences.
_TRIAL_POSITIONS = 1024


def _device_name(device: Any) -> str:
    import torch

    return torch.cuda.get_device_name(torch.device(device))


def _race_logits(log_weights: Any, rows: int, fraction_bits: int) -> Any:
    """fp32 [rows, V + 1] logits whose device Q10 rounding is exactly
    round(log_weights * 2^fraction_bits); column V is the (skipped) mask."""
    import torch

    scale = float(1 << fraction_bits)
    q = torch.round(log_weights.double() * scale)
    vocab = q.numel()
    row = torch.zeros(vocab + 1, dtype=torch.float32, device=log_weights.device)
    row[:vocab] = (q / scale).float()
    return row.expand(rows, vocab + 1).contiguous()


def _race_rows(rows: int, device: Any) -> tuple:
    """Row keying of a batch of trials laid out as canvases of
    _TRIAL_POSITIONS positions: (position, sequence) per row."""
    import torch

    r = torch.arange(rows, dtype=torch.int64)
    return r % _TRIAL_POSITIONS, r // _TRIAL_POSITIONS


def validate_candidate_cache_equivalence(
    *,
    positions: int = 64,
    vocabulary_size: int = 50_258,
    probability_bits: int = 16,
    analytic_vocabulary_size: int = 257,
    transitions: int = 16,
    monte_carlo_trials: int = 200_000,
    monte_carlo_vocabulary_size: int = 16,
    seed: int = 0,
    maximum_total_variation: float = 0.01,
    device: Any = "cuda",
) -> Dict[str, object]:
    """Analytic factorisation check plus a Monte-Carlo check of the GPU
    candidate sampler (candidate_cache.py:90-254)."""
    values = {
        "positions": positions,
        "vocabulary_size": vocabulary_size,
        "probability_bits": probability_bits,
        "analytic_vocabulary_size": analytic_vocabulary_size,
        "transitions": transitions,
        "monte_carlo_trials": monte_carlo_trials,
        "monte_carlo_vocabulary_size": monte_carlo_vocabulary_size,
    }
    if min(values.values()) <= 0:
        raise ValueError("all dimensions and trial counts must be positive")
    if probability_bits % 8:
        raise ValueError("probability_bits must be byte aligned")
    if not 0 < maximum_total_variation < 1:
        raise ValueError("maximum_total_variation must be between zero and one")
    if monte_carlo_vocabulary_size >= 65535:
        raise ValueError("monte_carlo_vocabulary_size must be below 65535")

    import torch

    dev = torch.device(device)
    generator = torch.Generator(device="cpu").manual_seed(seed)
    logits = torch.randn((positions, analytic_vocabulary_size), generator=generator, dtype=torch.float64)

    # -- analytic: the transition distribution factorises exactly (fp64, device)
    token_probabilities = torch.softmax(logits.to(dev), dim=-1)
    times = torch.linspace(1.0, 1e-5, transitions + 1, dtype=torch.float64, device=dev)
    maximum_absolute_error = 0.0
    maximum_row_sum_error = 0.0
    for transition in range(transitions):
        move_t = 0.999 * times[transition]
        move_s = 0.999 * times[transition + 1]
        token_mass = move_t - move_s
        original = torch.cat([token_probabilities * token_mass / move_t,
                              (move_s / move_t).expand(positions, 1)], dim=-1)
        reveal_probability = token_mass / move_t
        factored = torch.cat([token_probabilities * reveal_probability,
                              (1 - reveal_probability).expand(positions, 1)], dim=-1)
        maximum_absolute_error = max(maximum_absolute_error, float((original - factored).abs().max().item()))
        maximum_row_sum_error = max(maximum_row_sum_error, float((factored.sum(dim=-1) - 1).abs().max().item()))

    # -- Monte Carlo: baseline as the reference draws it, factored on the GPU
    mc_logits = torch.randn(monte_carlo_vocabulary_size, generator=generator, dtype=torch.float64)
    mc_probabilities = torch.softmax(mc_logits, dim=-1)
    move_t = torch.tensor(0.73, dtype=torch.float64)
    move_s = torch.tensor(0.41, dtype=torch.float64)
    original_distribution = torch.cat([mc_probabilities * (move_t - move_s) / move_t,
                                       (move_s / move_t).reshape(1)])
    baseline_samples = torch.multinomial(original_distribution, monte_carlo_trials, replacement=True,
                                         generator=generator)

    V = monte_carlo_vocabulary_size
    P = _TRIAL_POSITIONS
    sequences = -(-monte_carlo_trials // P)
    rows = sequences * P
    step = 0
    race_logits = _race_logits(torch.log(mc_probabilities).to(dev), rows, DEVICE_FRACTION_BITS)
    pos, seq = _race_rows(rows, dev)
    candidates = noisy_argmax_f32(race_logits, V, row_position=pos, row_key_hi=seq,
                                  row_eval=torch.full((rows,), step), key_lo=seed)
    threshold = min(1 << 32, math.floor(float((move_t - move_s) / move_t) * 4294967296.0))
    words = reveal_words(sequences, P, step, seed, device=dev)
    words32 = (words.to(torch.int64) & 0xFFFFFFFF).to(torch.int32)  # bit patterns of uint32
    tokens = torch.full((rows,), V, dtype=torch.int16, device=dev)
    cands16 = candidates.to(torch.int16)
    W = P // 64
    ones = torch.full((sequences * W,), -1, dtype=torch.int64, device=dev)
    active, valid = ones.clone(), ones.clone()
    results = torch.zeros(sequences, dtype=torch.int64, device=dev)
    _lib.call("dh_candidate_reveal", _lib.ptr(tokens), _lib.ptr(cands16), _lib.ptr(active), _lib.ptr(valid),
              _lib.ptr(words32.contiguous()), threshold, P, sequences, _lib.ptr(results), _lib.stream_handle())
    factored_samples = tokens[:monte_carlo_trials].to(torch.int64).cpu()

    baseline_histogram = torch.bincount(baseline_samples, minlength=V + 1).double() / monte_carlo_trials
    factored_histogram = torch.bincount(factored_samples, minlength=V + 1).double() / monte_carlo_trials
    total_variation = float((baseline_histogram - factored_histogram).abs().sum().item() / 2)
    total_variation_exact = float((original_distribution - factored_histogram).abs().sum().item() / 2)

    probability_cache_bytes = positions * vocabulary_size * (probability_bits // 8)
    candidate_id_bits = max(1, math.ceil(math.log2(vocabulary_size)))
    candidate_id_bytes = math.ceil(candidate_id_bits / 8)
    candidate_token_bytes = positions * candidate_id_bytes
    bitmap_bytes = 2 * math.ceil(positions / 8)
    candidate_cache_bytes = candidate_token_bytes + bitmap_bytes
    return {
        "method": "sample-token-on-model-evaluation-and-reuse-until-input-change",
        "correctness_class": "distribution-equivalent",
        "sampler": "b200",
        "device": _device_name(dev),
        "configuration": {**values, "seed": seed, "maximum_total_variation": maximum_total_variation},
        "analytic_factorization": {
            "maximum_absolute_probability_error": maximum_absolute_error,
            "maximum_row_sum_error": maximum_row_sum_error,
            "passed": maximum_absolute_error < 1e-12,
        },
        "monte_carlo": {
            "total_variation_distance": total_variation,
            "total_variation_to_exact_distribution": total_variation_exact,
            "candidate_source": "Philox4x32-10 + factorized Gumbel Q5.10 race (dh_noisy_argmax_f32)",
            "reveal_source": "dh_candidate_reveal, word < floor(p * 2^32)",
            "reveal_threshold_q32": threshold,
            "passed": total_variation <= maximum_total_variation,
        },
        "storage": {
            "full_probability_cache_bytes": probability_cache_bytes,
            "full_probability_cache_mib": probability_cache_bytes / 1024 ** 2,
            "candidate_token_bytes": candidate_token_bytes,
            "candidate_id_bits": candidate_id_bits,
            "candidate_id_bytes": candidate_id_bytes,
            "active_and_valid_bitmap_bytes": bitmap_bytes,
            "candidate_cache_bytes": candidate_cache_bytes,
            "storage_reduction_factor": probability_cache_bytes / candidate_cache_bytes,
        },
        "passed": maximum_absolute_error < 1e-12 and total_variation <= maximum_total_variation,
    }


def approximate_gumbel_q_from_words(words: Any, *, mantissa_bits: int = 8, fraction_bits: int = 10) -> Any:
    """Non-factorised leading-zero + mantissa Gumbel table (a design-space
    alternative the reference sweeps, rng.py:64-108), on the words' device:
    the bucket of d = 2^32-1-w keeps `mantissa_bits` bits below its leading
    one, its midpoint u gives round(-log(-log(u)) * 2^fraction_bits)."""
    import torch

    if not 1 <= mantissa_bits <= 16:
        raise ValueError("mantissa_bits must be between 1 and 16")
    if not 1 <= fraction_bits <= 12:
        raise ValueError("fraction_bits must be between 1 and 12")
    d = 0xFFFFFFFF - words.to(torch.int64)
    lg = torch.floor(torch.log2(d.clamp(min=1).double())).to(torch.int64)
    shift = (lg - mantissa_bits).clamp(min=0)
    width = torch.ones_like(shift) << shift
    mid = (torch.div(d, width, rounding_mode="floor") * width).double() + (width.double() - 1.0) / 2.0
    mid = torch.where(d == 0, torch.zeros_like(mid), mid)
    u = 1.0 - (mid + 0.5) / 4294967296.0
    return torch.round(-torch.log(-torch.log(u)) * (1 << fraction_bits)).to(torch.int64)


def _noise_words(rows: int, vocab: int, row_eval: int, key_lo: int, device: Any) -> Any:
    """The words the device race uses for `rows` x `vocab` (row r: position r,
    sequence 0): philox((v/4, r, row_eval, 0), (key_lo, 0))[v%4] -> int64."""
    import numpy as np

    groups = (vocab + 3) // 4
    r = np.repeat(np.arange(rows, dtype=np.int64), groups)
    g = np.tile(np.arange(groups, dtype=np.int64), rows)
    counters = np.stack([g, r, np.full_like(g, row_eval), np.zeros_like(g)], axis=1)
    keys = np.stack([np.full_like(g, key_lo), np.zeros_like(g)], axis=1)
    return philox4x32_10(counters, keys, device).view(rows, groups * 4)[:, :vocab]


def validate_rng_and_gumbel(
    *,
    distribution_trials: int = 200_000,
    distribution_vocabulary_size: int = 16,
    full_vocabulary_size: int = 50_258,
    full_vocabulary_batches: int = 16,
    full_vocabulary_batch_size: int = 64,
    mantissa_bits: Sequence[int] = (4, 6, 8),
    fraction_bits: int = 10,
    seed: int = 0,
    maximum_distribution_tv: float = 0.01,
    minimum_full_vocabulary_agreement: float = 0.995,
    device: Any = "cuda",
) -> Dict[str, object]:
    """Philox known answers, the race's distribution and its pathwise
    agreement with exact Gumbel-max, on the GPU (rng.py:196-380)."""
    integer_values = {
        "distribution_trials": distribution_trials,
        "distribution_vocabulary_size": distribution_vocabulary_size,
        "full_vocabulary_size": full_vocabulary_size,
        "full_vocabulary_batches": full_vocabulary_batches,
        "full_vocabulary_batch_size": full_vocabulary_batch_size,
        "fraction_bits": fraction_bits,
    }
    if min(integer_values.values()) <= 0 or not mantissa_bits:
        raise ValueError("trial counts, dimensions, and bit widths must be positive")
    if not 0 < maximum_distribution_tv < 1:
        raise ValueError("maximum_distribution_tv must be between zero and one")
    if not 0 < minimum_full_vocabulary_agreement <= 1:
        raise ValueError("minimum_full_vocabulary_agreement must be in (0, 1]")
    if max(mantissa_bits) != DEVICE_MANTISSA_BITS or fraction_bits != DEVICE_FRACTION_BITS:
        raise ValueError("the device race implements the 8-bit-mantissa Q5.10 tables: "
                         "max(mantissa_bits) must be 8 and fraction_bits 10")
    if max(distribution_vocabulary_size, full_vocabulary_size) >= 65535:
        raise ValueError("vocabulary sizes must be below 65535")

    import torch

    dev = torch.device(device)
    kat_counters = [c for c, _, _ in PHILOX4X32_10_KNOWN_ANSWERS]
    kat_keys = [k for _, k, _ in PHILOX4X32_10_KNOWN_ANSWERS]
    kat_out = philox4x32_10(kat_counters, kat_keys, dev).cpu().tolist()
    known_answers = []
    for (counter, key, expected), actual in zip(PHILOX4X32_10_KNOWN_ANSWERS, kat_out):
        known_answers.append({
            "counter": ["%08x" % w for w in counter],
            "key": ["%08x" % w for w in key],
            "expected": ["%08x" % w for w in expected],
            "actual": ["%08x" % w for w in actual],
            "passed": tuple(actual) == tuple(expected),
        })

    generator = torch.Generator(device="cpu").manual_seed(seed)
    scale = 1 << fraction_bits

    # -- distribution of the device race on a small vocabulary
    logits = torch.randn(distribution_vocabulary_size, generator=generator, dtype=torch.float64)
    target = torch.softmax(logits, dim=-1)
    V = distribution_vocabulary_size
    rows = distribution_trials
    pos, seq = _race_rows(rows, dev)
    ids = noisy_argmax_f32(_race_logits(logits.to(dev), rows, fraction_bits), V, row_position=pos,
                           row_key_hi=seq, row_eval=torch.zeros(rows, dtype=torch.int64), key_lo=seed)
    empirical = torch.bincount(ids.to(torch.int64).cpu(), minlength=V).double() / rows
    distribution_tv = float(0.5 * (empirical - target).abs().sum().item())

    # -- full vocabulary: device race vs exact Gumbel-max on the same words
    agreements = {bits: 0 for bits in mantissa_bits}
    factorized_matches = 0
    total = full_vocabulary_batches * full_vocabulary_batch_size
    FV, BS = full_vocabulary_size, full_vocabulary_batch_size
    for batch in range(full_vocabulary_batches):
        batch_logits = torch.randn((BS, FV), generator=generator, dtype=torch.float32).to(torch.float64).to(dev)
        words = _noise_words(BS, FV, batch, seed, dev)
        uniforms = (words.double() + 0.5) / 4294967296.0
        exact = (batch_logits - torch.log(-torch.log(uniforms))).argmax(dim=-1)
        logits_q = torch.round(batch_logits * scale)
        for bits in mantissa_bits:
            approx = approximate_gumbel_q_from_words(words, mantissa_bits=bits, fraction_bits=fraction_bits)
            agreements[bits] += int((logits_q.to(torch.int64) + approx).argmax(dim=-1).eq(exact).sum().item())
        race = torch.zeros((BS, FV + 1), dtype=torch.float32, device=dev)
        race[:, :FV] = (logits_q / scale).float()
        got = noisy_argmax_f32(race, FV, row_position=torch.arange(BS), row_key_hi=torch.zeros(BS),
                               row_eval=torch.full((BS,), batch), key_lo=seed)
        factorized_matches += int(got.to(torch.int64).eq(exact).sum().item())

    sweep = []
    for bits in mantissa_bits:
        agreement = agreements[bits] / total
        sweep.append({
            "mantissa_bits": bits,
            "conservative_lut_entries": 33 * (1 << bits),
            "int16_lut_bytes": 33 * (1 << bits) * 2,
            "matching_candidates": agreements[bits],
            "samples": total,
            "pathwise_agreement": agreement,
            "passed": agreement >= minimum_full_vocabulary_agreement,
        })
    factorized_agreement = factorized_matches / total
    factorized = {
        "mantissa_bits": DEVICE_MANTISSA_BITS,
        "correction_exponents": DEVICE_CORRECTION_EXPONENTS,
        "int16_lut_bytes": (1 + DEVICE_CORRECTION_EXPONENTS) * (1 << DEVICE_MANTISSA_BITS) * 2,
        "matching_candidates": factorized_matches,
        "samples": total,
        "pathwise_agreement": factorized_agreement,
        "source": "dh_noisy_argmax_f32 (device race)",
        "passed": factorized_agreement >= minimum_full_vocabulary_agreement,
    }
    kat_passed = all(item["passed"] for item in known_answers)
    return {
        "sampler": "b200",
        "device": _device_name(dev),
        "philox4x32_10": {
            "known_answer_source": "Random123 tests/kat_vectors, Philox4x32 10-round entries",
            "known_answers": known_answers,
            "passed": kat_passed,
        },
        "distribution_validation": {
            "trials": distribution_trials,
            "vocabulary_size": distribution_vocabulary_size,
            "mantissa_bits": DEVICE_MANTISSA_BITS,
            "fraction_bits": fraction_bits,
            "total_variation_distance": distribution_tv,
            "maximum_total_variation": maximum_distribution_tv,
            "passed": distribution_tv <= maximum_distribution_tv,
        },
        "full_vocabulary_stress": {
            "vocabulary_size": full_vocabulary_size,
            "batches": full_vocabulary_batches,
            "batch_size": full_vocabulary_batch_size,
            "samples": total,
            "fraction_bits": fraction_bits,
            "minimum_pathwise_agreement": minimum_full_vocabulary_agreement,
            "sweep": sweep,
            "full_table_reference": next(i for i in sweep if i["mantissa_bits"] == max(mantissa_bits)),
            "selected_design": "factorized-mantissa-plus-three-correction-tables",
            "factorized_design": factorized,
            "selected_passed": bool(factorized["passed"]),
        },
        "scope": ("philox-known-answer-and-device-gumbel-race-validation; "
                  "not-a-complete-rng-statistical-suite"),
        "passed": kat_passed and distribution_tv <= maximum_distribution_tv and factorized["passed"],
    }
