"""Command line of the B200 path: the reference's subcommands for this path
(src/diffusion_accel/cli.py) with their names and flags, backed by the
device kernels.

  trace-mdlm                  cli.py:375-396, 1209-1245 (mdlm.run_mdlm_trace)
  validate-candidate-cache    cli.py:552-563
  validate-rng-gumbel         cli.py:666-682
  analyze-mdlm-prefix-drift   cli.py:724-739
  generate-mdlm-conditioned   cli.py:769-787
  run-mdlm-two-turn               cli.py:788-807, 1616-1640 (multiturn.evaluate_two_turn_mdlm_session)
  export-mdlm-hardware-package    cli.py:155-163, 856-880
  validate-mdlm-hardware-package  cli.py:165-169, 882-885
  validate-hardware-fixed-mlp     cli.py:187-200, 905-917
  sweep-hardware-fixed-mlp        cli.py:202-213
  sweep-fixed-layernorm / sweep-fixed-rotary / sweep-fixed-attention   cli.py:240-258
  sweep-qkv-weight-precision      cli.py:260-272, 986-1000
  screen-packed-int8-attention / -heldout / -logits   cli.py:286-342, 1017-1058
  benchmark-mdlm-event        cli.py:397-409 (benchmark-mdlm-apple, apple_mdlm.py:203-390),
                              also accepted under the reference's name

Differences, all forced by what a run here has:
- no checkpoint: --model-id / --revision / --local-files-only are recorded
  but the weights are the seeded random-init stand-in (--weights-seed), or
  an HF-layout model.safetensors given by --checkpoint where a command
  takes one;
- no tokenizer: text is not decoded and --prefix-text is refused, while
  --prefix-tokens takes a seeded synthetic prefix;
- no dataset: windows are seeded synthetic ids;
- trace-mdlm offers the two candidate-cache samplers the device loop
  implements, and writes a JSON trace rather than the reference's
  workload-trace IR.
Lengths are multiples of 32 (the kernels' granule), so run-mdlm-two-turn's
answer and follow-up blocks default to 32 tokens where the reference's
default to 16.
"""

from __future__ import annotations

import argparse
import json
from pathlib import Path
from typing import Any, List, Optional

DEFAULT_MODEL_ID = "kuleshov-group/mdlm-owt"
DEFAULT_REVISION = "d0958fa851335ece6c15260ce0025f030673c0fb"


def build_parser() -> argparse.ArgumentParser:
    parser = argparse.ArgumentParser(prog="diffusionhard-b200")
    sub = parser.add_subparsers(dest="command", required=True)

    mdlm = sub.add_parser("trace-mdlm", help="run the MDLM candidate-cache loop on the GPU and write a trace")
    mdlm.add_argument("--out", type=Path, required=True)
    mdlm.add_argument("--model-id", default=DEFAULT_MODEL_ID)
    mdlm.add_argument("--revision", default=DEFAULT_REVISION)
    mdlm.add_argument("--device", default="cuda")
    mdlm.add_argument("--canvas-tokens", type=int, default=64)
    mdlm.add_argument("--steps", type=int, default=64)
    mdlm.add_argument("--warmup", type=int, default=1)
    mdlm.add_argument("--seed", type=int, default=0)
    mdlm.add_argument("--sampler", choices=["ddpm-cache", "ddpm-candidate-cache"], default="ddpm-cache")
    mdlm.add_argument("--local-files-only", action="store_true")
    mdlm.add_argument("--batch", type=int, default=1)
    mdlm.add_argument("--weights-seed", type=int, default=0)

    cand = sub.add_parser("validate-candidate-cache",
                          help="validate compact candidate caching against DDPM transition sampling")
    cand.add_argument("--positions", type=int, default=64)
    cand.add_argument("--vocabulary-size", type=int, default=50_258)
    cand.add_argument("--probability-bits", type=int, default=16)
    cand.add_argument("--analytic-vocabulary-size", type=int, default=257)
    cand.add_argument("--transitions", type=int, default=16)
    cand.add_argument("--monte-carlo-trials", type=int, default=200_000)
    cand.add_argument("--monte-carlo-vocabulary-size", type=int, default=16)
    cand.add_argument("--seed", type=int, default=0)
    cand.add_argument("--maximum-total-variation", type=float, default=0.01)
    cand.add_argument("--out", type=Path)
    cand.add_argument("--device", default="cuda")

    rng = sub.add_parser("validate-rng-gumbel", help="validate Philox vectors and the Gumbel race")
    rng.add_argument("--distribution-trials", type=int, default=200_000)
    rng.add_argument("--distribution-vocabulary-size", type=int, default=16)
    rng.add_argument("--full-vocabulary-size", type=int, default=50_258)
    rng.add_argument("--full-vocabulary-batches", type=int, default=16)
    rng.add_argument("--full-vocabulary-batch-size", type=int, default=64)
    rng.add_argument("--mantissa-bits", nargs="+", type=int, default=[4, 6, 8])
    rng.add_argument("--fraction-bits", type=int, default=10)
    rng.add_argument("--seed", type=int, default=0)
    rng.add_argument("--maximum-distribution-tv", type=float, default=0.01)
    rng.add_argument("--minimum-full-vocabulary-agreement", type=float, default=0.995)
    rng.add_argument("--out", type=Path)
    rng.add_argument("--device", default="cuda")

    drift = sub.add_parser("analyze-mdlm-prefix-drift",
                           help="measure per-layer prefix K/V drift after a suffix edit")
    drift.add_argument("--out", type=Path)
    drift.add_argument("--model-id", default=DEFAULT_MODEL_ID)
    drift.add_argument("--revision", default=DEFAULT_REVISION)
    drift.add_argument("--device", default="cuda")
    drift.add_argument("--prefix-text")
    drift.add_argument("--prefix-tokens", type=int, default=64)
    drift.add_argument("--suffix-tokens", type=int, default=32)
    drift.add_argument("--changed-suffix-tokens", type=int, default=1)
    drift.add_argument("--warmup", type=int, default=1)
    drift.add_argument("--timing-repeats", type=int, default=5)
    drift.add_argument("--seed", type=int, default=0)
    drift.add_argument("--local-files-only", action="store_true")
    drift.add_argument("--weights-seed", type=int, default=0)

    event = sub.add_parser("benchmark-mdlm-event", aliases=["benchmark-mdlm-apple"],
                           help="benchmark the event-driven selected-row MDLM sampler against the candidate cache")
    event.add_argument("--out", type=Path)
    event.add_argument("--model-id", default=DEFAULT_MODEL_ID)
    event.add_argument("--revision", default=DEFAULT_REVISION)
    event.add_argument("--device", default="cuda")
    event.add_argument("--canvas-tokens", type=int, default=64)
    event.add_argument("--steps", type=int, default=64)
    event.add_argument("--seeds", nargs="+", type=int, default=[0, 1, 2])
    event.add_argument("--local-files-only", action="store_true")
    event.add_argument("--weights-seed", type=int, default=0)

    turn = sub.add_parser("run-mdlm-two-turn", help="run an exact block-causal two-turn retained-K/V session")
    turn.add_argument("--out", type=Path)
    turn.add_argument("--model-id", default=DEFAULT_MODEL_ID)
    turn.add_argument("--revision", default=DEFAULT_REVISION)
    turn.add_argument("--device", default="cuda")
    turn.add_argument("--dataset-id", default="Salesforce/wikitext")
    turn.add_argument("--dataset-config", default="wikitext-2-raw-v1")
    turn.add_argument("--dataset-revision", default="b08601e04326c79dfdd32d625aee71d232d685c3")
    turn.add_argument("--split", default="test")
    turn.add_argument("--prefix-tokens", type=int, default=64)
    turn.add_argument("--first-answer-tokens", type=int, default=32)
    turn.add_argument("--followup-tokens", type=int, default=32)
    turn.add_argument("--second-answer-tokens", type=int, default=32)
    turn.add_argument("--samples", type=int, default=3)
    turn.add_argument("--steps", type=int, default=64)
    turn.add_argument("--seed", type=int, default=0)
    turn.add_argument("--local-files-only", action="store_true")
    turn.add_argument("--weights-seed", type=int, default=0)

    export = sub.add_parser("export-mdlm-hardware-package",
                            help="export 64-token goldens and constant-folded FP16 weights")
    export.add_argument("--out-dir", type=Path, required=True)
    export.add_argument("--model-id", default=DEFAULT_MODEL_ID)
    export.add_argument("--revision", default=DEFAULT_REVISION)
    export.add_argument("--device", default="cpu")
    export.add_argument("--local-files-only", action="store_true")
    export.add_argument("--checkpoint", type=Path, help="HF-layout model.safetensors (default: the stand-in)")
    export.add_argument("--weights-seed", type=int, default=0)

    vpkg = sub.add_parser("validate-mdlm-hardware-package",
                          help="verify package hashes, safetensors metadata, and aligned DDR layout")
    vpkg.add_argument("--package-dir", type=Path, required=True)

    hfm = sub.add_parser("validate-hardware-fixed-mlp",
                         help="validate one package MLP through RTL-equivalent requant and GELU on the GPU")
    hfm.add_argument("--package-dir", type=Path, required=True)
    hfm.add_argument("--block", type=int, default=0)
    hfm.add_argument("--activation-granularity", choices=["tensor", "token"], default="token")
    hfm.add_argument("--down-activation-granularity", choices=["tensor", "token"])
    hfm.add_argument("--smoothquant-alpha", type=float, default=0.75)
    hfm.add_argument("--out", type=Path)

    sfm = sub.add_parser("sweep-hardware-fixed-mlp",
                         help="run the RTL-equivalent fixed MLP validation across all 12 blocks")
    sfm.add_argument("--package-dir", type=Path, required=True)
    sfm.add_argument("--activation-granularity", choices=["tensor", "token"], default="token")
    sfm.add_argument("--down-activation-granularity", choices=["tensor", "token"])
    sfm.add_argument("--out", type=Path)

    for name, help_text in (("sweep-fixed-layernorm", "validate Q13.10 to Q5.12 LayerNorm at all H0 boundaries"),
                            ("sweep-fixed-rotary", "validate Q5.12 rotary Q/K transforms at all H0 blocks"),
                            ("sweep-fixed-attention", "validate fixed attention, output projection, and residual")):
        fx = sub.add_parser(name, help=help_text + " (on the GPU)")
        fx.add_argument("--package-dir", type=Path, required=True)
        fx.add_argument("--out", type=Path)

    qkvp = sub.add_parser("sweep-qkv-weight-precision",
                          help="compare INT8 and INT16 QKV weights at all H0 boundaries (on the GPU)")
    qkvp.add_argument("--package-dir", type=Path, required=True)
    qkvp.add_argument("--weight-bits", type=int, nargs="+", choices=[8, 16], default=[8, 16])
    qkvp.add_argument("--smoothquant-alphas", type=float, nargs="+", default=[])
    qkvp.add_argument("--out", type=Path)

    ia = sub.add_parser("screen-packed-int8-attention",
                        help="screen paired-token INT8 QK and PV on all captured H0 blocks (on the GPU)")
    ia.add_argument("--package-dir", type=Path, required=True)
    ia.add_argument("--out", type=Path)
    for name, help_text in (("screen-packed-int8-attention-heldout",
                             "apply captured INT8 attention calibration to fresh canvases"),
                            ("screen-packed-int8-attention-logits",
                             "propagate packed INT8 attention error through all twelve blocks")):
        sc = sub.add_parser(name, help=help_text + " (on the GPU)")
        sc.add_argument("--package-dir", type=Path, required=True)
        sc.add_argument("--device", choices=["auto", "cuda"], default="auto")
        sc.add_argument("--seeds", type=int, nargs="+")
        sc.add_argument("--model-id", default=DEFAULT_MODEL_ID)
        sc.add_argument("--revision", default=DEFAULT_REVISION)
        sc.add_argument("--checkpoint", type=Path, help="HF-layout model.safetensors (default: the stand-in)")
        sc.add_argument("--weights-seed", type=int, default=0)
        sc.add_argument("--out", type=Path)
        if name.endswith("-logits"):
            sc.add_argument("--preserve-qk18", action="store_true")
            sc.add_argument("--preserve-pv18", action="store_true")
            sc.add_argument("--qk-bits", type=int, choices=[8, 9], default=8)
            sc.add_argument("--qk-scale-mode", choices=["calibrated-head", "dynamic-vector"],
                            default="calibrated-head")
            sc.add_argument("--qk-multiplier-fraction-bits", type=int, choices=[17, 24], default=24)
            sc.add_argument("--pv-probability-levels", type=int, choices=[127, 255], default=127)
            sc.add_argument("--pv-probability-sum-correction", action="store_true")
            sc.add_argument("--pv-value-bits", type=int, choices=[8, 9], default=8)

    cond = sub.add_parser("generate-mdlm-conditioned",
                          help="compare conditioned DDPM generation with retained prefix K/V")
    cond.add_argument("--out", type=Path)
    cond.add_argument("--model-id", default=DEFAULT_MODEL_ID)
    cond.add_argument("--revision", default=DEFAULT_REVISION)
    cond.add_argument("--device", default="cuda")
    cond.add_argument("--prefix-tokens", type=int, default=64)
    cond.add_argument("--suffix-tokens", type=int, default=32)
    cond.add_argument("--samples", type=int, default=3)
    cond.add_argument("--steps", type=int, default=64)
    cond.add_argument("--seed", type=int, default=0)
    cond.add_argument("--local-files-only", action="store_true")
    cond.add_argument("--weights-seed", type=int, default=0)
    return parser


def _emit(result: Any, out: Optional[Path]) -> None:
    rendered = json.dumps(result, indent=2, sort_keys=True)
    if out is not None:
        out.parent.mkdir(parents=True, exist_ok=True)
        out.write_text(rendered + "\n", encoding="utf-8")
    print(rendered)


def _checkpoint_note(args: argparse.Namespace) -> dict:
    return {"model_id": args.model_id, "revision": args.revision,
            "weights": f"random-init N(0, 0.02) stand-in, seed {args.weights_seed} (no checkpoint on this host)"}


def run_trace_mdlm(args: argparse.Namespace) -> dict:
    import torch

    from .api import load_mdlm, run_ddpm_cache_sampler, run_ddpm_candidate_cache_sampler
    from .model import MDLMConfig

    if args.canvas_tokens <= 0 or args.steps <= 0 or args.warmup < 0 or args.batch <= 0:
        raise ValueError("canvas_tokens/steps/batch must be positive and warmup non-negative")
    cfg = MDLMConfig()
    if args.canvas_tokens > cfg.max_positions:
        raise ValueError(f"canvas_tokens exceeds the model context length {cfg.max_positions}")
    engine = load_mdlm(args.batch, args.canvas_tokens, seed=args.weights_seed, device=args.device)
    mask = cfg.mask_token_id
    ids = torch.full((args.batch, args.canvas_tokens), mask, dtype=torch.long)
    sampler = run_ddpm_cache_sampler if args.sampler == "ddpm-cache" else run_ddpm_candidate_cache_sampler
    for _ in range(args.warmup):
        sampler(engine, ids, mask_token_id=mask, steps=args.steps, seed=args.seed)
    out_ids, measurements, meta = sampler(engine, ids, mask_token_id=mask, steps=args.steps, seed=args.seed)
    decoded = out_ids.tolist()
    trace = {
        "metadata": {
            **meta, **_checkpoint_note(args),
            "sampler": {"ddpm-cache": "official-ddpm-cache",
                        "ddpm-candidate-cache": "distribution-equivalent-candidate-cache"}[args.sampler],
            "device": torch.cuda.get_device_name(engine.device),
            "parameter_count": cfg.parameter_count(),
            "canvas_tokens": args.canvas_tokens,
            "batch": args.batch,
            "generated_token_ids": decoded[0] if args.batch == 1 else decoded,
            "all_tokens_committed": not any(mask in row for row in decoded),
            "generated_text": None,
            "generation_device_ms": engine.generation_ms(),
        },
        "steps": [vars(m) for m in measurements],
    }
    args.out.parent.mkdir(parents=True, exist_ok=True)
    args.out.write_text(json.dumps(trace, indent=2) + "\n", encoding="utf-8")
    return {
        "trace": str(args.out),
        "steps": len(measurements),
        "sampling_transitions": meta.get("sampling_transitions", len(measurements)),
        "model_evaluations": meta.get("model_evaluations", len(measurements)),
        "probability_cache_hits": meta.get("probability_cache_hits", 0),
        "device": trace["metadata"]["device"],
        "parameter_count": cfg.parameter_count(),
        "all_tokens_committed": trace["metadata"]["all_tokens_committed"],
        "generated_text": None,
        "measured_latency_ms": sum(m.elapsed_s for m in measurements) * 1e3,
    }


def main(argv: Optional[List[str]] = None) -> int:
    args = build_parser().parse_args(argv)
    if args.command == "trace-mdlm":
        _emit(run_trace_mdlm(args), None)
        return 0
    if args.command == "validate-candidate-cache":
        from .validation import validate_candidate_cache_equivalence

        result = validate_candidate_cache_equivalence(
            positions=args.positions, vocabulary_size=args.vocabulary_size,
            probability_bits=args.probability_bits, analytic_vocabulary_size=args.analytic_vocabulary_size,
            transitions=args.transitions, monte_carlo_trials=args.monte_carlo_trials,
            monte_carlo_vocabulary_size=args.monte_carlo_vocabulary_size, seed=args.seed,
            maximum_total_variation=args.maximum_total_variation, device=args.device)
        _emit(result, args.out)
        return 0 if result["passed"] else 1
    if args.command == "validate-rng-gumbel":
        from .validation import validate_rng_and_gumbel

        result = validate_rng_and_gumbel(
            distribution_trials=args.distribution_trials,
            distribution_vocabulary_size=args.distribution_vocabulary_size,
            full_vocabulary_size=args.full_vocabulary_size, full_vocabulary_batches=args.full_vocabulary_batches,
            full_vocabulary_batch_size=args.full_vocabulary_batch_size, mantissa_bits=args.mantissa_bits,
            fraction_bits=args.fraction_bits, seed=args.seed, maximum_distribution_tv=args.maximum_distribution_tv,
            minimum_full_vocabulary_agreement=args.minimum_full_vocabulary_agreement, device=args.device)
        _emit(result, args.out)
        return 0 if result["passed"] else 1
    if args.command == "analyze-mdlm-prefix-drift":
        if args.prefix_text is not None:
            raise SystemExit("--prefix-text needs the GPT-2 tokenizer, which this host does not have; "
                             "use --prefix-tokens N for a seeded synthetic prefix")
        from .prefix import analyze_mdlm_prefix_drift

        result = analyze_mdlm_prefix_drift(
            prefix_tokens=args.prefix_tokens, suffix_tokens=args.suffix_tokens,
            changed_suffix_tokens=args.changed_suffix_tokens, warmup=args.warmup,
            timing_repeats=args.timing_repeats, seed=args.seed, weights_seed=args.weights_seed,
            device=args.device)
        result.update(_checkpoint_note(args))
        _emit(result, args.out)
        return 0
    if args.command in ("benchmark-mdlm-event", "benchmark-mdlm-apple"):
        from .event import benchmark_event_sampler

        result = benchmark_event_sampler(canvas_tokens=args.canvas_tokens, steps=args.steps,
                                         seeds=tuple(args.seeds), weights_seed=args.weights_seed,
                                         device=args.device)
        result.update(_checkpoint_note(args))
        _emit(result, args.out)
        return 0
    if args.command == "run-mdlm-two-turn":
        from .session import evaluate_two_turn_mdlm_session

        result = evaluate_two_turn_mdlm_session(
            prefix_tokens=args.prefix_tokens, first_answer_tokens=args.first_answer_tokens,
            followup_tokens=args.followup_tokens, second_answer_tokens=args.second_answer_tokens,
            samples=args.samples, steps=args.steps, seed=args.seed, weights_seed=args.weights_seed,
            device=args.device)
        result.update(_checkpoint_note(args))
        result["dataset"] = {"id": args.dataset_id, "config": args.dataset_config, "revision": args.dataset_revision,
                             "split": args.split, "used": False,
                             "note": "the dataset is not on this host: windows are seeded synthetic ids"}
        _emit(result, args.out)
        return 0
    if args.command == "export-mdlm-hardware-package":
        import numpy as np

        from .checkpoint import checkpoint_module, deterministic_hardware_input, export_hardware_package
        from .model import MDLMConfig, build_standin, ddit_forward, fold

        cfg = MDLMConfig()
        module = checkpoint_module(args.checkpoint, cfg) if args.checkpoint else build_standin(cfg, args.weights_seed)
        folded = fold(module)
        folded.config = cfg
        ids = np.asarray([deterministic_hardware_input(64, cfg.vocab_size, cfg.mask_token_id)])
        source = {"model_id": args.model_id, "revision": args.revision}
        if args.checkpoint:
            source["path"] = str(args.checkpoint)
        else:
            source["weights"] = _checkpoint_note(args)["weights"]
        manifest = export_hardware_package(folded, args.out_dir, source=source,
                                           unfolded_logits=ddit_forward(module, ids))
        _emit({"package_dir": str(args.out_dir), "constant_fold_validation": manifest["constant_fold_validation"],
               "golden_tensor_count": manifest["goldens"]["tensor_count"],
               "weight_tensor_count": manifest["weights"]["tensor_count"], "files": manifest["files"]}, None)
        return 0
    if args.command == "validate-mdlm-hardware-package":
        from .checkpoint import validate_hardware_package

        report = validate_hardware_package(args.package_dir)
        _emit(report, None)
        return 0 if report["passed"] else 1
    if args.command == "validate-hardware-fixed-mlp":
        from .fixed_mlp import validate_hardware_fixed_mlp

        _emit(validate_hardware_fixed_mlp(args.package_dir, block=args.block,
                                          activation_granularity=args.activation_granularity,
                                          down_activation_granularity=args.down_activation_granularity,
                                          smoothquant_alpha=args.smoothquant_alpha), args.out)
        return 0
    if args.command == "sweep-hardware-fixed-mlp":
        from .fixed_mlp import sweep_hardware_fixed_mlp

        _emit(sweep_hardware_fixed_mlp(args.package_dir, activation_granularity=args.activation_granularity,
                                       down_activation_granularity=args.down_activation_granularity), args.out)
        return 0
    if args.command in ("sweep-fixed-layernorm", "sweep-fixed-rotary", "sweep-fixed-attention"):
        from . import fixed_point

        fn = {"sweep-fixed-layernorm": fixed_point.sweep_fixed_layer_norm,
              "sweep-fixed-rotary": fixed_point.sweep_fixed_rotary,
              "sweep-fixed-attention": fixed_point.sweep_fixed_attention}[args.command]
        _emit(fn(args.package_dir), args.out)
        return 0
    if args.command == "sweep-qkv-weight-precision":
        from .fixed_point import sweep_qkv_weight_precision

        _emit(sweep_qkv_weight_precision(args.package_dir, weight_bits=tuple(args.weight_bits),
                                         smoothquant_alphas=tuple(args.smoothquant_alphas) or (None,)), args.out)
        return 0
    if args.command == "screen-packed-int8-attention":
        from .attention_int8 import screen_packed_int8_attention

        _emit(screen_packed_int8_attention(args.package_dir), args.out)
        return 0
    if args.command in ("screen-packed-int8-attention-heldout", "screen-packed-int8-attention-logits"):
        from . import attention_int8
        from .checkpoint import checkpoint_module
        from .model import MDLMConfig, build_standin

        cfg = MDLMConfig()
        module = checkpoint_module(args.checkpoint, cfg) if args.checkpoint else build_standin(cfg, args.weights_seed)
        if args.command.endswith("-heldout"):
            report = attention_int8.screen_packed_int8_attention_heldout(args.package_dir, seeds=args.seeds,
                                                                        device=args.device, model=module)
        else:
            report = attention_int8.screen_packed_int8_attention_logits(
                args.package_dir, seeds=args.seeds, device=args.device, quantize_qk=not args.preserve_qk18,
                quantize_pv=not args.preserve_pv18, qk_bits=args.qk_bits, qk_scale_mode=args.qk_scale_mode,
                qk_multiplier_fraction_bits=args.qk_multiplier_fraction_bits,
                pv_probability_levels=args.pv_probability_levels,
                pv_probability_sum_correction=args.pv_probability_sum_correction, pv_value_bits=args.pv_value_bits,
                model=module)
        if not args.checkpoint:
            report.update(_checkpoint_note(args))
        _emit(report, args.out)
        return 0
    if args.command == "generate-mdlm-conditioned":
        from .conditioned import evaluate_conditioned_mdlm_ddpm

        result = evaluate_conditioned_mdlm_ddpm(
            prefix_tokens=args.prefix_tokens, suffix_tokens=args.suffix_tokens, samples=args.samples,
            steps=args.steps, seed=args.seed, weights_seed=args.weights_seed, device=args.device)
        result.update(_checkpoint_note(args))
        _emit(result, args.out)
        return 0
    raise AssertionError(args.command)  # argparse restricts the choices


if __name__ == "__main__":
    raise SystemExit(main())
