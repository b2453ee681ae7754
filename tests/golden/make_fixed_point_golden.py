#!/usr/bin/env python3
"""Golden outputs of the reference's RTL fixed-point block stages
(src/diffusion_accel/fixed_norm.py and fixed_attention.py, imported in
place) on seeded inputs (fixed_point_cases below):

  * fixed_layer_norm_q12 on four activation regimes (unit, wide, saturating,
    near-constant rows);
  * fixed_rotary_q12 and fixed_attention_q12 (default and a coarse 4-bit /
    cutoff-8 exponential table) on seeded qkv with package-style fp16
    rotary tables;
  * fixed_attention_projection_q10 and fixed_qkv_projection_q12 (16-bit,
    8-bit and SmoothQuant alpha 0.5 weights);
  * sweep_fixed_layer_norm / sweep_fixed_rotary / sweep_fixed_attention on a
    synthetic 12-block package of integer-grid values (sweep_package below;
    its file digests are recorded so the tests can check that they rebuild
    the same package).
Integer outputs are stored as SHA-256 digests of their int64 arrays, metrics
as JSON.  Writes tests/golden/fixed_point_golden.json.

    python tests/golden/make_fixed_point_golden.py --reference <reference root>
"""

from __future__ import annotations

import argparse
import os
import hashlib
import json
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent


def digest(t) -> str:
    a = np.ascontiguousarray(t.detach().cpu().numpy().astype("<i8"))
    return hashlib.sha256(a.tobytes()).hexdigest()


def fixed_point_cases(torch):
    """Seeded inputs (generator seed 11)."""
    from diffusionhard_b200.model import rope_tables

    g = torch.Generator().manual_seed(11)
    base = torch.randn((64, 768), generator=g)
    ln = {
        "unit": base.clone(),
        "wide": base * 40.0,
        "saturating": base * 3000.0,
        "flat": 0.5 + base * 1e-4,
    }
    qkv = torch.randn((64, 2304), generator=g)
    cos, sin = rope_tables(64, 64)
    cos = torch.from_numpy(cos).half().float()
    sin = torch.from_numpy(sin).half().float()
    w_out = torch.randn((768, 768), generator=g) * 0.02
    w_qkv = torch.randn((2304, 768), generator=g) * 0.02
    b_qkv = torch.randn(2304, generator=g) * 0.02
    return ln, {"unit": qkv, "hot": qkv * 3.0, "saturating": qkv * 40.0}, cos, sin, w_out, w_qkv, b_qkv


def sweep_package(out_dir: Path):
    """A synthetic 12-block package with the tensor names and shapes the
    sweeps read.  Every value is an integer-grid number drawn with numpy's
    integer generator (seed 8), so the files are identical on every machine.
    Returns {file name: SHA-256}."""
    import torch
    from safetensors.torch import save_file

    rng = np.random.default_rng(8)

    def grid(shape, span, frac):
        return torch.from_numpy(rng.integers(-span, span + 1, size=shape).astype(np.float32) / float(1 << frac))

    goldens = {"folded.embedding": grid((1, 64, 768), 2048, 10),
               "folded.final.norm_unaffine": grid((1, 64, 768), 4096, 12)}
    weights = {"rotary.cos": grid((64, 32), 1024, 10).half(), "rotary.sin": grid((64, 32), 1024, 10).half()}
    for b in range(12):
        p = "folded.block_%02d" % b
        goldens[p + ".qkv"] = grid((1, 64, 2304), 4096, 12)
        for name in ("attention", "norm1_unaffine", "norm2_unaffine"):
            goldens[p + "." + name] = grid((1, 64, 768), 4096, 12)
        for name in ("attention_projection", "after_attention", "output"):
            goldens[p + "." + name] = grid((1, 64, 768), 4096, 10)
        weights["block_%02d.qkv.weight" % b] = grid((2304, 768), 200, 12).half()
        weights["block_%02d.qkv.bias" % b] = grid((2304,), 200, 12).half()
        weights["block_%02d.attention_out.weight" % b] = grid((768, 768), 200, 12).half()
    out_dir.mkdir(parents=True, exist_ok=True)
    save_file(goldens, out_dir / "golden_tensors.safetensors")
    save_file(weights, out_dir / "folded_fp16_weights.safetensors")
    (out_dir / "manifest.json").write_text(json.dumps({"fixed_graph": {"blocks": 12}}) + "\n")
    return {n: hashlib.sha256((out_dir / n).read_bytes()).hexdigest()
            for n in ("golden_tensors.safetensors", "folded_fp16_weights.safetensors")}


def strip(report):
    report = dict(report)
    report.pop("package_dir", None)
    return report


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--reference", default=os.environ.get("DH_REFERENCE_ROOT"),
                    required="DH_REFERENCE_ROOT" not in os.environ,
                    help="reference tree (default: $DH_REFERENCE_ROOT)")
    args = ap.parse_args()
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(Path(args.reference) / "src"))
    import torch

    from diffusion_accel import fixed_attention as fa  # reference, in place
    from diffusion_accel import fixed_norm as fn

    ln, qkvs, cos, sin, w_out, w_qkv, b_qkv = fixed_point_cases(torch)
    out = {"layer_norm": {}, "rotary": {}, "attention": {}, "projection": {}, "qkv_projection": {}}
    for name, act in ln.items():
        _, q, m = fn.fixed_layer_norm_q12(act)
        out["layer_norm"][name] = {"output_q": digest(q), "metrics": m}
    for name, qkv in qkvs.items():
        _, _, q12, k12, d = fa.fixed_rotary_q12(qkv, cos, sin)
        out["rotary"][name] = {"query_q12": digest(q12), "key_q12": digest(k12),
                               "qkv_q12": digest(d["tensors"]["qkv_q12"]), "metrics": d["metrics"]}
    for name, qkv in qkvs.items():
        for step, cutoff in ((6, 16.0), (4, 8.0)):
            _, aq, d = fa.fixed_attention_q12(qkv, cos, sin, exponential_step_bits=step, exponential_cutoff=cutoff)
            key = "%s_s%d_c%g" % (name, step, cutoff)
            out["attention"][key] = {"attention_q12": digest(aq),
                                     "scores_q10": digest(d["tensors"]["scores_q10"]),
                                     "probabilities_q16": digest(d["tensors"]["probabilities_q16"]),
                                     "metrics": d["metrics"]}
            if step == 6:
                _, pq, pd = fa.fixed_attention_projection_q10(aq, w_out)
                out["projection"][name] = {"projection_q10": digest(pq),
                                           "accumulators": digest(pd["tensors"]["accumulators"]),
                                           "metrics": pd["metrics"]}
    _, norm_q, _ = fn.fixed_layer_norm_q12(ln["unit"])
    for key, kwargs in (("int16", {}), ("int8", {"weight_bits": 8}), ("alpha0.5", {"smoothquant_alpha": 0.5})):
        _, oq, d = fa.fixed_qkv_projection_q12(norm_q, w_qkv, b_qkv, **kwargs)
        out["qkv_projection"][key] = {"output_q12": digest(oq), "accumulators": digest(d["tensors"]["accumulators"]),
                                      "metrics": d["metrics"]}
    with tempfile.TemporaryDirectory() as tmp:
        pkg = Path(tmp) / "pkg"
        out["sweep_package_files"] = sweep_package(pkg)
        out["sweep_layer_norm"] = strip(fn.sweep_fixed_layer_norm(pkg))
        out["sweep_rotary"] = strip(fa.sweep_fixed_rotary(pkg))
        out["sweep_attention"] = strip(fa.sweep_fixed_attention(pkg))
    (HERE / "fixed_point_golden.json").write_text(json.dumps(out, sort_keys=True) + "\n")
    print({k: (len(v) if isinstance(v, dict) else v) for k, v in out.items()})


if __name__ == "__main__":
    main()
