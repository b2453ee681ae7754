"""Pin the model-side oracle and host logic to the reference's own Python
(fixtures from tests/golden/make_model_golden.py)."""

import json

import numpy as np
import pytest

from conftest import GOLDEN
from diffusionhard_b200.model import (MDLMConfig, build_standin, fold, fp32_forward, rope_tables,
                                      smoothquant_linear)
from diffusionhard_b200.prefix import tensor_drift_metrics
from diffusionhard_b200.sampler import hardware_candidate_cache_bytes, reveal_thresholds_q32
from oracle import model_oracle

G = np.load(GOLDEN / "model_golden.npz")
GJ = json.loads((GOLDEN / "model_golden.json").read_text())


def test_parameter_count_matches_reference_spec():
    # configs/models/mdlm_owt_169m.yaml:4
    assert MDLMConfig().parameter_count() == 169_627_218
    m = build_standin(MDLMConfig(**GJ["config"]), seed=0)
    assert sum(p.numel() for p in m.parameters()) == MDLMConfig(**GJ["config"]).parameter_count()


def test_folded_fp32_forward_matches_reference_folded_forward():
    import torch

    cfg = MDLMConfig(**GJ["config"])
    folded = fold(build_standin(cfg, seed=0))
    h = fp32_forward(folded, G["ids"])
    logits = torch.nn.functional.linear(torch.from_numpy(h), torch.from_numpy(folded.head.weight),
                                        torch.from_numpy(folded.head.bias)).numpy()
    assert np.abs(logits - G["logits"]).max() < 1e-4


def test_static_smoothquant_w8a8_equals_reference_quantized_linear():
    """With the smoothing amax taken from the same activations, the static
    W8A8 path reproduces fixed_mlp.quantized_linear bit for bit."""
    import torch

    act = torch.from_numpy(G["act"])
    ql = smoothquant_linear(G["weight"], G["bias"], act.abs().amax(dim=0).numpy(), 0.5)
    out, q, scale, acc = model_oracle.w8a8_linear(act, ql, return_parts=True)
    assert np.array_equal(out.numpy(), G["ql_out"])
    m = GJ["quantized_linear_metrics"]
    assert int(acc.min()) == m["accumulator_min"] and int(acc.max()) == m["accumulator_max"]
    assert float(ql.w_scale.min()) == pytest.approx(m["weight_scale_min"], rel=1e-7)


def test_rotary_matches_reference():
    import torch

    cos, sin = rope_tables(1024)
    pos = G["positions"]
    got = model_oracle._rot(torch.from_numpy(G["vec"]), torch.from_numpy(cos[pos])[None, :, None, :],
                            torch.from_numpy(sin[pos])[None, :, None, :])
    assert np.abs(got.numpy() - G["rotated"]).max() < 1e-6


def test_drift_metrics_match_reference():
    import torch

    got = tensor_drift_metrics(torch.from_numpy(G["drift_a"]), torch.from_numpy(G["drift_b"]))
    for k, v in GJ["drift_metrics"].items():
        if isinstance(v, bool):
            assert got[k] == v
        else:
            assert got[k] == pytest.approx(v, rel=1e-6, abs=1e-9), k


def test_reveal_schedule_matches_reference_probability():
    import torch

    # mdlm.py:1116-1117, 1151-1153 in float32
    steps = 64
    t = torch.linspace(1.0, 1e-5, steps + 1)
    thr = reveal_thresholds_q32(steps)
    for k in range(steps):
        mt = (1 - 1e-3) * t[k]
        ms = (1 - 1e-3) * t[k + 1]
        p = float(((mt - ms) / mt).item())
        assert thr[k] == min(1 << 32, int(np.floor(p * 2.0 ** 32)))
    assert thr[0] == pytest.approx(2 ** 32 / 64, rel=1e-3)


def test_candidate_cache_bytes_match_reference_metadata():
    # tests/test_mdlm.py:170 (4 positions, mask 3) and test_conditioned.py:69 (8 positions)
    assert hardware_candidate_cache_bytes(4, 3) == (6, 1)
    assert hardware_candidate_cache_bytes(8, 3) == (10, 1)
    assert hardware_candidate_cache_bytes(64, 50257) == (144, 2)  # README.md:17-19
