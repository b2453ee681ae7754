"""RTL fixed-point block stages on the GPU against the reference's own
outputs (tests/golden/make_fixed_point_golden.py): integer outputs by SHA-256
digest (bit-exact), integer metrics exactly, float metrics to 1e-4 relative,
and the three package sweeps."""

import json
import sys

import pytest

from conftest import GOLDEN

sys.path.insert(0, str(GOLDEN))
from make_fixed_point_golden import digest, fixed_point_cases, strip, sweep_package  # noqa: E402

pytestmark = pytest.mark.gpu

GJ = json.loads((GOLDEN / "fixed_point_golden.json").read_text())


def _same(got, ref, path=""):
    if isinstance(ref, dict):
        assert set(got) == set(ref), (path, set(got) ^ set(ref))
        for k in ref:
            _same(got[k], ref[k], path + "." + k)
    elif isinstance(ref, list):
        assert len(got) == len(ref), path
        for i, (g, r) in enumerate(zip(got, ref)):
            _same(g, r, "%s[%d]" % (path, i))
    elif isinstance(ref, float):
        # float metrics compare against host float references (matmuls,
        # softmax) whose CPU summation order may differ between machines
        assert got == pytest.approx(ref, rel=1e-4, abs=1e-7), path
    else:
        assert got == ref, path


@pytest.fixture(scope="module")
def cases(cuda):
    return fixed_point_cases(cuda)


def test_layer_norm_bit_exact(cases):
    from diffusionhard_b200.fixed_point import fixed_layer_norm_q12

    for name, act in cases[0].items():
        _, q, m = fixed_layer_norm_q12(act)
        assert digest(q) == GJ["layer_norm"][name]["output_q"], name
        _same(m, GJ["layer_norm"][name]["metrics"], name)


def test_rotary_bit_exact(cases):
    from diffusionhard_b200.fixed_point import fixed_rotary_q12

    _, qkvs, cos, sin = cases[:4]
    for name, qkv in qkvs.items():
        _, _, q12, k12, d = fixed_rotary_q12(qkv, cos, sin)
        ref = GJ["rotary"][name]
        assert digest(q12) == ref["query_q12"] and digest(k12) == ref["key_q12"], name
        assert digest(d["tensors"]["qkv_q12"]) == ref["qkv_q12"], name
        _same(d["metrics"], ref["metrics"], name)


def test_attention_and_projection_bit_exact(cases):
    from diffusionhard_b200.fixed_point import fixed_attention_projection_q10, fixed_attention_q12

    _, qkvs, cos, sin, w_out = cases[:5]
    for name, qkv in qkvs.items():
        for step, cutoff in ((6, 16.0), (4, 8.0)):
            _, aq, d = fixed_attention_q12(qkv, cos, sin, exponential_step_bits=step, exponential_cutoff=cutoff)
            ref = GJ["attention"]["%s_s%d_c%g" % (name, step, cutoff)]
            assert digest(aq) == ref["attention_q12"], (name, step)
            assert digest(d["tensors"]["scores_q10"]) == ref["scores_q10"], (name, step)
            assert digest(d["tensors"]["probabilities_q16"]) == ref["probabilities_q16"], (name, step)
            _same(d["metrics"], ref["metrics"], name)
            if step == 6:
                _, pq, pd = fixed_attention_projection_q10(aq, w_out)
                pref = GJ["projection"][name]
                assert digest(pq) == pref["projection_q10"], name
                assert digest(pd["tensors"]["accumulators"]) == pref["accumulators"], name
                _same(pd["metrics"], pref["metrics"], name)


def test_qkv_projection_bit_exact(cases):
    from diffusionhard_b200.fixed_point import fixed_layer_norm_q12, fixed_qkv_projection_q12

    ln, _, _, _, _, w_qkv, b_qkv = cases
    _, norm_q, _ = fixed_layer_norm_q12(ln["unit"])
    for key, kwargs in (("int16", {}), ("int8", {"weight_bits": 8}), ("alpha0.5", {"smoothquant_alpha": 0.5})):
        _, oq, d = fixed_qkv_projection_q12(norm_q, w_qkv, b_qkv, **kwargs)
        ref = GJ["qkv_projection"][key]
        assert digest(oq) == ref["output_q12"], key
        assert digest(d["tensors"]["accumulators"]) == ref["accumulators"], key
        _same(d["metrics"], ref["metrics"], key)


def test_argument_errors(cuda):
    torch = cuda
    from diffusionhard_b200.fixed_point import fixed_attention_q12, fixed_layer_norm_q12, fixed_qkv_projection_q12

    with pytest.raises(ValueError, match="token by 768"):
        fixed_layer_norm_q12(torch.zeros(4, 64))
    with pytest.raises(ValueError, match="step_bits"):
        fixed_attention_q12(torch.zeros(4, 2304), torch.zeros(4, 32), torch.zeros(4, 32), exponential_step_bits=0)
    with pytest.raises(ValueError, match="rotary tables"):
        fixed_attention_q12(torch.zeros(4, 2304), torch.zeros(5, 32), torch.zeros(5, 32))
    with pytest.raises(ValueError, match="mutually exclusive"):
        fixed_qkv_projection_q12(torch.zeros(4, 768, dtype=torch.int64), torch.zeros(2304, 768), torch.zeros(2304),
                                 smoothquant_alpha=0.5, smoothquant_scales=torch.ones(768))


def test_package_sweeps_match_reference(cuda, tmp_path):
    from diffusionhard_b200.fixed_point import sweep_fixed_attention, sweep_fixed_layer_norm, sweep_fixed_rotary

    assert sweep_package(tmp_path / "pkg") == GJ["sweep_package_files"], "the rebuilt package differs"
    _same(strip(sweep_fixed_layer_norm(tmp_path / "pkg")), GJ["sweep_layer_norm"], "layer_norm")
    _same(strip(sweep_fixed_rotary(tmp_path / "pkg")), GJ["sweep_rotary"], "rotary")
    _same(strip(sweep_fixed_attention(tmp_path / "pkg")), GJ["sweep_attention"], "attention")
