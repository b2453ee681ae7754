"""Packed INT8 attention on the GPU (dh_packed_int8_attention_q12 and the
drop-ins of diffusionhard_b200.attention_int8) against the reference's own
outputs (tests/golden/make_attention_int8_golden.py): integer outputs by
SHA-256 digest (bit-exact), integer metrics exactly, float metrics to 1e-4
relative; then against the numpy oracle at other canvas lengths, and the
C-ABI argument checks."""

import json
import sys

import numpy as np
import pytest

from conftest import GOLDEN, ROOT

sys.path.insert(0, str(GOLDEN))
sys.path.insert(0, str(ROOT))
from make_attention_int8_golden import (EVALUATE_OPTIONS, HELDOUT_SEEDS, LOGIT_OPTIONS,  # noqa: E402
                                        STANDIN_SEED)
from make_fixed_point_golden import digest, fixed_point_cases, strip, sweep_package  # noqa: E402
from oracle import attention_int8_oracle as oracle  # noqa: E402

pytestmark = pytest.mark.gpu

GJ = json.loads((GOLDEN / "attention_int8_golden.json").read_text())


def _same(got, ref, path="", rel=1e-4):
    if isinstance(ref, dict):
        assert set(got) == set(ref), (path, set(got) ^ set(ref))
        for k in ref:
            _same(got[k], ref[k], path + "." + k, rel)
    elif isinstance(ref, list):
        assert len(got) == len(ref), path
        for i, (g, r) in enumerate(zip(got, ref)):
            _same(g, r, "%s[%d]" % (path, i), rel)
    elif isinstance(ref, float):
        # float metrics compare against host float references whose CPU
        # summation order may differ between machines
        assert got == pytest.approx(ref, rel=rel, abs=1e-7), path
    else:
        assert got == ref, path


@pytest.fixture(scope="module")
def cases(cuda):
    _, qkvs, cos, sin, _, _, _ = fixed_point_cases(cuda)
    return qkvs, cos, sin


@pytest.mark.parametrize("name", ["unit", "hot", "saturating"])
def test_dynamic_bit_exact(cases, name):
    from diffusionhard_b200.attention_int8 import dynamic_qk_fixed_pv_attention_q12

    qkvs, cos, sin = cases
    att, d = dynamic_qk_fixed_pv_attention_q12(qkvs[name], cos, sin)
    g = GJ["dynamic"][name]
    assert digest(att) == g["attention"]
    for key in ("attention_q12", "scores_q10", "probabilities_q16", "query_maxima_q12", "key_maxima_q12"):
        assert digest(d["tensors"][key]) == g[key], key


@pytest.mark.parametrize("opt", sorted(EVALUATE_OPTIONS))
@pytest.mark.parametrize("name", ["unit", "hot"])
def test_evaluate_bit_exact(cuda, cases, name, opt):
    from diffusionhard_b200.attention_int8 import _evaluate_with_fixed_maxima, _exponential_table

    qkvs, cos, sin = cases
    cand, base, heads = _evaluate_with_fixed_maxima(qkvs[name], cos, sin, GJ["calibration"], _exponential_table(),
                                                    **EVALUATE_OPTIONS[opt])
    g = GJ["evaluate"]["%s_%s" % (name, opt)]
    assert digest(cand) == g["candidate"]
    assert digest(base) == g["baseline"]
    _same(heads, g["heads"], "heads")


def test_package_screens_match_reference(cuda, tmp_path):
    from diffusionhard_b200.attention_int8 import screen_packed_int8_attention
    from diffusionhard_b200.fixed_point import sweep_qkv_weight_precision

    assert sweep_package(tmp_path / "pkg") == GJ["sweep_package_files"], "the rebuilt package differs"
    _same(strip(screen_packed_int8_attention(tmp_path / "pkg")), GJ["screen"], "screen")
    _same(strip(sweep_qkv_weight_precision(tmp_path / "pkg", smoothquant_alphas=(None, 0.5))),
          GJ["qkv_weight_precision"], "qkv_weight_precision")


def test_heldout_and_logit_screens_match_reference(cuda, tmp_path):
    """The reference ran these on the same full-size stand-in in place of the
    checkpoint; its float forward and the host one here agree, so the
    integer attention sees the same qkv.  The logit metrics (total variation,
    KL divergence) are small differences of sums over 50,257 host-float
    probabilities, whose vectorised reductions vary between CPUs by ~0.5%
    of the metric, so they compare to 2% (top-1 matches exactly)."""
    from diffusionhard_b200.attention_int8 import (screen_packed_int8_attention_heldout,
                                                   screen_packed_int8_attention_logits)
    from diffusionhard_b200.model import MDLMConfig, build_standin, fold

    sweep_package(tmp_path / "pkg")
    folded = fold(build_standin(MDLMConfig(), seed=STANDIN_SEED))

    def nodev(r):
        r = dict(r)
        r.pop("device")
        return r

    _same(nodev(screen_packed_int8_attention_heldout(tmp_path / "pkg", seeds=HELDOUT_SEEDS, model=folded)),
          nodev(GJ["heldout"]), "heldout")
    for k, kw in LOGIT_OPTIONS.items():
        got = screen_packed_int8_attention_logits(tmp_path / "pkg", seeds=HELDOUT_SEEDS, model=folded, **kw)
        _same(nodev(got), nodev(GJ["logits"][k]), "logits." + k, rel=2e-2)


@pytest.mark.parametrize("tokens", [1, 37, 256, 700])
@pytest.mark.parametrize("opt", ["default", "dynamic_q17", "sum_correction", "fixed18_pv"])
def test_matches_oracle_at_other_lengths(cuda, tokens, opt):
    """Canvases of other lengths (a single token, ragged, long) against the
    numpy oracle: candidate, baseline and per-head argmax agreement."""
    torch = cuda
    from diffusionhard_b200.attention_int8 import _evaluate_with_fixed_maxima, _exponential_table
    from diffusionhard_b200.model import rope_tables

    g = torch.Generator().manual_seed(tokens)
    qkv = torch.randn((tokens, 2304), generator=g) * 2.0
    cos, sin = (torch.from_numpy(t).half().float() for t in rope_tables(tokens, 64))
    cal = oracle.head_maxima((qkv * 0.7).numpy(), cos.numpy(), sin.numpy())  # some inputs saturate
    cand, base, heads = _evaluate_with_fixed_maxima(qkv, cos, sin, cal, _exponential_table(), **EVALUATE_OPTIONS[opt])
    r = oracle.packed_attention(qkv.numpy(), cos.numpy(), sin.numpy(), calibration=cal,
                                **oracle.evaluate_options(EVALUATE_OPTIONS[opt]))
    np.testing.assert_array_equal(cand.numpy(), r["attention"])
    np.testing.assert_array_equal(base.numpy(), r["baseline"])
    agree = (r["scores_q10"].argmax(-1) == r["baseline_scores"].argmax(-1)).mean(-1)
    assert [h["score_argmax_agreement_vs_fixed18"] for h in heads] == pytest.approx(agree.tolist(), abs=1e-6)


def test_c_abi_argument_checks(cuda):
    torch = cuda
    from diffusionhard_b200 import _lib

    buf = torch.zeros(4096, dtype=torch.int64, device="cuda")
    p = buf.data_ptr()

    def call(**kw):
        a = dict(q=p, k=p, qkv=p, tokens=4, heads=12, mode=1, scores=1, levels=127, frac=24, plevels=127, corr=0,
                 vlevels=127, params=p, step=6, cutoff=16384, lut=p, lut_n=1025, work=p, out=p, sc=None, pr=None,
                 pq=None, qm=p, km=p, st=None)
        a.update(kw)
        return _lib.raw("dh_packed_int8_attention_q12", a["q"], a["k"], a["qkv"], a["tokens"], a["heads"],
                        a["mode"], a["scores"], a["levels"], a["frac"], a["plevels"], a["corr"], a["vlevels"],
                        a["params"], a["step"], a["cutoff"], a["lut"], a["lut_n"], a["work"], a["out"], a["sc"],
                        a["pr"], a["pq"], a["qm"], a["km"], a["st"], None)

    assert call(q=None) == 100
    assert call(mode=3) == 105
    assert call(mode=0) == 105  # requantised scores need requantised vectors
    assert call(vlevels=0) == 105  # requantised probabilities need requantised values
    assert call(frac=31) == 105
    assert call(work=None) == 100
    assert call(mode=2, qm=None) == 100
    assert call(tokens=2049) == 103
    assert call(tokens=0) == 0


@pytest.mark.parametrize("tokens", [64, 2048])
def test_unquantized_candidate_equals_fixed18_baseline(cuda, tokens):
    """With neither phase requantised the K15 candidate is the fixed18
    attention itself, so it must equal K13's output bit for bit -- checked up
    to the 2,048-token limit, where the oracle would be slow."""
    torch = cuda
    from diffusionhard_b200.attention_int8 import _evaluate_with_fixed_maxima, _exponential_table
    from diffusionhard_b200.model import rope_tables

    g = torch.Generator().manual_seed(tokens + 1)
    qkv = torch.randn((tokens, 2304), generator=g) * 2.0
    cos, sin = (torch.from_numpy(t).half().float() for t in rope_tables(tokens, 64))
    cal = [{"query_q12": 4096, "key_q12": 4096, "value_q12": 4096}] * 12
    cand, base, heads = _evaluate_with_fixed_maxima(qkv, cos, sin, cal, _exponential_table(), quantize_qk=False,
                                                    quantize_pv=False)
    assert torch.equal(cand, base)
    assert all(h["score_argmax_agreement_vs_fixed18"] == 1.0 for h in heads)
