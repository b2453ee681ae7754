"""Engines built from a checkpoint and from a hardware package on the GPU."""

import numpy as np
import pytest

from diffusionhard_b200.model import MDLMConfig, build_standin, fold

pytestmark = pytest.mark.gpu

SMALL = MDLMConfig(vocab_size=1000, mask_token_id=999, blocks=2)


def test_checkpoint_engine_equals_standin_engine(cuda, tmp_path):
    torch = cuda
    from safetensors.torch import save_file

    from diffusionhard_b200.api import load_mdlm
    from diffusionhard_b200.checkpoint import export_hardware_package

    sd = {k: v.contiguous() for k, v in build_standin(SMALL, seed=0).state_dict().items()}
    save_file(sd, tmp_path / "model.safetensors")
    ref = load_mdlm(1, 64, seed=0, config=SMALL)
    ck = load_mdlm(1, 64, config=SMALL, checkpoint=tmp_path / "model.safetensors")
    g = torch.Generator().manual_seed(3)
    ids = torch.randint(0, 999, (64,), generator=g).to(torch.int32).cuda()
    for e in (ref, ck):
        e.tokens.copy_(ids)
        e.forward()
    torch.cuda.synchronize()
    assert torch.equal(ref.x, ck.x)

    folded = fold(build_standin(SMALL, seed=0))
    folded.config = SMALL
    export_hardware_package(folded, tmp_path / "pkg")
    with pytest.raises(ValueError, match="failed validation"):  # no unfolded model: fold not validated
        load_mdlm(1, 64, config=SMALL, package=tmp_path / "pkg")
    from diffusionhard_b200.checkpoint import load_hardware_package
    from diffusionhard_b200.engine import MDLMEngine
    from diffusionhard_b200.model import quantize

    pkg = MDLMEngine(quantize(load_hardware_package(tmp_path / "pkg", verify=False, config=SMALL)), 1, 64)
    pkg.tokens.copy_(ids)
    pkg.forward()
    a, b = ref.logits()[0], pkg.logits()[0]
    rel = float((a - b).abs().mean() / a.abs().mean())
    assert rel < 0.05, rel  # fp16 package weights
    agree = float(a.argmax(-1).eq(b.argmax(-1)).float().mean())
    assert agree >= 0.9, agree
    assert np.isfinite(b.cpu().numpy()).all()


def _same_report(got, ref, path=""):
    if isinstance(ref, dict):
        assert set(got) == set(ref), path
        for k in ref:
            _same_report(got[k], ref[k], path + "." + k)
    elif isinstance(ref, float):
        assert got == pytest.approx(ref, rel=1e-6, abs=1e-9), path
    else:
        assert got == ref, path


def test_fixed_mlp_package_validation_matches_reference(cuda):
    """validate_hardware_fixed_mlp on the reference-written package: the
    integer metrics equal the reference's report exactly, the float metrics
    to 1e-6 (tests/golden/make_package_golden.py)."""
    import json
    import sys

    from conftest import GOLDEN

    sys.path.insert(0, str(GOLDEN))
    from make_package_golden import FIXED_MLP_CASES

    from diffusionhard_b200.fixed_mlp import validate_hardware_fixed_mlp

    ref = json.loads((GOLDEN / "package_golden.json").read_text())["fixed_mlp"]
    for (block, gran, down_gran, alpha), r in zip(FIXED_MLP_CASES, ref):
        got = validate_hardware_fixed_mlp(GOLDEN / "package", block=block, activation_granularity=gran,
                                          down_activation_granularity=down_gran, smoothquant_alpha=alpha)
        got.pop("package_dir")
        _same_report(got, r)
    with pytest.raises(ValueError, match="between 0 and 11"):
        validate_hardware_fixed_mlp(GOLDEN / "package", block=12)
