"""Checkpoint and hardware-package I/O against the reference's own package
code (tests/golden/make_package_golden.py): the validator's verdicts, the
fp16 folded weights and DDR image read back, byte-identical export, and the
HF-layout state-dict loader.  No GPU."""

import json
import shutil
import sys

import numpy as np
import pytest
import torch

from conftest import GOLDEN

sys.path.insert(0, str(GOLDEN))
from make_package_golden import package_config, package_standin  # noqa: E402

from diffusionhard_b200 import checkpoint as ck  # noqa: E402
from diffusionhard_b200.model import ddit_forward, fold, fp32_forward  # noqa: E402

PKG = GOLDEN / "package"
GJ = json.loads((GOLDEN / "package_golden.json").read_text())


def _report(r):
    return {k: v for k, v in r.items() if k != "package_dir"}


def _folded():
    f = fold(package_standin())
    f.config = package_config()
    return f


def test_validator_matches_reference_verdicts(tmp_path):
    assert _report(ck.validate_hardware_package(PKG)) == GJ["reference_package"]
    bad = tmp_path / "bad"
    shutil.copytree(PKG, bad)
    raw = bytearray((bad / ck.BINARY_FILE).read_bytes())
    raw[4096 + 10] ^= 0x40
    (bad / ck.BINARY_FILE).write_bytes(bytes(raw))
    assert _report(ck.validate_hardware_package(bad)) == GJ["flipped_byte"]
    with pytest.raises(ValueError, match="failed validation"):
        ck.load_hardware_package(bad, config=package_config())


def test_layout_errors_are_reported():
    m = json.loads((PKG / ck.MANIFEST_FILE).read_text())
    assert ck.binary_layout_errors(m) == []
    names = ck.hardware_weight_order(m["weight_binary_layout"]["tensors"])
    entries = m["weight_binary_layout"]["tensors"]
    entries[names[1]]["offset_bytes"] += 2
    # names[1] fills its 4 KiB pages exactly, so shifting it also overlaps names[2]
    assert ck.binary_layout_errors(m) == ["%s offset is not aligned" % names[1],
                                          "%s overlaps the previous tensor" % names[2]]
    entries[names[1]]["offset_bytes"] = entries[names[0]]["offset_bytes"]
    assert ck.binary_layout_errors(m) == ["%s overlaps the previous tensor" % names[1]]
    last = names[-1]
    entries[names[1]]["offset_bytes"] = entries[names[2]]["offset_bytes"] - entries[names[1]]["length_bytes"]
    entries[last]["offset_bytes"] = m["weight_binary_layout"]["total_bytes"]
    assert ck.binary_layout_errors(m) == ["%s exceeds the declared binary size" % last]


@pytest.mark.parametrize("from_binary", [False, True])
def test_reference_package_loads_as_our_fold(from_binary):
    got = ck.load_hardware_package(PKG, from_binary=from_binary, config=package_config())
    exp = _folded()
    r16 = lambda a: np.asarray(a, np.float32).astype(np.float16).astype(np.float32)  # noqa: E731
    assert np.array_equal(got.embedding, r16(exp.embedding))
    for gb, eb in zip(got.blocks, exp.blocks):
        for name in ("qkv", "out", "up", "down"):
            assert np.array_equal(gb[name].weight, r16(eb[name].weight)), name
            if eb[name].bias is None:
                assert gb[name].bias is None
            else:
                assert np.array_equal(gb[name].bias, r16(eb[name].bias)), name
    assert np.array_equal(got.head.weight, r16(exp.head.weight))
    assert (got.config.hidden, got.config.heads, got.config.mlp, got.config.blocks, got.config.vocab_size) == \
        (64, 2, 256, 2, 101)


def test_export_is_byte_identical_to_reference(tmp_path):
    f = _folded()
    m = ck.export_hardware_package(f, tmp_path / "ours", unfolded_logits=ddit_forward(package_standin(), np.asarray(
        [ck.deterministic_hardware_input(64, 101, 100)])))
    ref = json.loads((PKG / ck.MANIFEST_FILE).read_text())
    for name in (ck.WEIGHTS_FILE, ck.BINARY_FILE):
        assert m["files"][name] == ref["files"][name], name
    assert m["weight_binary_layout"] == ref["weight_binary_layout"]
    assert m["weights"] == ref["weights"]
    assert m["constant_fold_validation"]["passed"]
    assert ck.validate_hardware_package(tmp_path / "ours")["passed"]
    assert m["files"][ck.BINARY_FILE]["sha256"] == GJ["our_export_weights_sha256"]
    with pytest.raises(ValueError, match="frozen to 64"):
        ck.export_hardware_package(f, tmp_path / "x", canvas_tokens=32)
    unvalidated = ck.export_hardware_package(f, tmp_path / "nofold")
    assert not unvalidated["constant_fold_validation"]["passed"]


def test_fold_matches_reference_folded_forward_and_unfolded_model():
    from safetensors.torch import load_file

    g = load_file(str(PKG / ck.GOLDEN_FILE))
    ids = g["input.ids"].numpy().astype(np.int64)
    assert ids[0].tolist() == ck.deterministic_hardware_input(64, 101, 100)
    f = _folded()
    logits = fp32_forward(f, ids) @ f.head.weight.T + f.head.bias
    np.testing.assert_allclose(logits, g["folded.final.logits"].numpy(), rtol=0, atol=2e-6)
    np.testing.assert_allclose(ddit_forward(package_standin(), ids).numpy(), logits, rtol=0, atol=2e-6)


def test_state_dict_loader(tmp_path):
    from safetensors.torch import save_file

    cfg = package_config()
    m = package_standin()
    sd = {k: v.contiguous() for k, v in m.state_dict().items()}
    exp = _folded()
    for src in (sd, {"model." + k: v for k, v in sd.items()}):
        got = ck.load_checkpoint(src, cfg)
        assert np.array_equal(got.blocks[1]["up"].weight, exp.blocks[1]["up"].weight)
        assert np.array_equal(got.head.bias, exp.head.bias)
    save_file(sd, tmp_path / "model.safetensors")
    got = ck.load_checkpoint(tmp_path / "model.safetensors", cfg)
    assert np.array_equal(got.embedding, exp.embedding)
    torch.save(sd, tmp_path / "model.pt")
    assert np.array_equal(ck.load_checkpoint(tmp_path / "model.pt", cfg).blocks[0]["qkv"].bias,
                          exp.blocks[0]["qkv"].bias)
    broken = dict(sd)
    broken.pop("backbone.blocks.0.attn_qkv.weight")
    with pytest.raises(ValueError, match="missing"):
        ck.load_checkpoint(broken, cfg)
    broken = dict(sd)
    broken["backbone.output_layer.linear.bias"] = torch.zeros(7)
    with pytest.raises(ValueError, match="shape mismatch"):
        ck.load_checkpoint(broken, cfg)


def test_hardware_input_and_decode():
    ids = ck.deterministic_hardware_input(64, 50258, 50257)
    assert ids[0] == 17 and ids[1] == 50257 and ids[3] == (3 * 7919 + 17) % 50257
    with pytest.raises(ValueError, match="final ID"):
        ck.deterministic_hardware_input(64, 50258, 5)
    text = ck.decode_tokens([1, 2, 3])
    assert text is None or isinstance(text, str)
