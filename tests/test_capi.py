"""CPU checks of the C ABI: the library loads, exports every declared symbol,
and argument validation returns the reference's status codes before any GPU
work (these calls return early, so they need no device)."""

import ctypes
import re

import pytest

from conftest import ROOT
from diffusionhard_b200 import _lib


def _declared():
    text = re.sub(r"/\*.*?\*/", " ", (ROOT / "include" / "dh_b200.h").read_text(), flags=re.S)
    return set(re.findall(r"\b(dh_\w+)\s*\(", text))


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    declared = _declared()
    assert declared == set(_lib.parse_header())
    missing = [name for name in declared if not hasattr(lib, name)]
    assert not missing


def test_rng_stream_status_codes_match_reference():
    # philox_rng.cpp:114-119
    assert _lib.raw("dh_philox_word_stream", None, 0, 1, 0, 0, 0, 0, None) == 1
    assert _lib.raw("dh_philox_word_stream", None, 65, 1, 0, 0, 0, 0, None) == 1
    assert _lib.raw("dh_philox_word_stream", None, 1, 0, 0, 0, 0, 0, None) == 2
    assert _lib.raw("dh_philox_gumbel_stream", None, 1, 65536, 0, 0, 0, 0, None) == 2
    assert _lib.raw("dh_philox_gumbel_stream", None, 1, 1, 0, 0, 0, 0, None) == 100


def test_reveal_status_codes_match_reference():
    # candidate_sampler.cpp:29-34: position count first, then threshold.
    assert _lib.raw("dh_candidate_reveal", None, None, None, None, None, 0, 0, 1, None, None) == 1
    assert _lib.raw("dh_candidate_reveal", None, None, None, None, None, (1 << 32) + 1, 8, 1, None, None) == 2
    assert _lib.raw("dh_candidate_reveal", None, None, None, None, None, 1 << 32, 8, 1, None, None) == 100


def test_argmax_validation():
    assert _lib.raw("dh_noisy_argmax_f32", None, 10, 0, 10, 0, None, None, None, 0, 0, None, None, None, 0, None) == 1
    assert _lib.raw("dh_noisy_argmax_f32", None, 10, 1, 10, 10, None, None, None, 0, 0, None, None, None, 0, None) == 2
    assert _lib.raw("dh_noisy_argmax_workspace_size", 64, 50258) == 64 * 13 * 8


def test_sampler_workspace_query_is_pure():
    a = _lib.lib().dh_sampler_workspace_size(2, 64, 1000)
    b = _lib.lib().dh_sampler_workspace_size(2, 64, 1000)
    assert a == b and a >= 2 * 64 * 8


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(_lib, "LIB_PATH", tmp_path / "nope.so")
    _lib.lib.cache_clear()
    try:
        with pytest.raises(_lib.DHLibraryError):
            _lib.lib()
    finally:
        monkeypatch.undo()
        _lib.lib.cache_clear()
        _lib.lib()


def test_noise_argmax_status_codes():
    # RNG family first (row count, vocabulary / mask), then the null sink
    assert _lib.raw("dh_noise_argmax", 0, 10, 0, None, None, None, 0, 0, 0, 0, None, None, None) == 1
    assert _lib.raw("dh_noise_argmax", 1, 0, 0, None, None, None, 0, 0, 0, 0, None, None, None) == 2
    assert _lib.raw("dh_noise_argmax", 1, 65536, 0, None, None, None, 0, 0, 0, 0, None, None, None) == 2
    assert _lib.raw("dh_noise_argmax", 1, 10, 10, None, None, None, 0, 0, 0, 0, None, None, None) == 2
    assert _lib.raw("dh_noise_argmax", 1, 10, 9, None, None, None, 0, 0, 0, 0, None, None, None) == 100
