"""Pin the CPU oracle to the reference: known answers, golden vectors, and the
reference's own compiled C++ (when oracle/_ref was built here)."""

import json
import subprocess
import sys

import numpy as np
import pytest

from conftest import GOLDEN, REFERENCE_ROOT, ROOT, load_npz_cases
from oracle import pyoracle

REF_TESTS = ["philox_rng_test", "output_head_test", "candidate_sampler_test",
             "rng_output_head_test", "int8_mac_tile_test"]


def test_philox_random123_known_answers():
    kats = json.loads((GOLDEN / "philox_kats.json").read_text())
    assert len(kats) == 3
    for ctr, key, expected in kats:
        assert pyoracle.philox(ctr, key) == tuple(expected)


def test_philox_matches_reference_on_random_counters():
    g = np.load(GOLDEN / "rng_golden.npz")
    for i in range(0, 512, 7):
        assert pyoracle.philox(g["ctr"][i], g["key"][i]) == tuple(int(x) for x in g["philox_out"][i])


def test_gumbel_golden_points():
    # philox_rng_test.cpp:84-92
    points = {0: -1983, 1: -1983, 0x7FFFFFFF: 372, 0x80000000: 377, 0xFFFFFF00: 17043,
              0xFFFFFFFE: 22718, 0xFFFFFFFF: 23423}
    got = pyoracle.gumbel_q10(np.array(list(points), dtype=np.uint32))
    assert got.tolist() == list(points.values())


def test_gumbel_matches_reference_vectors():
    g = np.load(GOLDEN / "rng_golden.npz")
    assert np.array_equal(pyoracle.gumbel_q10(g["words"]), g["scores"])


def test_gumbel_is_monotonic():
    words = np.array([0, 1, 100, 1 << 16, 1 << 24, (1 << 32) - 2, (1 << 32) - 1], dtype=np.uint32)
    s = pyoracle.gumbel_q10(words)
    assert np.all(s[1:] >= s[:-1])


def test_gumbel_tables_match_generator_and_reference():
    sys.path.insert(0, str(ROOT / "diffusionhard_b200" / "csrc"))
    import gen_gumbel_lut

    base, corr, top, l2 = gen_gumbel_lut.tables()
    obase, ocorr, otop, ol2 = pyoracle.gumbel_tables()
    assert obase.tolist() == base and ocorr.tolist() == corr and otop == top == 23423 and ol2 == l2 == 710
    header = (ROOT / "diffusionhard_b200" / "csrc" / "gumbel_lut.h").read_text()
    assert header == gen_gumbel_lut.render_header(), "gumbel_lut.h is stale; rerun gen_gumbel_lut.py"
    ref_header = REFERENCE_ROOT / "hls" / "rng" / "gumbel_lut.hpp"
    if ref_header.exists():
        import re

        text = ref_header.read_text()
        nums = [int(x) for x in re.findall(r"-?\d+", text.split("kGumbelBaseQ = {{")[1].split("}};")[0])]
        assert nums == base
        cnums = [int(x) for x in re.findall(r"-?\d+", text.split("kGumbelCorrectionQ = {{")[1].split("}};")[0])]
        assert cnums == [v for row in corr for v in row]


@pytest.mark.parametrize("name", ["s3x19", "s2x19", "s64x1000"])
def test_word_stream_order_matches_reference(name):
    g = np.load(GOLDEN / "rng_golden.npz")
    p, v, ev, st, lo, hi = (int(x) for x in g[name + "_params"])
    words = pyoracle.word_stream(p, v, ev, st, lo, hi)
    assert np.array_equal(words, g[name + "_words"])
    assert np.array_equal(pyoracle.gumbel_q10(words), g[name + "_scores"])


def _noise_from_stream(scores, positions, vocab):
    noise = np.zeros((positions, vocab), np.int32)
    i = 0
    for base in range(0, vocab, 16):
        n = min(16, vocab - base)
        for p in range(positions):
            noise[p, base:base + n] = scores[i:i + n]
            i += n
    return noise


@pytest.mark.parametrize("case", ["tiled", "rng_integration", "ties", "rand64x768x300", "rand64x256x1043"])
def test_head_requant_matches_reference(case):
    c = load_npz_cases("head_golden.npz")[case]
    if "noise" in c:
        noise = c["noise"]
    else:
        ev, st, lo, hi = (int(x) for x in c["rng"])
        p, v = c["hidden"].shape[0], c["weights"].shape[0]
        noise = _noise_from_stream(pyoracle.gumbel_q10(pyoracle.word_stream(p, v, ev, st, lo, hi)), p, v)
    ids, _ = pyoracle.head_i8(pyoracle.HEAD_REQUANT_Q20, c["hidden"], c["weights"], int(c["mask"]),
                              mult_q20=c["mult"], bias_q10=c["bias"], noise=noise)
    assert ids.tolist() == c["ids"].astype(np.int32).tolist()


def test_head_requant_in_place_philox_matches_stream_noise():
    c = load_npz_cases("head_golden.npz")["rand64x256x1043"]
    ev, st, lo, hi = (int(x) for x in c["rng"])
    p = c["hidden"].shape[0]
    ids, _ = pyoracle.head_i8(pyoracle.HEAD_REQUANT_Q20, c["hidden"], c["weights"], int(c["mask"]),
                              mult_q20=c["mult"], bias_q10=c["bias"], row_position=np.arange(p),
                              row_key_hi=np.full(p, hi), row_eval=np.full(p, ev), key_lo=lo, stream_id=st)
    assert ids.tolist() == c["ids"].astype(np.int32).tolist()


def test_reveal_matches_reference():
    # The reference arrays are fixed at 256 positions (4 bitmap words) and its
    # invalidation clears all 4 words; a canvas of P positions owns the first
    # ceil(P/64) words, which is what the batched layout stores per sequence.
    for name, c in load_npz_cases("reveal_golden.npz").items():
        t, a, v = c["tokens"].copy(), c["active"].copy(), c["valid"].copy()
        res = pyoracle.candidate_reveal(t, c["cands"], a, v, c["words"], int(c["thr"]), int(c["positions"]))
        nw = (int(c["positions"]) + 63) // 64
        assert res == int(c["result"]), name
        assert np.array_equal(t, c["tokens_out"]) and np.array_equal(a, c["active_out"]), name
        assert np.array_equal(v[:nw], c["valid_out"][:nw]), name


def test_reveal_invalid_controls_do_not_mutate():
    t = np.full(256, 5, np.uint16)
    c = np.zeros(256, np.uint16)
    a = np.full(4, np.uint64(0xFFFFFFFFFFFFFFFF))
    v = a.copy()
    w = np.zeros(256, np.uint32)
    assert pyoracle.candidate_reveal(t, c, a, v, w, 0, 0) >> 32 == 1
    assert pyoracle.candidate_reveal(t, c, a, v, w, (1 << 32) + 1, 8) >> 32 == 2
    assert np.all(t == 5) and np.all(a == np.uint64(0xFFFFFFFFFFFFFFFF))


def test_noisy_argmax_f32_matches_manual():
    rng = np.random.default_rng(0)
    logits = (3 * rng.standard_normal((4, 37))).astype(np.float32)
    ids, scores = pyoracle.noisy_argmax_f32(logits, 36, row_key_hi=np.arange(4), row_eval=np.full(4, 5), key_lo=9)
    for r in range(4):
        best, bid = None, None
        for v in range(36):
            w = pyoracle.philox((v // 4, r, 5, 0), (9, r))[v % 4]
            s = int(np.round(np.float32(logits[r, v]) * np.float32(1024))) + int(pyoracle.gumbel_q10(np.array([w]))[0])
            if best is None or s > best:
                best, bid = s, v
        assert ids[r] == bid and scores[r] == best


@pytest.mark.skipif(not (REFERENCE_ROOT / "hls").is_dir(), reason="reference tree not present")
def test_reference_cpp_tests_pass_from_oracle_ref():
    subprocess.run(["make", "-s", "-C", str(ROOT / "oracle"), "ref", f"REF={REFERENCE_ROOT}"], check=True)
    for name in REF_TESTS:
        out = subprocess.run([str(ROOT / "oracle" / "_ref" / name)], capture_output=True, text=True, check=True)
        assert "all checks passed" in out.stdout


@pytest.mark.skipif(pyoracle.reference_lib() is None, reason="oracle/_ref not built")
def test_oracle_equals_reference_lib_on_random_words():
    ref = pyoracle.reference_lib()
    rng = np.random.default_rng(5)
    words = rng.integers(0, 1 << 32, 20000, dtype=np.uint64).astype(np.uint32)
    ours = pyoracle.gumbel_q10(words)
    theirs = np.array([ref.ref_gumbel_q10(int(w)) for w in words], dtype=np.int32)
    assert np.array_equal(ours, theirs)
