#!/usr/bin/env python3
"""Generate the committed golden fixtures from the reference itself.

Run in a container that has the reference tree (--reference or DH_REFERENCE_ROOT) and
``make -C oracle ref`` built: the fixtures come from the reference's own code --
its HLS C++ compiled from source (oracle/_ref/libdh_ref.so) and its Python
package (src/diffusion_accel, imported in place).  The GPU box does not have
the reference; tests there compare against these files.

    python tests/golden/make_golden.py --reference <reference root>
"""

from __future__ import annotations

import argparse
import os
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

from oracle import pyoracle  # noqa: E402


def _ref_stream(lib, fn, positions, vocab, ev, st, lo, hi, dtype):
    out = np.zeros(positions * vocab, dtype=dtype)
    status = getattr(lib, fn)(out.ctypes.data, positions, vocab, ev, st, lo, hi)
    assert status == 0
    return out


def make_rng(lib, ref_py) -> dict:
    rng = np.random.default_rng(1234)
    edge = np.array([0, 1, 2, 3, 0xFF, 0x100, 0x7FFFFFFF, 0x80000000, 0xBFFFFFFF, 0xE0000000,
                     0xFFFFFF00, 0xFFFFFFFD, 0xFFFFFFFE, 0xFFFFFFFF], dtype=np.uint32)
    words = np.concatenate([edge, rng.integers(0, 1 << 32, 8192, dtype=np.uint64).astype(np.uint32),
                            (0xFFFFFFFF - rng.integers(0, 1 << 12, 1024)).astype(np.uint32)])
    scores_cpp = np.array([lib.ref_gumbel_q10(int(w)) for w in words], dtype=np.int32)
    import torch

    scores_py = ref_py.rng.approximate_factorized_gumbel_q_from_words(
        torch.tensor(words.astype(np.int64))).numpy().astype(np.int32)
    assert np.array_equal(scores_cpp, scores_py), "reference C++ and Python Gumbel disagree"
    kats = [[list(c), list(k), list(e)] for c, k, e in ref_py.rng.PHILOX4X32_10_KNOWN_ANSWERS]
    ctr = rng.integers(0, 1 << 32, (512, 4), dtype=np.uint64).astype(np.uint32)
    key = rng.integers(0, 1 << 32, (512, 2), dtype=np.uint64).astype(np.uint32)
    outs = np.zeros((512, 4), dtype=np.uint32)
    for i in range(512):
        o = np.zeros(4, dtype=np.uint32)
        lib.ref_philox4x32_10(np.ascontiguousarray(ctr[i]).ctypes.data,
                              np.ascontiguousarray(key[i]).ctypes.data, o.ctypes.data)
        outs[i] = o
    streams = {}
    for name, (p, v, ev, st, lo, hi) in {
        "s3x19": (3, 19, 7, 11, 13, 17),
        "s2x19": (2, 19, 3, 5, 7, 11),
        "s64x1000": (64, 1000, 5, 0, 0xDEADBEEF, 42),
        "s1x50258": (1, 50258, 63, 0, 0, 0),
    }.items():
        streams[name + "_params"] = np.array([p, v, ev, st, lo, hi], dtype=np.uint32)
        streams[name + "_words"] = _ref_stream(lib, "ref_philox_word_stream", p, v, ev, st, lo, hi, np.uint32)
        streams[name + "_scores"] = _ref_stream(lib, "ref_philox_gumbel_stream", p, v, ev, st, lo, hi, np.int32)
    np.savez_compressed(HERE / "rng_golden.npz", words=words, scores=scores_cpp, ctr=ctr, key=key,
                        philox_out=outs, **streams)
    (HERE / "philox_kats.json").write_text(json.dumps(kats, indent=1))
    return {"words": len(words)}


def _ref_head(lib, hidden, weights, mult, bias, noise, mask):
    p, h = hidden.shape
    v = weights.shape[0]
    cand = np.zeros(p, dtype=np.uint16)
    status = lib.ref_output_head_int8(hidden.ctypes.data, weights.ctypes.data, mult.ctypes.data,
                                      bias.ctypes.data, noise.ctypes.data, cand.ctypes.data, p, h, v, mask)
    return status, cand


def make_head(lib) -> dict:
    cases = {}
    # The two deterministic cases of hls/output_head/output_head_test.cpp and
    # hls/integration/rng_output_head_test.cpp, rebuilt with their formulas.
    P, H, V, M = 5, 7, 19, 18
    hidden = ((np.arange(P * H) * 7 + 3) % 17 - 8).astype(np.int8).reshape(P, H)
    weights = ((np.arange(V * H) * 11 + 5) % 23 - 11).astype(np.int8).reshape(V, H)
    mult = ((1 << 19) + np.arange(V) * 17003).astype(np.int32)
    bias = (np.arange(V) * 13 - 80).astype(np.int32)
    noise = ((np.arange(P * V) * 29 + 17) % 101 - 50).astype(np.int32).reshape(P, V)
    st, cand = _ref_head(lib, hidden, weights, mult, bias, noise, M)
    assert st == 0
    cases["tiled"] = dict(hidden=hidden, weights=weights, mult=mult, bias=bias, noise=noise, mask=M, ids=cand)

    hidden = ((np.arange(P * H) * 5 + 1) % 19 - 9).astype(np.int8).reshape(P, H)
    weights = ((np.arange(V * H) * 7 + 2) % 23 - 11).astype(np.int8).reshape(V, H)
    mult = ((1 << 19) + np.arange(V) * 19001).astype(np.int32)
    bias = (np.arange(V) * 17 - 90).astype(np.int32)
    gs = _ref_stream(lib, "ref_philox_gumbel_stream", P, V, 3, 5, 7, 11, np.int32)
    noise = np.zeros((P, V), np.int32)
    i = 0
    for base in range(0, V, 16):
        for p in range(P):
            for lane in range(16):
                t = base + lane
                if t < V:
                    noise[p, t] = gs[i]
                    i += 1
    st, cand = _ref_head(lib, hidden, weights, mult, bias, noise, M)
    assert st == 0
    cases["rng_integration"] = dict(hidden=hidden, weights=weights, mult=mult, bias=bias, noise=noise,
                                    mask=M, ids=cand, rng=np.array([3, 5, 7, 11], np.uint32))

    P, H, V = 2, 3, 5
    st, cand = _ref_head(lib, np.zeros((P, H), np.int8), np.zeros((V, H), np.int8),
                         np.full(V, 1 << 20, np.int32), np.zeros(V, np.int32), np.zeros((P, V), np.int32), 0)
    cases["ties"] = dict(hidden=np.zeros((P, H), np.int8), weights=np.zeros((V, H), np.int8),
                         mult=np.full(V, 1 << 20, np.int32), bias=np.zeros(V, np.int32),
                         noise=np.zeros((P, V), np.int32), mask=0, ids=cand)

    # Random full-width cases with Philox-Gumbel noise (64 positions, hidden 768).
    rng = np.random.default_rng(99)
    for name, (P, H, V, M) in {"rand64x768x300": (64, 768, 300, 299),
                               "rand64x256x1043": (64, 256, 1043, 17)}.items():
        hidden = rng.integers(-127, 128, (P, H)).astype(np.int8)
        weights = np.clip(np.round(rng.normal(0, 40, (V, H))), -127, 127).astype(np.int8)
        mult = rng.integers(1 << 10, 1 << 14, V).astype(np.int32)
        bias = rng.integers(-3000, 3000, V).astype(np.int32)
        gs = _ref_stream(lib, "ref_philox_gumbel_stream", P, V, 9, 0, 0x1234, 0x5678, np.int32)
        noise = np.zeros((P, V), np.int32)
        i = 0
        for base in range(0, V, 16):
            for p in range(P):
                n = min(16, V - base)
                noise[p, base:base + n] = gs[i:i + n]
                i += n
        st, cand = _ref_head(lib, hidden, weights, mult, bias, noise, M)
        assert st == 0
        # noise is not stored: it is the Philox-Gumbel stream of `rng`
        # (eval, stream, seed_lo, seed_hi), pinned separately in rng_golden.npz.
        cases[name] = dict(hidden=hidden, weights=weights, mult=mult, bias=bias, mask=M,
                           ids=cand, rng=np.array([9, 0, 0x1234, 0x5678], np.uint32))
    flat = {}
    for name, d in cases.items():
        for k, v in d.items():
            flat[f"{name}__{k}"] = np.asarray(v)
    np.savez_compressed(HERE / "head_golden.npz", **flat)
    return {"cases": list(cases)}


def make_reveal(lib) -> dict:
    rng = np.random.default_rng(7)
    cases = {}
    for ci, positions in enumerate([1, 7, 63, 64, 65, 70, 128, 200, 256]):
        for variant in range(3):
            tokens = np.full(256, 50257, np.uint16)
            tokens[:positions] = rng.integers(0, 50258, positions)
            cands = rng.integers(0, 50257, 256).astype(np.uint16)
            act = rng.integers(0, 1 << 63, 4, dtype=np.int64).astype(np.uint64) | (rng.integers(0, 1 << 63, 4, dtype=np.int64).astype(np.uint64) << np.uint64(1))
            val = np.full(4, np.uint64(0xFFFFFFFFFFFFFFFF)) if variant != 2 else rng.integers(0, 1 << 63, 4, dtype=np.int64).astype(np.uint64)
            words = rng.integers(0, 1 << 32, 256, dtype=np.uint64).astype(np.uint32)
            thr = [0, 1 << 31, 1 << 32][variant] if variant < 2 else int(rng.integers(0, 1 << 32))
            if variant == 1:
                thr = int(rng.integers(0, 1 << 32))
            t2, a2, v2 = tokens.copy(), act.copy(), val.copy()
            res = lib.ref_candidate_reveal(t2.ctypes.data, cands.ctypes.data, a2.ctypes.data,
                                           v2.ctypes.data, words.ctypes.data, thr, positions)
            cases[f"c{ci}_{variant}"] = dict(positions=positions, tokens=tokens, cands=cands, active=act,
                                             valid=val, words=words, thr=np.uint64(thr), result=np.uint64(res),
                                             tokens_out=t2, active_out=a2, valid_out=v2)
    flat = {}
    for name, d in cases.items():
        for k, v in d.items():
            flat[f"{name}__{k}"] = np.asarray(v)
    np.savez_compressed(HERE / "reveal_golden.npz", **flat)
    return {"cases": len(cases)}


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--reference", default=os.environ.get("DH_REFERENCE_ROOT"),
                    required="DH_REFERENCE_ROOT" not in os.environ,
                    help="reference tree (default: $DH_REFERENCE_ROOT)")
    args = parser.parse_args()
    sys.path.insert(0, str(Path(args.reference) / "src"))
    import diffusion_accel.rng  # noqa: F401  (reference package, imported in place)
    import diffusion_accel as ref_py

    lib = pyoracle.reference_lib()
    if lib is None:
        raise SystemExit("oracle/_ref/libdh_ref.so missing: run `make -C oracle ref REF=<reference>`")
    print("rng", make_rng(lib, ref_py))
    print("head", make_head(lib))
    print("reveal", make_reveal(lib))


if __name__ == "__main__":
    main()
