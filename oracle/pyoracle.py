"""numpy/ctypes front end of the CPU oracles.  TEST INFRASTRUCTURE ONLY.

* :data:`ORACLE` wraps ``oracle/lib/liboracle.so`` -- the plain-C restatement
  of the reference algorithms (dh_oracle.c); it is always available (built by
  ``make -C oracle``).
* :func:`reference_lib` wraps ``oracle/_ref/libdh_ref.so`` -- the reference's
  own HLS C++ compiled from its sources; present only where the reference tree
  was available at build time.

Only tests, ``__graft_entry__.smoke`` and bench.py's CPU-baseline / reference
arm use this module, as the checker.  The product never imports it.
"""

from __future__ import annotations

import ctypes
import subprocess
from functools import lru_cache
from pathlib import Path
from typing import Optional

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_PATH = HERE / "lib" / "liboracle.so"
REF_PATH = HERE / "_ref" / "libdh_ref.so"

_P = ctypes.c_void_p
_U32 = ctypes.c_uint32
_U64 = ctypes.c_uint64
_I32 = ctypes.c_int32


def _p(a: Optional[np.ndarray]) -> Optional[int]:
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data


@lru_cache(maxsize=1)
def oracle_lib() -> ctypes.CDLL:
    if not ORACLE_PATH.exists():
        subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    lib = ctypes.CDLL(str(ORACLE_PATH))
    sig = {
        "or_philox4x32_10": (None, [_P, _P, _P]),
        "or_philox_token_word": (_U32, [_U32] * 6),
        "or_reveal_word": (_U32, [_U32] * 4),
        "or_gumbel_tables": (None, [_P, _P, _P, _P]),
        "or_gumbel_q10": (_I32, [_U32]),
        "or_logit_q10": (_I32, [ctypes.c_float]),
        "or_noisy_argmax_f32": (None, [_P, _U32, _U32, _U32, _P, _P, _P, _U32, _U32, _P, _P]),
        "or_greedy_argmax_f32": (None, [_P, _U32, _U32, _U32, _P]),
        "or_requantize_q20": (_I32, [_I32, _I32]),
        "or_gemm_i8": (None, [_P, _P, _U32, _U32, _U32, _P]),
        "or_dequant_logit": (ctypes.c_float, [_I32, ctypes.c_float, ctypes.c_float, ctypes.c_float]),
        "or_head_i8": (None, [ctypes.c_int, _P, _P, _U32, _U32, _U32, _U32, _P, _P, _P, _P, _P,
                              _P, _P, _P, _P, _U32, _U32, _P, _P]),
        "or_candidate_reveal": (_U64, [_P, _P, _P, _P, _P, _U64, _U32]),
        "or_candidate_cache_sampler_f32": (_U32, [_P, _U32, _U32, _U32, _U32, _P, _U32, _U32, _P,
                                                  _P, _P, _P, _P, _P, _P, _P, _P]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


@lru_cache(maxsize=1)
def reference_lib() -> Optional[ctypes.CDLL]:
    """The reference HLS C++ (compiled from its own sources), or None."""
    if not REF_PATH.exists():
        return None
    lib = ctypes.CDLL(str(REF_PATH))
    sig = {
        "ref_philox4x32_10": (None, [_P, _P, _P]),
        "ref_gumbel_q10": (_I32, [_U32]),
        "ref_gumbel_lut_address": (_U32, [_U32]),
        "ref_philox_word_stream": (_U32, [_P, _U32, _U32, _U32, _U32, _U32, _U32]),
        "ref_philox_gumbel_stream": (_U32, [_P, _U32, _U32, _U32, _U32, _U32, _U32]),
        "ref_output_head_int8": (_U32, [_P, _P, _P, _P, _P, _P, _U32, _U32, _U32, _U32]),
        "ref_candidate_reveal": (_U64, [_P, _P, _P, _P, _P, _U64, _U32]),
        "ref_candidate_max_positions": (_U32, []),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


# ------------------------------------------------------------------ helpers

def philox(counter, key) -> tuple:
    c = np.ascontiguousarray(counter, dtype=np.uint32)
    k = np.ascontiguousarray(key, dtype=np.uint32)
    out = np.zeros(4, dtype=np.uint32)
    oracle_lib().or_philox4x32_10(_p(c), _p(k), _p(out))
    return tuple(int(x) for x in out)


def gumbel_q10(words: np.ndarray) -> np.ndarray:
    lib = oracle_lib()
    w = np.asarray(words, dtype=np.uint32).ravel()
    return np.array([lib.or_gumbel_q10(int(x)) for x in w], dtype=np.int32).reshape(np.shape(words))


def gumbel_tables() -> tuple:
    base = np.zeros(256, dtype=np.int16)
    corr = np.zeros(768, dtype=np.int16)
    top = ctypes.c_int32()
    l2 = ctypes.c_int32()
    oracle_lib().or_gumbel_tables(_p(base), _p(corr), ctypes.addressof(top), ctypes.addressof(l2))
    return base, corr.reshape(3, 256), top.value, l2.value


def word_stream(positions: int, vocab: int, eval_id: int, stream_id: int, seed_lo: int,
                seed_hi: int) -> np.ndarray:
    """Philox words in the reference stream order (philox_rng.cpp:95-149)."""
    lib = oracle_lib()
    out = []
    for base in range(0, vocab, 16):
        for p in range(positions):
            for lb in range(4):
                t0 = base + 4 * lb
                if t0 >= vocab:
                    continue
                w = philox((t0 // 4, p, eval_id, stream_id), (seed_lo, seed_hi))
                for i in range(4):
                    if t0 + i < vocab:
                        out.append(w[i])
    del lib
    return np.array(out, dtype=np.uint32)


def noisy_argmax_f32(logits: np.ndarray, mask_id: int, row_position=None, row_key_hi=None,
                     row_eval=None, key_lo: int = 0, stream_id: int = 0):
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    rows, vocab = logits.shape
    pos = np.ascontiguousarray(np.arange(rows) if row_position is None else row_position, dtype=np.uint32)
    khi = np.ascontiguousarray(np.zeros(rows) if row_key_hi is None else row_key_hi, dtype=np.uint32)
    ev = np.ascontiguousarray(np.zeros(rows) if row_eval is None else row_eval, dtype=np.uint32)
    ids = np.zeros(rows, dtype=np.int32)
    scores = np.zeros(rows, dtype=np.int32)
    oracle_lib().or_noisy_argmax_f32(_p(logits), rows, vocab, mask_id, _p(pos), _p(khi), _p(ev),
                                     key_lo, stream_id, _p(ids), _p(scores))
    return ids, scores


def greedy_argmax_f32(logits: np.ndarray, mask_id: int) -> np.ndarray:
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    rows, vocab = logits.shape
    ids = np.zeros(rows, dtype=np.int32)
    oracle_lib().or_greedy_argmax_f32(_p(logits), rows, vocab, mask_id, _p(ids))
    return ids


HEAD_REQUANT_Q20, HEAD_DEQUANT_NOISY, HEAD_DEQUANT_GREEDY = 0, 1, 2


def head_i8(mode: int, hidden: np.ndarray, weights: np.ndarray, mask_id: int, *, mult_q20=None,
            bias_q10=None, noise=None, a_scale=None, w_scale=None, bias=None, row_position=None,
            row_key_hi=None, row_eval=None, key_lo: int = 0, stream_id: int = 0):
    hidden = np.ascontiguousarray(hidden, dtype=np.int8)
    weights = np.ascontiguousarray(weights, dtype=np.int8)
    rows, k = hidden.shape
    vocab = weights.shape[0]
    c = lambda a, t: None if a is None else np.ascontiguousarray(a, dtype=t)  # noqa: E731
    args = [c(mult_q20, np.int32), c(bias_q10, np.int32), c(noise, np.int32), c(a_scale, np.float32),
            c(w_scale, np.float32), c(bias, np.float32), c(row_position, np.uint32),
            c(row_key_hi, np.uint32), c(row_eval, np.uint32)]
    ids = np.zeros(rows, dtype=np.int32)
    scores = np.zeros(rows, dtype=np.int32)
    oracle_lib().or_head_i8(mode, _p(hidden), _p(weights), rows, k, vocab, mask_id,
                            *[_p(a) for a in args], key_lo, stream_id, _p(ids), _p(scores))
    return ids, scores


def gemm_i8(a: np.ndarray, w: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.int8)
    w = np.ascontiguousarray(w, dtype=np.int8)
    out = np.zeros((a.shape[0], w.shape[0]), dtype=np.int32)
    oracle_lib().or_gemm_i8(_p(a), _p(w), a.shape[0], w.shape[0], a.shape[1], _p(out))
    return out


def candidate_reveal(tokens, cands, active, valid, words, threshold: int, positions: int):
    """In-place on numpy arrays; returns the packed (status << 32) | changed."""
    return int(oracle_lib().or_candidate_reveal(_p(tokens), _p(cands), _p(active), _p(valid),
                                                _p(words), threshold, positions))


def reveal_words(positions: int, step: int, seed: int, seq: int) -> np.ndarray:
    lib = oracle_lib()
    return np.array([lib.or_reveal_word(p, step, seed, seq) for p in range(positions)], dtype=np.uint32)


def candidate_cache_sampler_f32(logits_per_eval: np.ndarray, tokens: np.ndarray, mask_id: int,
                                thr_q32: np.ndarray, seed: int, seq_index: int = 0,
                                snapshots: bool = True) -> dict:
    """Run the oracle sampler loop for one sequence; returns a dict of arrays."""
    logits_per_eval = np.ascontiguousarray(logits_per_eval, dtype=np.float32)
    steps = len(thr_q32)
    assert logits_per_eval.shape[0] == steps + 1
    positions, vocab = logits_per_eval.shape[1:]
    words_n = (positions + 63) // 64
    tok = np.ascontiguousarray(tokens, dtype=np.int32).copy()
    thr = np.ascontiguousarray(thr_q32, dtype=np.uint64)
    snap_t = np.zeros((steps, positions), np.int32) if snapshots else None
    snap_c = np.zeros((steps, positions), np.int32) if snapshots else None
    snap_a = np.zeros((steps, words_n), np.uint64) if snapshots else None
    snap_v = np.zeros((steps, words_n), np.uint64) if snapshots else None
    act = np.zeros(steps, np.int32)
    chg = np.zeros(steps, np.int32)
    evl = np.zeros(steps, np.int32)
    trans = ctypes.c_uint32()
    evals = oracle_lib().or_candidate_cache_sampler_f32(
        _p(logits_per_eval), positions, vocab, mask_id, steps, _p(thr), seed, seq_index, _p(tok),
        _p(snap_t), _p(snap_c), _p(snap_a), _p(snap_v), _p(act), _p(chg), _p(evl),
        ctypes.addressof(trans))
    return {"tokens": tok, "snap_tokens": snap_t, "snap_candidates": snap_c, "snap_active": snap_a,
            "snap_valid": snap_v, "step_active": act, "step_changed": chg, "step_evaluated": evl,
            "evaluations": int(evals), "transitions": int(trans.value)}
