"""numpy restatement of the reference's fixed-point rotary, fixed18 attention
and packed INT8 attention candidates.  TEST INFRASTRUCTURE ONLY: the tests
use it as the checker of dh_fixed_rotary_q12 / dh_fixed_attention_q12 /
dh_packed_int8_attention_q12; the product never imports it.

Follows src/diffusion_accel/fixed_attention.py:17-113 (symmetric rounding
shift, Q5.12 rotary with Q1.15 constants), :174-298 (Q7.10 scores, LUT
softmax, Q16 x Q12 P . V) and src/diffusion_accel/attention_int8.py:28-123
(dynamic per-vector INT8 Q / K) and :126-315 (calibrated / dynamic Q / K,
requantised probabilities and values), in int64 numpy arithmetic.
"""

from __future__ import annotations

import math
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np

Q12_MIN, Q12_MAX = -(1 << 17), (1 << 17) - 1


def sym_round_shift(v: np.ndarray, shift: int) -> np.ndarray:
    """sign(v) * ((|v| + 2^(shift-1)) >> shift) (fixed_attention.py:17-21)."""
    v = np.asarray(v, dtype=np.int64)
    return np.sign(v) * ((np.abs(v) + (1 << (shift - 1))) >> shift)


def exponential_lut_q16(step_bits: int = 6, cutoff: float = 16.0) -> np.ndarray:
    return np.array([min(65535, round(math.exp(-i / (1 << step_bits)) * 65536))
                     for i in range(int(cutoff * (1 << step_bits)) + 1)], dtype=np.int64)


def rotary_q12(qkv: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> Tuple[np.ndarray, np.ndarray, np.ndarray]:
    """qkv fp32 [T, 2304] -> (qkv_q12 [T, 3, 12, 64], rotated query, key
    [T, 12, 64]) (fixed_attention.py:24-78)."""
    T = qkv.shape[0]
    q = np.clip(np.rint(qkv.astype(np.float64).reshape(T, 3, 12, 64) * 4096.0), Q12_MIN, Q12_MAX).astype(np.int64)
    c = np.clip(np.rint(cos.astype(np.float64) * 32768.0), -(1 << 15), (1 << 15) - 1).astype(np.int64)[:, None, :]
    s = np.clip(np.rint(sin.astype(np.float64) * 32768.0), -(1 << 15), (1 << 15) - 1).astype(np.int64)[:, None, :]

    def rotate(x):
        a, b = x[..., :32], x[..., 32:]
        return np.clip(np.concatenate((sym_round_shift(a * c - b * s, 15), sym_round_shift(b * c + a * s, 15)), -1),
                       Q12_MIN, Q12_MAX)

    return q, rotate(q[:, 0]), rotate(q[:, 1])


def lut_softmax(scores: np.ndarray, lut: np.ndarray) -> np.ndarray:
    """Q0.16 probabilities of Q7.10 score rows, step 6 / cutoff 16
    (fixed_attention.py:226-247, attention_int8.py:92-102)."""
    delta = np.clip(scores - scores.max(axis=-1, keepdims=True), -16384, 0)
    e = lut[np.minimum((-delta + 8) >> 4, 1024)]
    s = e.sum(axis=-1, keepdims=True)
    recip = ((1 << 30) + s // 2) // s
    return np.minimum((e * recip + (1 << 13)) >> 14, 65535)


def _quantize(values: np.ndarray, multiplier, levels: int, frac: int) -> np.ndarray:
    return np.clip(sym_round_shift(values * multiplier, frac), -levels, levels)


def fixed18_scores(q: np.ndarray, k: np.ndarray) -> np.ndarray:
    """[T, 64] x [T, 64] Q5.12 -> Q7.10 (fixed_attention.py:198-212)."""
    return np.clip(sym_round_shift(q @ k.T, 17), Q12_MIN, Q12_MAX)


def packed_attention(qkv: np.ndarray, cos: np.ndarray, sin: np.ndarray, *, qk_mode: str, quantize_qk: bool = True,
                     qk_levels: int = 127, qk_frac: int = 17,
                     calibration: Optional[Sequence[Dict[str, int]]] = None, p_levels: int = 0,
                     sum_correction: bool = False, v_levels: int = 0) -> Dict[str, np.ndarray]:
    """The candidate attention of one canvas.  qk_mode "dynamic" or
    "calibrated" (calibration = per-head maxima); p_levels = 0 keeps the
    fixed18 P . V.  Returns attention [T, 768], scores / probabilities
    [12, T, T], dynamic maxima [12, T] and the fixed18 baseline attention
    and scores."""
    T = qkv.shape[0]
    lut = exponential_lut_q16()
    qkv_q, q12, k12 = rotary_q12(qkv, cos, sin)
    v12 = qkv_q[:, 2]
    out = np.zeros((T, 12, 64), dtype=np.int64)
    base = np.zeros((T, 12, 64), dtype=np.int64)
    scores = np.zeros((12, T, T), dtype=np.int64)
    base_scores = np.zeros((12, T, T), dtype=np.int64)
    probs = np.zeros((12, T, T), dtype=np.int64)
    qmaxs = np.zeros((12, T), dtype=np.int64)
    kmaxs = np.zeros((12, T), dtype=np.int64)
    for h in range(12):
        q, k, v = q12[:, h], k12[:, h], v12[:, h]
        bs = fixed18_scores(q, k)
        base_scores[h] = bs
        base[:, h] = np.clip(sym_round_shift(lut_softmax(bs, lut) @ v, 16), Q12_MIN, Q12_MAX)
        if qk_mode == "dynamic":
            qm = np.maximum(np.abs(q).max(axis=1), 1)
            km = np.maximum(np.abs(k).max(axis=1), 1)
            qmult = np.rint(float(qk_levels * (1 << qk_frac)) / qm.astype(np.float64)).astype(np.int64)
            kmult = np.rint(float(qk_levels * (1 << qk_frac)) / km.astype(np.float64)).astype(np.int64)
            q8 = _quantize(q, qmult[:, None], qk_levels, qk_frac)
            k8 = _quantize(k, kmult[:, None], qk_levels, qk_frac)
            smult = np.rint(qm[:, None].astype(np.float64) * km[None, :].astype(np.float64) * float(1 << 28)
                            / float(qk_levels * qk_levels * (1 << 17))).astype(np.int64)
            qmaxs[h], kmaxs[h] = qm, km
        else:
            m = calibration[h]
            q8 = _quantize(q, round(qk_levels * (1 << qk_frac) / max(1, m["query_q12"])), qk_levels, qk_frac)
            k8 = _quantize(k, round(qk_levels * (1 << qk_frac) / max(1, m["key_q12"])), qk_levels, qk_frac)
            smult = round(m["query_q12"] * m["key_q12"] * (1 << 28) / (qk_levels * qk_levels * (1 << 17)))
        sc = np.clip(sym_round_shift((q8 @ k8.T) * smult, 28), Q12_MIN, Q12_MAX) if quantize_qk else bs
        p = lut_softmax(sc, lut)
        scores[h], probs[h] = sc, p
        if p_levels:
            vmax = calibration[h]["value_q12"]
            v8 = _quantize(v, round(v_levels * (1 << 24) / max(1, vmax)), v_levels, 24)
            pq = np.clip((p * p_levels + (1 << 15)) >> 16, 0, p_levels)
            if sum_correction:
                pq[np.arange(T), p.argmax(axis=-1)] += p_levels - pq.sum(axis=-1)
            mult = round(vmax * (1 << 24) / (v_levels * p_levels))
            out[:, h] = np.clip(sym_round_shift((pq @ v8) * mult, 24), Q12_MIN, Q12_MAX)
        else:
            out[:, h] = np.clip(sym_round_shift(p @ v, 16), Q12_MIN, Q12_MAX)
    return {"attention": out.reshape(T, 768), "scores_q10": scores, "probabilities_q16": probs,
            "query_maxima_q12": qmaxs, "key_maxima_q12": kmaxs, "baseline": base.reshape(T, 768),
            "baseline_scores": base_scores}


def evaluate_options(kw: Dict[str, object]) -> Dict[str, object]:
    """_evaluate_with_fixed_maxima keyword arguments (attention_int8.py:126-161)
    -> packed_attention keyword arguments."""
    qk_bits = int(kw.get("qk_bits", 8))
    v_bits = int(kw.get("pv_value_bits", 8))
    quantize_pv = bool(kw.get("quantize_pv", True))
    return {
        "qk_mode": "dynamic" if kw.get("qk_scale_mode", "calibrated-head") == "dynamic-vector" else "calibrated",
        "quantize_qk": bool(kw.get("quantize_qk", True)),
        "qk_levels": (1 << (qk_bits - 1)) - 1,
        "qk_frac": int(kw.get("qk_multiplier_fraction_bits", 24)),
        "p_levels": int(kw.get("pv_probability_levels", 127)) if quantize_pv else 0,
        "sum_correction": bool(kw.get("pv_probability_sum_correction", False)),
        "v_levels": (1 << (v_bits - 1)) - 1,
    }


def head_maxima(qkv: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> List[Dict[str, int]]:
    """Per-head calibration maxima of one canvas (attention_int8.py:567-583)."""
    qkv_q, q12, k12 = rotary_q12(qkv, cos, sin)
    return [{"query_q12": max(1, int(np.abs(q12[:, h]).max())), "key_q12": max(1, int(np.abs(k12[:, h]).max())),
             "value_q12": max(1, int(np.abs(qkv_q[:, 2, h]).max()))} for h in range(12)]
