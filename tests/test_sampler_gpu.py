"""GPU parity of the sampler kernels (K1 noisy argmax, K2 reveal, Philox
streams, the device candidate-cache loop) against the oracle and the
reference golden vectors.  Everything here is bit-exact."""

import json

import numpy as np
import pytest

from conftest import GOLDEN, load_npz_cases
from diffusionhard_b200 import _lib
from diffusionhard_b200.sampler import (CandidateCacheState, reveal_thresholds_q32,
                                        run_candidate_cache_sampler_f32)
from oracle import pyoracle

pytestmark = pytest.mark.gpu


def _dev(torch, a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.to(dtype)
    return t.cuda()


def test_philox_known_answers_on_device(cuda):
    torch = cuda
    kats = json.loads((GOLDEN / "philox_kats.json").read_text())
    g = np.load(GOLDEN / "rng_golden.npz")
    ctr = np.concatenate([np.array([k[0] for k in kats], np.uint32), g["ctr"]])
    key = np.concatenate([np.array([k[1] for k in kats], np.uint32), g["key"]])
    exp = np.concatenate([np.array([k[2] for k in kats], np.uint32), g["philox_out"]])
    c, k = _dev(torch, ctr.view(np.int32)), _dev(torch, key.view(np.int32))
    out = torch.zeros_like(c)
    _lib.call("dh_philox4x32_10", _lib.ptr(c), _lib.ptr(k), _lib.ptr(out), len(ctr), None)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy().view(np.uint32), exp)


def test_gumbel_q10_on_device_matches_reference(cuda):
    torch = cuda
    g = np.load(GOLDEN / "rng_golden.npz")
    w = _dev(torch, g["words"].view(np.int32))
    out = torch.zeros_like(w)
    _lib.call("dh_gumbel_q10", _lib.ptr(w), _lib.ptr(out), w.numel(), None)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), g["scores"])
    # exhaustive over the tail binade and a strided sweep of the whole range
    words = np.concatenate([np.arange(0xFFF00000, 0x100000000, dtype=np.uint64),
                            np.arange(0, 1 << 32, 65537, dtype=np.uint64)]).astype(np.uint32)
    w = _dev(torch, words.view(np.int32))
    out = torch.zeros_like(w)
    _lib.call("dh_gumbel_q10", _lib.ptr(w), _lib.ptr(out), w.numel(), None)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), pyoracle.gumbel_q10(words))


@pytest.mark.parametrize("name", ["s3x19", "s2x19", "s64x1000", "s1x50258"])
def test_streams_match_reference_order(cuda, name):
    torch = cuda
    g = np.load(GOLDEN / "rng_golden.npz")
    p, v, ev, st, lo, hi = (int(x) for x in g[name + "_params"])
    words = torch.zeros(p * v, dtype=torch.int32, device="cuda")
    scores = torch.zeros(p * v, dtype=torch.int32, device="cuda")
    _lib.call("dh_philox_word_stream", _lib.ptr(words), p, v, ev, st, lo, hi, None)
    _lib.call("dh_philox_gumbel_stream", _lib.ptr(scores), p, v, ev, st, lo, hi, None)
    torch.cuda.synchronize()
    assert np.array_equal(words.cpu().numpy().view(np.uint32), g[name + "_words"])
    assert np.array_equal(scores.cpu().numpy(), g[name + "_scores"])


def _noisy(torch, logits, mask, pos=None, khi=None, ev=None, key_lo=0, stream=0, greedy=False):
    rows, vocab = logits.shape
    L = _dev(torch, logits.astype(np.float32))
    ids = torch.zeros(rows, dtype=torch.int32, device="cuda")
    scores = torch.zeros(rows, dtype=torch.int32, device="cuda")
    ws = torch.empty(max(1, _lib.lib().dh_noisy_argmax_workspace_size(rows, vocab)), dtype=torch.uint8,
                     device="cuda")
    arr = lambda a: None if a is None else _dev(torch, np.asarray(a, np.uint32).view(np.int32))  # noqa: E731
    p_, k_, e_ = arr(pos), arr(khi), arr(ev)
    if greedy:
        _lib.call("dh_greedy_argmax_f32", _lib.ptr(L), vocab, rows, vocab, mask, _lib.ptr(ids),
                  _lib.ptr(ws), ws.numel(), None)
    else:
        _lib.call("dh_noisy_argmax_f32", _lib.ptr(L), vocab, rows, vocab, mask, _lib.ptr(p_),
                  _lib.ptr(k_), _lib.ptr(e_), key_lo, stream, _lib.ptr(ids), _lib.ptr(scores),
                  _lib.ptr(ws), ws.numel(), None)
    torch.cuda.synchronize()
    return ids.cpu().numpy(), scores.cpu().numpy()


@pytest.mark.parametrize("rows,vocab,mask", [(64, 50258, 50257), (3, 19, 18), (5, 7, 0), (2, 1, 0),
                                             (17, 4097, 4096), (300, 1000, 3)])
def test_noisy_argmax_matches_oracle(cuda, rows, vocab, mask):
    rng = np.random.default_rng(rows * 7 + vocab)
    logits = (3 * rng.standard_normal((rows, vocab))).astype(np.float32)
    pos = rng.integers(0, 1024, rows)
    khi = rng.integers(0, 512, rows)
    ev = rng.integers(0, 64, rows)
    ids, scores = _noisy(cuda, logits, mask, pos, khi, ev, key_lo=11, stream=0)
    oids, oscores = pyoracle.noisy_argmax_f32(logits, mask, pos, khi, ev, key_lo=11)
    assert np.array_equal(ids, oids)
    if vocab > 1:
        assert np.array_equal(scores, oscores)


def test_noisy_argmax_ties_and_extremes(cuda):
    # identical logits: only the noise decides; huge logits saturate the Q10 clamp.
    logits = np.zeros((8, 300), np.float32)
    logits[1, :] = 1e30
    logits[2, 7] = np.inf
    logits[3, :] = -np.inf
    ids, _ = _noisy(cuda, logits, 299)
    oids, _ = pyoracle.noisy_argmax_f32(logits, 299)
    assert np.array_equal(ids, oids)


def test_greedy_argmax_lowest_id_on_ties(cuda):
    logits = np.zeros((4, 100), np.float32)
    logits[0, [5, 9, 40]] = 2.0
    logits[1, 0] = 5.0  # masked below
    logits[2] = np.linspace(-1, 1, 100)
    logits[3, [98, 99]] = 3.0
    ids, _ = _noisy(cuda, logits, 0, greedy=True)
    assert ids.tolist() == pyoracle.greedy_argmax_f32(logits, 0).tolist()
    assert ids[0] == 5 and ids[1] == 1 and ids[3] == 98


def test_candidate_reveal_matches_reference(cuda):
    torch = cuda
    for name, c in load_npz_cases("reveal_golden.npz").items():
        P = int(c["positions"])
        nw = (P + 63) // 64
        t = _dev(torch, c["tokens"][:P].view(np.int16))
        cand = _dev(torch, c["cands"][:P].view(np.int16))
        a = _dev(torch, c["active"][:nw].view(np.int64))
        v = _dev(torch, c["valid"][:nw].view(np.int64))
        w = _dev(torch, c["words"][:P].view(np.int32))
        res = torch.zeros(1, dtype=torch.int64, device="cuda")
        _lib.call("dh_candidate_reveal", _lib.ptr(t), _lib.ptr(cand), _lib.ptr(a), _lib.ptr(v),
                  _lib.ptr(w), int(c["thr"]), P, 1, _lib.ptr(res), None)
        torch.cuda.synchronize()
        assert int(res.item()) == int(c["result"]), name
        assert np.array_equal(t.cpu().numpy().view(np.uint16), c["tokens_out"][:P]), name
        assert np.array_equal(a.cpu().numpy().view(np.uint64), c["active_out"][:nw]), name
        assert np.array_equal(v.cpu().numpy().view(np.uint64), c["valid_out"][:nw]), name


def test_candidate_reveal_batched_sequences_are_independent(cuda):
    torch = cuda
    rng = np.random.default_rng(3)
    S, P = 37, 1024
    nw = P // 64
    tokens = np.full((S, P), 50257, np.uint16)
    cands = rng.integers(0, 50257, (S, P)).astype(np.uint16)
    act = rng.integers(0, 1 << 63, (S, nw), dtype=np.int64).astype(np.uint64) * np.uint64(2) + np.uint64(1)
    val = np.full((S, nw), np.uint64(0xFFFFFFFFFFFFFFFF))
    val[5] = 0  # a sequence with an empty cache never reveals
    words = rng.integers(0, 1 << 32, (S, P), dtype=np.uint64).astype(np.uint32)
    thr = 1 << 27
    exp = []
    et, ea, ev = tokens.copy(), act.copy(), val.copy()
    for s in range(S):
        exp.append(pyoracle.candidate_reveal(et[s], cands[s], ea[s], ev[s], words[s], thr, P))
    t, cd = _dev(torch, tokens.view(np.int16)), _dev(torch, cands.view(np.int16))
    a, v = _dev(torch, act.view(np.int64)), _dev(torch, val.view(np.int64))
    w = _dev(torch, words.view(np.int32))
    res = torch.zeros(S, dtype=torch.int64, device="cuda")
    _lib.call("dh_candidate_reveal", _lib.ptr(t), _lib.ptr(cd), _lib.ptr(a), _lib.ptr(v), _lib.ptr(w),
              thr, P, S, _lib.ptr(res), None)
    torch.cuda.synchronize()
    assert res.cpu().numpy().tolist() == exp
    assert np.array_equal(t.cpu().numpy().view(np.uint16), et)
    assert np.array_equal(a.cpu().numpy().view(np.uint64), ea)
    assert np.array_equal(v.cpu().numpy().view(np.uint64), ev)


def _config1_logits(steps, positions, vocab, seed=0):
    import torch

    g = torch.Generator().manual_seed(seed)
    return np.stack([(3 * torch.randn((positions, vocab), generator=g)).numpy() for _ in range(steps + 1)])


@pytest.mark.parametrize("positions,vocab,steps", [(64, 50258, 64), (128, 1000, 16)])
def test_candidate_cache_loop_bit_exact_per_step(cuda, positions, vocab, steps):
    """Standalone sampler (64 x 50258, 64 transitions): per-step tokens,
    candidates and bitmaps equal the oracle's bit for bit."""
    torch = cuda
    mask = vocab - 1
    blocks = _config1_logits(steps, positions, vocab)
    thr = reveal_thresholds_q32(steps)
    ids0 = np.full(positions, mask, np.int32)
    o = pyoracle.candidate_cache_sampler_f32(blocks, ids0, mask, np.array(thr, np.uint64), seed=0)
    dev_blocks = torch.from_numpy(blocks).cuda()
    snaps = []

    def snapshot(k, st: CandidateCacheState):
        snaps.append((st.tokens.cpu().numpy().copy(), st.candidates.cpu().numpy().view(np.uint16).copy(),
                      st.active.cpu().numpy().view(np.uint64).copy(),
                      st.valid.cpu().numpy().view(np.uint64).copy()))

    ids, _, meta = run_candidate_cache_sampler_f32(
        lambda tokens, k: dev_blocks[k], torch.from_numpy(ids0).view(1, positions), mask_token_id=mask,
        steps=steps, seed=0, vocabulary_size=vocab, snapshot=snapshot)
    n = o["transitions"]
    for k in range(n):
        t, c, a, v = snaps[k]
        assert np.array_equal(t, o["snap_tokens"][k]), k
        assert np.array_equal(c.astype(np.int32), o["snap_candidates"][k]), k
        assert np.array_equal(a, o["snap_active"][k]), k
        assert np.array_equal(v, o["snap_valid"][k]), k
    assert np.array_equal(ids.cpu().numpy().ravel(), o["tokens"])
    assert meta["sampling_transitions"] == n
    assert meta["transition_active_tokens"] == o["step_active"][:n].tolist()
    assert meta["transition_changed_tokens"] == o["step_changed"][:n].tolist()
    assert meta["model_evaluations"] == o["evaluations"]
    assert mask not in ids.cpu().numpy().tolist()
    assert meta["hardware_candidate_cache_bytes"] == positions * 2 + 2 * (positions // 8)


@pytest.mark.parametrize("rows,vocab,mask", [(64, 50258, 50257), (3, 19, 18), (2, 1, 0), (300, 1000, 3),
                                             (7, 513, 512), (5, 1024, 0)])
def test_noise_only_argmax_is_the_race_over_zero_logits(cuda, rows, vocab, mask):
    """dh_noise_argmax: the head's noise race with every logit zero equals
    the oracle's noisy argmax of an all-zero logit matrix, ids and scores."""
    torch = cuda
    rng = np.random.default_rng(rows + vocab)
    pos = rng.integers(0, 1024, rows)
    khi = rng.integers(0, 512, rows)
    ev = rng.integers(0, 64, rows)
    zeros = np.zeros((rows, vocab), np.float32)
    oids, oscores = pyoracle.noisy_argmax_f32(zeros, mask, pos, khi, ev, key_lo=11, stream_id=2)
    arr = lambda a: _dev(torch, np.asarray(a, np.uint32).view(np.int32))  # noqa: E731
    packed = torch.zeros(rows, dtype=torch.int64, device="cuda")
    ids = torch.full((rows,), -1, dtype=torch.int32, device="cuda")
    p_, k_, e_ = arr(pos), arr(khi), arr(ev)
    _lib.call("dh_noise_argmax", rows, vocab, mask, _lib.ptr(p_), _lib.ptr(k_), _lib.ptr(e_), 0, 0, 11, 2,
              _lib.ptr(packed), _lib.ptr(ids), None)
    torch.cuda.synchronize()
    assert np.array_equal(ids.cpu().numpy(), oids)
    if vocab > 1:
        got = packed.cpu().numpy().view(np.uint64)
        score = ((got >> np.uint64(32)).astype(np.uint32) ^ np.uint32(0x80000000)).view(np.int32)
        assert np.array_equal(score, oscores)
    # constant key / evaluation instead of per-row arrays
    packed.zero_()
    _lib.call("dh_noise_argmax", rows, vocab, mask, None, None, None, 9, 5, 11, 2, _lib.ptr(packed),
              _lib.ptr(ids), None)
    torch.cuda.synchronize()
    cids, _ = pyoracle.noisy_argmax_f32(zeros, mask, None, np.full(rows, 5), np.full(rows, 9), key_lo=11,
                                        stream_id=2)
    assert np.array_equal(ids.cpu().numpy(), cids)
