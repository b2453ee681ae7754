"""GPU parity of the W8A8 DDiT forward, the fused head and the device loop.

Bars (from the path's contract): bit-exact for Philox words, int32
accumulators, argmax ids and candidate-cache state; within 1e-2 relative for
fp32/bf16 LayerNorm, softmax and dequantised activations.  The forward is
compared with the CPU oracle (the reference W8A8 arithmetic), the head and the
loop bookkeeping bit-exactly with the oracle given the GPU's own inputs
(teacher forcing), since the fp32 forward itself is only tolerance-exact.
"""

import numpy as np
import pytest

from diffusionhard_b200 import _lib
from diffusionhard_b200.engine import MDLMEngine
from diffusionhard_b200.model import MDLMConfig, build_quantized
from diffusionhard_b200.sampler import reveal_thresholds_q32
from oracle import model_oracle, pyoracle

pytestmark = pytest.mark.gpu

SMALL = MDLMConfig(vocab_size=1000, mask_token_id=999, blocks=2)


@pytest.fixture(scope="module")
def small_model():
    return build_quantized(SMALL, seed=0)


def _device_error():
    err = np.zeros(1, np.uint32)
    _lib.call("dh_device_error", err.ctypes.data, 1)
    return int(err[0])


def _ids(B, L, seed, mask_every=3, vocab=999):
    import torch

    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(0, vocab, (B, L), generator=g)
    ids[:, ::mask_every] = vocab
    return ids


@pytest.mark.parametrize("L", [256, 64, 96])
def test_forward_matches_oracle(cuda, small_model, L):
    torch = cuda
    qm = small_model
    B = 2
    eng = MDLMEngine(qm, B, L)
    ids = _ids(B, L, 3)
    eng.tokens.copy_(ids.view(-1).to(torch.int32))
    per_block = {}
    eng.forward(hook=lambda i: per_block.__setitem__(i, eng.x.clone()))
    hq, hs = eng.final_hidden_q()
    torch.cuda.synchronize()
    assert _device_error() == 0
    rec = {}
    model_oracle.forward(qm, ids.numpy(), record=rec)
    for i in range(SMALL.blocks):
        got = per_block[i].cpu().view(B, L, 768)
        ref = rec[f"x{i}"]
        assert ((got - ref).norm() / ref.norm()).item() < 1e-2, i
    gq = hq.cpu().numpy()
    oq = rec["head_q"].numpy()
    assert (gq == oq).mean() > 0.95
    assert np.abs(gq.astype(np.int32) - oq.astype(np.int32)).max() <= 1
    assert np.allclose(hs.cpu().numpy(), rec["head_scale"].numpy(), rtol=1e-2)


def _head(torch, hq, hs, qm, mode, pos=None, key=None, ev=None, key_lo=0):
    rows = hq.shape[0]
    wq = torch.from_numpy(qm.head.weight_q).cuda()
    ws = torch.from_numpy(qm.head.w_scale).cuda()
    bias = torch.from_numpy(qm.head.bias).cuda()
    packed = torch.zeros(rows, dtype=torch.int64, device="cuda")
    ids = torch.zeros(rows, dtype=torch.int32, device="cuda")
    sc = torch.zeros(rows, dtype=torch.int32, device="cuda")
    dev = lambda a: None if a is None else torch.from_numpy(np.asarray(a, np.int32)).cuda()  # noqa: E731
    p_, k_, e_ = dev(pos), dev(key), dev(ev)
    _lib.call("dh_head_argmax_i8", _lib.ptr(hq), 768, _lib.ptr(wq), 768, rows, None, 768,
              qm.config.vocab_size, 0, qm.config.mask_token_id, mode, _lib.ptr(hs), _lib.ptr(ws), _lib.ptr(bias),
              None, None, None, _lib.ptr(p_), _lib.ptr(k_), _lib.ptr(e_), 0, key_lo, 0, _lib.ptr(packed),
              _lib.ptr(ids), _lib.ptr(sc), None)
    torch.cuda.synchronize()
    return ids.cpu().numpy(), sc.cpu().numpy()


@pytest.mark.parametrize("vocab,rows", [(1000, 300), (50258, 129), (50258, 16), (50258, 32), (1000, 1),
                                       (1000, 33)])
def test_head_bit_exact(cuda, vocab, rows):
    """Up to 32 rows the head runs in its few-row mode (the rows loaded into
    all four lane quadrants, the columns split four ways); 33 and more rows
    take the one-row-per-thread path."""
    torch = cuda
    cfg = MDLMConfig(vocab_size=vocab, mask_token_id=vocab - 1, blocks=1)
    rng = np.random.default_rng(vocab)

    class Q:  # a head-only quantised model: int8 W ~ round(clip(N(0,40))), scales U(0.5e-3, 2e-3)
        pass

    qm = Q()
    qm.config = cfg
    qm.head = Q()
    qm.head.weight_q = np.clip(np.round(rng.normal(0, 40, (vocab, 768))), -127, 127).astype(np.int8)
    qm.head.w_scale = rng.uniform(0.5e-3, 2e-3, vocab).astype(np.float32)
    qm.head.bias = rng.normal(0, 0.02, vocab).astype(np.float32)
    h = rng.integers(-127, 128, (rows, 768)).astype(np.int8)
    a = rng.uniform(0.01, 0.05, rows).astype(np.float32)
    pos, key, ev = rng.integers(0, 1024, rows), rng.integers(0, 64, rows), rng.integers(0, 64, rows)
    hq, hs = torch.from_numpy(h).cuda(), torch.from_numpy(a).cuda()
    for mode in (1, 2):
        ids, sc = _head(torch, hq, hs, qm, mode, pos, key, ev, key_lo=7)
        oids, osc = pyoracle.head_i8(mode, h, qm.head.weight_q, cfg.mask_token_id, a_scale=a,
                                     w_scale=qm.head.w_scale, bias=qm.head.bias, row_position=pos,
                                     row_key_hi=key, row_eval=ev, key_lo=7)
        assert np.array_equal(ids, oids), mode
        assert np.array_equal(sc, osc), mode
    assert _device_error() == 0


def test_head_few_rows_by_device_count(cuda):
    """The few-row mode is chosen on the device: a launch over 300 host rows
    whose device row count is 20 gives the oracle's ids for those 20 rows and
    leaves the rest untouched."""
    torch = cuda
    vocab, rows, live = 50258, 300, 20
    rng = np.random.default_rng(5)
    w = np.clip(np.round(rng.normal(0, 40, (vocab, 768))), -127, 127).astype(np.int8)
    ws = rng.uniform(0.5e-3, 2e-3, vocab).astype(np.float32)
    bias = rng.normal(0, 0.02, vocab).astype(np.float32)
    h = rng.integers(-127, 128, (rows, 768)).astype(np.int8)
    a = rng.uniform(0.01, 0.05, rows).astype(np.float32)
    pos, key, ev = (rng.integers(0, 1024, rows).astype(np.int32), rng.integers(0, 64, rows).astype(np.int32),
                    rng.integers(0, 64, rows).astype(np.int32))
    dev = lambda x: torch.from_numpy(np.ascontiguousarray(x)).cuda()  # noqa: E731
    hq, hs, wq, wsd, bd, pd, kd, ed = map(dev, (h, a, w, ws, bias, pos, key, ev))
    count = torch.tensor([live], dtype=torch.int32, device="cuda")
    packed = torch.zeros(rows, dtype=torch.int64, device="cuda")
    ids = torch.full((rows,), -5, dtype=torch.int32, device="cuda")
    sc = torch.zeros(rows, dtype=torch.int32, device="cuda")
    p = _lib.ptr
    _lib.call("dh_head_argmax_i8", p(hq), 768, p(wq), 768, rows, p(count), 768, vocab, 0, vocab - 1, 1, p(hs),
              p(wsd), p(bd), None, None, None, p(pd), p(kd), p(ed), 0, 7, 0, p(packed), p(ids), p(sc), None)
    torch.cuda.synchronize()
    oids, osc = pyoracle.head_i8(1, h[:live], w, vocab - 1, a_scale=a[:live], w_scale=ws, bias=bias,
                                 row_position=pos[:live], row_key_hi=key[:live], row_eval=ev[:live], key_lo=7)
    got = ids.cpu().numpy()
    assert np.array_equal(got[:live], oids)
    assert np.array_equal(sc.cpu().numpy()[:live], osc)
    assert (got[live:] == -5).all()
    assert _device_error() == 0


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
def test_output_head_mirror_matches_reference(cuda, case):
    """dh_output_head_int8 against output_head_int8_kernel's own results
    (golden vectors made by the reference C++).  Hidden sizes below 16 are
    zero-padded, which leaves every accumulator unchanged."""
    torch = cuda
    from conftest import load_npz_cases

    c = load_npz_cases("head_golden.npz")[case]
    P, H = c["hidden"].shape
    V = c["weights"].shape[0]
    Hp = (H + 15) // 16 * 16
    hid = np.zeros((P, Hp), np.int8)
    hid[:, :H] = c["hidden"]
    w = np.zeros((V, Hp), np.int8)
    w[:, :H] = c["weights"]
    d = lambda a, t: torch.from_numpy(np.ascontiguousarray(a, t)).cuda()  # noqa: E731
    cand = torch.zeros(P, dtype=torch.int16, device="cuda")
    ws = torch.zeros(P, dtype=torch.int64, device="cuda")
    if "noise" in c:
        noise = d(c["noise"], np.int32)
        ev = st = lo = hi = 0
    else:
        noise = None
        ev, st, lo, hi = (int(x) for x in c["rng"])
    # keep every device buffer referenced until the asynchronous kernel has run
    hid_d, w_d, mult_d, bias_d = d(hid, np.int8), d(w, np.int8), d(c["mult"], np.int32), d(c["bias"], np.int32)
    _lib.call("dh_output_head_int8", _lib.ptr(hid_d), _lib.ptr(w_d), _lib.ptr(mult_d), _lib.ptr(bias_d),
              _lib.ptr(noise), _lib.ptr(cand), P, Hp, V, int(c["mask"]), ev, st, lo, hi, _lib.ptr(ws), None)
    torch.cuda.synchronize()
    assert cand.cpu().numpy().view(np.uint16).tolist() == c["ids"].tolist()


def test_output_head_mirror_status_codes():
    assert _lib.raw("dh_output_head_int8", None, None, None, None, None, None, 0, 16, 5, 0, 0, 0, 0, 0, None, None) == 1
    assert _lib.raw("dh_output_head_int8", None, None, None, None, None, None, 1, 769, 5, 0, 0, 0, 0, 0, None, None) == 2
    assert _lib.raw("dh_output_head_int8", None, None, None, None, None, None, 1, 16, 0, 0, 0, 0, 0, 0, None, None) == 3
    assert _lib.raw("dh_output_head_int8", None, None, None, None, None, None, 1, 16, 5, 5, 0, 0, 0, 0, None, None) == 4


def test_attention_matches_sdpa(cuda):
    torch = cuda
    import torch.nn.functional as F

    B, H, Lq, P = 2, 12, 256, 128
    kv_stride = P + Lq
    g = torch.Generator(device="cuda").manual_seed(0)
    q = torch.randn((B, H, Lq, 64), device="cuda", generator=g).to(torch.bfloat16)
    k = torch.randn((B, H, kv_stride, 64), device="cuda", generator=g).to(torch.bfloat16)
    vt = torch.randn((B, H, 64, kv_stride), device="cuda", generator=g).to(torch.float16)
    k[:, :, :P] *= 3  # a prefix with larger scores exercises the rescale path
    vt_dev = vt
    for kv_len in (Lq, kv_stride):
        out = torch.empty((B * Lq, 768), dtype=torch.bfloat16, device="cuda")
        _lib.call("dh_attention", _lib.ptr(q), _lib.ptr(k), _lib.ptr(vt_dev), _lib.ptr(out), B, Lq, kv_len,
                  kv_stride, None, None)
        torch.cuda.synchronize()
        ref = F.scaled_dot_product_attention(q.float(), k[:, :, :kv_len].float(),
                                             vt[:, :, :, :kv_len].float().transpose(-1, -2))
        got = out.float().view(B, Lq, H, 64).transpose(1, 2)
        assert ((got - ref).norm() / ref.norm()).item() < 1e-2, kv_len
    assert _device_error() == 0


@pytest.mark.parametrize("Lq,P", [(64, 0), (96, 0), (160, 0), (96, 32), (64, 96)])
def test_attention_ragged_lengths(cuda, Lq, P):
    """q_len / kv_len multiples of 32 but not of 128: keys past kv_len are
    masked (they are set huge here, so a leak would show), rows past q_len
    are not written (a guard region after the output stays untouched)."""
    torch = cuda
    import torch.nn.functional as F

    B, H = 3, 12
    kv_len = P + Lq
    kv_stride = ((kv_len + 127) // 128) * 128 + 32  # padding inside the stride
    g = torch.Generator(device="cuda").manual_seed(Lq + P)
    q = torch.randn((B, H, Lq, 64), device="cuda", generator=g).to(torch.bfloat16)
    k = torch.randn((B, H, kv_stride, 64), device="cuda", generator=g).to(torch.bfloat16)
    vt = torch.randn((B, H, 64, kv_stride), device="cuda", generator=g).to(torch.float16)
    k[:, :, kv_len:] = 50.0  # would dominate every softmax row if not masked
    vt[:, :, :, kv_len:] = 1000.0
    guard = 4096
    buf = torch.full((B * Lq * 768 + guard,), 7.0, dtype=torch.bfloat16, device="cuda")
    out = buf[: B * Lq * 768].view(B * Lq, 768)
    vt_dev = vt
    _lib.call("dh_attention", _lib.ptr(q), _lib.ptr(k), _lib.ptr(vt_dev), _lib.ptr(out), B, Lq, kv_len,
              kv_stride, None, None)
    torch.cuda.synchronize()
    ref = F.scaled_dot_product_attention(q.float(), k[:, :, :kv_len].float(),
                                         vt[:, :, :, :kv_len].float().transpose(-1, -2))
    got = out.float().view(B, Lq, H, 64).transpose(1, 2)
    assert ((got - ref).norm() / ref.norm()).item() < 1e-2
    assert bool((buf[B * Lq * 768:] == 7.0).all())
    assert _device_error() == 0
    assert _lib.raw("dh_attention", _lib.ptr(q), _lib.ptr(k), _lib.ptr(vt_dev), _lib.ptr(out), B, 48, kv_len,
                    kv_stride, None, None) == 103


@pytest.mark.parametrize("L", [256, 96])
def test_loop_teacher_forced_bit_exact(cuda, small_model, L):
    """Each transition: the revealed row set equals the oracle's reveal
    decision on the GPU's state, and every revealed row's candidate equals the
    oracle's noisy argmax on the GPU's own int8 hidden row."""
    torch = cuda
    qm = small_model
    B, steps, seed = 2, 12, 5
    eng = MDLMEngine(qm, B, L)
    eng.seq_offset = 3
    mask = SMALL.mask_token_id
    eng.init_loop(torch.full((B, L), mask, dtype=torch.int64, device="cuda"), steps)
    thr = reveal_thresholds_q32(steps)
    eval_of = np.zeros(B, np.int64)
    for k in range(steps + 1):
        tokens_before = eng.tokens.cpu().numpy().reshape(B, L)
        need_before = eng.need_eval.cpu().numpy()
        eng.enqueue_transition(k, steps, seed, thr[k] if k < steps else 0)
        torch.cuda.synchronize()
        n = int(eng.sel_count.item())
        rows = eng.sel_rows[:n].cpu().numpy()
        assert np.all(np.diff(rows.astype(np.int64)) > 0)  # deterministic position-major order
        active = tokens_before == mask
        if k < steps:
            for b in range(B):
                if need_before[b] and active[b].any():
                    eval_of[b] = k
            exp = set()
            for b in range(B):
                words = pyoracle.reveal_words(L, k, seed, 3 + b)
                for p in np.nonzero(active[b])[0]:
                    if int(words[p]) < thr[k]:
                        exp.add(b * L + int(p))
            assert set(rows.tolist()) == exp, k
        else:
            assert set(rows.tolist()) == {int(i) for i in np.nonzero(active.ravel())[0]}
        if n == 0:
            continue
        hq = eng.head_q[:n].cpu().numpy()
        hs = eng.head_scale[:n].cpu().numpy()
        got = eng.tokens.cpu().numpy()[rows]
        b_idx, p_idx = rows // L, rows % L
        mode = 2 if k == steps else 1
        oids, _ = pyoracle.head_i8(mode, hq, qm.head.weight_q, mask, a_scale=hs, w_scale=qm.head.w_scale,
                                   bias=qm.head.bias, row_position=p_idx, row_key_hi=3 + b_idx,
                                   row_eval=eval_of[b_idx], key_lo=seed)
        assert np.array_equal(got, oids), k
    assert not (eng.tokens.cpu().numpy() == mask).any()
    meta = eng.metadata(steps)
    assert meta["sampling_transitions"] == steps
    assert sum(meta["transition_changed_tokens"]) + (meta["transition_active_tokens"][-1]
                                                     - meta["transition_changed_tokens"][-1]) == B * L
    assert _device_error() == 0


def test_graph_replay_equals_eager_and_batch_split_invariant(cuda, small_model):
    torch = cuda
    qm = small_model
    mask = SMALL.mask_token_id
    full = MDLMEngine(qm, 4, 256)
    ids = torch.full((4, 256), mask, dtype=torch.int64, device="cuda")
    eager, _ = full.generate(ids, steps=10, seed=9, graph=False)
    eager = eager.clone()
    graph, _ = full.generate(ids, steps=10, seed=9, graph=True)
    assert torch.equal(eager, graph)
    half = MDLMEngine(qm, 2, 256)
    parts = []
    for off in (0, 2):
        half.seq_offset = off
        out, _ = half.generate(ids[:2], steps=10, seed=9, graph=False)
        parts.append(out.clone())
    assert torch.equal(torch.cat(parts), eager)


def test_prefix_cached_suffix_matches_oracle(cuda, small_model):
    """Prefix K/V computed once by an isolated prefix forward and reused by
    the suffix forward (prefix_drift._cached_suffix_forward)."""
    torch = cuda
    qm = small_model
    B, P, S = 2, 128, 256
    kv = MDLMEngine.kv_cache(qm, B, P + S)
    pre = MDLMEngine(qm, B, P, kv_len=P, kv_buffers=kv)
    suf = MDLMEngine(qm, B, S, pos_offset=P, kv_len=P + S, kv_offset=P, kv_buffers=kv)
    ids = _ids(B, P + S, 11)
    ids[:, :P] = torch.randint(0, 999, (B, P), generator=torch.Generator().manual_seed(2))
    pre.tokens.copy_(ids[:, :P].reshape(-1).to(torch.int32))
    pre.forward()
    suf.tokens.copy_(ids[:, P:].reshape(-1).to(torch.int32))
    suf.forward()
    hq, hs = suf.final_hidden_q()
    torch.cuda.synchronize()
    rec_p = {}
    model_oracle.forward(qm, ids[:, :P].numpy(), capture_kv=True, record=rec_p)
    rec_s = {}
    h = model_oracle.forward(qm, ids[:, P:].numpy(), positions=np.arange(P, P + S), prefix_kv=rec_p["kv"],
                             record=rec_s)
    assert (hq.cpu().numpy() == rec_s["head_q"].numpy()).mean() > 0.95
    got_x = suf.x.cpu().view(B, S, 768)
    ref_x = rec_s[f"x{SMALL.blocks - 1}"]
    assert ((got_x - ref_x).norm() / ref_x.norm()).item() < 1e-2
    del h
    assert _device_error() == 0


@pytest.mark.parametrize("rows", [257, 16])
def test_vocab_sharded_head_equals_unsharded(cuda, rows):
    """Head rows split into 4 slices (global ids via vocab_offset); the MAX of
    the packed words equals the unsharded head, ids and scores, both modes
    (16 rows: the few-row mode on every slice)."""
    torch = cuda
    from diffusionhard_b200.distributed import decode_packed, to_signed_, vocab_shards

    V, mask = 50258, 50257
    rng = np.random.default_rng(42)
    W = torch.from_numpy(np.clip(np.round(rng.normal(0, 40, (V, 768))), -127, 127).astype(np.int8)).cuda()
    ws = torch.from_numpy(rng.uniform(0.5e-3, 2e-3, V).astype(np.float32)).cuda()
    bias = torch.from_numpy(rng.normal(0, 0.02, V).astype(np.float32)).cuda()
    h = torch.from_numpy(rng.integers(-127, 128, (rows, 768)).astype(np.int8)).cuda()
    a = torch.from_numpy(rng.uniform(0.01, 0.05, rows).astype(np.float32)).cuda()
    pos = torch.from_numpy(rng.integers(0, 1024, rows).astype(np.int32)).cuda()

    def run(v0, v1, mode):
        packed = torch.zeros(rows, dtype=torch.int64, device="cuda")
        wsl, wss, bsl = W[v0:v1].contiguous(), ws[v0:v1].contiguous(), bias[v0:v1].contiguous()
        _lib.call("dh_head_argmax_i8", _lib.ptr(h), 768, _lib.ptr(wsl), 768, rows, None, 768, v1 - v0, v0, mask,
                  mode, _lib.ptr(a), _lib.ptr(wss), _lib.ptr(bsl), None, None, None, _lib.ptr(pos), None, None,
                  9, 3, 0, _lib.ptr(packed), None, None, None)
        torch.cuda.synchronize()
        return packed

    for mode in (1, 2):
        full = run(0, V, mode)
        merged = None
        for v0, v1 in vocab_shards(V, 4):
            part = to_signed_(run(v0, v1, mode))
            merged = part if merged is None else torch.maximum(merged, part)
        to_signed_(merged)
        assert torch.equal(merged, full), mode
        ids, _ = decode_packed(full)
        assert not (ids == mask).any()
    assert _device_error() == 0
