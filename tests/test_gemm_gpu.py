"""tcgen05 int8 GEMM: int32 accumulators bit-exact against the oracle
(fixed_mlp._integer_matmul / the HLS MAC tile contract)."""

import numpy as np
import pytest

from diffusionhard_b200 import _lib
from oracle import pyoracle

pytestmark = pytest.mark.gpu


def _gemm(torch, a, w):
    m, k = a.shape
    n = w.shape[0]
    lda = (k + 15) // 16 * 16
    A = torch.zeros((m, lda), dtype=torch.int8, device="cuda")
    W = torch.zeros((n, lda), dtype=torch.int8, device="cuda")
    A[:, :k] = torch.from_numpy(a).cuda()
    W[:, :k] = torch.from_numpy(w).cuda()
    C = torch.full((m, n), -7, dtype=torch.int32, device="cuda")
    _lib.call("dh_gemm_i8_s32", _lib.ptr(A), lda, _lib.ptr(W), lda, _lib.ptr(C), n, m, n, k, None)
    torch.cuda.synchronize()
    err = np.zeros(1, np.uint32)
    _lib.call("dh_device_error", err.ctypes.data, 1)
    assert err[0] == 0
    return C.cpu().numpy()


def _ref(a, w):
    return (a.astype(np.float64) @ w.astype(np.float64).T).astype(np.int64).astype(np.int32)


@pytest.mark.parametrize("m,n,k", [(128, 256, 128), (256, 512, 768), (1, 1, 16), (129, 257, 144),
                                   (300, 1000, 768), (1000, 2304, 768), (777, 768, 3072)])
def test_gemm_i8_accumulators_bit_exact(cuda, m, n, k):
    rng = np.random.default_rng(m * 31 + n * 7 + k)
    a = rng.integers(-127, 128, (m, k)).astype(np.int8)
    w = rng.integers(-127, 128, (n, k)).astype(np.int8)
    got = _gemm(cuda, a, w)
    exp = _ref(a, w) if m * n * k > 4_000_000 else pyoracle.gemm_i8(a, w)
    assert np.array_equal(got, exp)


def test_gemm_i8_extreme_values(cuda):
    # all -128 / 127 saturating patterns: accumulator range of K=3072 stays in int32
    m, n, k = 256, 256, 3072
    a = np.full((m, k), -128, np.int8)
    w = np.full((n, k), -128, np.int8)
    a[::2] = 127
    got = _gemm(cuda, a, w)
    assert np.array_equal(got, _ref(a, w))


@pytest.mark.parametrize("k", [768, 3072])
def test_residual_narrow_tiles_match_wide_tiles(cuda, k):
    """dh_gemm_residual takes 128 x 64 tiles when they fit one wave of the
    SMs (a forward of one sequence), 128 x 192 otherwise: the same rows give
    the same bits either way (here 1,000 rows alone, and as the live rows of
    an 8,192-row launch)."""
    torch = cuda
    g = torch.Generator().manual_seed(k)
    m, big = 1000, 8192
    a = torch.randint(-127, 128, (big, k), generator=g, dtype=torch.int8).cuda()
    a_scale = (torch.rand(big, generator=g) * 1e-2 + 1e-3).cuda()
    w = torch.randint(-127, 128, (768, k), generator=g, dtype=torch.int8).cuda()
    w_scale = (torch.rand(768, generator=g) * 1e-3 + 1e-4).cuda()
    bias = (torch.randn(768, generator=g) * 0.02).cuda()
    x0 = torch.randn((big, 768), generator=g).cuda()
    p = _lib.ptr
    narrow = x0.clone()
    _lib.call("dh_gemm_residual", p(a), p(a_scale), p(w), p(w_scale), p(bias), p(narrow), m, 768, k, None, None)
    wide = x0.clone()
    live = torch.tensor([m], dtype=torch.int32, device="cuda")
    _lib.call("dh_gemm_residual", p(a), p(a_scale), p(w), p(w_scale), p(bias), p(wide), big, 768, k, p(live), None)
    torch.cuda.synchronize()
    assert torch.equal(narrow[:m], wide[:m])
    assert torch.equal(narrow[m:], x0[m:]) and torch.equal(wide[m:], x0[m:])
    # and the values are the dequantised products plus the residual
    acc = (a[:m].double() @ w.double().T)
    ref = x0[:m].double() + acc * (a_scale[:m].double()[:, None] * w_scale.double()[None, :]) + bias.double()
    assert float((narrow[:m].double() - ref).abs().max()) < 1e-3
    err = np.zeros(1, np.uint32)
    _lib.call("dh_device_error", err.ctypes.data, 1)
    assert err[0] == 0


@pytest.mark.parametrize("m", [1000, 64])
def test_gelu_narrow_tiles_match_wide_tiles(cuda, m):
    """dh_gemm_gelu takes 128 x 128 tiles when every CTA then holds at most
    one tile per epilogue group (one 1,024-token sequence, or a 64-token
    canvas), 128 x 256 otherwise: the same rows give the same bf16 outputs
    and row maxima either way (the rows alone, and as the live rows of an
    8,192-row launch)."""
    torch = cuda
    g = torch.Generator().manual_seed(m)
    big, n, k = 8192, 3072, 768
    a = torch.randint(-127, 128, (big, k), generator=g, dtype=torch.int8).cuda()
    a_scale = (torch.rand(big, generator=g) * 1e-3 + 1e-4).cuda()
    w = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8).cuda()
    w_scale = (torch.rand(n, generator=g) * 1e-3 + 1e-4).cuda()
    bias = (torch.randn(n, generator=g) * 0.1).cuda()
    out_scale = (torch.rand(n, generator=g) + 0.5).cuda()
    p = _lib.ptr
    outs = []
    for rows, live in ((m, None), (big, torch.tensor([m], dtype=torch.int32, device="cuda"))):
        out = torch.full((big, n), 3.0, dtype=torch.bfloat16, device="cuda")
        amax = torch.zeros(big, dtype=torch.int32, device="cuda")
        _lib.call("dh_gemm_gelu", p(a), p(a_scale), p(w), p(w_scale), p(bias), p(out_scale), p(out), p(amax), rows,
                  n, k, p(live), None)
        torch.cuda.synchronize()
        assert bool((out[m:] == 3.0).all()) and int(amax[m:].abs().sum()) == 0
        outs.append((out[:m].clone(), amax[:m].clone()))
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])
    assert torch.equal(outs[0][1].view(torch.float32), outs[0][0].float().abs().amax(dim=1))
    # and the values are bias + dequantised products through GELU(tanh), times out_scale
    x = (a[:m].double() @ w.double().T) * (a_scale[:m].double()[:, None] * w_scale.double()[None, :]) + bias.double()
    ref = 0.5 * x * (1 + torch.tanh(0.7978845608028654 * (x + 0.044715 * x ** 3))) * out_scale.double()
    assert float(((outs[0][0].double() - ref).norm() / ref.norm())) < 1e-2
    err = np.zeros(1, np.uint32)
    _lib.call("dh_device_error", err.ctypes.data, 1)
    assert err[0] == 0


def test_qkv_narrow_tiles_match_wide_tiles(cuda):
    """dh_gemm_qkv_rope takes 128 x 128 tiles when they fit one wave (one
    1,024-token sequence), 128 x 256 otherwise: q, k and V^T of the same
    rows are the same bits either way (one sequence alone, and as the live
    rows of an eight-sequence launch)."""
    torch = cuda
    from diffusionhard_b200.model import MDLMConfig, build_quantized
    from diffusionhard_b200.engine import MDLMEngine

    qm = build_quantized(MDLMConfig(vocab_size=1000, mask_token_id=999, blocks=1), seed=0)
    L = 1024
    g = torch.Generator().manual_seed(3)
    a_all = torch.randint(-127, 128, (8 * L, 768), generator=g, dtype=torch.int8)
    s_all = torch.rand(8 * L, generator=g) * 1e-2 + 1e-3
    outs = []
    for B in (1, 8):
        eng = MDLMEngine(qm, B, L)
        # the GEMM reads the activations as [rows, 768], row after row
        eng.act_q.view(-1)[: B * L * 768].view(B * L, 768).copy_(a_all[: B * L])
        eng.act_scale.copy_(s_all[: B * L])
        qkv, out = eng.blocks[0]["qkv"], eng.blocks[0]["out"]
        k, vt = eng.kv_buffers[0]
        live = torch.tensor([L], dtype=torch.int32, device="cuda")
        p = _lib.ptr
        _lib.call("dh_gemm_qkv_rope", p(eng.act_q), p(eng.act_scale), p(qkv.w), p(qkv.w_scale), p(qkv.bias),
                  p(eng.rope_cos), p(eng.rope_sin), p(out.inv_smooth), B * L, L, 0, eng.kv_stride, 0, p(eng.q), p(k),
                  p(vt), p(live) if B > 1 else None, None)
        torch.cuda.synchronize()
        outs.append((eng.q[0].clone(), k[0].clone(), vt[0].clone()))
    for a, b in zip(*outs):
        assert torch.equal(a, b)
    err = np.zeros(1, np.uint32)
    _lib.call("dh_device_error", err.ctypes.data, 1)
    assert err[0] == 0
