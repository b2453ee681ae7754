"""The per-token int8 quantiser of the W8A8 linears (K3 / K3') against the
reference's fixed_mlp._quantize_symmetric (fixed_mlp.py:11-35), whose
outputs on seeded rows are the golden fixture tests/golden/quant_golden.npz
(made by tests/golden/make_quant_golden.py).

Bars: dh_quant_rows_bf16 is bit-exact -- the same int8 bytes and the same
fp32 row scales -- because it divides exactly as the reference does.
dh_ln_smooth_quant adds the LayerNorm, whose fp32 mean and variance the GPU
sums in another order than the CPU: its int8 bytes may differ by one step
where the normalised value lies within rounding of a half-integer quotient
(at most 0.2% of the bytes here), and its row scales by a few ulps.
"""

import sys

import numpy as np
import pytest

from conftest import GOLDEN, load_npz_cases
from diffusionhard_b200 import _lib
from oracle import model_oracle

sys.path.insert(0, str(GOLDEN))
from make_quant_golden import quant_cases  # noqa: E402


def _cases():
    import torch

    gold = load_npz_cases("quant_golden.npz")
    return {name: (x, s, ln, gold[name]) for name, (x, s, ln) in quant_cases(torch).items()}


def test_oracle_quantiser_matches_reference_golden():
    import torch
    import torch.nn.functional as F

    for name, (x, s, ln, g) in _cases().items():
        a = F.layer_norm(x, [x.shape[1]]) if ln else x
        q, scale = model_oracle.quantize_rows(a, None if s is None else s.numpy())
        assert np.array_equal(q.numpy(), g["q"]), name
        assert np.array_equal(scale.numpy(), g["scale"]), name
    del torch


def _quant_rows(torch, x, s, with_reciprocal=True):
    rows, cols = x.shape
    xin = x.to(torch.bfloat16).cuda()
    sd = None if s is None else s.cuda()
    inv = None if s is None or not with_reciprocal else (1.0 / s).cuda()  # fp32 reciprocals, rounded
    q = torch.empty((rows, cols), dtype=torch.int8, device="cuda")
    sc = torch.empty(rows, dtype=torch.float32, device="cuda")
    _lib.call("dh_quant_rows_bf16", _lib.ptr(xin), _lib.ptr(sd), _lib.ptr(inv), _lib.ptr(q), _lib.ptr(sc), rows, cols,
              None, None)
    torch.cuda.synchronize()
    return q.cpu().numpy(), sc.cpu().numpy()


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["bf16_768", "bf16_768_smooth", "bf16_3072", "bf16_3072_smooth", "edge_768"])
@pytest.mark.parametrize("with_reciprocal", [True, False])
def test_quant_rows_bit_exact(cuda, name, with_reciprocal):
    torch = cuda
    x, s, _, g = _cases()[name]
    q, sc = _quant_rows(torch, x, s, with_reciprocal)
    assert np.array_equal(q, g["q"]), name
    assert np.array_equal(sc, g["scale"]), name
    oq, osc = model_oracle.quantize_rows(x, None if s is None else s.numpy())
    assert np.array_equal(q, oq.numpy()) and np.array_equal(sc, osc.numpy())


@pytest.mark.gpu
@pytest.mark.parametrize("cols", [768, 3072])
def test_quant_rows_bit_exact_on_many_rows(cuda, cols):
    """4,096 rows over 2^-20 .. 2^20 magnitudes (12.6 M quotients at 3,072
    columns): the corrected-reciprocal division equals the CPU oracle's IEEE
    division everywhere."""
    torch = cuda
    g = torch.Generator().manual_seed(cols)
    rows = 4096
    mag = 2.0 ** (torch.randint(-20, 21, (rows, 1), generator=g).float())
    x = (torch.randn((rows, cols), generator=g) * mag).to(torch.bfloat16).float()
    s = torch.rand(cols, generator=g) * 9.9 + 0.1
    for smooth in (None, s):
        q, sc = _quant_rows(torch, x, smooth)
        oq, osc = model_oracle.quantize_rows(x, None if smooth is None else smooth.numpy())
        assert np.array_equal(sc, osc.numpy())
        assert np.array_equal(q, oq.numpy())


@pytest.mark.gpu
def test_ln_smooth_quant_matches_reference(cuda):
    torch = cuda
    x, s, _, g = _cases()["ln_768"]
    rows = x.shape[0]
    xd, sd, inv = x.cuda(), s.cuda(), (1.0 / s).cuda()
    q = torch.empty((rows, 768), dtype=torch.int8, device="cuda")
    sc = torch.empty(rows, dtype=torch.float32, device="cuda")
    _lib.call("dh_ln_smooth_quant", _lib.ptr(xd), _lib.ptr(sd), _lib.ptr(inv), _lib.ptr(q), _lib.ptr(sc), rows, None,
              None, None, None)
    torch.cuda.synchronize()
    gq = q.cpu().numpy().astype(np.int32)
    diff = np.abs(gq - g["q"].astype(np.int32))
    assert diff.max() <= 1
    assert (diff == 0).mean() >= 0.998
    assert np.allclose(sc.cpu().numpy(), g["scale"], rtol=4e-6, atol=0)


@pytest.mark.gpu
@pytest.mark.parametrize("m", [4096, 1000])
def test_gelu_row_amax_and_single_pass_quantiser(cuda, m):
    """dh_gemm_gelu merges each row's max |out| into row_amax (the bits of
    the max over the stored bf16 values); dh_quant_rows_bf16_amax then gives
    the same bytes and scales as the two-pass dh_quant_rows_bf16 and clears
    the words for the next launch.  m = 4,096 gives every persistent CTA
    several tiles; 1,000 ends in a ragged tile."""
    torch = cuda
    g = torch.Generator(device="cuda").manual_seed(m)
    n, k = 3072, 768
    a = torch.randint(-127, 128, (m, k), dtype=torch.int8, device="cuda", generator=g)
    w = torch.randint(-127, 128, (n, k), dtype=torch.int8, device="cuda", generator=g)
    a_scale = torch.rand(m, device="cuda", generator=g) * 1e-3 + 1e-4
    w_scale = torch.rand(n, device="cuda", generator=g) * 1e-3 + 1e-4
    bias = torch.randn(n, device="cuda", generator=g) * 0.1
    out_scale = torch.rand(n, device="cuda", generator=g) + 0.5
    mlp = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")
    amax = torch.zeros(m, dtype=torch.int32, device="cuda")
    _lib.call("dh_gemm_gelu", _lib.ptr(a), _lib.ptr(a_scale), _lib.ptr(w), _lib.ptr(w_scale), _lib.ptr(bias),
              _lib.ptr(out_scale), _lib.ptr(mlp), _lib.ptr(amax), m, n, k, None, None)
    torch.cuda.synchronize()
    expect = mlp.float().abs().amax(dim=1)
    assert torch.equal(amax.view(torch.float32), expect)
    q1 = torch.empty((m, n), dtype=torch.int8, device="cuda")
    s1 = torch.empty(m, dtype=torch.float32, device="cuda")
    q2, s2 = torch.empty_like(q1), torch.empty_like(s1)
    _lib.call("dh_quant_rows_bf16", _lib.ptr(mlp), None, None, _lib.ptr(q1), _lib.ptr(s1), m, n, None, None)
    _lib.call("dh_quant_rows_bf16_amax", _lib.ptr(mlp), _lib.ptr(amax), _lib.ptr(q2), _lib.ptr(s2), m, n, None,
              None)
    torch.cuda.synchronize()
    assert torch.equal(q1, q2) and torch.equal(s1, s2)
    assert int(amax.abs().sum()) == 0


@pytest.mark.gpu
@pytest.mark.parametrize("row_bytes", [16, 1536, 3072, 12288])
def test_gather_rows_copies_the_listed_rows(cuda, row_bytes):
    """dh_gather_rows / dh_gather_rows_i8: dst row i = src row rows_index[i]
    for i < min(rows, *rows_count), nothing past the count."""
    torch = cuda
    from diffusionhard_b200 import _lib

    rows = 300
    g = torch.Generator().manual_seed(row_bytes)
    src = torch.randint(0, 256, (rows, row_bytes), generator=g, dtype=torch.uint8).cuda()
    index = torch.randperm(rows, generator=g)[:200].to(torch.int32).cuda()
    count = torch.tensor([173], dtype=torch.int32, device="cuda")
    dst = torch.full((rows, row_bytes), 7, dtype=torch.uint8, device="cuda")
    _lib.call("dh_gather_rows", _lib.ptr(src), row_bytes, _lib.ptr(index), _lib.ptr(count), 200, _lib.ptr(dst), None)
    torch.cuda.synchronize()
    assert torch.equal(dst[:173], src[index[:173].long()])
    assert bool((dst[173:] == 7).all())
    if row_bytes == 16:
        assert _lib.raw("dh_gather_rows", _lib.ptr(src), 8, _lib.ptr(index), _lib.ptr(count), 200, _lib.ptr(dst),
                        None) == 105
        assert _lib.raw("dh_gather_rows", None, 16, _lib.ptr(index), _lib.ptr(count), 200, _lib.ptr(dst), None) == 100
    # the int8 head-input form carries each row's scale along
    if row_bytes == 1536:
        q = torch.randint(-127, 128, (rows, 768), generator=g, dtype=torch.int8).cuda()
        sc = torch.rand(rows, generator=g).cuda()
        dq = torch.zeros((rows, 768), dtype=torch.int8, device="cuda")
        ds = torch.zeros(rows, device="cuda")
        _lib.call("dh_gather_rows_i8", _lib.ptr(q), _lib.ptr(sc), _lib.ptr(index), _lib.ptr(count), 200, _lib.ptr(dq),
                  _lib.ptr(ds), None)
        torch.cuda.synchronize()
        sel = index[:173].long()
        assert torch.equal(dq[:173], q[sel]) and torch.equal(ds[:173], sc[sel])
