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
