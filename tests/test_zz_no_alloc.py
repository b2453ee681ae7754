"""The no-allocation entry point dh_noisy_argmax_f32_noalloc.

Some callers cannot allocate device memory: a plugin running inside a host
framework that owns every device allocation, or a serving path that must not
call cudaMalloc (which can synchronise the whole device) once it is running.
For them the Gumbel-max kernel keeps its scratch in an array inside the
library.  This test calls it through the C ABI and checks it against the
workspace entry point dh_noisy_argmax_f32 and against the CPU oracle, bit for
bit (argmax ids and scores are exact), on two calls in a row: the second call
runs on the scratch the first one left behind.  It also runs the largest row
count the scratch accepts.
"""

import numpy as np
import pytest

from diffusionhard_b200 import _lib
from oracle import pyoracle

pytestmark = pytest.mark.gpu


def _call(torch, noalloc, logits, rows, vocab, mask, pos, key, ev, key_lo):
    ids = torch.full((rows,), -1, dtype=torch.int32, device="cuda")
    scores = torch.zeros(rows, dtype=torch.int32, device="cuda")
    if noalloc:
        _lib.call("dh_noisy_argmax_f32_noalloc", _lib.ptr(logits), vocab, rows, vocab, mask, _lib.ptr(pos),
                  _lib.ptr(key), _lib.ptr(ev), key_lo, 0, _lib.ptr(ids), _lib.ptr(scores), None)
    else:
        ws = torch.empty(_lib.lib().dh_noisy_argmax_workspace_size(rows, vocab), dtype=torch.uint8,
                         device="cuda")
        _lib.call("dh_noisy_argmax_f32", _lib.ptr(logits), vocab, rows, vocab, mask, _lib.ptr(pos),
                  _lib.ptr(key), _lib.ptr(ev), key_lo, 0, _lib.ptr(ids), _lib.ptr(scores), _lib.ptr(ws),
                  ws.numel(), None)
    torch.cuda.synchronize()
    return ids.cpu().numpy(), scores.cpu().numpy()


def test_noalloc_matches_workspace_entry_on_two_calls(cuda):
    torch = cuda
    for call, (rows, vocab) in enumerate([(64, 50258), (300, 1000)]):
        rng = np.random.default_rng(100 + call)
        logits = torch.from_numpy((3 * rng.standard_normal((rows, vocab))).astype(np.float32)).cuda()
        pos = torch.from_numpy(rng.integers(0, 1024, rows).astype(np.int32)).cuda()
        key = torch.from_numpy(rng.integers(0, 64, rows).astype(np.int32)).cuda()
        ev = torch.from_numpy(rng.integers(0, 64, rows).astype(np.int32)).cuda()
        mask = vocab - 1
        got = _call(torch, True, logits, rows, vocab, mask, pos, key, ev, 17)
        ref = _call(torch, False, logits, rows, vocab, mask, pos, key, ev, 17)
        assert np.array_equal(got[0], ref[0]), call
        assert np.array_equal(got[1], ref[1]), call
        assert (got[0] >= 0).all() and not (got[0] == mask).any()
        oids, oscores = pyoracle.noisy_argmax_f32(logits.cpu().numpy(), mask, row_position=pos.cpu().numpy(),
                                                  row_key_hi=key.cpu().numpy(), row_eval=ev.cpu().numpy(),
                                                  key_lo=17)
        assert np.array_equal(got[0], oids), call
        assert np.array_equal(got[1], oscores), call


def test_noalloc_accepts_the_largest_row_count(cuda):
    # 5,041 rows x 13 chunks of the 50,258-token vocabulary = 65,533 of the
    # 65,536 scratch slots; the oracle checks a sample of the rows
    torch = cuda
    rows, vocab = 5041, 50258
    g = torch.Generator(device="cuda").manual_seed(3)
    logits = 3 * torch.randn((rows, vocab), device="cuda", generator=g)
    pos = torch.arange(rows, dtype=torch.int32, device="cuda") % 1024
    key = torch.arange(rows, dtype=torch.int32, device="cuda") // 1024
    ev = torch.full((rows,), 5, dtype=torch.int32, device="cuda")
    got = _call(torch, True, logits, rows, vocab, vocab - 1, pos, key, ev, 4)
    ref = _call(torch, False, logits, rows, vocab, vocab - 1, pos, key, ev, 4)
    assert np.array_equal(got[0], ref[0]) and np.array_equal(got[1], ref[1])
    sample = np.r_[0:16, rows - 16:rows]
    oids, oscores = pyoracle.noisy_argmax_f32(logits[sample].cpu().numpy(), vocab - 1,
                                              row_position=pos[sample].cpu().numpy(),
                                              row_key_hi=key[sample].cpu().numpy(),
                                              row_eval=ev[sample].cpu().numpy(), key_lo=4)
    assert np.array_equal(got[0][sample], oids) and np.array_equal(got[1][sample], oscores)


def test_noalloc_rejects_rows_beyond_the_scratch(cuda):
    # 5,042 rows x 13 chunks of the 50,258-token vocabulary exceed 65,536 slots
    assert _lib.raw("dh_noisy_argmax_f32_noalloc", 1, 50258, 5042, 50258, 50257, None, None, None, 0, 0, 1,
                    None, None) == 106
