"""The no-allocation entry point dh_noisy_argmax_f32_noalloc.

Some callers cannot allocate device memory: a plugin running inside a host
framework that owns every device allocation, or a serving path that must not
call cudaMalloc (which can synchronise the whole device) once it is running.
For them the Gumbel-max kernel keeps its scratch in an array inside the
library.  This test calls it through the C ABI and checks it against the
workspace entry point dh_noisy_argmax_f32, bit for bit (argmax ids and scores
are exact), on two calls in a row: the second call runs on the scratch the
first one left behind.
"""

import numpy as np
import pytest

from diffusionhard_b200 import _lib

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


def test_noalloc_rejects_rows_beyond_the_scratch(cuda):
    # 5,042 rows x 13 chunks of the 50,258-token vocabulary exceed 65,536 slots
    assert _lib.raw("dh_noisy_argmax_f32_noalloc", 1, 50258, 5042, 50258, 50257, None, None, None, 0, 0, 1,
                    None, None) == 106
