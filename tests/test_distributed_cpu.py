"""N > 1 host logic on CPU ranks (gloo, world size 2): batch shards, vocab
shards, and the packed (score, ~id) MAX all-reduce of the vocab-sharded head.
No GPU: per-shard results come from the oracle."""

import os
import socket

import numpy as np
import pytest

from diffusionhard_b200.distributed import decode_packed, shard_batch, vocab_shards


def test_shard_batch_covers_the_batch():
    for gb in (1, 7, 32, 512):
        for world in (1, 2, 3, 8):
            parts = [shard_batch(gb, world, r) for r in range(world)]
            assert sum(c for _, c in parts) == gb
            assert [o for o, _ in parts] == [sum(c for _, c in parts[:r]) for r in range(world)]


def test_vocab_shards_align_to_philox_groups():
    for world in (1, 2, 4, 8):
        sh = vocab_shards(50258, world)
        assert sh[0][0] == 0 and sh[-1][1] == 50258
        assert all(a % 256 == 0 for a, _ in sh)
        assert all(sh[i][1] == sh[i + 1][0] for i in range(world - 1))


def _pack(score, tid):
    return ((score ^ 0x80000000) & 0xFFFFFFFF) << 32 | (0xFFFFFFFF - tid)


def _as_i64(u):
    return u - (1 << 64) if u >= 1 << 63 else u


def test_decode_packed_roundtrip():
    import torch

    vals = [(-5, 3), (0, 0), (23423, 50256), (-(2 ** 30), 7)]
    p = torch.tensor([_as_i64(_pack(s & 0xFFFFFFFF, t)) for s, t in vals], dtype=torch.int64)
    ids, scores = decode_packed(p)
    assert ids.tolist() == [t for _, t in vals]
    assert scores.tolist() == [s for s, _ in vals]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, scores, shards, out):
    import torch
    import torch.distributed as dist

    from diffusionhard_b200.distributed import all_reduce_packed_max_

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        v0, v1 = shards[rank]
        rows = scores.shape[0]
        packed = []
        for r in range(rows):
            best = 0
            for t in range(v0, v1):
                best = max(best, _pack(int(scores[r, t]) & 0xFFFFFFFF, t))
            packed.append(_as_i64(best))
        t = torch.tensor(packed, dtype=torch.int64)
        all_reduce_packed_max_(t)
        out[rank] = t.tolist()
    finally:
        dist.destroy_process_group()


def test_vocab_sharded_packed_max_matches_unsharded_argmax():
    import torch.multiprocessing as mp

    rng = np.random.default_rng(0)
    rows, vocab = 6, 600
    scores = rng.integers(-3000, 3000, (rows, vocab))
    scores[1, 100] = scores[1, 400] = 10 ** 6  # tie across shards -> lowest id
    scores[2, :] = 5                             # all equal -> id 0
    shards = vocab_shards(vocab, 2)
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    out = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, scores, shards, out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    import torch

    for r in range(2):
        ids, sc = decode_packed(torch.tensor(out[r], dtype=torch.int64))
        exp = [int(np.argmax(scores[i])) for i in range(rows)]
        assert ids.tolist() == exp
        assert sc.tolist() == [int(scores[i].max()) for i in range(rows)]
    assert out[0] == out[1]
