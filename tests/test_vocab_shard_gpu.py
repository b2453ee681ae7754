"""The vocab-sharded head on two GPUs: each rank holds half of the head rows,
the composite loop (dh_sample_loop) merges the per-row results with
dh_vocab_shard_reduce over NCCL after every head launch, and both ranks
commit the tokens of the unsharded head.  Needs two GPUs (skipped on one);
NVLS is off and every collective has a short timeout."""

import os
import socket

import pytest

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank: int, world: int, port: int, out_dir: str) -> None:
    import datetime

    import torch
    import torch.distributed as dist

    from diffusionhard_b200.distributed import vocab_shards
    from diffusionhard_b200.engine import MDLMEngine
    from diffusionhard_b200.model import MDLMConfig, build_quantized

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    try:
        cfg = MDLMConfig(vocab_size=1000, mask_token_id=999, blocks=2)
        qm = build_quantized(cfg, seed=0)
        L, steps = 256, 16
        ids = torch.full((1, L), cfg.mask_token_id, dtype=torch.int64, device="cuda")
        whole = MDLMEngine(qm, 1, L)
        ref, _ = whole.generate(ids, steps=steps, seed=3)
        ref = ref.clone()
        shard = MDLMEngine(qm, 1, L)
        v0, v1 = vocab_shards(cfg.vocab_size, world)[rank]
        shard.shard_head(v0, v1, group=dist.group.WORLD)
        assert shard.native_loop_ok()
        out, _ = shard.generate(ids, steps=steps, seed=3, graph=False)
        torch.cuda.synchronize()
        with open(os.path.join(out_dir, f"rank{rank}"), "w") as f:
            f.write("equal" if torch.equal(out, ref) else "differ")
    finally:
        dist.barrier()
        dist.destroy_process_group()


def test_sharded_head_over_nccl_equals_unsharded(cuda, tmp_path):
    torch = cuda
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    mp.start_processes(_rank, args=(2, _free_port(), str(tmp_path)), nprocs=2, start_method="spawn", join=True)
    assert [(tmp_path / f"rank{r}").read_text() for r in range(2)] == ["equal", "equal"]
