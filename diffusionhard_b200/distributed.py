"""Multi-GPU plumbing for the MDLM loop (torch.distributed; NCCL on GPUs).

* Batch sharding: sequences are independent, so rank r of N runs sequences
  [offset, offset + count) of the global batch with no collective on the hot
  path; the Philox key uses the global sequence index (engine.seq_offset), so
  the tokens do not depend on N.
* Vocab-sharded head (single-sequence latency): the backbone is replicated,
  each rank projects a contiguous slice of the 50,258 head rows, and the
  per-row packed (score, ~token id) words are MAX-reduced over ranks.  The
  packed word's order is unsigned; flipping its top bit makes it a signed
  int64 with the same order, which every backend reduces natively.  The tie
  rule (equal scores -> lowest id) survives the reduction because ~id is the
  low word (ordered_noisy_argmax_reducer.sv:106-133).
"""

from __future__ import annotations

from typing import Any, List, Tuple

SIGN_FLIP = -(1 << 63)  # int64 with only the top bit set


def shard_batch(global_batch: int, world: int, rank: int) -> Tuple[int, int]:
    """(offset, count) of rank's sequences; the first `global_batch % world`
    ranks take one extra sequence."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad world / rank")
    base, extra = divmod(global_batch, world)
    count = base + (1 if rank < extra else 0)
    offset = rank * base + min(rank, extra)
    return offset, count


def vocab_shards(vocab: int, world: int, align: int = 256) -> List[Tuple[int, int]]:
    """Contiguous head-row ranges, boundaries multiples of `align` (a
    multiple of 4 keeps every Philox group of 4 tokens inside one shard)."""
    if align % 4:
        raise ValueError("shard boundaries must be multiples of 4")
    per = -(-vocab // world)
    per = -(-per // align) * align
    out = []
    for r in range(world):
        v0 = min(r * per, vocab)
        v1 = min(v0 + per, vocab)
        out.append((v0, v1))
    return out


def to_signed_(packed: Any) -> Any:
    """In place: unsigned-ordered packed words -> signed-ordered (and back)."""
    packed.bitwise_xor_(SIGN_FLIP)
    return packed


def all_reduce_packed_max_(packed: Any, group: Any = None) -> Any:
    """In place: per-row (max score, lowest id) over all ranks."""
    import torch.distributed as dist

    to_signed_(packed)
    dist.all_reduce(packed, op=dist.ReduceOp.MAX, group=group)
    return to_signed_(packed)


def decode_packed(packed: Any) -> Tuple[Any, Any]:
    """(ids, integer scores) of unsigned-ordered packed words (int64 tensor)."""
    import torch

    low = packed & 0xFFFFFFFF
    ids = (0xFFFFFFFF - low).to(torch.int64)
    high = (packed >> 32) & 0xFFFFFFFF  # score + 2^31 (sign bit flipped)
    scores = high - (1 << 31)
    return ids, scores


def nccl_comm_handle(group: Any, device: Any) -> Any:
    """The ncclComm_t (as an int) behind a process group's NCCL backend on
    `device`, for dh_vocab_shard_reduce; None when the group has no NCCL
    backend (gloo, or a torch without the accessor).  A communicator that
    torch creates lazily is created by one collective, which every rank of
    the group takes at the same point."""
    import torch
    import torch.distributed as dist

    try:
        backend = group._get_backend(torch.device(device))
    except Exception:
        return None
    get = getattr(backend, "_comm_ptr", None)
    if get is None:
        return None
    ptr = int(get())
    if ptr == 0:
        t = torch.zeros(1, device=device)
        dist.all_reduce(t, group=group)
        torch.cuda.synchronize(device)
        ptr = int(get())
    return ptr or None
