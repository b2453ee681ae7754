"""The composite entry points dh_ddit_forward, dh_sample_loop and
dh_vocab_shard_reduce, called through the C ABI with no Python orchestration
of the kernels.

GPU: the forward equals the per-kernel forward bit for bit, and a whole
generation equals the one the per-kernel entry points produce when driven
from Python (engine.generate(native=False)) -- tokens and the per-transition
counters.  CPU: argument checks return their status before any GPU work.
"""

import ctypes

import numpy as np
import pytest

from diffusionhard_b200 import _lib
from diffusionhard_b200.model import MDLMConfig, build_quantized
from diffusionhard_b200.sampler import reveal_thresholds_q32

SMALL = MDLMConfig(vocab_size=1000, mask_token_id=999, blocks=2)


def test_composite_argument_checks_need_no_gpu():
    assert _lib.raw("dh_ddit_forward", None, 1, 1, 64, 1, 1, 1 << 20, None, None) == 100
    assert _lib.raw("dh_vocab_shard_reduce", None, 1, 1, None) == 100
    w = _lib.MDLMWeights()
    w.blocks = 0
    w.vocabulary_size = 1000
    w.mask_token_id = 999
    w.max_positions = 1024
    assert _lib.raw("dh_ddit_forward", ctypes.addressof(w), 1, 1, 64, 1, 1, 1 << 20, None, None) == 105
    w.blocks = 2
    assert _lib.raw("dh_ddit_forward", ctypes.addressof(w), 1, 1, 48, 1, 1, 1 << 20, None, None) == 103
    assert _lib.raw("dh_ddit_forward", ctypes.addressof(w), 1, 1, 64, 1, 1, 1 << 20, None, None) == 100
    thr = (ctypes.c_uint64 * 2)(1 << 31, (1 << 32) + 1)
    assert _lib.raw("dh_sample_loop", ctypes.addressof(w), 1, 1, 1, 64, 2, ctypes.addressof(thr), 0, 0, 1,
                    None, 0, 1, 1 << 20, None) == 100
    assert _lib.lib().dh_sample_loop_workspace_size(4, 1024) > _lib.lib().dh_ddit_forward_workspace_size(4, 1024)


def test_weight_struct_layout():
    # four uint32, three pointers, the block array pointer, the head's five
    # pointers, two uint32 (natural alignment, LP64)
    assert ctypes.sizeof(_lib.LinearWeights) == 40
    assert _lib.MDLMWeights.head.offset == 16 + 4 * 8
    assert ctypes.sizeof(_lib.MDLMWeights) == 16 + 32 + 40 + 8


@pytest.mark.gpu
def test_ddit_forward_equals_per_kernel_forward(cuda):
    torch = cuda
    from diffusionhard_b200.engine import MDLMEngine

    qm = build_quantized(SMALL, seed=0)
    B, L = 3, 256
    eng = MDLMEngine(qm, B, L)
    ids = torch.randint(0, 1000, (B * L,), generator=torch.Generator().manual_seed(4)).to(torch.int32).cuda()
    eng.tokens.copy_(ids)
    eng.forward()
    ref = eng.x.clone()
    x = torch.empty_like(ref)
    ws = torch.empty(_lib.lib().dh_ddit_forward_workspace_size(B, L), dtype=torch.uint8, device="cuda")
    w = eng.native_weights()
    _lib.call("dh_ddit_forward", ctypes.addressof(w), _lib.ptr(ids), B, L, _lib.ptr(x), _lib.ptr(ws), ws.numel(),
              None, _lib.stream_handle())
    torch.cuda.synchronize()
    assert torch.equal(x, ref)
    assert _lib.raw("dh_ddit_forward", ctypes.addressof(w), _lib.ptr(ids), B, L, _lib.ptr(x), _lib.ptr(ws),
                    ws.numel() - 1, None, None) == 102


@pytest.mark.gpu
@pytest.mark.parametrize("B,L,steps,compact", [(2, 256, 12, 0), (3, 96, 8, 0), (3, 96, 8, 1), (4, 64, 64, 1)])
def test_sample_loop_equals_per_kernel_loop(cuda, B, L, steps, compact):
    torch = cuda
    from diffusionhard_b200.engine import MDLMEngine

    qm = build_quantized(SMALL, seed=0)
    eng = MDLMEngine(qm, B, L)
    eng.seq_offset = 5
    ids = torch.full((B, L), SMALL.mask_token_id, dtype=torch.int64)
    ids[:, ::7] = 3  # a few clean positions
    eng.compact = False
    ref, _ = eng.generate(ids.cuda(), steps=steps, seed=11, native=False)
    ref = ref.clone()
    ref_counters = eng.counters.clone()
    # the composite entry point through ctypes, on fresh buffers
    w = eng.native_weights()
    ids_in = ids.reshape(-1).to(torch.int32).cuda()
    tokens = torch.empty(B * L, dtype=torch.int32, device="cuda")
    counters = torch.empty(3 * steps, dtype=torch.int32, device="cuda")
    ws = torch.empty(_lib.lib().dh_sample_loop_workspace_size(B, L), dtype=torch.uint8, device="cuda")
    thr = (ctypes.c_uint64 * steps)(*reveal_thresholds_q32(steps))
    _lib.call("dh_sample_loop", ctypes.addressof(w), _lib.ptr(ids_in), _lib.ptr(tokens), B, L, steps,
              ctypes.addressof(thr), 11, 5, _lib.ptr(counters), None, compact, _lib.ptr(ws), ws.numel(),
              _lib.stream_handle())
    torch.cuda.synchronize()
    assert torch.equal(tokens.view(B, L), ref)
    assert torch.equal(counters, ref_counters)
    assert not (tokens == SMALL.mask_token_id).any()
    # and engine.generate's default route (the composite) gives the same
    eng.compact = bool(compact)
    out, _ = eng.generate(ids.cuda(), steps=steps, seed=11, graph=True)
    assert torch.equal(out, ref)
    err = np.zeros(1, np.uint32)
    _lib.call("dh_device_error", err.ctypes.data, 1)
    assert err[0] == 0


@pytest.mark.gpu
def test_vocab_shard_reduce_on_one_rank(cuda, tmp_path):
    """One-rank NCCL communicator: the all-reduce leaves the packed words as
    they are.  (The multi-rank merge is tests/test_vocab_shard_gpu.py.)"""
    torch = cuda
    import torch.distributed as dist

    from diffusionhard_b200.distributed import nccl_comm_handle

    if dist.is_initialized():
        pytest.skip("a process group is already initialised")
    dist.init_process_group("nccl", init_method=f"file://{tmp_path}/pg", rank=0, world_size=1,
                            device_id=torch.device("cuda", 0))
    try:
        comm = nccl_comm_handle(dist.group.WORLD, torch.device("cuda", 0))
        assert comm
        packed = torch.randint(0, 1 << 62, (257,), dtype=torch.int64, device="cuda")
        before = packed.clone()
        _lib.call("dh_vocab_shard_reduce", comm, _lib.ptr(packed), packed.numel(), _lib.stream_handle())
        torch.cuda.synchronize()
        assert torch.equal(packed, before)
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_packed_forward_computes_only_the_refilling_sequences(cuda):
    """Per-sequence ddpm_cache skip (mdlm.py:1134-1174 per canvas): with half
    of the batch already clean, the packed loop runs the forward over the
    other half only -- half the rows of the whole-batch loop -- and commits
    the same tokens.  Transition by transition through the per-kernel entry
    points, reading the planned forward rows (at most half of the
    whole-batch rows: fewer when one of the masked sequences also goes a
    transition unchanged)."""
    torch = cuda
    from diffusionhard_b200.engine import MDLMEngine

    qm = build_quantized(SMALL, seed=0)
    B, L, steps = 4, 64, 16
    ids = torch.full((B, L), SMALL.mask_token_id, dtype=torch.int64)
    ids[1] = torch.randint(0, 999, (L,), generator=torch.Generator().manual_seed(1))
    ids[3] = torch.randint(0, 999, (L,), generator=torch.Generator().manual_seed(3))
    thr = reveal_thresholds_q32(steps)
    results = {}
    for compact in (False, True):
        eng = MDLMEngine(qm, B, L)
        eng._compact_now = compact
        eng.init_loop(ids.cuda(), steps)
        rows = 0
        for k in range(steps + 1):
            eng.enqueue_transition(k, steps, 5, thr[k] if k < steps else 0)
            torch.cuda.synchronize()
            rows += int(eng.fwd_rows.item())
        results[compact] = (eng.tokens.clone(), rows, eng.metadata(steps))
    (t0, r0, m0), (t1, r1, m1) = results[False], results[True]
    assert torch.equal(t0, t1)
    assert 0 < r1 <= r0 // 2
    assert m0 == m1
    assert not (t1 == SMALL.mask_token_id).any()


@pytest.mark.gpu
@pytest.mark.parametrize("B,L,steps", [(2, 256, 8), (4, 64, 64)])
def test_launch_count_is_the_captured_kernel_count(cuda, B, L, steps):
    """engine.launches_per_generation (the bench's gpu_launches claim) equals
    the kernel nodes of the CUDA graph that captures one whole generation
    through dh_sample_loop, unpacked (the last block finished for the revealed
    rows only) and packed."""
    torch = cuda
    from cuda.bindings import runtime as rt

    from diffusionhard_b200.engine import MDLMEngine

    qm = build_quantized(SMALL, seed=0)
    eng = MDLMEngine(qm, B, L)
    ids = torch.full((B, L), SMALL.mask_token_id, dtype=torch.int64, device="cuda")
    eng.generate(ids, steps=steps, seed=1)  # sets the loop buffers up, eagerly
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph(keep_graph=True)
    with torch.cuda.graph(g):
        eng._enqueue_native(steps, 1, reveal_thresholds_q32(steps))
    graph = rt.cudaGraph_t(init_value=g.raw_cuda_graph())
    err, _, count = rt.cudaGraphGetNodes(graph, 0)
    assert err == rt.cudaError_t.cudaSuccess
    err, nodes, count = rt.cudaGraphGetNodes(graph, count)
    assert err == rt.cudaError_t.cudaSuccess
    kernels = 0
    for node in nodes[:count]:
        err, kind = rt.cudaGraphNodeGetType(node)
        assert err == rt.cudaError_t.cudaSuccess
        kernels += kind == rt.cudaGraphNodeType.cudaGraphNodeTypeKernel
    assert kernels == eng.launches_per_generation(steps)
    del g
