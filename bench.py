#!/usr/bin/env python3
"""Benchmark: generated tokens/s of the MDLM-169.6M W8A8 denoising loop.

Workload per GPU (the full-model configuration the metric is quoted on):
random-init MDLM-OWT-169.6M (N(0, 0.02) weights, folded, W8A8 with SmoothQuant
alpha=0.5 from a seeded calibration batch), batch 32 x L=1024 all-masked
canvases, 64 ddpm_cache transitions of the log-linear schedule + the final
greedy pass, on the candidate-cache loop with the fused int8 head.
One bench step = one complete generation.  With N GPUs every rank runs its
own 32 sequences (weak scaling, no collective on the hot path); the Philox key
uses the global sequence index, so tokens do not depend on N.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

Prints one JSON line (rank 0).  `value` is device-timed (CUDA events, max
over ranks) with inputs resident on the GPU; `e2e` is the same metric
through the public drop-in API (run_ddpm_candidate_cache_sampler) from
pinned host ids, with the host<->device copies inside the timed region.
The line also carries, each measured after the headline on the same ranks:
the whole-generation roofline (`step_roofline`), the measured int8 peak the
int8 fractions use (`int8_peak`), the speed-mode throughput sweep of 512 x
1024 canvases and 32 steps split over the N ranks (`strong_sweep`), and the
single-sequence latency with the head vocab-sharded over the N ranks and the
cost of its per-transition all-reduce (`vocab_shard`).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "generated tok/s, MDLM-169.6M int8 L=1024 64 steps, 1/2/4/8 B200; head GB/s+TC util"
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def load_peaks() -> tuple[dict, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text()), "measured"
    return dict(PEAKS_FALLBACK), "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int) -> None:
        self.gpu = gpu_index
        self.proc = None
        self.path = Path(os.environ.get("TMPDIR", "/tmp")) / f"dh_clocks_{os.getpid()}.csv"

    def __enter__(self):
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=self.fh, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.fh.close()

    def summary(self) -> dict:
        if self.proc is None or not self.path.exists():
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        rows = []
        for line in self.path.read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9 and parts[1].isdigit():
                rows.append(parts)
        self.path.unlink(missing_ok=True)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [int(r[1]) for r in rows]
        loaded = [s for s in sm if s > 600] or sm
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": int(statistics.median(loaded)), "sm_max_mhz": int(rows[0][2]),
                "reasons": reasons, "samples": len(rows), "power_w_max": max(float(r[3]) for r in rows)}


def dist_setup():
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(local)
    return world, rank, local


def max_over_ranks(value: float, world: int) -> float:
    if world == 1:
        return value
    import torch
    import torch.distributed as dist

    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int) -> None:
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def time_kernel(fn, iters: int = 20) -> float:
    """Average ms of `fn` (enqueue on the current stream) over `iters` launches."""
    import torch

    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters


def measure_int8_peak() -> dict:
    """Dense int8 tensor throughput of this GPU, measured the way the bf16
    peak is: a library int8 GEMM (torch._int_mm -> cuBLASLt, int32
    accumulation) of 8192^3, best of 10 timed launches after warm-up
    (2 * 8192^3 ops per launch)."""
    import torch

    n = 8192
    g = torch.Generator(device="cuda").manual_seed(0)
    a = torch.randint(-127, 128, (n, n), dtype=torch.int8, device="cuda", generator=g)
    b = torch.randint(-127, 128, (n, n), dtype=torch.int8, device="cuda", generator=g).t()
    for _ in range(3):
        torch._int_mm(a, b)
    torch.cuda.synchronize()
    best = float("inf")
    for _ in range(10):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        torch._int_mm(a, b)
        e.record()
        e.synchronize()
        best = min(best, s.elapsed_time(e))
    del a, b
    torch.cuda.empty_cache()
    return {"tops": round(2.0 * n ** 3 / (best * 1e-3) / 1e12, 1),
            "how": "torch._int_mm (cuBLASLt) int8 x int8 -> int32, 8192^3, best of 10 launches, CUDA events"}


# Algorithmic work of one forward, per row (the units of the MDLM
# specification, model_spec.py:29-84): backbone int8 ops, attention FLOP per
# key, and the bytes the memory-bound row kernels must move.
# The forward runs every block over every row up to the last block's
# attention; the rest of the last block (attention-out, MLP, their
# quantisers) runs only for the rows whose candidates are drawn (the head's
# rows), which is all the head reads.
QKV_OPS_PER_ROW = 2 * 768 * 2304
POST_ATTN_OPS_PER_ROW = 2 * (768 * 768 + 2 * 768 * 3072)
BACKBONE_OPS_PER_ROW = 11 * (QKV_OPS_PER_ROW + POST_ATTN_OPS_PER_ROW) + QKV_OPS_PER_ROW  # 159,252,480
ATTN_FLOP_PER_ROW_PER_KEY = 36864
HEAD_OPS_PER_ROW = 2 * 768 * 50258 + POST_ATTN_OPS_PER_ROW  # 87,813,120
LN_BYTES = 768 * 4 + 768 + 4
Q768_BYTES = 768 * 2 + 768 + 4
Q3072_BYTES = 3072 * 2 + 3072 + 4
STREAM_BYTES_PER_ROW = 11 * (2 * LN_BYTES + Q768_BYTES + Q3072_BYTES) + LN_BYTES + (768 * 4 * 2 + 4)
# per head row: the last block's LayerNorm and quantisers, the final
# LayerNorm, and the gather of its residual row and attention output
HEAD_STREAM_BYTES_PER_ROW = 2 * LN_BYTES + Q768_BYTES + Q3072_BYTES + 768 * 4 * 2 + 768 * 2 * 2


def step_roofline(ms_per_generation: float, rows: int, kv_len: int, evaluations: int, head_rows: int,
                  int8_tops: float, bf16_tflops: float, hbm_gbs: float) -> dict:
    """Whole-generation roofline: the time the algorithmic work would take at
    the peaks, each kind of work at its own peak and summed
    (int8 ops / int8 peak + bf16 FLOP / bf16 peak + stream bytes / HBM), over
    the measured time."""
    int8_ops = evaluations * rows * BACKBONE_OPS_PER_ROW + head_rows * HEAD_OPS_PER_ROW
    bf16_flop = evaluations * rows * ATTN_FLOP_PER_ROW_PER_KEY * kv_len
    stream = evaluations * rows * STREAM_BYTES_PER_ROW + head_rows * HEAD_STREAM_BYTES_PER_ROW
    t = {"int8": int8_ops / (int8_tops * 1e12), "bf16": bf16_flop / (bf16_tflops * 1e12),
         "hbm": stream / (hbm_gbs * 1e9)}
    ideal_ms = sum(t.values()) * 1e3
    return {"ideal_ms": round(ideal_ms, 2), "measured_ms": round(ms_per_generation, 2),
            "frac": round(ideal_ms / ms_per_generation, 4),
            "ideal_ms_by_kind": {k: round(v * 1e3, 2) for k, v in t.items()},
            "work": {"int8_ops": int8_ops, "bf16_flop": bf16_flop, "stream_bytes": stream,
                     "evaluations": evaluations, "rows_per_evaluation": rows, "head_rows": head_rows},
            "peaks": {"int8_tops": int8_tops, "bf16_tflops": bf16_tflops, "hbm_gbs": hbm_gbs}}


def strong_sweep(qm, world: int, rank: int, global_batch: int = 512, steps: int = 32, warmup: int = 3,
                 iters: int = 2) -> dict:
    """The throughput sweep of the speed mode: global_batch x 1024 all-masked
    canvases split over the ranks (strong scaling), `steps` transitions +
    the final pass; device time, max over ranks."""
    import torch

    from diffusionhard_b200.distributed import shard_batch
    from diffusionhard_b200.engine import MDLMEngine

    offset, B = shard_batch(global_batch, world, rank)
    eng = MDLMEngine(qm, B, 1024)
    eng.seq_offset = offset
    ids = torch.full((B, 1024), qm.config.mask_token_id, dtype=torch.int64, device="cuda")
    for _ in range(warmup):
        eng.generate(ids, steps=steps, seed=0, graph=True)
    torch.cuda.synchronize()
    barrier(world)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        eng.generate(ids, steps=steps, seed=0, graph=True)
    e.record()
    torch.cuda.synchronize()
    ms = max_over_ranks(s.elapsed_time(e), world) / iters
    meta = eng.metadata(steps)
    eng._graphs.clear()
    del eng
    torch.cuda.empty_cache()
    return {"value": round(global_batch * 1024 / (ms * 1e-3), 1), "unit": "tok/s", "scaling": "strong",
            "n_gpus": world, "global_batch": global_batch, "sequences_per_gpu": B, "seq_len": 1024,
            "steps": steps, "ms_per_generation": round(ms, 3), "warmup": warmup, "timed": iters,
            "model_evaluations": meta["model_evaluations"]}


def vocab_shard_latency(qm, world: int, rank: int, steps: int = 64, warmup: int = 3, iters: int = 3,
                        graph: bool = True) -> dict:
    """Single-sequence latency with the head split over the ranks and merged
    by dh_vocab_shard_reduce (NCCL all-reduce of the packed per-row words)
    after every head launch; beside it, the time of that all-reduce alone
    (back-to-back calls on the 1024 packed words of a transition)."""
    import torch

    from diffusionhard_b200 import _lib
    from diffusionhard_b200.distributed import vocab_shards
    from diffusionhard_b200.engine import MDLMEngine

    L = 1024
    eng = MDLMEngine(qm, 1, L)
    if world > 1:
        import torch.distributed as dist

        v0, v1 = vocab_shards(qm.config.vocab_size, world)[rank]
        eng.shard_head(v0, v1, group=dist.group.WORLD)
    ids = torch.full((1, L), qm.config.mask_token_id, dtype=torch.int64, device="cuda")
    for _ in range(warmup):
        eng.generate(ids, steps=steps, seed=0, graph=graph)
    torch.cuda.synchronize()
    barrier(world)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        eng.generate(ids, steps=steps, seed=0, graph=graph)
    e.record()
    torch.cuda.synchronize()
    ms = max_over_ranks(s.elapsed_time(e), world) / iters
    tokens = eng.tokens.clone()
    agree = True
    reduce_us = None
    if world > 1:
        import torch.distributed as dist

        gathered = [torch.empty_like(tokens) for _ in range(world)]
        dist.all_gather(gathered, tokens)
        agree = all(torch.equal(g, tokens) for g in gathered)
        comm = eng._nccl_comm()
        packed = torch.zeros(L, dtype=torch.int64, device="cuda")
        for _ in range(10):
            _lib.call("dh_vocab_shard_reduce", comm, _lib.ptr(packed), L, _lib.stream_handle())
        torch.cuda.synchronize()
        barrier(world)
        n = 200
        s.record()
        for _ in range(n):
            _lib.call("dh_vocab_shard_reduce", comm, _lib.ptr(packed), L, _lib.stream_handle())
        e.record()
        torch.cuda.synchronize()
        reduce_us = max_over_ranks(s.elapsed_time(e), world) / n * 1e3
    meta = eng.metadata(steps)
    eng._graphs.clear()  # graphs holding NCCL calls go before the process group does
    del eng
    torch.cuda.empty_cache()
    out = {"value": round(L / (ms * 1e-3), 1), "unit": "tok/s", "ms_per_generation": round(ms, 3),
           "n_gpus": world, "head_split": world, "seq_len": L, "steps": steps,
           "model_evaluations": meta["model_evaluations"], "ranks_agree_on_tokens": agree,
           "loop": "dh_sample_loop" + (" in a CUDA graph (the all-reduce captured with it)" if graph else
                                       ", eager launches")}
    if reduce_us is not None:
        transitions = steps + 1
        out["allreduce_us_per_transition"] = round(reduce_us, 2)
        out["allreduce_ms_per_generation"] = round(reduce_us * transitions / 1e3, 3)
        out["allreduce_share"] = round(reduce_us * transitions / 1e3 / ms, 4)
    return out


def kernel_breakdown(eng) -> dict:
    """Per-kernel average launch time of one forward's kernels (ms)."""
    from diffusionhard_b200 import _lib

    p, s, M, L = _lib.ptr, _lib.stream_handle(), eng.M, eng.L
    blk = eng.blocks[0]
    k, vt = eng.kv_buffers[0]
    qkv, out, up, down = blk["qkv"], blk["out"], blk["up"], blk["down"]
    c = _lib.call
    fns = {
        "embed_gather": lambda: c("dh_embed_gather", p(eng.tokens), p(eng.embedding), p(eng.x), M,
                                  eng.cfg.vocab_size, None, s),
        "ln_smooth_quant": lambda: c("dh_ln_smooth_quant", p(eng.x), p(qkv.smooth), p(qkv.inv_smooth), p(eng.act_q),
                                     p(eng.act_scale), M, None, None, None, s),
        "gemm_qkv_rope": lambda: c("dh_gemm_qkv_rope", p(eng.act_q), p(eng.act_scale), p(qkv.w),
                                   p(qkv.w_scale), p(qkv.bias), p(eng.rope_cos), p(eng.rope_sin), p(out.inv_smooth), M, L, 0,
                                   eng.kv_stride, 0, p(eng.q), p(k), p(vt), None, s),
        "attention": lambda: c("dh_attention", p(eng.q), p(k), p(vt), p(eng.attn), eng.B, L, eng.kv_len,
                               eng.kv_stride, None, s),
        "quant_rows_768": lambda: c("dh_quant_rows_bf16", p(eng.attn), None, None, p(eng.act_q),
                                    p(eng.act_scale), M, 768, None, s),
        "gemm_out_residual": lambda: c("dh_gemm_residual", p(eng.act_q), p(eng.act_scale), p(out.w),
                                       p(out.w_scale), p(out.bias), p(eng.x), M, 768, 768, None, s),
        "gemm_up_gelu": lambda: c("dh_gemm_gelu", p(eng.act_q), p(eng.act_scale), p(up.w), p(up.w_scale),
                                  p(up.bias), p(down.inv_smooth), p(eng.mlp), p(eng.row_amax), M, 3072, 768,
                                  None, s),
        "quant_rows_3072": lambda: c("dh_quant_rows_bf16_amax", p(eng.mlp), p(eng.row_amax), p(eng.act_q),
                                     p(eng.act_scale), M, 3072, None, s),
        "gemm_down_residual": lambda: c("dh_gemm_residual", p(eng.act_q), p(eng.act_scale), p(down.w),
                                        p(down.w_scale), p(down.bias), p(eng.x), M, 768, 3072, None, s),
    }
    return {name: time_kernel(fn) for name, fn in fns.items()}


# The kernels that finish the last block run over the head's rows only (a
# few hundred of the 32,768 per evaluation): per forward, the full-size
# launches of kernel_breakdown are those of the other blocks.
LAST_BLOCK_ROWS_ONLY = ("quant_rows_768", "gemm_out_residual", "gemm_up_gelu", "quant_rows_3072",
                        "gemm_down_residual")


def launches_per_forward(name: str, blocks: int) -> int:
    if name == "embed_gather":
        return 1
    if name == "ln_smooth_quant":
        return 2 * blocks - 1
    if name in LAST_BLOCK_ROWS_ONLY:
        return blocks - 1
    return blocks


def roofline_for(name: str, ms: float, eng, peaks: dict, peaks_kind: str, int8: dict) -> dict:
    M, L, B = eng.M, eng.L, eng.B
    int8_peak = int8["tops"]
    gemm = {"gemm_qkv_rope": (768, 2304), "gemm_out_residual": (768, 768), "gemm_up_gelu": (768, 3072),
            "gemm_down_residual": (3072, 768)}
    if name in gemm:
        K, N = gemm[name]
        ach = 2.0 * M * N * K / (ms * 1e-3) / 1e12
        return {"kernel": name, "bound": "tensor", "achieved": round(ach, 1),
                "peak": round(int8_peak, 1), "unit": "TOP/s", "frac": round(ach / int8_peak, 4),
                "peak_source": "measured int8: " + int8["how"],
                "work_per_launch": f"2*{M}*{N}*{K} int8 ops"}
    if name == "attention":
        flops = 4.0 * B * 12 * L * eng.kv_len * 64
        ach = flops / (ms * 1e-3) / 1e12
        return {"kernel": name, "bound": "tensor", "achieved": round(ach, 1), "peak": peaks["bf16_tflops"],
                "unit": "TFLOP/s", "frac": round(ach / peaks["bf16_tflops"], 4),
                "peak_source": f"{peaks_kind} bf16 burst", "work_per_launch": "4*B*12*L*kv_len*64 bf16 FLOP"}
    bytes_per = {"ln_smooth_quant": M * (768 * 4 + 768 + 4), "quant_rows_768": M * (768 * 2 + 768 + 4),
                 "quant_rows_3072": M * (3072 * 2 + 3072 + 4), "embed_gather": M * (768 * 4 * 2 + 4)}[name]
    ach = bytes_per / (ms * 1e-3) / 1e9
    return {"kernel": name, "bound": "hbm", "achieved": round(ach, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
            "frac": round(ach / peaks["hbm_gbs"], 4), "peak_source": f"{peaks_kind} copy bandwidth",
            "work_per_launch": f"{bytes_per} bytes"}


def head_microbench(qm, peaks: dict, peaks_kind: str, int8: dict) -> dict:
    """The fused head + sampler microbench as the configuration specifies it:
    bf16 hidden [64, 1024, 768] ~ N(0, 1), conditioning [64, 128] ~ N(0, 1),
    adaLN Linear(128 -> 1536) ~ N(0, 0.02), int8 weight [50258, 768] =
    round(clip(N(0, 40), +-127)) with fp32 scales ~ U(0.5e-3, 2e-3) and bias
    ~ N(0, 0.02), 50% of the positions masked by a Bernoulli draw of
    Generator(seed 0), Philox key (seed, b).  Timed per step, all on the
    device: the mask load, adaLN, masked-row compaction, LayerNorm +
    modulation + per-token int8 of the masked rows, and the fused head with
    its Philox-Gumbel argmax (diffusionhard_b200.final_head).  Beside it the
    head kernel alone over the same rows."""
    import numpy as np
    import torch

    from diffusionhard_b200 import _lib
    from diffusionhard_b200.final_head import ConditionedHead

    B, L, V, C = 64, 1024, qm.config.vocab_size, 128
    g = torch.Generator().manual_seed(0)
    masked = torch.rand((B, L), generator=g) < 0.5
    gd = torch.Generator(device="cuda").manual_seed(0)
    hidden = torch.randn((B, L, 768), device="cuda", generator=gd).to(torch.bfloat16)
    cond = torch.randn((B, C), device="cuda", generator=gd)
    rng = np.random.default_rng(0)
    ada_w = (rng.standard_normal((1536, C)) * 0.02).astype(np.float32)
    w = np.clip(np.round(rng.normal(0, 40, (V, 768))), -127, 127).astype(np.int8)
    w_scale = rng.uniform(0.5e-3, 2e-3, V).astype(np.float32)
    bias = (rng.standard_normal(V) * 0.02).astype(np.float32)
    head = ConditionedHead(w, w_scale, bias, ada_w, None, None, qm.config.mask_token_id, B, L)
    masked_dev = masked.cuda()

    def step():
        head.load_mask(masked_dev)
        head.enqueue(hidden, cond, seed=0)

    ms = time_kernel(step, iters=10)
    rows = int(head.sel_count.item())
    p = _lib.ptr

    def head_only():
        _lib.call("dh_head_argmax_i8", p(head.head_q), 768, p(head.w), 768, B * L, p(head.sel_count), 768, V, 0,
                  qm.config.mask_token_id, 1, p(head.head_scale), p(head.w_scale), p(head.bias), None, None, None,
                  p(head.sel_pos), p(head.sel_key), p(head.sel_eval), 0, 0, 0, p(head.packed), p(head.out_ids), None,
                  _lib.stream_handle())

    head_ms = time_kernel(head_only, iters=10)
    # the head's noise alone over the same rows, vocabulary and Philox keys,
    # on every SM with nothing else to compute: the integer-pipe floor
    packed_n = torch.zeros(rows, dtype=torch.int64, device="cuda")

    def noise_only():
        packed_n.zero_()
        _lib.call("dh_noise_argmax", rows, V, qm.config.mask_token_id, p(head.sel_pos), p(head.sel_key),
                  p(head.sel_eval), 0, 0, 0, 0, p(packed_n), None, _lib.stream_handle())

    noise_ms = time_kernel(noise_only, iters=10)
    ops = 2.0 * rows * V * 768
    ach = ops / (head_ms * 1e-3) / 1e12
    return {"workload": "64 x 1024 bf16 hidden, 50% masked (Bernoulli, seed 0), adaLN final LayerNorm + per-token "
                        "int8 + 768 x 50258 int8 head + Philox-Gumbel argmax",
            "masked_rows": rows, "vocab": V, "ms": round(ms, 4), "head_kernel_ms": round(head_ms, 4),
            "prologue_ms": round(ms - head_ms, 4), "rows_per_s": round(rows / (ms * 1e-3), 1),
            "achieved_top_s": round(ach, 1), "int8_peak_top_s": int8["tops"],
            "tensor_frac": round(ach / int8["tops"], 4),
            "integer_roofline": {"noise_only_ms": round(noise_ms, 4), "frac": round(noise_ms / head_ms, 4),
                                 "how": "dh_noise_argmax over the same rows x vocabulary and Philox keys (the "
                                        "head's Philox-4x32-10 / Gumbel Q10 race with zero logits, all SMs, no "
                                        "GEMM) over the fused head's time"},
            "note": "per logit: 1/4 of a Philox4x32-10 block, the Gumbel Q10 lookup, the exact fp64 dequant and "
                    "the Q10 rounding on the integer / fp64 pipes; see profiles/ for the pipe utilisation"}


def profile_forward(args) -> None:
    """One forward over B x L rows plus the head over 512 selected rows."""
    import torch

    from diffusionhard_b200.engine import MDLMEngine
    from diffusionhard_b200.model import MDLMConfig, build_quantized

    cfg = MDLMConfig()
    qm = build_quantized(cfg, seed=0)
    eng = MDLMEngine(qm, args.batch, args.seq_len)
    eng.tokens.fill_(cfg.mask_token_id)
    rows = torch.arange(512, dtype=torch.int32, device="cuda") * 61
    count = torch.tensor([512], dtype=torch.int32, device="cuda")
    pos = rows % args.seq_len
    key = rows // args.seq_len
    for _ in range(2):
        eng.forward()
        eng.final_hidden_q(rows, count)
        eng.head_argmax(eng.M, 1, rows_count=count, row_position=pos, row_key_hi=key, key_lo=0)
    torch.cuda.synchronize()
    print("profile-forward done", flush=True)


def profile_head(args) -> None:
    """The head microbench's pipeline (adaLN, masked-row compaction,
    LayerNorm + modulation + int8, fused head) on --batch x 1024 bf16 hidden
    states, 50% masked, three times: a short launch list for ncu."""
    import numpy as np
    import torch

    from diffusionhard_b200.final_head import ConditionedHead

    B, L, V, C = args.batch, 1024, 50258, 128
    g = torch.Generator().manual_seed(0)
    masked = torch.rand((B, L), generator=g) < 0.5
    gd = torch.Generator(device="cuda").manual_seed(0)
    hidden = torch.randn((B, L, 768), device="cuda", generator=gd).to(torch.bfloat16)
    cond = torch.randn((B, C), device="cuda", generator=gd)
    rng = np.random.default_rng(0)
    ada_w = (rng.standard_normal((1536, C)) * 0.02).astype(np.float32)
    w = np.clip(np.round(rng.normal(0, 40, (V, 768))), -127, 127).astype(np.int8)
    w_scale = rng.uniform(0.5e-3, 2e-3, V).astype(np.float32)
    bias = (rng.standard_normal(V) * 0.02).astype(np.float32)
    head = ConditionedHead(w, w_scale, bias, ada_w, None, None, V - 1, B, L)
    for _ in range(3):
        head.load_mask(masked.cuda())
        head.enqueue(hidden, cond, seed=0)
    torch.cuda.synchronize()
    print("profile-head done:", int(head.sel_count.item()), "masked rows", flush=True)


def run_vocab_shard(args, world: int, rank: int) -> None:
    """Single-sequence latency: every rank runs the same backbone forward and
    projects its slice of the head; the packed (score, ~id) words are
    MAX-reduced over NCCL every transition, so all ranks commit the same
    tokens (identical to the unsharded head)."""
    import torch

    from diffusionhard_b200.distributed import vocab_shards
    from diffusionhard_b200.engine import MDLMEngine
    from diffusionhard_b200.model import MDLMConfig, build_quantized

    cfg = MDLMConfig()
    qm = build_quantized(cfg, seed=0)
    L, S = args.seq_len, args.denoise_steps
    eng = MDLMEngine(qm, 1, L)
    if world > 1:
        import torch.distributed as dist

        v0, v1 = vocab_shards(cfg.vocab_size, world)[rank]
        eng.shard_head(v0, v1, group=dist.group.WORLD)
    ids = torch.full((1, L), cfg.mask_token_id, dtype=torch.int64, device="cuda")
    for _ in range(args.warmup):
        eng.generate(ids, steps=S, seed=0, graph=True)
    torch.cuda.synchronize()
    barrier(world)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(args.steps):
        eng.generate(ids, steps=S, seed=0, graph=True)
    end.record()
    torch.cuda.synchronize()
    ms = max_over_ranks(start.elapsed_time(end), world)
    tokens_here = eng.tokens.clone()
    if world > 1:
        import torch.distributed as dist

        gathered = [torch.empty_like(tokens_here) for _ in range(world)]
        dist.all_gather(gathered, tokens_here)
        consistent = all(torch.equal(g, tokens_here) for g in gathered)
    else:
        consistent = True
    if rank == 0:
        per = ms / args.steps
        print(json.dumps({
            "metric": "single-sequence generation latency, MDLM-169.6M int8, vocab-sharded head",
            "value": round(L / (per * 1e-3), 1), "unit": "tok/s", "ms_per_generation": round(per, 3),
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
            "scaling": "strong", "dtype": "int8", "data": "synthetic",
            "config": {"workload": f"1 x L={L}, {S} ddpm_cache steps, head 768x50258 split over {world} GPU(s), "
                                   "packed-u64 MAX all-reduce per transition", "global_batch": 1, "seq_len": L,
                       "steps": S, "parallelism": f"vocab{world}"},
            "ranks_agree_on_tokens": consistent,
            "model_evaluations": eng.metadata(S)["model_evaluations"]}), flush=True)
    eng._graphs.clear()  # graphs holding NCCL calls go before the process group does
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()


def run_prefix_conditioned(args, world: int, rank: int) -> None:
    """Prefix-conditioned generation with prefix K/V reuse: B sequences of a
    clean prefix (uniform ids, seed 2) and a fully masked suffix.  Each timed
    generation runs the isolated prefix forward once and the candidate-cache
    loop over the suffix only (suffix rows attend to [prefix ; suffix]).
    Beside it: the same generation on the whole canvas with full
    bidirectional attention (every evaluation recomputes the prefix), the
    drift of the isolated prefix K/V against a full-attention forward, and a
    check that the suffix loop left the prefix K/V bit-identical."""
    import torch

    from diffusionhard_b200.engine import MDLMEngine
    from diffusionhard_b200.model import MDLMConfig, build_quantized
    from diffusionhard_b200.prefix import PrefixConditionedGenerator

    cfg = MDLMConfig()
    qm = build_quantized(cfg, seed=0)
    B, P, S, T = args.batch, args.prefix_tokens, args.seq_len - args.prefix_tokens, args.denoise_steps
    offset = rank * B
    gen = PrefixConditionedGenerator(qm, B, P, S)
    gen.suffix.seq_offset = offset
    prefix = torch.randint(0, cfg.mask_token_id, (world * B, P), generator=torch.Generator().manual_seed(2))
    prefix = prefix[offset:offset + B].cuda()
    suffix = torch.full((B, S), cfg.mask_token_id, dtype=torch.int64, device="cuda")

    def timed(fn) -> float:
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        barrier(world)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(args.steps):
            fn()
        b.record()
        torch.cuda.synchronize()
        return max_over_ranks(a.elapsed_time(b), world) / args.steps

    with ClockSampler(torch.cuda.current_device()) as clocks:
        cached_ms = timed(lambda: gen.generate(prefix, suffix, steps=T, seed=0, graph=True))
    clock_info = clocks.summary()
    cached_tokens = gen.suffix.tokens.view(B, S).clone()
    meta = gen.suffix.metadata(T)
    prefill_ms = timed(lambda: gen.set_prefix(prefix))
    kv_before = [(k[:, :, :P].clone(), vt[:, :, :, :P].clone()) for k, vt in gen.kv]
    gen.suffix.generate(suffix, steps=T, seed=0, graph=True)
    torch.cuda.synchronize()
    prefix_kv_untouched = all(torch.equal(a, k[:, :, :P]) and torch.equal(b, vt[:, :, :, :P])
                              for (a, b), (k, vt) in zip(kv_before, gen.kv))
    del kv_before

    full = MDLMEngine(qm, B, P + S)
    full.seq_offset = offset
    canvas = torch.cat([prefix, suffix], dim=1)
    full_ms = timed(lambda: full.generate(canvas, steps=T, seed=0, graph=True))
    full_suffix = full.tokens.view(B, P + S)[:, P:]
    agreement = float(full_suffix.eq(cached_tokens).float().mean().item())
    full._graphs.clear()
    del full
    torch.cuda.empty_cache()

    drift = gen.drift_report(prefix, cached_tokens.to(torch.int64))
    layers = [{"layer": d["layer"], "key_normalized_rmse": round(d["key"]["normalized_rmse"], 6),
               "value_normalized_rmse": round(d["value"]["normalized_rmse"], 6),
               "key_cosine": round(d["key"]["cosine_similarity"], 6),
               "key_exact": d["key"]["exact_equal"], "value_exact": d["value"]["exact_equal"]}
              for d in drift["layers"]]
    gen.suffix._graphs.clear()
    if rank == 0:
        tokens = world * B * S
        print(json.dumps({
            "metric": "generated suffix tok/s, prefix-conditioned MDLM-169.6M int8 (prefix K/V reused)",
            "value": round(tokens / (cached_ms * 1e-3), 1), "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(cached_ms, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
            "data": "synthetic (random-init weights, prefix ids uniform in [0, 50257) seed 2)",
            "config": {"workload": f"{B} x (prefix {P} + suffix {S}) per GPU, {T} ddpm_cache steps + final pass; "
                                   "prefix forward once per generation, suffix-only loop",
                       "global_batch": world * B, "seq_len": P + S, "prefix": P, "suffix": S, "steps": T,
                       "parallelism": f"dp{world} batch-sharded"},
            "prefix_prefill_ms": round(prefill_ms, 3),
            "full_recompute": {"ms_per_generation": round(full_ms, 3),
                               "value": round(tokens / (full_ms * 1e-3), 1),
                               "speedup_of_prefix_reuse": round(full_ms / cached_ms, 3),
                               "note": "whole canvas, full bidirectional attention, every evaluation "
                                       "recomputes all P + S rows",
                               "suffix_token_agreement_with_prefix_reuse": round(agreement, 4)},
            "isolated_prefix_kv_exact_after_generation": prefix_kv_untouched,
            "full_attention_prefix_kv_drift": {"first_drifting_layer": drift["first_drifting_layer"],
                                               "layers": layers},
            "generation": {"model_evaluations": meta["model_evaluations"],
                           "sampling_transitions": meta["sampling_transitions"],
                           "masks_left": int((cached_tokens == cfg.mask_token_id).sum().item())},
            "gpu_launches": (gen.suffix.launches_per_generation(T) + gen.prefix.launches_per_forward) * args.steps,
            "clocks": clock_info}), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()


def run_reference(args, world: int, rank: int) -> None:
    if rank != 0:
        return
    from diffusionhard_b200.model import MDLMConfig, build_quantized
    from oracle import cpu_baseline

    qm = build_quantized(MDLMConfig(), seed=0)
    samples = []
    for i in range(args.warmup + args.steps):
        r = cpu_baseline.measure_reference_sampler(qm, positions=args.seq_len, sample_steps=4,
                                                   steps=args.denoise_steps)
        if r is None:  # the reference package is not installed: the restated transition
            r = cpu_baseline.measure(qm, positions=args.seq_len, transitions=1, steps=args.denoise_steps)
        if i >= args.warmup:
            samples.append(r["seconds_per_evaluated_transition"])
    dt = statistics.mean(samples)
    L = args.seq_len
    value = L / (dt * (args.denoise_steps + 1))
    line = {"metric": METRIC, "value": round(value, 3), "unit": "tok/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 1),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
            "data": "synthetic", "impl": "reference",
            "config": {"workload": f"MDLM-169.6M W8A8 random-init, L={L} all-masked, {args.denoise_steps} "
                                   "ddpm_cache steps (CPU: per step one bounded call of the sampler on 1 "
                                   "sequence, extrapolated per model evaluation)",
                       "global_batch": 1, "seq_len": L, "steps": args.denoise_steps},
            "cpu_baseline": {"value": round(value, 3), "unit": "tok/s", "cores": r["cores"], "kind": r["kind"],
                             "sample": r["sample"]},
            "e2e": {"value": round(value, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--batch", type=int, default=32, help="sequences per GPU")
    ap.add_argument("--seq-len", type=int, default=1024)
    ap.add_argument("--denoise-steps", type=int, default=64)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--global-batch", type=int, default=0,
                    help="split this many sequences over the ranks (strong scaling, e.g. 512 "
                         "with --denoise-steps 32); default: --batch per GPU (weak scaling)")
    ap.add_argument("--vocab-shard", action="store_true",
                    help="single-sequence latency: backbone replicated, 768x50258 head split over "
                         "the ranks, per-transition packed-max all-reduce (one line, impl ours)")
    ap.add_argument("--prefix-conditioned", action="store_true",
                    help="prefix K/V reuse workload: --batch sequences of --prefix-tokens clean ids + "
                         "(--seq-len - --prefix-tokens) masked suffix per GPU (one line, impl ours)")
    ap.add_argument("--prefix-tokens", type=int, default=512)
    ap.add_argument("--profile-forward", action="store_true",
                    help="run one warm-up forward, then one forward + one head call "
                         "(a short launch list for ncu)")
    ap.add_argument("--profile-head", action="store_true",
                    help="run the conditioned head pipeline of the head microbench three times on "
                         "--batch x 1024 canvases (a short launch list for ncu)")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")

    import torch

    world, rank, local = dist_setup() if args.impl == "ours" or int(os.environ.get("WORLD_SIZE", "1")) > 1 \
        else (1, 0, 0)
    if args.impl == "reference":
        run_reference(args, world, rank)
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
        return

    from diffusionhard_b200 import _lib
    from diffusionhard_b200.api import run_ddpm_candidate_cache_sampler
    from diffusionhard_b200.engine import MDLMEngine
    from diffusionhard_b200.model import MDLMConfig, build_quantized

    peaks, peaks_kind = load_peaks()
    if args.profile_forward:
        profile_forward(args)
        return
    if args.profile_head:
        profile_head(args)
        return
    if args.vocab_shard:
        run_vocab_shard(args, world, rank)
        return
    if args.prefix_conditioned:
        run_prefix_conditioned(args, world, rank)
        return
    cfg = MDLMConfig()
    qm = build_quantized(cfg, seed=0)
    L, S = args.seq_len, args.denoise_steps
    if args.global_batch:
        from diffusionhard_b200.distributed import shard_batch

        offset, B = shard_batch(args.global_batch, world, rank)
        scaling = "strong"
    else:
        B, offset, scaling = args.batch, rank * args.batch, "weak"
    eng = MDLMEngine(qm, B, L)
    eng.seq_offset = offset
    ids_dev = torch.full((B, L), cfg.mask_token_id, dtype=torch.int64, device="cuda")
    host_ids = torch.full((B, L), cfg.mask_token_id, dtype=torch.int64).pin_memory()

    for _ in range(args.warmup):
        eng.generate(ids_dev, steps=S, seed=0, graph=True)
    torch.cuda.synchronize()
    barrier(world)

    # ------------------------------------------------ device-timed region
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(torch.cuda.current_device()) as clocks:
        barrier(world)
        torch.cuda.synchronize()
        start.record()
        for _ in range(args.steps):
            eng.generate(ids_dev, steps=S, seed=0, graph=True)
        end.record()
        torch.cuda.synchronize()
        barrier(world)
    ms = max_over_ranks(start.elapsed_time(end), world)
    clock_info = clocks.summary()
    global_batch = args.global_batch or world * B
    tokens = global_batch * L * args.steps
    value = tokens / (ms * 1e-3)
    meta = eng.metadata(S)
    masks_left = int((eng.tokens == cfg.mask_token_id).sum().item())

    # ------------------------------------------------ end-to-end (public API, host buffers)
    for _ in range(2):
        run_ddpm_candidate_cache_sampler(eng, host_ids, mask_token_id=cfg.mask_token_id, steps=S, seed=0)
    torch.cuda.synchronize()
    barrier(world)
    t0 = time.perf_counter()
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_start.record()
    for _ in range(args.steps):
        ids_out, _, meta_e2e = run_ddpm_candidate_cache_sampler(eng, host_ids, mask_token_id=cfg.mask_token_id,
                                                                steps=S, seed=0)
    e_end.record()
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e_start.elapsed_time(e_end), world)
    wall_e2e = max_over_ranks((time.perf_counter() - t0) * 1e3, world)
    e2e_value = tokens / (e2e_ms * 1e-3)

    # ------------------------------------------------ kernel breakdown / roofline
    int8 = measure_int8_peak()
    bd = kernel_breakdown(eng)
    per_gen = {k: v * launches_per_forward(k, len(eng.blocks)) for k, v in bd.items()}
    dominant = max(per_gen, key=per_gen.get)
    roof = roofline_for(dominant, bd[dominant], eng, peaks, peaks_kind, int8)
    traffic_file = ROOT / "profiles" / "traffic.json"
    traffic = None
    if traffic_file.exists():
        traffic = json.loads(traffic_file.read_text()).get(dominant)
    roof["traffic"] = traffic
    head = head_microbench(qm, peaks, peaks_kind, int8) if rank == 0 else None
    step_roof = step_roofline(ms / args.steps, B * L, eng.kv_len, meta["model_evaluations"], B * L,
                              int8["tops"], peaks["bf16_tflops"], peaks["hbm_gbs"])
    eng._graphs.clear()
    sweep = strong_sweep(qm, world, rank)
    shard = vocab_shard_latency(qm, world, rank)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import cpu_baseline

        r = cpu_baseline.measure_best(qm, steps=S)
        cpu = {k: (round(v, 3) if isinstance(v, float) else v) for k, v in r.items()
               if k in ("value", "unit", "cores", "kind", "sample")}

    err = __import__("numpy").zeros(1, "uint32")
    _lib.call("dh_device_error", err.ctypes.data, 0)
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 3),
            "higher_is_better": True, "scaling": scaling, "vs_baseline": None, "dtype": "int8",
            "data": "synthetic (random-init N(0,0.02) weights, all-masked canvases)",
            "config": {"workload": (f"MDLM-169.6M W8A8, batch {B} x L={L} per GPU, {S} ddpm_cache steps + final pass"
                                    if scaling == "weak" else
                                    f"MDLM-169.6M W8A8, {global_batch} x L={L} split over {world} GPU(s), "
                                    f"{S} ddpm_cache steps + final pass"),
                       "global_batch": global_batch, "seq_len": L, "steps": S, "parallelism": f"dp{world} batch-sharded",
                       "l2": "activations per forward (> 1 GB) exceed L2; no flush needed"},
            "e2e": {"value": round(e2e_value, 1), "unit": "tok/s", "h2d_bytes_per_step": B * L * 8,
                    "d2h_bytes_per_step": B * L * 8 + 3 * S * 4, "wall_ms_per_step": round(wall_e2e / args.steps, 3)},
            "roofline": roof,
            "step_roofline": step_roof,
            "int8_peak": int8,
            "cpu_baseline": cpu,
            "gpu_launches": eng.launches_per_generation(S) * args.steps,
            "clocks": clock_info,
            "kernel_ms": {k: round(v, 4) for k, v in bd.items()},
            "kernel_ms_per_generation_est": {k: round(v * (S + 1), 2) for k, v in per_gen.items()},
            "head_microbench": head,
            "strong_sweep": sweep,
            "vocab_shard": shard,
            "generation": {"model_evaluations": meta["model_evaluations"],
                           "sampling_transitions": meta["sampling_transitions"], "masks_left": masks_left,
                           "e2e_matches_device": bool(torch.equal(ids_out.cuda().to(torch.int32), eng.tokens.view(B, L)))},
            "device_error": int(err[0]),
        }
        print(json.dumps(line), flush=True)
    eng._graphs.clear()
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
