"""MDLM engine: device-resident W8A8 DDiT + fused head + candidate-cache loop.

Host side of the C ABI (include/dh_b200.h).  Per forward and block:
LN+SmoothQuant+int8 -> QKV GEMM (+rotary) -> attention -> requant ->
attention-out GEMM (+residual) -> LN+quant -> MLP-up GEMM (+GELU) -> requant ->
MLP-down GEMM (+residual).  `generate` hands the whole generation to the
library's composite entry point dh_sample_loop (one C call enqueues every
launch); the per-kernel orchestration here serves the loop variants the
composite does not cover (prefix K/V offsets, Python hooks, a non-NCCL head
reduction) and the per-transition tests.  Every launch is enqueued on one
stream with no host synchronisation; a whole generation can be captured in
one CUDA graph (`generate(..., graph=True)`).

The transition structure follows mdlm._run_ddpm_candidate_cache_sampler
(mdlm.py:1104-1218); candidates are computed only for the rows revealed at a
transition (loop.cu), which is pathwise identical to the full-row candidate
cache.
"""

from __future__ import annotations

import ctypes
import functools
from typing import Any, Dict, List, Optional

import numpy as np

from . import _lib
from .model import QuantizedMDLM
from .sampler import NOISE_EPSILON, MDLMStepMeasurement, hardware_candidate_cache_bytes, reveal_thresholds_q32


class _DevLinear:
    def __init__(self, torch, ql, device) -> None:
        self.w = torch.from_numpy(np.ascontiguousarray(ql.weight_q)).to(device)
        self.w_scale = torch.from_numpy(ql.w_scale.astype(np.float32)).to(device)
        self.bias = torch.from_numpy(ql.bias.astype(np.float32)).to(device)
        self.smooth = torch.from_numpy(ql.smooth.astype(np.float32)).to(device)
        self.inv_smooth = torch.from_numpy(ql.inv_smooth.astype(np.float32)).to(device)
        self.out_features, self.in_features = ql.weight_q.shape


def _on_device(method):
    """Run an engine method with the engine's GPU as the current device.
    Every launch goes to the current device's current stream and reads the
    current device's error word, so an engine on cuda:1 must not launch
    while cuda:0 is current."""

    @functools.wraps(method)
    def wrapper(self, *args, **kwargs):
        with self.torch.cuda.device(self.device):
            return method(self, *args, **kwargs)

    return wrapper


class MDLMEngine:
    """Weights and activation buffers for `batch` sequences of `seq_len` rows.

    Attention keys: this forward writes its K / V rows at key offset
    `kv_offset` of K / V^T buffers with `kv_stride` keys per (sequence, head)
    and attends over the first `kv_len` keys.  Default: kv_len = kv_stride =
    seq_len, offset 0.  Prefix reuse (prefix_drift._cached_suffix_forward,
    prefix_drift.py:155-238) shares per-block K / V buffers between a prefix
    engine (seq_len = P, kv_len = P, offset 0: the isolated prefix) and a
    suffix engine (seq_len = S, pos_offset = P, kv_offset = P,
    kv_len = P + S): the prefix K / V are written once and never recomputed.
    """

    def __init__(self, qm: QuantizedMDLM, batch: int, seq_len: int, device: Any = "cuda", *,
                 pos_offset: int = 0, kv_len: Optional[int] = None, kv_offset: int = 0,
                 kv_buffers: Optional[List[tuple]] = None) -> None:
        import torch

        self.torch = torch
        cfg = qm.config
        if cfg.hidden != 768 or cfg.heads != 12 or cfg.head_dim != 64 or cfg.mlp != 3072:
            raise ValueError("the kernels are specialised for d=768, 12x64 heads, MLP 3072")
        kv_len = seq_len if kv_len is None else kv_len
        if seq_len % 32 or kv_len % 32 or kv_offset % 32:
            raise ValueError("seq_len, kv_len and kv_offset must be multiples of 32")
        if pos_offset + seq_len > cfg.max_positions or kv_offset + seq_len > max(kv_len, kv_offset + seq_len):
            raise ValueError("rotary positions exceed the model length")
        self.cfg, self.qm = cfg, qm
        self.B, self.L = batch, seq_len
        self.pos_offset, self.kv_len, self.kv_offset = pos_offset, kv_len, kv_offset
        self.M = batch * seq_len
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("the engine runs on a CUDA device")
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        d = self.device
        self.embedding = torch.from_numpy(qm.embedding).to(d)
        self.rope_cos = torch.from_numpy(np.ascontiguousarray(qm.rope_cos)).to(d)
        self.rope_sin = torch.from_numpy(np.ascontiguousarray(qm.rope_sin)).to(d)
        self.blocks = [{k: _DevLinear(torch, v, d) for k, v in blk.items()} for blk in qm.blocks]
        self.head = _DevLinear(torch, qm.head, d)
        M, H = self.M, cfg.heads
        bf16 = torch.bfloat16
        self.x = torch.empty((M, 768), dtype=torch.float32, device=d)
        self.act_q = torch.empty((M, 3072), dtype=torch.int8, device=d)
        self.act_scale = torch.empty(M, dtype=torch.float32, device=d)
        self.q = torch.empty((batch, H, seq_len, 64), dtype=bf16, device=d)
        if kv_buffers is None:
            # zeros: attention reads whole 128-key tiles and needs finite V
            # past kv_len (the keys there are masked)
            k = torch.zeros((batch, H, kv_len, 64), dtype=bf16, device=d)
            vt = torch.zeros((batch, H, 64, kv_len), dtype=torch.float16, device=d)
            kv_buffers = [(k, vt)] * len(self.blocks)
        self.kv_buffers = kv_buffers
        self.kv_stride = kv_buffers[0][0].shape[2]
        if kv_offset + seq_len > self.kv_stride or kv_len > self.kv_stride:
            raise ValueError("K / V buffers too short")
        self.attn = torch.empty((M, 768), dtype=bf16, device=d)
        self.mlp = torch.empty((M, 3072), dtype=bf16, device=d)
        self.row_amax = torch.zeros(M, dtype=torch.int32, device=d)  # MLP-up row amax (cleared by its quantiser)
        # head input (gathered rows) and loop state
        self.head_q = torch.empty((M, 768), dtype=torch.int8, device=d)
        self.head_scale = torch.empty(M, dtype=torch.float32, device=d)
        self.packed = torch.zeros(M, dtype=torch.int64, device=d)
        W = (seq_len + 63) // 64
        u32 = torch.int32
        self.tokens = torch.empty(M, dtype=torch.int32, device=d)
        self.ids_in = torch.empty(M, dtype=torch.int32, device=d)  # input canvas of the composite loop
        self.active = torch.empty(batch * W, dtype=torch.int64, device=d)
        self.need_eval = torch.empty(batch, dtype=u32, device=d)
        self.eval_id = torch.empty(batch, dtype=u32, device=d)
        self.fwd_rows = torch.full((1,), M, dtype=u32, device=d)
        self.sel_count = torch.zeros(1, dtype=u32, device=d)
        self.sel_rows = torch.empty(M, dtype=u32, device=d)
        self.sel_pos = torch.empty(M, dtype=u32, device=d)
        self.sel_key = torch.empty(M, dtype=u32, device=d)
        self.sel_eval = torch.empty(M, dtype=u32, device=d)
        self.counters: Optional[Any] = None
        self._counters: Dict[int, Any] = {}  # per step count: captured graphs keep their buffer
        self._native: Optional[tuple] = None   # (dh_mdlm_weights, its block array)
        self._loop_ws: Optional[Any] = None    # workspace of dh_sample_loop
        self.seq_offset = 0  # global index of local sequence 0 (Philox key_hi)
        self.head_vocab_offset = 0  # global id of the first head row held here (vocab-sharded head)
        self.head_group = None      # process group reducing the sharded head, or None
        self.head_reduce = None     # callable(packed) merging shard results (testing / custom groups)
        self.pre_forward = None     # callable(fwd_rows) enqueued before each transition's forward
        # forward only the sequences that refill (True), the whole batch when
        # one does (False), or choose per generation (None): packing pays when
        # sequences often go a transition without a change, i.e. when the
        # expected reveals per transition L / steps are few
        self.compact: Optional[bool] = None
        self._compact_now = False
        self._compact_bufs: Optional[tuple] = None  # seq_list, per-row head input and scale
        self._graphs: Dict[Any, Any] = {}
        self._events = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
        self.launches_per_forward = 1 + 9 * len(self.blocks)

    def shard_head(self, v0: int, v1: int, group: Any = None, reduce: Any = None) -> None:
        """Keep only head rows [v0, v1) (vocab-sharded head).  After every head
        launch the packed per-row results are MAX-reduced over `group` (or
        passed to `reduce`), so each rank commits the unsharded argmax."""
        if v0 % 4:
            raise ValueError("shard start must be a multiple of 4")
        h = self.head
        h.w = h.w[v0:v1].contiguous()
        h.w_scale = h.w_scale[v0:v1].contiguous()
        h.bias = h.bias[v0:v1].contiguous()
        h.out_features = v1 - v0
        self.head_vocab_offset = v0
        self._native = None
        self.head_group = group
        self.head_reduce = reduce

    @staticmethod
    def kv_cache(qm: QuantizedMDLM, batch: int, kv_stride: int, device: Any = "cuda") -> List[tuple]:
        """Per-block K [B, 12, kv_stride, 64] bf16 and V^T [B, 12, 64, kv_stride]
        f16 (zero-filled: positions not yet written must hold finite V)."""
        import torch

        return [(torch.zeros((batch, 12, kv_stride, 64), dtype=torch.bfloat16, device=device),
                 torch.zeros((batch, 12, 64, kv_stride), dtype=torch.float16, device=device))
                for _ in qm.blocks]

    # ------------------------------------------------------------ forward

    def _p(self, t):
        return _lib.ptr(t)

    @_on_device
    def forward(self, tokens: Any = None, run_rows: Any = None, hook: Any = None, seq_list: Any = None) -> None:
        """Forward over self.tokens (or `tokens`, int32 [M] on the device);
        leaves the residual stream in self.x.  run_rows: device word, only
        its first *run_rows rows are computed (0: none).  seq_list: the rows
        are the packed positions of the listed sequences.  hook(i) runs after
        block i."""
        s = _lib.stream_handle()
        tok = self.tokens if tokens is None else tokens
        rr = self._p(run_rows) if run_rows is not None else None
        if seq_list is not None:
            _lib.call("dh_embed_gather_seqs", self._p(tok), self._p(seq_list), self.L, self._p(self.embedding),
                      self._p(self.x), self.M, self.cfg.vocab_size, rr, s)
        else:
            _lib.call("dh_embed_gather", self._p(tok), self._p(self.embedding), self._p(self.x), self.M,
                      self.cfg.vocab_size, rr, s)
        for i, blk in enumerate(self.blocks):
            self._forward_block(i, blk, rr, s)
            if hook is not None:
                hook(i)

    def _forward_block(self, i: int, blk: dict, rr: Any, s: Any) -> None:
        M, L = self.M, self.L
        p = self._p
        call = _lib.call
        k, vt = self.kv_buffers[i]
        qkv, out, up, down = blk["qkv"], blk["out"], blk["up"], blk["down"]
        call("dh_ln_smooth_quant", p(self.x), p(qkv.smooth), p(qkv.inv_smooth), p(self.act_q), p(self.act_scale), M,
             None, None, rr, s)
        call("dh_gemm_qkv_rope", p(self.act_q), p(self.act_scale), p(qkv.w), p(qkv.w_scale), p(qkv.bias),
             p(self.rope_cos), p(self.rope_sin), p(out.inv_smooth), M, L, self.pos_offset, self.kv_stride, self.kv_offset,
             p(self.q), p(k), p(vt), rr, s)
        call("dh_attention", p(self.q), p(k), p(vt), p(self.attn), self.B, L, self.kv_len, self.kv_stride,
             rr, s)
        call("dh_quant_rows_bf16", p(self.attn), None, None, p(self.act_q), p(self.act_scale), M,
             768, rr, s)
        call("dh_gemm_residual", p(self.act_q), p(self.act_scale), p(out.w), p(out.w_scale), p(out.bias),
             p(self.x), M, 768, 768, rr, s)
        call("dh_ln_smooth_quant", p(self.x), p(up.smooth), p(up.inv_smooth), p(self.act_q), p(self.act_scale), M,
             None, None, rr, s)
        call("dh_gemm_gelu", p(self.act_q), p(self.act_scale), p(up.w), p(up.w_scale), p(up.bias),
             p(down.inv_smooth), p(self.mlp), p(self.row_amax), M, 3072, 768, rr, s)
        call("dh_quant_rows_bf16_amax", p(self.mlp), p(self.row_amax), p(self.act_q), p(self.act_scale), M,
             3072, rr, s)
        call("dh_gemm_residual", p(self.act_q), p(self.act_scale), p(down.w), p(down.w_scale),
             p(down.bias), p(self.x), M, 768, 3072, rr, s)

    @_on_device
    def final_hidden_q(self, rows_index: Any = None, rows_count: Any = None):
        """Final LayerNorm + head SmoothQuant + int8 of (selected) rows."""
        s = _lib.stream_handle()
        _lib.call("dh_ln_smooth_quant", self._p(self.x), self._p(self.head.smooth), self._p(self.head.inv_smooth),
                  self._p(self.head_q), self._p(self.head_scale), self.M,
                  self._p(rows_index) if rows_index is not None else None,
                  self._p(rows_count) if rows_count is not None else None, None, s)
        return self.head_q, self.head_scale

    @_on_device
    def logits(self) -> Any:
        """fp32 logits [B, L, V] of the last forward: a debug / drift-analysis
        path (the samplers never materialise logits).  int32 accumulators of
        the int8 head from the tensor-core GEMM, then the reference dequant
        out = fp32(acc * fp64(a_scale * w_scale) + bias)
        (fixed_mlp.quantized_linear, fixed_mlp.py:120-136)."""
        torch = self.torch
        hq, hs = self.final_hidden_q()
        h = self.head
        V = h.out_features
        acc = torch.empty((self.M, V), dtype=torch.int32, device=self.device)
        _lib.call("dh_gemm_i8_s32", self._p(hq), 768, self._p(h.w), 768, self._p(acc), V, self.M, V, 768,
                  _lib.stream_handle())
        combined = (hs[:, None] * h.w_scale[None, :]).double()
        out = (acc.double() * combined + h.bias.double()[None, :]).float()
        return out.view(self.B, self.L, V)

    @_on_device
    def selected_logits(self, input_ids: Any, selected: Any) -> Any:
        """fp32 logits [n, V] of the selected positions of a single-sequence
        canvas (apple_mdlm._AppleSelectedLogits, apple_mdlm.py:159-200): the
        forward over the whole canvas, then the final LayerNorm, quantisation
        and head GEMM of the selected rows only, dequantised as
        fixed_mlp.quantized_linear (fixed_mlp.py:120-136)."""
        torch = self.torch
        if self.B != 1 or input_ids.numel() != self.L:
            raise ValueError("selected_logits takes one sequence of the engine's length")
        self.tokens.copy_(input_ids.reshape(-1).to(device=self.device, dtype=torch.int32))
        self.forward()
        rows = selected.reshape(-1).to(device=self.device, dtype=torch.int32).contiguous()
        n = rows.numel()
        if n == 0 or int(rows.min()) < 0 or int(rows.max()) >= self.L:
            raise ValueError("selected positions must be non-empty and inside the canvas")
        cnt = torch.tensor([n], dtype=torch.int32, device=self.device)
        hq, hs = self.final_hidden_q(rows, cnt)
        h = self.head
        V = h.out_features
        acc = torch.empty((n, V), dtype=torch.int32, device=self.device)
        _lib.call("dh_gemm_i8_s32", self._p(hq), 768, self._p(h.w), 768, self._p(acc), V, n, V, 768,
                  _lib.stream_handle())
        combined = (hs[:n, None] * h.w_scale[None, :]).double()
        return (acc.double() * combined + h.bias.double()[None, :]).float()

    @_on_device
    def head_argmax(self, rows: int, mode: int, rows_count: Any = None, row_position: Any = None,
                    row_key_hi: Any = None, row_eval: Any = None, key_lo: int = 0,
                    out_ids: Any = None, out_scores: Any = None, const_eval: int = 0) -> None:
        s = _lib.stream_handle()
        h = self.head
        _lib.call("dh_head_argmax_i8", self._p(self.head_q), 768, self._p(h.w), 768, rows,
                  self._p(rows_count) if rows_count is not None else None, 768, h.out_features,
                  self.head_vocab_offset, self.cfg.mask_token_id, mode, self._p(self.head_scale), self._p(h.w_scale),
                  self._p(h.bias), None, None, None, self._p(row_position), self._p(row_key_hi),
                  self._p(row_eval), const_eval, key_lo, 0, self._p(self.packed), self._p(out_ids),
                  self._p(out_scores), s)

    # ------------------------------------------------------------- loop

    @_on_device
    def enqueue_transition(self, k: int, steps: int, seed: int, threshold_q32: int) -> None:
        """Transition k of `steps` (k == steps: the final greedy pass)."""
        s = _lib.stream_handle()
        B, L = self.B, self.L
        p = self._p
        call = _lib.call
        final = 1 if k == steps else 0
        kk = min(k, steps - 1)
        seqs = self._compact_buffers()[0] if self._compact_now else None
        call("dh_loop_plan_seqs", B, L, kk, steps, final, p(self.active), p(self.need_eval), p(self.eval_id),
             p(self.fwd_rows), p(self.sel_count), p(self.counters), p(seqs), s)
        if self.pre_forward is not None:
            self.pre_forward(self.fwd_rows)
        self.forward(run_rows=self.fwd_rows, seq_list=seqs)
        if seqs is not None:
            _, head_all, head_all_scale = self._compact_buffers()
            call("dh_ln_smooth_quant_scatter", p(self.x), p(self.head.smooth), p(self.head.inv_smooth),
                 p(head_all), p(head_all_scale), self.M, p(seqs), L, p(self.fwd_rows), s)
        call("dh_loop_select", B, L, kk, seed, self.seq_offset, self.pos_offset, 0 if final else threshold_q32,
             final,
             p(self.active), p(self.eval_id), p(self.sel_rows), p(self.sel_pos), p(self.sel_key),
             p(self.sel_eval), p(self.sel_count), s)
        if seqs is not None:
            call("dh_gather_rows_i8", p(head_all), p(head_all_scale), p(self.sel_rows), p(self.sel_count), self.M,
                 p(self.head_q), p(self.head_scale), s)
        else:
            self.final_hidden_q(self.sel_rows, self.sel_count)
        self.head_argmax(self.M, 2 if final else 1, rows_count=self.sel_count, row_position=self.sel_pos,
                         row_key_hi=self.sel_key, row_eval=self.sel_eval, key_lo=seed)
        if self.head_reduce is not None:
            self.head_reduce(self.packed)
        elif self.head_group is not None:
            from .distributed import all_reduce_packed_max_

            all_reduce_packed_max_(self.packed, self.head_group)
        call("dh_loop_commit", B, L, kk, steps, final, p(self.packed), p(self.sel_rows), p(self.sel_count),
             p(self.tokens), p(self.active), p(self.need_eval), p(self.counters), s)

    def _compact_buffers(self) -> tuple:
        if self._compact_bufs is None:
            torch = self.torch
            self._compact_bufs = (torch.empty(self.B, dtype=torch.int32, device=self.device),
                                  torch.empty((self.M, 768), dtype=torch.int8, device=self.device),
                                  torch.empty(self.M, dtype=torch.float32, device=self.device))
        return self._compact_bufs

    def compact_for(self, steps: int) -> bool:
        """Whether a `steps`-transition generation packs the forward to the
        refilling sequences: as set in `compact`, else when the batch holds
        several sequences and fewer than 4 reveals per transition are expected
        (L < 4 steps), so that a sequence often goes a transition unchanged."""
        if self.compact is not None:
            return bool(self.compact)
        return self.B > 1 and self.L < 4 * steps

    def _enqueue_generation(self, steps: int, seed: int, thresholds: List[int]) -> None:
        for k in range(steps + 1):
            self.enqueue_transition(k, steps, seed, thresholds[k] if k < steps else 0)

    def _use_counters(self, steps: int) -> Any:
        """The per-transition counters of a `steps`-transition generation.
        One buffer per step count, kept for the engine's life: a captured
        graph holds the address it was captured with."""
        c = self._counters.get(steps)
        if c is None:
            c = self.torch.zeros(3 * steps, dtype=self.torch.int32, device=self.device)
            self._counters[steps] = c
        self.counters = c
        return c

    @_on_device
    def init_loop(self, input_ids: Any, steps: int) -> None:
        """Load ids [B, L] (device) and reset the loop state."""
        torch = self.torch
        self._use_counters(steps)
        ids = input_ids.to(device=self.device, dtype=torch.int32).contiguous().view(-1)
        if ids.numel() != self.M:
            raise ValueError("input_ids must be [batch, seq_len]")
        self._ids_in = ids
        _lib.call("dh_loop_init", _lib.ptr(ids), self.B, self.L, self.cfg.mask_token_id, steps,
                  _lib.ptr(self.tokens), _lib.ptr(self.active), _lib.ptr(self.need_eval),
                  _lib.ptr(self.eval_id), _lib.ptr(self.counters), _lib.stream_handle())

    # ------------------------------------------- composite (C-ABI) loop

    def native_weights(self) -> Any:
        """dh_mdlm_weights over this engine's device tensors (built once; the
        engine keeps the structs and the tensors alive)."""
        if self._native is None:
            p = _lib.ptr

            def lin(d: _DevLinear) -> Any:
                return _lib.LinearWeights(p(d.w), p(d.w_scale), p(d.bias), p(d.smooth), p(d.inv_smooth))

            names = ("qkv", "out", "up", "down")
            arr = (_lib.LinearWeights * (4 * len(self.blocks)))(*[lin(b[n]) for b in self.blocks for n in names])
            w = _lib.MDLMWeights(len(self.blocks), self.cfg.vocab_size, self.cfg.mask_token_id,
                                 int(self.rope_cos.shape[0]), p(self.embedding), p(self.rope_cos), p(self.rope_sin),
                                 ctypes.cast(arr, ctypes.POINTER(_lib.LinearWeights)), lin(self.head),
                                 self.head.out_features, self.head_vocab_offset)
            self._native = (w, arr)
        return self._native[0]

    def _nccl_comm(self) -> Any:
        if self.head_group is None:
            return None
        from .distributed import nccl_comm_handle

        return nccl_comm_handle(self.head_group, self.device)

    def native_loop_ok(self) -> bool:
        """Whether dh_sample_loop covers this engine's configuration: whole
        canvases (no prefix K/V offsets), no Python hooks, and a head that is
        whole or merged over NCCL."""
        if self.pre_forward is not None or self.head_reduce is not None:
            return False
        if self.pos_offset or self.kv_offset or self.kv_len != self.L or self.kv_stride != self.L:
            return False
        return self.head_group is None or self._nccl_comm() is not None

    def _enqueue_native(self, steps: int, seed: int, thresholds: List[int]) -> None:
        torch = self.torch
        if self._loop_ws is None:
            size = _lib.lib().dh_sample_loop_workspace_size(self.B, self.L)
            self._loop_ws = torch.empty(size, dtype=torch.uint8, device=self.device)
        thr = (ctypes.c_uint64 * steps)(*thresholds[:steps])
        w = self.native_weights()
        _lib.call("dh_sample_loop", ctypes.addressof(w), _lib.ptr(self.ids_in), _lib.ptr(self.tokens), self.B,
                  self.L, steps, ctypes.addressof(thr), seed, self.seq_offset, _lib.ptr(self.counters),
                  self._nccl_comm(), 1 if self._compact_now else 0, _lib.ptr(self._loop_ws), self._loop_ws.numel(),
                  _lib.stream_handle())

    def launches_per_generation(self, steps: int) -> int:
        """Kernels one generation launches (the loop set-up, then per
        transition: plan, the forward, select, the head's input rows, the head
        (zeroing + fused GEMM) and commit).  The composite loop over an
        unpacked batch stops the forward after the last block's attention (six
        launches fewer) and finishes that block for the revealed rows: two row
        gathers, the block's six remaining kernels and the final LayerNorm.
        Packed, the head input is also scattered per sequence."""
        compact = self.compact_for(steps)
        per_transition = 1 + self.launches_per_forward + 1 + 1 + 2 + 1 + (1 if compact else 0)
        if self.native_loop_ok() and not compact:
            per_transition += -6 + (2 + 6 + 1) - 1
        return 1 + (steps + 1) * per_transition

    @_on_device
    def generate(self, input_ids: Any, *, steps: int, seed: int = 0, sampling_epsilon: float = 1e-5,
                 graph: bool = False, native: Optional[bool] = None) -> tuple[Any, dict]:
        """Candidate-cache generation of B sequences (input_ids int [B, L],
        any device).  native: run the loop through the composite entry point
        dh_sample_loop (default when native_loop_ok()), else through the
        per-kernel entry points from Python.  Both launch the same kernels
        with the same arguments.  Returns (device int32 ids [B, L],
        metadata)."""
        torch = self.torch
        thresholds = reveal_thresholds_q32(steps, sampling_epsilon)
        native = self.native_loop_ok() if native is None else native
        self._compact_now = self.compact_for(steps)
        if native:
            if input_ids.numel() != self.M:
                raise ValueError("input_ids must be [batch, seq_len]")
            self.ids_in.copy_(input_ids.reshape(-1))
            self._use_counters(steps)

            def enqueue() -> None:
                self._enqueue_native(steps, seed, thresholds)
        else:
            self.init_loop(input_ids, steps)

            def enqueue() -> None:
                self._enqueue_generation(steps, seed, thresholds)
        if graph:
            key = (native, self._compact_now, steps, seed, sampling_epsilon, self.seq_offset)
            g = self._graphs.get(key)
            if g is None:
                # warm-up outside capture (function attributes, tensor maps)
                enqueue()
                if not native:
                    self.init_loop(input_ids, steps)
                torch.cuda.synchronize()
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    enqueue()
                self._graphs[key] = g
            self._events[0].record()
            g.replay()
            self._events[1].record()
        else:
            self._events[0].record()
            enqueue()
            self._events[1].record()
        return self.tokens.view(self.B, self.L), {}

    # ------------------------------------------------- event-driven loop

    @_on_device
    def _load_schedule(self, sched: Any) -> Any:
        """Copy a host EventSchedule into the selected-row buffers: rows,
        canvas positions, Philox key_hi and per-transition counts."""
        torch = self.torch
        if (sched.sequences, sched.positions) != (self.B, self.L):
            raise ValueError(f"schedule must cover [{self.B}, {self.L}]")
        n = int(sched.order.numel())
        order = sched.order
        b = order // self.L
        p = order % self.L
        host = torch.stack([order, self.pos_offset + p, self.seq_offset + b]).to(torch.int32)
        if n:
            self.sel_rows[:n].copy_(host[0])
            self.sel_pos[:n].copy_(host[1])
            self.sel_key[:n].copy_(host[2])
        counts = getattr(self, "_event_counts", None)
        if counts is None or counts.numel() != sched.steps + 1:
            counts = torch.empty(sched.steps + 1, dtype=torch.int32, device=self.device)
            self._event_counts = counts
        counts.copy_(torch.tensor([sched.count(k) for k in range(sched.steps + 1)], dtype=torch.int32))
        return counts

    def _enqueue_event_generation(self, sched: Any, seed: int, counts: Any) -> None:
        s = _lib.stream_handle()
        B, L, steps = self.B, self.L, sched.steps
        p = self._p
        for k in range(steps + 1):
            if sched.count(k) == 0:
                continue
            off = sched.offsets[k]
            final = 1 if k == steps else 0
            rows, cnt = self.sel_rows[off:], counts[k:k + 1]
            self.forward()
            self.final_hidden_q(rows, cnt)
            self.head_argmax(self.M, 2 if final else 1, rows_count=cnt, row_position=self.sel_pos[off:],
                             row_key_hi=self.sel_key[off:], const_eval=k, key_lo=seed)
            if self.head_reduce is not None:
                self.head_reduce(self.packed)
            elif self.head_group is not None:
                from .distributed import all_reduce_packed_max_

                all_reduce_packed_max_(self.packed, self.head_group)
            _lib.call("dh_loop_commit", B, L, min(k, steps - 1), steps, final, p(self.packed), p(rows), p(cnt),
                      p(self.tokens), p(self.active), p(self.need_eval), p(self.counters), s)

    @_on_device
    def generate_event_driven(self, input_ids: Any, sched: Any, *, seed: int = 0,
                              graph: bool = False) -> Any:
        """Event-driven generation (apple_mdlm.py:62-156, batched): only the
        transitions of `sched` (an event.EventSchedule over [B, L]) that reveal
        a row run a forward, and the head projects only those rows; the final
        pass takes the greedy argmax.  Returns device int32 ids [B, L]."""
        torch = self.torch
        self.init_loop(input_ids, sched.steps)
        counts = self._load_schedule(sched)
        if graph:
            key = ("event", sched.steps, seed, self.seq_offset, tuple(sched.offsets))
            g = self._graphs.get(key)
            if g is None:
                self._enqueue_event_generation(sched, seed, counts)
                self.init_loop(input_ids, sched.steps)
                torch.cuda.synchronize()
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    self._enqueue_event_generation(sched, seed, counts)
                self._graphs[key] = g
            self._events[0].record()
            g.replay()
            self._events[1].record()
        else:
            self._events[0].record()
            self._enqueue_event_generation(sched, seed, counts)
            self._events[1].record()
        return self.tokens.view(self.B, self.L)

    def generation_ms(self) -> float:
        """Device time of the last generate() (the loop only, CUDA events)."""
        self._events[1].synchronize()
        return float(self._events[0].elapsed_time(self._events[1]))

    def measurements(self, steps: int, sampling_epsilon: float = 1e-5) -> list:
        """The reference's per-evaluation records of the last generation
        (mdlm.py:1133-1200): one MDLMStepMeasurement per transition that ran a
        model evaluation, then the final greedy pass when masks remained.
        sigma_t = -log1p(-(1 - 1e-3) t_k) in float32 as the reference computes
        it.  The loop runs as one device program, so elapsed_s is the
        generation's device time divided evenly over the evaluations."""
        torch = self.torch
        meta = self.metadata(steps)
        counters = self.counters.view(steps, 3).cpu().tolist()
        n = meta["sampling_transitions"]
        t = torch.linspace(1.0, sampling_epsilon, steps + 1)
        sigma = (-torch.log1p(-(1 - NOISE_EPSILON) * t)).tolist()
        evaluations = max(1, meta["model_evaluations"])
        per_eval = self.generation_ms() / 1e3 / evaluations
        out = [MDLMStepMeasurement(k, counters[k][0], counters[k][1], per_eval, float(sigma[k]))
               for k in range(n) if counters[k][2]]
        remaining = counters[n - 1][0] - counters[n - 1][1] if n else 0
        if remaining > 0:
            final_sigma = float(-torch.log1p(-(1 - NOISE_EPSILON) * torch.tensor([sampling_epsilon])).item())
            out.append(MDLMStepMeasurement(n, remaining, remaining, per_eval, final_sigma))
        return out

    def metadata(self, steps: int) -> dict:
        counters = self.counters.view(steps, 3).cpu().tolist()
        active = [c[0] for c in counters if c[0] > 0]
        n = len(active)
        changed = [c[1] for c in counters[:n]]
        evaluated = [c[2] for c in counters[:n]]
        remaining_before_final = active[-1] - changed[-1] if n else 0
        evaluations = sum(evaluated) + (1 if remaining_before_final > 0 else 0)
        cache_bytes, id_bytes = hardware_candidate_cache_bytes(self.M, self.cfg.mask_token_id)
        return {
            "sampling_transitions": n,
            "model_evaluations": evaluations,
            "probability_cache_hits": n - sum(evaluated),
            "candidate_cache_hits": n - sum(evaluated),
            "transition_active_tokens": active,
            "transition_changed_tokens": changed,
            "cache_hit_sampling_overhead_modeled": False,
            "cache_correctness_class": "distribution-equivalent",
            "hardware_candidate_cache_bytes": cache_bytes,
            "candidate_id_bytes": id_bytes,
        }
