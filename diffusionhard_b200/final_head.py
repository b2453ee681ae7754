"""The output head with a per-sequence conditioning vector: the final layer of
the DDiT unfolded (mlx_mdlm._FinalLayer, mlx_mdlm.py:456-498) followed by the
fused int8 head and the Philox-Gumbel noisy argmax.

For every masked position of a [B, L] canvas: LayerNorm of the bf16 hidden
row, adaLN modulation h = n (1 + scale_b) + shift_b with [shift | scale] =
adaLN(cond_b), per-token int8 (fixed_mlp._quantize_symmetric), the int8
768 x V projection and the race round_half_even(logit * 1024) +
gumbel_q10(philox((v/4, p, 0, 0), (seed, b))[v % 4]) with the mask token
skipped.  Four launches on one stream, no host synchronisation: adaLN,
masked-row compaction (dh_loop_init / dh_loop_select), LayerNorm + modulation
+ quantisation of the masked rows, head.  Logits never reach HBM.
"""

from __future__ import annotations

from typing import Any, Optional

import numpy as np

from . import _lib


class ConditionedHead:
    """Device weights and buffers for canvases of `batch` x `seq_len`.

    weight_q int8 [V, 768], w_scale / bias fp32 [V], ada_weight fp32
    [1536, C], ada_bias fp32 [1536] or None, ln_weight fp32 [768] or None
    (ones)."""

    def __init__(self, weight_q: np.ndarray, w_scale: np.ndarray, bias: np.ndarray, ada_weight: np.ndarray,
                 ada_bias: Optional[np.ndarray], ln_weight: Optional[np.ndarray], mask_token_id: int, batch: int,
                 seq_len: int, device: Any = "cuda") -> None:
        import torch

        self.torch = torch
        d = torch.device(device)
        if d.index is None:
            d = torch.device("cuda", torch.cuda.current_device())
        self.device = d
        f32 = lambda a: None if a is None else torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(d)  # noqa: E731
        self.w = torch.from_numpy(np.ascontiguousarray(weight_q, np.int8)).to(d)
        self.w_scale, self.bias = f32(w_scale), f32(bias)
        self.ada_w, self.ada_b, self.ln_w = f32(ada_weight), f32(ada_bias), f32(ln_weight)
        self.V, self.C = int(self.w.shape[0]), int(self.ada_w.shape[1])
        if self.w.shape[1] != 768 or self.ada_w.shape[0] != 1536:
            raise ValueError("the head is 768 wide and the modulation 2 x 768")
        self.mask = mask_token_id
        self.B, self.L = batch, seq_len
        M = batch * seq_len
        i32 = torch.int32
        self.modulation = torch.empty((batch, 1536), dtype=torch.float32, device=d)
        self.ids_in = torch.empty(M, dtype=i32, device=d)
        self.tokens = torch.empty(M, dtype=i32, device=d)
        self.active = torch.empty(batch * ((seq_len + 63) // 64), dtype=torch.int64, device=d)
        self.need_eval = torch.empty(batch, dtype=i32, device=d)
        self.eval_id = torch.empty(batch, dtype=i32, device=d)
        self.counters = torch.zeros(3, dtype=i32, device=d)
        self.sel_rows = torch.empty(M, dtype=i32, device=d)
        self.sel_pos = torch.empty(M, dtype=i32, device=d)
        self.sel_key = torch.empty(M, dtype=i32, device=d)
        self.sel_eval = torch.empty(M, dtype=i32, device=d)
        self.sel_count = torch.zeros(1, dtype=i32, device=d)
        self.head_q = torch.empty((M, 768), dtype=torch.int8, device=d)
        self.head_scale = torch.empty(M, dtype=torch.float32, device=d)
        self.packed = torch.zeros(M, dtype=torch.int64, device=d)
        self.out_ids = torch.empty(M, dtype=i32, device=d)

    def load_mask(self, masked: Any) -> None:
        """masked: bool [B, L] (any device): the positions that need a
        candidate."""
        torch = self.torch
        ids = torch.where(masked.to(self.device), self.mask, 0).to(torch.int32)
        self.ids_in.copy_(ids.reshape(-1))

    def enqueue(self, hidden: Any, cond: Any, seed: int = 0) -> None:
        """hidden: bf16 [B, L, 768], cond: fp32 [B, C], both on the device;
        the masked rows come from the last load_mask.  Results: out_ids[:n]
        (token ids in position-major order of the masked rows, n = sel_count)
        and sel_rows[:n] (their b * L + p)."""
        p, s, call = _lib.ptr, _lib.stream_handle(), _lib.call
        B, L, M = self.B, self.L, self.B * self.L
        call("dh_adaln_modulation", p(cond), p(self.ada_w), p(self.ada_b), p(self.modulation), B, self.C, 1536, s)
        call("dh_loop_init", p(self.ids_in), B, L, self.mask, 1, p(self.tokens), p(self.active), p(self.need_eval),
             p(self.eval_id), p(self.counters), s)
        call("dh_loop_select", B, L, 0, seed, 0, 0, 0, 1, p(self.active), p(self.eval_id), p(self.sel_rows),
             p(self.sel_pos), p(self.sel_key), p(self.sel_eval), p(self.sel_count), s)
        call("dh_ln_modulate_quant_bf16", p(hidden), p(self.ln_w), p(self.modulation), L, p(self.sel_rows),
             p(self.sel_count), M, p(self.head_q), p(self.head_scale), s)
        call("dh_head_argmax_i8", p(self.head_q), 768, p(self.w), 768, M, p(self.sel_count), 768, self.V, 0,
             self.mask, 1, p(self.head_scale), p(self.w_scale), p(self.bias), None, None, None, p(self.sel_pos),
             p(self.sel_key), p(self.sel_eval), 0, seed, 0, p(self.packed), p(self.out_ids), None, s)

    def candidates(self, hidden: Any, cond: Any, masked: Any, seed: int = 0) -> tuple[Any, Any]:
        """(rows b * L + p, token ids) of the masked positions, on the host."""
        with self.torch.cuda.device(self.device):
            self.load_mask(masked)
            self.enqueue(hidden, cond, seed)
            n = int(self.sel_count.item())
            return self.sel_rows[:n].cpu().numpy(), self.out_ids[:n].cpu().numpy()
