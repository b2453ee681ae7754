"""CPU oracle of the W8A8 DDiT forward.  TEST INFRASTRUCTURE ONLY.

Restates, in torch-CPU float32 / float64, the reference arithmetic:
  * W8A8 linear with static SmoothQuant scales: fixed_mlp.quantized_linear
    (src/diffusion_accel/fixed_mlp.py:65-136; _quantize_symmetric :11-35),
    with the activation amax of the smoothing scale taken from calibration
    instead of the live batch (the static pattern of fixed_attention.py:410-420);
  * the folded DDiT block and final layer: hardware_package.folded_mdlm_forward
    (hardware_package.py:195-289), mlx_mdlm._DDiTBlock (mlx_mdlm.py:397-453);
  * rotate-half rotary (mlx_mdlm.py:316-329) and fp32 SDPA with scale 1/8;
  * prefix-cached suffix forward (prefix_drift._cached_suffix_forward,
    prefix_drift.py:155-238) over K/V = [prefix ; suffix];
  * block-causal attention (mdlm.block_isolation, mdlm.py:61-77, applied as
    the additive -inf bias of mdlm.py:424-441): a row of a completed block
    attends to its own and earlier blocks; rows after the last boundary form
    the active bidirectional block.
Pinned to the reference in tests/test_model_oracle.py (golden fixtures made by
tests/golden/make_model_golden.py from the reference's own functions).
"""

from __future__ import annotations

from typing import Dict, List, Optional, Tuple

import numpy as np


# When True, the int8 product uses torch._int_mm -- the reference's own CPU
# path (fixed_mlp._integer_matmul, fixed_mlp.py:55-62); otherwise an exact
# float64 matmul (identical int32 results, no int8 kernel needed).
USE_INT_MM = False


def quantize_rows(a, smooth=None):
    """Per-token symmetric int8 of fp32 rows a [R, C], after division by the
    SmoothQuant scale when given: fixed_mlp._quantize_symmetric(a / s, 8,
    "token") (fixed_mlp.py:11-35; quantized_linear divides by s first,
    :82-96).  Returns (int8 [R, C], fp32 row scales [R])."""
    import torch

    if smooth is not None:
        a = a / torch.as_tensor(smooth, dtype=torch.float32)[None, :]
    maximum = a.abs().amax(dim=1)
    scale = torch.where(maximum > 0, maximum / 127.0, torch.ones_like(maximum))
    q = torch.round(a / scale[:, None]).clamp(-127, 127).to(torch.int8)
    return q, scale


def w8a8_linear(a, ql, return_parts: bool = False):
    """Reference quantized_linear arithmetic with a static smoothing scale."""
    import torch

    q, scale = quantize_rows(a, ql.smooth)
    w_scale = torch.from_numpy(ql.w_scale)
    if USE_INT_MM:
        wq = getattr(ql, "_wq_t", None)
        if wq is None:
            wq = torch.from_numpy(ql.weight_q).t().contiguous()
            ql._wq_t = wq
        acc = torch._int_mm(q.contiguous(), wq).to(torch.int64)
    else:
        acc = torch.matmul(q.double(), torch.from_numpy(ql.weight_q).double().t()).to(torch.int64)
    combined = scale[:, None] * w_scale[None, :]
    out = (acc.double() * combined.double() + torch.from_numpy(ql.bias).double()[None, :]).float()
    if return_parts:
        return out, q, scale, acc
    return out


def _rot(t, cos, sin):
    import torch

    h = t.shape[-1] // 2
    a, b = t[..., :h], t[..., h:]
    return torch.cat((a * cos - b * sin, b * cos + a * sin), dim=-1)


def block_causal_bias(length: int, block_ends):
    """Additive attention bias [L, L] of mdlm.py:424-441: for consecutive
    completed blocks [start, end), keys at or after `end` are -inf."""
    import torch

    bias = torch.zeros((length, length), dtype=torch.float32)
    start = 0
    for end in (min(int(e), length) for e in block_ends if int(e) > 0):
        bias[start:end, end:] = -torch.inf
        start = end
    return bias


def forward(qm, ids: np.ndarray, *, positions: Optional[np.ndarray] = None,
            prefix_kv: Optional[List[Tuple[object, object]]] = None, capture_kv: bool = False,
            record: Optional[Dict[str, object]] = None, block_ends: Optional[List[int]] = None,
            ln_fp64: bool = False):
    """W8A8 forward of `ids` [B, L].  Returns the final LayerNorm output [B, L, d].

    ln_fp64: compute every LayerNorm in float64 and round its output to
        float32 -- the same arithmetic with other rounding, which measures how
        far two CPU evaluations of the reference agree.

    positions: rotary positions of the rows (default 0..L-1).
    block_ends: completed block boundaries for block-causal attention.
    prefix_kv: per block (K_rot, V) [B, P, H, 64] prepended to the keys/values.
    capture_kv: store per-block (K_rot, V) of these rows in record["kv"].
    record: optional dict receiving "x{i}" (residual after block i),
        "head_q" / "head_scale" (int8 head input and its row scales).
    """
    import torch
    import torch.nn.functional as F

    cfg = qm.config
    B, L = ids.shape
    pos = np.arange(L) if positions is None else positions

    def layer_norm(t, shape):
        return F.layer_norm(t.double(), shape).float() if ln_fp64 else F.layer_norm(t, shape)

    cos = torch.from_numpy(qm.rope_cos[pos])[None, :, None, :]
    sin = torch.from_numpy(qm.rope_sin[pos])[None, :, None, :]
    kv = []
    bias = block_causal_bias(L, block_ends) if block_ends else None
    if bias is not None and prefix_kv is not None:
        raise ValueError("block_ends apply to a whole-sequence forward")
    with torch.no_grad():
        x = torch.from_numpy(qm.embedding)[torch.from_numpy(ids.astype(np.int64))]
        for i, blk in enumerate(qm.blocks):
            h = layer_norm(x, [cfg.hidden]).reshape(B * L, cfg.hidden)
            qkv = w8a8_linear(h, blk["qkv"]).view(B, L, 3, cfg.heads, cfg.head_dim)
            q, k, v = qkv.unbind(dim=2)
            q, k = _rot(q, cos, sin), _rot(k, cos, sin)
            if capture_kv:
                kv.append((k.clone(), v.clone()))
            if prefix_kv is not None:
                k = torch.cat([prefix_kv[i][0], k], dim=1)
                v = torch.cat([prefix_kv[i][1], v], dim=1)
            a = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                               attn_mask=bias)
            a = a.transpose(1, 2).reshape(B * L, cfg.hidden)
            x = x + w8a8_linear(a, blk["out"]).view(B, L, cfg.hidden)
            h = layer_norm(x, [cfg.hidden]).reshape(B * L, cfg.hidden)
            u = F.gelu(w8a8_linear(h, blk["up"]), approximate="tanh")
            x = x + w8a8_linear(u, blk["down"]).view(B, L, cfg.hidden)
            if record is not None:
                record[f"x{i}"] = x.clone()
        h = layer_norm(x, [cfg.hidden])
        if record is not None:
            record["head_q"], record["head_scale"] = quantize_rows(h.reshape(B * L, cfg.hidden), qm.head.smooth)
            if capture_kv:
                record["kv"] = kv
        return h


def logits(qm, h):
    """Head logits from the final hidden (reference W8A8 output, fp32)."""
    B, L, d = h.shape
    return w8a8_linear(h.reshape(B * L, d), qm.head).view(B, L, -1)


def final_layer_candidates(hidden, cond, ada_weight, ada_bias, ln_weight, head_weight_q, head_w_scale, head_bias,
                           masked, mask_id: int, seed: int):
    """Candidates of the masked positions of a [B, L] canvas when the
    conditioning varies per sequence: mlx_mdlm._FinalLayer (mlx_mdlm.py:
    456-498) unfolded -- [shift | scale] = adaLN(cond), h = LayerNorm(x)
    (eps 1e-5, weight) * (1 + scale_b) + shift_b -- then the per-token int8 of
    fixed_mlp._quantize_symmetric and the int8 head's noisy argmax
    (pyoracle.head_i8 mode 1, Philox counter (v/4, p, 0, 0), key (seed, b)).
    hidden: fp32 [B, L, 768]; returns (rows b * L + p in position-major
    order, ids, int8 rows, row scales)."""
    import torch
    import torch.nn.functional as F

    from oracle import pyoracle

    B, L, d = hidden.shape
    mod = torch.nn.functional.linear(cond, ada_weight, ada_bias)
    shift, scale = mod.chunk(2, dim=-1)
    n = F.layer_norm(hidden, [d], ln_weight)
    h = n * (1 + scale[:, None]) + shift[:, None]
    rows = np.nonzero(np.asarray(masked).reshape(-1))[0]
    q, s = quantize_rows(h.reshape(B * L, d)[torch.from_numpy(rows)])
    qn, sn = q.numpy(), s.numpy()
    ids, _ = pyoracle.head_i8(1, qn, head_weight_q, mask_id, a_scale=sn, w_scale=head_w_scale, bias=head_bias,
                              row_position=rows % L, row_key_hi=rows // L, row_eval=np.zeros(rows.size),
                              key_lo=seed)
    return rows, ids, qn, sn
