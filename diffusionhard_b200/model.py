"""MDLM-OWT DDiT weights: random init, constant-condition folding, SmoothQuant
calibration and W8A8 quantisation (host side, run once per model).

Architecture (mlx_mdlm.py:251-575, hardware_package.py:195-289): 12 DDiT blocks,
d=768, 12 heads x 64, MLP 3072 (GELU tanh), rotary positions, adaLN on a
128-d sigma embedding, vocab 50258 with mask id 50257.  The checkpoint is not
time-conditioned (configs/models/mdlm_owt_169m.yaml:15), so the conditioning
vector is the constant silu(sigma_map(0)) and every adaLN shift / scale / gate
folds into the adjacent linear (model_specialization.py:10-38).

W8A8 (fixed_mlp.quantized_linear, fixed_mlp.py:65-136) with static SmoothQuant
scales s = amax_a^alpha / amax_w^(1-alpha) per input channel, amax_a from a
seeded calibration batch: W' = W * s, per-output-channel int8 weights
w_scale = max|W'_row| / 127; at run time a' = a / s is quantised per token.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Dict, List, Optional

import numpy as np


@dataclass(frozen=True)
class MDLMConfig:
    vocab_size: int = 50258
    mask_token_id: int = 50257
    hidden: int = 768
    heads: int = 12
    head_dim: int = 64
    mlp: int = 3072
    blocks: int = 12
    cond: int = 128
    freq: int = 256
    max_positions: int = 1024

    def parameter_count(self) -> int:
        """Parameter inventory of model_spec.parameter_breakdown (model_spec.py:29-59)."""
        h, c, m, v = self.hidden, self.cond, self.mlp, self.vocab_size
        per_block = 2 * h + h * 3 * h + h * h + h * m + m + m * h + h + c * 6 * h + 6 * h
        return (v * h + (256 * c + c + c * c + c) + per_block * self.blocks + h + h * v + v
                + c * 2 * h + 2 * h)


def build_standin(config: MDLMConfig = MDLMConfig(), seed: int = 0, std: float = 0.02):
    """A torch module with the HF DDiT attribute names, weights ~ N(0, std).

    backbone.vocab_embed.embedding, backbone.sigma_map.mlp[0|2],
    backbone.rotary_emb, backbone.blocks[i].{norm1, attn_qkv, attn_out, norm2,
    mlp[0|2], adaLN_modulation}, backbone.output_layer.{norm_final, linear,
    adaLN_modulation}; LayerNorm weights are 1, biases 0.
    """
    import torch
    import torch.nn as nn

    g = torch.Generator().manual_seed(seed)

    def lin(i: int, o: int, bias: bool = True) -> nn.Linear:
        m = nn.Linear(i, o, bias=bias)
        with torch.no_grad():
            m.weight.copy_(torch.randn((o, i), generator=g) * std)
            if bias:
                m.bias.zero_()
        return m

    class LayerNormW(nn.Module):
        def __init__(self, d: int) -> None:
            super().__init__()
            self.weight = nn.Parameter(torch.ones(d))

        def forward(self, x):
            return torch.nn.functional.layer_norm(x.float(), [x.shape[-1]]) * self.weight[None, None, :]

    class Embedding(nn.Module):
        def __init__(self) -> None:
            super().__init__()
            self.embedding = nn.Parameter(torch.randn((config.vocab_size, config.hidden), generator=g) * std)

        def forward(self, ids):
            return self.embedding[ids]

    class SigmaMap(nn.Module):
        def __init__(self) -> None:
            super().__init__()
            self.mlp = nn.Sequential(lin(config.freq, config.cond), nn.SiLU(), lin(config.cond, config.cond))

        def forward(self, t):
            half = config.freq // 2
            freqs = torch.exp(-math.log(10000.0) * torch.arange(half, dtype=torch.float32) / half)
            args = t[:, None].float() * freqs[None]
            emb = torch.cat([torch.cos(args), torch.sin(args)], dim=-1)
            return self.mlp(emb)

    class Rotary(nn.Module):
        def __init__(self) -> None:
            super().__init__()
            d = config.head_dim
            self.register_buffer("inv_freq", 1.0 / (10000 ** (torch.arange(0, d, 2).float() / d)))

        def forward(self, x):
            # flash-attention layout [1, seq, 3, 1, head_dim] (hardware_package.py:221)
            t = torch.arange(x.shape[1], dtype=self.inv_freq.dtype)
            freqs = torch.einsum("i,j->ij", t, self.inv_freq)
            emb = torch.cat((freqs, freqs), dim=-1)
            cos = emb.cos()[None, :, None, None, :].repeat(1, 1, 3, 1, 1)
            sin = emb.sin()[None, :, None, None, :].repeat(1, 1, 3, 1, 1)
            return cos, sin

    class Block(nn.Module):
        def __init__(self) -> None:
            super().__init__()
            d = config.hidden
            self.norm1 = LayerNormW(d)
            self.attn_qkv = lin(d, 3 * d, bias=False)
            self.attn_out = lin(d, d, bias=False)
            self.norm2 = LayerNormW(d)
            self.mlp = nn.Sequential(lin(d, config.mlp), nn.GELU(approximate="tanh"), lin(config.mlp, d))
            self.adaLN_modulation = lin(config.cond, 6 * d)

    class FinalLayer(nn.Module):
        def __init__(self) -> None:
            super().__init__()
            self.norm_final = LayerNormW(config.hidden)
            self.linear = lin(config.hidden, config.vocab_size)
            self.adaLN_modulation = lin(config.cond, 2 * config.hidden)

    class Backbone(nn.Module):
        def __init__(self) -> None:
            super().__init__()
            self.vocab_embed = Embedding()
            self.sigma_map = SigmaMap()
            self.rotary_emb = Rotary()
            self.blocks = nn.ModuleList([Block() for _ in range(config.blocks)])
            self.output_layer = FinalLayer()

    class Config:
        n_heads = config.heads
        hidden_dim = config.hidden
        n_blocks = config.blocks
        vocab_size = config.vocab_size
        model_length = config.max_positions
        time_conditioning = False

    class Model(nn.Module):
        def __init__(self) -> None:
            super().__init__()
            self.backbone = Backbone()
            self.config = Config()

    return Model().eval()


def ddit_forward(model, ids) -> "object":
    """Unfolded DDiT forward of a module with the HF attribute names (the
    stand-in above or a loaded checkpoint), fp32 on the CPU: the adaLN
    conditioning c = silu(sigma_map(0)) is applied as modulate / gate at run
    time rather than folded.  The block and final-layer structure follows
    the reference's MLX restatement (mlx_mdlm.py:397-498): per block,
    x += gate_msa * attn_out(attn(rotary(qkv(norm1(x) * (1 + scale_msa) + shift_msa)))), then
    x += gate_mlp * mlp(norm2(x) * (1 + scale_mlp) + shift_mlp); logits =
    linear(norm_final(x) * (1 + scale) + shift).  Returns fp32 logits [B, L, V]."""
    import torch
    import torch.nn.functional as F

    with torch.no_grad():
        bb = model.backbone
        ids_t = torch.as_tensor(ids, dtype=torch.long)
        x = bb.vocab_embed(ids_t).float()
        B, L, d = x.shape
        heads = int(model.config.n_heads)
        hd = d // heads
        c = F.silu(bb.sigma_map(torch.zeros(1)))
        cos, sin = bb.rotary_emb(x)
        half = hd // 2
        cos = cos[0, :, 0, 0, :half][None, :, None, :]
        sin = sin[0, :, 0, 0, :half][None, :, None, :]

        def rot(t):
            a, b = t[..., :half], t[..., half:]
            return torch.cat((a * cos - b * sin, b * cos + a * sin), dim=-1)

        for blk in bb.blocks:
            sa, ca, ga, sm, cm, gm = blk.adaLN_modulation(c)[:, None].chunk(6, dim=2)
            h = blk.norm1(x) * (1 + ca) + sa
            qkv = blk.attn_qkv(h).view(B, L, 3, heads, hd)
            q, k, v = qkv.unbind(dim=2)
            a = F.scaled_dot_product_attention(rot(q).transpose(1, 2), rot(k).transpose(1, 2), v.transpose(1, 2))
            x = x + ga * blk.attn_out(a.transpose(1, 2).reshape(B, L, d))
            h = blk.norm2(x) * (1 + cm) + sm
            x = x + gm * blk.mlp(h)
        ol = bb.output_layer
        shift, scale = ol.adaLN_modulation(c)[:, None].chunk(2, dim=2)
        return ol.linear(ol.norm_final(x) * (1 + scale) + shift)


@dataclass
class FoldedLinear:
    weight: np.ndarray          # fp32 [out, in]
    bias: Optional[np.ndarray]  # fp32 [out] or None


@dataclass
class FoldedMDLM:
    """fp32 weights after folding the constant adaLN conditioning."""

    config: MDLMConfig
    embedding: np.ndarray                      # [V, d]
    blocks: List[Dict[str, FoldedLinear]]      # qkv, out, up, down
    head: FoldedLinear                         # [V, d]


def fold(model) -> FoldedMDLM:
    """Fold silu(sigma_map(0)) through every adaLN (hardware_package.py:126-192)."""
    import torch
    import torch.nn.functional as F

    with torch.no_grad():
        bb = model.backbone
        cond = F.silu(bb.sigma_map(torch.zeros(1)))
        blocks = []
        for blk in bb.blocks:
            mod = blk.adaLN_modulation(cond)[0]
            shift_a, scale_a, gate_a, shift_m, scale_m, gate_m = mod.chunk(6, dim=0)

            def affine(w, b, nw, shift, scale):
                s = nw * (1 + scale)
                fw = w * s.unsqueeze(0)
                fb = torch.mv(w, shift)
                if b is not None:
                    fb = fb + b
                return fw, fb

            qw, qb = affine(blk.attn_qkv.weight, None, blk.norm1.weight, shift_a, scale_a)
            ow = blk.attn_out.weight * gate_a.unsqueeze(1)
            uw, ub = affine(blk.mlp[0].weight, blk.mlp[0].bias, blk.norm2.weight, shift_m, scale_m)
            dw = blk.mlp[2].weight * gate_m.unsqueeze(1)
            db = blk.mlp[2].bias * gate_m
            blocks.append({
                "qkv": FoldedLinear(qw.numpy().copy(), qb.numpy().copy()),
                "out": FoldedLinear(ow.numpy().copy(), None),
                "up": FoldedLinear(uw.numpy().copy(), ub.numpy().copy()),
                "down": FoldedLinear(dw.numpy().copy(), db.numpy().copy()),
            })
        ol = bb.output_layer
        shift, scale = ol.adaLN_modulation(cond)[0].chunk(2, dim=0)
        hs = ol.norm_final.weight * (1 + scale)
        hw = ol.linear.weight * hs.unsqueeze(0)
        hb = torch.mv(ol.linear.weight, shift) + ol.linear.bias
        cfg = MDLMConfig(vocab_size=ol.linear.weight.shape[0], hidden=ol.linear.weight.shape[1],
                         blocks=len(bb.blocks))
        return FoldedMDLM(cfg, bb.vocab_embed.embedding.detach().numpy().copy(), blocks,
                          FoldedLinear(hw.numpy().copy(), hb.numpy().copy()))


def rope_tables(positions: int, head_dim: int = 64):
    """cos / sin [positions, head_dim/2] fp32, computed as the reference does
    (inv_freq = 1/10000^(arange(0, d, 2)/d), freqs = pos * inv_freq in fp32;
    mlx_mdlm.py:298-313, prefix_drift.py:135-152)."""
    import torch

    inv_freq = 1.0 / (10000 ** (torch.arange(0, head_dim, 2).float() / head_dim))
    t = torch.arange(positions, dtype=torch.float32)
    freqs = torch.einsum("i,j->ij", t, inv_freq)
    return freqs.cos().numpy().copy(), freqs.sin().numpy().copy()


def fp32_forward(folded: FoldedMDLM, ids: np.ndarray, record_amax: Optional[Dict[str, np.ndarray]] = None,
                 threads: Optional[int] = None, captured: Optional[Dict[str, object]] = None,
                 attention: Optional[object] = None) -> np.ndarray:
    """Folded fp32 forward (hardware_package.folded_mdlm_forward semantics);
    returns the final hidden state after LayerNorm (unaffine).  When
    `record_amax` is given, the per-input-channel max |activation| of every
    linear is accumulated into it (keys "b{i}.qkv", ..., "head").  When
    `captured` is given, it receives the intermediate tensors under the
    reference's golden names (hardware_package.py:195-289):
    folded.embedding, folded.block_NN.{norm1_unaffine, qkv, attention,
    attention_projection, after_attention, norm2_unaffine, mlp_up, gelu,
    mlp_down, output}, folded.final.norm_unaffine.  `attention(block,
    normalized, qkv)`, when given, replaces the float attention of each
    block: normalized is the unaffine LayerNorm output [B, L, hidden], qkv
    its fp32 [B, L, 3 * hidden] projection, and the result the [B, L,
    hidden] attention output (the error-propagating screens of
    attention_int8.py:689-936 substitute an integer attention there)."""
    import torch
    import torch.nn.functional as F

    cfg = folded.config
    B, L = ids.shape
    cos, sin = rope_tables(L, cfg.head_dim)
    cos_t, sin_t = torch.from_numpy(cos)[None, :, None, :], torch.from_numpy(sin)[None, :, None, :]

    def rec(name, a):
        if record_amax is None:
            return
        m = a.abs().reshape(-1, a.shape[-1]).amax(dim=0).numpy()
        record_amax[name] = np.maximum(record_amax.get(name, m), m)

    def rot(t):
        h = cfg.head_dim // 2
        a, b = t[..., :h], t[..., h:]
        return torch.cat((a * cos_t - b * sin_t, b * cos_t + a * sin_t), dim=-1)

    def cap(name, t):
        if captured is not None:
            captured[name] = t.detach().contiguous().clone()

    with torch.no_grad():
        x = torch.from_numpy(folded.embedding)[torch.from_numpy(ids.astype(np.int64))]
        cap("folded.embedding", x)
        for i, blk in enumerate(folded.blocks):
            pre = "folded.block_%02d" % i
            h = F.layer_norm(x, [cfg.hidden])
            rec(f"b{i}.qkv", h)
            cap(pre + ".norm1_unaffine", h)
            qkv = F.linear(h, torch.from_numpy(blk["qkv"].weight), torch.from_numpy(blk["qkv"].bias))
            cap(pre + ".qkv", qkv)
            if attention is not None:
                a = attention(i, h, qkv).to(torch.float32).reshape(B, L, cfg.hidden)
            else:
                qkv = qkv.view(B, L, 3, cfg.heads, cfg.head_dim)
                q, k, v = qkv.unbind(dim=2)
                q, k = rot(q), rot(k)
                a = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2))
                a = a.transpose(1, 2).reshape(B, L, cfg.hidden)
            rec(f"b{i}.out", a)
            cap(pre + ".attention", a)
            proj = F.linear(a, torch.from_numpy(blk["out"].weight))
            x = x + proj
            cap(pre + ".attention_projection", proj)
            cap(pre + ".after_attention", x)
            h = F.layer_norm(x, [cfg.hidden])
            rec(f"b{i}.up", h)
            cap(pre + ".norm2_unaffine", h)
            up = F.linear(h, torch.from_numpy(blk["up"].weight), torch.from_numpy(blk["up"].bias))
            cap(pre + ".mlp_up", up)
            u = F.gelu(up, approximate="tanh")
            rec(f"b{i}.down", u)
            cap(pre + ".gelu", u)
            dn = F.linear(u, torch.from_numpy(blk["down"].weight), torch.from_numpy(blk["down"].bias))
            cap(pre + ".mlp_down", dn)
            x = x + dn
            cap(pre + ".output", x)
        h = F.layer_norm(x, [cfg.hidden])
        rec("head", h)
        cap("folded.final.norm_unaffine", h)
        return h.numpy()


@dataclass
class QuantLinear:
    """W8A8 linear: int8 weight [out, in], per-output scale, fp32 bias, the
    SmoothQuant scale s [in] and its reciprocal (the device multiplies)."""

    weight_q: np.ndarray
    w_scale: np.ndarray
    bias: np.ndarray
    smooth: np.ndarray
    inv_smooth: np.ndarray


@dataclass
class QuantizedMDLM:
    config: MDLMConfig
    embedding: np.ndarray
    blocks: List[Dict[str, QuantLinear]]
    head: QuantLinear
    rope_cos: np.ndarray
    rope_sin: np.ndarray
    meta: Dict[str, object] = field(default_factory=dict)


def smoothquant_linear(w: np.ndarray, b: Optional[np.ndarray], act_amax: np.ndarray,
                       alpha: float = 0.5) -> QuantLinear:
    """Static-scale restatement of fixed_mlp.py:82-90 + :38-52 in fp32 torch ops."""
    import torch

    W = torch.from_numpy(w)
    a_max = torch.from_numpy(act_amax.astype(np.float32)).clamp_min(1e-8)
    w_max = W.abs().amax(dim=0).clamp_min(1e-8)
    s = (a_max.pow(alpha) / w_max.pow(1.0 - alpha)).clamp_min(1e-8)
    Ws = W * s[None, :]
    maximum = Ws.abs().amax(dim=1)
    scales = torch.where(maximum > 0, maximum / 127.0, torch.ones_like(maximum))
    q = torch.round(Ws / scales[:, None]).clamp(-127, 127).to(torch.int8)
    bias = np.zeros(w.shape[0], np.float32) if b is None else b.astype(np.float32)
    return QuantLinear(q.numpy().copy(), scales.numpy().astype(np.float32), bias,
                       s.numpy().astype(np.float32), (1.0 / s).numpy().astype(np.float32))


def calibration_ids(config: MDLMConfig, batch: int = 2, length: int = 256, seed: int = 1,
                    masked_fraction: float = 0.5) -> np.ndarray:
    """Seeded calibration batch: ids uniform in [0, mask) with a masked share."""
    import torch

    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(0, config.mask_token_id, (batch, length), generator=g)
    mask = torch.rand((batch, length), generator=g) < masked_fraction
    ids[mask] = config.mask_token_id
    return ids.numpy()


def quantize(folded: FoldedMDLM, alpha: float = 0.5, calib: Optional[np.ndarray] = None) -> QuantizedMDLM:
    cfg = folded.config
    if calib is None:
        calib = calibration_ids(cfg)
    amax: Dict[str, np.ndarray] = {}
    fp32_forward(folded, calib, record_amax=amax)
    blocks = []
    for i, blk in enumerate(folded.blocks):
        blocks.append({name: smoothquant_linear(blk[name].weight, blk[name].bias, amax[f"b{i}.{name}"], alpha)
                       for name in ("qkv", "out", "up", "down")})
    head = smoothquant_linear(folded.head.weight, folded.head.bias, amax["head"], alpha)
    cos, sin = rope_tables(cfg.max_positions, cfg.head_dim)
    return QuantizedMDLM(cfg, folded.embedding.astype(np.float32), blocks, head, cos, sin,
                         {"alpha": alpha, "calibration_shape": list(calib.shape)})


def build_quantized(config: MDLMConfig = MDLMConfig(), seed: int = 0, alpha: float = 0.5,
                    calib: Optional[np.ndarray] = None) -> QuantizedMDLM:
    """Random-init MDLM (N(0, 0.02)), folded and W8A8-quantised."""
    import torch

    torch.set_num_threads(max(1, torch.get_num_threads()))
    model = build_standin(config, seed)
    folded = fold(model)
    folded.config = config
    return quantize(folded, alpha, calib)
