"""The head with a per-sequence conditioning vector (the final layer of the
DDiT unfolded, mlx_mdlm._FinalLayer, mlx_mdlm.py:456-498): adaLN
modulation, LayerNorm + modulation + per-token int8 of the masked rows, and
the fused int8 head + Philox-Gumbel argmax, against the CPU oracle
(model_oracle.final_layer_candidates).

Bars: the modulation within 1e-5; the int8 rows within one step of the
oracle's (the LayerNorm's fp32 reductions differ in order), at least 99%
identical; given the GPU's own int8 rows the candidate ids are bit-exact;
against the oracle's own rows at least 99% of the ids agree.
"""

import numpy as np
import pytest

from diffusionhard_b200.final_head import ConditionedHead
from oracle import model_oracle, pyoracle

pytestmark = pytest.mark.gpu


def test_conditioned_head_matches_oracle(cuda):
    torch = cuda
    B, L, V, C = 3, 256, 50258, 128
    g = torch.Generator().manual_seed(0)
    hidden = torch.randn((B, L, 768), generator=g).to(torch.bfloat16)
    cond = torch.randn((B, C), generator=g)
    ada_w = torch.randn((1536, C), generator=g) * 0.02
    ln_w = 1 + 0.1 * torch.randn(768, generator=g)
    rng = np.random.default_rng(1)
    w = np.clip(np.round(rng.normal(0, 40, (V, 768))), -127, 127).astype(np.int8)
    w_scale = rng.uniform(0.5e-3, 2e-3, V).astype(np.float32)
    bias = rng.normal(0, 0.02, V).astype(np.float32)
    masked = torch.rand((B, L), generator=g) < 0.5
    head = ConditionedHead(w, w_scale, bias, ada_w.numpy(), None, ln_w.numpy(), V - 1, B, L)
    rows, ids = head.candidates(hidden.cuda(), cond.cuda(), masked, seed=9)
    n = rows.size
    mod_ref = torch.nn.functional.linear(cond, ada_w)
    assert torch.allclose(head.modulation.cpu(), mod_ref, rtol=1e-5, atol=1e-6)
    orows, oids, oq, osc = model_oracle.final_layer_candidates(hidden.float(), cond, ada_w, None, ln_w, w, w_scale,
                                                               bias, masked.numpy(), V - 1, seed=9)
    assert np.array_equal(rows, orows)
    gq = head.head_q[:n].cpu().numpy()
    assert np.abs(gq.astype(np.int32) - oq.astype(np.int32)).max() <= 1
    assert (gq == oq).mean() >= 0.99
    assert np.allclose(head.head_scale[:n].cpu().numpy(), osc, rtol=1e-5)
    # bit-exact given the GPU's own int8 rows
    tids, _ = pyoracle.head_i8(1, gq, w, V - 1, a_scale=head.head_scale[:n].cpu().numpy(), w_scale=w_scale,
                               bias=bias, row_position=rows % L, row_key_hi=rows // L, row_eval=np.zeros(n),
                               key_lo=9)
    assert np.array_equal(ids, tids)
    agree = float((ids == oids).mean())
    print(f"\nconditioned head, {n} masked rows: ids identical to the oracle's {agree:.4f}")
    assert agree >= 0.99
