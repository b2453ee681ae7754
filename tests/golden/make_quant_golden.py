#!/usr/bin/env python3
"""Golden outputs of the reference's per-token int8 activation quantiser,
fixed_mlp._quantize_symmetric(a / s, 8, "token") (src/diffusion_accel/
fixed_mlp.py:11-35, the activation path of quantized_linear :82-96),
imported in place from the reference tree, on the seeded rows of
`quant_cases` below:

  * bf16-valued rows of 768 and 3072 columns, with and without a SmoothQuant
    divisor s (the inputs of dh_quant_rows_bf16);
  * edge rows: all zero, a single non-zero, exact rounding ties (amax 127, so
    the scale is 1 and x / scale = k + 1/2), one sign only, tiny magnitudes;
  * fp32 rows through F.layer_norm (eps 1e-5, no affine) and then the
    quantiser (the inputs of dh_ln_smooth_quant).
The inputs are regenerated from their seeds by `quant_cases`, so only the
int8 rows and row scales are stored.  Writes tests/golden/quant_golden.npz.

    python tests/golden/make_quant_golden.py --reference <reference root>
"""

from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def quant_cases(torch):
    """name -> (fp32 rows, smooth divisor or None, layer_norm first)."""
    g = torch.Generator().manual_seed(11)
    out = {}
    for cols, rows in ((768, 48), (3072, 16)):
        scale = 2.0 ** (torch.arange(rows) % 9 - 4).float()[:, None]
        x = (torch.randn((rows, cols), generator=g) * scale).to(torch.bfloat16).float()
        s = torch.rand(cols, generator=g) * 2.7 + 0.3
        out[f"bf16_{cols}"] = (x, None, False)
        out[f"bf16_{cols}_smooth"] = (x, s, False)
    edge = torch.zeros((6, 768))
    edge[1, 17] = -3.25
    edge[2, :] = torch.tensor([(k % 255) - 127 + 0.5 for k in range(768)]).clamp(-127, 127)
    edge[2, 0] = 127.0
    edge[3] = torch.rand(768, generator=g) * 5 + 0.01
    edge[4] = -edge[3]
    edge[5] = torch.randn(768, generator=g) * 1e-20
    out["edge_768"] = (edge.to(torch.bfloat16).float(), None, False)
    ln = torch.randn((64, 768), generator=g) * (torch.rand((64, 1), generator=g) * 4 + 0.1) + \
        torch.randn((64, 1), generator=g)
    out["ln_768"] = (ln, torch.rand(768, generator=g) * 2.7 + 0.3, True)
    return out


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--reference", default=os.environ.get("DH_REFERENCE_ROOT"),
                    required="DH_REFERENCE_ROOT" not in os.environ,
                    help="reference tree (default: $DH_REFERENCE_ROOT)")
    args = ap.parse_args()
    sys.path.insert(0, str(Path(args.reference) / "src"))
    import torch
    import torch.nn.functional as F

    from diffusion_accel.fixed_mlp import _quantize_symmetric  # reference, in place

    arrays = {}
    for name, (x, s, ln) in quant_cases(torch).items():
        a = F.layer_norm(x, [x.shape[1]]) if ln else x
        if s is not None:
            a = a / s[None, :]
        q, scale = _quantize_symmetric(a, 8, "token")
        arrays[f"{name}__q"] = q.numpy()
        arrays[f"{name}__scale"] = scale.numpy().astype(np.float32)
    np.savez_compressed(HERE / "quant_golden.npz", **arrays)
    print(sorted(arrays))


if __name__ == "__main__":
    main()
