#!/usr/bin/env python3
"""Golden outputs of the reference's block-causal attention
(src/diffusion_accel/mdlm.py:61-77 block_isolation and the attention bias of
its FlashAttention compatibility path, mdlm.py:366-468), imported in place.

The compatibility module is installed only when flash_attn cannot be
imported, so this script hides the installed flash_attn behind an import
blocker first.  For seeded packed qkv [S, 3, H, D] (qkv_case below) and each
boundary list in CASES, it records flash_attn_varlen_qkvpacked_func's output
under block_isolation.  Writes tests/golden/block_golden.npz.

    python tests/golden/make_block_golden.py --reference <reference root>
"""

from __future__ import annotations

import argparse
import os
import importlib.abc
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
CASES = [[], [32], [32, 64], [16, 40, 80], [96], [200]]


def qkv_case(torch):
    """Packed qkv [96, 3, 2, 16] ~ N(0, 1), seed 4."""
    return torch.randn((96, 3, 2, 16), generator=torch.Generator().manual_seed(4))


class _Block(importlib.abc.MetaPathFinder):
    def find_spec(self, name, path, target=None):
        if name == "flash_attn" or name.startswith("flash_attn."):
            raise ImportError("hidden so that the reference installs its compatibility path")
        return None


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--reference", default=os.environ.get("DH_REFERENCE_ROOT"),
                    required="DH_REFERENCE_ROOT" not in os.environ,
                    help="reference tree (default: $DH_REFERENCE_ROOT)")
    args = ap.parse_args()
    sys.path.insert(0, str(Path(args.reference) / "src"))
    sys.meta_path.insert(0, _Block())
    import torch

    from diffusion_accel import mdlm  # reference, in place

    mdlm.install_flash_attention_compat()
    sys.meta_path.pop(0)
    from flash_attn.flash_attn_interface import flash_attn_varlen_qkvpacked_func

    qkv = qkv_case(torch)
    cu = torch.tensor([0, qkv.shape[0]], dtype=torch.int32)
    out = {}
    for i, ends in enumerate(CASES):
        if ends:
            with mdlm.block_isolation(ends):
                o = flash_attn_varlen_qkvpacked_func(qkv, cu, qkv.shape[0], 0.0, causal=False)
        else:
            o = flash_attn_varlen_qkvpacked_func(qkv, cu, qkv.shape[0], 0.0, causal=False)
        out[f"case{i}"] = o.numpy()
    np.savez_compressed(HERE / "block_golden.npz", **out)
    print({k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main()
