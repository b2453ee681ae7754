"""Checkpoints and the fixed-shape hardware package.

* ``load_checkpoint``: an MDLM-OWT state dict in the HF DDiT layout
  (``model.safetensors`` or a torch file) -> folded fp32 weights, through
  the stand-in module that carries the same attribute names (model.py) and
  the constant-condition fold.
* The hardware package of the reference (hardware_package.py:83-116,
  300-613): ``folded_fp16_weights.safetensors`` (the folded weights in fp16,
  named ``embedding.weight``, ``block_NN.{qkv,attention_out,mlp_up,mlp_down}.*``,
  ``output.*``, ``rotary.{cos,sin}``), the same tensors as one little-endian
  DDR image with 4 KiB-aligned entries (``folded_fp16_weights.bin``),
  golden tensors, and ``manifest.json`` with sizes, SHA-256 digests and the
  binary layout.  ``export_hardware_package`` writes it from folded weights,
  ``validate_hardware_package`` checks it as the reference's validator does,
  and ``load_hardware_package`` reads it back as folded weights for the
  engine (W8A8 quantisation then follows, as for the stand-in).
* ``decode_tokens``: GPT-2 text of token ids when the tokenizer is cached
  locally (mdlm.py:1356-1365), else None.
"""

from __future__ import annotations

import hashlib
import json
from pathlib import Path
from typing import Any, Dict, Iterable, List, Optional, Sequence, Tuple

import numpy as np

from .model import FoldedLinear, FoldedMDLM, MDLMConfig, build_standin, fold, fp32_forward

PACKAGE_SCHEMA_VERSION = "0.1"
WEIGHTS_FILE = "folded_fp16_weights.safetensors"
BINARY_FILE = "folded_fp16_weights.bin"
GOLDEN_FILE = "golden_tensors.safetensors"
MANIFEST_FILE = "manifest.json"
_LINEARS = (("qkv", "qkv", True), ("out", "attention_out", False), ("up", "mlp_up", True),
            ("down", "mlp_down", True))


def deterministic_hardware_input(canvas_tokens: int, vocabulary_size: int, mask_token_id: int) -> List[int]:
    """The package's mixed masked / visible input (hardware_package.py:26-40):
    position p holds (7919 p + 17) mod mask when p % 3 == 0, else the mask."""
    if canvas_tokens <= 0:
        raise ValueError("canvas_tokens must be positive")
    if vocabulary_size <= 1:
        raise ValueError("vocabulary_size must be greater than one")
    if mask_token_id != vocabulary_size - 1:
        raise ValueError("MDLM hardware package expects the final ID as mask")
    return [mask_token_id if p % 3 else (p * 7919 + 17) % mask_token_id for p in range(canvas_tokens)]


def _sha256(path: Path) -> str:
    h = hashlib.sha256()
    with path.open("rb") as f:
        for chunk in iter(lambda: f.read(1 << 20), b""):
            h.update(chunk)
    return h.hexdigest()


def hardware_weight_order(names: Iterable[str]) -> List[str]:
    """DDR image order (hardware_package.py:69-80): the embedding, then the
    blocks, then the output layer, then the rest, each group by name."""
    def rank(name: str) -> Tuple[int, str]:
        if name == "embedding.weight":
            return (0, name)
        if name.startswith("block_"):
            return (1, name)
        if name.startswith("output."):
            return (2, name)
        return (3, name)

    return sorted(names, key=rank)


def tensor_manifest(tensors: Dict[str, Any]) -> Dict[str, object]:
    """Per-tensor dtype / shape / bytes and totals (hardware_package.py:52-66)."""
    entries: Dict[str, object] = {}
    total = 0
    for name in sorted(tensors):
        t = tensors[name]
        nbytes = t.numel() * t.element_size()
        total += nbytes
        entries[name] = {"dtype": str(t.dtype).replace("torch.", ""), "shape": list(t.shape), "bytes": nbytes}
    return {"tensor_count": len(entries), "tensor_bytes": total, "tensors": entries}


def write_weight_binary(tensors: Dict[str, Any], path: Path, alignment: int = 4096) -> Dict[str, object]:
    """The DDR image: fp16 tensors, row-major, each starting on `alignment`
    bytes, zero padding between and at the end (hardware_package.py:83-116)."""
    if alignment <= 0 or alignment & (alignment - 1):
        raise ValueError("binary alignment must be a positive power of two")
    entries: Dict[str, object] = {}
    offset = 0
    with path.open("wb") as f:
        for name in hardware_weight_order(tensors):
            pad = (-offset) % alignment
            f.write(bytes(pad))
            offset += pad
            payload = tensors[name].contiguous().numpy().astype("<f2").tobytes(order="C")
            entries[name] = {"offset_bytes": offset, "length_bytes": len(payload),
                             "dtype": "little-endian-float16", "shape": list(tensors[name].shape),
                             "order": "row-major"}
            f.write(payload)
            offset += len(payload)
        pad = (-offset) % alignment
        f.write(bytes(pad))
        offset += pad
    return {"alignment_bytes": alignment, "total_bytes": offset, "tensor_count": len(entries), "tensors": entries}


def read_weight_binary(path: Path, layout: Dict[str, Any]) -> Dict[str, np.ndarray]:
    """fp16 arrays of the DDR image by its layout (memory-mapped)."""
    raw = np.memmap(path, dtype=np.uint8, mode="r")
    if raw.size < int(layout["total_bytes"]):
        raise ValueError("weight binary is shorter than its declared size")
    out = {}
    for name, e in layout["tensors"].items():
        o, n = int(e["offset_bytes"]), int(e["length_bytes"])
        out[name] = np.frombuffer(raw[o:o + n], dtype="<f2").reshape(e["shape"])
    return out


def binary_layout_errors(manifest: Dict[str, Any]) -> List[str]:
    """Alignment, overlap, length and bounds of every image entry
    (hardware_package.py:542-562)."""
    errors: List[str] = []
    layout = manifest["weight_binary_layout"]
    alignment = int(layout["alignment_bytes"])
    total = int(layout["total_bytes"])
    weights = manifest["weights"]["tensors"]
    end = 0
    for name in hardware_weight_order(layout["tensors"]):
        e = layout["tensors"][name]
        o, n = int(e["offset_bytes"]), int(e["length_bytes"])
        if o % alignment:
            errors.append("%s offset is not aligned" % name)
        if o < end:
            errors.append("%s overlaps the previous tensor" % name)
        if name not in weights or n != int(weights[name]["bytes"]):
            errors.append("%s binary length does not match tensor bytes" % name)
        if o + n > total:
            errors.append("%s exceeds the declared binary size" % name)
        end = o + n
    return errors


def folded_to_package_tensors(folded: FoldedMDLM, rotary_positions: int = 64) -> Dict[str, Any]:
    """Folded weights under the package names, in fp16
    (hardware_package._export_folded_weights, hardware_package.py:322-355)."""
    import torch

    from .model import rope_tables

    def h(a: np.ndarray) -> Any:
        return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(torch.float16)

    out = {"embedding.weight": h(folded.embedding)}
    for i, blk in enumerate(folded.blocks):
        for ours, theirs, has_bias in _LINEARS:
            out["block_%02d.%s.weight" % (i, theirs)] = h(blk[ours].weight)
            if has_bias:
                out["block_%02d.%s.bias" % (i, theirs)] = h(blk[ours].bias)
    out["output.weight"] = h(folded.head.weight)
    out["output.bias"] = h(folded.head.bias)
    cos, sin = rope_tables(rotary_positions, folded.config.head_dim)
    out["rotary.cos"] = h(cos)
    out["rotary.sin"] = h(sin)
    return out


def package_tensors_to_folded(tensors: Dict[str, Any], config: Optional[MDLMConfig] = None) -> FoldedMDLM:
    """Inverse of folded_to_package_tensors: fp16 package tensors (torch or
    numpy) -> fp32 folded weights.  The shapes give vocabulary, width, MLP
    width and block count; heads come from `config` (default 12 x 64)."""
    def f32(name: str) -> np.ndarray:
        if name not in tensors:
            raise ValueError("package is missing tensor %s" % name)
        t = tensors[name]
        a = t.float().numpy() if hasattr(t, "float") else np.asarray(t, dtype=np.float32)
        return np.ascontiguousarray(a, dtype=np.float32)

    n_blocks = len({k.split(".")[0] for k in tensors if k.startswith("block_")})
    emb = f32("embedding.weight")
    head_w = f32("output.weight")
    vocab, hidden = head_w.shape
    blocks = []
    for i in range(n_blocks):
        blk = {}
        for ours, theirs, has_bias in _LINEARS:
            w = f32("block_%02d.%s.weight" % (i, theirs))
            b = f32("block_%02d.%s.bias" % (i, theirs)) if has_bias else None
            blk[ours] = FoldedLinear(w, b)
        blocks.append(blk)
    mlp = blocks[0]["up"].weight.shape[0] if blocks else 4 * hidden
    base = config or MDLMConfig()
    heads = base.heads if hidden == base.heads * base.head_dim else max(1, hidden // base.head_dim)
    cfg = MDLMConfig(vocab_size=vocab, mask_token_id=vocab - 1, hidden=hidden, heads=heads,
                     head_dim=hidden // heads, mlp=mlp, blocks=n_blocks, cond=base.cond, freq=base.freq,
                     max_positions=base.max_positions)
    if emb.shape != (vocab, hidden):
        raise ValueError("embedding and output shapes disagree")
    return FoldedMDLM(cfg, emb, blocks, FoldedLinear(head_w, f32("output.bias")))


def export_hardware_package(folded: FoldedMDLM, out_dir: Path, *, canvas_tokens: int = 64,
                            source: Optional[Dict[str, object]] = None,
                            unfolded_logits: Optional[Any] = None) -> Dict[str, object]:
    """Write the hardware package of folded weights (the layout of
    hardware_package.export_mdlm_hardware_package, hardware_package.py:366-540).

    Goldens are the folded fp32 forward on deterministic_hardware_input
    under the reference's names: ``input.ids``, ``folded.embedding``, every
    block's ``folded.block_NN.*`` intermediates (what the fixed-point MLP
    validation reads), ``folded.final.norm_unaffine``,
    ``folded.final.logits`` and ``folded.top1``.  When ``unfolded_logits``
    (the unfolded model's logits on the same input, e.g. model.ddit_forward)
    is given, the manifest's constant-fold validation compares them with the
    folded logits under the reference's acceptance (max error 1e-4, top-1
    agreement 1); otherwise it records that no unfolded model was available
    and does not pass."""
    import torch
    from safetensors.torch import save_file

    if canvas_tokens != 64:
        raise ValueError("the first hardware package is frozen to 64 tokens")
    cfg = folded.config
    mask = cfg.vocab_size - 1
    ids = deterministic_hardware_input(canvas_tokens, cfg.vocab_size, mask)
    ids_np = np.asarray([ids], dtype=np.int64)
    captured: Dict[str, Any] = {}
    hidden = torch.from_numpy(fp32_forward(folded, ids_np, captured=captured))
    logits = hidden @ torch.from_numpy(folded.head.weight).t() + torch.from_numpy(folded.head.bias)
    scores = logits.clone()
    scores[..., mask] = -torch.inf
    top1 = scores.argmax(dim=-1)
    goldens = dict(captured)
    goldens.update({
        "input.ids": torch.tensor([ids], dtype=torch.int32),
        "folded.final.logits": logits.contiguous(),
        "folded.top1": top1.to(torch.int32).contiguous(),
    })
    if unfolded_logits is not None:
        ref = torch.as_tensor(unfolded_logits).float().reshape(logits.shape)
        diff = (ref - logits).abs()
        ref_scores = ref.clone()
        ref_scores[..., mask] = -torch.inf
        ref_top1 = ref_scores.argmax(dim=-1)
        agreement = float(ref_top1.eq(top1).float().mean().item())
        goldens["reference.top1"] = ref_top1.to(torch.int32).contiguous()
        validation = {"folded_vs_reference_max_abs_error": float(diff.max().item()),
                      "folded_vs_reference_mean_abs_error": float(diff.mean().item()),
                      "top1_agreement": agreement, "acceptance_max_abs_error": 1e-4}
        validation["passed"] = validation["folded_vs_reference_max_abs_error"] <= 1e-4 and agreement == 1.0
    else:
        ref_top1 = None
        validation = {"acceptance_max_abs_error": 1e-4, "passed": False,
                      "note": "no unfolded model given: the fold was not validated"}
    weights = folded_to_package_tensors(folded)
    out_dir = Path(out_dir)
    out_dir.mkdir(parents=True, exist_ok=True)
    paths = [out_dir / GOLDEN_FILE, out_dir / WEIGHTS_FILE, out_dir / BINARY_FILE]
    save_file(goldens, paths[0])
    save_file(weights, paths[1])
    layout = write_weight_binary(weights, paths[2])
    manifest = {
        "schema_version": PACKAGE_SCHEMA_VERSION,
        "source_checkpoint": dict(source or {"weights": "folded weights supplied by the caller"}),
        "fixed_graph": {"canvas_tokens": canvas_tokens, "batch_size": 1, "hidden_size": cfg.hidden,
                        "blocks": len(folded.blocks), "heads": cfg.heads, "vocabulary_size": cfg.vocab_size,
                        "mask_token_id": mask, "time_conditioning": False},
        "input": {"construction": "position*7919+17 modulo mask ID; positions not divisible by three are masked",
                  "visible_tokens": sum(v != mask for v in ids), "masked_tokens": sum(v == mask for v in ids),
                  "reference_top1_token_ids": None if ref_top1 is None else ref_top1[0].tolist(),
                  "reference_top1_decoded_text": None},
        "constant_fold_validation": validation,
        "goldens": tensor_manifest(goldens),
        "weights": tensor_manifest(weights),
        "weight_binary_layout": layout,
        "files": {p.name: {"bytes": p.stat().st_size, "sha256": _sha256(p)} for p in paths},
        "device_used_for_reference": "cpu",
    }
    (out_dir / MANIFEST_FILE).write_text(json.dumps(manifest, indent=2, sort_keys=True) + "\n", encoding="utf-8")
    return manifest


def validate_hardware_package(package_dir: Path) -> Dict[str, object]:
    """Hashes, sizes, tensor names / shapes and the DDR layout of a package,
    the checks of hardware_package.validate_mdlm_hardware_package
    (hardware_package.py:565-613), with the same report keys."""
    from safetensors import safe_open

    package_dir = Path(package_dir)
    manifest = json.loads((package_dir / MANIFEST_FILE).read_text(encoding="utf-8"))
    errors: List[str] = []
    verified: Dict[str, object] = {}
    for name, expected in manifest["files"].items():
        path = package_dir / name
        if not path.exists():
            errors.append("missing file %s" % name)
            continue
        size, digest = path.stat().st_size, _sha256(path)
        if size != int(expected["bytes"]):
            errors.append("%s byte size mismatch" % name)
        if digest != str(expected["sha256"]):
            errors.append("%s SHA-256 mismatch" % name)
        verified[name] = {"bytes": size, "sha256": digest}
    for filename, section in ((GOLDEN_FILE, "goldens"), (WEIGHTS_FILE, "weights")):
        if not (package_dir / filename).exists():
            continue
        with safe_open(package_dir / filename, framework="pt", device="cpu") as handle:
            keys = list(handle.keys())
            expected = manifest[section]["tensors"]
            if set(keys) != set(expected):
                errors.append("%s tensor names do not match manifest" % filename)
                continue
            for key in keys:
                if list(handle.get_slice(key).get_shape()) != expected[key]["shape"]:
                    errors.append("%s shape mismatch for %s" % (filename, key))
    errors.extend(binary_layout_errors(manifest))
    if not bool(manifest["constant_fold_validation"]["passed"]):
        errors.append("constant-fold validation did not pass")
    return {
        "schema_version": manifest["schema_version"],
        "package_dir": str(package_dir),
        "passed": not errors,
        "errors": errors,
        "verified_files": verified,
        "golden_tensor_count": int(manifest["goldens"]["tensor_count"]),
        "weight_tensor_count": int(manifest["weights"]["tensor_count"]),
        "binary_alignment_bytes": int(manifest["weight_binary_layout"]["alignment_bytes"]),
    }


def load_hardware_package(package_dir: Path, *, verify: bool = True, from_binary: bool = False,
                          config: Optional[MDLMConfig] = None) -> FoldedMDLM:
    """Folded fp32 weights of a hardware package, from the safetensors file
    or (``from_binary``) from the DDR image by the manifest's layout.  With
    ``verify`` a package that fails validate_hardware_package is refused."""
    package_dir = Path(package_dir)
    if verify:
        report = validate_hardware_package(package_dir)
        if not report["passed"]:
            raise ValueError("hardware package failed validation: " + "; ".join(report["errors"]))
    if from_binary:
        manifest = json.loads((package_dir / MANIFEST_FILE).read_text(encoding="utf-8"))
        tensors = read_weight_binary(package_dir / BINARY_FILE, manifest["weight_binary_layout"])
    else:
        from safetensors.torch import load_file

        tensors = load_file(str(package_dir / WEIGHTS_FILE))
    return package_tensors_to_folded(tensors, config)


def _read_state_dict(path: Path) -> Dict[str, Any]:
    path = Path(path)
    if path.suffix == ".safetensors":
        from safetensors.torch import load_file

        return load_file(str(path))
    import torch

    sd = torch.load(str(path), map_location="cpu", weights_only=True)
    return sd.get("state_dict", sd) if isinstance(sd, dict) else sd


def checkpoint_module(checkpoint: Any, config: MDLMConfig = MDLMConfig()) -> Any:
    """The DDiT module (stand-in class, HF attribute names) holding the
    weights of an MDLM checkpoint in the HF layout
    (``backbone.vocab_embed.embedding``, ``backbone.blocks.N.attn_qkv.weight``,
    ``backbone.blocks.N.adaLN_modulation.*``, ``backbone.output_layer.*``,
    ``backbone.sigma_map.mlp.{0,2}.*``; a ``model.`` prefix is accepted).
    ``checkpoint`` is a path (.safetensors or a torch file) or a state dict;
    every parameter of the architecture must be present."""
    import torch

    sd = _read_state_dict(checkpoint) if isinstance(checkpoint, (str, Path)) else dict(checkpoint)
    sd = {(k[len("model."):] if k.startswith("model.") else k): v for k, v in sd.items()}
    model = build_standin(config, seed=0)
    own = model.state_dict()
    missing = [k for k in own if k not in sd and not k.endswith("inv_freq")]
    if missing:
        raise ValueError("checkpoint is missing %d parameters, e.g. %s" % (len(missing), missing[:3]))
    for k, v in own.items():
        if k in sd and tuple(sd[k].shape) != tuple(v.shape):
            raise ValueError("checkpoint shape mismatch for %s: %s vs %s" % (k, tuple(sd[k].shape), tuple(v.shape)))
    with torch.no_grad():
        model.load_state_dict({k: sd[k].float() for k in own if k in sd}, strict=False)
    return model


def load_checkpoint(checkpoint: Any, config: MDLMConfig = MDLMConfig()) -> FoldedMDLM:
    """Folded fp32 weights of an MDLM checkpoint (checkpoint_module): the
    constant conditioning folds as in hardware_package._fold_block."""
    folded = fold(checkpoint_module(checkpoint, config))
    folded.config = config
    return folded


def decode_tokens(ids: Sequence[int], *, local_files_only: bool = True) -> Optional[str]:
    """GPT-2 text of token ids (mdlm.py:1356-1365) when the tokenizer is
    available locally; None otherwise, as the reference does on OSError."""
    try:
        from transformers import AutoTokenizer

        tok = AutoTokenizer.from_pretrained("gpt2", local_files_only=local_files_only)
    except Exception:  # noqa: BLE001 -- any loader failure means no tokenizer here
        return None
    return tok.decode([int(i) for i in ids])
