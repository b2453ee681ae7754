"""Device-resident candidate-cache sampler (host orchestration).

Mirrors the reference samplers' call protocol and return shape
(src/diffusion_accel/mdlm.py:995-1218, conditioned.py:132-242): a sampler takes
``input_ids`` and a model / logits function and returns
``(ids, measurements, metadata)`` with the reference metadata keys.

The loop state lives on the device (tokens, uint16 candidates, active/valid
bitmaps, per-transition counters); no host synchronisation happens inside the
loop -- the counters are read once at the end.  Randomness is counter-based:
noise word of token v at position p of sequence b after an evaluation at
transition k is philox((v/4, p, k, 0), (seed, b))[v%4]; the reveal word is
philox((p/4, 0, k, 1), (seed, b))[p%4].
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Any, Callable, List, Optional

from . import _lib

NOISE_EPSILON = 1e-3


def reveal_thresholds_q32(steps: int, sampling_epsilon: float = 1e-5) -> List[int]:
    """Q32 reveal thresholds of the log-linear schedule.

    The probability is computed exactly as the reference does, in float32
    (mdlm.py:1116-1117, 1151-1153): t = linspace(1, eps, steps+1),
    move = (1 - 1e-3) t, p_k = (move_k - move_{k+1}) / move_k; then
    threshold = min(2^32, floor(p_k * 2^32)) so that P(word < threshold) = p_k
    up to 2^-32.
    """
    import torch

    if steps <= 0:
        raise ValueError("steps must be positive")
    t = torch.linspace(1.0, sampling_epsilon, steps + 1)
    out = []
    for k in range(steps):
        move_t = ((1 - NOISE_EPSILON) * t[k].reshape(1)).reshape(1, 1)
        move_s = ((1 - NOISE_EPSILON) * t[k + 1].reshape(1)).reshape(1, 1)
        p = float(((move_t - move_s) / move_t).item())
        out.append(max(0, min(1 << 32, math.floor(p * 4294967296.0))))
    return out


def hardware_candidate_cache_bytes(positions: int, mask_token_id: int) -> tuple[int, int]:
    """(cache bytes, candidate id bytes) as reported by mdlm.py:1202-1212."""
    candidate_id_bytes = max(1, math.ceil(mask_token_id.bit_length() / 8))
    return positions * candidate_id_bytes + 2 * math.ceil(positions / 8), candidate_id_bytes


@dataclass
class MDLMStepMeasurement:
    """Same fields as mdlm.MDLMStepMeasurement (mdlm.py:105-111)."""

    step_id: int
    active_tokens: int
    changed_tokens: int
    elapsed_s: float
    sigma: float


class CandidateCacheState:
    """Device buffers of the candidate-cache loop for B sequences of L positions."""

    def __init__(self, sequences: int, positions: int, vocab: int, mask_token_id: int,
                 steps: int, device: Any = "cuda") -> None:
        import torch

        self.B, self.L, self.V = sequences, positions, vocab
        self.mask = mask_token_id
        self.steps = steps
        self.device = torch.device(device)
        words = (positions + 63) // 64
        d = self.device
        self.tokens = torch.empty(sequences * positions, dtype=torch.int32, device=d)
        self.candidates = torch.empty(sequences * positions, dtype=torch.uint16, device=d)
        self.active = torch.empty(sequences * words, dtype=torch.uint64, device=d)
        self.valid = torch.empty(sequences * words, dtype=torch.uint64, device=d)
        self.eval_id = torch.empty(sequences, dtype=torch.int32, device=d)
        self.counters = torch.zeros(3 * steps, dtype=torch.int32, device=d)
        ws = _lib.lib().dh_sampler_workspace_size(sequences, positions, vocab)
        self.workspace = torch.empty(max(int(ws), 256), dtype=torch.uint8, device=d)

    def init(self, input_ids: Any) -> None:
        import torch

        ids = input_ids.to(device=self.device, dtype=torch.int32).contiguous().view(-1)
        if ids.numel() != self.B * self.L:
            raise ValueError("input_ids must have B*L entries")
        self._ids_in = ids
        _lib.call("dh_sampler_init", _lib.ptr(ids), self.B, self.L, self.mask, self.steps,
                  _lib.ptr(self.tokens), _lib.ptr(self.candidates), _lib.ptr(self.active),
                  _lib.ptr(self.valid), _lib.ptr(self.eval_id), _lib.ptr(self.counters),
                  _lib.stream_handle())

    def transition_f32(self, logits: Any, seed: int, step: int, threshold_q32: int) -> None:
        _lib.call("dh_sampler_transition_f32", _lib.ptr(logits), self.B, self.L, self.V, self.mask,
                  seed, step, self.steps, threshold_q32, _lib.ptr(self.tokens),
                  _lib.ptr(self.candidates), _lib.ptr(self.active), _lib.ptr(self.valid),
                  _lib.ptr(self.eval_id), _lib.ptr(self.counters), _lib.ptr(self.workspace),
                  self.workspace.numel(), _lib.stream_handle())

    def finalize_f32(self, logits: Any) -> None:
        _lib.call("dh_sampler_finalize_f32", _lib.ptr(logits), self.B, self.L, self.V, self.mask,
                  _lib.ptr(self.tokens), _lib.ptr(self.active), _lib.ptr(self.workspace),
                  self.workspace.numel(), _lib.stream_handle())

    def any_active(self) -> Any:
        """Device bool tensor: some position is still masked."""
        import torch

        return self.active.view(torch.int64).ne(0).any()

    def metadata(self) -> dict:
        counters = self.counters.view(self.steps, 3).cpu().tolist()
        active = [c[0] for c in counters if c[0] > 0]
        changed = [c[1] for c in counters[: len(active)]]
        evaluated = [c[2] for c in counters[: len(active)]]
        return {"transition_active_tokens": active, "transition_changed_tokens": changed,
                "evaluated": evaluated}


def run_candidate_cache_sampler_f32(
    logits_function: Callable[[Any, int], Any],
    input_ids: Any,
    *,
    mask_token_id: int,
    steps: int,
    seed: int = 0,
    vocabulary_size: int,
    sampling_epsilon: float = 1e-5,
    snapshot: Optional[Callable[[int, CandidateCacheState], None]] = None,
) -> tuple[Any, List[MDLMStepMeasurement], dict]:
    """Candidate-cache DDPM over an fp32 logits function (mdlm.py:1104-1218).

    ``logits_function(token_ids, transition)`` returns fp32 logits
    ``[B*L, vocabulary_size]`` on the device for the current canvas (the model
    protocol of the reference with the transition index in place of sigma --
    the pinned checkpoint ignores sigma, mdlm.py:1004).  It is called every
    transition while some sequence may need a refill; sequences whose cache
    is valid ignore the logits, exactly like a cache hit.  Returns
    ``(ids, measurements, metadata)`` with the reference keys.
    """
    import torch

    if input_ids.ndim != 2:
        raise ValueError("input_ids must be [batch, positions]")
    B, L = input_ids.shape
    state = CandidateCacheState(B, L, vocabulary_size, mask_token_id, steps, device="cuda")
    state.init(input_ids)
    thresholds = reveal_thresholds_q32(steps, sampling_epsilon)
    for k in range(steps):
        logits = logits_function(state.tokens.view(B, L), k)
        state.transition_f32(logits, seed, k, thresholds[k])
        if snapshot is not None:
            snapshot(k, state)
    final_logits = logits_function(state.tokens.view(B, L), steps)
    remaining = int(state.active.view(torch.int64).ne(0).sum().item())
    if remaining:
        state.finalize_f32(final_logits)
    meta = state.metadata()
    evaluations = sum(meta["evaluated"]) + (1 if remaining else 0)
    hits = len(meta["transition_active_tokens"]) - sum(meta["evaluated"])
    cache_bytes, id_bytes = hardware_candidate_cache_bytes(B * L, mask_token_id)
    ids = state.tokens.view(B, L).to(torch.int64)
    metadata = {
        "sampling_transitions": len(meta["transition_active_tokens"]),
        "model_evaluations": evaluations,
        "probability_cache_hits": hits,
        "candidate_cache_hits": hits,
        "transition_active_tokens": meta["transition_active_tokens"],
        "transition_changed_tokens": meta["transition_changed_tokens"],
        "cache_hit_sampling_overhead_modeled": False,
        "cache_correctness_class": "distribution-equivalent",
        "hardware_candidate_cache_bytes": cache_bytes,
        "candidate_id_bytes": id_bytes,
    }
    return ids, [], metadata


def _u32(x: Any, device: Any) -> Any:
    """uint32 values (python ints / numpy / torch) as a device int32 tensor of
    the same bit patterns."""
    import numpy as np
    import torch

    if isinstance(x, torch.Tensor):
        x = x.cpu().numpy()
    a = np.ascontiguousarray(np.asarray(x, dtype=np.int64).astype(np.uint32).view(np.int32))
    return torch.from_numpy(a).to(device)


def philox4x32_10(counters: Any, keys: Any, device: Any = "cuda") -> Any:
    """Philox4x32-10 blocks on the GPU (dh_philox4x32_10): counters [n, 4] and
    keys [n, 2] of uint32 values -> int64 tensor [n, 4] of the output words."""
    import torch

    c = _u32(counters, device).reshape(-1, 4).contiguous()
    k = _u32(keys, device).reshape(-1, 2).contiguous()
    if c.shape[0] != k.shape[0]:
        raise ValueError("one key per counter")
    out = torch.empty_like(c)
    n = c.shape[0]
    for i in range(0, n, 1 << 30):
        j = min(n, i + (1 << 30))
        _lib.call("dh_philox4x32_10", _lib.ptr(c[i:j]), _lib.ptr(k[i:j]), _lib.ptr(out[i:j]), j - i,
                  _lib.stream_handle())
    return out.to(torch.int64) & 0xFFFFFFFF


def noisy_argmax_f32(logits: Any, mask_token_id: int, *, row_position: Any, row_key_hi: Any,
                     row_eval: Any, key_lo: int, stream_id: int = 0) -> Any:
    """Gumbel-max race of fp32 logit rows on the GPU (dh_noisy_argmax_f32):
    the token with the largest round(logit * 1024) + Gumbel_Q10(word), word =
    philox((v/4, row_position, row_eval, stream_id), (key_lo, row_key_hi))[v%4],
    the mask token excluded, lowest id on ties.  Any number of rows (calls of
    at most 65,535 rows).  Returns int32 ids [rows] on the logits' device."""
    import torch

    if logits.dim() != 2 or logits.dtype != torch.float32 or not logits.is_cuda:
        raise ValueError("logits must be a CUDA float32 [rows, vocab] tensor")
    logits = logits.contiguous()
    rows, vocab = logits.shape
    dev = logits.device
    pos, khi, ev = (_u32(a, dev) for a in (row_position, row_key_hi, row_eval))
    if not (pos.numel() == khi.numel() == ev.numel() == rows):
        raise ValueError("one position / key / evaluation per row")
    ids = torch.empty(rows, dtype=torch.int32, device=dev)
    chunk = 65535
    ws_bytes = int(_lib.lib().dh_noisy_argmax_workspace_size(min(rows, chunk), vocab))
    ws = torch.empty(max(ws_bytes, 256), dtype=torch.uint8, device=dev)
    for i in range(0, rows, chunk):
        j = min(rows, i + chunk)
        _lib.call("dh_noisy_argmax_f32", _lib.ptr(logits[i:j]), vocab, j - i, vocab, mask_token_id,
                  _lib.ptr(pos[i:j]), _lib.ptr(khi[i:j]), _lib.ptr(ev[i:j]), key_lo & 0xFFFFFFFF, stream_id,
                  _lib.ptr(ids[i:j]), None, _lib.ptr(ws), ws.numel(), _lib.stream_handle())
    return ids


def reveal_words(sequences: int, positions: int, step: int, seed: int, seq_offset: int = 0,
                 device: Any = "cuda") -> Any:
    """Reveal words of the loop, philox((p/4, 0, step, 1), (seed, b))[p%4], as
    int64 [sequences, positions] (computed on the GPU)."""
    import numpy as np

    groups = (positions + 3) // 4
    b = np.repeat(np.arange(sequences, dtype=np.int64) + seq_offset, groups)
    g = np.tile(np.arange(groups, dtype=np.int64), sequences)
    counters = np.stack([g, np.zeros_like(g), np.full_like(g, step), np.ones_like(g)], axis=1)
    keys = np.stack([np.full_like(g, seed), b], axis=1)
    words = philox4x32_10(counters, keys, device)
    return words.view(sequences, groups * 4)[:, :positions]
