"""Batched-segment decoding over several GPUs: the data-parallel mode of the
reference's segmented transcription (crates/qwen-asr/src/transcribe.rs:354-420,
independent segments when past_text_conditioning is false, context.rs:512).

One process per GPU.  Segments are split statically and evenly over the
ranks; every rank decodes its share on its own engine (full weight replica),
in micro-batches of up to `max_batch` sequences (one KV slot each); the
token ids are gathered to rank 0 on the host in segment order at the end.
There is no collective on the data path: the only cross-rank traffic is the
final gather of the ids (and whatever timing reductions a caller adds).
"""
from __future__ import annotations

from typing import Callable, Sequence

import numpy as np


def segment_range(n_segments: int, rank: int, world: int) -> range:
    """Segments of `rank`: a contiguous, even static split (sizes differ by <= 1)."""
    if world <= 0 or not 0 <= rank < world or n_segments < 0:
        raise ValueError(f"bad partition request: n={n_segments} rank={rank} world={world}")
    return range(n_segments * rank // world, n_segments * (rank + 1) // world)


def decode_batch(dec, prompts: Sequence[np.ndarray], first_tokens: Sequence[int], n_new: int) -> list[list[int]]:
    """Greedy decode of up to dec.max_batch segments on one engine.

    prompts[i]: the prompt rows [P_i, hidden] (f32 embeddings, the prompt
    without its last token); first_tokens[i]: the last prompt token, fed at
    position P_i by the first decode step (the reference prefills the prompt
    but its last token, then runs decoder_forward_int8 on it).  Returns the
    n_new generated ids of every segment.
    """
    M = len(prompts)
    if M == 0:
        return []
    if M > dec.max_batch:
        raise ValueError(f"{M} segments > engine batch {dec.max_batch}")
    pos = np.empty(M, np.int32)
    for i, p in enumerate(prompts):
        p = np.ascontiguousarray(p, dtype=np.float32)
        if len(p):
            dec.prefill(i, p, 0)
        pos[i] = len(p)
    tok = np.asarray(first_tokens, dtype=np.int32).copy()
    out = [[] for _ in range(M)]
    for _ in range(n_new):
        tok = dec.step(tok, pos)
        for i in range(M):
            out[i].append(int(tok[i]))
        pos += 1
    return out


def run_rank(decode_fn: Callable[[list[int]], list[list[int]]], n_segments: int, batch: int, rank: int,
             world: int) -> dict[int, list[int]]:
    """Decode this rank's segments in micro-batches: {segment: ids}."""
    mine = list(segment_range(n_segments, rank, world))
    res: dict[int, list[int]] = {}
    for b in range(0, len(mine), batch):
        segs = mine[b:b + batch]
        for s, ids in zip(segs, decode_fn(segs)):
            res[s] = ids
    return res


def gather_in_order(local: dict[int, list[int]], n_segments: int, dist=None) -> list[list[int]] | None:
    """Concatenate every rank's results in segment order on rank 0 (None on
    the other ranks).  Without a process group, `local` must hold them all."""
    if dist is None or not dist.is_initialized() or dist.get_world_size() == 1:
        parts = [local]
    else:
        parts = [None] * dist.get_world_size() if dist.get_rank() == 0 else None
        dist.gather_object(local, parts, dst=0)
        if dist.get_rank() != 0:
            return None
    merged: dict[int, list[int]] = {}
    for p in parts:
        dup = merged.keys() & p.keys()
        if dup:
            raise RuntimeError(f"segments decoded twice: {sorted(dup)[:4]}")
        merged.update(p)
    missing = [s for s in range(n_segments) if s not in merged]
    if missing:
        raise RuntimeError(f"segments missing from the gather: {missing[:4]}")
    return [merged[s] for s in range(n_segments)]
