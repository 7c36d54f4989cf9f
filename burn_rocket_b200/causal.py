"""Chunked causal attention (the reference's `causal_chunk_plan` /
`causal_attention`, src/util/causal.rs:64-163).

Queries are split into chunks of `chunk` rows; chunk (q0..q1) attends to the
key prefix k0..k1 with k1 = min(q_offset + q1, kn) (causal: no later key is
visible) and, for a sliding window w, k0 = max(q_offset + q0 - (w - 1), 0).
Each chunk runs the fused attention kernel with the causal block mask at its
absolute query / key offsets. A single chunk with q_offset == 0 and kn == s
takes the dense causal(-window) op, as the reference does, so short runs are
bit-identical to it. On B200 one fused launch already handles a whole causal
prefill without an O(S^2) mask, so the default here is `chunk=0` (dense); the
chunked form is kept for callers that bound per-launch work.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional

DEFAULT_CAUSAL_CHUNK = 1024


@dataclass(frozen=True)
class CausalChunk:
    q0: int  # query rows q0..q1 (local)
    q1: int
    k0: int  # keys k0..k1 (local)
    k1: int

    def q_pos(self, q_offset: int) -> int:
        """Absolute position of the chunk's first query row."""
        return q_offset + self.q0


def causal_chunk_plan(s: int, kn: int, q_offset: int, window: Optional[int], chunk: int) -> List[CausalChunk]:
    """causal_chunk_plan (src/util/causal.rs:64-101)."""
    if s <= 0:
        raise ValueError("causal attention needs at least one query")
    if kn <= 0:
        raise ValueError("causal attention needs at least one key")
    if chunk == 0 or s <= chunk:
        k0 = 0 if window is None else max(q_offset - max(window - 1, 0), 0)
        return [CausalChunk(0, s, k0, kn)]
    plan = []
    q0 = 0
    while q0 < s:
        q1 = min(q0 + chunk, s)
        p0, p1 = q_offset + q0, q_offset + q1 - 1
        k0 = 0 if window is None else max(p0 - max(window - 1, 0), 0)
        plan.append(CausalChunk(q0, q1, k0, min(p1 + 1, kn)))
        q0 = q1
    return plan


def causal_attention(q, k, v, n_head: int, n_kv_heads: int, head_dim: int, scale: float,
                     softcap: Optional[float] = None, window: Optional[int] = None, q_offset: int = 0,
                     chunk: int = 0):
    """causal_attention (src/util/causal.rs:103-163) over [S, H*D] / [Kn, KV*D] CUDA tensors."""
    import torch
    from . import attention_causal_block, attention_causal_window
    s, kn = q.shape[-2], k.shape[-2]
    plan = causal_chunk_plan(s, kn, q_offset, window, chunk)
    win = -1 if window is None else int(window)
    if len(plan) == 1 and q_offset == 0 and kn == s:
        return attention_causal_window(q, k, v, n_head, n_kv_heads, head_dim, scale, softcap, win)
    outs = []
    for c in plan:
        outs.append(attention_causal_block(q[..., c.q0:c.q1, :], k[..., c.k0:c.k1, :], v[..., c.k0:c.k1, :],
                                           n_head, n_kv_heads, head_dim, scale, softcap, win,
                                           q_start=c.q_pos(q_offset), kv_start=c.k0))
    return outs[0] if len(outs) == 1 else torch.cat(outs, dim=-2)
