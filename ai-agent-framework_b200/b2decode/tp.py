"""Tensor-parallel helpers: the shares each rank keeps, and connecting the
ranks of one model through torch.distributed (one process per GPU).

The shares mirror the loader (csrc/model.cu, b2_load with tp_size > 1):
heads split evenly (q, k, v rows and Wo input columns), the FFN split at
32-element block granularity (gate / up rows, down input columns; uneven
shares allowed), the lm_head split by vocab rows.
"""
from __future__ import annotations


def shares(hidden: int, heads: int, kv_heads: int, ffn: int, vocab: int, tp: int, rank: int) -> dict:
    """This rank's slices of a model of the given shape (row / column ranges
    in the GGUF tensors)."""
    if tp < 1 or not 0 <= rank < tp:
        raise ValueError("rank outside the degree")
    if heads % tp or kv_heads % tp:
        raise ValueError("heads and KV heads must be divisible by the degree")
    hd = hidden // heads
    nh, nkv = heads // tp, kv_heads // tp
    nbf = ffn // 32
    fb0, fb1 = rank * nbf // tp, (rank + 1) * nbf // tp
    v0, v1 = rank * vocab // tp, (rank + 1) * vocab // tp
    return {
        "q_rows": (rank * nh * hd, (rank + 1) * nh * hd),
        "kv_rows": (rank * nkv * hd, (rank + 1) * nkv * hd),
        "wo_cols": (rank * nh * hd, (rank + 1) * nh * hd),
        "ffn_rows": (32 * fb0, 32 * fb1),
        "down_cols": (32 * fb0, 32 * fb1),
        "vocab_rows": (v0, v1),
    }


def exchange_handles(handle: bytes, group=None) -> list:
    """All ranks' 64-byte handles in rank order (torch.distributed
    all_gather_object over the given group, any backend)."""
    import torch.distributed as dist
    out = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, bytes(handle), group=group)
    return out


def connect(model, group=None) -> None:
    """Maps every rank's exchange buffer into this rank's model."""
    model.tp_connect(exchange_handles(model.tp_handle(), group))
