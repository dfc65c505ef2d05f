"""Tensor parallelism on the host side: the NCCL group bootstrap over
torch.distributed, and which share of each tensor a rank holds.

The reference runs on one Metal device and has no counterpart.  The split
follows the usual row partition of a Llama layer over R ranks: rank r owns
query heads [r H/R, (r+1) H/R) and KV heads [r Hkv/R, (r+1) Hkv/R) (their
rows of wq / wk / wv and their KV-cache heads), FFN rows [r F/R, (r+1) F/R)
of w_gate and w_up, the matching input columns of wo (r H/R heads x 128)
and w_down (the same FFN rows), and vocabulary rows [r V/R, (r+1) V/R) of
the output head.  wo and w_down then produce partial sums that one sum
all-reduce per projection combines (the runner does this in
mlm_llama_*); norms and the token embedding are replicated.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, Tuple


def bootstrap(ctx, group=None) -> Tuple[int, int]:
    """Join this context to an NCCL group spanning the torch.distributed
    group: rank 0 draws the NCCL unique id, a broadcast hands it to the
    others, every rank calls mlm_tp_init.  Returns (rank, size)."""
    import torch.distributed as dist
    rank, size = dist.get_rank(group), dist.get_world_size(group)
    obj = [ctx.tp_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0, group=group)
    ctx.tp_init(size, rank, obj[0])
    return rank, size


@dataclass(frozen=True)
class Shard:
    """Rank `rank` of `size`: the index ranges it owns along each split axis."""
    rank: int
    size: int

    def span(self, n: int) -> Tuple[int, int]:
        if n % self.size:
            raise ValueError(f"{n} does not split over {self.size} ranks")
        k = n // self.size
        return self.rank * k, (self.rank + 1) * k


def layer_shards(cfg, shard: Shard) -> Dict[str, dict]:
    """Per Q4_K tensor of a layer: the rows (row0, rows) and 256-element
    block columns (kb0, nkb) of the whole-model tensor this rank stores,
    with the whole tensor's block-column count nb."""
    hd, d = cfg.head_dim, cfg.dim
    q0, q1 = shard.span(cfg.n_heads)
    k0, k1 = shard.span(cfg.n_kv_heads)
    f0, f1 = shard.span(cfg.ffn_dim)
    nbd, nbf = d // 256, cfg.ffn_dim // 256
    if (q0 * hd) % 256 or (q1 * hd) % 256 or f0 % 256 or f1 % 256:
        raise ValueError("a split column range is not whole Q4_K blocks")
    whole = lambda r0, r1, nb: {"row0": r0, "rows": r1 - r0, "kb0": 0, "nkb": nb, "nb": nb}
    return {
        "wq": whole(q0 * hd, q1 * hd, nbd),
        "wk": whole(k0 * hd, k1 * hd, nbd),
        "wv": whole(k0 * hd, k1 * hd, nbd),
        "wo": {"row0": 0, "rows": d, "kb0": q0 * hd // 256, "nkb": (q1 - q0) * hd // 256,
               "nb": nbd},
        "w_gate": whole(f0, f1, nbd),
        "w_up": whole(f0, f1, nbd),
        "w_down": {"row0": 0, "rows": d, "kb0": f0 // 256, "nkb": (f1 - f0) // 256, "nb": nbf},
    }


def output_shard(cfg, shard: Shard) -> dict:
    v0, v1 = shard.span(cfg.vocab)
    nb = cfg.dim // 256
    return {"row0": v0, "rows": v1 - v0, "kb0": 0, "nkb": nb, "nb": nb}
