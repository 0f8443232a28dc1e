"""Bulk drivers of the hot path: saturation mutagenesis (ISM), ref/alt
variant scoring, and example-sharded multi-GPU execution.

Upstream delegates these to the third-party ``tangermeme`` package
(``cherimoya_cli/commands/attribute.py:54-64``;
``docs/tutorials/variant_effect.rst:50-69``), which builds mutant batches
on the host and moves them to the GPU. Here mutants are generated on the
device from (sequence, position, alternative) indices inside the stem
kernel, and scores are produced by a fused epilogue:

  d_logcount = logcount(mutant) - logcount(reference)
  jsd        = Jensen-Shannon distance between softmax(profile(reference))
               and softmax(profile(mutant)), flattened over channels and
               positions (upstream performance.py:171-207).

Multi-GPU: examples are independent (the per-example LayerNorm couples all
positions of one example and nothing else), so sequences / pairs are split
into contiguous shards, one per rank, with no collective on the data path;
one NCCL all-gather collects the scores at the end.
"""

import torch

from . import ops
from ._lib import MODE_BF16, MODE_FP32


def to_bases(X):
    """One-hot (N, 4, L) -> int8 base indices (N, L); all-zero columns -> 4."""
    if X.dim() == 2:
        return X.to(torch.int8)
    if X.dim() != 3 or X.shape[1] != 4:
        raise RuntimeError("expected one-hot (N, 4, L) or bases (N, L)")
    idx = X.argmax(dim=1).to(torch.int8)
    idx[X.abs().sum(dim=1) == 0] = 4
    return idx


def _mode(model, precision):
    p = precision or model.precision
    return MODE_BF16 if p == "bf16" else MODE_FP32


def saturation_mutagenesis(model, X, start=None, end=None, mutant_batch=2048, precision=None):
    """Score every single-base substitution in [start, end) of each sequence.

    X: one-hot (N, 4, L) or bases (N, L), on a CUDA device. Defaults to the
    model's output window [trimming, L - trimming). Returns
    (d_logcount (N, n_groups, 4, W), jsd (N, 4, W)); entries whose base is
    the reference base are 0.
    """
    bases = to_bases(X)
    if not bases.is_cuda:
        raise RuntimeError("cherimoya_b200: ISM needs CUDA input")
    L = bases.shape[1]
    start = model.trimming if start is None else int(start)
    end = L - model.trimming if end is None else int(end)
    buf, off = model.engine_weights(bases.device)
    desc = model.engine_desc(L, _mode(model, precision))
    with torch.no_grad():
        return ops.ism(bases, start, end, int(mutant_batch), buf, off, desc,
                       float(model.residual_scale))


def variant_effect(model, X_ref, X_alt, precision=None):
    """Ref/alt scoring: (d_logcount (N, n_groups), jsd (N,))."""
    ref, alt = to_bases(X_ref), to_bases(X_alt)
    if not ref.is_cuda:
        raise RuntimeError("cherimoya_b200: variant scoring needs CUDA input")
    buf, off = model.engine_weights(ref.device)
    desc = model.engine_desc(ref.shape[1], _mode(model, precision))
    with torch.no_grad():
        return ops.variant(ref, alt.to(ref.device), buf, off, desc, float(model.residual_scale))


# ----------------------------------------------------------------- sharding
def shard_range(n, rank, world):
    """Contiguous shard of n items for `rank`; the remainder goes to the
    lowest ranks."""
    base, rem = divmod(n, world)
    lo = rank * base + min(rank, rem)
    return lo, lo + base + (1 if rank < rem else 0)


def gather_shards(local, n_total, group=None):
    """All-gather per-rank shards (first dim) into the full (n_total, ...)
    tensor on every rank. Shards may differ by one row; they are padded to
    equal size for the collective and trimmed after."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    sizes = [shard_range(n_total, r, world) for r in range(world)]
    max_rows = max(hi - lo for lo, hi in sizes)
    padded = local.new_zeros((max_rows,) + tuple(local.shape[1:]))
    padded[:local.shape[0]] = local
    bufs = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(bufs, padded, group=group)
    return torch.cat([b[:hi - lo] for b, (lo, hi) in zip(bufs, sizes)], dim=0)


def sharded_saturation_mutagenesis(model, X, start=None, end=None, mutant_batch=2048,
                                   precision=None, group=None):
    """ISM over all ranks of the default (or given) process group: each rank
    scores its contiguous shard of sequences on its own GPU, then the
    scores are all-gathered. Every rank passes the same full X."""
    import torch.distributed as dist
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    lo, hi = shard_range(X.shape[0], rank, world)
    d, j = saturation_mutagenesis(model, X[lo:hi], start, end, mutant_batch, precision)
    return gather_shards(d, X.shape[0], group), gather_shards(j, X.shape[0], group)


def sharded_variant_effect(model, X_ref, X_alt, precision=None, group=None):
    """Variant scoring sharded by pair across ranks, then all-gathered."""
    import torch.distributed as dist
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    lo, hi = shard_range(X_ref.shape[0], rank, world)
    d, j = variant_effect(model, X_ref[lo:hi], X_alt[lo:hi], precision)
    return gather_shards(d, X_ref.shape[0], group), gather_shards(j, X_ref.shape[0], group)
