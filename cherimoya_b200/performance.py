"""Profile-comparison metrics used to score ISM and variants, drop-in for the
scoring part of upstream ``cherimoya/performance.py``."""

import torch


def _kl_divergence(probs1, probs2):
    """sum p1 log(p1/p2) over the last axis; zero-probability terms
    contribute 0 (upstream performance.py:138-168)."""
    idxs = (probs1 != 0) & (probs2 != 0)
    quot = torch.ones_like(probs1)
    quot[idxs] = (probs1 / probs2)[idxs]
    return torch.sum(probs1 * torch.log(quot), dim=-1)


def jensen_shannon_distance(logps, true_counts):
    """JS divergence between exp(logps) and true_counts, each renormalised
    over the last axis (upstream performance.py:171-207)."""
    probs1 = torch.exp(logps)
    probs1 = torch.divide(probs1, torch.sum(probs1, dim=-1, keepdims=True))
    probs2 = torch.divide(true_counts, torch.sum(true_counts, dim=-1, keepdims=True))
    probs2 = probs2.type(probs1.dtype)
    mid = 0.5 * (probs1 + probs2)
    return 0.5 * (_kl_divergence(probs1, mid) + _kl_divergence(probs2, mid))


def pearson_corr(arr1, arr2):
    """Pearson correlation over the last axis, 0 where a variance is 0
    (upstream performance.py:210-246)."""
    dev1 = arr1 - torch.mean(arr1, dim=-1, keepdim=True)
    dev2 = arr2 - torch.mean(arr2, dim=-1, keepdim=True)
    numer = torch.sum(dev1 * dev2, dim=-1)
    denom = torch.sqrt(torch.sum(dev1 * dev1, dim=-1) * torch.sum(dev2 * dev2, dim=-1))
    out = torch.zeros_like(numer)
    nz = denom != 0
    out[nz] = numer[nz] / denom[nz]
    return out
