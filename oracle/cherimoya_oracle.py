"""CPU oracle for the Cherimoya inference hot path.  TEST INFRASTRUCTURE ONLY.

This module restates, in plain PyTorch CPU fp32 ops, the algorithm of the
upstream Cherimoya v0.2.1 inference path so that the CUDA engine can be
checked against it. It is imported only by ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py``; the engine (``cherimoya_b200``) never imports it.

Parity is pinned: ``tests/test_oracle.py`` checks every function here
against golden vectors produced by the upstream package itself
(``tests/golden/make_golden.py``).

Each function cites the upstream file:line it restates (paths relative to
the upstream project root).
"""

import math

import torch
import torch.nn.functional as F

CONV_NORM_EPS = 1e-3          # cherimoya/cheri.py:49
GELU_K = math.sqrt(2.0 / math.pi)


def gelu_tanh(x):
    """GELU, tanh approximation (torch.nn.GELU(approximate='tanh'),
    cherimoya/cherimoya.py:174 and cherimoya/cheri.py:935):
    0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3)))."""
    return 0.5 * x * (1.0 + torch.tanh(GELU_K * (x + 0.044715 * x * x * x)))


def dilated_depthwise_conv(x, w, dilation):
    """3-tap depthwise dilated conv over (N, L, C), zero padding.

    y[n, i, c] = w[0,c] x[n,i-d,c] + w[1,c] x[n,i,c] + w[2,c] x[n,i+d,c]
    with x outside [0, L) read as zero (cherimoya/cheri.py:84-90; tap
    semantics pinned by tests/test_cheri.py:49-73 upstream).
    """
    N, L, C = x.shape
    d = int(dilation)
    y = x * w[1]
    if d < L:
        y[:, d:, :] += x[:, :L - d, :] * w[0]
        y[:, :L - d, :] += x[:, d:, :] * w[2]
    return y


def conv_norm(x, w, dilation, eps=CONV_NORM_EPS):
    """Fused dilated conv + per-example LayerNorm over the (L, C) plane.

    cherimoya/cheri.py:52-98: mean and biased variance over all L*C values
    of each example, computed in fp32; no affine; result cast back to x's
    dtype.
    """
    N, L, C = x.shape
    y = dilated_depthwise_conv(x.float(), w.float(), dilation)
    flat = y.reshape(N, -1)
    mean = flat.mean(dim=1, keepdim=True)
    var = flat.var(dim=1, keepdim=True, unbiased=False)
    flat = (flat - mean) * torch.rsqrt(var + eps)
    return flat.reshape(N, L, C).to(x.dtype)


def cheri_block(x, conv_w, w1, w2, dilation, residual_scale):
    """One Cheri Block, CPU branch (cherimoya/cheri.py:1080-1082):
    out = x + residual_scale * (gelu(conv_norm(x) @ w1^T) @ w2^T)."""
    h = conv_norm(x, conv_w, dilation)
    h = gelu_tanh(h @ w1.t())
    return x + (h @ w2.t()) * residual_scale


def block_weights(sd, i):
    """Block i's (conv_w, w1, w2) from a state_dict in the checkpoint layout
    (legacy ``blocks.i.conv_weight`` key, cherimoya/cheri.py:829-855;
    ``blocks.i.conv.conv_weight`` also accepted, cheri.py:986-1002)."""
    p = "blocks.{}.".format(i)
    cw = sd.get(p + "conv_weight", sd.get(p + "conv.conv_weight"))
    return cw, sd[p + "linear1.weight"], sd[p + "linear2.weight"]


def default_trimming(n_layers):
    """cherimoya/cherimoya.py:170-171."""
    return 46 + sum(2 ** i for i in range(n_layers))


def forward(sd, config, X, X_ctl=None):
    """Cherimoya._forward_impl (cherimoya/cherimoya.py:340-400), CPU fp32.

    X: (N, 4, L) float; X_ctl: (N, n_control_tracks, L) or None.
    Returns (profile (N, n_outputs, L - 2T), logcounts (N, n_groups)).
    """
    n_layers = int(config["n_layers"])
    rs = float(config.get("residual_scale", 0.15))
    T = config.get("trimming")
    if T is None:
        T = default_trimming(n_layers)
    L = X.shape[2]
    start, end = T, L - T
    X = X.float()
    # stem: Conv1d(4, C, 21, padding=10) + GELU(tanh)   (cherimoya.py:173-174, 373)
    h = gelu_tanh(F.conv1d(X, sd["iconv.weight"], sd["iconv.bias"], padding=10))
    h = h.transpose(1, 2).contiguous()                 # (N, L, C)    (cherimoya.py:374)
    for i in range(n_layers):                          # (cherimoya.py:375-376)
        cw, w1, w2 = block_weights(sd, i)
        h = cheri_block(h, cw, w1, w2, 2 ** i, rs)
    h = h.transpose(1, 2).contiguous()                 # (N, C, L)    (cherimoya.py:378)
    h_ctl = h if X_ctl is None else torch.cat([h, X_ctl.float()], dim=1)
    # profile head: Conv1d(C(+ctl), n_out, 75, padding=37), trimmed (cherimoya.py:182-184, 384)
    profile = F.conv1d(h_ctl, sd["fconv.weight"], sd["fconv.bias"], padding=37)[:, :, start:end]
    # count head: mean over the trimmed window, then Linear (cherimoya.py:387-399)
    m = h[:, :, start:end].float().mean(dim=2)
    if X_ctl is not None:
        c = X_ctl[:, :, start:end].float().sum(dim=(1, 2)).unsqueeze(-1)
        m = torch.cat([m, torch.log(c + 1)], dim=-1)
    logcounts = m @ sd["linear.weight"].t() + sd["linear.bias"]
    return profile, logcounts


# ----------------------------------------------------------------------------
# wrappers (cherimoya/wrappers.py)

def control_inputs(config, X, X_ctl=None):
    """ControlWrapper (wrappers.py:38-47): zero control tracks of X's shape
    when the model expects controls and none are given."""
    n_ctl = int(config.get("n_control_tracks", 0))
    if X_ctl is not None or n_ctl == 0:
        return X_ctl
    return torch.zeros(X.shape[0], n_ctl, X.shape[-1], dtype=X.dtype)


def profile_wrapper(profile):
    """ProfileWrapper (wrappers.py:95-99): flatten, mean-centre, then
    sum(softmax(l) * l) per example -> (N, 1)."""
    lg = profile.reshape(profile.shape[0], -1)
    lg = lg - lg.mean(dim=-1, keepdim=True)
    return (lg * torch.softmax(lg, dim=-1)).sum(dim=-1, keepdim=True)


def expected_counts(profile, logcounts, signal_groups):
    """ExpectedCountsWrapper (wrappers.py:154-166): per signal group, a joint
    softmax over (channels, positions) times expm1(group logcount)."""
    counts = torch.expm1(logcounts)
    outs = []
    for i, lg in enumerate(torch.split(profile, list(signal_groups), dim=1)):
        N, c, L = lg.shape
        p = torch.softmax(lg.reshape(N, -1), dim=-1).reshape(N, c, L)
        outs.append(p * counts[:, i, None, None])
    return torch.cat(outs, dim=1)


# ----------------------------------------------------------------------------
# metrics (cherimoya/performance.py)

def kl_divergence(p1, p2):
    """_kl_divergence (performance.py:138-168): sum p1 log(p1/p2) over the
    last axis, terms where either probability is zero contribute 0."""
    ok = (p1 != 0) & (p2 != 0)
    q = torch.ones_like(p1)
    q[ok] = (p1 / p2)[ok]
    return torch.sum(p1 * torch.log(q), dim=-1)


def jensen_shannon_distance(logps, counts):
    """jensen_shannon_distance (performance.py:171-207): exp + renormalise
    the first argument, renormalise the second, JS divergence over the last
    axis (natural log)."""
    p1 = torch.exp(logps)
    p1 = p1 / p1.sum(dim=-1, keepdim=True)
    p2 = (counts / counts.sum(dim=-1, keepdim=True)).to(p1.dtype)
    mid = 0.5 * (p1 + p2)
    return 0.5 * (kl_divergence(p1, mid) + kl_divergence(p2, mid))


def pearson_corr(a, b):
    """pearson_corr (performance.py:210-246), 0 where a variance is 0."""
    da = a - a.mean(dim=-1, keepdim=True)
    db = b - b.mean(dim=-1, keepdim=True)
    num = (da * db).sum(dim=-1)
    den = torch.sqrt((da * da).sum(dim=-1) * (db * db).sum(dim=-1))
    out = torch.zeros_like(num)
    nz = den != 0
    out[nz] = num[nz] / den[nz]
    return out


# ----------------------------------------------------------------------------
# bulk drivers: saturation mutagenesis and ref/alt variant scoring

def one_hot(bases, dtype=torch.float32):
    """(N, L) integer bases in 0..3 (A, C, G, T) -> (N, 4, L) one-hot."""
    return F.one_hot(bases.long(), 4).permute(0, 2, 1).to(dtype).contiguous()


def ism_scores(sd, config, bases, start, end, batch=256):
    """Saturation mutagenesis over positions [start, end) of each sequence.

    For sequence n, position p and base b the mutant is the reference with
    base b at p (b equal to the reference base reproduces the reference).
    Scores, following the upstream ISM metric:
      d_logcount[n, b, p-start] = logcount(mutant)[0] - logcount(ref)[0]
      jsd[n, b, p-start] = jensen_shannon_distance(profile(mutant) flattened,
                                                   softmax(profile(ref)) flattened)
    Returns (d_logcount, jsd), each (N, 4, end - start) fp32, and the
    reference outputs.
    """
    X = one_hot(bases)
    N, _, L = X.shape
    W = end - start
    dlc = torch.zeros(N, 4, W)
    jsd = torch.zeros(N, 4, W)
    with torch.no_grad():
        p_ref, c_ref = forward(sd, config, X)
        for n in range(N):
            pos = torch.arange(start, end).repeat_interleave(4)
            alt = torch.arange(4).repeat(W)
            for s in range(0, 4 * W, batch):
                pp, aa = pos[s:s + batch], alt[s:s + batch]
                Xm = X[n].unsqueeze(0).repeat(len(pp), 1, 1)
                Xm[torch.arange(len(pp)), :, pp] = 0.0
                Xm[torch.arange(len(pp)), aa, pp] = 1.0
                pm, cm = forward(sd, config, Xm)
                d = cm[:, 0] - c_ref[n, 0]
                pr = torch.softmax(p_ref[n].reshape(1, -1), dim=-1).expand(len(pp), -1)
                j = jensen_shannon_distance(pm.reshape(len(pp), -1), pr)
                dlc[n, aa, pp - start] = d
                jsd[n, aa, pp - start] = j
    return dlc, jsd, p_ref, c_ref


def ism_wrapper_deltas(sd, config, bases, start, end, kind, target=0, batch=256):
    """Change of an attribution target's scalar in every single-base mutant
    of positions [start, end) (the targets of the upstream attribute command,
    cherimoya_cli/commands/attribute.py:46-51): kind "logcount" -> the
    LogCountWrapper output column `target` (wrappers.py:102-122), kind
    "profile" -> the ProfileWrapper value (wrappers.py:71-99), each through a
    ControlWrapper (zero controls, wrappers.py:38-47). Returns (N, 4, W):
    y(reference with base b at p) - y(reference), by explicit mutant
    forwards."""
    def y(X):
        p, c = forward(sd, config, X, control_inputs(config, X))
        return c[:, target] if kind == "logcount" else profile_wrapper(p)[:, 0]

    X = one_hot(bases)
    N, _, L = X.shape
    W = end - start
    out = torch.zeros(N, 4, W)
    with torch.no_grad():
        y_ref = y(X)
        pos = torch.arange(start, end).repeat_interleave(4)
        alt = torch.arange(4).repeat(W)
        for n in range(N):
            for s in range(0, 4 * W, batch):
                pp, aa = pos[s:s + batch], alt[s:s + batch]
                Xm = X[n].unsqueeze(0).repeat(len(pp), 1, 1)
                Xm[torch.arange(len(pp)), :, pp] = 0.0
                Xm[torch.arange(len(pp)), aa, pp] = 1.0
                out[n, aa, pp - start] = y(Xm) - y_ref[n]
    return out


def variant_scores(sd, config, ref_bases, alt_bases):
    """Ref/alt variant-effect scoring (the pattern of the upstream tutorial
    docs/tutorials/variant_effect.rst:50-69: predict both, take the delta).

    Returns d_logcount (N, n_groups) = logcount(alt) - logcount(ref) and
    jsd (N,) between softmax(profile(ref)) and profile(alt) (flattened).
    """
    with torch.no_grad():
        p_r, c_r = forward(sd, config, one_hot(ref_bases))
        p_a, c_a = forward(sd, config, one_hot(alt_bases))
    N = p_r.shape[0]
    pr = torch.softmax(p_r.reshape(N, -1), dim=-1)
    j = jensen_shannon_distance(p_a.reshape(N, -1), pr)
    return c_a - c_r, j


def reverse_complement_average(sd, config, X, X_ctl=None):
    """Forward / reverse-complement averaging of the upstream evaluate command
    (cherimoya_cli/commands/evaluate.py:80-96): the reverse complement flips
    the base and position axes of X (and of X_ctl), its profile is flipped
    back over channels and positions, and both outputs are averaged with the
    forward strand's."""
    with torch.no_grad():
        p, c = forward(sd, config, X, X_ctl)
        p_rc, c_rc = forward(sd, config, torch.flip(X, dims=(-1, -2)),
                             None if X_ctl is None else torch.flip(X_ctl, dims=(-1, -2)))
    return (p + torch.flip(p_rc, dims=(-1, -2))) / 2, (c + c_rc) / 2
