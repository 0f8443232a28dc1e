"""Parity of the benchmark configurations' production kernels, and of the
output wrappers on the CUDA path.

* Multi-task backbone: ``Cherimoya(signal_groups=[1, 2, 2, 2, 2])`` at
  n_filters 128, 9 layers, 2114 bp (9 profile tracks, 5 count heads;
  upstream cherimoya/cherimoya.py:182-186, 384-399), on GC-skewed inputs.
  In bf16 mode this runs the warp-specialised MLP kernel and the fused
  tensor-core head with 9 (track, example) items per sequence and the five
  count Linears in the spare MMA operand rows; in fp32 mode the fp32 MLP and
  the split-precision head.
* Wrappers (upstream cherimoya/wrappers.py:11-166) on CUDA models against
  the upstream-produced ``wrap_*`` golden outputs.
* A batch of 1024 default-model sequences (the throughput configuration's
  launch shape: more tiles than CTAs, many per CTA) against the oracle on a
  sample of rows spread over the batch.

Tolerances as elsewhere: fp32 mode max abs error <= 1e-4; bf16 mode max abs
error <= 1e-2 and per-track profile Pearson >= 0.9999. Expected counts
(softmax x expm1(log-count)) are held to the bound those tolerances imply.
"""

import pytest
import torch

import cherimoya_b200 as cb
from oracle import cherimoya_oracle as O

pytestmark = pytest.mark.gpu

DEV = "cuda"
TOL = {"fp32": 1e-4, "bf16": 1e-2}
BF16_PEARSON = 0.9999
L = 2114


def _gc_bases(n, seed):
    """Per-sequence GC fraction gc ~ U(0.35, 0.65); C and G each gc / 2."""
    g = torch.Generator().manual_seed(seed)
    gc = 0.35 + 0.3 * torch.rand(n, 1, generator=g)
    u = torch.rand(n, L, generator=g)
    return torch.where(u < gc / 2, 1, torch.where(u < gc, 2,
                       torch.where(u < gc + (1 - gc) / 2, 0, 3)))


def _pearson_min(a, b):
    a = a.reshape(-1, a.shape[-1]).double()
    b = b.reshape(-1, b.shape[-1]).double()
    return float(O.pearson_corr(a, b).min())


def _check(mode, p, c, rp, rc, label):
    ep = (p - rp).abs().max().item()
    ec = (c - rc).abs().max().item()
    r = _pearson_min(p, rp)
    print(label, mode, "max|dprofile| %.3e max|dlogcount| %.3e pearson %.7f" % (ep, ec, r))
    assert ep <= TOL[mode] and ec <= TOL[mode]
    if mode == "bf16":
        assert r >= BF16_PEARSON


@pytest.mark.parametrize("mode", ["fp32", "bf16"])
def test_multitask_c128_9layer_against_oracle(mode):
    torch.manual_seed(0)
    m = cb.Cherimoya(signal_groups=[1, 2, 2, 2, 2], compile=False, precision=mode).eval()
    sd = {k: v.clone() for k, v in m.state_dict().items()}
    assert m.n_outputs == 9 and m.n_groups == 5 and m.n_filters == 128 and m.n_layers == 9
    X = O.one_hot(_gc_bases(24, 2))
    with torch.no_grad():
        rp, rc = O.forward(sd, m._init_kwargs(), X)
        p, c = m.to(DEV)(X.to(DEV))
    torch.cuda.synchronize()
    assert p.shape == (24, 9, 1000) and c.shape == (24, 5)
    _check(mode, p.cpu(), c.cpu(), rp, rc, "multitask")


@pytest.mark.parametrize("N,Lseq,T,groups,C", [
    (1, 129, 60, None, 128),       # 83-row window: one tile
    (3, 300, 53, None, 128),       # three tiles
    (200, 300, 53, None, 128),     # more items than CTAs: item boundaries inside a CTA
    (160, 400, 100, [2, 1], 128),  # three tracks, two count heads, 480 items
    (2, 2114, 0, None, 128),       # 2188-row window: eighteen tiles
    (4, 1000, 37, None, 128),      # eight tiles
    (150, 300, 53, None, 256),     # n_filters 256: two channel halves per tile
])
def test_fused_head_window_lengths_bf16(N, Lseq, T, groups, C):
    """The bf16 fused head sums each profile diagonal per tile and carries the
    74 outputs that straddle two tiles to the next tile's epilogue group; the
    count columns travel in the same carry. Window lengths of 1 to 18 tiles,
    odd and even tile counts, several items per CTA and several tracks."""
    torch.manual_seed(5)
    kw = {} if groups is None else {"signal_groups": groups}
    m = cb.Cherimoya(n_filters=C, n_layers=2, trimming=T, compile=False, precision="bf16",
                     **kw).eval()
    sd = {k: v.clone() for k, v in m.state_dict().items()}
    g = torch.Generator().manual_seed(6)
    X = O.one_hot(torch.randint(0, 4, (N, Lseq), generator=g))
    with torch.no_grad():
        rp, rc = O.forward(sd, m._init_kwargs(), X)
        p, c = m.to(DEV)(X.to(DEV))
    torch.cuda.synchronize()
    assert p.shape == rp.shape and c.shape == rc.shape
    _check("bf16", p.cpu(), c.cpu(), rp, rc, "head L=%d T=%d N=%d" % (Lseq, T, N))


def _golden_model(case, mode):
    m = cb.Cherimoya(**case["config"], compile=False, precision=mode)
    m.load_state_dict(case["state_dict"])
    return m.eval().to(DEV)


def _golden_inputs(case):
    X = case["X"] if case["X"] is not None else O.one_hot(case["bases"])
    X_ctl = case.get("X_ctl")
    return X.to(DEV), None if X_ctl is None else X_ctl.to(DEV)


@pytest.mark.parametrize("name,mode", [
    ("model_default_L2114", "fp32"), ("model_default_L2114", "bf16"),
    ("model_multitask", "fp32"), ("model_multitask", "bf16"),
    ("model_control_tracks", "fp32"),
])
def test_wrappers_on_cuda_match_upstream(golden, name, mode):
    case = golden(name)
    m = _golden_model(case, mode)
    X, X_ctl = _golden_inputs(case)
    out = case["outputs"]
    tol = TOL[mode]
    with torch.no_grad():
        ctl_p, ctl_c = cb.ControlWrapper(m)(X)
        prof = cb.ProfileWrapper(cb.ControlWrapper(m))(X)
        lc = cb.LogCountWrapper(cb.ControlWrapper(m))(X)
        exp = cb.ExpectedCountsWrapper(m)(X, X_ctl)
    torch.cuda.synchronize()
    assert ctl_p.is_cuda and prof.shape == out["wrap_profile"].shape
    e_ctl = (ctl_p.cpu() - out["wrap_control"]).abs().max().item()
    e_prof = (prof.cpu() - out["wrap_profile"]).abs().max().item()
    e_lc = (lc.cpu() - out["wrap_logcount"]).abs().max().item()
    # expected counts s * expm1(lc), s the group softmax: logit errors <= tol
    # move s by <= 2 tol s, a log-count error <= tol moves expm1(lc) by
    # <= tol exp(lc), so |d| <= tol s (2 |expm1(lc)| + exp(lc)) (1.5x margin)
    ref_exp = out["wrap_expected"]
    groups = case["config"]["signal_groups"]
    s_ref = torch.cat([torch.softmax(g.reshape(g.shape[0], -1), -1).reshape(g.shape)
                       for g in torch.split(out["profile"], groups, dim=1)], dim=1)
    lc_ref = torch.repeat_interleave(out["logcounts"], torch.tensor(groups), dim=1)[..., None]
    bound = 1.5 * tol * s_ref * (2 * torch.expm1(lc_ref).abs() + torch.exp(lc_ref))
    e_exp = ((exp.cpu() - ref_exp).abs() / bound).max().item()
    print(name, mode, "control %.2e profile %.2e logcount %.2e expected/bound %.2f"
          % (e_ctl, e_prof, e_lc, e_exp))
    assert e_ctl <= tol and e_prof <= tol and e_lc <= tol
    assert e_exp <= 1.0


def test_batch1024_bf16_rows_against_oracle(golden):
    """The throughput configuration (batch 1024, bf16 mode) on the engine;
    16 rows spread over the batch, first and last included, against the
    oracle."""
    case = golden("model_default_L2114")
    m = _golden_model(case, "bf16")
    g = torch.Generator().manual_seed(1)
    bases = torch.randint(0, 4, (1024, L), generator=g)
    with torch.no_grad():
        p, c = m(O.one_hot(bases).to(DEV))
    torch.cuda.synchronize()
    rows = torch.linspace(0, 1023, 16).round().long()
    with torch.no_grad():
        rp, rc = O.forward(case["state_dict"], case["config"], O.one_hot(bases[rows]))
    _check("bf16", p.cpu()[rows], c.cpu()[rows], rp, rc, "batch1024")
    assert torch.isfinite(p).all() and torch.isfinite(c).all()


def test_wrapper_epilogue_kernels_against_oracle():
    """The fused ExpectedCountsWrapper / ProfileWrapper kernels on random
    logits (grouped, 9 tracks) against the oracle's restatement of upstream
    wrappers.py:71-99, 125-166: fp32, relative error <= 1e-5."""
    from cherimoya_b200 import ops
    g = torch.Generator().manual_seed(7)
    p = torch.randn(5, 9, 1000, generator=g) * 3.0
    c = torch.randn(5, 5, generator=g)
    groups = [1, 2, 2, 2, 2]
    e = ops.expected_counts(p.to(DEV), c.to(DEV), groups).cpu()
    pw = ops.profile_wrapper(p.to(DEV)).cpu()
    ref_e = O.expected_counts(p, c, groups)
    ref_pw = O.profile_wrapper(p)
    assert e.shape == ref_e.shape and pw.shape == ref_pw.shape
    rel_e = ((e - ref_e).abs() / (ref_e.abs() + 1e-30)).max().item()
    rel_pw = ((pw - ref_pw).abs() / ref_pw.abs().clamp_min(1e-3)).max().item()
    print("epilogues: expected counts rel %.2e, profile wrapper rel %.2e" % (rel_e, rel_pw))
    assert rel_e <= 1e-5 and rel_pw <= 1e-5
