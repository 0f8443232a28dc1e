"""The MLP kernel's fused next-block LayerNorm statistics.

In bf16 mode at the default width, a batch large enough for whole examples
per CTA (at least one example per SM, e.g. 296 = 2 x 148 sequences) runs
every block's MLP launch with the next block's statistics computed inside it
from the rows it has just stored; a small batch computes them in a standalone
pass. Both use the same fixed decomposition of the statistics into work
units and the same combine order, and the per-tile MLP arithmetic does not
depend on which CTA runs a tile, so a sequence's outputs must be bitwise
equal on both paths. The large batch is also checked against the oracle on
sampled rows (bf16 tolerances: max abs error <= 1e-2, per-track profile
Pearson >= 0.9999).
"""

import pytest
import torch

import cherimoya_b200 as cb
from oracle import cherimoya_oracle as O

pytestmark = pytest.mark.gpu

DEV = "cuda"
L = 2114


def _model(**kw):
    torch.manual_seed(0)
    m = cb.Cherimoya(compile=False, precision="bf16", **kw).eval()
    sd = {k: v.clone() for k, v in m.state_dict().items()}
    return m.to(DEV), sd


def _run(m, X):
    with torch.no_grad():
        p, c = m(X.to(DEV))
    torch.cuda.synchronize()
    return p.cpu(), c.cpu()


@pytest.mark.parametrize("kw", [{}, {"signal_groups": [1, 2, 2, 2, 2]}],
                         ids=["default", "multitask"])
def test_fused_statistics_path_is_bitwise_equal_to_standalone(kw):
    m, _ = _model(**kw)
    g = torch.Generator().manual_seed(11)
    X = O.one_hot(torch.randint(0, 4, (296, L), generator=g))
    p_big, c_big = _run(m, X)                       # fused statistics
    rows = [0, 1, 147, 148, 200, 295]
    p_small, c_small = _run(m, X[rows])             # standalone statistics pass
    assert torch.equal(p_big[rows], p_small) and torch.equal(c_big[rows], c_small)


def test_fused_statistics_against_oracle():
    m, sd = _model()
    g = torch.Generator().manual_seed(12)
    bases = torch.randint(0, 4, (444, L), generator=g)
    p, c = _run(m, O.one_hot(bases))
    rows = torch.tensor([0, 73, 147, 148, 296, 443])
    with torch.no_grad():
        rp, rc = O.forward(sd, m._init_kwargs(), O.one_hot(bases[rows]))
    ep = (p[rows] - rp).abs().max().item()
    ec = (c[rows] - rc).abs().max().item()
    a, b = p[rows].reshape(-1, 1000).double(), rp.reshape(-1, 1000).double()
    r = float(O.pearson_corr(a, b).min())
    print("fused stats batch 444: max|dprofile| %.3e max|dlogcount| %.3e pearson %.7f"
          % (ep, ec, r))
    assert ep <= 1e-2 and ec <= 1e-2 and r >= 0.9999


def test_fused_statistics_repeatable():
    m, _ = _model()
    g = torch.Generator().manual_seed(13)
    X = O.one_hot(torch.randint(0, 4, (300, L), generator=g))
    p1, c1 = _run(m, X)
    p2, c2 = _run(m, X)
    assert torch.equal(p1, p2) and torch.equal(c1, c2)
