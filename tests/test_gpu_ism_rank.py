"""Saturation mutagenesis on the default model (n_filters 128, 9 layers,
2114 bp) against the oracle: score errors, and whether the four bases at
each position come out in the same order (the rank order that ISM
attributions are read from).

With random-init weights the Delta-logcounts are of order 1e-5 and two
bases at one position can differ by a few 1e-8, below the fp32 rounding of
a log-count itself. The test therefore requires identical order at every
position whose adjacent sorted oracle scores are at least RESOLVED apart
(far above the fp32 error of the engine's log-counts) and reports the rate
over all positions; bf16 mode reports both rates and holds the score
errors to the bf16 tolerance."""

import os

import pytest
import torch

import cherimoya_b200 as cb
from oracle import cherimoya_oracle as O

pytestmark = pytest.mark.gpu

START, END = 1041, 1073          # 32 positions around the centre of the output window
RESOLVED = 1e-6


@pytest.fixture(scope="module")
def ism_case():
    case = torch.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden",
                                   "model_default_L2114.pt"), weights_only=False)
    g = torch.Generator().manual_seed(31)
    bases = torch.randint(0, 4, (2, 2114), generator=g)
    dlc, jsd, _, _ = O.ism_scores(case["state_dict"], case["config"], bases, START, END)
    return case, bases, dlc, jsd


def _engine(case, bases, precision):
    m = cb.Cherimoya(**case["config"], compile=False, precision=precision)
    m.load_state_dict(case["state_dict"])
    m = m.eval().to("cuda")
    d, j = cb.saturation_mutagenesis(m, bases.to("cuda"), START, END)
    torch.cuda.synchronize()
    return d[:, 0].cpu(), j.cpu()


def _agreement(ref, got):
    """(rate over all positions, rate over resolved positions, number of
    resolved positions) of identical base order."""
    same = (ref.argsort(dim=1) == got.argsort(dim=1)).all(dim=1)
    srt = ref.sort(dim=1).values
    resolved = (srt[:, 1:] - srt[:, :-1]).min(dim=1).values >= RESOLVED
    n_res = int(resolved.sum())
    res_rate = same[resolved].float().mean().item() if n_res else 1.0
    return same.float().mean().item(), res_rate, n_res


@pytest.mark.parametrize("precision", ["fp32", "bf16"])
def test_default_model_ism_rank_order(ism_case, precision):
    case, bases, ref_d, ref_j = ism_case
    d, j = _engine(case, bases, precision)
    ed, ej = (d - ref_d).abs().max().item(), (j - ref_j).abs().max().item()
    full, res_rate, n_res = _agreement(ref_d, d)
    print("%s ism max|d dlogcount| %.3e max|d jsd| %.3e rank order: all %d positions %.4f, "
          "%d resolved positions %.4f" % (precision, ed, ej, d.shape[0] * d.shape[2], full,
                                          n_res, res_rate))
    if precision == "fp32":
        assert ed <= 1e-4 and ej <= 1e-4
        assert res_rate == 1.0
    else:
        assert ed <= 1e-2 and ej <= 1e-2
