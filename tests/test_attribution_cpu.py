"""Host logic of the tangermeme-call-shape ISM front end: target resolution,
the attribution convention, and the control-free model a zero-control
ControlWrapper amounts to (checked against the oracle forward on CPU)."""

import pytest
import torch

import cherimoya_b200 as cb
from cherimoya_b200 import attribution as A
from oracle import cherimoya_oracle as O


def test_resolve_target():
    m = cb.Cherimoya(n_filters=16, n_layers=2, compile=False)
    assert A.resolve_target(cb.LogCountWrapper(cb.ControlWrapper(m))) == (A.LOGCOUNT, m)
    assert A.resolve_target(cb.ProfileWrapper(m)) == (A.PROFILE, m)
    with pytest.raises(TypeError):
        A.resolve_target(m)
    with pytest.raises(TypeError):
        A.resolve_target(cb.ExpectedCountsWrapper(m))


def test_convention_centres_and_masks():
    delta = torch.randn(2, 4, 5)
    X = O.one_hot(torch.randint(0, 4, (2, 5)))
    hyp = A.attributions(delta, X, hypothetical=True)
    assert torch.allclose(hyp.mean(dim=1), torch.zeros(2, 5), atol=1e-6)
    obs = A.attributions(delta, X, hypothetical=False)
    assert torch.equal(obs, hyp * X)
    assert torch.equal(A.attributions(delta, X, center=False), delta)


def test_control_free_model_equals_zero_controls():
    torch.manual_seed(1)
    m = cb.Cherimoya(n_filters=16, n_layers=2, n_control_tracks=2, signal_groups=[2],
                     trimming=20, compile=False).eval()
    X = O.one_hot(torch.randint(0, 4, (2, 120)))
    m0 = A.control_free(m)
    assert m0.n_control_tracks == 0 and A.control_free(m) is m0
    with torch.no_grad():
        p, c = cb.ControlWrapper(m)(X)
        p0, c0 = m0(X)
    assert torch.allclose(p, p0, atol=1e-6) and torch.allclose(c, c0, atol=1e-6)


def test_rejects_extra_inputs_and_cpu():
    m = cb.Cherimoya(n_filters=16, n_layers=2, compile=False)
    X = O.one_hot(torch.randint(0, 4, (1, 100)))
    with pytest.raises(RuntimeError):
        A.saturation_mutagenesis(cb.LogCountWrapper(m), X, args=(X,))
    with pytest.raises(RuntimeError):
        A.saturation_mutagenesis(cb.LogCountWrapper(m), X, device="cpu")
