"""Batched prediction and reverse-complement averaging on CPU: the batching
and argument handling of ``cherimoya_b200.predict`` (the call shape of the
upstream ``predict`` call sites, cherimoya/cherimoya.py:567-568 and
cherimoya_cli/commands/evaluate.py:70-78) and the strand averaging of
cherimoya_cli/commands/evaluate.py:80-96 against the oracle."""

import pytest
import torch

import cherimoya_b200 as cb
from oracle import cherimoya_oracle as O

TOL = 2e-5


def _model(case):
    m = cb.Cherimoya(**case["config"], compile=False)
    m.load_state_dict(case["state_dict"])
    return m.eval()


def _bases(n, L, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, 4, (n, L), generator=g)


def _ctl(n, tracks, L, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.poisson(torch.full((n, tracks, L), 0.5), generator=g)


def _maxdiff(a, b):
    return float((a - b).abs().max())


@pytest.mark.parametrize("batch_size", [1, 3, 7, 64])
def test_predict_matches_one_forward(golden, batch_size):
    case = golden("model_multitask")
    m = _model(case)
    X = O.one_hot(_bases(7, 400, 11))
    p, c = cb.predict(m, X, batch_size=batch_size, device="cpu")
    ref_p, ref_c = O.forward(case["state_dict"], case["config"], X)
    assert p.shape == ref_p.shape and c.shape == ref_c.shape
    assert _maxdiff(p, ref_p) < TOL and _maxdiff(c, ref_c) < TOL


def test_predict_passes_control_tracks(golden):
    case = golden("model_control_tracks")
    m = _model(case)
    X = O.one_hot(_bases(5, 300, 12))
    X_ctl = _ctl(5, 2, 300, 13)
    p, c = cb.predict(m, X, args=(X_ctl,), batch_size=2, device="cpu")
    ref_p, ref_c = O.forward(case["state_dict"], case["config"], X, X_ctl)
    assert _maxdiff(p, ref_p) < TOL and _maxdiff(c, ref_c) < TOL


def test_predict_single_output_wrapper(golden):
    case = golden("model_multitask")
    m = _model(case)
    X = O.one_hot(_bases(5, 400, 14))
    lc = cb.predict(cb.LogCountWrapper(m), X, batch_size=2, device="cpu")
    assert isinstance(lc, torch.Tensor) and lc.shape == (5, 5)
    _, ref_c = O.forward(case["state_dict"], case["config"], X)
    assert _maxdiff(lc, ref_c) < TOL


@pytest.mark.parametrize("name", ["model_multitask", "model_control_tracks"])
def test_reverse_complement_average_matches_oracle(golden, name):
    case = golden(name)
    m = _model(case)
    L = 400 if name == "model_multitask" else 300
    X = O.one_hot(_bases(5, L, 15))
    X_ctl = _ctl(5, 2, L, 16) if name == "model_control_tracks" else None
    args = None if X_ctl is None else (X_ctl,)
    p, c = cb.predict(m, X, args=args, batch_size=2, device="cpu",
                      reverse_complement_average=True)
    ref_p, ref_c = O.reverse_complement_average(case["state_dict"], case["config"], X, X_ctl)
    assert _maxdiff(p, ref_p) < TOL and _maxdiff(c, ref_c) < TOL


def test_oracle_reverse_complement_average_is_strand_symmetric(golden):
    """Averaging the reverse complement of X gives the strand-flipped
    average of X: the same two sums with the operands swapped."""
    case = golden("model_multitask")
    X = O.one_hot(_bases(3, 400, 17))
    p, c = O.reverse_complement_average(case["state_dict"], case["config"], X)
    p2, c2 = O.reverse_complement_average(case["state_dict"], case["config"],
                                          torch.flip(X, dims=(-1, -2)))
    assert torch.equal(p2, torch.flip(p, dims=(-1, -2))) and torch.equal(c2, c)


def test_predict_bfloat16_is_cpu_autocast(golden):
    case = golden("model_small_float_input")
    m = _model(case)
    X = case["X"]
    p, c = cb.predict(m, X, batch_size=2, device="cpu", dtype="bfloat16")
    with torch.no_grad(), torch.autocast("cpu", dtype=torch.bfloat16):
        ref = [m(X[s:s + 2]) for s in range(0, X.shape[0], 2)]
    assert torch.equal(p, torch.cat([r[0] for r in ref]))
    assert torch.equal(c, torch.cat([r[1] for r in ref]))


def test_predict_argument_errors(golden):
    case = golden("model_small_float_input")
    m = _model(case)
    X = case["X"]
    with pytest.raises(ValueError):
        cb.predict(m, X, device="cpu", dtype="float16")
    with pytest.raises(ValueError):
        cb.predict(m, X, args=(X[:1],), device="cpu")
    with pytest.raises(ValueError):
        cb.predict(m, X[:0], device="cpu")
    with pytest.raises(ValueError):
        cb.predict(m, X, batch_size=0, device="cpu")
    with pytest.raises(RuntimeError):
        cb.predict(cb.LogCountWrapper(m), X, device="cpu", reverse_complement_average=True)
