"""Batched prediction through the engine: host inputs pipelined through
pinned staging and a copy stream, device-resident inputs, control tracks,
reverse-complement averaging (cherimoya_cli/commands/evaluate.py:80-96) as
one doubled-batch forward, and bf16 mode; each compared with the oracle
on the same inputs and state_dict."""

import pytest
import torch

import cherimoya_b200 as cb
from oracle import cherimoya_oracle as O

pytestmark = pytest.mark.gpu

FP32_TOL = 1e-4
BF16_TOL = 1e-2
BF16_PEARSON = 0.9999


def _model(case, precision="auto"):
    m = cb.Cherimoya(**case["config"], compile=False, precision=precision)
    m.load_state_dict(case["state_dict"])
    return m.eval().to("cuda")


def _bases(n, L, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, 4, (n, L), generator=g)


def _maxdiff(a, b):
    return float((a - b).abs().max())


@pytest.mark.parametrize("pinned", [False, True])
def test_predict_host_input_default_model(golden, pinned):
    case = golden("model_default_L2114")
    m = _model(case)
    X = O.one_hot(_bases(11, 2114, 21))
    if pinned:
        X = X.pin_memory()
    p, c = cb.predict(m, X, batch_size=4, device="cuda")
    assert not p.is_cuda and not c.is_cuda
    ref_p, ref_c = O.forward(case["state_dict"], case["config"], X)
    assert _maxdiff(p, ref_p) <= FP32_TOL and _maxdiff(c, ref_c) <= FP32_TOL


def test_predict_reverse_complement_with_controls(golden):
    case = golden("model_control_tracks")
    m = _model(case)
    X = O.one_hot(_bases(5, 300, 22))
    g = torch.Generator().manual_seed(23)
    X_ctl = torch.poisson(torch.full((5, 2, 300), 0.5), generator=g)
    p, c = cb.predict(m, X, args=(X_ctl,), batch_size=2, device="cuda",
                      reverse_complement_average=True)
    ref_p, ref_c = O.reverse_complement_average(case["state_dict"], case["config"], X, X_ctl)
    assert _maxdiff(p, ref_p) <= FP32_TOL and _maxdiff(c, ref_c) <= FP32_TOL


def test_predict_device_resident_reverse_complement_multitask(golden):
    case = golden("model_multitask")
    m = _model(case)
    X = O.one_hot(_bases(6, 400, 24))
    p, c = cb.predict(m, X.cuda(), batch_size=4, device="cuda",
                      reverse_complement_average=True)
    ref_p, ref_c = O.reverse_complement_average(case["state_dict"], case["config"], X)
    assert _maxdiff(p, ref_p) <= FP32_TOL and _maxdiff(c, ref_c) <= FP32_TOL


def test_predict_bfloat16_default_model(golden):
    case = golden("model_default_L2114")
    m = _model(case)
    X = O.one_hot(_bases(6, 2114, 25))
    p, c = cb.predict(m, X, batch_size=4, device="cuda", dtype="bfloat16")
    ref_p, ref_c = O.forward(case["state_dict"], case["config"], X)
    r = O.pearson_corr(p.reshape(-1, p.shape[-1]).double(),
                       ref_p.reshape(-1, ref_p.shape[-1]).double())
    assert _maxdiff(p, ref_p) <= BF16_TOL and _maxdiff(c, ref_c) <= BF16_TOL
    assert float(r.min()) >= BF16_PEARSON
