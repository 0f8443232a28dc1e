"""The tangermeme-call-shape ISM front end (cherimoya_b200.attribution) on
the upstream attribute command's targets, against the oracle.

The command (upstream cherimoya_cli/commands/attribute.py:43-64) builds
LogCountWrapper(ControlWrapper(model)) or ProfileWrapper(ControlWrapper(model))
and calls saturation_mutagenesis(wrapper, X, dtype=..., device=...,
batch_size=..., hypothetical=True, start=mid - 200, end=mid + 200). Here the
same call runs the engine's fused ISM; the oracle forwards every mutant
explicitly (oracle.ism_wrapper_deltas) and the same convention (centre over
the four bases, times X unless hypothetical) is applied to its deltas.

Tolerances: fp32 mode max abs error <= 1e-4 on the attributions; the base
order per position must agree wherever the oracle's sorted values are at
least 1e-6 apart (random-init deltas are ~1e-5 with near ties).
"""

import pytest
import torch

import cherimoya_b200 as cb
from cherimoya_b200 import attribution as A
from oracle import cherimoya_oracle as O

pytestmark = pytest.mark.gpu

L = 2114


def _order_agreement(a, b, gap=1e-6):
    """Positions whose oracle base values are resolvable (consecutive sorted
    values >= gap apart) and of those the fraction with the same base order."""
    sb, ib = torch.sort(b, dim=1)
    ia = torch.argsort(a, dim=1)
    resolved = (sb[:, 1:] - sb[:, :-1]).min(dim=1).values >= gap
    same = (ia == ib).all(dim=1)
    return int(resolved.sum()), float(same[resolved].float().mean()) if resolved.any() else 1.0


@pytest.mark.parametrize("kind", ["counts", "profile"])
def test_attribute_command_call_against_oracle(kind):
    torch.manual_seed(0)
    model = cb.Cherimoya(compile=False).eval()
    sd = {k: v.clone() for k, v in model.state_dict().items()}
    model = model.to("cuda")
    g = torch.Generator().manual_seed(21)
    bases = torch.randint(0, 4, (2, L), generator=g)
    X = O.one_hot(bases)
    mid = L // 2
    start, end = mid - 16, mid + 16
    wrapped = cb.ControlWrapper(model)
    wrapper = cb.LogCountWrapper(wrapped) if kind == "counts" else cb.ProfileWrapper(wrapped)
    attr = A.saturation_mutagenesis(wrapper, X, dtype=torch.float32, device="cuda",
                                    batch_size=64, verbose=False, hypothetical=True,
                                    start=start, end=end).float()
    assert attr.shape == (2, 4, end - start) and attr.device.type == "cpu"
    delta = O.ism_wrapper_deltas(sd, model._init_kwargs(), bases, start, end,
                                 "logcount" if kind == "counts" else "profile")
    ref = A.attributions(delta, X[:, :, start:end], hypothetical=True)
    err = (attr - ref).abs().max().item()
    n_res, agree = _order_agreement(attr.permute(0, 2, 1).reshape(-1, 4),
                                    ref.permute(0, 2, 1).reshape(-1, 4))
    print(kind, "max|dattr| %.3e, order agreement %.3f over %d resolved positions"
          % (err, agree, n_res))
    assert err <= 1e-4
    assert agree == 1.0
    # hypothetical=False keeps the observed base's value only
    obs = A.saturation_mutagenesis(wrapper, X, device="cuda", start=start, end=end)
    assert torch.allclose(obs, attr * X[:, :, start:end], atol=0, rtol=0)


def test_raw_outputs_and_control_track_model():
    """A model with control tracks under ControlWrapper (zero controls) and
    raw_outputs: y(reference) and y(mutant) against the oracle."""
    torch.manual_seed(3)
    model = cb.Cherimoya(n_filters=32, n_layers=3, n_control_tracks=2, signal_groups=[2],
                         trimming=60, compile=False).eval()
    sd = {k: v.clone() for k, v in model.state_dict().items()}
    model = model.to("cuda")
    Ls = 400
    bases = torch.randint(0, 4, (3, Ls), generator=torch.Generator().manual_seed(5))
    X = O.one_hot(bases)
    wrapper = cb.ProfileWrapper(cb.ControlWrapper(model))
    y_ref, y_mut = A.saturation_mutagenesis(wrapper, X, device="cuda", start=190, end=210,
                                            raw_outputs=True)
    delta = O.ism_wrapper_deltas(sd, model._init_kwargs(), bases, 190, 210, "profile")
    with torch.no_grad():
        p, _ = O.forward(sd, model._init_kwargs(), X, O.control_inputs(model._init_kwargs(), X))
    yr = O.profile_wrapper(p)
    assert (y_ref - yr).abs().max().item() <= 1e-4
    assert (y_mut - (yr[:, :, None] + delta)).abs().max().item() <= 1e-4
