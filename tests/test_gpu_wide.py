"""Wide models on the sm_100a engine: C = 256 (and any H > 256) run the
streamed-weight MLP kernel, whose W1 / W2 chunks move through shared memory
one 64-unit hidden chunk at a time.

Cases:
  * the upstream-produced golden model with n_filters 256 (2 layers);
  * the variant-scoring configuration: 12 layers, n_filters 256, expansion 2,
    trimming 557, full 2114-bp inputs, forward and ref/alt scoring vs the
    oracle on the same state_dict;
  * a default-width model with expansion 3 (H = 384), which also takes the
    streamed kernel.

Tolerances as in test_gpu_parity: fp32 1e-4 max abs; bf16 1e-2 max abs and
per-track profile Pearson >= 0.9999.
"""

import pytest
import torch

import cherimoya_b200 as cb
from oracle import cherimoya_oracle as O

pytestmark = pytest.mark.gpu

FP32_TOL = 1e-4
BF16_TOL = 1e-2
BF16_PEARSON = 0.9999


def _pearson_min(a, b):
    a = a.reshape(-1, a.shape[-1]).double()
    b = b.reshape(-1, b.shape[-1]).double()
    return float(O.pearson_corr(a, b).min())


def _check(mode, p, c, rp, rc, label):
    ep, ec = (p - rp).abs().max().item(), (c - rc).abs().max().item()
    r = _pearson_min(p, rp)
    print(label, mode, "max|dprofile| %.3e max|dlogcount| %.3e pearson %.7f" % (ep, ec, r))
    if mode == "fp32":
        assert ep <= FP32_TOL and ec <= FP32_TOL
    else:
        assert ep <= BF16_TOL and ec <= BF16_TOL and r >= BF16_PEARSON


def _engine(model, X):
    with torch.no_grad():
        p, c = model(X.cuda())
    torch.cuda.synchronize()
    return p.cpu(), c.cpu()


@pytest.mark.parametrize("mode", ["fp32", "bf16"])
def test_wide_c256_matches_upstream(golden, mode):
    case = golden("model_wide_c256")
    m = cb.Cherimoya(**case["config"], compile=False, precision=mode)
    m.load_state_dict(case["state_dict"])
    m = m.eval().cuda()
    X = O.one_hot(case["bases"])
    p, c = _engine(m, X)
    out = case["outputs"]
    assert p.shape == out["profile"].shape and c.shape == out["logcounts"].shape
    _check(mode, p, c, out["profile"], out["logcounts"], "c256 golden")


def _variant_model():
    torch.manual_seed(0)
    return cb.Cherimoya(n_filters=256, n_layers=12, trimming=557, compile=False).eval()


@pytest.mark.parametrize("mode", ["fp32", "bf16"])
def test_variant_config_forward_against_oracle(mode):
    m = _variant_model()
    sd = {k: v.float() for k, v in m.state_dict().items()}
    cfg = {"n_layers": 12, "residual_scale": 0.15, "trimming": 557}
    g = torch.Generator().manual_seed(3)
    X = O.one_hot(torch.randint(0, 4, (2, 2114), generator=g))
    with torch.no_grad():
        rp, rc = O.forward(sd, cfg, X)
    m.precision = mode
    p, c = _engine(m.cuda(), X)
    _check(mode, p, c, rp, rc, "12-layer c256")


def test_variant_config_scores_against_oracle():
    m = _variant_model()
    sd = {k: v.float() for k, v in m.state_dict().items()}
    cfg = {"n_layers": 12, "residual_scale": 0.15, "trimming": 557}
    g = torch.Generator().manual_seed(4)
    ref = torch.randint(0, 4, (3, 2114), generator=g)
    alt = ref.clone()
    alt[:, 1057] = (ref[:, 1057] + 1 + torch.randint(0, 3, (3,), generator=g)) % 4
    rd, rj = O.variant_scores(sd, cfg, ref, alt)
    m.precision = "fp32"
    m = m.cuda()
    d, j = cb.variant_effect(m, O.one_hot(ref).cuda(), O.one_hot(alt).cuda())
    torch.cuda.synchronize()
    assert (d.cpu() - rd).abs().max().item() <= FP32_TOL
    assert (j.cpu() - rj).abs().max().item() <= FP32_TOL


@pytest.mark.parametrize("mode", ["fp32", "bf16"])
def test_expansion3_streamed_mlp_against_oracle(mode):
    torch.manual_seed(5)
    m = cb.Cherimoya(n_filters=128, n_layers=3, expansion=3, trimming=200,
                     compile=False).eval()
    sd = {k: v.float() for k, v in m.state_dict().items()}
    cfg = {"n_layers": 3, "residual_scale": 0.15, "trimming": 200}
    g = torch.Generator().manual_seed(6)
    X = O.one_hot(torch.randint(0, 4, (3, 1000), generator=g))
    with torch.no_grad():
        rp, rc = O.forward(sd, cfg, X)
    m.precision = mode
    p, c = _engine(m.cuda(), X)
    _check(mode, p, c, rp, rc, "expansion 3")


@pytest.mark.parametrize("mode", ["fp32", "bf16"])
@pytest.mark.parametrize("n_filters,expansion", [(256, 1), (200, 2)])
def test_wide_widths_against_oracle(mode, n_filters, expansion):
    """n_filters 256 with expansion 1 (four hidden chunks in the streamed-weight
    kernel) and n_filters 200 (padded to 256 channels: the padded channels must
    stay zero through the stem halves, the MLP and the 256-wide head)."""
    torch.manual_seed(7)
    m = cb.Cherimoya(n_filters=n_filters, n_layers=3, expansion=expansion, trimming=300,
                     compile=False).eval()
    sd = {k: v.float() for k, v in m.state_dict().items()}
    cfg = {"n_layers": 3, "residual_scale": 0.15, "trimming": 300}
    g = torch.Generator().manual_seed(8)
    X = O.one_hot(torch.randint(0, 4, (3, 1300), generator=g))
    with torch.no_grad():
        rp, rc = O.forward(sd, cfg, X)
    m.precision = mode
    p, c = _engine(m.cuda(), X)
    _check(mode, p, c, rp, rc, "n_filters %d expansion %d" % (n_filters, expansion))
