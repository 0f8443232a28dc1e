"""The CPU oracle against golden vectors produced by the upstream package.

These pin the oracle before it is trusted as the checker for the CUDA
engine. Fixtures: tests/golden/make_golden.py.
"""

import torch

from oracle import cherimoya_oracle as O


def _inputs(case):
    X = case["X"]
    if X is None:
        X = O.one_hot(case["bases"])
    return X, case.get("X_ctl")


def test_conv_norm_matches_upstream(golden):
    for c in golden("conv_norm")["cases"]:
        y = O.conv_norm(c["x"], c["w"], c["dilation"])
        assert y.dtype == c["x"].dtype
        assert torch.allclose(y, c["y"], atol=1e-5, rtol=0), (y - c["y"]).abs().max()


def test_conv_norm_zero_mean_unit_var():
    # mirrors upstream tests/test_cheri.py:33-46
    g = torch.Generator().manual_seed(0)
    x = torch.randn(4, 128, 16, generator=g)
    w = torch.randn(3, 16, generator=g)
    y = O.conv_norm(x, w, 4).reshape(4, -1)
    assert torch.allclose(y.mean(1), torch.zeros(4), atol=1e-4)
    assert torch.allclose(y.var(1, unbiased=False), torch.ones(4), atol=2e-3)


def test_conv_taps_manual():
    # mirrors upstream tests/test_cheri.py:49-73 (explicit loop reference)
    g = torch.Generator().manual_seed(0)
    x = torch.randn(1, 10, 2, generator=g)
    w = torch.randn(3, 2, generator=g) * 0.1
    d = 3
    y = O.dilated_depthwise_conv(x, w, d)
    for c in range(2):
        for i in range(10):
            v = w[1, c] * x[0, i, c]
            if i - d >= 0:
                v = v + w[0, c] * x[0, i - d, c]
            if i + d < 10:
                v = v + w[2, c] * x[0, i + d, c]
            assert abs(float(v - y[0, i, c])) < 1e-6


def test_dilation_longer_than_sequence():
    x = torch.randn(2, 5, 3)
    w = torch.randn(3, 3)
    y = O.dilated_depthwise_conv(x, w, 8)
    assert torch.allclose(y, x * w[1])


def test_cheri_block_matches_upstream(golden):
    for c in golden("cheri_block")["cases"]:
        sd = c["state_dict"]
        assert list(sd.keys()) == ["conv_weight", "linear1.weight", "linear2.weight"]
        y = O.cheri_block(c["x"], sd["conv_weight"], sd["linear1.weight"],
                          sd["linear2.weight"], c["dilation"], c["residual_scale"])
        assert torch.allclose(y, c["y"], atol=2e-5, rtol=0), (y - c["y"]).abs().max()


def _check_model(case, atol):
    X, X_ctl = _inputs(case)
    p, lc = O.forward(case["state_dict"], case["config"], X, X_ctl)
    out = case["outputs"]
    assert p.shape == out["profile"].shape and lc.shape == out["logcounts"].shape
    assert (p - out["profile"]).abs().max() < atol
    assert (lc - out["logcounts"]).abs().max() < atol
    return X, X_ctl, p, lc


def test_model_forward_matches_upstream(golden):
    for name in ["model_default_L2114", "model_small_float_input", "model_multitask",
                 "model_control_tracks", "model_wide_c256"]:
        _check_model(golden(name), atol=2e-5)


def test_state_dict_layout(golden):
    case = golden("model_default_L2114")
    keys = case["state_dict_keys"]
    assert keys[:4] == ["lw0", "lw1", "iconv.weight", "iconv.bias"]
    assert keys[4:7] == ["blocks.0.conv_weight", "blocks.0.linear1.weight",
                         "blocks.0.linear2.weight"]
    assert keys[-4:] == ["fconv.weight", "fconv.bias", "linear.weight", "linear.bias"]


def test_wrappers_match_upstream(golden):
    for name in ["model_default_L2114", "model_multitask", "model_control_tracks"]:
        case = golden(name)
        X, X_ctl, _, _ = _check_model(case, atol=2e-5)
        cfg, sd, out = case["config"], case["state_dict"], case["outputs"]
        ctl0 = O.control_inputs(cfg, X)
        p0, c0 = O.forward(sd, cfg, X, ctl0)
        assert torch.allclose(p0, out["wrap_control"], atol=2e-5)
        assert torch.allclose(O.profile_wrapper(p0), out["wrap_profile"], atol=2e-5)
        assert torch.allclose(c0, out["wrap_logcount"], atol=2e-5)
        pe, ce = O.forward(sd, cfg, X, X_ctl)
        ec = O.expected_counts(pe, ce, cfg["signal_groups"])
        assert torch.allclose(ec, out["wrap_expected"], atol=1e-6, rtol=1e-4)


def test_metrics_match_upstream(golden):
    m = golden("metrics")
    assert torch.allclose(O.jensen_shannon_distance(m["logps"], m["counts"]), m["jsd"],
                          atol=1e-6)
    assert torch.allclose(O.pearson_corr(m["logps"], m["counts"]), m["pearson"], atol=1e-6)


def test_ism_matches_upstream(golden):
    case = golden("ism_small")
    dlc, jsd, _, _ = O.ism_scores(case["state_dict"], case["config"], case["bases"],
                                  case["start"], case["end"])
    assert torch.allclose(dlc, case["d_logcount"], atol=1e-6)
    assert torch.allclose(jsd, case["jsd"], atol=1e-7)
    # reference-base rows re-score the reference: zero up to batch-size rounding
    ref = case["bases"][:, case["start"]:case["end"]].long()
    assert dlc.gather(1, ref.unsqueeze(1)).abs().max() < 1e-8


def test_bf16_autocast_golden_is_close_to_fp32(golden):
    """The upstream bf16 mode (CPU autocast) stays within the bf16 tolerance
    of the fp32 path: the bar the bf16 engine is held to."""
    out = golden("model_default_L2114")["outputs"]
    assert (out["profile_bf16_autocast"] - out["profile"]).abs().max() < 1e-2
    assert (out["logcounts_bf16_autocast"] - out["logcounts"]).abs().max() < 1e-2
