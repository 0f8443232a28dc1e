"""Drop-in surface of the engine package on CPU: constructor, init order,
state_dict layout, checkpoint payload, CPU forward semantics, wrappers.
Mirrors upstream tests/test_model.py and tests/test_cheri.py checkpoint
and semantics tests."""

import torch

import cherimoya_b200 as cb
from oracle import cherimoya_oracle as O


def _inputs(case):
    X = case["X"]
    if X is None:
        X = O.one_hot(case["bases"])
    return X, case.get("X_ctl")


def _model(case):
    m = cb.Cherimoya(**case["config"], compile=False)
    m.load_state_dict(case["state_dict"])
    return m.eval()


def test_state_dict_keys_and_order_match_upstream(golden):
    for name in ["model_default_L2114", "model_multitask", "model_control_tracks"]:
        case = golden(name)
        m = cb.Cherimoya(**case["config"])
        assert list(m.state_dict().keys()) == case["state_dict_keys"]


def test_seeded_init_matches_upstream(golden):
    """Same constructor RNG draw order as upstream (cherimoya.py:173-197,
    cheri.py:932-939): a seed gives the upstream weights."""
    case = golden("model_default_L2114")
    torch.manual_seed(0)
    m = cb.Cherimoya(**case["config"])
    for k, v in m.state_dict().items():
        assert torch.equal(v, case["state_dict"][k]), k


def test_cpu_forward_matches_upstream(golden):
    for name in ["model_default_L2114", "model_small_float_input", "model_multitask",
                 "model_control_tracks", "model_wide_c256"]:
        case = golden(name)
        m = _model(case)
        X, X_ctl = _inputs(case)
        with torch.no_grad():
            p, c = m(X, X_ctl)
        assert (p - case["outputs"]["profile"]).abs().max() < 2e-5
        assert (c - case["outputs"]["logcounts"]).abs().max() < 2e-5


def test_block_cpu_matches_upstream(golden):
    for c in golden("cheri_block")["cases"]:
        blk = cb.CheriBlock(c["n_filters"], c["dilation"], c["expansion"], c["residual_scale"])
        blk.load_state_dict(c["state_dict"])
        assert list(blk.state_dict().keys()) == c["state_dict_keys"]
        with torch.no_grad():
            y = blk(c["x"])
        assert (y - c["y"]).abs().max() < 2e-5


def test_legacy_and_new_conv_keys_load():
    blk = cb.CheriBlock(8, 2)
    sd = blk.state_dict()
    assert "conv_weight" in sd and "conv.conv_weight" not in sd
    sd2 = {("conv.conv_weight" if k == "conv_weight" else k): v for k, v in sd.items()}
    blk2 = cb.CheriBlock(8, 2)
    blk2.load_state_dict(sd2)
    assert torch.equal(blk2.conv_weight, blk.conv_weight)
    assert blk2.conv_weight is blk2.conv.conv_weight


def test_save_load_roundtrip(tmp_path):
    torch.manual_seed(3)
    m = cb.Cherimoya(n_filters=16, n_layers=3, signal_groups=[1, 2], compile=False)
    path = str(tmp_path / "m.torch")
    m.save(path)
    payload = torch.load(path, weights_only=True)
    assert set(payload) == {"config", "state_dict"}
    assert payload["config"]["signal_groups"] == [1, 2]
    m2 = cb.Cherimoya.load(path, compile=False)
    for (k, a), (k2, b) in zip(m.state_dict().items(), m2.state_dict().items()):
        assert k == k2 and torch.equal(a, b)
    X = O.one_hot(torch.randint(0, 4, (2, 200)))
    with torch.no_grad():
        a, b = m(X), m2(X)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])


def test_signal_group_validation():
    import pytest
    for bad in ([], [0], [1, -2], "1", [True]):
        with pytest.raises(ValueError):
            cb.Cherimoya(signal_groups=bad)


def test_wrappers_cpu_match_upstream(golden):
    for name in ["model_default_L2114", "model_multitask", "model_control_tracks"]:
        case = golden(name)
        m = _model(case)
        X, X_ctl = _inputs(case)
        out = case["outputs"]
        with torch.no_grad():
            assert torch.allclose(cb.ControlWrapper(m)(X)[0], out["wrap_control"], atol=2e-5)
            assert torch.allclose(cb.ProfileWrapper(cb.ControlWrapper(m))(X), out["wrap_profile"],
                                  atol=2e-5)
            assert torch.allclose(cb.LogCountWrapper(cb.ControlWrapper(m))(X),
                                  out["wrap_logcount"], atol=2e-5)
            assert torch.allclose(cb.ExpectedCountsWrapper(m)(X, X_ctl), out["wrap_expected"],
                                  atol=1e-6, rtol=1e-4)


def test_wrong_channel_count_raises_runtime_error():
    import pytest
    m = cb.Cherimoya(n_filters=16, n_layers=2)
    with pytest.raises(RuntimeError):
        with torch.no_grad():
            m(torch.zeros(1, 5, 200))


def test_grad_path_is_differentiable():
    m = cb.Cherimoya(n_filters=16, n_layers=2)
    X = O.one_hot(torch.randint(0, 4, (2, 200))).requires_grad_(True)
    p, c = m(X)
    (p.sum() + c.sum()).backward()
    assert X.grad is not None and torch.isfinite(X.grad).all()


def test_metrics_match_upstream(golden):
    from cherimoya_b200 import performance as P
    mt = golden("metrics")
    assert torch.allclose(P.jensen_shannon_distance(mt["logps"], mt["counts"]), mt["jsd"],
                          atol=1e-6)
    assert torch.allclose(P.pearson_corr(mt["logps"], mt["counts"]), mt["pearson"], atol=1e-6)


def test_to_bases_and_shard_ranges():
    from cherimoya_b200.ism import shard_range, to_bases
    b = torch.randint(0, 4, (3, 50))
    X = O.one_hot(b)
    X[1, :, 7] = 0
    got = to_bases(X)
    exp = b.to(torch.int8).clone()
    exp[1, 7] = 4
    assert torch.equal(got, exp)
    for n in (0, 1, 7, 256, 1000):
        for world in (1, 2, 3, 8):
            spans = [shard_range(n, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
            sizes = [hi - lo for lo, hi in spans]
            assert max(sizes) - min(sizes) <= 1


def test_conv_norm_output_is_zero_mean_unit_variance():
    """Per-example LayerNorm over the (L, C) plane (upstream tests/test_cheri.py:33-46):
    mean 0 and biased variance var / (var + eps) ~ 1 for each example."""
    g = torch.Generator().manual_seed(4)
    x = torch.randn(3, 257, 24, generator=g) * 3.0 + 1.5
    w = torch.randn(3, 24, generator=g)
    y = cb.fused_dilated_conv_norm(x, w, 5)
    flat = y.reshape(3, -1)
    assert flat.mean(dim=1).abs().max().item() <= 1e-4
    assert (flat.var(dim=1, unbiased=False) - 1.0).abs().max().item() <= 2e-3
