"""Parity of the sm_100a engine with the upstream implementation.

Every test here runs the CUDA path through the C-ABI library
(libcherimoya_b200.so) and compares it with the golden vectors produced by
the upstream package (tests/golden) or with the CPU oracle on the same
seeded inputs and the same state_dict.

Tolerances:
  fp32 mode: max abs error <= 1e-4 on profile logits and log-counts
  bf16 mode: max abs error <= 1e-2 and per-track profile Pearson >= 0.9999
"""

import pytest
import torch

import cherimoya_b200 as cb
from oracle import cherimoya_oracle as O

pytestmark = pytest.mark.gpu

DEV = "cuda"
FP32_TOL = 1e-4
BF16_TOL = 1e-2
BF16_PEARSON = 0.9999


def _inputs(case):
    X = case["X"]
    if X is None:
        X = O.one_hot(case["bases"])
    return X, case.get("X_ctl")


def _model(case, precision="auto", device=DEV):
    m = cb.Cherimoya(**case["config"], compile=False, precision=precision)
    m.load_state_dict(case["state_dict"])
    return m.eval().to(device)


def _run(m, X, X_ctl=None):
    with torch.no_grad():
        p, c = m(X.to(DEV), None if X_ctl is None else X_ctl.to(DEV))
    torch.cuda.synchronize()
    return p.cpu(), c.cpu()


def _pearson_min(a, b):
    a = a.reshape(-1, a.shape[-1]).double()
    b = b.reshape(-1, b.shape[-1]).double()
    return float(O.pearson_corr(a, b).min())


GOLDEN_MODELS = ["model_default_L2114", "model_small_float_input", "model_multitask",
                 "model_control_tracks"]


@pytest.mark.parametrize("name", GOLDEN_MODELS)
def test_forward_fp32_matches_upstream(golden, name):
    case = golden(name)
    m = _model(case, "fp32")
    X, X_ctl = _inputs(case)
    p, c = _run(m, X, X_ctl)
    out = case["outputs"]
    assert p.shape == out["profile"].shape and c.shape == out["logcounts"].shape
    ep = (p - out["profile"]).abs().max().item()
    ec = (c - out["logcounts"]).abs().max().item()
    print(name, "fp32 max|dprofile| %.3e max|dlogcount| %.3e" % (ep, ec))
    assert ep <= FP32_TOL and ec <= FP32_TOL


@pytest.mark.parametrize("name", ["model_default_L2114", "model_small_float_input"])
def test_forward_bf16_matches_upstream(golden, name):
    case = golden(name)
    m = _model(case, "bf16")
    X, X_ctl = _inputs(case)
    p, c = _run(m, X, X_ctl)
    out = case["outputs"]
    for ref_p, ref_c in [(out["profile"], out["logcounts"]),
                         (out["profile_bf16_autocast"], out["logcounts_bf16_autocast"])]:
        ep = (p - ref_p).abs().max().item()
        ec = (c - ref_c).abs().max().item()
        r = _pearson_min(p, ref_p)
        print(name, "bf16 max|dprofile| %.3e max|dlogcount| %.3e pearson %.6f" % (ep, ec, r))
        assert ep <= BF16_TOL and ec <= BF16_TOL and r >= BF16_PEARSON


def test_bf16_input_selects_bf16_mode(golden):
    case = golden("model_default_L2114")
    m = _model(case)
    X, _ = _inputs(case)
    p16, c16 = _run(m, X.to(torch.bfloat16))
    m.precision = "bf16"
    pb, cb_ = _run(m, X)
    assert torch.equal(p16, pb) and torch.equal(c16, cb_)


@pytest.mark.parametrize("mode", ["fp32", "bf16"])
def test_full_size_batch64_against_oracle(golden, mode):
    """Default model, 64 uniform random one-hot 2114-bp sequences (the
    upstream CPU-benchmark shape), engine vs the oracle."""
    case = golden("model_default_L2114")
    g = torch.Generator().manual_seed(1)
    X = O.one_hot(torch.randint(0, 4, (64, 2114), generator=g))
    with torch.no_grad():
        rp, rc = O.forward(case["state_dict"], case["config"], X)
    m = _model(case, mode)
    p, c = _run(m, X)
    ep, ec = (p - rp).abs().max().item(), (c - rc).abs().max().item()
    r = _pearson_min(p, rp)
    print(mode, "batch64 max|dprofile| %.3e max|dlogcount| %.3e pearson %.7f" % (ep, ec, r))
    if mode == "fp32":
        assert ep <= FP32_TOL and ec <= FP32_TOL
    else:
        assert ep <= BF16_TOL and ec <= BF16_TOL and r >= BF16_PEARSON


def test_forward_bases_equals_onehot_forward(golden):
    case = golden("model_default_L2114")
    m = _model(case, "bf16")
    bases = case["bases"]
    p1, c1 = _run(m, O.one_hot(bases))
    with torch.no_grad():
        p2, c2 = m.forward_bases(bases.to(DEV), precision="bf16")
    assert torch.equal(p1, p2.cpu()) and torch.equal(c1, c2.cpu())


@pytest.mark.parametrize("mode", ["fp32", "bf16"])
def test_deterministic_and_batch_invariant(golden, mode):
    """Repeated calls are bitwise equal (upstream tests/test_model.py:739-759)
    and a sequence's output does not depend on the rest of its batch."""
    case = golden("model_default_L2114")
    m = _model(case, mode)
    g = torch.Generator().manual_seed(7)
    X = O.one_hot(torch.randint(0, 4, (5, 2114), generator=g))
    p1, c1 = _run(m, X)
    p2, c2 = _run(m, X)
    assert torch.equal(p1, p2) and torch.equal(c1, c2)
    p3, c3 = _run(m, X[2:3])
    assert torch.equal(p3, p1[2:3]) and torch.equal(c3, c1[2:3])


@pytest.mark.parametrize("mode", ["fp32", "bf16"])
@pytest.mark.parametrize("dil", [1, 64, 256])
def test_block_repeatable_over_many_tiles(mode, dil):
    """Several 128-row tiles per CTA (64 x 2114 rows = 1057 tiles): the
    pipelined kernel's buffer reuse is exercised; repeated calls must be
    bitwise equal and match the oracle."""
    torch.manual_seed(dil)
    blk = cb.CheriBlock(128, dil).eval()
    sd = {k: v.clone() for k, v in blk.state_dict().items()}
    x = torch.randn(64, 2114, 128) * 0.3
    ref = O.cheri_block(x, sd["conv_weight"], sd["linear1.weight"], sd["linear2.weight"], dil,
                        0.15)
    blk = blk.to(DEV)
    dt = torch.float32 if mode == "fp32" else torch.bfloat16
    with torch.no_grad():
        outs = [blk(x.to(DEV, dt)).float().cpu() for _ in range(3)]
    assert all(torch.equal(outs[0], o) for o in outs[1:])
    err = (outs[0] - ref).abs().max().item()
    assert err <= (FP32_TOL if mode == "fp32" else 3e-2), err


@pytest.mark.parametrize("idx", [0, 1, 2])
def test_block_engine_matches_upstream(golden, idx):
    c = golden("cheri_block")["cases"][idx]
    blk = cb.CheriBlock(c["n_filters"], c["dilation"], c["expansion"], c["residual_scale"])
    blk.load_state_dict(c["state_dict"])
    blk = blk.eval().to(DEV)
    with torch.no_grad():
        y = blk(c["x"].to(DEV)).cpu()
    e = (y - c["y"]).abs().max().item()
    print("block", idx, "fp32 max|dy| %.3e" % e)
    assert e <= FP32_TOL
    with torch.no_grad():
        y16 = blk(c["x"].to(DEV, torch.bfloat16)).float().cpu()
    e16 = (y16 - c["y"]).abs().max().item()
    print("block", idx, "bf16 max|dy| %.3e" % e16)
    assert e16 <= 5e-2  # bf16 storage of unit-scale activations (upstream test_cheri.py:535-559)


def test_block_zero_mlp_is_exact_identity():
    """Zero linear2 -> the block returns its input bit for bit (upstream
    tests/test_cheri.py:590-608)."""
    torch.manual_seed(0)
    blk = cb.CheriBlock(128, 8).eval().to(DEV)
    with torch.no_grad():
        blk.linear2.weight.zero_()
        x = torch.randn(2, 300, 128, device=DEV)
        y = blk(x)
    assert torch.equal(x, y)


def test_in_place_update_invalidates_packed_weights(golden):
    """Weights changed in place after the first call are seen by the next
    (upstream tests/test_cheri.py:303-356, 904-930)."""
    case = golden("model_small_float_input")
    m = _model(case, "fp32")
    X, _ = _inputs(case)
    p1, _ = _run(m, X)
    with torch.no_grad():
        m.blocks[1].linear1.weight.mul_(3.0)
        m.fconv.bias.add_(0.5)
    p2, c2 = _run(m, X)
    sd = {k: v.cpu() for k, v in m.state_dict().items()}
    with torch.no_grad():
        rp, rc = O.forward(sd, case["config"], X)
    assert not torch.equal(p1, p2)
    assert (p2 - rp).abs().max() <= FP32_TOL and (c2 - rc).abs().max() <= FP32_TOL


@pytest.mark.parametrize("N,L,T", [(1, 300, 53), (3, 300, 53), (2, 129, 60), (7, 2114, 557),
                                   (1, 2114, 0), (4, 1000, 37)])
def test_edge_shapes_against_oracle(N, L, T):
    """Ragged batches (rows not a multiple of the 128-row tile), a single
    example, short sequences, trimming 0 and windows touching the padding."""
    torch.manual_seed(11)
    m = cb.Cherimoya(n_filters=128, n_layers=9 if L >= 1000 else 3, trimming=T,
                     compile=False, precision="fp32").eval()
    sd = {k: v.clone() for k, v in m.state_dict().items()}
    g = torch.Generator().manual_seed(12)
    X = O.one_hot(torch.randint(0, 4, (N, L), generator=g))
    with torch.no_grad():
        rp, rc = O.forward(sd, m._init_kwargs(), X)
    p, c = _run(m.to(DEV), X)
    assert (p - rp).abs().max() <= FP32_TOL and (c - rc).abs().max() <= FP32_TOL


def test_empty_batch_and_wrong_channels():
    m = cb.Cherimoya(n_filters=32, n_layers=2, compile=False).eval().to(DEV)
    with torch.no_grad():
        p, c = m(torch.zeros(0, 4, 300, device=DEV))
        assert p.shape == (0, 1, 300 - 2 * m.trimming) and c.shape == (0, 1)
        with pytest.raises(RuntimeError):
            m(torch.zeros(2, 5, 300, device=DEV))


def test_ism_matches_upstream(golden):
    case = golden("ism_small")
    m = _model(case, "fp32")
    bases = case["bases"].to(DEV)
    dlc, jsd = cb.saturation_mutagenesis(m, bases, case["start"], case["end"], mutant_batch=97)
    torch.cuda.synchronize()
    dlc, jsd = dlc[:, 0].cpu(), jsd.cpu()
    e1 = (dlc - case["d_logcount"]).abs().max().item()
    e2 = (jsd - case["jsd"]).abs().max().item()
    print("ism max|d dlogcount| %.3e max|d jsd| %.3e" % (e1, e2))
    assert e1 <= 2e-6 and e2 <= 2e-6
    # rank order of the four bases at every position
    ref_rank = case["d_logcount"].argsort(dim=1)
    got_rank = dlc.argsort(dim=1)
    agree = (ref_rank == got_rank).all(dim=1).float().mean().item()
    print("ism rank-order agreement %.4f" % agree)
    assert agree == 1.0


def test_ism_full_length_properties(golden):
    """Default model at 2114 bp: reference-base entries are 0, a mutant's
    score equals the forward of the explicitly mutated sequence."""
    case = golden("model_default_L2114")
    m = _model(case, "fp32")
    bases = case["bases"][:1].to(DEV)
    dlc, jsd = cb.saturation_mutagenesis(m, bases, 1000, 1010)
    ref = bases[0, 1000:1010].long().cpu()
    d0 = dlc[0, 0].cpu()
    assert torch.all(d0.gather(0, ref.unsqueeze(0)) == 0)
    # explicit check of one mutant through the plain forward
    alt = (int(ref[3]) + 2) % 4
    mut = bases.clone()
    mut[0, 1003] = alt
    with torch.no_grad():
        _, c_ref = m.forward_bases(bases, precision="fp32")
        _, c_mut = m.forward_bases(mut, precision="fp32")
    assert abs(float(c_mut[0, 0] - c_ref[0, 0]) - float(d0[alt, 3])) < 1e-7


def test_variant_effect_matches_oracle(golden):
    case = golden("model_small_float_input")
    cfg = dict(case["config"])
    torch.manual_seed(5)
    m = cb.Cherimoya(**cfg, compile=False, precision="fp32").eval()
    sd = {k: v.clone() for k, v in m.state_dict().items()}
    g = torch.Generator().manual_seed(6)
    ref = torch.randint(0, 4, (37, 300), generator=g)
    alt = ref.clone()
    alt[:, 150] = (alt[:, 150] + torch.randint(1, 4, (37,), generator=g)) % 4
    rd, rj = O.variant_scores(sd, m._init_kwargs(), ref, alt)
    m = m.to(DEV)
    d, j = cb.variant_effect(m, ref.to(DEV), alt.to(DEV))
    assert (d.cpu() - rd).abs().max() <= 2e-6
    assert (j.cpu() - rj).abs().max() <= 2e-6


def test_forward_captures_in_cuda_graph(golden):
    """The engine forward has no host synchronisation or allocation of its
    own, so a whole model call records into a CUDA graph; replays with new
    input contents give the eager results."""
    case = golden("model_default_L2114")
    m = _model(case, "bf16")
    X = O.one_hot(case["bases"]).to(DEV)
    Xs = X.clone()
    with torch.no_grad():
        ref_p, ref_c = m(X)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(2):
                m(Xs)                                   # warm-up on the side stream
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            gp, gc = m(Xs)
        Xs.copy_(X.flip(0))
        g.replay()
        torch.cuda.synchronize()
        fp, fc = m(X.flip(0))
        assert torch.equal(gp, fp) and torch.equal(gc, fc)
        Xs.copy_(X)
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(gp, ref_p) and torch.equal(gc, ref_c)


@pytest.mark.parametrize("mode", ["fp32", "bf16"])
def test_hidden_width_not_a_multiple_of_16(mode):
    """Hidden widths the kernels pad (upstream tests/test_cheri.py:358-372,
    611-629: H % 16 != 0 must still work): n_filters 24, expansion 1."""
    torch.manual_seed(5)
    m = cb.Cherimoya(n_filters=24, expansion=1, n_layers=4, trimming=80, compile=False,
                     precision=mode).eval()
    sd = {k: v.clone() for k, v in m.state_dict().items()}
    X = O.one_hot(torch.randint(0, 4, (3, 500), generator=torch.Generator().manual_seed(6)))
    with torch.no_grad():
        rp, rc = O.forward(sd, m._init_kwargs(), X)
    p, c = _run(m.to(DEV), X)
    tol = FP32_TOL if mode == "fp32" else BF16_TOL
    assert (p - rp).abs().max() <= tol and (c - rc).abs().max() <= tol


def test_engine_matches_grad_path_on_cuda(golden):
    """CUDA no_grad (the engine) against CUDA with gradients enabled (the
    differentiable PyTorch ops) on the same model (upstream
    tests/test_model.py:583-631: fp32 within 1e-4)."""
    case = golden("model_default_L2114")
    m = _model(case, "fp32")
    X = O.one_hot(case["bases"]).to(DEV)
    with torch.no_grad():
        p0, c0 = m(X)
    # the grad path's convolutions in plain fp32 (cuDNN would otherwise use TF32)
    tf32 = torch.backends.cudnn.allow_tf32
    torch.backends.cudnn.allow_tf32 = False
    try:
        p1, c1 = m(X.clone().requires_grad_(True))
    finally:
        torch.backends.cudnn.allow_tf32 = tf32
    assert p1.requires_grad
    assert (p0 - p1.detach()).abs().max().item() <= FP32_TOL
    assert (c0 - c1.detach()).abs().max().item() <= FP32_TOL


def test_block_hooks_bypassed_by_the_engine():
    """Forward hooks on the blocks fire on the PyTorch path and not when the
    engine runs the whole model (the documented upstream asymmetry,
    tests/test_cheri.py:734-761)."""
    m = cb.Cherimoya(n_filters=32, n_layers=2, compile=False, precision="fp32").eval().to(DEV)
    calls = []
    h = m.blocks[0].register_forward_hook(lambda mod, inp, out: calls.append(1))
    X = torch.zeros(1, 4, 300, device=DEV)
    X[:, 0] = 1.0
    with torch.no_grad():
        m(X)
    assert calls == []
    m(X.requires_grad_(True))
    assert calls == [1]
    h.remove()
