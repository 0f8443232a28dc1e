"""Generate golden input/output vectors from the upstream Cherimoya package.

Run from the repository root on a machine with an upstream copy, named by
$CHERIMOYA_REFERENCE (a checkout) or installed into baseline/_ref (see
oracle/upstream.py):

    CHERIMOYA_REFERENCE=<upstream checkout> python tests/golden/make_golden.py

Each case is a ``.pt`` file holding the model config, its fp32 state_dict,
the inputs and the outputs of the upstream CPU path (eager, ``no_grad``).
The parity tests load the state_dict into both the oracle and the CUDA
engine, so they do not depend on torch's RNG reproducing the weights.

Upstream code exercised (paths relative to the upstream project):
  cherimoya/cheri.py:52-98       _cheri_conv_norm_cpu
  cherimoya/cheri.py:1072-1082   CheriBlock.forward (CPU branch)
  cherimoya/cherimoya.py:340-400 Cherimoya._forward_impl
  cherimoya/wrappers.py:11-166   ControlWrapper / ProfileWrapper /
                                 LogCountWrapper / ExpectedCountsWrapper
  cherimoya/performance.py:138-246  _kl_divergence, jensen_shannon_distance,
                                 pearson_corr
"""

import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle.upstream import import_upstream  # noqa: E402


def one_hot(idx):
    """(N, L) int64 base indices -> (N, 4, L) fp32 one-hot (A, C, G, T)."""
    return torch.nn.functional.one_hot(idx, 4).permute(0, 2, 1).float().contiguous()


def save(name, payload):
    path = os.path.join(HERE, name + ".pt")
    torch.save(payload, path)
    print("wrote", path, os.path.getsize(path), "bytes")


def model_case(ref, name, config, N, L, seed, input_kind="onehot",
               ctl=False, autocast=False, wrappers=False):
    torch.manual_seed(seed)
    model = ref.Cherimoya(**config, verbose=False, compile=False).eval()
    g = torch.Generator().manual_seed(seed + 1)
    if input_kind == "onehot":
        idx = torch.randint(0, 4, (N, L), generator=g)
        X = one_hot(idx)
    else:
        idx = None
        X = torch.randn(N, 4, L, generator=g)
    X_ctl = None
    if ctl:
        X_ctl = torch.rand(N, config["n_control_tracks"], L, generator=g) * 3.0
    with torch.no_grad():
        prof, lc = model(X, X_ctl)
        out = {"profile": prof.clone(), "logcounts": lc.clone()}
        if autocast:
            with torch.autocast("cpu", dtype=torch.bfloat16):
                p16, c16 = model(X, X_ctl)
            out["profile_bf16_autocast"] = p16.float().clone()
            out["logcounts_bf16_autocast"] = c16.float().clone()
        if wrappers:
            W = ref.wrappers
            inner = W.ControlWrapper(model)
            out["wrap_control"] = inner(X)[0].clone()
            out["wrap_profile"] = W.ProfileWrapper(inner)(X).clone()
            out["wrap_logcount"] = W.LogCountWrapper(inner)(X).clone()
            out["wrap_expected"] = W.ExpectedCountsWrapper(model)(X, X_ctl).clone()
    payload = {
        "config": model._init_kwargs(),
        "state_dict": {k: v.clone() for k, v in model.state_dict().items()},
        "state_dict_keys": list(model.state_dict().keys()),
        "X": X if idx is None else None,
        "bases": idx.to(torch.int8) if idx is not None else None,
        "X_ctl": X_ctl,
        "outputs": out,
    }
    save(name, payload)
    return model


def ism_case(ref, name, config, N, L, start, end, seed):
    """Saturation-mutagenesis scores computed with the upstream forward.

    For every reference sequence, position p in [start, end) and each of
    the three non-reference bases, the mutant is scored as
    d_logcount = logcount(mutant) - logcount(reference) and
    jsd = jensen_shannon_distance(profile(mutant), softmax(profile(reference)))
    flattened over (channels, positions), using the upstream metric.
    """
    torch.manual_seed(seed)
    model = ref.Cherimoya(**config, verbose=False, compile=False).eval()
    g = torch.Generator().manual_seed(seed + 1)
    idx = torch.randint(0, 4, (N, L), generator=g)
    X = one_hot(idx)
    W = end - start
    dlc = torch.zeros(N, 4, W)
    jsd = torch.zeros(N, 4, W)
    jsd_fn = ref.performance.jensen_shannon_distance
    with torch.no_grad():
        p_ref, c_ref = model(X)
        for n in range(N):
            muts = []
            for p in range(start, end):
                for b in range(4):
                    Xm = X[n].clone()
                    Xm[:, p] = 0.0
                    Xm[b, p] = 1.0
                    muts.append(Xm)
            Xm = torch.stack(muts)
            pm, cm = model(Xm)
            d = (cm[:, 0] - c_ref[n, 0]).reshape(W, 4).T
            pr = torch.softmax(p_ref[n].reshape(1, -1), dim=-1).expand(pm.shape[0], -1)
            j = jsd_fn(pm.reshape(pm.shape[0], -1), pr).reshape(W, 4).T
            dlc[n] = d
            jsd[n] = j
    payload = {
        "config": model._init_kwargs(),
        "state_dict": {k: v.clone() for k, v in model.state_dict().items()},
        "bases": idx.to(torch.int8),
        "start": start, "end": end,
        "d_logcount": dlc, "jsd": jsd,
        "profile_ref": p_ref.clone(), "logcounts_ref": c_ref.clone(),
    }
    save(name, payload)


def main():
    ref = import_upstream()
    torch.set_num_threads(8)
    cheri = ref.cheri

    # 1. fused conv + norm (cheri.py:52-98)
    cases = []
    for (N, L, C, d, seed) in [(2, 64, 8, 2, 0), (1, 300, 16, 7, 1), (3, 130, 128, 64, 2)]:
        g = torch.Generator().manual_seed(seed)
        x = torch.randn(N, L, C, generator=g)
        w = torch.randn(3, C, generator=g) * 0.1
        y = cheri._cheri_conv_norm_cpu(x, w, d)
        cases.append({"x": x, "w": w, "dilation": d, "y": y})
    save("conv_norm", {"cases": cases})

    # 2. one CheriBlock, CPU branch (cheri.py:1072-1082)
    blocks = []
    for (C, d, exp, rs, N, L, seed) in [(16, 4, 2, 0.15, 2, 100, 3), (128, 16, 2, 0.15, 1, 211, 4),
                                         (24, 1, 3, 0.5, 2, 50, 5)]:
        torch.manual_seed(seed)
        blk = cheri.CheriBlock(C, d, expansion=exp, residual_scale=rs).eval()
        g = torch.Generator().manual_seed(seed + 100)
        x = torch.randn(N, L, C, generator=g)
        with torch.no_grad():
            y = blk(x)
        blocks.append({"n_filters": C, "dilation": d, "expansion": exp, "residual_scale": rs,
                       "state_dict": {k: v.clone() for k, v in blk.state_dict().items()},
                       "state_dict_keys": list(blk.state_dict().keys()),
                       "x": x, "y": y})
    save("cheri_block", {"cases": blocks})

    # 3. models (cherimoya.py:340-400)
    model_case(ref, "model_default_L2114",
               dict(n_filters=128, n_layers=9, signal_groups=[1]), N=2, L=2114, seed=0,
               autocast=True, wrappers=True)
    model_case(ref, "model_small_float_input",
               dict(n_filters=16, n_layers=3, signal_groups=[1]), N=3, L=300, seed=10,
               input_kind="randn", autocast=True)
    model_case(ref, "model_multitask",
               dict(n_filters=32, n_layers=4, signal_groups=[1, 2, 2, 2, 2]), N=2, L=400,
               seed=20, wrappers=True)
    model_case(ref, "model_control_tracks",
               dict(n_filters=16, n_layers=3, signal_groups=[2], n_control_tracks=2), N=2,
               L=300, seed=30, ctl=True, wrappers=True)
    model_case(ref, "model_wide_c256",
               dict(n_filters=256, n_layers=2, signal_groups=[1], trimming=100), N=2, L=400,
               seed=40)

    # 4. metrics (performance.py:138-246)
    g = torch.Generator().manual_seed(50)
    a = torch.randn(3, 2, 500, generator=g)
    b = torch.rand(3, 2, 500, generator=g)
    b[0, 0, :10] = 0.0
    perf = ref.performance
    save("metrics", {"logps": a, "counts": b,
                     "jsd": perf.jensen_shannon_distance(a, b),
                     "pearson": perf.pearson_corr(a, b)})

    # 5. ISM definition pinned on the upstream forward + JSD
    ism_case(ref, "ism_small", dict(n_filters=16, n_layers=3, signal_groups=[1]),
             N=2, L=200, start=80, end=120, seed=60)


if __name__ == "__main__":
    main()
