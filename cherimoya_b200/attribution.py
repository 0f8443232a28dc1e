"""Saturation-mutagenesis attributions in the call shape of tangermeme's
``saturation_mutagenesis``, computed by the engine's fused ISM.

The upstream ``cherimoya attribute`` command
(``cherimoya_cli/commands/attribute.py:43-64``) wraps the model as
``LogCountWrapper(ControlWrapper(model))`` or
``ProfileWrapper(ControlWrapper(model))`` and calls

    saturation_mutagenesis(wrapper, X, dtype=..., device=..., batch_size=...,
                           verbose=..., hypothetical=True, start=mid - 200,
                           end=mid + 200).float()

from tangermeme (pinned ``tangermeme 1.4.0``, upstream ``uv.lock:2748-2749``;
its source is not part of the upstream tree). ``saturation_mutagenesis``
below accepts that call unchanged and returns the tensor the command saves.

What is computed. For reference sequence n, base b and position p in
[start, end), the mutant is the reference with base b at p, and

    delta[n, b, p] = y(mutant) - y(reference)

with y the wrapper's scalar output: the log-count of group ``target`` for a
LogCountWrapper (upstream ``wrappers.py:102-122``), the ProfileWrapper value
(mean-centred flattened profile logits weighted by their softmax, summed;
``wrappers.py:71-99``) for a ProfileWrapper. The base the reference already
has gives 0. The returned attributions follow tangermeme's documented ISM
convention: delta minus its mean over the four bases of each position
(``center=True``, as hypothetical contributions are reported), multiplied by
the one-hot input unless ``hypothetical=True``. ``raw_outputs=True`` returns
(y(reference) (N, 1), y(mutant) (N, 4, W)) instead.

All 3 x W substitutions of every sequence run through the engine's ISM
(mutants built on the device, scores in a fused epilogue); ``batch_size``
only bounds the engine's pass size, which does not change any result (the
engine's outputs do not depend on the batch they are computed in).

A ControlWrapper around a model with control tracks supplies all-zero
controls; the profile head then gets zero control channels and the count
head log(0 + 1) = 0, so the scores equal those of the same model without its
control weights, which is what the engine runs.
"""

import torch

from . import ops
from ._lib import MODE_BF16, MODE_FP32
from .ism import to_bases
from .model import Cherimoya
from .wrappers import ControlWrapper, LogCountWrapper, ProfileWrapper

LOGCOUNT, PROFILE = "logcount", "profile"


def resolve_target(module):
    """(kind, model) of an attribution target: kind is LOGCOUNT for a
    LogCountWrapper, PROFILE for a ProfileWrapper, each optionally around a
    ControlWrapper around a Cherimoya."""
    if isinstance(module, LogCountWrapper):
        kind = LOGCOUNT
    elif isinstance(module, ProfileWrapper):
        kind = PROFILE
    else:
        raise TypeError("cherimoya_b200.saturation_mutagenesis: the target must be a "
                        "LogCountWrapper or ProfileWrapper (optionally around a "
                        "ControlWrapper) of a Cherimoya model; got {}".format(
                            type(module).__name__))
    inner = module.model
    if isinstance(inner, ControlWrapper):
        inner = inner.model
    if not isinstance(inner, Cherimoya):
        raise TypeError("cherimoya_b200.saturation_mutagenesis: the wrapped model must be a "
                        "Cherimoya; got {}".format(type(inner).__name__))
    return kind, inner


def control_free(model):
    """The model a zero-control ControlWrapper amounts to: the same weights
    without the control inputs (cached on the model; rebuilt when a
    parameter changes)."""
    if model.n_control_tracks == 0:
        return model
    key = tuple(p._version for p in model.parameters())
    cached = getattr(model, "_control_free_cache", None)
    dev = next(model.parameters()).device
    if cached is not None and cached[0] == key and cached[1] == dev:
        return cached[2]
    kw = model._init_kwargs()
    kw["n_control_tracks"] = 0
    kw["verbose"] = False
    m0 = Cherimoya(**kw, compile=False, precision=model.precision)
    sd = {k: v.detach().clone() for k, v in model.state_dict().items()}
    C = model.n_filters
    sd["fconv.weight"] = sd["fconv.weight"][:, :C].contiguous()
    sd["linear.weight"] = sd["linear.weight"][:, :C].contiguous()
    m0.load_state_dict(sd)
    m0 = m0.eval().to(dev)
    model._control_free_cache = (key, dev, m0)
    return m0


def _precision(model, dtype):
    if dtype is None:
        return MODE_BF16 if model.precision == "bf16" else MODE_FP32
    if dtype in (torch.bfloat16, "bfloat16", "bf16"):
        return MODE_BF16
    if dtype in (torch.float32, "float32", "float", "fp32"):
        return MODE_FP32
    raise ValueError("cherimoya_b200.saturation_mutagenesis: dtype must be float32 or "
                     "bfloat16; got {!r}".format(dtype))


def attributions(delta, X_window, hypothetical=True, center=True):
    """tangermeme's ISM convention on (N, 4, W) deltas: minus the mean over
    the four bases of each position, times the one-hot window unless
    hypothetical."""
    attr = delta - delta.mean(dim=1, keepdim=True) if center else delta
    if not hypothetical:
        attr = attr * X_window.to(attr.dtype)
    return attr


def saturation_mutagenesis(model, X, args=None, start=0, end=-1, batch_size=32, device="cuda",
                           hypothetical=False, raw_outputs=False, dtype=None, verbose=False,
                           target=0, center=True):
    """ISM attributions of ``model`` (a LogCountWrapper / ProfileWrapper of a
    Cherimoya) for one-hot sequences X (N, 4, L) over positions [start, end)
    (end = -1: L). Returns an (N, 4, end - start) fp32 CPU tensor; see the
    module docstring for the exact quantity."""
    if args is not None:
        raise RuntimeError("cherimoya_b200.saturation_mutagenesis: extra model inputs "
                           "(args) are not supported; a ControlWrapper supplies zero controls")
    kind, cm = resolve_target(model)
    if X.dim() != 3 or X.shape[1] != 4:
        raise RuntimeError("cherimoya_b200.saturation_mutagenesis: X must be one-hot (N, 4, L)")
    L = X.shape[-1]
    start = int(start)
    end = L if end is None or int(end) < 0 else int(end)
    if not (0 <= start < end <= L):
        raise ValueError("invalid window [{}, {}) for length {}".format(start, end, L))
    n_groups = cm.n_groups
    if kind == LOGCOUNT and not (0 <= int(target) < n_groups):
        raise ValueError("target {} out of range for {} count outputs".format(target, n_groups))
    dev = torch.device(device)
    if dev.type != "cuda":
        raise RuntimeError("cherimoya_b200.saturation_mutagenesis runs on CUDA devices")
    mode = _precision(cm, dtype)
    engine_model = control_free(cm).to(dev)
    bases = to_bases(X.to(dev))
    buf, off = engine_model.engine_weights(dev)
    desc = engine_model.engine_desc(L, mode)
    mb = max(int(batch_size), 2048)
    if verbose:
        print("cherimoya_b200 ISM: {} sequences x 3 x {} substitutions".format(
            X.shape[0], end - start))
    with torch.no_grad():
        dlc, _, dpw = ops.ism_targets(bases, start, end, mb, buf, off, desc,
                                      float(engine_model.residual_scale))
        delta = dlc[:, int(target)] if kind == LOGCOUNT else dpw
        if raw_outputs:
            # y of the references through the same engine forward
            prof, lc = ops.forward_bases(bases, None, buf, off, desc,
                                         float(engine_model.residual_scale))
            if kind == LOGCOUNT:
                y_ref = lc[:, int(target):int(target) + 1]
            else:
                flat = prof.reshape(prof.shape[0], -1)
                y_ref = (torch.softmax(flat, -1) * (flat - flat.mean(-1, keepdim=True))).sum(
                    -1, keepdim=True)
            return y_ref.float().cpu(), (y_ref[:, :, None] + delta).float().cpu()
        attr = attributions(delta, X[:, :, start:end].to(dev), hypothetical, center)
    return attr.float().cpu()
