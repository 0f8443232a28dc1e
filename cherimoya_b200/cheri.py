"""The Cheri Block, drop-in for upstream ``cherimoya/cheri.py``.

Same module tree, parameter names, init order and checkpoint keys as
upstream (``CheriBlock`` -> ``conv`` (``FusedDilatedConvNorm`` holding
``conv_weight``), ``linear1``, ``linear2``, ``activation``; the depthwise
weight is serialised under its legacy key ``conv_weight``).

Dispatch (mirrors upstream ``CheriBlock._can_use_inference_path``,
cheri.py:1027-1038):
  * CUDA input and ``torch.is_grad_enabled() == False`` -> the sm_100a
    engine (``cherimoya_b200::block_forward``); raises if the engine cannot
    run, never falls back.
  * CPU input, or gradients enabled -> differentiable PyTorch ops with the
    upstream semantics (cheri.py:52-98, 1080-1082). This is the training /
    attribution path; it is not used for CUDA inference.
"""

import torch
import torch.nn.functional as F

CONV_NORM_EPS = 1e-3


def conv_norm_torch(x, w, dilation, eps=CONV_NORM_EPS):
    """3-tap depthwise dilated conv + per-example LayerNorm over (L, C) in
    differentiable PyTorch ops (upstream cheri.py:52-98)."""
    N, L, C = x.shape
    y = F.conv1d(x.transpose(1, 2), w.t().unsqueeze(1).to(x.dtype), padding=dilation,
                 dilation=dilation, groups=C).transpose(1, 2)
    flat = y.reshape(N, -1).float()
    mean = flat.mean(dim=1, keepdim=True)
    var = flat.var(dim=1, keepdim=True, unbiased=False)
    flat = (flat - mean) * torch.rsqrt(var + eps)
    return flat.reshape(N, L, C).to(y.dtype)


def fused_dilated_conv_norm(x, w, dilation):
    """Fused 3-tap dilated depthwise conv + per-example norm (upstream
    cheri.py:757-783)."""
    return conv_norm_torch(x, w, dilation)


class FusedDilatedConvNorm(torch.nn.Module):
    """Module owning the depthwise weight (upstream cheri.py:786-826).

    The engine path calls the fused kernel directly, so hooks registered on
    this module fire on the PyTorch path only (same asymmetry as upstream,
    cheri.py:795-799)."""

    def __init__(self, n_filters, dilation):
        super().__init__()
        self.n_filters = n_filters
        self.dilation = dilation
        # allocated here, initialised by CheriBlock (RNG draw order as upstream)
        self.conv_weight = torch.nn.Parameter(torch.randn(3, n_filters))

    def forward(self, X):
        assert X.ndim == 3, f"expected (N, L, C), got {tuple(X.shape)}"
        assert X.shape[-1] == self.n_filters, (
            f"channel dim {X.shape[-1]} != n_filters {self.n_filters}")
        return fused_dilated_conv_norm(X, self.conv_weight, self.dilation)


def _rename_conv_key(module, destination, prefix, _local_metadata):
    """Serialise ``conv.conv_weight`` under the legacy ``conv_weight`` key,
    keeping its position (upstream cheri.py:829-855)."""
    new_key = prefix + "conv.conv_weight"
    if new_key not in destination:
        return
    old_key = prefix + "conv_weight"
    items = [(old_key if k == new_key else k, v) for k, v in destination.items()]
    destination.clear()
    destination.update(items)


class CheriBlock(torch.nn.Module):
    """One Cheri Block: depthwise dilated conv + per-example LayerNorm, then
    a bias-free C -> expansion*C -> C GELU(tanh) MLP, scaled residual
    (upstream cheri.py:858-1082)."""

    def __init__(self, n_filters, dilation, expansion=2, residual_scale=0.15):
        super().__init__()
        self.n_filters = n_filters
        self.dilation = dilation
        self.expansion = expansion
        self.residual_scale = residual_scale
        hidden = expansion * n_filters
        self.conv = FusedDilatedConvNorm(n_filters, dilation)
        self.linear1 = torch.nn.Linear(n_filters, hidden, bias=False)
        self.linear2 = torch.nn.Linear(hidden, n_filters, bias=False)
        self.activation = torch.nn.GELU(approximate="tanh")
        torch.nn.init.trunc_normal_(self.conv.conv_weight, std=0.02)
        torch.nn.init.trunc_normal_(self.linear1.weight, std=0.02)
        torch.nn.init.trunc_normal_(self.linear2.weight, std=0.02)
        self._engine_cache = None
        self.register_state_dict_post_hook(_rename_conv_key)

    @property
    def conv_weight(self):
        """Read-only alias of ``self.conv.conv_weight`` (upstream cheri.py:972-984)."""
        return self.conv.conv_weight

    def _load_from_state_dict(self, state_dict, prefix, *args, **kwargs):
        """Accept the legacy ``conv_weight`` key (upstream cheri.py:986-1002)."""
        old_key, new_key = prefix + "conv_weight", prefix + "conv.conv_weight"
        if old_key in state_dict and new_key not in state_dict:
            state_dict[new_key] = state_dict.pop(old_key)
        super()._load_from_state_dict(state_dict, prefix, *args, **kwargs)

    def _engine_weights(self, device):
        """Packed engine weights, rebuilt whenever a parameter changes
        (tracked through the parameters' version counters)."""
        params = (self.conv.conv_weight, self.linear1.weight, self.linear2.weight)
        key = (str(device), float(self.residual_scale),
               tuple((p.data_ptr(), p._version) for p in params))
        if self._engine_cache is None or self._engine_cache[0] != key:
            from . import ops
            buf, off = ops.pack_block(*params, self.residual_scale, device)
            self._engine_cache = (key, buf, off)
        return self._engine_cache[1], self._engine_cache[2]

    def forward(self, X):
        if X.is_cuda and not torch.is_grad_enabled():
            from . import ops
            buf, off = self._engine_weights(X.device)
            out = ops.block_forward(X, buf, off, self.expansion * self.n_filters, self.dilation)
            return out if out.dtype == X.dtype else out.to(X.dtype)
        X_conv = self.conv(X)
        X_mlp = self.linear2(self.activation(self.linear1(X_conv)))
        return X + X_mlp * self.residual_scale
