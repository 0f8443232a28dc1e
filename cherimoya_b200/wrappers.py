"""Output wrappers, drop-in for upstream ``cherimoya/wrappers.py``.

They call ``model(...)``, so on CUDA under ``no_grad`` they run the engine;
there the ProfileWrapper and ExpectedCountsWrapper arithmetic on the
forward's outputs also runs as one fused kernel each (``ops.profile_wrapper``,
``ops.expected_counts``).
"""

import torch


def _engine_epilogue(profile):
    """The fused epilogue kernels serve CUDA inference on fp32 outputs (what
    the engine's forward returns); anything else keeps the PyTorch ops."""
    return (profile.is_cuda and not torch.is_grad_enabled() and profile.dtype == torch.float32
            and profile.dim() == 3)


class ControlWrapper(torch.nn.Module):
    """Supplies an all-zero control track when the model expects controls and
    none is given (upstream wrappers.py:11-47)."""

    def __init__(self, model):
        super().__init__()
        self.model = model

    def forward(self, X, X_ctl=None):
        if X_ctl is not None:
            return self.model(X, X_ctl)
        if self.model.n_control_tracks == 0:
            return self.model(X)
        X_ctl = torch.zeros(X.shape[0], self.model.n_control_tracks, X.shape[-1],
                            dtype=X.dtype, device=X.device)
        return self.model(X, X_ctl)


class _ProfileLogitScaling(torch.nn.Module):
    """logits * softmax(logits), isolated as its own module for attribution
    tools (upstream wrappers.py:50-68)."""

    def __init__(self):
        super().__init__()
        self.softmax = torch.nn.Softmax(dim=-1)

    def forward(self, logits):
        return logits * self.softmax(logits)


class ProfileWrapper(torch.nn.Module):
    """sum(softmax(l) * l) of the mean-centred flattened profile logits
    (upstream wrappers.py:71-99)."""

    def __init__(self, model):
        super().__init__()
        self.model = model
        self.flatten = torch.nn.Flatten()
        self.scaling = _ProfileLogitScaling()

    def forward(self, X, X_ctl=None):
        profile = self.model(X, X_ctl=X_ctl)[0]
        if _engine_epilogue(profile):
            from . import ops
            return ops.profile_wrapper(profile)
        logits = self.flatten(profile)
        logits = logits - torch.mean(logits, dim=-1, keepdims=True)
        return self.scaling(logits).sum(dim=-1, keepdims=True)


class LogCountWrapper(torch.nn.Module):
    """The log-count output (upstream wrappers.py:102-122)."""

    def __init__(self, model):
        super().__init__()
        self.model = model

    def forward(self, X, X_ctl=None):
        return self.model(X, X_ctl=X_ctl)[1]


class ExpectedCountsWrapper(torch.nn.Module):
    """expm1(group log-count) distributed by a joint softmax over each signal
    group's channels and positions (upstream wrappers.py:125-166)."""

    def __init__(self, model):
        super().__init__()
        self.model = model

    def forward(self, X, X_ctl=None):
        y_logits, y_logcounts = self.model(X, X_ctl=X_ctl)
        if _engine_epilogue(y_logits):
            from . import ops
            return ops.expected_counts(y_logits, y_logcounts, list(self.model.signal_groups))
        y_counts = torch.expm1(y_logcounts)
        out = []
        for i, logits in enumerate(torch.split(y_logits, self.model.signal_groups, dim=1)):
            n, c, length = logits.shape
            probs = torch.softmax(logits.reshape(n, -1), dim=-1).reshape(n, c, length)
            out.append(probs * y_counts[:, i, None, None])
        return torch.cat(out, dim=1)
