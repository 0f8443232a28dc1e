"""The Cherimoya model, drop-in for upstream ``cherimoya/cherimoya.py``.

Same constructor arguments and defaults, same submodules, parameter
initialisation order, ``state_dict`` keys and ``save``/``load`` payload
(``{'config', 'state_dict'}``, loadable with ``weights_only=True``), same
``forward(X, X_ctl=None) -> (profile logits, log-counts)``.

``forward`` dispatch:
  * CUDA input under ``torch.no_grad()`` with stock Cheri Blocks -> one
    call of the sm_100a engine for the whole model
    (``cherimoya_b200::forward``: stem, every block, both heads). The
    engine raises if it cannot run; there is no fallback.
  * Otherwise (CPU input, gradients enabled, or a subclass that replaced
    the blocks) -> differentiable PyTorch ops with the upstream semantics
    (cherimoya.py:340-400).

Arithmetic of the engine path (``precision``):
  * ``'fp32'``: fp32 residual stream and heads, bf16 tensor-core MLP
    contractions with fp32 accumulation (max abs error vs the fp32 CPU path
    ~3e-5 on the default model).
  * ``'bf16'``: bf16 residual stream, the upstream autocast-bf16 mode.
  * ``'auto'`` (default): bf16 when X is bf16 or CUDA autocast is active
    with bf16, else fp32.
"""

import torch

from .cheri import CheriBlock
from ._lib import MODE_BF16, MODE_FP32


def _validate_signal_groups(groups, label="signal_groups"):
    """Upstream cherimoya/io.py:11-46: a non-empty list of positive ints."""
    if not isinstance(groups, (list, tuple)):
        raise ValueError("{} must be a list of positive ints; got {!r}".format(label, groups))
    if len(groups) == 0:
        raise ValueError("{} must be non-empty; got an empty list".format(label))
    for g in groups:
        if (not isinstance(g, int)) or isinstance(g, bool) or g < 1:
            raise ValueError("{} entries must be positive ints; got {!r} in {!r}".format(
                label, g, list(groups)))


class Cherimoya(torch.nn.Module):
    """The Cherimoya sequence-to-function model (upstream cherimoya.py:97-400).

    ``compile`` and ``compile_mode`` are accepted for call compatibility;
    the engine path is already one fused native call, so no
    ``torch.compile`` wrapping is applied.
    """

    def __init__(self, n_filters=128, n_layers=9, signal_groups=None, n_control_tracks=0,
                 expansion=2, residual_scale=0.15, name=None, trimming=None, verbose=True,
                 compile=True, compile_mode="max-autotune", precision="auto"):
        super().__init__()
        if signal_groups is None:
            signal_groups = [1]
        signal_groups = list(signal_groups)
        _validate_signal_groups(signal_groups)
        self.signal_groups = signal_groups
        self.n_outputs = sum(signal_groups)
        self.n_groups = len(signal_groups)
        self.n_filters = n_filters
        self.n_layers = n_layers
        self.n_control_tracks = n_control_tracks
        self.expansion = expansion
        self.residual_scale = residual_scale
        self.name = name or "cherimoya.{}.{}".format(n_filters, n_layers)
        self.trimming = trimming if trimming is not None else (
            46 + sum(2 ** i for i in range(n_layers)))
        self.verbose = verbose
        if precision not in ("auto", "fp32", "bf16"):
            raise ValueError("precision must be 'auto', 'fp32' or 'bf16'")
        self.precision = precision

        # construction order = upstream RNG draw order (cherimoya.py:173-197)
        self.iconv = torch.nn.Conv1d(4, n_filters, kernel_size=21, padding=10)
        self.igelu = torch.nn.GELU(approximate="tanh")
        self.blocks = torch.nn.ModuleList([
            CheriBlock(n_filters, 2 ** i, expansion=expansion, residual_scale=residual_scale)
            for i in range(self.n_layers)])
        self.fconv = torch.nn.Conv1d(n_filters + n_control_tracks, self.n_outputs,
                                     kernel_size=75, padding=37)
        n_count_control = 1 if n_control_tracks > 0 else 0
        self.linear = torch.nn.Linear(n_filters + n_count_control, self.n_groups)
        self.lw0 = torch.nn.Parameter(torch.ones(self.n_groups))
        self.lw1 = torch.nn.Parameter(torch.ones(self.n_groups))
        torch.nn.init.trunc_normal_(self.iconv.weight, std=0.02)
        torch.nn.init.trunc_normal_(self.fconv.weight, std=0.02)
        torch.nn.init.trunc_normal_(self.linear.weight, std=0.02)
        torch.nn.init.zeros_(self.iconv.bias)
        torch.nn.init.zeros_(self.fconv.bias)
        torch.nn.init.zeros_(self.linear.bias)

        self._compile = bool(compile)
        self._compile_mode = compile_mode
        self._engine_cache = None

    # ------------------------------------------------------------ checkpoint
    def _init_kwargs(self):
        """Constructor kwargs stored in checkpoints (upstream cherimoya.py:246-258)."""
        return {
            "n_filters": self.n_filters,
            "n_layers": self.n_layers,
            "signal_groups": list(self.signal_groups),
            "n_control_tracks": self.n_control_tracks,
            "expansion": self.expansion,
            "residual_scale": self.residual_scale,
            "name": self.name,
            "trimming": self.trimming,
            "verbose": False,
        }

    def save(self, path):
        """Write ``{'config', 'state_dict'}`` (upstream cherimoya.py:260-278)."""
        torch.save({"config": self._init_kwargs(), "state_dict": self.state_dict()}, path)

    @classmethod
    def load(cls, path, device="cpu", compile=True, compile_mode="max-autotune",
             precision="auto"):
        """Load a checkpoint written by ``save`` (upstream cherimoya.py:280-327)."""
        payload = torch.load(path, map_location=device, weights_only=True)
        model = cls(**payload["config"], compile=compile, compile_mode=compile_mode,
                    precision=precision)
        model.load_state_dict(payload["state_dict"])
        return model.to(device)

    # ------------------------------------------------------------ engine
    def _stock_blocks(self):
        return (isinstance(self.blocks, torch.nn.ModuleList) and len(self.blocks) == self.n_layers
                and all(type(b) is CheriBlock and b.dilation == 2 ** i
                        and b.expansion == self.expansion and b.residual_scale == self.residual_scale
                        for i, b in enumerate(self.blocks)))

    def engine_mode(self, X):
        """Arithmetic mode the engine uses for input X."""
        if self.precision == "bf16":
            return MODE_BF16
        if self.precision == "fp32":
            return MODE_FP32
        if X.dtype == torch.bfloat16:
            return MODE_BF16
        if torch.is_autocast_enabled("cuda") and \
                torch.get_autocast_dtype("cuda") == torch.bfloat16:
            return MODE_BF16
        return MODE_FP32

    def engine_desc(self, seq_len, mode):
        """The op-level model description list (see ``ops``)."""
        return [int(self.n_filters), int(self.n_layers), int(self.expansion),
                int(self.n_outputs), int(self.n_groups), int(self.n_control_tracks),
                int(self.trimming), int(seq_len), int(mode)]

    def engine_weights(self, device):
        """Packed engine weights for `device`, rebuilt when any parameter is
        replaced or updated in place (parameter version counters)."""
        from . import ops
        params = [self.iconv.weight, self.iconv.bias]
        for b in self.blocks:
            params += [b.conv.conv_weight, b.linear1.weight, b.linear2.weight]
        params += [self.fconv.weight, self.fconv.bias, self.linear.weight, self.linear.bias]
        key = (str(device), float(self.residual_scale),
               tuple((p.data_ptr(), p._version, p.dtype) for p in params))
        if self._engine_cache is None or self._engine_cache[0] != key:
            sd = {
                "iconv_weight": self.iconv.weight, "iconv_bias": self.iconv.bias,
                "conv_weight": [b.conv.conv_weight for b in self.blocks],
                "linear1_weight": [b.linear1.weight for b in self.blocks],
                "linear2_weight": [b.linear2.weight for b in self.blocks],
                "fconv_weight": self.fconv.weight, "fconv_bias": self.fconv.bias,
                "linear_weight": self.linear.weight, "linear_bias": self.linear.bias,
            }
            desc = self.engine_desc(1 + 2 * self.trimming, MODE_FP32)
            buf, off = ops.pack_weights(sd, desc, self.residual_scale, device)
            self._engine_cache = (key, buf, off)
        return self._engine_cache[1], self._engine_cache[2]

    def use_engine(self, X):
        return X.is_cuda and not torch.is_grad_enabled() and self._stock_blocks()

    # ------------------------------------------------------------ forward
    def forward(self, X, X_ctl=None):
        """(profile logits (N, n_outputs, L - 2T), log-counts (N, n_groups))."""
        if self.use_engine(X):
            from . import ops
            mode = self.engine_mode(X)
            buf, off = self.engine_weights(X.device)
            desc = self.engine_desc(X.shape[-1], mode)
            return ops.forward(X, X_ctl, buf, off, desc, float(self.residual_scale))
        return self._forward_torch(X, X_ctl)

    def _forward_torch(self, X, X_ctl=None):
        """PyTorch path with the upstream semantics (cherimoya.py:340-400)."""
        start, end = self.trimming, X.shape[2] - self.trimming
        X = self.igelu(self.iconv(X))
        X = X.transpose(1, 2).contiguous()
        for i in range(self.n_layers):
            X = self.blocks[i](X)
        X = X.transpose(1, 2).contiguous()
        X_w_ctl = X if X_ctl is None else torch.cat([X, X_ctl], dim=1)
        y_profile = self.fconv(X_w_ctl)[:, :, start:end]
        X = torch.mean(X[:, :, start:end].float(), dim=2)
        if X_ctl is not None:
            X_ctl = torch.sum(X_ctl[:, :, start:end].float(), dim=(1, 2)).unsqueeze(-1)
            X = torch.cat([X, torch.log(X_ctl + 1)], dim=-1)
        y_counts = self.linear(X)
        return y_profile, y_counts

    def forward_bases(self, bases, X_ctl=None, precision=None):
        """Engine forward on base indices (N, L) int8 in 0..3 (A, C, G, T):
        one byte per position crosses PCIe instead of 16."""
        from . import ops
        if not bases.is_cuda:
            raise RuntimeError("cherimoya_b200: forward_bases needs CUDA input")
        mode = {"fp32": MODE_FP32, "bf16": MODE_BF16}.get(precision or self.precision, MODE_FP32)
        buf, off = self.engine_weights(bases.device)
        desc = self.engine_desc(bases.shape[-1], mode)
        with torch.no_grad():
            return ops.forward_bases(bases, X_ctl, buf, off, desc, float(self.residual_scale))
