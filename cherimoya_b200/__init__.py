"""cherimoya_b200 -- a B200 (sm_100a) inference engine for the Cherimoya
model's hot path, drop-in for the upstream ``cherimoya`` package's model
API: ``Cherimoya``, ``CheriBlock``, the output wrappers, the checkpoint
layout, plus on-device saturation mutagenesis and variant scoring, and
pipelined batched prediction with reverse-complement averaging.
"""

from .cheri import CheriBlock, FusedDilatedConvNorm, fused_dilated_conv_norm
from .model import Cherimoya
from .wrappers import ControlWrapper, ExpectedCountsWrapper, LogCountWrapper, ProfileWrapper
from .ism import (saturation_mutagenesis, sharded_saturation_mutagenesis,
                  sharded_variant_effect, variant_effect)
from .predict import predict, rc_forward
from . import attribution

__version__ = "0.1.0"

__all__ = [
    "Cherimoya", "CheriBlock", "FusedDilatedConvNorm", "fused_dilated_conv_norm",
    "ControlWrapper", "ProfileWrapper", "LogCountWrapper", "ExpectedCountsWrapper",
    "saturation_mutagenesis", "variant_effect", "sharded_saturation_mutagenesis",
    "sharded_variant_effect", "predict", "rc_forward", "attribution",
]
