"""xcalibur_b200: a B200-native (sm_100a) NVFP4-weight / BF16-activation mixture-of-experts layer.

The hot path of lingster/xCalibur (its ``kernels/moe_w4a16_h200`` operator), rebuilt for Blackwell:
hand-written CUDA behind a C-ABI library (``include/xcb_moe.h``), driven from PyTorch for memory and streams.
"""
from . import gf2, packer  # noqa: F401  (pure-Python layout machinery)

__all__ = ["gf2", "packer", "moe_w4a16", "prepare", "kernel_fn", "PreparedMoE"]


def __getattr__(name):
    # the torch-facing layer is imported lazily so that gf2/packer load without torch or the built library
    if name in ("moe_w4a16", "prepare", "kernel_fn", "PreparedMoE", "Weights", "Inputs", "Config"):
        from . import moe

        return getattr(moe, name)
    raise AttributeError(name)
