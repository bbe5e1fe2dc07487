"""``greyhound::scale_by(t, g) = t * g`` for a device scalar ``g``.

The backward of every op whose gradients are computed in the forward
(src/greyhound/ops/chunked_linear_cross_entropy.py:175-185,
src/greyhound/ops/cross_entropy.py:79-85, ops/chunked_linear_loss.py:160-166)
multiplies the saved gradients by ``grad_output``. Here that is one
vectorised kernel that reads ``g`` on the device and keeps the saved
tensor's (possibly transposed) layout.
"""

from __future__ import annotations

import torch
from torch import Tensor

from greyhound_b200 import _lib

__all__ = ["scale_by"]


@torch.library.custom_op("greyhound::scale_by", mutates_args=())
def scale_by(t: Tensor, g: Tensor) -> Tensor:
    return _lib.scaled(t, g)


@scale_by.register_fake
def _(t: Tensor, g: Tensor) -> Tensor:
    return torch.empty_like(t)
