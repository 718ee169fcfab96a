"""int8 NHWC pooling over the C ABI (the layers between the convs of the int8 network stacks)."""
from __future__ import annotations

import torch

from . import _lib
from .conv import _ptr, _stream


def maxpool_s8(x: torch.Tensor, r: int, s: int, stride: int, pad: int, out: torch.Tensor | None = None,
               stream=None) -> torch.Tensor:
    """Max over R x S windows; padded positions take no part (b200q_maxpool_s8)."""
    if x.dtype != torch.int8:
        raise TypeError("maxpool_s8 takes int8 activations")
    n, h, w, c = x.shape
    ho, wo = (h + 2 * pad - r) // stride + 1, (w + 2 * pad - s) // stride + 1
    if out is None:
        out = torch.empty((n, ho, wo, c), dtype=torch.int8, device=x.device)
    _lib.check(_lib.lib().b200q_maxpool_s8(_ptr(x.contiguous()), _ptr(out), n, h, w, c, r, s, stride, stride, pad,
                                           pad, _stream(stream)))
    return out


def global_avgpool_s8(x: torch.Tensor, out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """[n, h, w, c] -> [n, c]: clamp(rint(sum / (h*w)), -128, 127) (b200q_global_avgpool_s8)."""
    if x.dtype != torch.int8:
        raise TypeError("global_avgpool_s8 takes int8 activations")
    n, h, w, c = x.shape
    if out is None:
        out = torch.empty((n, c), dtype=torch.int8, device=x.device)
    _lib.check(_lib.lib().b200q_global_avgpool_s8(_ptr(x.contiguous()), _ptr(out), n, h, w, c, _stream(stream)))
    return out
