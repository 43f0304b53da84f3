"""Drop-in for the 1.5-entmax prior of ANANTA_OCR ``dash_attention.py``.

``entmax15`` / ``_Entmax15`` keep the reference's names and autograd contract
(dash_attention.py:637-662): forward y = relu(z - tau)^2 with z = (x - max)/2
and sum(y) = 1, backward dx = dy*g - g * sum(dy*g) / max(sum g, 1e-12) with
g = sqrt(y).  Both run as kernels of ``libdash_b200.so``
(``dash_entmax15_fwd`` / ``dash_entmax15_bwd``) over the rows of the last
dim of any other dim order (moved last and back).  fp32 (inputs of other
dtypes are computed in fp32 and returned in their dtype).
"""
from __future__ import annotations

import torch

from . import ops


class _Entmax15(torch.autograd.Function):
    @staticmethod
    def forward(ctx, X, dim):
        ctx.dim = dim
        x = X.movedim(dim, -1)
        y = ops.entmax15(x).to(X.dtype)
        ctx.save_for_backward(y)
        return y.movedim(-1, dim)

    @staticmethod
    def backward(ctx, dY):
        (y,) = ctx.saved_tensors
        dx = ops.entmax15_backward(y, dY.movedim(ctx.dim, -1)).to(dY.dtype)
        return dx.movedim(-1, ctx.dim), None


def entmax15(X, dim=-1):
    return _Entmax15.apply(X, dim)
