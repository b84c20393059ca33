"""When the ops route through the ``d2p_py::`` custom ops instead of the
dispatcher ops.

The ``torch.library.custom_op`` wrappers in ``_pt2_ops`` carry their own fake
kernels and autograd formulas, which is what torch.compile and fake-tensor
tracing need.  Eager calls on real tensors go straight to ``torch.ops.d2p``.
(Behaviour of the reference's selector, d2p/_pt2_utils.py.)
"""
from __future__ import annotations

import torch
from torch._subclasses.fake_tensor import FakeTensor


def _tracing() -> bool:
    return bool(torch.compiler.is_compiling())


def is_fake(value: object) -> bool:
    """A fake tensor: shapes and dtypes only, no data to read."""
    return isinstance(value, FakeTensor)


def use_pt2_ops(*args: object) -> bool:
    """True while Dynamo traces the caller, or when an argument is a fake tensor."""
    return _tracing() or any(is_fake(a) for a in args)
