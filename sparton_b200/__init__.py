"""sparton_b200 — B200-native SPLADE projection head.

Drop-in for hhkbble/sparton: ``from sparton_b200 import SpartonHead``. As
upstream (src/sparton/__init__.py:1-13), the module is exported only when CUDA
is available; without it a warning is issued and ``__all__`` is empty. The
implementation modules (``sparton_b200.head``, ``sparton_b200.ops``) import on
any machine; calling the operators needs an sm_100 GPU and the native library
built by ``python -m sparton_b200.build``.
"""
import warnings

import torch

if not torch.cuda.is_available():
    warnings.warn(
        "CUDA is not available. Sparton only runs on CUDA devices.",
        stacklevel=2,
    )
    __all__ = []
else:
    __all__ = ["SpartonHead"]
    from .head import SpartonHead
