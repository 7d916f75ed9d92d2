"""Ops: ``functional`` (kernels / CPU reference dispatch), ``autograd``
(training functions with fp32 main-grad accumulation), ``reference`` (fp32
PyTorch oracle)."""
from . import autograd, functional, reference  # noqa: F401
