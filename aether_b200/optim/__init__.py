"""Optimisers over a ParamArena (flat fp32 master, one kernel launch per group)."""
from .adamw import FlatAdamW, cosine_lr  # noqa: F401
