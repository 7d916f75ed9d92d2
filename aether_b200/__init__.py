"""aether_b200 -- a Blackwell-native (sm_100a) train/serve stack.

Layers:
  * ``aether_b200._C``        hand-written sm_100a kernels (tcgen05 GEMM, attention,
                              norms, RoPE, SwiGLU, fused cross-entropy, AdamW, ...)
  * ``aether_b200.ops``       functional + autograd wrappers (CPU tensors use the
                              fp32 PyTorch reference in ``ops.reference``)
  * ``aether_b200.models``    GPT (training bench), Qwen2/2.5 (serving), AetherLM-Nano
  * ``aether_b200.parallel``  DP (ZeRO-1), TP, PP engines over torch.distributed/NCCL
  * ``aether_b200.serving``   KV cache, CUDA-graph decode, scheduler, HTTP server
  * ``aether_b200.formats``   .weights/.meta, safetensors, GGUF
"""
from . import _ext  # noqa: F401

__version__ = "0.1.0"
