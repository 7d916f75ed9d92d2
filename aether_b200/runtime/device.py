"""ctypes bindings to ``libaether_dev.so`` -- the device-handle C ABI
(``aether_dev_*`` buffer registry and graphs, ``aether_op_*_cuda`` ops).

    from aether_b200.runtime.device import Dev
    d = Dev()                      # loads the library and runs aether_dev_init
    a = d.upload(np.ones((4, 8), np.float32))
    b = d.upload(np.ones((8, 2), np.float32))
    c = d.alloc_f32(8)
    d.call("aether_op_matmul_f32_cuda", a, b, c, 4, 8, 2)
    d.download(c, (4, 2))

Every op checks its handles' kinds and sizes and returns -1 instead of
launching when they do not fit; -2 means a CUDA error, whose text
``last_error()`` returns.

Reference: the i64-handle device ABI of runtime/src/cuda.rs:7230-11760.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

_PKG = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(_PKG, "libaether_dev.so")
_LIB = None

I, L, Fl, P = C.c_int, C.c_int64, C.c_float, C.c_char_p

# (result, [arguments]) for every export; i64 handles, int extents, float scalars.
SIGNATURES = {
    "aether_dev_init": (I, []),
    "aether_dev_set_device": (I, [I]),
    "aether_dev_count": (I, []),
    "aether_dev_last_error": (P, []),
    "aether_dev_mem_free_bytes": (L, []),
    "aether_dev_alloc_f32": (L, [I]),
    "aether_dev_alloc_i32": (L, [I]),
    "aether_dev_alloc_u8": (L, [I]),
    "aether_dev_free_f32": (I, [L]),
    "aether_dev_free_i32": (I, [L]),
    "aether_dev_free_u8": (I, [L]),
    "aether_dev_h2d_f32": (I, [L, L, I]),
    "aether_dev_d2h_f32": (I, [L, L, I]),
    "aether_dev_h2d_i32": (I, [L, L, I]),
    "aether_dev_d2h_i32": (I, [L, L, I]),
    "aether_dev_h2d_u8": (I, [L, L, I]),
    "aether_dev_d2h_u8": (I, [L, L, I]),
    "aether_dev_h2d_f32_n": (I, [L, L, I]),
    "aether_dev_d2h_f32_n": (I, [L, L, I]),
    "aether_dev_h2d_i32_n": (I, [L, L, I]),
    "aether_dev_d2d_f32_offset": (I, [L, I, L, I, I]),
    "aether_wall_us": (L, []),
    "aether_dev_sync": (I, []),
    "aether_dev_graph_begin": (I, []),
    "aether_dev_graph_end": (I, []),
    "aether_dev_graph_launch": (I, []),
    "aether_dev_graph_destroy": (I, []),
    "aether_op_matmul_f32_cuda": (I, [L, L, L, I, I, I]),
    "aether_op_matmul_tn_f32_cuda": (I, [L, L, L, I, I, I]),
    "aether_op_matmul_nt_f32_cuda": (I, [L, L, L, I, I, I]),
    "aether_op_matmul_gelu_f32_cuda": (I, [L, L, L, I, I, I]),
    "aether_op_matmul_f32_cuda_profile": (I, [L, L, L, I, I, I]),
    "aether_op_matmul_backward_rhs_f32_cuda": (I, [L, L, L, I, I, I]),
    "aether_op_matmul_backward_lhs_f32_cuda": (I, [L, L, L, I, I, I]),
    "aether_bench_matmul_batch": (I, [L, L, L, I, I, I, I]),
    "aether_op_quant_matmul_backward_lhs_f32_cuda": (I, [L, I, L, L, I, I]),
    "aether_op_add_f32_cuda": (I, [L, L, L, I]),
    "aether_op_add_inplace_f32_cuda": (I, [L, L, I]),
    "aether_op_mul_inplace_f32_cuda": (I, [L, L, I]),
    "aether_op_scale_f32_cuda": (I, [L, Fl, I]),
    "aether_op_gelu_f32_cuda": (I, [L, L, I]),
    "aether_op_gelu_backward_f32_cuda": (I, [L, L, L, I]),
    "aether_op_gelu_erf_f32_cuda": (I, [L, L, I]),
    "aether_op_silu_f32_cuda": (I, [L, I]),
    "aether_op_silu_backward_f32_cuda": (I, [L, L, L, I]),
    "aether_op_bias_add_f32_cuda": (I, [L, L, I, I]),
    "aether_op_transpose_021_f32_cuda": (I, [L, L, I, I, I]),
    "aether_op_embed_lookup_f32_cuda": (I, [L, L, L, I, I]),
    "aether_op_embed_scatter_add_f32_cuda": (I, [L, L, L, I, I]),
    "aether_op_gqa_repeat_kv_f32_cuda": (I, [L, L, I, I, I, I]),
    "aether_op_gqa_reduce_kv_grad_f32_cuda": (I, [L, L, I, I, I, I]),
    "aether_op_append_kv_f32_cuda": (I, [L, L, L, L, I, I]),
    "aether_op_adamw_step_f32_cuda": (I, [L, L, L, L, Fl, Fl, Fl, Fl, Fl, L, I]),
    "aether_op_rope_apply_f32_cuda": (I, [L, I, I, I, Fl, I]),
    "aether_op_rope_apply_backward_f32_cuda": (I, [L, I, I, I, Fl, I]),
    "aether_op_softmax_f32_cuda": (I, [L, L, I, I]),
    "aether_op_softmax_backward_f32_cuda": (I, [L, L, L, I, I]),
    "aether_op_softmax_backward_scaled_f32_cuda": (I, [L, L, L, Fl, I, I]),
    "aether_op_layer_norm_f32_cuda": (I, [L, L, L, L, L, L, Fl, I, I]),
    "aether_op_add_layer_norm_f32_cuda": (I, [L, L, L, L, L, L, L, Fl, I, I]),
    "aether_op_layer_norm_backward_dx_f32_cuda": (I, [L, L, L, L, L, L, I, I]),
    "aether_op_layer_norm_backward_params_f32_cuda": (I, [L, L, L, L, L, L, I, I]),
    "aether_op_rms_norm_f32_cuda": (I, [L, L, L, Fl, I, I]),
    "aether_op_fused_add_rmsnorm_f32_cuda": (I, [L, L, L, L, Fl, I, I]),
    "aether_op_rms_norm_backward_dx_f32_cuda": (I, [L, L, L, L, L, Fl, I, I]),
    "aether_op_rms_norm_backward_gamma_f32_cuda": (I, [L, L, L, L, I, I]),
    "aether_op_cross_entropy_f32_cuda": (Fl, [L, L, L, I, I]),
    "aether_op_cross_entropy_backward_f32_cuda": (I, [L, L, L, I, I]),
    "aether_op_sdpa_causal_forward_f32_cuda": (I, [L, L, L, L, L, I, I, I]),
    "aether_op_sdpa_causal_backward_f32_cuda": (I, [L, L, L, L, L, L, L, L, L, I, I, I]),
    "aether_op_attention_seq1_f32_cuda": (I, [L, L, L, L, I, I, I, I, Fl]),
    "aether_op_dequant_q4_k_m_f32_cuda": (I, [L, L, I]),
    "aether_op_dequant_q6_k_f32_cuda": (I, [L, L, I]),
    "aether_op_dequant_f32_cuda": (I, [I, L, L, I]),
    "aether_op_fused_q4k_ffn_gate_up_silu_mul_cuda": (I, [L, L, L, L, I, I]),
    "aether_op_fused_q4k_ffn_gate_up_silu_mul_v2_cuda": (I, [L, L, L, L, I, I]),
    "aether_op_fused_f16_matmul_seq1_cuda": (I, [L, L, L, I, I]),
    "aether_op_fused_f32_matmul_seq1_cuda": (I, [L, L, L, I, I]),
    "aether_nccl_real_init_multi_gpu": (I, [I]),
    "aether_nccl_real_get_handle": (L, [I]),
    "aether_nccl_real_all_reduce_f32": (I, [L, L, I, I, L]),
    "aether_nccl_real_comm_world_size": (I, [L]),
    "aether_nccl_real_comm_rank": (I, [L]),
    "aether_nccl_real_finalize": (I, []),
}
for _n in ("q4k", "q4_0", "q5_0", "q8_0", "q5_k", "q3_k", "iq4_nl", "iq4_xs"):
    SIGNATURES[f"aether_op_fused_{_n}_matmul_seq1_cuda"] = (I, [L, L, L, I, I])
for _v in ("v2", "v3", "v4", "v5", "v6"):
    SIGNATURES[f"aether_op_fused_q4k_matmul_seq1_{_v}_cuda"] = (I, [L, L, L, I, I])
SIGNATURES["aether_op_fused_q6k_matmul_seq1_v2_cuda"] = (I, [L, L, L, I, I])
for _n in ("q4k", "q8_0", "q5_0", "q3_k", "q6_k", "q5_k", "iq4_xs"):
    SIGNATURES[f"aether_op_fused_{_n}_expert_matmul_seq1_cuda"] = (I, [L, L, L, I, I, I])


SIGNATURES.update({
    "aether_op_rope_apply_devarg_f32_cuda": (I, [L, I, I, I, Fl, L]),
    "aether_op_batched_rope_apply_devarg_f32_cuda": (I, [L, I, I, I, Fl, L]),
    "aether_op_qkv_bias_rope_devarg_f32_cuda": (I, [L, L, L, L, L, L, I, I, I, Fl, L]),
    "aether_op_append_kv_devarg_f32_cuda": (I, [L, L, L, L, I, L]),
    "aether_op_attention_seq1_devarg_f32_cuda": (I, [L, L, L, L, I, I, I, Fl, I, L]),
    "aether_op_paged_append_kv_devarg_f32_cuda": (I, [L, L, L, L, L, I, I, L]),
    "aether_op_paged_append_kv_mla_devarg_f32_cuda": (I, [L, L, L, L, L, I, I, I, L]),
    "aether_op_paged_attention_seq1_v4_devarg_f32_cuda": (I, [L, L, L, L, L, L, L, L, I, I, I, I, Fl, I, I, L]),
    "aether_op_paged_attention_flex_devarg_f32_cuda": (I, [L, L, L, L, L, I, I, I, I, I, Fl, I, L]),
    "aether_op_paged_attention_mla_devarg_f32_cuda": (I, [L, L, L, L, L, I, I, I, I, Fl, I, L]),
    "aether_op_batched_paged_append_kv_seqB_devarg_f32_cuda": (I, [L, L, L, L, L, I, I, I, I, L]),
    "aether_op_batched_paged_append_kv_hetero_devarg_f32_cuda": (I, [L, L, L, L, L, I, I, I, I, L]),
    "aether_op_batched_paged_attention_seqB_devarg_f32_cuda": (I, [L, L, L, L, L, I, I, I, I, I, I, Fl, I, L]),
    "aether_op_batched_paged_attention_hetero_devarg_f32_cuda": (I, [L, L, L, L, L, I, I, I, I, I, I, Fl, I, L]),
    "aether_op_bert_self_attention_fwd_f32_cuda": (I, [L, L, L, L, I, I, I, Fl]),
    "aether_op_bert_embed_sum_f32_cuda": (I, [L, L, L, L, L, L, I, I]),
    "aether_op_dinov3_rope2d_f32_cuda": (I, [L, L, L, I, I, I, I, I]),
    "aether_op_mla_split_kv_a_f32_cuda": (I, [L, L, L, I, I]),
    "aether_op_mla_assemble_k_f32_cuda": (I, [L, L, L, I, I, I, I]),
    "aether_op_mla_extract_v_f32_cuda": (I, [L, L, I, I, I]),
    "aether_op_mla_broadcast_kv_for_mqa_f32_cuda": (I, [L, L, L, L, I, I, I]),
    "aether_op_mla_rope_q_partial_f32_cuda": (I, [L, I, I, I, Fl, L]),
    "aether_op_mla_rope_k_shared_f32_cuda": (I, [L, I, Fl, L]),
    "aether_op_mla_rope_q_partial_yarn_f32_cuda": (I, [L, I, I, I, Fl, Fl, Fl, Fl, Fl, L]),
    "aether_op_mla_rope_k_shared_yarn_f32_cuda": (I, [L, I, Fl, Fl, Fl, Fl, Fl, L]),
    "aether_op_quantize_q8_1_llama_cuda": (I, [L, L, L, L, I]),
    "aether_op_mmvq_q4k_q8_1_single_cuda": (I, [L, L, L, L, I, I]),
    "aether_op_mmvq_q6k_q8_1_single_cuda": (I, [L, L, L, L, I, I]),
    "aether_op_mmvq_q4k_q8_1_swiglu_cuda": (I, [L, L, L, L, L, I, I]),
    "aether_op_fused_q4k_membw_probe_cuda": (I, [L, L, L, I, I]),
    "aether_llm_inference_bench_tps_cuda": (Fl, [I, I, I, I, I]),
    "aether_llm_inference_bench_tps_cuda_resident": (Fl, [I, I, I, I, I]),
})
for _v in ("", "_v2", "_v3"):
    SIGNATURES[f"aether_op_paged_attention_seq1{_v}_devarg_f32_cuda"] = (I, [L, L, L, L, L, I, I, I, I, Fl, I, L])
for _n in ("q8_0", "q4_k", "q5_k", "q6_k", "iq4_nl", "f16"):
    SIGNATURES[f"aether_op_mla_absorb_q_{_n}_cuda"] = (I, [L, L, L, I, I, I, I, I])
    SIGNATURES[f"aether_op_mla_absorb_v_{_n}_cuda"] = (I, [L, L, L, I, I, I, I])
for _n in ("q4k_matmul_seqB_v3", "q4k_matmul_seqB_fp16", "q6k_matmul_seqB_v3", "q6k_matmul_seqB_fp16"):
    SIGNATURES[f"aether_op_fused_{_n}_cuda"] = (I, [L, L, L, I, I, I])


def lib():
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `make -C csrc/rt`")
        lb = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            f = getattr(lb, name)
            f.restype, f.argtypes = res, args
        _LIB = lb
    return _LIB


def last_error() -> str:
    return (lib().aether_dev_last_error() or b"").decode()


class Dev:
    """A thin host-side wrapper: numpy in / out, handles everywhere else."""

    def __init__(self, device: int | None = None):
        self.lib = lib()
        rc = self.lib.aether_dev_init() if device is None else self.lib.aether_dev_set_device(device)
        if rc != 0:
            raise RuntimeError(f"aether_dev_init failed ({rc}): {last_error()}")

    def call(self, name: str, *args):
        rc = getattr(self.lib, name)(*args)
        if isinstance(rc, int) and rc != 0:
            raise RuntimeError(f"{name} returned {rc}: {last_error()}")
        return rc

    def alloc_f32(self, n: int) -> int:
        h = self.lib.aether_dev_alloc_f32(int(n))
        if not h:
            raise MemoryError(last_error())
        return h

    def alloc_i32(self, n: int) -> int:
        h = self.lib.aether_dev_alloc_i32(int(n))
        if not h:
            raise MemoryError(last_error())
        return h

    def alloc_u8(self, n: int) -> int:
        h = self.lib.aether_dev_alloc_u8(int(n))
        if not h:
            raise MemoryError(last_error())
        return h

    def upload(self, a: np.ndarray) -> int:
        a = np.ascontiguousarray(a)
        if a.dtype == np.float32:
            h = self.alloc_f32(a.size)
            self.call("aether_dev_h2d_f32", a.ctypes.data, h, a.size)
        elif a.dtype == np.int32:
            h = self.alloc_i32(a.size)
            self.call("aether_dev_h2d_i32", a.ctypes.data, h, a.size)
        elif a.dtype == np.uint8:
            h = self.alloc_u8(a.size)
            self.call("aether_dev_h2d_u8", a.ctypes.data, h, a.size)
        else:
            raise TypeError(a.dtype)
        return h

    def download(self, h: int, shape, dtype=np.float32) -> np.ndarray:
        out = np.empty(shape, dtype)
        fn = {np.dtype(np.float32): "aether_dev_d2h_f32", np.dtype(np.int32): "aether_dev_d2h_i32",
              np.dtype(np.uint8): "aether_dev_d2h_u8"}[np.dtype(dtype)]
        self.call(fn, h, out.ctypes.data, out.size)
        return out

    def free(self, h: int, kind: str = "f32") -> None:
        getattr(self.lib, f"aether_dev_free_{kind}")(h)
