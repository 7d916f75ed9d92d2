"""ctypes bindings to ``libaether_rt.so`` -- the C ABI that compiled Aether
programs link against (CPU op bodies, autodiff tape, AetherLM-Nano trainer,
checkpoint I/O, serving structures, observability).

    from aether_b200 import runtime as rt
    rt.call("aether_op_matmul_f32", rt.ptr(a), rt.ptr(b), rt.ptr(c), m, k, n)
    nano = rt.Nano(vocab=256, d_model=64, n_layers=2, n_heads=4, d_ff=128, seq_len=32, seed=42)

Argument and return types come from ``SIGNATURES`` (floats must be declared
for ctypes to pass them correctly); functions not listed default to int
arguments and an int result.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

_PKG = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(_PKG, "libaether_rt.so")
_LIB = None

P, I, L, Fl, U64 = C.c_void_p, C.c_int, C.c_int64, C.c_float, C.c_uint64

SIGNATURES = {
    # core ops
    "aether_op_matmul_f32": (I, [P, P, P, I, I, I]),
    # developer tooling, host communicator, autotune, audio
    "aether_hot_reload_arm": (I, [P, L]),
    "aether_hot_reload_check": (I, [P, L]),
    "aether_sbom_reset": (I, []),
    "aether_sbom_add": (I, [P, L, P, L]),
    "aether_sbom_count": (L, []),
    "aether_sbom_emit": (I, [P, L]),
    "aether_autotune_matmul_tile_f32": (L, [L, L, L]),
    "aether_autotune_unpack_tile_m": (L, [L]),
    "aether_autotune_unpack_tile_n": (L, [L]),
    "aether_autotune_unpack_tile_k": (L, [L]),
    "aether_autotune_unpack_unroll": (L, [L]),
    "aether_cov_record": (I, [L, L]),
    "aether_cov_hits": (L, [L, L]),
    "aether_cov_reset": (I, []),
    "aether_cov_dump": (I, []),
    "aether_pgo_record_branch": (I, [L, L]),
    "aether_pgo_record_call": (I, [L]),
    "aether_pgo_branch_freq": (Fl, [L]),
    "aether_pgo_call_count": (L, [L]),
    "aether_pgo_reset": (I, []),
    "aether_prefetch_t0": (I, [L]),
    "aether_nccl_init": (I, []),
    "aether_nccl_init_count": (I, []),
    "aether_nccl_finalize": (I, []),
    "aether_nccl_comm_create": (L, [I, I]),
    "aether_nccl_comm_destroy": (I, [L]),
    "aether_nccl_comm_world_size": (I, [L]),
    "aether_nccl_comm_rank": (I, [L]),
    "aether_nccl_all_reduce_f32": (I, [P, P, I, I, L]),
    "aether_llm_inference_bench_tps": (Fl, [I, I, I, I, I]),
    "aether_print_bench": (I, [L, I, I, I, I, L]),
    "aether_img_normalize_f32": (I, [P, P, I, Fl, Fl]),
    "aether_img_patchify_f32": (I, [P, P, I, I, I]),
    "aether_audio_hann_window": (I, [P, I]),
    "aether_audio_dft_magnitude_f32": (I, [P, I, P, I]),
    # chat templates and tool calls
    "aether_template_new": (L, []),
    "aether_template_free": (I, [L]),
    "aether_template_set_var": (I, [L, P, I, P, I]),
    "aether_template_push_message": (I, [L, P, I, P, I]),
    "aether_template_render": (I, [L, P, I, P, I]),
    "aether_template_render_from_file": (I, [L, L, I, P, I]),
    "aether_tool_render_call": (I, [P, I, P, I, P, I]),
    # distributed layout arithmetic
    "aether_tp_simulate_column_parallel_linear_f32": (I, [P, P, P, I, I, I, I]),
    "aether_pp_simulate_2stage_forward_f32": (I, [P, P, P, P, I, I, I, I]),
    "aether_zero_simulate_stage_bytes_f32": (L, [I, I, I]),
    "aether_overlap_simulate_overlapped_us": (I, [I, I]),
    "aether_overlap_simulate_serial_us": (I, [I, I]),
    "aether_grad_compress_lowrank_f32": (I, [P, P, I, I, I]),
    "aether_fsdp_simulate_shard_alltoall_f32": (I, [P, P, I, I]),
    "aether_op_softmax_f32": (I, [P, I, I, I]),
    "aether_op_layer_norm_f32": (I, [P, P, P, Fl, P, P, P, I, I]),
    "aether_op_cross_entropy_f32": (Fl, [P, P, P, I, I]),
    "aether_op_adamw_step_f32": (I, [P, P, P, P, Fl, Fl, Fl, Fl, Fl, L, I]),
    "aether_op_clip_grad_norm_f32": (Fl, [P, Fl, I]),
    "aether_rt_self_check": (I, []),
    "aether_alloc_f32": (L, [I]),
    "aether_free": (None, [L]),
    # extended ops
    "aether_op_pow_f32": (I, [P, Fl, I]),
    "aether_op_clamp_f32": (I, [P, Fl, Fl, I]),
    "aether_op_sum_f32": (Fl, [P, I]),
    "aether_op_mean_f32": (Fl, [P, I]),
    "aether_op_var_f32": (Fl, [P, I]),
    "aether_op_std_f32": (Fl, [P, I]),
    "aether_op_argmax_f32": (L, [P, I]),
    "aether_op_lion_step_f32": (I, [P, P, P, I, Fl, Fl, Fl, Fl]),
    "aether_op_lamb_step_f32": (I, [P, P, P, P, I, Fl, Fl, Fl, Fl, Fl, Fl, Fl]),
    "aether_op_adafactor_step_f32": (I, [P, P, P, P, I, I, Fl, Fl, Fl]),
    "aether_op_sgd_momentum_step_f32": (I, [P, P, P, Fl, Fl, Fl, I]),
    "aether_op_rmsprop_step_f32": (I, [P, P, P, Fl, Fl, Fl, I]),
    "aether_op_adagrad_step_f32": (I, [P, P, P, Fl, Fl, I]),
    "aether_op_max_pool_2d_f32": (I, [P, P] + [I] * 10),
    "aether_op_avg_pool_2d_f32": (I, [P, P] + [I] * 10),
    "aether_op_adaptive_avg_pool_2d_f32": (I, [P, P] + [I] * 6),
    "aether_op_embedding_bag_f32": (I, [P, P, P, P, I, I, I, I, I]),
    "aether_op_masked_fill_f32": (I, [P, P, Fl, I]),
    "aether_op_mish_backward_f32": (I, [P, P, I]),
    # dtype conversions and dequantisers
    "aether_f32_to_bf16": (I, [Fl]),
    "aether_bf16_to_f32": (Fl, [I]),
    "aether_f32_to_f16": (I, [Fl]),
    "aether_f16_to_f32": (Fl, [I]),
    "aether_op_matmul_bf16_f32_out": (I, [L, L, L, I, I, I]),
    "aether_pack_f32_to_bf16": (I, [L, L, I]),
    "aether_dequant_q4_0": (I, [P, P, I]),
    "aether_dequant_q8_0": (I, [P, P, I]),
    "aether_dequant_q4_k_m": (I, [P, P, I]),
    "aether_dequant_q6_k": (I, [P, P, I]),
    "aether_dequant_q3_k": (I, [P, P, I]),
    # serving structures
    "aether_pkv_new": (L, [I, I]),
    "aether_pkv_destroy": (I, [L]),
    "aether_pkv_allocate": (I, [L]),
    "aether_pkv_touch": (I, [L, I]),
    "aether_pkv_free_block": (I, [L, I]),
    "aether_pkv_evict_lru": (I, [L]),
    "aether_pkv_n_allocated": (I, [L]),
    "aether_pkv_pagetable_new": (L, [I]),
    "aether_pkv_pagetable_set": (I, [L, I, I]),
    "aether_pkv_pagetable_get": (L, [L, I]),
    "aether_pkv_pagetable_translate": (L, [L, I, I]),
    "aether_batch_sched_new": (L, [L, I, I]),
    "aether_batch_sched_destroy": (L, [L]),
    "aether_batch_sched_admit": (L, [L, I, I, I]),
    "aether_batch_sched_record_token": (L, [L, I, I]),
    "aether_batch_sched_finish": (L, [L, I]),
    "aether_batch_sched_reap": (L, [L]),
    "aether_batch_sched_n_active": (L, [L]),
    "aether_batch_sched_position": (L, [L, I]),
    "aether_batch_sched_pagetable_for": (L, [L, I]),
    "aether_cb_new": (L, [I]),
    "aether_cb_admit": (I, [L, I]),
    "aether_cb_step": (I, [L]),
    "aether_cb_complete": (I, [L, I]),
    "aether_cb_n_active": (I, [L]),
    "aether_specdec_accept": (I, [Fl, Fl, Fl]),
    "aether_mm_new": (L, []),
    "aether_mm_register": (I, [L, P, I, I]),
    "aether_mm_lookup": (I, [L, P, I]),
    "aether_mm_total_vram_mb": (I, [L]),
    "aether_rl_new": (L, [I, I]),
    "aether_rl_check": (I, [L, P, I, L]),
    # observability
    "aether_obs_counter_inc": (I, [P, I, I]),
    "aether_obs_counter_get": (L, [P, I]),
    "aether_obs_dump_prometheus": (I, [P, I]),
    "aether_crash_dump": (I, [P, L, L]),
    "aether_gpu_alloc_track": (L, [L]),
    "aether_gpu_free_track": (L, [L]),
    "aether_gpu_live_bytes": (L, []),
    "aether_oom_signal": (L, [L]),
    "aether_oom_check": (L, []),
    "aether_prof_alloc_total": (L, []),
    "aether_prof_alloc_live": (L, []),
    "aether_prof_alloc_peak": (L, []),
    "aether_prof_reset": (I, []),
    "aether_timer_start": (L, []),
    "aether_timer_elapsed_us": (L, [L]),
    # scalar helpers, extra losses, witnesses, GGUF reader (float arguments / results)
    "aether_init_normal_f32": (I, [P, I, Fl, L]),
    "aether_fill_labels_i32": (I, [P, I, I, L]),
    "aether_fill_f32": (None, [P, I, Fl]),
    "aether_init_constant_f32": (None, [P, I, Fl]),
    "aether_abs_f32": (Fl, [Fl]),
    "aether_cos_f32": (Fl, [Fl]),
    "aether_sin_f32": (Fl, [Fl]),
    "aether_exp_f32": (Fl, [Fl]),
    "aether_log_f32": (Fl, [Fl]),
    "aether_sqrt_f32": (Fl, [Fl]),
    "aether_max_f32": (Fl, [Fl, Fl]),
    "aether_min_f32": (Fl, [Fl, Fl]),
    "aether_max_i64": (L, [L, L]),
    "aether_min_i64": (L, [L, L]),
    "aether_abs_i64": (L, [L]),
    "aether_sum_f32": (Fl, [P, I]),
    "aether_dot_f32_scalar": (Fl, [P, P, L]),
    "aether_op_bce_f32": (Fl, [P, P, I]),
    "aether_op_bce_backward_f32": (I, [P, P, P, I]),
    "aether_op_kl_div_f32": (Fl, [P, P, I]),
    "aether_op_kl_div_backward_f32": (I, [P, P, P, I]),
    "aether_op_contrastive_f32": (Fl, [P, P, Fl, I, Fl]),
    "aether_op_contrastive_backward_f32": (I, [P, P, P, Fl, I, Fl]),
    "aether_op_smooth_l1_f32": (Fl, [P, P, I, Fl]),
    "aether_op_smooth_l1_backward_f32": (I, [P, P, P, I, Fl]),
    "aether_op_triplet_f32": (Fl, [P, P, P, I, Fl]),
    "aether_op_triplet_backward_f32": (I, [P, P, P, P, I, Fl]),
    "aether_op_matmul_bf16": (I, [P, P, P, I, I, I]),
    "aether_print_loss": (I, [I, Fl]),
    "aether_print_f32_default": (I, [Fl]),
    "aether_print_kv_f32": (I, [C.c_char_p, Fl]),
    "aether_print_kv_i64": (I, [C.c_char_p, L]),
    "aether_f32_close_exit": (I, [Fl, Fl]),
    "aether_f32_in_band_exit": (I, [Fl, Fl, Fl]),
    "aether_bpe_tokenizer_new": (L, []),
    "aether_bpe_tokenizer_free": (I, [L]),
    "aether_bpe_add_token_with_id": (I, [L, I, P, I]),
    "aether_bpe_add_merge": (I, [L, I, I, I, P, I]),
    "aether_bpe_add_merge_by_id": (I, [L, I, I, I, I]),
    "aether_bpe_encode": (I, [L, P, I, P, I]),
    "aether_bpe_encode_ids": (I, [L, P, I, P, I]),
    "aether_bpe_decode": (I, [L, P, I, P, I]),
    "aether_bpe_lookup_bytes": (I, [L, P, I]),
    "aether_tokenizer_json_load": (I, [L, P, I]),
    "aether_safetensors_n_tensors": (I, [P, L]),
    "aether_safetensors_get_dtype": (I, [P, L, P, L]),
    "aether_safetensors_get_shape": (I, [P, L, P, L, P, I]),
    "aether_gguf_open": (L, [P, I]),
    "aether_gguf_close": (I, [L]),
    "aether_gguf_version": (I, [L]),
    "aether_gguf_n_tensors": (I, [L]),
    "aether_gguf_get_tensor_name": (I, [L, I, P, I]),
    "aether_gguf_get_tensor_dtype": (I, [L, I]),
    "aether_gguf_get_tensor_shape": (I, [L, I, P, I]),
    "aether_gguf_get_tensor_abs_offset": (L, [L, I]),
    "aether_gguf_get_tensor_data_ptr": (L, [L, I]),
    "aether_gguf_find_tensor_by_name": (I, [L, P, I]),
    "aether_gguf_get_tensor_n_elems": (L, [L, I]),
    "aether_gguf_get_metadata_u32": (L, [L, P, I]),
    "aether_gguf_get_metadata_bool": (L, [L, P, I]),
    "aether_gguf_get_metadata_f32": (C.c_double, [L, P, I]),
    "aether_gguf_get_metadata_string": (I, [L, P, I, P, I]),
    "aether_gguf_get_metadata_array_string_n": (I, [L, P, I]),
    "aether_gguf_get_metadata_array_string_get": (I, [L, P, I, I, P, I]),
    "aether_gguf_get_metadata_array_f32_n": (I, [L, P, I]),
    "aether_gguf_get_metadata_array_f32": (I, [L, P, I, P, I]),
    # crypto and wire codecs
    "aether_sha256": (I, [P, I, P]),
    "aether_sha512": (I, [P, I, P]),
    "aether_hmac_sha256": (I, [P, I, P, I, P]),
    "aether_hkdf_extract": (I, [P, I, P, I, P]),
    "aether_hkdf_expand": (I, [P, I, P, I, P, I]),
    "aether_tls13_hkdf_expand_label": (I, [P, I, P, I, P, I, P, I]),
    "aether_chacha20_poly1305_encrypt": (I, [P, P, P, I, P, I, P, I]),
    "aether_chacha20_poly1305_decrypt": (I, [P, P, P, I, P, I, P, I]),
    "aether_x25519_derive_public": (I, [P, P]),
    "aether_x25519_shared_secret": (I, [P, P, P]),
    "aether_ed25519_derive_public": (I, [P, P]),
    "aether_ed25519_sign": (I, [P, P, P, I, P]),
    "aether_ed25519_verify": (I, [P, P, I, P]),
    "aether_random_bytes": (I, [P, I]),
    "aether_ws_encode_text_frame": (I, [P, I, P, I]),
    "aether_ws_decode_frame_payload": (I, [P, I, P, I]),
    "aether_http_parse_request": (I, [P, I, P, I, C.POINTER(C.c_int), C.POINTER(C.c_int)]),
    "aether_http_write_response_200": (I, [P, I, P, I]),
    "aether_openai_render_completion": (I, [P, I, P, I, P, I, I, I, P, I]),
    # TLS 1.3 sessions
    "aether_tls13_server_new": (L, [P, P, P, P, I, P, I]),
    "aether_tls13_client_new": (L, [P, P, P, I]),
    "aether_tls13_self_loopback_smoke": (I, []),
    # AetherLM-Nano
    "aether_nano_create": (P, [I, I, I, I, I, I, U64]),
    "aether_nano_destroy": (None, [P]),
    "aether_nano_num_params": (L, [P]),
    "aether_nano_params": (C.POINTER(C.c_float), [P]),
    "aether_nano_train_step": (Fl, [P, P, P, I, Fl, Fl, Fl, L]),
    "aether_nano_loss": (Fl, [P, P, P, I]),
    "aether_nano_generate": (I, [P, P, I, I, P]),
    "aether_nano_synthetic_corpus": (L, [P, L, U64, I]),
    "aether_nano_pattern_corpus": (L, [P, L]),
    "aether_nano_sample_batch": (None, [P, L, I, I, P, P, P]),
    "aether_nano_cosine_lr": (Fl, [I, I, Fl, I]),
    "aether_nano_save": (I, [P, C.c_char_p]),
    "aether_nano_load_weights": (I, [P, C.c_char_p]),
}


def lib():
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            from .._build import build_runtime

            build_runtime()  # plain g++ / make: seconds, no GPU needed
        _LIB = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(_LIB, name)
            fn.restype, fn.argtypes = res, args
    return _LIB


def call(name: str, *args):
    return getattr(lib(), name)(*args)


def ptr(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(C.c_void_p)


class Nano:
    """AetherLM-Nano on the native CPU trainer (reference trainer/src/model.rs)."""

    def __init__(self, vocab=256, d_model=64, n_layers=2, n_heads=4, d_ff=128, seq_len=32, seed=42):
        self.seq_len = seq_len
        self.step = 0
        self.h = call("aether_nano_create", vocab, d_model, n_layers, n_heads, d_ff, seq_len, seed)

    def __del__(self):
        if getattr(self, "h", None) and _LIB is not None:
            try:
                _LIB.aether_nano_destroy(self.h)
            except Exception:  # noqa: BLE001 -- interpreter shutdown
                pass
            self.h = None

    @property
    def n_params(self) -> int:
        return int(call("aether_nano_num_params", self.h))

    def params(self) -> np.ndarray:
        return np.ctypeslib.as_array(call("aether_nano_params", self.h), shape=(self.n_params,)).copy()

    def train_step(self, ids: np.ndarray, labels: np.ndarray, lr: float, wd: float = 0.0, clip: float = 1.0) -> float:
        B = ids.shape[0]
        self.step += 1
        return float(call("aether_nano_train_step", self.h, ptr(ids), ptr(labels), B, lr, wd, clip, self.step))

    def loss(self, ids, labels) -> float:
        return float(call("aether_nano_loss", self.h, ptr(ids), ptr(labels), ids.shape[0]))

    def generate(self, prompt, max_new: int) -> list:
        p = np.asarray(prompt, dtype=np.int32)
        out = np.zeros(max_new, dtype=np.int32)
        n = call("aether_nano_generate", self.h, ptr(p), len(p), max_new, ptr(out))
        return out[:n].tolist()

    def save(self, stem: str) -> int:
        return int(call("aether_nano_save", self.h, stem.encode()))

    def load(self, path: str) -> int:
        return int(call("aether_nano_load_weights", self.h, path.encode()))


def synthetic_corpus(n_bytes: int, seed: int = 42, n_words: int = 200) -> np.ndarray:
    buf = np.zeros(n_bytes, dtype=np.uint8)
    n = call("aether_nano_synthetic_corpus", ptr(buf), n_bytes, seed, n_words)
    return buf[:n]


def pattern_corpus(n_bytes: int) -> np.ndarray:
    """The reference trainer's default smoke corpus (one sentence repeated)."""
    buf = np.zeros(n_bytes, dtype=np.uint8)
    call("aether_nano_pattern_corpus", ptr(buf), n_bytes)
    return buf


def sample_batch(data: np.ndarray, B: int, S: int, rng_state: np.ndarray):
    ids = np.zeros((B, S), dtype=np.int32)
    labels = np.zeros((B, S), dtype=np.int32)
    call("aether_nano_sample_batch", ptr(data), data.size, B, S, ptr(rng_state), ptr(ids), ptr(labels))
    return ids, labels


def render_template(template: str, messages, variables=None, max_out: int = 1 << 20) -> str:
    """Render a chat template (the native Jinja subset) over (role, content) messages."""
    h = call("aether_template_new")
    try:
        for k, v in (variables or {}).items():
            kb, vb = k.encode(), str(v).encode()
            if call("aether_template_set_var", h, kb, len(kb), vb, len(vb)) != 0:
                raise ValueError(f"bad variable {k!r}")
        for role, content in messages:
            rb, cb = role.encode(), content.encode()
            if call("aether_template_push_message", h, rb, len(rb), cb, len(cb)) != 0:
                raise ValueError("bad message")
        tb = template.encode()
        out = C.create_string_buffer(max_out)
        n = call("aether_template_render", h, tb, len(tb), out, max_out)
        if n < 0:
            raise ValueError("template render failed (malformed template or output too large)")
        return out.raw[:n].decode()
    finally:
        call("aether_template_free", h)


def render_tool_call(name: str, arguments: str, max_out: int = 1 << 16) -> str:
    nb, ab = name.encode(), arguments.encode()
    out = C.create_string_buffer(max_out)
    n = call("aether_tool_render_call", nb, len(nb), ab, len(ab), out, max_out)
    if n < 0:
        raise ValueError("tool call render failed")
    return out.raw[:n].decode()
