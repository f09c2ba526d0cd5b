"""ctypes binding of libiris_cuda.so (the C ABI declared in include/iris_cuda.h).

Used by the tests, bench.py and __graft_entry__.py.  It loads the in-tree
library built by ``make -C iris.c_b200 cuda`` and fails loudly when it is
missing: there is no CPU or framework fallback behind these calls.
"""
from __future__ import annotations

import ctypes as C
import os
import weakref

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libiris_cuda.so")

OK = 0
ERR_ARG, ERR_OOM, ERR_CUDA, ERR_IO, ERR_TIMEOUT, ERR_NODEV, ERR_INJECTED = -1, -2, -3, -4, -5, -6, -7

_fp = C.POINTER(C.c_float)
_u16p = C.POINTER(C.c_uint16)


class FluxConfig(C.Structure):
    _fields_ = [("hidden", C.c_int), ("heads", C.c_int), ("head_dim", C.c_int), ("mlp", C.c_int),
                ("n_double", C.c_int), ("n_single", C.c_int), ("text_dim", C.c_int),
                ("channels", C.c_int), ("rope_theta", C.c_float)]

    @classmethod
    def from_hf(cls, cfg: dict) -> "FluxConfig":
        h = cfg["num_attention_heads"] * cfg["attention_head_dim"]
        return cls(hidden=h, heads=cfg["num_attention_heads"], head_dim=cfg["attention_head_dim"],
                   mlp=int(h * cfg.get("mlp_ratio", 3.0)), n_double=cfg["num_layers"],
                   n_single=cfg["num_single_layers"], text_dim=cfg["joint_attention_dim"],
                   channels=cfg["in_channels"], rope_theta=float(cfg.get("rope_theta", 2000.0)))


class KernelTime(C.Structure):
    _fields_ = [("name", C.c_char * 32), ("flops", C.c_double), ("bytes", C.c_double), ("ms", C.c_float)]


class ZImageConfig(C.Structure):
    _fields_ = [("dim", C.c_int), ("heads", C.c_int), ("n_layers", C.c_int), ("n_refiner", C.c_int),
                ("cap_feat_dim", C.c_int), ("in_channels", C.c_int), ("patch_size", C.c_int),
                ("ffn_dim", C.c_int), ("adaln_dim", C.c_int), ("t_mid", C.c_int), ("rope_theta", C.c_float),
                ("axes_dims", C.c_int * 3)]

    @classmethod
    def from_dict(cls, c: dict) -> "ZImageConfig":
        return cls(dim=c["dim"], heads=c["dim"] // 128, n_layers=c["n_layers"], n_refiner=c["n_refiner"],
                   cap_feat_dim=c["cap_feat_dim"], in_channels=c["in_channels"], patch_size=c["patch_size"],
                   ffn_dim=c["ffn_dim"], adaln_dim=min(c["dim"], 256), t_mid=c["t_mid"],
                   rope_theta=float(c["rope_theta"]), axes_dims=(C.c_int * 3)(*c["axes_dims"]))


class Qwen3Config(C.Structure):
    """iris_cuda_qwen3_config_t."""
    _fields_ = [("hidden", C.c_int), ("intermediate", C.c_int), ("heads", C.c_int), ("kv_heads", C.c_int),
                ("head_dim", C.c_int), ("vocab", C.c_int), ("layers", C.c_int), ("rope_theta", C.c_float)]

    @classmethod
    def from_hf(cls, c: dict) -> "Qwen3Config":
        return cls(c["hidden_size"], c["intermediate_size"], c["num_attention_heads"], c["num_key_value_heads"],
                   c.get("head_dim", 128), c["vocab_size"], c["num_hidden_layers"], c.get("rope_theta", 1e6))


class Image(C.Structure):
    """iris_cuda_image_t (the reference's iris_image layout, iris.h:73-78)."""
    _fields_ = [("width", C.c_int), ("height", C.c_int), ("channels", C.c_int),
                ("data", C.POINTER(C.c_uint8))]


class Ref(C.Structure):
    _fields_ = [("latent", _fp), ("h", C.c_int), ("w", C.c_int), ("t_offset", C.c_int)]


PROGRESS_CB = C.CFUNCTYPE(None, C.c_int, C.c_int)

# name -> (restype, argtypes) for every exported entry point of include/iris_cuda.h
SIGNATURES = {
    "iris_cuda_init": (C.c_int, [C.c_int]),
    "iris_cuda_available": (C.c_int, []),
    "iris_cuda_cleanup": (None, []),
    "iris_cuda_last_error": (C.c_char_p, []),
    "iris_cuda_device_status": (C.c_int, [C.c_int]),
    "iris_cuda_synchronize": (C.c_int, []),
    "iris_cuda_stream": (C.c_void_p, []),
    "iris_cuda_kernel_launches": (C.c_uint64, []),
    "iris_cuda_selftest_wait_timeout": (C.c_int, []),
    "iris_cuda_flux_load": (C.c_void_p, [C.c_char_p]),
    "iris_cuda_flux_random": (C.c_void_p, [C.POINTER(FluxConfig), C.c_uint64, C.c_float, C.c_int]),
    "iris_cuda_flux_load_tp": (C.c_void_p, [C.c_char_p, C.c_int, C.c_int]),
    "iris_cuda_flux_random_tp": (C.c_void_p, [C.POINTER(FluxConfig), C.c_uint64, C.c_float, C.c_int,
                                              C.c_int, C.c_int]),
    "iris_cuda_flux_free": (None, [C.c_void_p]),
    "iris_cuda_flux_get_config": (C.c_int, [C.c_void_p, C.POINTER(FluxConfig)]),
    "iris_cuda_flux_read_weight": (C.c_int, [C.c_void_p, C.c_char_p, _u16p, C.c_size_t]),
    "iris_cuda_flux_weight_bytes": (C.c_size_t, [C.c_void_p]),
    "iris_cuda_flux_load_lora": (C.c_int, [C.c_void_p, C.c_char_p, C.c_float]),
    "iris_cuda_flux_unload_lora": (C.c_int, [C.c_void_p]),
    "iris_cuda_flux_lora_adapters": (C.c_int, [C.c_void_p]),
    "iris_cuda_flux_lora_stats": (C.c_int, [C.c_void_p, C.POINTER(C.c_double), C.POINTER(C.c_double)]),
    "iris_cuda_lora_probe": (C.c_int, [C.c_char_p, C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(C.c_int)]),
    "iris_cuda_flux_load_ip_adapter": (C.c_int, [C.c_void_p, C.c_char_p, C.c_char_p, C.c_float]),
    "iris_cuda_flux_load_ip_adapter_mem": (C.c_int, [C.c_void_p, C.c_char_p, _fp, C.c_int, C.c_float]),
    "iris_cuda_flux_unload_ip_adapter": (C.c_int, [C.c_void_p]),
    "iris_cuda_flux_set_ip_schedule": (C.c_int, [C.c_void_p, C.c_char_p]),
    "iris_cuda_flux_set_ip_step": (C.c_int, [C.c_void_p, C.c_int, C.c_int]),
    "iris_cuda_flux_ip_embeds": (C.c_int, [C.c_void_p, _fp, C.c_int]),
    "iris_cuda_flux_set_sref_csd": (C.c_int, [C.c_void_p, C.c_char_p, _fp, C.c_int, C.c_float]),
    "iris_cuda_flux_set_csd_delta": (C.c_int, [C.c_void_p, _fp]),
    "iris_cuda_flux_set_csd_skip": (C.c_int, [C.c_void_p, C.c_int]),
    "iris_cuda_flux_set_sref_bands": (C.c_int, [C.c_void_p, C.c_float, C.c_float]),
    "iris_cuda_transformer_forward": (C.c_void_p, [C.c_void_p, _fp, C.c_int, C.c_int, _fp, C.c_int,
                                                   C.c_float]),
    "iris_cuda_transformer_forward_with_multi_refs": (C.c_void_p, [C.c_void_p, _fp, C.c_int, C.c_int,
                                                                   C.POINTER(Ref), C.c_int, _fp,
                                                                   C.c_int, C.c_float]),
    "iris_cuda_flux_forward_dev": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int,
                                             C.POINTER(Ref), C.c_int, C.c_void_p, C.c_int,
                                             C.c_float, C.c_void_p]),
    "iris_cuda_flux_run_block": (C.c_int, [C.c_void_p, C.c_int, C.c_int, _fp, C.c_int, C.c_int,
                                           C.c_int, C.c_float]),
    "iris_cuda_flux_profile": (C.c_int, [C.c_void_p, C.c_float, C.POINTER(KernelTime), C.c_int]),
    "iris_cuda_official_schedule": (C.c_void_p, [C.c_int, C.c_int]),
    "iris_cuda_linear_schedule": (C.c_void_p, [C.c_int]),
    "iris_cuda_zimage_schedule": (C.c_void_p, [C.c_int, C.c_int]),
    "iris_cuda_init_noise": (C.c_void_p, [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int64]),
    "iris_cuda_sample_euler": (C.c_void_p, [C.c_void_p, _fp, C.c_int, C.c_int, C.c_int, C.c_int,
                                            _fp, C.c_int, _fp, C.c_int, PROGRESS_CB]),
    "iris_cuda_sample_euler_cfg": (C.c_void_p, [C.c_void_p, _fp, C.c_int, C.c_int, C.c_int, C.c_int,
                                                _fp, C.c_int, _fp, C.c_int, C.c_float, _fp, C.c_int,
                                                PROGRESS_CB]),
    "iris_cuda_sample_euler_with_multi_refs": (C.c_void_p, [C.c_void_p, _fp, C.c_int, C.c_int,
                                                            C.c_int, C.c_int, C.POINTER(Ref), C.c_int,
                                                            _fp, C.c_int, _fp, C.c_int, PROGRESS_CB]),
    "iris_cuda_sample_euler_dev": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p,
                                             C.c_int, C.c_void_p, C.c_int, C.c_float, _fp, C.c_int]),
    "iris_cuda_comm_unique_id": (C.c_int, [C.c_void_p, C.c_size_t]),
    "iris_cuda_comm_init": (C.c_int, [C.c_void_p, C.c_int, C.c_int]),
    "iris_cuda_comm_destroy": (None, []),
    "iris_cuda_comm_world": (C.c_int, []),
    "iris_cuda_comm_rank": (C.c_int, []),
    "iris_cuda_sample_euler_cfg_pair": (C.c_void_p, [C.c_void_p, _fp, C.c_int, C.c_int, C.c_int, C.c_int,
                                                     _fp, C.c_int, _fp, C.c_int, C.c_float, _fp, C.c_int,
                                                     PROGRESS_CB]),
    "iris_cuda_sample_euler_cfg_pair_dev": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int,
                                                      C.c_void_p, C.c_void_p, C.c_int, C.c_float, _fp,
                                                      C.c_int]),
    "iris_cuda_zimage_load": (C.c_void_p, [C.c_char_p]),
    "iris_cuda_zimage_random": (C.c_void_p, [C.POINTER(ZImageConfig), C.c_uint64, C.c_float, C.c_int]),
    "iris_cuda_zimage_free": (None, [C.c_void_p]),
    "iris_cuda_zimage_get_config": (C.c_int, [C.c_void_p, C.POINTER(ZImageConfig)]),
    "iris_cuda_zimage_weight_bytes": (C.c_size_t, [C.c_void_p]),
    "iris_cuda_zi_transformer_forward": (C.c_void_p, [C.c_void_p, _fp, C.c_int, C.c_int, C.c_float, _fp,
                                                      C.c_int]),
    "iris_cuda_sample_euler_zimage": (C.c_void_p, [C.c_void_p, _fp, C.c_int, C.c_int, C.c_int, C.c_int,
                                                   C.c_int, _fp, C.c_int, _fp, C.c_int, PROGRESS_CB]),
    "iris_cuda_sample_euler_zimage_dev": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p,
                                                    C.c_int, _fp, C.c_int]),
    "iris_cuda_vae_load": (C.c_void_p, [C.c_char_p, C.c_int, C.c_float, C.c_float]),
    "iris_cuda_vae_free": (None, [C.c_void_p]),
    "iris_cuda_vae_weight_bytes": (C.c_size_t, [C.c_void_p]),
    "iris_cuda_vae_decode": (C.c_void_p, [C.c_void_p, _fp, C.c_int, C.c_int, C.c_int]),
    "iris_cuda_image_free": (None, [C.c_void_p]),
    "iris_cuda_vae_decode_f32": (C.c_int, [C.c_void_p, _fp, C.c_int, C.c_int, _fp]),
    "iris_cuda_vae_decode_dev": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p,
                                           C.c_void_p]),
    "iris_cuda_vae_graph_kernels": (C.c_uint64, [C.c_void_p]),
    "iris_cuda_vae_random": (C.c_void_p, [C.c_int, C.c_float, C.c_float, C.c_uint64]),
    "iris_cuda_qwen3_load": (C.c_void_p, [C.c_char_p]),
    "iris_cuda_qwen3_random": (C.c_void_p, [C.POINTER(Qwen3Config), C.c_uint64]),
    "iris_cuda_qwen3_free": (None, [C.c_void_p]),
    "iris_cuda_qwen3_get_config": (C.c_int, [C.c_void_p, C.POINTER(Qwen3Config)]),
    "iris_cuda_qwen3_weight_bytes": (C.c_size_t, [C.c_void_p]),
    "iris_cuda_qwen3_set_extraction_mode": (C.c_int, [C.c_void_p, C.c_int]),
    "iris_cuda_qwen3_text_dim": (C.c_int, [C.c_void_p]),
    "iris_cuda_qwen3_forward": (C.c_void_p, [C.c_void_p, C.POINTER(C.c_int), C.POINTER(C.c_int), C.c_int]),
    "iris_cuda_qwen3_forward_dev": (C.c_int, [C.c_void_p, C.POINTER(C.c_int), C.POINTER(C.c_int), C.c_int,
                                              C.c_void_p]),
    "iris_cuda_qwen3_graph_kernels": (C.c_uint64, [C.c_void_p]),
    "iris_cuda_qwen3_profile": (C.c_int, [C.c_void_p, C.POINTER(KernelTime), C.c_int]),
    "iris_cuda_vae_profile": (C.c_int, [C.c_void_p, C.POINTER(KernelTime), C.c_int]),
    # iris_gpu_* surface (iris_metal.h names)
    "iris_gpu_tensor_create": (C.c_void_p, [_fp, C.c_size_t]),
    "iris_gpu_tensor_alloc": (C.c_void_p, [C.c_size_t]),
    "iris_gpu_tensor_alloc_persistent": (C.c_void_p, [C.c_size_t]),
    "iris_gpu_tensor_set_persistent": (None, [C.c_void_p, C.c_int]),
    "iris_gpu_tensor_read": (None, [C.c_void_p, _fp]),
    "iris_gpu_tensor_write": (None, [C.c_void_p, _fp]),
    "iris_gpu_tensor_free": (None, [C.c_void_p]),
    "iris_gpu_tensor_size": (C.c_size_t, [C.c_void_p]),
    "iris_gpu_tensor_is_f16": (C.c_int, [C.c_void_p]),
    "iris_gpu_tensor_alloc_f16": (C.c_void_p, [C.c_size_t]),
    "iris_gpu_tensor_create_bf16": (C.c_void_p, [_fp, C.c_size_t]),
    "iris_gpu_tensor_f32_to_bf16": (C.c_void_p, [C.c_void_p]),
    "iris_gpu_tensor_bf16_to_f32": (C.c_void_p, [C.c_void_p]),
    "iris_gpu_convert_f32_to_bf16_into": (C.c_int, [C.c_void_p, C.c_void_p]),
    "iris_gpu_convert_bf16_to_f32_into": (C.c_int, [C.c_void_p, C.c_void_p]),
    "iris_gpu_sync": (None, []),
    "iris_gpu_batch_begin": (None, []),
    "iris_gpu_batch_end": (None, []),
    "iris_gpu_linear_bf16_native": (C.c_void_p, [C.c_void_p, _u16p, C.c_int, C.c_int, C.c_int]),
    "iris_gpu_linear_bf16_native_into": (C.c_int, [C.c_void_p, C.c_void_p, _u16p, C.c_int, C.c_int,
                                                   C.c_int]),
    "iris_gpu_adaln_norm_bf16": (None, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int,
                                        C.c_int, C.c_float]),
    "iris_gpu_adaln_norm_bf16_noalloc": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                                   C.c_int, C.c_int, C.c_float, C.c_void_p]),
    "iris_gpu_qk_rms_norm_bf16": (None, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int,
                                         C.c_int, C.c_int, C.c_float]),
    "iris_gpu_rope_unified_bf16": (None, [C.c_void_p, C.c_void_p, _fp, _fp, _fp, _fp, _fp, _fp,
                                          C.c_int, C.c_int, C.c_int, C.c_int, C.c_int]),
    "iris_gpu_rope_2d_bf16": (None, [C.c_void_p, _fp, _fp, C.c_int, C.c_int, C.c_int, C.c_int]),
    "iris_gpu_attention_fused_bf16": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                                C.c_int, C.c_int, C.c_int, C.c_int, C.c_float]),
    "iris_gpu_silu_mul_bf16": (None, [C.c_void_p, C.c_void_p, C.c_int]),
    "iris_gpu_gated_add_bf16": (None, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int]),
    "iris_gpu_concat_seq_bf16": (None, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int,
                                        C.c_int]),
    "iris_gpu_slice_seq_bf16": (None, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int]),
    "iris_gpu_split_qkv_mlp_bf16": (None, [C.c_void_p] * 6 + [C.c_int] * 3),
    "iris_gpu_concat_attn_mlp_bf16": (None, [C.c_void_p] * 3 + [C.c_int] * 3),
    "iris_metal_available": (C.c_int, []),
    "iris_metal_shaders_available": (C.c_int, []),
    "iris_bf16_pipeline_available": (C.c_int, []),
    "iris_gpu_add_bf16": (None, [C.c_void_p] * 3 + [C.c_int]),
    "iris_gpu_copy_bf16": (None, [C.c_void_p, C.c_void_p, C.c_size_t]),
    "iris_gpu_head_rms_norm_bf16": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_float]),
    "iris_gpu_linear_bf16_bf16out": (C.c_void_p, [C.c_void_p, _u16p, C.c_int, C.c_int, C.c_int]),
    "iris_gpu_attention_mps_bf16": (C.c_int, [C.c_void_p] * 4 + [C.c_int] * 4 + [C.c_float]),
    "iris_gpu_attention_bf16_native": (C.c_int, [C.c_void_p] * 4 + [C.c_int] * 4 + [C.c_float]),
    "iris_gpu_tensor_data": (_fp, [C.c_void_p]),
    "iris_gpu_linear": (C.c_void_p, [C.c_void_p, _fp, _fp, C.c_int, C.c_int, C.c_int]),
    "iris_gpu_linear_bf16": (C.c_void_p, [C.c_void_p, _u16p, C.c_int, C.c_int, C.c_int]),
    "iris_gpu_linear_bf16_into": (C.c_int, [C.c_void_p, C.c_void_p, _u16p, C.c_int, C.c_int, C.c_int]),
    "iris_gpu_adaln_norm": (None, [C.c_void_p, C.c_void_p, _fp, _fp, C.c_int, C.c_int, C.c_float]),
    "iris_gpu_rms_norm_f32": (None, [C.c_void_p, C.c_void_p, _fp, C.c_int, C.c_int, C.c_float]),
    "iris_gpu_qk_rms_norm": (None, [C.c_void_p, C.c_void_p, _fp, _fp, C.c_int, C.c_int, C.c_int, C.c_float]),
    "iris_gpu_rope_single_f32": (None, [C.c_void_p, _fp, _fp, C.c_int, C.c_int, C.c_int]),
    "iris_gpu_rope_single_pair_f32": (None, [C.c_void_p, C.c_void_p, _fp, _fp, C.c_int, C.c_int, C.c_int]),
    "iris_gpu_rope_unified": (None, [C.c_void_p, C.c_void_p, _fp, _fp, _fp, _fp] + [C.c_int] * 5),
    "iris_gpu_silu_mul": (None, [C.c_void_p, C.c_void_p, C.c_int]),
    "iris_gpu_gated_add": (None, [C.c_void_p, _fp, C.c_void_p, C.c_int, C.c_int]),
    "iris_gpu_split_qkv_mlp": (None, [C.c_void_p] * 6 + [C.c_int] * 3),
    "iris_gpu_concat_attn_mlp": (None, [C.c_void_p] * 3 + [C.c_int] * 3),
    "iris_gpu_attention_fused": (C.c_int, [C.c_void_p] * 4 + [C.c_int] * 4 + [C.c_float]),
    "iris_gpu_attention_bf16": (C.c_int, [C.c_void_p] * 4 + [C.c_int] * 4 + [C.c_float]),
    "iris_gpu_add_f32": (None, [C.c_void_p] * 3 + [C.c_int]),
    "iris_gpu_copy_f32": (None, [C.c_void_p, C.c_void_p, C.c_size_t]),
    "iris_gpu_copy_region_f32": (None, [C.c_void_p, C.c_size_t, C.c_void_p, C.c_size_t, C.c_size_t]),
    "iris_metal_attention_fused": (C.c_int, [_fp] * 4 + [C.c_int] * 4 + [C.c_float]),
    "iris_metal_attention": (None, [_fp] * 5 + [C.c_int] * 4 + [C.c_float]),
    "iris_metal_set_attention_bias": (None, [C.c_int, C.c_float]),
    "iris_gpu_chain_begin": (None, []),
    "iris_gpu_chain_end": (None, []),
    "iris_gpu_in_chain": (C.c_int, []),
    "iris_metal_begin_batch": (None, []),
    "iris_metal_end_batch": (None, []),
    "iris_metal_in_batch": (C.c_int, []),
    "iris_metal_sync": (None, []),
    "iris_metal_wait_idle": (None, []),
    "iris_metal_init": (C.c_int, []),
    "iris_metal_cleanup": (None, []),
    "iris_metal_reset": (None, []),
    "iris_metal_reset_transient": (None, []),
    "iris_metal_rope_cache_begin": (None, []),
    "iris_metal_clear_weight_cache_only": (None, []),
    "iris_metal_clear_bf16_cache_only": (None, []),
    "iris_metal_clear_f16_cache_only": (None, []),
    "iris_metal_clear_activation_pool_only": (None, []),
    "iris_metal_memory_used": (C.c_size_t, []),
    "iris_metal_warmup_bf16": (None, [_u16p, C.c_size_t]),
    "iris_metal_warmup_bf16_buffer": (None, [_u16p, C.c_size_t]),
    "iris_metal_warmup_bf16_buffers_parallel": (None, [C.POINTER(_u16p), C.POINTER(C.c_size_t), C.c_int]),
    "iris_gpu_op_failures": (C.c_ulong, []),
}

_libc = C.CDLL(None)
_libc.free.argtypes = [C.c_void_p]
_libc.free.restype = None


class IrisCudaError(RuntimeError):
    pass


def load(path: str = LIB_PATH) -> C.CDLL:
    if not os.path.exists(path):
        raise IrisCudaError(f"{path} not built: run `make -C iris.c_b200 cuda` (no fallback path exists)")
    lib = C.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


_LIB = None


def lib() -> C.CDLL:
    global _LIB
    if _LIB is None:
        _LIB = load()
    return _LIB


def last_error() -> str:
    return (lib().iris_cuda_last_error() or b"").decode()


def _f(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(_fp)


def _take_floats(ptr, n, shape=None) -> np.ndarray:
    if not ptr:
        raise IrisCudaError(last_error() or "call failed")
    # the library's malloc'd buffer becomes the array's memory (no copy); it is
    # freed when the last view of it goes away
    buf = (C.c_float * n).from_address(ptr)
    weakref.finalize(buf, _libc.free, ptr)
    arr = np.frombuffer(buf, np.float32)
    return arr.reshape(shape) if shape is not None else arr


class Flux:
    """Resident Flux.2 Klein transformer (libiris_cuda)."""

    def __init__(self, handle):
        if not handle:
            raise IrisCudaError(last_error() or "model creation failed")
        self.h = handle
        cfg = FluxConfig()
        lib().iris_cuda_flux_get_config(self.h, C.byref(cfg))
        self.cfg = cfg

    @classmethod
    def load(cls, model_dir: str, tp_rank: int = 0, tp_size: int = 1) -> "Flux":
        if tp_size == 1:
            return cls(lib().iris_cuda_flux_load(model_dir.encode()))
        return cls(lib().iris_cuda_flux_load_tp(model_dir.encode(), tp_rank, tp_size))

    @classmethod
    def random(cls, cfg: FluxConfig, seed: int, std: float = 0.02, norm_unit: bool = False,
               tp_rank: int = 0, tp_size: int = 1) -> "Flux":
        if tp_size == 1:
            return cls(lib().iris_cuda_flux_random(C.byref(cfg), seed, std, int(norm_unit)))
        return cls(lib().iris_cuda_flux_random_tp(C.byref(cfg), seed, std, int(norm_unit), tp_rank, tp_size))

    def close(self):
        if self.h:
            lib().iris_cuda_flux_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def weight_bytes(self) -> int:
        return lib().iris_cuda_flux_weight_bytes(self.h)

    def read_weight(self, name: str, shape) -> np.ndarray:
        out = np.zeros(int(np.prod(shape)), np.uint16)
        rc = lib().iris_cuda_flux_read_weight(self.h, name.encode(), out.ctypes.data_as(_u16p), out.size)
        if rc:
            raise IrisCudaError(last_error())
        return out.reshape(shape)

    def load_lora(self, path: str, scale: float = 1.0) -> int:
        """iris_load_lora: fold a LoRA file (XLabs / Kohya / Diffusers / BFL) into
        the weights at strength `scale`; returns the number of adapters applied."""
        if lib().iris_cuda_flux_load_lora(self.h, path.encode(), float(scale)):
            raise IrisCudaError(last_error())
        return lib().iris_cuda_flux_lora_adapters(self.h)

    def unload_lora(self) -> None:
        if lib().iris_cuda_flux_unload_lora(self.h):
            raise IrisCudaError(last_error())

    @property
    def lora_adapters(self) -> int:
        return lib().iris_cuda_flux_lora_adapters(self.h)

    def lora_stats(self) -> tuple[float, float]:
        """(device ms, bytes moved) of the last LoRA fold."""
        ms, nb = C.c_double(), C.c_double()
        lib().iris_cuda_flux_lora_stats(self.h, C.byref(ms), C.byref(nb))
        return ms.value, nb.value

    def load_ip_adapter(self, bundle_dir: str, features, scale_mult: float = 1.0) -> None:
        """iris_load_ip_adapter: features = a path to raw f32 rows, or an array."""
        if isinstance(features, str):
            rc = lib().iris_cuda_flux_load_ip_adapter(self.h, bundle_dir.encode(), features.encode(), scale_mult)
        else:
            f = np.ascontiguousarray(features, np.float32)
            n = f.shape[0] if f.ndim > 1 else 1
            rc = lib().iris_cuda_flux_load_ip_adapter_mem(self.h, bundle_dir.encode(), _f(f), n, scale_mult)
        if rc:
            raise IrisCudaError(last_error())

    def unload_ip_adapter(self) -> None:
        if lib().iris_cuda_flux_unload_ip_adapter(self.h):
            raise IrisCudaError(last_error())

    def set_ip_schedule(self, spec: str) -> None:
        if lib().iris_cuda_flux_set_ip_schedule(self.h, spec.encode()):
            raise IrisCudaError(last_error())

    def set_ip_step(self, step: int, num_steps: int) -> None:
        if lib().iris_cuda_flux_set_ip_step(self.h, step, num_steps):
            raise IrisCudaError(last_error())

    def ip_embeds(self, tokens: int) -> np.ndarray:
        out = np.zeros(tokens * self.cfg.hidden, np.float32)
        n = lib().iris_cuda_flux_ip_embeds(self.h, _f(out), out.size)
        if n < 0:
            raise IrisCudaError(last_error())
        return out[:n].reshape(-1, self.cfg.hidden)

    def set_sref_csd(self, csdmod_path, csd, scale: float) -> None:
        """iris_set_sref_csd: the CSD modulation delta on the timestep embedding (None: off)."""
        if csdmod_path is None:
            rc = lib().iris_cuda_flux_set_sref_csd(self.h, None, None, 0, 0.0)
        else:
            c = np.ascontiguousarray(csd, np.float32).ravel()
            rc = lib().iris_cuda_flux_set_sref_csd(self.h, csdmod_path.encode(), _f(c), c.size, scale)
        if rc:
            raise IrisCudaError(last_error())

    def set_sref_bands(self, shf: float, slf: float) -> None:
        if lib().iris_cuda_flux_set_sref_bands(self.h, shf, slf):
            raise IrisCudaError(last_error())

    def run_block(self, kind: int, idx: int, hidden: np.ndarray, txt_seq: int, img_h: int, img_w: int,
                  t: float) -> np.ndarray:
        hid = np.ascontiguousarray(hidden, np.float32).copy()
        rc = lib().iris_cuda_flux_run_block(self.h, kind, idx, _f(hid), txt_seq, img_h, img_w, t)
        if rc:
            raise IrisCudaError(last_error())
        return hid

    def forward(self, latent: np.ndarray, txt: np.ndarray, t: float, refs=()) -> np.ndarray:
        lat = np.ascontiguousarray(latent, np.float32)
        tx = np.ascontiguousarray(txt, np.float32)
        c, h, w = lat.shape
        if refs:
            keep = [np.ascontiguousarray(r, np.float32) for r in refs]
            arr = (Ref * len(keep))(*[Ref(_f(r), r.shape[1], r.shape[2], 10 * (i + 1))
                                      for i, r in enumerate(keep)])
            p = lib().iris_cuda_transformer_forward_with_multi_refs(self.h, _f(lat), h, w, arr, len(keep),
                                                                    _f(tx), tx.shape[0], t)
        else:
            p = lib().iris_cuda_transformer_forward(self.h, _f(lat), h, w, _f(tx), tx.shape[0], t)
        return _take_floats(p, c * h * w, (c, h, w))

    def profile(self, t: float, max_entries: int = 512):
        """Per-kernel CUDA-event times of one forward over the last input shape."""
        buf = (KernelTime * max_entries)()
        n = lib().iris_cuda_flux_profile(self.h, t, buf, max_entries)
        if n < 0:
            raise IrisCudaError(last_error())
        return [dict(name=buf[i].name.decode(), flops=buf[i].flops, bytes=buf[i].bytes, ms=buf[i].ms)
                for i in range(n)]

    def sample_euler(self, z, txt, schedule, refs=(), txt_uncond=None, guidance=1.0, cfg_pair=False):
        """Euler sampler; cfg_pair=True splits the CFG branches over the
        process's 2-rank communicator (comm_init)."""
        zz = np.ascontiguousarray(z, np.float32)
        tx = np.ascontiguousarray(txt, np.float32)
        sc = np.ascontiguousarray(schedule, np.float32)
        c, h, w = zz.shape
        cb = PROGRESS_CB(0)
        if cfg_pair:
            tu = np.ascontiguousarray(txt_uncond, np.float32)
            p = lib().iris_cuda_sample_euler_cfg_pair(self.h, _f(zz), 1, c, h, w, _f(tx), tx.shape[0], _f(tu),
                                                      tu.shape[0], guidance, _f(sc), len(sc) - 1, cb)
        elif txt_uncond is not None:
            tu = np.ascontiguousarray(txt_uncond, np.float32)
            p = lib().iris_cuda_sample_euler_cfg(self.h, _f(zz), 1, c, h, w, _f(tx), tx.shape[0], _f(tu),
                                                 tu.shape[0], guidance, _f(sc), len(sc) - 1, cb)
        elif refs:
            keep = [np.ascontiguousarray(r, np.float32) for r in refs]
            arr = (Ref * len(keep))(*[Ref(_f(r), r.shape[1], r.shape[2], 10 * (i + 1))
                                      for i, r in enumerate(keep)])
            p = lib().iris_cuda_sample_euler_with_multi_refs(self.h, _f(zz), 1, c, h, w, arr, len(keep),
                                                             _f(tx), tx.shape[0], _f(sc), len(sc) - 1, cb)
        else:
            p = lib().iris_cuda_sample_euler(self.h, _f(zz), 1, c, h, w, _f(tx), tx.shape[0], _f(sc),
                                             len(sc) - 1, cb)
        return _take_floats(p, c * h * w, (c, h, w))


def comm_unique_id() -> bytes:
    """A new NCCL unique id (IRIS_CUDA_COMM_ID_BYTES bytes) for comm_init."""
    buf = C.create_string_buffer(128)
    if lib().iris_cuda_comm_unique_id(buf, 128):
        raise IrisCudaError(last_error())
    return buf.raw


def comm_init(uid: bytes, world: int, rank: int) -> None:
    buf = C.create_string_buffer(bytes(uid), 128)
    if lib().iris_cuda_comm_init(buf, world, rank):
        raise IrisCudaError(last_error())


def comm_destroy() -> None:
    lib().iris_cuda_comm_destroy()


def comm_groups(world: int, group_size: int):
    """Rank groups of `group_size` consecutive ranks ((0,1), (2,3), ... for CFG
    pairs); every rank is in exactly one."""
    if group_size < 1 or world % group_size:
        raise ValueError(f"world {world} is not a multiple of group size {group_size}")
    return [tuple(range(g, g + group_size)) for g in range(0, world, group_size)]


def comm_init_group(exchange, rank: int, world: int, group_size: int) -> tuple:
    """Create this rank's NCCL communicator over its group of `group_size`
    consecutive ranks.  `exchange(obj)` must return the list of every rank's
    obj (e.g. torch.distributed.all_gather_object); the first rank of each
    group creates the id.  Returns (group, rank in group)."""
    groups = comm_groups(world, group_size)
    group = next(g for g in groups if rank in g)
    mine = comm_unique_id() if rank == group[0] else None
    ids = exchange(mine)
    comm_init(ids[group[0]], len(group), group.index(rank))
    return group, group.index(rank)


LORA_FORMATS = {1: "xlabs", 2: "kohya", 3: "diffusers", 4: "bfl"}


def lora_probe(path: str, n_double: int, n_single: int, hidden: int, mlp: int) -> dict:
    """Host-only: adapters of a LoRA file matching a model of this shape."""
    k = (C.c_int * 5)()
    n = lib().iris_cuda_lora_probe(path.encode(), n_double, n_single, hidden, mlp, k)
    if n < 0:
        raise IrisCudaError(last_error())
    return {"format": LORA_FORMATS[k[0]], "adapters": n, "qkv": k[1], "proj": k[2], "linear1": k[3],
            "linear2": k[4]}


def official_schedule(steps: int, seq: int) -> np.ndarray:
    return _take_floats(lib().iris_cuda_official_schedule(steps, seq), steps + 1)


def zimage_schedule(steps: int, seq: int) -> np.ndarray:
    return _take_floats(lib().iris_cuda_zimage_schedule(steps, seq), steps + 1)


def init_noise(c: int, h: int, w: int, seed: int) -> np.ndarray:
    return _take_floats(lib().iris_cuda_init_noise(1, c, h, w, seed), c * h * w, (c, h, w))


class ZImage:
    """Resident Z-Image S3-DiT transformer (libiris_cuda)."""

    def __init__(self, handle):
        if not handle:
            raise IrisCudaError(last_error() or "model creation failed")
        self.h = handle
        cfg = ZImageConfig()
        lib().iris_cuda_zimage_get_config(self.h, C.byref(cfg))
        self.cfg = cfg

    @classmethod
    def load(cls, model_dir: str) -> "ZImage":
        return cls(lib().iris_cuda_zimage_load(model_dir.encode()))

    @classmethod
    def random(cls, cfg: ZImageConfig, seed: int, std: float = 0.02, norm_unit: bool = False) -> "ZImage":
        return cls(lib().iris_cuda_zimage_random(C.byref(cfg), seed, std, int(norm_unit)))

    def close(self):
        if self.h:
            lib().iris_cuda_zimage_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def forward(self, latent: np.ndarray, cap: np.ndarray, t: float) -> np.ndarray:
        lat = np.ascontiguousarray(latent, np.float32)
        cp = np.ascontiguousarray(cap, np.float32)
        c, h, w = lat.shape
        p = lib().iris_cuda_zi_transformer_forward(self.h, _f(lat), h, w, t, _f(cp), cp.shape[0])
        return _take_floats(p, c * h * w, (c, h, w))

    def sample_euler(self, z: np.ndarray, cap: np.ndarray, schedule) -> np.ndarray:
        zz = np.ascontiguousarray(z, np.float32)
        cp = np.ascontiguousarray(cap, np.float32)
        sc = np.ascontiguousarray(schedule, np.float32)
        c, h, w = zz.shape
        p = lib().iris_cuda_sample_euler_zimage(self.h, _f(zz), 1, c, h, w, self.cfg.patch_size, _f(cp),
                                                cp.shape[0], _f(sc), len(sc) - 1, PROGRESS_CB(0))
        return _take_floats(p, c * h * w, (c, h, w))


class Vae:
    """Resident autoencoder decoder (libiris_cuda): latent -> RGB image."""

    def __init__(self, handle, z: int):
        if not handle:
            raise IrisCudaError(last_error() or "VAE load failed")
        self.h = handle
        self.z = z

    @classmethod
    def load(cls, vae_dir: str, z: int = 0, scaling: float = 0.0, shift: float = 0.0) -> "Vae":
        """z <= 0: latent channels, scaling and shift from vae_dir/config.json."""
        h = lib().iris_cuda_vae_load(vae_dir.encode(), z, scaling, shift)
        zz = z
        if zz <= 0:
            import json
            import os
            cfg = os.path.join(vae_dir, "config.json")
            zz = json.load(open(cfg)).get("latent_channels", 32) if os.path.exists(cfg) else 32
        return cls(h, zz)

    @classmethod
    def random(cls, z: int = 32, seed: int = 1, scaling: float = 0.0, shift: float = 0.0) -> "Vae":
        return cls(lib().iris_cuda_vae_random(z, scaling, shift, seed), z)

    def profile(self, max_entries: int = 512):
        """Per-kernel CUDA-event times of one decode at the last latent size."""
        arr = (KernelTime * max_entries)()
        n = lib().iris_cuda_vae_profile(self.h, arr, max_entries)
        if n < 0:
            raise IrisCudaError(last_error())
        return [dict(name=arr[i].name.decode(), ms=arr[i].ms, flops=arr[i].flops, bytes=arr[i].bytes)
                for i in range(n)]

    def close(self):
        if self.h:
            lib().iris_cuda_vae_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def weight_bytes(self) -> int:
        return lib().iris_cuda_vae_weight_bytes(self.h)

    def decode(self, latent: np.ndarray) -> np.ndarray:
        """[4z, h, w] latent -> uint8 [16h, 16w, 3] (iris_vae_decode)."""
        lat = np.ascontiguousarray(latent, np.float32)
        _, h, w = lat.shape
        p = lib().iris_cuda_vae_decode(self.h, _f(lat), 1, h, w)
        if not p:
            raise IrisCudaError(last_error())
        img = C.cast(p, C.POINTER(Image)).contents
        out = np.ctypeslib.as_array(img.data, shape=(img.height, img.width, img.channels)).copy()
        lib().iris_cuda_image_free(p)
        return out

    def decode_f32(self, latent: np.ndarray) -> np.ndarray:
        """[4z, h, w] latent -> f32 RGB planes [3, 16h, 16w] before the uint8 conversion."""
        lat = np.ascontiguousarray(latent, np.float32)
        _, h, w = lat.shape
        out = np.zeros((3, 16 * h, 16 * w), np.float32)
        if lib().iris_cuda_vae_decode_f32(self.h, _f(lat), h, w, _f(out)):
            raise IrisCudaError(last_error())
        return out

    def graph_kernels(self) -> int:
        return lib().iris_cuda_vae_graph_kernels(self.h)


class Qwen3:
    """Resident Qwen3 text encoder (libiris_cuda): token ids -> text embeddings."""

    def __init__(self, handle):
        if not handle:
            raise IrisCudaError(last_error() or "text encoder creation failed")
        self.h = handle

    @classmethod
    def load(cls, model_dir: str) -> "Qwen3":
        return cls(lib().iris_cuda_qwen3_load(model_dir.encode()))

    @classmethod
    def random(cls, cfg: Qwen3Config, seed: int) -> "Qwen3":
        return cls(lib().iris_cuda_qwen3_random(C.byref(cfg), seed))

    def close(self):
        if self.h:
            lib().iris_cuda_qwen3_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_extraction_mode(self, mode: int) -> None:
        if lib().iris_cuda_qwen3_set_extraction_mode(self.h, mode):
            raise IrisCudaError(last_error())

    def text_dim(self) -> int:
        return lib().iris_cuda_qwen3_text_dim(self.h)

    def profile(self, max_entries: int = 1024):
        """Per-kernel CUDA-event times of one forward at the last sequence length."""
        arr = (KernelTime * max_entries)()
        n = lib().iris_cuda_qwen3_profile(self.h, arr, max_entries)
        if n < 0:
            raise IrisCudaError(last_error())
        return [dict(name=arr[i].name.decode(), ms=arr[i].ms, flops=arr[i].flops) for i in range(n)]

    def forward(self, ids, mask=None) -> np.ndarray:
        """ids / mask [S] -> f32 [S, text_dim] (qwen3_forward)."""
        ip = C.POINTER(C.c_int)
        ids = np.ascontiguousarray(ids, np.int32)
        m = None if mask is None else np.ascontiguousarray(mask, np.int32)
        p = lib().iris_cuda_qwen3_forward(self.h, ids.ctypes.data_as(ip),
                                          None if m is None else m.ctypes.data_as(ip), len(ids))
        return _take_floats(p, len(ids) * self.text_dim(), (len(ids), self.text_dim()))
