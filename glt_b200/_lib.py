"""ctypes binding of include/glt_graft.h.

Loads the in-tree ``libglt_b200.so``.  There is no fallback: if the library
is missing the import fails loudly (build it with ``python -m glt_b200.build``).
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libglt_b200.so")

GLT_OK = 0
STATUS_NAMES = {
    0: "GLT_OK", 1: "GLT_EINVAL", 2: "GLT_ECUDA", 3: "GLT_ENCCL", 4: "GLT_EIO",
    5: "GLT_ETIMEOUT", 6: "GLT_ESTATE", 7: "GLT_ENOMEM",
}


class GltError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {msg}")
        self.status = status


def _load() -> C.CDLL:
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} not found: the CUDA library is required (python -m glt_b200.build)"
        )
    return C.CDLL(LIB_PATH)


lib = _load()

_vp, _i32, _i64, _f32, _u32 = C.c_void_p, C.c_int, C.c_int64, C.c_float, C.c_uint
_u64 = C.c_uint64


class GltModelConfig(C.Structure):
    """ctypes mirror of GltModelConfig (include/glt_graft.h)."""
    _fields_ = [
        ("hidden_dim", _i32), ("intermediate_dim", _i32), ("slice_dim", _i32), ("vocab_size", _i32),
        ("num_layers", _i32), ("num_heads", _i32), ("num_kv_heads", _i32), ("head_dim", _i32),
        ("max_domains", _i32), ("domain_id", _i32), ("layout", _i32), ("tie_embeddings", _i32),
        ("rms_norm_eps", _f32), ("lm_loss_scale", _f32), ("lambda_silence", _f32), ("rope_theta", _f32),
        ("graft_layer_start", _i32), ("graft_layer_end", _i32),
        ("graft_proj_gate", _i32), ("graft_proj_up", _i32), ("graft_proj_down", _i32),
        ("allow_expansion_trap", _i32),
        ("adam_beta1", _f32), ("adam_beta2", _f32), ("adam_eps", _f32), ("adam_weight_decay", _f32),
        ("gradient_clip_norm", _f32),
        ("lr_warmup_steps", _i32), ("lr_peak", _f32),
        ("no_rope_mask_len", _i32), ("no_rope_mask", _i32 * 256),
    ]


class GltStepStats(C.Structure):
    _fields_ = [(n, _f32) for n in (
        "lm_loss", "silence_loss", "domain_graft_energy", "ood_graft_energy",
        "domain_ood_energy_ratio", "total_loss", "lr", "grad_norm")]


class GltEvalStats(C.Structure):
    _fields_ = [("tokens", C.c_int64), ("total_nll", C.c_double), ("mean_ce", C.c_double),
                ("ppl", C.c_double), ("logits_sum", C.c_double), ("logits_l2", C.c_double),
                ("logits_hash", C.c_uint64), ("graft_forward_calls", C.c_int64)]


class GltGraftWeights(C.Structure):
    """ctypes mirror of GltGraftWeights (include/glt_graft.h)."""
    _fields_ = [("weight", _vp), ("weight_bf16", _vp), ("weight_elems", C.c_int64), ("domain_id", _i32),
                ("allocated", _i32), ("active", _i32)]


class GltMlpSaved(C.Structure):
    """ctypes mirror of GltMlpSaved (include/glt_graft.h)."""
    _fields_ = [("x_ffn", _vp), ("variance", _vp), ("energy_sq", _vp), ("delta_down", _vp)]


_cfgp = C.POINTER(GltModelConfig)
_gwp = C.POINTER(GltGraftWeights)
_svp = C.POINTER(GltMlpSaved)
_fp = C.POINTER(C.c_void_p)

# (name, restype, argtypes) for every exported symbol; tests check that each
# declaration of include/glt_graft.h appears here and in the library.
SIGNATURES: dict[str, tuple] = {
    "glt_last_error": (C.c_char_p, []),
    "glt_version": (C.c_char_p, []),
    "glt_device_error": (_i32, [C.POINTER(_u32)]),
    "glt_selftest_wait_timeout": (_i32, [_i32, _i32, _vp]),
    "glt_gemm": (_i32, [_vp, _i64, _i32, _vp, _i64, _i32, _vp, _i64, _i32,
                        _i32, _i32, _i32, _f32, _f32, _vp]),
    "glt_gemm_pair_mode": (_i32, [_i32]),
    "glt_config_default": (_i32, [_cfgp]),
    "glt_config_validate": (_i32, [_cfgp, _i32, _i32]),
    "glt_get_lr": (_f32, [_cfgp, _i32, _i32]),
    "glt_delta_offset": (_i64, [_i32, _i32, _i32, _i32]),
    "glt_adamw_all": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _f32, _vp]),
    "glt_grad_clip": (_i32, [_vp, _i64, _f32, _i32, _vp, _i64, _vp, _vp, _vp]),
    "glt_swiglu_fwd": (_i32, [_vp, _vp, _vp, _i32, _i32, _i64, _i64, _i64, _vp]),
    "glt_swiglu_bwd": (_i32, [_vp, _vp, _vp, _vp, _vp, _i64, _vp]),
    "glt_stack_grafts": (_i32, [C.POINTER(_vp), _i32, _i32, _i32, _i32, _vp, _vp]),
    "glt_model_create": (_i32, [_cfgp, _i32, _i32, _i32, C.POINTER(_vp)]),
    "glt_graft_weights_alloc": (_i32, [_cfgp, _i32, _i32, _gwp]),
    "glt_graft_weights_free": (_i32, [_gwp]),
    "glt_mlp_create": (_i32, [_cfgp, _i32, C.POINTER(_vp)]),
    "glt_mlp_destroy": (_i32, [_vp]),
    "glt_mlp_set_weight": (_i32, [_vp, _i32, _i32, _vp, _i64, _i32, _vp]),
    "glt_mlp_set_graft": (_i32, [_vp, _gwp, _vp]),
    "glt_mlp_recompute_bytes": (_i32, [_vp, C.POINTER(_i64)]),
    "glt_mlp_fwd": (_i32, [_vp, _i32, _vp, _vp, _svp, _i32, _vp]),
    "glt_mlp_recompute": (_i32, [_vp, _i32, _svp, _vp, _vp]),
    "glt_mlp_bwd": (_i32, [_vp, _i32, _vp, _vp, _svp, _vp, _vp, _f32, _vp, _vp]),
    "glt_model_destroy": (_i32, [_vp]),
    "glt_train_state_save": (_i32, [C.c_char_p, _vp, _vp, _vp, _i64, _i32, C.c_char_p, _i32, _i32, _i32,
                                    _i32, _i32, _i64]),
    "glt_train_state_load": (_i32, [C.c_char_p, _vp, _vp, _vp, _i64, _i32, C.c_char_p, _i32, _i32, _i32,
                                    _i32, C.POINTER(_i64)]),
    "glt_model_save_train_state": (_i32, [_vp, C.c_char_p, C.c_char_p, _i32, _i64]),
    "glt_model_load_train_state": (_i32, [_vp, C.c_char_p, C.c_char_p, _i32, C.POINTER(_i64)]),
    "glt_model_save_stack": (_i32, [_vp, C.POINTER(C.c_char_p), _i32, C.c_char_p]),
    "glt_model_load_stack": (_i32, [_vp, C.POINTER(C.c_char_p), _i32, C.c_char_p]),
    "glt_model_step_stats": (_i32, [_vp, _i32, C.c_void_p]),
    "glt_model_memory": (_i32, [_vp, C.POINTER(_i64), C.POINTER(_i64)]),
    "glt_model_mlp_store": (_i32, [_vp, _i32, C.POINTER(_i32), C.POINTER(_i64)]),
    "glt_model_init_random": (_i32, [_vp, _u64, _f32, _f32, _f32]),
    "glt_model_set_weight": (_i32, [_vp, _i32, _i32, _vp, _i64, _i32, _vp]),
    "glt_model_graft_buffers": (_i32, [_vp, _fp, _fp, _fp, _fp, C.POINTER(_i64)]),
    "glt_model_refresh_graft": (_i32, [_vp, _vp]),
    "glt_train_step": (_i32, [_vp, _vp, _vp, _i32, _i32, _i32, C.POINTER(GltStepStats), _vp]),
    "glt_forward": (_i32, [_vp, _vp, _i32, _i32, _vp, _vp]),
    "glt_model_eval": (_i32, [_vp, _vp, C.c_int64, _i32, _i32, C.POINTER(GltEvalStats), _vp]),
    "glt_model_shadow_bake": (_i32, [_vp, _vp]),
    "glt_model_load_safetensors": (_i32, [_vp, C.c_char_p, _vp]),
    "glt_safetensors_tensor_info": (_i32, [C.c_char_p, C.c_char_p, C.POINTER(_i32),
                                           C.POINTER(C.c_int64), C.POINTER(_i32)]),
    "glt_device_memory": (_i32, [C.POINTER(C.c_int64), C.POINTER(C.c_int64)]),
    "glt_malloc": (_i32, [C.POINTER(C.c_void_p), C.c_int64]),
    "glt_free": (_i32, [_vp]),
    "glt_block_step": (_i32, [_vp, _vp, _vp, _f32, _i32, C.POINTER(_f32), _vp, _vp, _vp]),
    "glt_model_activation": (_i32, [_vp, _i32, _i32, C.POINTER(_vp), C.POINTER(_i64)]),
    "glt_dp_unique_id": (_i32, [_vp, _i32]),
    "glt_dp_init": (_i32, [_vp, _vp, _i32, _i32]),
    "glt_dp_finalize": (_i32, [_vp]),
    "glt_dp_async_error": (_i32, [_vp, C.POINTER(_i32)]),
    "glt_dp_abort": (_i32, [_vp]),
    "glt_memcpy": (_i32, [_vp, _vp, _i64, _vp, _i32]),
    "glt_launch_count": (_i32, [C.POINTER(_u64)]),
    "glt_model_profile": (_i32, [_vp, _i32]),
    "glt_model_profile_read": (_i32, [_vp, C.POINTER(C.c_double), C.POINTER(_i64), _i32]),
    "glt_attention_fwd": (_i32, [_vp, _i64, _vp, _i64, _vp, _i32, _i32, _i32, _i32, _i32, _i32, _vp]),
    "glt_attention_bwd": (_i32, [_vp, _i64, _vp, _vp, _i64, _vp, _vp, _vp, _vp, _i32, _i32, _i32,
                                 _i32, _i32, _i32, _vp]),
    "glt_rope": (_i32, [_vp, _i64, _i32, _i32, _i32, _i32, _i32, _f32, _i32, _vp]),
    "glt_rmsnorm_fwd": (_i32, [_vp, _vp, _vp, _vp, _i32, _i32, _f32, _vp]),
    "glt_rmsnorm_bwd": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _f32, _vp]),
    "glt_arena_create": (_i32, [_i64, C.POINTER(_vp)]),
    "glt_arena_destroy": (_i32, [_vp]),
    "glt_graft_op": (_i32, [_i32, _i32, _i32, _i32, _vp, _vp, _vp, _i32, _i64, _vp, _i32, _i64,
                            _vp, _i64, _f32, _f32, _vp, _vp]),
    "glt_graft_op_noalloc": (_i32, [_i32, _i32, _i32, _i32, _vp, _vp, _vp, _i32, _i64, _vp, _i32,
                                    _i64, _vp, _i64, _f32, _f32, _vp]),
    "glt_shadow_bake": (_i32, [_vp, _i64, _vp, _i32, _i32, _i32, _i32, _i32, _vp]),
    "glt_apply_graft_to_shadow": (_i32, [_cfgp, _vp, _vp, _vp, _i64, _i64, _vp,
                                         C.POINTER(_i32), _vp]),
    "glt_checkpoint_save": (_i32, [C.c_char_p, _vp, _i64, _i32, C.c_char_p, _i32, _i32, _i32,
                                   _i32, _i32]),
    "glt_checkpoint_load": (_i32, [C.c_char_p, _vp, _i64, _i32, _i32, C.c_char_p, _i32, _i32,
                                   _i32, C.POINTER(_i32)]),
    "glt_model_save_checkpoint": (_i32, [_vp, C.c_char_p, C.c_char_p, _i32]),
    "glt_model_load_checkpoint": (_i32, [_vp, C.c_char_p, C.c_char_p, _i32]),
    "glt_load_bin": (_i32, [C.c_char_p, C.POINTER(_i32), C.POINTER(_i32), _vp, _i64]),
    "glt_batch_walk_start": (_i32, [_u64, _i32, _i32, C.POINTER(_i32), C.POINTER(_i32)]),
    "glt_batch_step": (_i32, [_vp, _i32, _vp, _i32, _i32, _i32, C.POINTER(_i32), C.POINTER(_i32),
                              _vp, _vp]),
}

for _name, (_res, _args) in SIGNATURES.items():
    _fn = getattr(lib, _name)
    _fn.restype = _res
    _fn.argtypes = _args


def last_error() -> str:
    return lib.glt_last_error().decode(errors="replace")


def check(status: int) -> None:
    if status != GLT_OK:
        raise GltError(status, last_error())


def call(name: str, *args) -> None:
    check(getattr(lib, name)(*args))
