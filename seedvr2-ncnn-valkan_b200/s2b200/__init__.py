"""Python host mirror of the SeedVR2 windowed MM-attention path (B200, sm_100a).

Everything here is a thin ctypes layer over ``lib/libs2b200.so`` (C ABI:
``include/s2_b200.h``). PyTorch supplies device memory and streams only; all
compute runs in the library's CUDA kernels. There is no CPU fallback: if the
library is missing or no sm_100 GPU is present, the device entry points raise.

Mirrors the reference's layer surface (czwdysj/seedvr2-ncnn-valkan):
  * ``make_windows``            <- SeedVR2DiTBlock::make_windows (src/layers/seedvr2_dit_block.cpp:827-868)
  * ``SeedVR2DiTBlockAttention`` <- SeedVR2DiTBlock's attention stage: load_param (:643-655),
    load_model norm/freqs part (:657-688), set_runtime_shape (.h:55), attention() (:870-1091)
  * ``SeedVR2DiT``               <- the DiT (src/model/dit.cpp:277-383: input head, 32 blocks,
    output head) and one Euler step (src/core/engine.cpp:125-149, src/model/sampler.cpp:276-286)
  * ``SeedVR2DiTBlock``          <- the whole block (seedvr2_dit_block.cpp: load_param :643-655,
    load_model :657-688, forward :1114-1267)
  * ``DynamicFramewiseSpatialAttention`` <- the VAE mid-block attention layer
    (src/layers/dynamic_framewise_spatial_attention.cpp: load_param :50-59,
    load_model :61-77, forward :106-210)
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(os.path.dirname(HERE), "lib", "libs2b200.so")
HEAD_DIM = 128

S2_OK, S2_INVALID_ARGUMENT, S2_NOT_LOADED, S2_INFERENCE_FAILED, S2_UNSUPPORTED, S2_OUT_OF_MEMORY = 0, -1, -2, -5, -6, -7
S2_F32, S2_F16, S2_BF16 = 0, 1, 2
MODE_BF16_REF, MODE_F16, MODE_BF16_F16 = 0, 1, 2

_STATUS_NAMES = {0: "Ok", -1: "InvalidArgument", -2: "NotLoaded", -5: "InferenceFailed", -6: "UnsupportedBackend",
                 -7: "OutOfMemory"}


class S2Error(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{_STATUS_NAMES.get(status, status)} ({status}): {message}")
        self.status = status


class BlockParams(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in ("block_index", "shared", "last", "shifted", "dim", "heads", "head_dim",
                                            "mlp_hidden")] + [("eps", ctypes.c_float)]


class HeadParams(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in ("dim", "video_channels", "text_channels", "sinusoidal_dim",
                                            "embedding_dim", "out_channels")] + [("eps", ctypes.c_float)]


class GemmDesc(ctypes.Structure):
    """s2_gemm_desc (include/s2_b200.h)."""
    _fields_ = ([(n, ctypes.c_int) for n in ("epilogue", "M", "N", "K")]
                + [(n, ctypes.c_void_p) for n in ("a", "b", "bias", "gmul", "resid", "resid2", "out0", "out1", "out2",
                                                  "y", "y2")]
                + [("split", ctypes.c_int), ("split_row", ctypes.c_int), ("out_scale", ctypes.c_float),
                   ("workspace", ctypes.c_void_p), ("workspace_floats", ctypes.c_size_t), ("err", ctypes.c_void_p),
                   ("row_dest", ctypes.c_void_p)])


GEMM_SPLIT_F16, GEMM_GATED_RESID_F32, GEMM_SWIGLU_F16 = 0, 2, 3


DEBUG_TENSORS = ("qkv_vid", "qkv_txt", "norm_q_vid", "norm_q_txt", "norm_k_vid", "norm_k_txt", "attention_q",
                 "attention_k", "attention_v", "attention_output", "projected_vid", "projected_txt", "output_vid",
                 "output_txt")


class BlockDebug(ctypes.Structure):
    """s2_block_debug: device fp32 buffers of the block's 14 capture points."""
    _fields_ = [(n, ctypes.c_void_p) for n in DEBUG_TENSORS]


class Window(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in ("t0", "t1", "h0", "h1", "w0", "w1")]


class Row(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in ("src", "pt", "ph", "pw")]


_vp = ctypes.c_void_p
_i32p = ctypes.POINTER(ctypes.c_int32)
_f32p = ctypes.POINTER(ctypes.c_float)
_lib = None

# name -> (restype, argtypes); mirrors include/s2_b200.h
_SIGS = {
    "s2_make_windows": (ctypes.c_int, [ctypes.c_int] * 7 + [ctypes.POINTER(Window), ctypes.c_int, _i32p]),
    "s2_build_varlen": (ctypes.c_int, [ctypes.c_int] * 3 + [ctypes.POINTER(Window), ctypes.c_int, ctypes.c_int,
                                                           _i32p, ctypes.POINTER(Row), _i32p]),
    "s2_plan_work": (ctypes.c_int, [_i32p, ctypes.c_int, _i32p, ctypes.c_int, _i32p]),
    "s2_shard_windows": (ctypes.c_int, [ctypes.POINTER(Window), ctypes.c_int, ctypes.c_int, ctypes.c_int, _i32p]),
    "s2_shard_windows_joint": (ctypes.c_int, [ctypes.c_int] * 8 + [_i32p, _i32p]),
    "s2_shard_exchange": (ctypes.c_int, [ctypes.c_int] * 10 + [_i32p, _i32p, _i32p, _i32p, _i32p, _i32p, _i32p,
                                                              _i32p, ctypes.POINTER(ctypes.c_longlong)]),
    "s2_shard_row_destinations": (ctypes.c_int, [ctypes.c_int] * 10 + [_i32p, _i32p, ctypes.POINTER(ctypes.c_int)]),
    "s2_rope_table_bytes": (ctypes.c_size_t, [ctypes.c_int]),
    "s2_rope_table": (ctypes.c_int, [_vp, _vp, ctypes.c_int, _vp]),
    "s2_qk_norm_rope": (ctypes.c_int, [_vp, _vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_float, _vp, _vp, _vp,
                                       ctypes.c_int, ctypes.c_int, _vp, _vp, _vp]),
    "s2_window_attention": (ctypes.c_int, [_vp, ctypes.c_int, _vp, _vp, _vp, ctypes.c_int, ctypes.c_int, _vp,
                                           ctypes.c_int, ctypes.c_int, _vp, _vp, ctypes.c_int, _vp, _vp, _vp]),
    "s2_text_window_sum": (ctypes.c_int, [_vp, ctypes.c_int, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                          ctypes.c_float, ctypes.c_int, _vp]),
    "s2_attention_layer_create": (ctypes.c_int, [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float,
                                                 ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                                 ctypes.c_int, ctypes.POINTER(_vp)]),
    "s2_attention_layer_destroy": (ctypes.c_int, [_vp]),
    "s2_attention_layer_load": (ctypes.c_int, [_vp] + [_f32p] * 5),
    "s2_attention_layer_set_runtime_shape": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_int, ctypes.c_int]),
    "s2_attention_layer_set_window_subset": (ctypes.c_int, [_vp, _i32p, ctypes.c_int]),
    "s2_attention_layer_forward": (ctypes.c_int, [_vp, _vp, _vp, ctypes.c_int, ctypes.c_int, _vp, ctypes.c_int,
                                                  _vp, _vp]),
    "s2_attention_layer_forward_host": (ctypes.c_int, [_vp, _vp, _vp, _vp, ctypes.c_int, ctypes.c_int,
                                                       ctypes.c_int, _i32p, _vp, _vp]),
    "s2_attention_layer_last_launches": (ctypes.c_int, [_vp]),
    "s2_attention_layer_device_error": (ctypes.c_int, [_vp, _i32p]),
    "s2_dit_window_attention_noalloc": (ctypes.c_int, [_vp, ctypes.c_int, _vp, _vp, ctypes.c_int] + [ctypes.c_int] * 5
                                        + [ctypes.c_float] + [ctypes.c_int] * 4 + [_vp] * 5),
    "s2_dit_create": (ctypes.c_int, [ctypes.c_int] * 6 + [ctypes.c_float] + [ctypes.c_int] * 7
                      + [ctypes.POINTER(ctypes.c_void_p)]),
    "s2_dit_destroy": (ctypes.c_int, [_vp]),
    "s2_dit_input_weight_count": (ctypes.c_size_t, [_vp]),
    "s2_dit_output_weight_count": (ctypes.c_size_t, [_vp]),
    "s2_dit_load_input": (ctypes.c_int, [_vp, _f32p, ctypes.c_size_t]),
    "s2_dit_load_block": (ctypes.c_int, [_vp] + [ctypes.c_int] * 4 + [_f32p, ctypes.c_size_t]),
    "s2_dit_load_output": (ctypes.c_int, [_vp, _f32p, ctypes.c_size_t]),
    "s2_dit_forward": (ctypes.c_int, [_vp, _vp, _vp] + [ctypes.c_int] * 3 + [_vp, ctypes.c_int, ctypes.c_float, _vp]),
    "s2_dit_euler_step": (ctypes.c_int, [_vp, _vp, _vp, _vp] + [ctypes.c_int] * 3
                          + [_vp, ctypes.c_int, ctypes.c_float, _vp]),
    "s2_dit_euler_step_host": (ctypes.c_int, [_vp, _vp, _vp, _vp] + [ctypes.c_int] * 3
                               + [_vp, ctypes.c_int, ctypes.c_float, _vp]),
    "s2_dit_set_graph": (ctypes.c_int, [_vp, ctypes.c_int]),
    "s2_dit_set_comm": (ctypes.c_int, [_vp, _vp]),
    "s2_ncnn_read_block": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_char_p, ctypes.POINTER(BlockParams), _f32p,
                                          ctypes.c_size_t, ctypes.POINTER(ctypes.c_size_t)]),
    "s2_ncnn_read_input": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_char_p, ctypes.POINTER(HeadParams), _f32p,
                                          ctypes.c_size_t, ctypes.POINTER(ctypes.c_size_t)]),
    "s2_ncnn_read_output": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_char_p, ctypes.POINTER(HeadParams), _f32p,
                                           ctypes.c_size_t, ctypes.POINTER(ctypes.c_size_t)]),
    "s2_dit_load_dir": (ctypes.c_int, [_vp, ctypes.c_char_p]),
    "s2_comm_unique_id": (ctypes.c_int, [ctypes.c_char_p]),
    "s2_comm_init": (ctypes.c_int, [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_char_p,
                                    ctypes.POINTER(ctypes.c_void_p)]),
    "s2_comm_destroy": (ctypes.c_int, [_vp]),
    "s2_comm_init_timeout": (ctypes.c_int, [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_char_p,
                                            ctypes.c_longlong, ctypes.POINTER(ctypes.c_void_p)]),
    "s2_comm_set_timeout": (ctypes.c_int, [_vp, ctypes.c_longlong]),
    "s2_comm_wait": (ctypes.c_int, [_vp, _vp]),
    "s2_comm_size": (ctypes.c_int, [_vp]),
    "s2_comm_rank": (ctypes.c_int, [_vp]),
    "s2_attention_layer_set_local_rows": (ctypes.c_int, [_vp, ctypes.c_int]),
    "s2_attention_layer_local_rows": (ctypes.c_int, [_vp, ctypes.c_int, _i32p]),
    "s2_dit_block_set_local_rows": (ctypes.c_int, [_vp, ctypes.c_int]),
    "s2_dit_last_launches": (ctypes.c_int, [_vp]),
    "s2_dit_device_error": (ctypes.c_int, [_vp, _i32p]),
    "s2_dit_block_create": (ctypes.c_int, [ctypes.c_int] * 9 + [ctypes.c_float] + [ctypes.c_int] * 3
                            + [ctypes.POINTER(ctypes.c_void_p)]),
    "s2_dit_block_destroy": (ctypes.c_int, [_vp]),
    "s2_dit_block_weight_count": (ctypes.c_size_t, [_vp]),
    "s2_dit_block_load": (ctypes.c_int, [_vp, _f32p, ctypes.c_size_t]),
    "s2_dit_block_set_runtime_shape": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_int, ctypes.c_int]),
    "s2_dit_block_set_window_subset": (ctypes.c_int, [_vp, _i32p, ctypes.c_int]),
    "s2_dit_block_forward": (ctypes.c_int, [_vp, _vp, _vp, ctypes.c_int, _vp, ctypes.c_int, _vp, _vp, _vp]),
    "s2_dit_block_forward_host": (ctypes.c_int, [_vp, _vp, _vp, ctypes.c_int, _vp, ctypes.c_int, _vp, _i32p, _vp,
                                                 _vp]),
    "s2_dit_block_last_launches": (ctypes.c_int, [_vp]),
    "s2_dit_block_set_debug_tensors": (ctypes.c_int, [_vp, ctypes.POINTER(BlockDebug)]),
    "s2_dit_block_set_debug_tensors_host": (ctypes.c_int, [_vp, ctypes.POINTER(BlockDebug)]),
    "s2_dit_block_debug_rows": (ctypes.c_int, [_vp, ctypes.c_int, _i32p]),
    "s2_dit_block_device_error": (ctypes.c_int, [_vp, _i32p]),
    "s2_spatial_attention": (ctypes.c_int, [_vp, _vp, _vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                            ctypes.c_int, _vp, _vp]),
    "s2_vae_attention_create": (ctypes.c_int, [ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_void_p)]),
    "s2_vae_attention_destroy": (ctypes.c_int, [_vp]),
    "s2_vae_attention_load": (ctypes.c_int, [_vp] + [_f32p] * 10),
    "s2_vae_attention_forward": (ctypes.c_int, [_vp, _vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                                ctypes.c_longlong, _vp]),
    "s2_vae_attention_forward_host": (ctypes.c_int, [_vp, _vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                                     ctypes.c_longlong, _vp]),
    "s2_vae_attention_last_launches": (ctypes.c_int, [_vp]),
    "s2_vae_attention_device_error": (ctypes.c_int, [_vp, _i32p]),
    "s2_dit_sample": (ctypes.c_int, [_vp, _vp, _vp, _vp] + [ctypes.c_int] * 3 + [_vp, _vp, ctypes.c_int, ctypes.c_int,
                                                                             ctypes.c_float, ctypes.c_float, _vp]),
    "s2_dit_sample_texts": (ctypes.c_int, [_vp, _vp, _vp, _vp] + [ctypes.c_int] * 3
                            + [_vp, ctypes.c_int, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_float,
                               _vp]),
    "s2_sampler_timesteps": (ctypes.c_int, [ctypes.c_int, _f32p]),
    "s2_apply_cfg_workspace_bytes": (ctypes.c_size_t, []),
    "s2_apply_cfg": (ctypes.c_int, [_vp, _vp, _vp, ctypes.c_longlong, ctypes.c_float, ctypes.c_float, _vp, _vp]),
    "s2_euler_step_to": (ctypes.c_int, [_vp, _vp, _vp, ctypes.c_longlong, ctypes.c_float, ctypes.c_float, _vp]),
    "s2_euler_endpoint": (ctypes.c_int, [_vp, _vp, _vp, ctypes.c_longlong, ctypes.c_float, _vp]),
    "s2_condition_ratio": (ctypes.c_float, [ctypes.c_float, ctypes.c_int, ctypes.c_int, ctypes.c_int]),
    "s2_make_condition": (ctypes.c_int, [_vp, _vp, _vp] + [ctypes.c_int] * 4 + [ctypes.c_float, _vp]),
    "s2_gemm": (ctypes.c_int, [_vp, ctypes.POINTER(GemmDesc), ctypes.POINTER(ctypes.c_int)]),
    "s2_vae_group_norm_create": (ctypes.c_int, [ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_void_p)]),
    "s2_vae_group_norm_destroy": (ctypes.c_int, [_vp]),
    "s2_vae_group_norm_load": (ctypes.c_int, [_vp, _f32p, _f32p]),
    "s2_vae_group_norm_forward": (ctypes.c_int, [_vp, _vp, _vp] + [ctypes.c_int] * 3
                                  + [ctypes.c_longlong, _vp, ctypes.c_longlong]),
    "s2_vae_group_norm_forward_host": (ctypes.c_int, [_vp, _vp, _vp] + [ctypes.c_int] * 3 + [_vp]),
    "s2_vae_group_norm_last_launches": (ctypes.c_int, [_vp]),
    "s2_vae_space_time_shuffle_create": (ctypes.c_int, [ctypes.c_int] * 3 + [ctypes.POINTER(ctypes.c_void_p)]),
    "s2_vae_space_time_shuffle_destroy": (ctypes.c_int, [_vp]),
    "s2_vae_space_time_shuffle_load": (ctypes.c_int, [_vp, _f32p, _f32p]),
    "s2_vae_space_time_shuffle_output_shape": (ctypes.c_int, [_vp] + [ctypes.c_int] * 3 + [_i32p] * 3),
    "s2_vae_space_time_shuffle_forward": (ctypes.c_int, [_vp, _vp, _vp] + [ctypes.c_int] * 3
                                          + [ctypes.c_longlong, _vp, ctypes.c_longlong]),
    "s2_vae_space_time_shuffle_forward_host": (ctypes.c_int, [_vp, _vp, _vp] + [ctypes.c_int] * 3 + [_vp]),
    "s2_vae_space_time_shuffle_last_launches": (ctypes.c_int, [_vp]),
    "s2_vae_space_time_shuffle_device_error": (ctypes.c_int, [_vp, _i32p]),
    "s2_vae_conv3d_create": (ctypes.c_int, [ctypes.c_int] * 18 + [ctypes.c_float, ctypes.c_int,
                                                                  ctypes.POINTER(ctypes.c_void_p)]),
    "s2_vae_conv3d_destroy": (ctypes.c_int, [_vp]),
    "s2_vae_conv3d_load": (ctypes.c_int, [_vp, _f32p, _f32p]),
    "s2_vae_conv3d_output_shape": (ctypes.c_int, [_vp] + [ctypes.c_int] * 3 + [_i32p] * 3),
    "s2_vae_conv3d_forward": (ctypes.c_int, [_vp, _vp, _vp] + [ctypes.c_int] * 3
                              + [ctypes.c_longlong, _vp, ctypes.c_longlong]),
    "s2_vae_conv3d_forward_host": (ctypes.c_int, [_vp, _vp, _vp] + [ctypes.c_int] * 3 + [_vp]),
    "s2_vae_conv3d_last_launches": (ctypes.c_int, [_vp]),
    "s2_vae_conv3d_device_error": (ctypes.c_int, [_vp, _i32p]),
    "s2_debug_fail_allocations": (ctypes.c_int, [ctypes.c_int]),
    "s2_debug_attention_fault": (ctypes.c_int, [ctypes.c_int, ctypes.c_ulonglong]),
    "s2_last_error": (ctypes.c_char_p, []),
    "s2_device_check": (ctypes.c_int, [ctypes.c_int]),
    "s2_version": (ctypes.c_int, []),
}


def lib():
    """Load libs2b200.so (raises if it was not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise FileNotFoundError(f"{LIB_PATH} not built (run __graft_entry__.build())")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def exported_symbols():
    return list(_SIGS)


def last_error() -> str:
    return lib().s2_last_error().decode()


def _check(status: int, what: str = ""):
    if status != S2_OK:
        raise S2Error(status, f"{what}: {last_error()}")


# ---- host planning (runs without a GPU) --------------------------------------

def make_windows(frames, height, width, shifted, override=(0, 0, 0)) -> np.ndarray:
    """Window boxes [n, 6] = (t0, t1, h0, h1, w0, w1), in the reference's order."""
    n = ctypes.c_int32(0)
    _check(lib().s2_make_windows(frames, height, width, int(shifted), *override, None, 0, ctypes.byref(n)),
           "s2_make_windows")
    buf = (Window * max(n.value, 1))()
    _check(lib().s2_make_windows(frames, height, width, int(shifted), *override, buf, n.value, ctypes.byref(n)),
           "s2_make_windows")
    return np.array([[w.t0, w.t1, w.h0, w.h1, w.w0, w.w1] for w in buf[:n.value]], dtype=np.int32).reshape(-1, 6)


def build_varlen(frames, height, width, windows: np.ndarray, text_len: int):
    """(cu_seqlens [n+1] int32, rows [N, 4] int32 = src, pt, ph, pw)."""
    n = len(windows)
    wb = (Window * n)(*[Window(*map(int, w)) for w in windows])
    total = ctypes.c_int32(0)
    _check(lib().s2_build_varlen(frames, height, width, wb, n, text_len, None, None, ctypes.byref(total)),
           "s2_build_varlen")
    cu = np.zeros(n + 1, np.int32)
    rows = np.zeros((max(total.value, 1), 4), np.int32)
    _check(lib().s2_build_varlen(frames, height, width, wb, n, text_len, cu.ctypes.data_as(_i32p),
                                 ctypes.cast(rows.ctypes.data, ctypes.POINTER(Row)), ctypes.byref(total)),
           "s2_build_varlen")
    return cu, rows[:total.value]


def plan_work(cu_seqlens: np.ndarray) -> np.ndarray:
    cu = np.ascontiguousarray(cu_seqlens, np.int32)
    n = ctypes.c_int32(0)
    _check(lib().s2_plan_work(cu.ctypes.data_as(_i32p), len(cu) - 1, None, 0, ctypes.byref(n)), "s2_plan_work")
    work = np.zeros(max(n.value, 1), np.int32)
    _check(lib().s2_plan_work(cu.ctypes.data_as(_i32p), len(cu) - 1, work.ctypes.data_as(_i32p), n.value,
                              ctypes.byref(n)), "s2_plan_work")
    return work[:n.value]


# ---- sampler (EulerSampler, src/model/sampler.cpp) ---------------------------

def sampler_timesteps(steps: int) -> np.ndarray:
    """Timesteps of an n-step Euler schedule, 1000 (1 - i / steps)."""
    out = np.zeros(max(int(steps), 1), np.float32)
    _check(lib().s2_sampler_timesteps(int(steps), out.ctypes.data_as(_f32p)), "s2_sampler_timesteps")
    return out


def condition_ratio(noise_scale: float, frames: int, height: int, width: int) -> float:
    """Mixing ratio of the augmentation noise into the condition latent."""
    return float(lib().s2_condition_ratio(ctypes.c_float(noise_scale), frames, height, width))


def apply_cfg(positive, negative, scale, rescale=0.0, out=None, stream=None):
    """Classifier-free guidance on device fp32 tensors (EulerSampler::apply_cfg)."""
    torch = _torch()
    if out is None:
        out = torch.empty_like(positive)
    ws = None
    if rescale != 0.0:
        ws = torch.empty(int(lib().s2_apply_cfg_workspace_bytes()), dtype=torch.uint8, device=positive.device)
    _check(lib().s2_apply_cfg(_stream_ptr(stream), _ptr(positive), _ptr(negative), positive.numel(),
                              ctypes.c_float(scale), ctypes.c_float(rescale), _ptr(ws), _ptr(out)), "s2_apply_cfg")
    return out


def euler_step_to(prediction, current, timestep, next_timestep, out=None, stream=None):
    """EulerSampler::step_to on device fp32 tensors."""
    torch = _torch()
    if out is None:
        out = torch.empty_like(current)
    _check(lib().s2_euler_step_to(_stream_ptr(stream), _ptr(prediction), _ptr(current), current.numel(),
                                  ctypes.c_float(timestep), ctypes.c_float(next_timestep), _ptr(out)),
           "s2_euler_step_to")
    return out


def euler_endpoint(prediction, current, timestep, out=None, stream=None):
    """EulerSampler::endpoint on device fp32 tensors."""
    torch = _torch()
    if out is None:
        out = torch.empty_like(current)
    _check(lib().s2_euler_endpoint(_stream_ptr(stream), _ptr(prediction), _ptr(current), current.numel(),
                                   ctypes.c_float(timestep), _ptr(out)), "s2_euler_endpoint")
    return out


def make_condition(encoded, noise, noise_scale, out=None, stream=None):
    """Condition latent (1 - r) encoded + r noise on device fp32 [C, T, H, W]."""
    torch = _torch()
    if out is None:
        out = torch.empty_like(encoded)
    C, T, H, W = encoded.shape
    _check(lib().s2_make_condition(_stream_ptr(stream), _ptr(encoded), _ptr(noise), C, T, H, W,
                                   ctypes.c_float(noise_scale), _ptr(out)), "s2_make_condition")
    return out


def window_costs(windows: np.ndarray, text_len: int) -> np.ndarray:
    """Attention cost of each window, proportional to S_w^2 with S_w = L_w + text_len."""
    w = np.asarray(windows)
    s = (w[:, 1] - w[:, 0]) * (w[:, 3] - w[:, 2]) * (w[:, 5] - w[:, 4]) + text_len
    return s.astype(np.float64) ** 2


def shard_windows(windows: np.ndarray, text_len: int, n_ranks: int) -> list[np.ndarray]:
    """Deterministic longest-processing-time assignment of a layer's windows to
    ranks (cost S_w^2, ties to the lowest rank). Every window goes to exactly one
    rank, so every video token has exactly one owner; returns the sorted window
    ids of each rank."""
    costs = window_costs(windows, text_len)
    order = np.argsort(-costs, kind="stable")
    load = np.zeros(n_ranks)
    owner = np.zeros(len(costs), np.int32)
    for i in order:
        r = int(np.argmin(load))
        owner[i] = r
        load[r] += costs[i]
    return [np.nonzero(owner == r)[0].astype(np.int32) for r in range(n_ranks)]


def shard_exchange(grid, text_len: int, n_ranks: int, rank: int, kind: int, override=(0, 0, 0)) -> dict:
    """s2_shard_exchange: rank `rank`'s windows, local rows and row-exchange maps
    from window kind `kind` to the other kind (host planning, no GPU)."""
    T, H, W = grid
    L = T * H * W
    ids, tok = np.zeros(L, np.int32), np.zeros(L, np.int32)
    sc, rc = np.zeros(n_ranks, np.int32), np.zeros(n_ranks, np.int32)
    sr, rr = np.zeros(L, np.int32), np.zeros(L, np.int32)
    nw, nl, moved = ctypes.c_int(0), ctypes.c_int(0), ctypes.c_longlong(0)
    p = lambda a: a.ctypes.data_as(_i32p)  # noqa: E731
    _check(lib().s2_shard_exchange(T, H, W, *override, text_len, n_ranks, rank, kind, p(ids), ctypes.byref(nw),
                                   p(tok), ctypes.byref(nl), p(sc), p(sr), p(rc), p(rr), ctypes.byref(moved)),
           "s2_shard_exchange")
    return {"window_ids": ids[:nw.value].copy(), "local_tokens": tok[:nl.value].copy(), "send_counts": sc,
            "send_rows": sr[:int(sc.sum())].copy(), "recv_counts": rc, "recv_rows": rr[:int(rc.sum())].copy(),
            "moved_rows": moved.value}


def shard_row_destinations(grid, text_len: int, n_ranks: int, rank: int, kind: int, override=(0, 0, 0)):
    """s2_shard_row_destinations: (dest_rank, dest_row) of each of rank `rank`'s
    kind-`kind` local rows under the other kind (host planning, no GPU)."""
    T, H, W = grid
    L = T * H * W
    dr, dw = np.zeros(L, np.int32), np.zeros(L, np.int32)
    nl = ctypes.c_int(0)
    p = lambda a: a.ctypes.data_as(_i32p)  # noqa: E731
    _check(lib().s2_shard_row_destinations(T, H, W, *override, text_len, n_ranks, rank, kind, p(dr), p(dw),
                                           ctypes.byref(nl)), "s2_shard_row_destinations")
    return dr[:nl.value].copy(), dw[:nl.value].copy()


def shard_owners(windows: np.ndarray, text_len: int, n_ranks: int) -> np.ndarray:
    """Owner rank of every window as the library assigns it (s2_shard_windows)."""
    w = np.ascontiguousarray(windows, np.int32)
    owner = np.zeros(len(w), np.int32)
    _check(lib().s2_shard_windows(w.ctypes.data_as(ctypes.POINTER(Window)), len(w), text_len, n_ranks,
                                  owner.ctypes.data_as(_i32p)), "s2_shard_windows")
    return owner


# ---- device helpers (torch tensors as plumbing) ------------------------------

def _torch():
    import torch
    return torch


def _dtype_code(t) -> int:
    torch = _torch()
    return {torch.float32: S2_F32, torch.float16: S2_F16, torch.bfloat16: S2_BF16}[t.dtype]


def _stream_ptr(stream=None):
    torch = _torch()
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def mode_dtype(mode: int):
    torch = _torch()
    return torch.bfloat16 if mode == MODE_BF16_REF else torch.float16


class SeedVR2DiTBlockAttention:
    """The attention stage of SeedVR2DiTBlock on a B200 (drop-in for attention()).

    ``load_param`` takes the reference's ParamDict keys; ``load_model`` the
    QK-norm gammas of the video and text branches and the RoPE freqs;
    ``forward`` takes device tensors vid_qkv [L, 3*dim] and txt_qkv [Lt, 3*dim]
    and returns (vid_out [L, dim] in the mode dtype, txt_out [Lt, dim] fp32).
    Errors raise S2Error carrying the reference-style status code.
    """

    def __init__(self, device: int = 0, mode: int = MODE_BF16_REF, window_override=(0, 0, 0)):
        self.device = device
        self.mode = mode
        self.window_override = tuple(int(x) for x in window_override)
        self.handle = None
        self.heads = 20
        self.shifted = False
        self.shape = None

    # ParamDict keys 0..8 (seedvr2_dit_block.cpp:643-655)
    def load_param(self, block_index=0, shared=False, last=False, shifted=False, dim=2560, heads=20, head_dim=128,
                   mlp_hidden=6912, eps=1e-5):
        if dim != heads * head_dim:
            return S2_INVALID_ARGUMENT
        self.heads, self.shifted, self.eps = heads, bool(shifted), float(eps)
        h = ctypes.c_void_p()
        _check(lib().s2_attention_layer_create(self.device, heads, head_dim, ctypes.c_float(eps), int(shifted),
                                               *self.window_override, self.mode, ctypes.byref(h)),
               "s2_attention_layer_create")
        self.close()
        self.handle = h
        return S2_OK

    def load_model(self, norm_q_vid, norm_k_vid, freqs21, norm_q_txt=None, norm_k_txt=None):
        """Shared blocks (>= 10) pass no text gammas: the video branch is reused."""
        g = [np.ascontiguousarray(x, np.float32) for x in
             (norm_q_vid, norm_k_vid, norm_q_vid if norm_q_txt is None else norm_q_txt,
              norm_k_vid if norm_k_txt is None else norm_k_txt, freqs21)]
        _check(lib().s2_attention_layer_load(self.handle, *[x.ctypes.data_as(_f32p) for x in g]),
               "s2_attention_layer_load")
        self._keep = g
        return S2_OK

    def set_runtime_shape(self, frames, height, width):
        _check(lib().s2_attention_layer_set_runtime_shape(self.handle, frames, height, width), "set_runtime_shape")
        self.shape = (frames, height, width)

    def set_window_subset(self, ids=None):
        ids = np.ascontiguousarray([] if ids is None else ids, np.int32)
        _check(lib().s2_attention_layer_set_window_subset(self.handle, ids.ctypes.data_as(_i32p) if ids.size else None,
                                                          int(ids.size)), "set_window_subset")

    def forward(self, vid_qkv, txt_qkv, vid_out=None, txt_out=None, stream=None):
        torch = _torch()
        dim = self.heads * HEAD_DIM
        L, Lt = vid_qkv.shape[0], txt_qkv.shape[0]
        if vid_out is None:
            vid_out = torch.zeros((L, dim), dtype=mode_dtype(self.mode), device=vid_qkv.device)
        if txt_out is None:
            txt_out = torch.empty((Lt, dim), dtype=torch.float32, device=vid_qkv.device)
        _check(lib().s2_attention_layer_forward(self.handle, _stream_ptr(stream), _ptr(vid_qkv), _dtype_code(vid_qkv),
                                                L, _ptr(txt_qkv), Lt, _ptr(vid_out), _ptr(txt_out)),
               "s2_attention_layer_forward")
        return vid_out, txt_out

    def forward_host(self, vid_qkv: np.ndarray, txt_qkv: np.ndarray, vid_shape, io_dtype=S2_F32,
                     vid_out: np.ndarray | None = None, txt_out: np.ndarray | None = None, stream=None):
        """ncnn::Mat-style host buffers in, host buffers out (copies inside)."""
        dim = self.heads * HEAD_DIM
        L, Lt = vid_qkv.shape[0], txt_qkv.shape[0]
        np_out = {S2_F32: np.float32, S2_F16: np.float16, S2_BF16: np.uint16}[io_dtype]
        if vid_out is None:
            vid_out = np.zeros((L, dim), np_out)
        if txt_out is None:
            txt_out = np.zeros((Lt, dim), np.float32)
        shape = np.ascontiguousarray(vid_shape, np.int32)
        _check(lib().s2_attention_layer_forward_host(
            self.handle, _stream_ptr(stream) if stream is not None else None, ctypes.c_void_p(vid_qkv.ctypes.data),
            ctypes.c_void_p(txt_qkv.ctypes.data), io_dtype, L, Lt, shape.ctypes.data_as(_i32p),
            ctypes.c_void_p(vid_out.ctypes.data), ctypes.c_void_p(txt_out.ctypes.data)), "forward_host")
        return vid_out, txt_out

    def last_launches(self) -> int:
        return lib().s2_attention_layer_last_launches(self.handle)

    def device_error(self) -> int:
        code = ctypes.c_int32(0)
        lib().s2_attention_layer_device_error(self.handle, ctypes.byref(code))
        return code.value

    def close(self):
        if self.handle is not None and self.handle.value:
            lib().s2_attention_layer_destroy(self.handle)
        self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ---- explicit-buffer kernel entry points -------------------------------------

def rope_table(freqs21, max_pos, stream=None):
    torch = _torch()
    tab = torch.empty(lib().s2_rope_table_bytes(max_pos) // 4, dtype=torch.float32, device=freqs21.device)
    _check(lib().s2_rope_table(_stream_ptr(stream), _ptr(freqs21), max_pos, _ptr(tab)), "s2_rope_table")
    return tab


def qk_norm_rope(vid_qkv, txt_qkv, heads, gammas, table, rows, mode=MODE_BF16_REF, eps=1e-5, stream=None):
    """Returns packed (q, k, v), each fp16 [heads, n_rows, 128] holding the bf16-rounded values."""
    torch = _torch()
    n_rows = rows.shape[0]
    out = [torch.empty((heads, n_rows, HEAD_DIM), dtype=torch.float16, device=vid_qkv.device) for _ in range(3)]
    _check(lib().s2_qk_norm_rope(_stream_ptr(stream), _ptr(vid_qkv), _ptr(txt_qkv), _dtype_code(vid_qkv), heads,
                                 ctypes.c_float(eps), _ptr(gammas), _ptr(table), _ptr(rows), n_rows, mode,
                                 *[_ptr(t) for t in out]), "s2_qk_norm_rope")
    return out


def window_attention(q, k, v, cu_seqlens, text_len, rows, work, vid_out, txt_partial, err, mode=MODE_BF16_REF,
                     stream=None):
    heads, n_rows = q.shape[0], q.shape[1]
    _check(lib().s2_window_attention(_stream_ptr(stream), mode, _ptr(q), _ptr(k), _ptr(v), heads, n_rows,
                                     _ptr(cu_seqlens), cu_seqlens.shape[0] - 1, text_len, _ptr(rows), _ptr(work),
                                     work.shape[0], _ptr(vid_out), _ptr(txt_partial), _ptr(err)),
           "s2_window_attention")


def text_window_sum(txt_partial, n_windows, text_len, dim, scale, txt_out, accumulate=False, mode=MODE_BF16_REF,
                    stream=None):
    _check(lib().s2_text_window_sum(_stream_ptr(stream), mode, _ptr(txt_partial), n_windows, text_len, dim,
                                    ctypes.c_float(scale), int(accumulate), _ptr(txt_out)), "s2_text_window_sum")


def gemm(epilogue, a, b, *, bias=None, gmul=None, resid=None, resid2=None, outs=(), y=None, y2=None, split=0,
         split_row=0, out_scale=1.0, workspace=None, err=None, stream=None, row_dest=None) -> int:
    """s2_gemm: the block's InnerProduct on tcgen05 (a [M][K], b [N][K] fp16 CUDA
    tensors). Returns the number of extra kernels launched (split-K finish).
    err: device int32 error word (a zeroed one is made when None). row_dest:
    device int32 [rows][2] of {0, destination row of y} (gated residual only)."""
    if err is None:
        err = _torch().zeros(1, dtype=_torch().int32, device=a.device)
    M, K = a.shape
    N = b.shape[0]
    o = list(outs) + [None] * (3 - len(outs))

    def _ptr(t):
        return None if t is None else t.data_ptr()

    d = GemmDesc(epilogue=int(epilogue), M=M, N=N, K=K, a=_ptr(a), b=_ptr(b), bias=_ptr(bias), gmul=_ptr(gmul),
                 resid=_ptr(resid), resid2=_ptr(resid2), out0=_ptr(o[0]), out1=_ptr(o[1]), out2=_ptr(o[2]),
                 y=_ptr(y), y2=_ptr(y2), split=int(split), split_row=int(split_row), out_scale=float(out_scale),
                 workspace=_ptr(workspace), workspace_floats=0 if workspace is None else workspace.numel(),
                 err=_ptr(err), row_dest=_ptr(row_dest))
    extra = ctypes.c_int(0)
    _check(lib().s2_gemm(_stream_ptr(stream), ctypes.byref(d), ctypes.byref(extra)), "s2_gemm")
    return extra.value


def block_flags(index: int, n_blocks: int = 32) -> dict:
    """Per-block flags of the exported model (shared weights from block 10 on,
    odd blocks shifted, the final block last)."""
    return dict(shared=index >= 10, shifted=index % 2 == 1, last=index == n_blocks - 1)


class SeedVR2DiT:
    """The DiT on a B200: input head, blocks, output head, and one Euler step.

    ``load_input`` / ``load_block`` / ``load_output`` take the host fp32
    weight streams in the reference's load orders; ``forward`` the 33-channel
    latent; ``euler_step`` noise + condition latents and the text embedding
    (device tensors), ``euler_step_host`` the same on numpy arrays.
    """

    def __init__(self, device=0, n_blocks=32, dim=2560, heads=20, head_dim=128, mlp_hidden=6912, eps=1e-5,
                 video_channels=33, text_channels=5120, sinusoidal_dim=256, out_channels=16, window_override=(0, 0, 0)):
        h = ctypes.c_void_p()
        _check(lib().s2_dit_create(device, n_blocks, dim, heads, head_dim, mlp_hidden, ctypes.c_float(eps),
                                   video_channels, text_channels, sinusoidal_dim, out_channels,
                                   *[int(x) for x in window_override], ctypes.byref(h)), "s2_dit_create")
        self.handle = h
        self.n_blocks, self.dim, self.out_channels, self.text_channels = n_blocks, dim, out_channels, text_channels

    def input_weight_count(self) -> int:
        return int(lib().s2_dit_input_weight_count(self.handle))

    def output_weight_count(self) -> int:
        return int(lib().s2_dit_output_weight_count(self.handle))

    def load_input(self, weights):
        w = np.ascontiguousarray(weights, np.float32).ravel()
        _check(lib().s2_dit_load_input(self.handle, w.ctypes.data_as(_f32p), w.size), "s2_dit_load_input")

    def load_block(self, index, weights, shared=None, last=None, shifted=None):
        f = block_flags(index, self.n_blocks)
        f.update({k: v for k, v in dict(shared=shared, last=last, shifted=shifted).items() if v is not None})
        w = np.ascontiguousarray(weights, np.float32).ravel()
        _check(lib().s2_dit_load_block(self.handle, index, int(f["shared"]), int(f["last"]), int(f["shifted"]),
                                       w.ctypes.data_as(_f32p), w.size), "s2_dit_load_block")

    def load_output(self, weights):
        w = np.ascontiguousarray(weights, np.float32).ravel()
        _check(lib().s2_dit_load_output(self.handle, w.ctypes.data_as(_f32p), w.size), "s2_dit_load_output")

    def load_dir(self, model_dir: str):
        """Loads the reference's exported model directory (SeedVR2DiT::load)."""
        _check(lib().s2_dit_load_dir(self.handle, os.fsencode(model_dir)), "s2_dit_load_dir")

    def forward(self, latent, text, timestep, prediction=None, stream=None):
        torch = _torch()
        vc, T, H, W = latent.shape
        if prediction is None:
            prediction = torch.empty((self.out_channels, T, H, W), dtype=torch.float32, device=latent.device)
        _check(lib().s2_dit_forward(self.handle, _stream_ptr(stream), _ptr(latent), T, H, W, _ptr(text),
                                    text.shape[0], ctypes.c_float(timestep), _ptr(prediction)), "s2_dit_forward")
        return prediction

    def euler_step(self, noise, condition, text, timestep=1000.0, x0=None, stream=None):
        torch = _torch()
        _, T, H, W = noise.shape
        if x0 is None:
            x0 = torch.empty_like(noise)
        _check(lib().s2_dit_euler_step(self.handle, _stream_ptr(stream), _ptr(noise), _ptr(condition), T, H, W,
                                       _ptr(text), text.shape[0], ctypes.c_float(timestep), _ptr(x0)),
               "s2_dit_euler_step")
        return x0

    def euler_step_host(self, noise, condition, text, timestep=1000.0, x0=None, stream=None):
        noise, condition, text = (np.ascontiguousarray(a, np.float32) for a in (noise, condition, text))
        _, T, H, W = noise.shape
        if x0 is None:
            x0 = np.empty_like(noise)
        _check(lib().s2_dit_euler_step_host(self.handle, _stream_ptr(stream) if stream is not None else None,
                                            ctypes.c_void_p(noise.ctypes.data), ctypes.c_void_p(condition.ctypes.data),
                                            T, H, W, ctypes.c_void_p(text.ctypes.data), text.shape[0],
                                            ctypes.c_float(timestep), ctypes.c_void_p(x0.ctypes.data)),
               "s2_dit_euler_step_host")
        return x0

    def sample(self, noise, condition, positive_text, negative_text=None, steps=1, cfg_scale=1.0, cfg_rescale=0.0,
               out=None, stream=None):
        """The engine's sampling loop (engine.cpp:308-347): ``steps`` Euler
        steps from ``noise``, with classifier-free guidance against
        ``negative_text`` when ``cfg_scale != 1``. Device fp32 tensors; returns
        the final latent (x0)."""
        torch = _torch()
        _, T, H, W = noise.shape
        if out is None:
            out = torch.empty_like(noise)
        neg_len = negative_text.shape[0] if negative_text is not None else 0
        _check(lib().s2_dit_sample_texts(self.handle, _stream_ptr(stream), _ptr(noise), _ptr(condition), T, H, W,
                                         _ptr(positive_text), positive_text.shape[0], _ptr(negative_text), neg_len,
                                         int(steps), ctypes.c_float(cfg_scale), ctypes.c_float(cfg_rescale),
                                         _ptr(out)),
               "s2_dit_sample_texts")
        return out

    def set_comm(self, comm: "Comm | None"):
        """Shard the step over the communicator's ranks (None: this GPU alone)."""
        self._comm = comm
        _check(lib().s2_dit_set_comm(self.handle, comm.handle if comm is not None else None), "s2_dit_set_comm")

    def set_graph(self, enable: bool):
        _check(lib().s2_dit_set_graph(self.handle, int(enable)), "s2_dit_set_graph")

    def last_launches(self) -> int:
        return lib().s2_dit_last_launches(self.handle)

    def device_error(self) -> int:
        code = ctypes.c_int32(0)
        lib().s2_dit_device_error(self.handle, ctypes.byref(code))
        return code.value

    def close(self):
        if self.handle is not None and self.handle.value:
            lib().s2_dit_destroy(self.handle)
        self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class SeedVR2DiTBlock:
    """One DiT block on a B200 (drop-in for the ncnn layer's forward).

    ``load_param`` takes the reference's ParamDict keys 0..8, ``load_model``
    the flat fp32 weight stream in the reference's load order,
    ``set_runtime_shape`` the token grid; ``forward`` takes device fp32
    tensors vid [L, dim], txt [Lt, dim], emb [6*dim] and returns
    (vid_out, txt_out); ``forward_host`` the same on numpy arrays with the
    vid_shape blob. Errors raise S2Error with the reference-style status.
    """

    def __init__(self, device: int = 0, window_override=(0, 0, 0)):
        self.device = device
        self.window_override = tuple(int(x) for x in window_override)
        self.handle = None
        self.dim = 0

    def load_param(self, block_index=0, shared=False, last=False, shifted=False, dim=2560, heads=20, head_dim=128,
                   mlp_hidden=6912, eps=1e-5):
        h = ctypes.c_void_p()
        _check(lib().s2_dit_block_create(self.device, block_index, int(shared), int(last), int(shifted), dim, heads,
                                         head_dim, mlp_hidden, ctypes.c_float(eps), *self.window_override,
                                         ctypes.byref(h)), "s2_dit_block_create")
        self.close()
        self.handle, self.dim = h, dim
        return S2_OK

    def weight_count(self) -> int:
        return int(lib().s2_dit_block_weight_count(self.handle))

    def load_model(self, weights):
        w = np.ascontiguousarray(weights, np.float32).ravel()
        _check(lib().s2_dit_block_load(self.handle, w.ctypes.data_as(_f32p), w.size), "s2_dit_block_load")
        return S2_OK

    def set_runtime_shape(self, frames, height, width):
        _check(lib().s2_dit_block_set_runtime_shape(self.handle, frames, height, width), "set_runtime_shape")

    def set_window_subset(self, ids=None):
        ids = np.ascontiguousarray([] if ids is None else ids, np.int32)
        _check(lib().s2_dit_block_set_window_subset(self.handle, ids.ctypes.data_as(_i32p) if ids.size else None,
                                                    int(ids.size)), "set_window_subset")

    def forward(self, vid, txt, emb, vid_out=None, txt_out=None, stream=None):
        torch = _torch()
        L, Lt = vid.shape[0], (txt.shape[0] if txt is not None else 0)
        if vid_out is None:
            vid_out = torch.empty_like(vid)
        if txt_out is None and Lt:
            txt_out = torch.empty_like(txt)
        _check(lib().s2_dit_block_forward(self.handle, _stream_ptr(stream), _ptr(vid), L,
                                          _ptr(txt) if Lt else None, Lt, _ptr(emb), _ptr(vid_out),
                                          _ptr(txt_out) if Lt else None), "s2_dit_block_forward")
        return vid_out, txt_out

    def forward_host(self, vid: np.ndarray, txt: np.ndarray, emb: np.ndarray, vid_shape, stream=None):
        vid, txt, emb = (np.ascontiguousarray(a, np.float32) for a in (vid, txt, emb))
        vo, to = np.empty_like(vid), np.empty_like(txt)
        shape = np.ascontiguousarray(vid_shape, np.int32)
        _check(lib().s2_dit_block_forward_host(self.handle, _stream_ptr(stream) if stream is not None else None,
                                               ctypes.c_void_p(vid.ctypes.data), vid.shape[0],
                                               ctypes.c_void_p(txt.ctypes.data), txt.shape[0],
                                               ctypes.c_void_p(emb.ctypes.data), shape.ctypes.data_as(_i32p),
                                               ctypes.c_void_p(vo.ctypes.data), ctypes.c_void_p(to.ctypes.data)),
               "s2_dit_block_forward_host")
        return vo, to

    def debug_rows(self, text_len: int) -> int:
        n = ctypes.c_int32(0)
        _check(lib().s2_dit_block_debug_rows(self.handle, int(text_len), ctypes.byref(n)), "s2_dit_block_debug_rows")
        return n.value

    def set_debug_tensors(self, L: int, text_len: int, names=DEBUG_TENSORS):
        """set_debug_tensors (seedvr2_dit_block.h:58): allocate device fp32
        buffers for the named capture points and return them as a dict; the
        next forwards fill them. None switches capturing off."""
        if names is None:
            _check(lib().s2_dit_block_set_debug_tensors(self.handle, None), "s2_dit_block_set_debug_tensors")
            self._debug = None
            return None
        torch = _torch()
        d, rows = self.dim, self.debug_rows(text_len)
        shapes = {"qkv_vid": (L, 3 * d), "qkv_txt": (text_len, 3 * d), "norm_q_vid": (L, d), "norm_k_vid": (L, d),
                  "norm_q_txt": (text_len, d), "norm_k_txt": (text_len, d), "attention_q": (rows, d),
                  "attention_k": (rows, d), "attention_v": (rows, d), "attention_output": (rows, d),
                  "projected_vid": (L, d), "projected_txt": (text_len, d), "output_vid": (L, d),
                  "output_txt": (text_len, d)}
        bufs = {n: torch.zeros(shapes[n], dtype=torch.float32, device=f"cuda:{self.device}") for n in names}
        dbg = BlockDebug(**{n: t.data_ptr() for n, t in bufs.items()})
        _check(lib().s2_dit_block_set_debug_tensors(self.handle, ctypes.byref(dbg)), "s2_dit_block_set_debug_tensors")
        self._debug = bufs
        return bufs

    def last_launches(self) -> int:
        return lib().s2_dit_block_last_launches(self.handle)

    def device_error(self) -> int:
        code = ctypes.c_int32(0)
        lib().s2_dit_block_device_error(self.handle, ctypes.byref(code))
        return code.value

    def close(self):
        if self.handle is not None and self.handle.value:
            lib().s2_dit_block_destroy(self.handle)
        self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


COMM_ID_BYTES = 128


class Comm:
    """One rank of the library's multi-GPU communicator (NCCL, loaded on first use).

    ``Comm.create(device, rank, world, pg=None)`` makes rank 0's unique id and
    broadcasts it with torch.distributed (the default process group unless
    ``pg`` is given); pass ``unique_id`` to supply the bytes yourself."""

    def __init__(self, device: int, rank: int, world: int, unique_id: bytes):
        h = ctypes.c_void_p()
        _check(lib().s2_comm_init(device, world, rank, ctypes.create_string_buffer(unique_id, COMM_ID_BYTES),
                                  ctypes.byref(h)), "s2_comm_init")
        self.handle, self.rank, self.world = h, rank, world

    @staticmethod
    def unique_id() -> bytes:
        buf = ctypes.create_string_buffer(COMM_ID_BYTES)
        _check(lib().s2_comm_unique_id(buf), "s2_comm_unique_id")
        return buf.raw

    @classmethod
    def create(cls, device: int, rank: int, world: int, pg=None):
        torch = _torch()
        import torch.distributed as dist
        uid = cls.unique_id() if rank == 0 else bytes(COMM_ID_BYTES)
        t = torch.tensor(list(uid), dtype=torch.uint8)
        if dist.get_backend(pg) == "nccl":
            t = t.cuda(device)
        dist.broadcast(t, 0, group=pg)
        return cls(device, rank, world, bytes(t.cpu().tolist()))

    def set_timeout(self, ms: int):
        """Deadline of this communicator's host-side waits (s2_comm_set_timeout)."""
        _check(lib().s2_comm_set_timeout(self.handle, int(ms)), "s2_comm_set_timeout")

    def close(self):
        if self.handle is not None and self.handle.value:
            lib().s2_comm_destroy(self.handle)
        self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _read_ncnn(fn, ptype, param_path, bin_path):
    p = ptype()
    n = ctypes.c_size_t(0)
    _check(fn(os.fsencode(param_path), os.fsencode(bin_path), ctypes.byref(p), None, 0, ctypes.byref(n)), fn.__name__)
    w = np.zeros(n.value, np.float32)
    _check(fn(os.fsencode(param_path), os.fsencode(bin_path), ctypes.byref(p), w.ctypes.data_as(_f32p), w.size,
              ctypes.byref(n)), fn.__name__)
    return {f: getattr(p, f) for f, _ in ptype._fields_}, w


def read_ncnn_block(param_path, bin_path):
    """(ParamDict values, fp32 weight stream) of an exported SeedVR2DiTBlock."""
    return _read_ncnn(lib().s2_ncnn_read_block, BlockParams, param_path, bin_path)


def read_ncnn_input(param_path, bin_path):
    return _read_ncnn(lib().s2_ncnn_read_input, HeadParams, param_path, bin_path)


def read_ncnn_output(param_path, bin_path):
    return _read_ncnn(lib().s2_ncnn_read_output, HeadParams, param_path, bin_path)


def padded_channels(channels: int) -> int:
    """Head dim the spatial attention runs at: channels padded to 128, 256 or 512."""
    return 128 if channels <= 128 else (256 if channels <= 256 else 512)


def spatial_attention(q, k, v, channels, frames, tokens, out, err, stream=None):
    """Per-frame single-head attention; q/k/v/out fp16 [frames*tokens, padded_channels(channels)]."""
    _check(lib().s2_spatial_attention(_stream_ptr(stream), _ptr(q), _ptr(k), _ptr(v), channels, q.shape[1], frames,
                                      tokens, _ptr(out), _ptr(err)), "s2_spatial_attention")


VAE_WEIGHT_ORDER = ("norm_bias", "norm_weight", "k_bias", "k_weight", "out_bias", "out_weight", "q_bias", "q_weight",
                    "v_bias", "v_weight")


class DynamicFramewiseSpatialAttention:
    """The VAE mid-block attention layer on a B200 (drop-in for the ncnn layer's forward).

    ``load_param(channels)`` / ``load_model(weights)`` take what the reference's
    ParamDict key 10 and ModelBin hold (weights: a dict by name, or the flat
    fp32 stream in the reference's load order); ``forward`` takes a device fp32
    tensor x [C, T, H, W] (or an ncnn [C, cstep] blob with ``shape``) and
    returns y of the same layout; ``forward_host`` does the same on numpy
    arrays. Errors raise S2Error with the reference-style status code.
    """

    def __init__(self, device: int = 0):
        self.device = device
        self.handle = None
        self.channels = 0

    def load_param(self, channels: int):
        h = ctypes.c_void_p()
        _check(lib().s2_vae_attention_create(self.device, int(channels), ctypes.byref(h)), "s2_vae_attention_create")
        self.close()
        self.handle, self.channels = h, int(channels)
        return S2_OK

    def load_model(self, weights):
        C = self.channels
        if not isinstance(weights, dict):
            flat = np.ascontiguousarray(weights, np.float32).ravel()
            sizes = [C if name.endswith("bias") or name == "norm_weight" else C * C for name in VAE_WEIGHT_ORDER]
            if flat.size != sum(sizes):
                raise S2Error(S2_INVALID_ARGUMENT, f"load_model: {flat.size} floats, expected {sum(sizes)}")
            offs = np.cumsum([0] + sizes)
            weights = {n: flat[offs[i]:offs[i + 1]] for i, n in enumerate(VAE_WEIGHT_ORDER)}
        arrs = [np.ascontiguousarray(weights[n], np.float32).ravel() for n in VAE_WEIGHT_ORDER]
        _check(lib().s2_vae_attention_load(self.handle, *[a.ctypes.data_as(_f32p) for a in arrs]),
               "s2_vae_attention_load")
        self._keep = arrs
        return S2_OK

    def forward(self, x, y=None, shape=None, stream=None):
        """x: device fp32 [C, T, H, W], or [C, cstep] with shape=(T, H, W)."""
        torch = _torch()
        if shape is None:
            C, T, H, W = x.shape
            cstep = T * H * W
        else:
            (T, H, W), C, cstep = shape, x.shape[0], x.shape[1]
        if y is None:
            y = torch.empty_like(x)
        _check(lib().s2_vae_attention_forward(self.handle, _stream_ptr(stream), _ptr(x), T, H, W, cstep, _ptr(y)),
               "s2_vae_attention_forward")
        return y

    def forward_host(self, x: np.ndarray, stream=None, y: np.ndarray | None = None) -> np.ndarray:
        """x: host fp32 [C, T, H, W] -> y (copies in and out, synchronises);
        y may be given (e.g. pinned host memory)."""
        x = np.ascontiguousarray(x, np.float32)
        C, T, H, W = x.shape
        if y is None:
            y = np.empty_like(x)
        elif y.shape != x.shape or y.dtype != np.float32 or not y.flags["C_CONTIGUOUS"]:
            raise ValueError("y must be a contiguous fp32 array of x's shape")
        _check(lib().s2_vae_attention_forward_host(self.handle, _stream_ptr(stream) if stream is not None else None,
                                                   ctypes.c_void_p(x.ctypes.data), T, H, W, T * H * W,
                                                   ctypes.c_void_p(y.ctypes.data)), "s2_vae_attention_forward_host")
        return y

    def last_launches(self) -> int:
        return lib().s2_vae_attention_last_launches(self.handle)

    def device_error(self) -> int:
        code = ctypes.c_int32(0)
        lib().s2_vae_attention_device_error(self.handle, ctypes.byref(code))
        return code.value

    def close(self):
        if self.handle is not None and self.handle.value:
            lib().s2_vae_attention_destroy(self.handle)
        self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def device_check(device: int = 0) -> int:
    return lib().s2_device_check(device)


class _VaeLayer:
    """Common plumbing of the VAE layers on ncnn 4-D blobs (fp32 [C, T, H, W])."""

    _prefix = ""

    def __init__(self, device: int = 0):
        self.device = device
        self.handle = None
        self._keep = ()

    def _out_shape(self, T, H, W):
        return T, H, W

    def _out_channels(self):
        raise NotImplementedError

    def forward(self, x, y=None, stream=None):
        """x: device fp32 [C, T, H, W] -> y [C_out, T', H', W'] (new tensor unless given)."""
        torch = _torch()
        C, T, H, W = x.shape
        oT, oH, oW = self._out_shape(T, H, W)
        if y is None:
            y = torch.empty((self._out_channels(), oT, oH, oW), dtype=torch.float32, device=x.device)
        _check(getattr(lib(), self._prefix + "_forward")(self.handle, _stream_ptr(stream), _ptr(x), T, H, W, T * H * W,
                                                          _ptr(y), oT * oH * oW), self._prefix + "_forward")
        return y

    def forward_host(self, x: np.ndarray, stream=None) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        C, T, H, W = x.shape
        oT, oH, oW = self._out_shape(T, H, W)
        y = np.empty((self._out_channels(), oT, oH, oW), np.float32)
        _check(getattr(lib(), self._prefix + "_forward_host")(
            self.handle, _stream_ptr(stream) if stream is not None else None, ctypes.c_void_p(x.ctypes.data), T, H, W,
            ctypes.c_void_p(y.ctypes.data)), self._prefix + "_forward_host")
        return y

    def last_launches(self) -> int:
        return getattr(lib(), self._prefix + "_last_launches")(self.handle)

    def close(self):
        if self.handle is not None and self.handle.value:
            getattr(lib(), self._prefix + "_destroy")(self.handle)
        self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class DynamicFramewiseGroupNorm(_VaeLayer):
    """The VAE's framewise GroupNorm (src/layers/dynamic_framewise_group_norm.cpp):
    load_param(channels) (ParamDict key 10), load_model(bias, weight), forward."""

    _prefix = "s2_vae_group_norm"

    def load_param(self, channels: int):
        h = ctypes.c_void_p()
        _check(lib().s2_vae_group_norm_create(self.device, int(channels), ctypes.byref(h)), "s2_vae_group_norm_create")
        self.close()
        self.handle, self.channels = h, int(channels)
        return S2_OK

    def load_model(self, bias, weight):
        b, w = (np.ascontiguousarray(a, np.float32).ravel() for a in (bias, weight))
        _check(lib().s2_vae_group_norm_load(self.handle, b.ctypes.data_as(_f32p), w.ctypes.data_as(_f32p)),
               "s2_vae_group_norm_load")
        return S2_OK

    def _out_channels(self):
        return self.channels


class DynamicSpaceTimeShuffle(_VaeLayer):
    """The VAE decoder's space-time shuffle (src/layers/dynamic_space_time_shuffle.cpp):
    load_param(in_channels, projected_channels) (ParamDict keys 11 and 10),
    load_model(bias [P], weight [P, in]), forward -> [in, T', 2H, 2W]."""

    _prefix = "s2_vae_space_time_shuffle"

    def load_param(self, in_channels: int, projected_channels: int):
        h = ctypes.c_void_p()
        _check(lib().s2_vae_space_time_shuffle_create(self.device, int(in_channels), int(projected_channels),
                                                      ctypes.byref(h)), "s2_vae_space_time_shuffle_create")
        self.close()
        self.handle, self.in_channels, self.projected = h, int(in_channels), int(projected_channels)
        return S2_OK

    def load_model(self, bias, weight):
        b, w = (np.ascontiguousarray(a, np.float32).ravel() for a in (bias, weight))
        _check(lib().s2_vae_space_time_shuffle_load(self.handle, b.ctypes.data_as(_f32p), w.ctypes.data_as(_f32p)),
               "s2_vae_space_time_shuffle_load")
        return S2_OK

    def _out_shape(self, T, H, W):
        o = [ctypes.c_int32(0) for _ in range(3)]
        _check(lib().s2_vae_space_time_shuffle_output_shape(self.handle, T, H, W, *[ctypes.byref(v) for v in o]),
               "s2_vae_space_time_shuffle_output_shape")
        return tuple(v.value for v in o)

    def _out_channels(self):
        return self.in_channels

    def device_error(self) -> int:
        code = ctypes.c_int32(0)
        lib().s2_vae_space_time_shuffle_device_error(self.handle, ctypes.byref(code))
        return code.value


class Convolution3D(_VaeLayer):
    """ncnn's Convolution3D as the VAE uses it (the layer the reference patches,
    patches/0001-feat-Convolution3D-Vulkan-pack1.patch). load_param takes the
    layer's ParamDict fields; load_model(weight [out, in, kd, kh, kw], bias)."""

    _prefix = "s2_vae_conv3d"

    def load_param(self, in_channels, num_output, kernel=(3, 3, 3), dilation=(1, 1, 1), stride=(1, 1, 1),
                   pad=(0, 0, 0, 0, 0, 0), pad_value=0.0, bias_term=True):
        """pad = (front, top, left, behind, bottom, right), or all -233 / -234 (SAME)."""
        h = ctypes.c_void_p()
        _check(lib().s2_vae_conv3d_create(self.device, int(in_channels), int(num_output), *map(int, kernel),
                                          *map(int, dilation), *map(int, stride), *map(int, pad),
                                          ctypes.c_float(pad_value), int(bool(bias_term)), ctypes.byref(h)),
               "s2_vae_conv3d_create")
        self.close()
        self.handle, self.in_channels, self.num_output, self.bias_term = h, int(in_channels), int(num_output), bias_term
        return S2_OK

    def load_model(self, weight, bias=None):
        w = np.ascontiguousarray(weight, np.float32).ravel()
        b = None if bias is None else np.ascontiguousarray(bias, np.float32).ravel()
        _check(lib().s2_vae_conv3d_load(self.handle, w.ctypes.data_as(_f32p),
                                        None if b is None else b.ctypes.data_as(_f32p)), "s2_vae_conv3d_load")
        return S2_OK

    def _out_shape(self, T, H, W):
        o = [ctypes.c_int32(0) for _ in range(3)]
        _check(lib().s2_vae_conv3d_output_shape(self.handle, T, H, W, *[ctypes.byref(v) for v in o]),
               "s2_vae_conv3d_output_shape")
        return tuple(v.value for v in o)

    def _out_channels(self):
        return self.num_output

    def device_error(self) -> int:
        code = ctypes.c_int32(0)
        lib().s2_vae_conv3d_device_error(self.handle, ctypes.byref(code))
        return code.value

