"""ctypes binding of ``libbeatlm_b200.so`` (the C ABI in
``include/beatlm_b200.h``).

The library is loaded from this directory only; there is no fallback: if it
is missing or fails to load, every call raises. Build it with
``python -m beatlm_b200.build``.
"""
from __future__ import annotations

import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libbeatlm_b200.so")

BL_OK = 0
BL_F32, BL_F16, BL_BF16 = 0, 1, 2

_lock = threading.Lock()
_lib = None


class BackendError(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, code: int, message: str):
        super().__init__("beatlm_b200 error %d: %s" % (code, message))
        self.code = code


class AttentionArgs(ctypes.Structure):
    _fields_ = [
        ("batch", ctypes.c_uint32), ("tokens", ctypes.c_uint32), ("heads", ctypes.c_uint32),
        ("head_dim", ctypes.c_uint32), ("head_begin", ctypes.c_uint32),
        ("head_end", ctypes.c_uint32), ("row_begin", ctypes.c_uint32),
        ("row_end", ctypes.c_uint32), ("scale", ctypes.c_float), ("qk_dtype", ctypes.c_int32),
        ("v_dtype", ctypes.c_int32), ("out_dtype", ctypes.c_int32), ("qkv", ctypes.c_void_p),
        ("qkv_row_stride", ctypes.c_uint64), ("out", ctypes.c_void_p),
        ("out_row_stride", ctypes.c_uint64), ("out_head_base", ctypes.c_uint32),
        ("kv_splits", ctypes.c_uint32), ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_uint64), ("trace", ctypes.c_void_p),
        ("query_tiles", ctypes.c_uint32),
    ]


class Status(ctypes.Structure):
    _fields_ = [("code", ctypes.c_uint32), ("block", ctypes.c_uint32),
                ("where", ctypes.c_uint32), ("count", ctypes.c_uint32)]


# name -> (restype, argtypes), every symbol include/beatlm_b200.h declares.
SIGNATURES = {
    "bl_last_error": (ctypes.c_size_t, [ctypes.c_char_p, ctypes.c_size_t]),
    "bl_version": (ctypes.c_char_p, []),
    "bl_status": (ctypes.c_int, [ctypes.POINTER(Status), ctypes.c_int]),
    "bl_attention": (ctypes.c_int, [ctypes.POINTER(AttentionArgs), ctypes.c_void_p]),
    "bl_attention_workspace_bytes": (ctypes.c_uint64, [ctypes.POINTER(AttentionArgs)]),
    "bl_attention_noalloc": (ctypes.c_int, [ctypes.POINTER(AttentionArgs), ctypes.c_void_p]),
    "bl_attention_choice": (ctypes.c_int, [ctypes.POINTER(AttentionArgs),
                                           ctypes.POINTER(ctypes.c_uint32),
                                           ctypes.POINTER(ctypes.c_uint32),
                                           ctypes.POINTER(ctypes.c_uint32)]),
}


def lib():
    """The loaded library (raises if it is missing)."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError("beatlm_b200: %s is missing; build it with "
                                  "`python -m beatlm_b200.build`" % LIB_PATH)
            L = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
            _lib = L
    return _lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(1024)
    lib().bl_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(rc: int) -> None:
    if rc != BL_OK:
        raise BackendError(rc, last_error())


def status(reset: bool = False) -> Status:
    s = Status()
    check(lib().bl_status(ctypes.byref(s), 1 if reset else 0))
    return s


class GemmArgs(ctypes.Structure):
    _fields_ = [
        ("m", ctypes.c_uint32), ("n", ctypes.c_uint32), ("k", ctypes.c_uint32),
        ("ab_dtype", ctypes.c_int32), ("a", ctypes.c_void_p), ("lda", ctypes.c_uint64),
        ("b", ctypes.c_void_p), ("ldb", ctypes.c_uint64), ("ln_x", ctypes.c_void_p),
        ("ln_ldx", ctypes.c_uint64), ("ln_gamma", ctypes.c_void_p), ("ln_beta", ctypes.c_void_p),
        ("ln_eps", ctypes.c_float), ("bias", ctypes.c_void_p), ("act", ctypes.c_int32),
        ("scale", ctypes.c_float), ("chan_scale", ctypes.c_void_p), ("residual", ctypes.c_void_p),
        ("res_dtype", ctypes.c_int32), ("res_ld", ctypes.c_uint64), ("res_period", ctypes.c_uint32),
        ("out", ctypes.c_void_p), ("out_dtype", ctypes.c_int32), ("out_ld", ctypes.c_uint64),
        ("split_col", ctypes.c_uint32), ("out_dtype_hi", ctypes.c_int32),
        ("out_row_offset", ctypes.c_uint32), ("out_group_rows", ctypes.c_uint32),
        ("out_group_gap", ctypes.c_uint32), ("tile_n", ctypes.c_uint32),
        ("stats_out", ctypes.c_void_p), ("stats_parts", ctypes.c_uint32),
        ("ln_stats", ctypes.c_void_p), ("ln_stats_parts", ctypes.c_uint32),
        ("norm_out", ctypes.c_void_p), ("norm_out_dtype", ctypes.c_int32),
        ("norm_out_ld", ctypes.c_uint64), ("norm_gamma", ctypes.c_void_p),
        ("norm_beta", ctypes.c_void_p), ("norm_eps", ctypes.c_float),
        ("norm_sync", ctypes.c_void_p), ("norm_sync_bytes", ctypes.c_uint64),
        ("weights_static", ctypes.c_uint32), ("trace", ctypes.c_void_p),
        ("pair_tiles", ctypes.c_uint32), ("split_k", ctypes.c_uint32),
        ("stream_k", ctypes.c_uint32), ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_uint64), ("dot_w", ctypes.c_void_p),
        ("dot_bias", ctypes.c_float), ("dot_act", ctypes.c_int32),
    ]


class LayerNormArgs(ctypes.Structure):
    _fields_ = [
        ("rows", ctypes.c_uint32), ("cols", ctypes.c_uint32), ("x", ctypes.c_void_p),
        ("ldx", ctypes.c_uint64), ("gamma", ctypes.c_void_p), ("beta", ctypes.c_void_p),
        ("eps", ctypes.c_float), ("out", ctypes.c_void_p), ("out_dtype", ctypes.c_int32),
        ("ldo", ctypes.c_uint64), ("in_row_offset", ctypes.c_uint32),
        ("in_group_rows", ctypes.c_uint32), ("in_group_gap", ctypes.c_uint32),
    ]


class PatchifyArgs(ctypes.Structure):
    _fields_ = [
        ("frames", ctypes.c_uint32), ("side", ctypes.c_uint32), ("patch", ctypes.c_uint32),
        ("cin", ctypes.c_uint32), ("k_pad", ctypes.c_uint32), ("dim", ctypes.c_uint32),
        ("image", ctypes.c_void_p), ("a", ctypes.c_void_p), ("a_dtype", ctypes.c_int32),
        ("cls", ctypes.c_void_p), ("pos", ctypes.c_void_p), ("x", ctypes.c_void_p),
    ]


class KernelSpec(ctypes.Structure):
    _fields_ = [("op", ctypes.c_int32), ("args", ctypes.c_void_p), ("label", ctypes.c_char_p),
                ("parts", ctypes.c_uint32)]


class Substitution(ctypes.Structure):
    _fields_ = [("from_", ctypes.c_void_p), ("to", ctypes.c_void_p), ("bytes", ctypes.c_uint64)]


class BindingSet(ctypes.Structure):
    _fields_ = [("subs", ctypes.POINTER(Substitution)), ("n", ctypes.c_size_t)]


class SliceTime(ctypes.Structure):
    _fields_ = [("frame", ctypes.c_uint64), ("slice", ctypes.c_uint32),
                ("kernel", ctypes.c_uint32), ("begin_us", ctypes.c_double),
                ("micros", ctypes.c_double)]


class TimerStats(ctypes.Structure):
    _fields_ = [("frames_skipped", ctypes.c_uint64), ("frames_collected", ctypes.c_uint64),
                ("frames_failed", ctypes.c_uint64)]


_vp, _sz, _u32, _i32 = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_uint32, ctypes.c_int32
SIGNATURES.update({
    "bl_split_edges": (_u32, [_u32, _u32, _u32, ctypes.POINTER(_u32)]),
    "bl_parts_within": (_u32, [ctypes.c_uint64, ctypes.c_uint64, _u32]),
    "bl_kernels_create": (ctypes.c_int, [ctypes.POINTER(KernelSpec), _sz,
                                         ctypes.POINTER(BindingSet), _sz, ctypes.POINTER(_vp)]),
    "bl_kernels_destroy": (None, [_vp]),
    "bl_kernels_len": (_sz, [_vp]),
    "bl_kernels_sets": (_sz, [_vp]),
    "bl_kernels_launches": (_sz, [_vp]),
    "bl_kernels_label": (ctypes.c_char_p, [_vp, _sz]),
    "bl_kernels_encode": (ctypes.c_int, [_vp, _sz, _sz, _vp, _vp, _i32]),
    "bl_kernels_encode_range": (ctypes.c_int, [_vp, _sz, _sz, _sz, _vp, _vp, _i32]),
    "bl_kernels_capture": (ctypes.c_int, [_vp, _sz, _vp, ctypes.POINTER(_vp)]),
    "bl_graph_launch": (ctypes.c_int, [_vp, _vp]),
    "bl_graph_destroy": (None, [_vp]),
    "bl_timer_create": (ctypes.c_int, [_u32, ctypes.POINTER(_vp)]),
    "bl_timer_destroy": (None, [_vp]),
    "bl_timer_max_slices": (_u32, [_vp]),
    "bl_timer_begin_frame": (ctypes.c_int, [_vp, ctypes.c_uint64, ctypes.POINTER(_i32)]),
    "bl_timer_submitted": (ctypes.c_int, [_vp, _i32]),
    "bl_timer_submitted_held": (ctypes.c_int, [_vp, _i32]),
    "bl_timer_settle": (ctypes.c_int, [_vp, _i32, ctypes.c_int]),
    "bl_timer_drop": (ctypes.c_int, [_vp, _i32]),
    "bl_timer_invalidate_submitted": (_sz, [_vp]),
    "bl_timer_in_flight": (_sz, [_vp]),
    "bl_timer_collect_ready": (ctypes.c_int, [_vp, ctypes.POINTER(SliceTime), _sz,
                                              ctypes.POINTER(_sz), ctypes.POINTER(_sz)]),
    "bl_timer_get_stats": (ctypes.c_int, [_vp, ctypes.POINTER(TimerStats)]),
    "bl_gemm": (ctypes.c_int, [ctypes.POINTER(GemmArgs), ctypes.c_void_p]),
    "bl_gemm_norm_sync_bytes": (ctypes.c_uint64, [ctypes.POINTER(GemmArgs)]),
    "bl_gemm_workspace_bytes": (ctypes.c_uint64, [ctypes.POINTER(GemmArgs)]),
    "bl_layernorm": (ctypes.c_int, [ctypes.POINTER(LayerNormArgs), ctypes.c_void_p]),
    "bl_patchify": (ctypes.c_int, [ctypes.POINTER(PatchifyArgs), ctypes.c_void_p]),
})


class Estimator(ctypes.Structure):
    _fields_ = [("kind", ctypes.c_int32), ("window", ctypes.c_uint32),
                ("frame_window", ctypes.c_uint32), ("reserved", ctypes.c_uint32),
                ("alpha", ctypes.c_double), ("sigmas", ctypes.c_double),
                ("cap", ctypes.c_double), ("quantile", ctypes.c_double)]


class SyncPolicy(ctypes.Structure):
    _fields_ = [("kind", ctypes.c_int32), ("frames", ctypes.c_uint32),
                ("margin_us", ctypes.c_uint64), ("grid_origin_us", ctypes.c_uint64),
                ("grid_beat_us", ctypes.c_uint64)]


class FrameInfo(ctypes.Structure):
    _fields_ = [("index", ctypes.c_uint64), ("start_us", ctypes.c_uint64),
                ("period_us", ctypes.c_uint64)]


class SliceRun(ctypes.Structure):
    _fields_ = [("job", ctypes.c_uint64), ("slice", ctypes.c_uint32),
                ("reserved", ctypes.c_uint32), ("position", ctypes.c_uint64)]


class Delivery(ctypes.Structure):
    _fields_ = [("job", ctypes.c_uint64), ("input", ctypes.c_uint64)]


class Due(ctypes.Structure):
    _fields_ = [("kind", ctypes.c_int32), ("reserved", ctypes.c_uint32), ("at", ctypes.c_uint64)]


class Missed(ctypes.Structure):
    _fields_ = [("job", ctypes.c_uint64), ("input", ctypes.c_uint64), ("due", Due),
                ("policy", ctypes.c_int32), ("reserved", ctypes.c_uint32)]


class FramePlanInfo(ctypes.Structure):
    _fields_ = [("runs", ctypes.c_size_t), ("delivered", ctypes.c_size_t),
                ("missed", ctypes.c_size_t), ("spent_estimate_us", ctypes.c_uint64),
                ("budget_us", ctypes.c_uint64)]


class Im2colArgs(ctypes.Structure):
    _fields_ = [("input", ctypes.c_void_p), ("h", ctypes.c_uint32), ("w", ctypes.c_uint32),
                ("cin", ctypes.c_uint32), ("ksize", ctypes.c_uint32), ("stride", ctypes.c_uint32),
                ("relu", ctypes.c_uint32), ("out", ctypes.c_void_p), ("out_dtype", ctypes.c_int32),
                ("k_pad", ctypes.c_uint32), ("in_dtype", ctypes.c_int32)]


class Conv3x3Args(ctypes.Structure):
    _fields_ = [("input", ctypes.c_void_p), ("h", ctypes.c_uint32), ("w", ctypes.c_uint32),
                ("cin", ctypes.c_uint32), ("relu", ctypes.c_uint32)]


class PassCostArgs(ctypes.Structure):
    _fields_ = [("variant", ctypes.c_int32), ("passes", ctypes.c_uint32),
                ("every", ctypes.c_uint32), ("groups", ctypes.c_uint32),
                ("sink", ctypes.c_void_p), ("kernels", ctypes.c_void_p),
                ("stream", ctypes.c_void_p)]


class PassCostFrame(ctypes.Structure):
    _fields_ = [("span_us", ctypes.c_double), ("passes_us", ctypes.c_double),
                ("encode_us", ctypes.c_double), ("pairs", ctypes.c_uint32),
                ("reserved", ctypes.c_uint32)]


_u64 = ctypes.c_uint64
SIGNATURES.update({
    "bl_estimator_default": (None, [ctypes.POINTER(Estimator)]),
    "bl_cost_create": (ctypes.c_int, [_u64, ctypes.POINTER(Estimator), ctypes.POINTER(_vp),
                                      ctypes.POINTER(_i32)]),
    "bl_cost_clone": (ctypes.c_int, [_vp, ctypes.POINTER(_vp)]),
    "bl_cost_destroy": (None, [_vp]),
    "bl_cost_estimator": (ctypes.c_int, [_vp, ctypes.POINTER(Estimator)]),
    "bl_cost_record": (None, [_vp, _u32, _u64]),
    "bl_cost_record_calibration": (None, [_vp, _u32, _u64]),
    "bl_cost_frame_estimate": (ctypes.c_int, [_vp, _u32, ctypes.POINTER(_u64)]),
    "bl_cost_record_frame": (None, [_vp, _u64, _u64]),
    "bl_cost_frame_scale": (_i32, [_vp, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(_u64),
                                   ctypes.POINTER(_u64)]),
    "bl_cost_frames_recorded": (_u64, [_vp]),
    "bl_cost_planning_estimate": (_u64, [_vp, _u32]),
    "bl_cost_estimate": (_u64, [_vp, _u32]),
    "bl_cost_samples": (_u32, [_vp, _u32]),
    "bl_micros_nearest": (_u64, [ctypes.c_double]),
    "bl_kernel_spec_max_parts": (_u32, [ctypes.POINTER(KernelSpec)]),
    "bl_im2col": (ctypes.c_int, [ctypes.POINTER(Im2colArgs), _vp]),
    "bl_conv3x3": (ctypes.c_int, [ctypes.POINTER(GemmArgs), ctypes.POINTER(Conv3x3Args), _vp]),
    "bl_blocks_to_map": (ctypes.c_int, [_vp, _vp, _vp, _u32, _u32, _u32, _u32, _vp]),
    "bl_resize_bilinear": (ctypes.c_int, [_vp, _vp, _u32, _u32, _u32, _u32, _u32, _vp]),
    "bl_resize_bilinear_rows16": (ctypes.c_int, [_vp, _vp, _u32, _u32, _u32, _u32, _u32, _u32,
                                                 ctypes.c_int32, _vp]),
    "bl_conv1x1_one": (ctypes.c_int, [_vp, _vp, ctypes.c_float, _vp, _u32, _u32, ctypes.c_int32,
                                      _vp]),
    "bl_budget_for_frame": (_u64, [_u64, _u64, _u64]),
    "bl_beat_map_next": (ctypes.c_int, [ctypes.POINTER(_u64), _sz, _u64, ctypes.POINTER(_u64)]),
    "bl_scheduler_create": (ctypes.c_int, [ctypes.POINTER(SyncPolicy), _i32, _u64,
                                           ctypes.POINTER(_vp)]),
    "bl_scheduler_destroy": (None, [_vp]),
    "bl_scheduler_set_expected_budget": (None, [_vp, _u64]),
    "bl_scheduler_expected_budget": (_u64, [_vp]),
    "bl_scheduler_replace_beat_grid": (ctypes.c_int, [_vp, _u64, _u64, _u64]),
    "bl_scheduler_submit": (ctypes.c_int, [_vp, ctypes.POINTER(FrameInfo), ctypes.POINTER(_u32),
                                           _sz, _vp, ctypes.POINTER(_u64)]),
    "bl_scheduler_plan_frame": (ctypes.c_int, [_vp, ctypes.POINTER(FrameInfo), _u64, _vp,
                                               ctypes.POINTER(FramePlanInfo)]),
    "bl_scheduler_plan_runs": (_sz, [_vp, ctypes.POINTER(SliceRun), _sz]),
    "bl_scheduler_plan_delivered": (_sz, [_vp, ctypes.POINTER(Delivery), _sz]),
    "bl_scheduler_plan_missed": (_sz, [_vp, ctypes.POINTER(Missed), _sz]),
    "bl_scheduler_pending": (_sz, [_vp]),
    "bl_scheduler_due": (ctypes.c_int, [_vp, _u64, ctypes.POINTER(Due)]),
    "bl_pass_cost_frame_run": (ctypes.c_int, [ctypes.POINTER(PassCostArgs),
                                              ctypes.POINTER(PassCostFrame)]),
    "bl_program_parts_within": (ctypes.c_int, [ctypes.POINTER(KernelSpec), _sz,
                                               ctypes.POINTER(_u64), _sz, _u64,
                                               ctypes.POINTER(_u32)]),
    "bl_cost_record_passes": (_sz, [_vp, ctypes.POINTER(SliceTime), _sz, ctypes.c_int]),
})


class TensorDesc(ctypes.Structure):
    _fields_ = [("id", ctypes.c_uint32), ("elem_bytes", ctypes.c_uint32),
                ("elements", ctypes.c_uint64), ("first_use", ctypes.c_uint32),
                ("last_use", ctypes.c_uint32)]


class DeviceProfile(ctypes.Structure):
    _fields_ = [("max_binding_bytes", ctypes.c_uint64), ("max_buffer_bytes", ctypes.c_uint64),
                ("offset_alignment", ctypes.c_uint32)]


class PlanErrorInfo(ctypes.Structure):
    _fields_ = [("kind", ctypes.c_int32), ("id", ctypes.c_uint32), ("a", ctypes.c_uint64),
                ("b", ctypes.c_uint64)]


class Placement(ctypes.Structure):
    _fields_ = [("arena", ctypes.c_uint32), ("reserved", ctypes.c_uint32),
                ("offset", ctypes.c_uint64), ("size", ctypes.c_uint64)]


_u64 = ctypes.c_uint64
SIGNATURES.update({
    "bl_device_profile_webgpu_baseline": (ctypes.c_int, [ctypes.POINTER(DeviceProfile)]),
    "bl_device_profile_cuda": (ctypes.c_int, [ctypes.c_int, ctypes.POINTER(DeviceProfile)]),
    "bl_plan_create": (ctypes.c_int, [ctypes.POINTER(TensorDesc), _sz,
                                      ctypes.POINTER(DeviceProfile), ctypes.POINTER(_vp),
                                      ctypes.POINTER(PlanErrorInfo)]),
    "bl_plan_destroy": (None, [_vp]),
    "bl_plan_arenas": (_sz, [_vp, ctypes.POINTER(_u64), _sz]),
    "bl_plan_placement": (ctypes.c_int, [_vp, ctypes.c_uint32, ctypes.POINTER(Placement)]),
    "bl_plan_peak_live_bytes": (_u64, [_vp]),
    "bl_plan_total_bytes": (_u64, [_vp]),
    "bl_plan_valid_on": (ctypes.c_int, [_vp, ctypes.POINTER(DeviceProfile)]),
    "bl_arenas_create": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.POINTER(_vp)]),
    "bl_arenas_destroy": (None, [_vp]),
    "bl_arenas_bytes": (_u64, [_vp]),
    "bl_arenas_base": (ctypes.c_int, [_vp, ctypes.c_uint32, ctypes.POINTER(_vp)]),
    "bl_arenas_binding": (ctypes.c_int, [_vp, ctypes.POINTER(Placement), ctypes.POINTER(_vp)]),
    "bl_arenas_write": (ctypes.c_int, [_vp, ctypes.POINTER(Placement), _u64, _vp, _u64, _vp]),
    "bl_arenas_read": (ctypes.c_int, [_vp, ctypes.POINTER(Placement), _u64, _vp, _u64, _vp]),
})
SIGNATURES["bl_stream_hold"] = (ctypes.c_int, [_vp, ctypes.c_uint32])
SIGNATURES["bl_set_wait_limit"] = (ctypes.c_int, [ctypes.c_uint64])
SIGNATURES["bl_wait_limit"] = (ctypes.c_uint64, [])
SIGNATURES.update({
    "bl_peers_buffer_bytes": (ctypes.c_uint64, [ctypes.c_uint64]),
    "bl_peers_create": (ctypes.c_int, [ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint64,
                                       ctypes.POINTER(ctypes.c_void_p)]),
    "bl_peers_handle": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p]),
    "bl_peers_open": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t]),
    "bl_peers_attach": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_uint32, ctypes.c_void_p]),
    "bl_peers_slot": (ctypes.c_void_p, [ctypes.c_void_p, ctypes.c_uint32]),
    "bl_peers_next_epoch": (ctypes.c_uint32, [ctypes.c_void_p]),
    "bl_peers_destroy": (None, [ctypes.c_void_p]),
    "bl_attention_peers": (ctypes.c_int, [ctypes.POINTER(AttentionArgs), ctypes.c_void_p,
                                          ctypes.c_uint32, ctypes.POINTER(ctypes.c_uint32),
                                          ctypes.c_void_p]),
})
PEER_HANDLE_BYTES = 64


class AllGatherArgs(ctypes.Structure):
    _fields_ = [("comm", ctypes.c_void_p), ("send", ctypes.c_void_p), ("recv", ctypes.c_void_p),
                ("bytes", ctypes.c_uint64)]


COMM_ID_BYTES = 128
BL_ERR_COMM, BL_ERR_TIMEOUT = 6, 7
SIGNATURES.update({
    "bl_comm_available": (ctypes.c_int, []),
    "bl_comm_unique_id": (ctypes.c_int, [ctypes.c_void_p]),
    "bl_comm_init": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint32,
                                    ctypes.c_uint32, ctypes.POINTER(ctypes.c_void_p)]),
    "bl_comm_all_gather": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                          ctypes.c_uint64, ctypes.c_void_p]),
    "bl_comm_check": (ctypes.c_int, [ctypes.c_void_p]),
    "bl_comm_abort": (ctypes.c_int, [ctypes.c_void_p]),
    "bl_comm_aborted": (ctypes.c_int, [ctypes.c_void_p]),
    "bl_comm_destroy": (ctypes.c_int, [ctypes.c_void_p]),
})
