"""Loader of libferryb.so (the C ABI declared in include/ferryb.h).

The library is built in-tree (ferry_b200/libferryb.so, see build.py).  There
is no fallback: if it is missing or a call fails, a RuntimeError is raised,
as the reference's TORCH_CHECKs raise RuntimeError into Python
(ferry/csrc/expert_ops.cpp:20-34).
"""
import ctypes
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / 'libferryb.so'

_i64, _i32, _vp, _u64 = ctypes.c_int64, ctypes.c_int, ctypes.c_void_p, ctypes.c_uint64
_dbl, _f32 = ctypes.c_double, ctypes.c_float

_i32c, _u8p = ctypes.c_int32, ctypes.c_void_p


class Planner(ctypes.Structure):
    """ferryb_planner (include/ferryb.h)."""
    _fields_ = [('world', _i32c), ('experts', _i32c), ('layers', _i32c), ('topk', _i32c),
                ('window', _i32c), ('policy', _i32c), ('balance_tol_bps', _i64), ('salt', _i64),
                ('maxcap', _i32c), ('total_slots', _i32c), ('n_domains', _i32c),
                ('lut_rows', _i32c)] + [(n, _vp) for n in (
                    'capacities', 'slot_rank', 'slot_index', 'lut', 'masks', 'seconds', 'slots',
                    'owner', 'last', 'scores', 'ring', 'ring_p', 'hist_count', 'hist_head',
                    'order_meta', 'order_rec')] + [('order_cap', _i32c)]


class LayoutSummary(ctypes.Structure):
    """ferryb_layout_summary (include/ferryb.h)."""
    _fields_ = [(n, _i32c) for n in ('n_fetch_mine', 'n_hit', 'n_groups', 'n_recv', 'n_send',
                                      'n_routes', 'err', 'reserved')] + [
        ('fetch_keys', _i32c * 256), ('fetch_slots', _i32c * 256),
        ('send_counts', _i32c * 32), ('recv_counts', _i32c * 32), ('fetch_counts', _i32c * 32)]


class LayoutArgs(ctypes.Structure):
    """ferryb_layout_args (include/ferryb.h)."""
    _fields_ = [('ids', _vp), ('dest', _vp), ('world', _i32c), ('tokens_per_rank', _i32c),
                ('topk', _i32c), ('experts', _i32c), ('rank', _i32c)] + [(n, _vp) for n in (
                    'fetches', 'n_fetches', 'layer_slot', 'slots_row')] + [
        ('slots_count', _i32c), ('layer', _i32c)] + [(n, _vp) for n in (
                    'send_idx', 'send_ids', 'send_counts',
                    'recv_counts', 'starts', 'rows', 'cols', 'n_send', 'n_recv', 'recv_token',
                    'csr_pos', 'peer_row', 'groups', 'summary', 'err')]


class LayerConfig(ctypes.Structure):
    """ferryb_layer_config (include/ferryb.h)."""
    _fields_ = [(n, _i32c) for n in ('world', 'rank', 'tokens_per_rank', 'topk', 'experts', 'hidden',
                                      'intermediate', 'router_mode', 'norm_topk')] + [
        ('scaling', ctypes.c_float), ('probability_score', _i32c), ('timing', _i32c),
        ('sync_fetch', _i32c), ('shared_intermediate', _i32c)]


class LayerStats(ctypes.Structure):
    """ferryb_layer_stats (include/ferryb.h)."""
    _fields_ = [(n, _i64) for n in ('layers', 'fetches', 'routes', 'recv_rows', 'dispatch_bytes',
                                     'combine_bytes', 'launches', 'hit_experts', 'hit_weight_bytes',
                                     'timed_layers')] + [
        ('host_wait_us', _dbl), ('phase_us', _dbl * 5), ('host_us', _dbl * 6),
        ('copy_us', _dbl * 3), ('hit_gemm_kernel_us', _dbl), ('hit_gemm_kernel_launches', _i64),
        ('dispatch_permute_us', _dbl), ('combine_store_us', _dbl),
        ('kernel_us', _dbl * 9), ('kernel_launches', _i64 * 9), ('hit_gemm_kernel_bytes', _i64)]


# name -> (restype, argtypes); every symbol declared in include/ferryb.h.
SIGNATURES = {
    'ferryb_last_error': (ctypes.c_char_p, []),
    'ferryb_version': (_i32, []),
    'ferryb_device_sm_count': (_i32, [_i32]),
    'ferryb_stream_mem_ops_supported': (_i32, [_i32]),
    'ferryb_execute_experts_workspace': (_i64, [_i64, _i64, _i64, _i64]),
    'ferryb_execute_experts': (_i32, [_vp, _i64, _vp, _i64, _vp, _i64, _vp, _vp, _i64, _vp, _vp,
                                      _i64, _i64, _vp, _vp, _i64, _vp]),
    'ferryb_execute_experts_noalloc_limit': (_i64, []),
    'ferryb_execute_experts_noalloc': (_i32, [_vp, _i64, _vp, _i64, _vp, _i64, _vp, _vp, _i64, _vp,
                                              _vp, _i64, _i64, _vp, _vp]),
    'ferryb_plan_layer': (_i32, [ctypes.POINTER(Planner), _i64, _i32c, _vp, _i32c, _i32c, _vp, _vp,
                                 _vp, _i32c, _vp, _vp, _vp, _vp, _vp, _vp]),
    'ferryb_greedy_quota_rows': (_i32, [_i32c, _vp, _vp, _i32c, _vp, _i32c, _i32c, _vp, _vp, _vp]),
    'ferryb_demand': (_i32, [_vp, _vp, _i32c, _i32c, _i32c, _i32c, _vp, _vp, _vp]),
    'ferryb_admission_capacity': (_i32, [_vp, _i32c, _vp, _i32c, _i32c, _vp, _i32c, _vp, _vp]),
    'ferryb_load_balanced_assignment': (_i32, [_vp, _i32c, _i32c, _vp, _i32c, _vp, _i32c, _vp,
                                               _i64, _vp, _vp]),
    'ferryb_choose_slot': (_i32, [_i32c, _i32c, _vp, _vp, _i32c, _vp, _vp, _vp, _i32c, _vp, _vp]),
    'ferryb_build_layout': (_i32, [ctypes.POINTER(LayoutArgs), _vp]),
    'ferryb_layer_slots': (_i32, [_vp, _i32c, _i32c, _i32c, _vp, _vp]),
    'ferryb_h2d_create': (_i32, [_vp, _i64, _i64, _vp, _i64, _i32c, ctypes.POINTER(_vp)]),
    'ferryb_h2d_fetch': (_i32, [_vp, _vp, _vp, _i64]),
    'ferryb_h2d_fetch_flagged': (_i32, [_vp, _vp, _vp, _i64, _vp, ctypes.c_uint32]),
    'ferryb_h2d_wait_host': (_i32, [_vp, _vp, _i64]),
    'ferryb_h2d_wait_device': (_i32, [_vp, _vp, _i64, _vp]),
    'ferryb_h2d_mark_used': (_i32, [_vp, _vp, _i64, _vp]),
    'ferryb_h2d_synchronize': (_i32, [_vp]),
    'ferryb_h2d_copies': (_i64, [_vp]),
    'ferryb_h2d_destroy': (_i32, [_vp]),
    'ferryb_pack_dispatch': (_i32, [_vp, _i64, _i64, _vp, _vp, _i64, _vp, _vp, _i64, _i64, _vp, _vp,
                                    _vp]),
    'ferryb_unpack_dispatch': (_i32, [_vp, _i64, _i64, _i64, _vp, _vp, _vp]),
    'ferryb_segment_sum_workspace': (_i64, [_i64, _i64]),
    'ferryb_reduce_partials': (_i32, [_vp, _vp, _i64, _i64, _i64, _vp, _vp, _i64, _vp]),
    'ferryb_scatter_returned': (_i32, [_vp, _vp, _i64, _i64, _i64, _vp, _vp, _i64, _vp]),
    'ferryb_symm_alloc': (_i32, [_i64, ctypes.POINTER(_vp), _vp]),
    'ferryb_symm_open': (_i32, [_vp, ctypes.POINTER(_vp)]),
    'ferryb_symm_close': (_i32, [_vp]),
    'ferryb_symm_free': (_i32, [_vp]),
    'ferryb_history_update': (_i32, [_vp, _vp, _vp, _i32c, _i32c, _i32c, _i32c, _vp, _i64, _vp]),
    'ferryb_history_scores': (_i32, [_vp, _vp, _i32c, _i32c, _i32c, _i32c, _vp, _vp]),
    'ferryb_symm_allgather': (_i32, [_vp, _i32c, _i32c, _i64, _vp, _i64, _i64, ctypes.c_uint64, _vp]),
    'ferryb_symm_wait': (_i32, [_vp, _i64, _i32c, ctypes.c_uint64, _vp, _vp]),
    'ferryb_layer_workspace_bytes': (_i64, [ctypes.POINTER(LayerConfig)]),
    'ferryb_layer_symm_bytes': (_i64, [ctypes.POINTER(LayerConfig), _i32c]),
    'ferryb_layer_create': (_i32, [ctypes.POINTER(LayerConfig), ctypes.POINTER(Planner), _vp, _i64,
                                   _vp, _vp, _vp, _vp, _i64, ctypes.POINTER(_vp)]),
    'ferryb_layer_forward': (_i32, [_vp, _i64, _i32c, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    'ferryb_layer_execute': (_i32, [_vp, _i64, _i32c, _vp, _vp, _vp, _vp, _i32c, _vp, _vp]),
    'ferryb_layer_status': (_i32, [_vp, _vp]),
    'ferryb_layer_set_fault_hooks': (_i32, [_vp, ctypes.c_uint32, ctypes.c_uint64]),
    'ferryb_layer_get_stats': (_i32, [_vp, ctypes.POINTER(LayerStats)]),
    'ferryb_layer_reset_stats': (_i32, [_vp]),
    'ferryb_layer_set_shared': (_i32, [_vp, _i32c, _vp]),
    'ferryb_layer_last_summary': (_i32, [_vp, ctypes.POINTER(LayoutSummary)]),
    'ferryb_layer_collect_timing': (_i32, [_vp]),
    'ferryb_debug_plan_timestamps': (_i32, [_vp]),
    'ferryb_debug_layout_timestamps': (_i32, [_vp]),
    'ferryb_debug_router_timestamps': (_i32, [_vp]),
    'ferryb_layer_destroy': (_i32, [_vp]),
}

_lib = None


class FerrybError(RuntimeError):
    pass


# ferryb_layer_set_fault_hooks bits (include/ferryb.h)
HOOK_NO_READY_FLAGS = 1
HOOK_NO_DISPATCH_SIGNAL = 2
HOOK_NO_COMBINE_SIGNAL = 4


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise FerrybError(f'{LIB_PATH} is missing: build it with `python -m ferry_b200.build`')
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype, fn.argtypes = res, args
        _lib = handle
    return _lib


def call(name, *args):
    status = getattr(lib(), name)(*args)
    if status != 0:
        msg = lib().ferryb_last_error().decode(errors='replace')
        raise FerrybError(f'{name} failed (status {status}): {msg}')
    return status


def ptr(t):
    """Device/host address of a tensor (None -> NULL)."""
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def addr(t):
    """Integer address for ctypes structure fields (None -> 0)."""
    return 0 if t is None else t.data_ptr()


DEVICE_ERRORS = {1: 'a bounded device wait timed out', 2: 'missing experts exceed the total admission capacity',
                 3: 'no cache slot available for an expert scheduled on this rank',
                 4: 'an expert id or index is out of range', 5: 'a layout buffer is too small'}


def check_device_error(err_tensor, what):
    """Raise like the reference would (AssertionError for its asserts)."""
    code = int(err_tensor.item())
    if code == 2:
        raise AssertionError('missing experts exceed the total admission capacity')
    if code == 3:
        raise AssertionError(f'{what}: ' + DEVICE_ERRORS[3])
    if code:
        raise FerrybError(f'{what}: ' + DEVICE_ERRORS.get(code, f'device error {code}'))


def stream_ptr(device=None):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def require_cuda(*tensors):
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise FerrybError('expected CUDA tensors (this path has no CPU fallback)')


def check_tensor(t, name, shape, dtype=None, contiguous=False):
    """Raise FerrybError unless `t` has `shape` (None entries match any size),
    `dtype` and, if asked, a contiguous layout.  The C ABI receives bare
    pointers, so every buffer size it relies on is checked here first."""
    if t is None:
        raise FerrybError(f'{name} is required')
    if t.dim() != len(shape) or any(s is not None and t.shape[i] != s for i, s in enumerate(shape)):
        want = ', '.join('*' if s is None else str(s) for s in shape)
        raise FerrybError(f'{name} must have shape [{want}], got {list(t.shape)}')
    if dtype is not None and t.dtype != dtype:
        raise FerrybError(f'{name} must be {dtype}, got {t.dtype}')
    if contiguous and not t.is_contiguous():
        raise FerrybError(f'{name} must be contiguous')


def host_i64(values):
    arr = (ctypes.c_int64 * max(1, len(values)))(*[int(v) for v in values])
    return arr
