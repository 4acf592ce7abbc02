"""ctypes binding of libleanstream_b200.so (include/leanstream_b200.h).

The structures below mirror the C header field for field. Loading fails
loudly when the sm_100a library has not been built: there is no fallback.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIBRARY = Path(__file__).resolve().parent / "libleanstream_b200.so"

SOURCE_CACHE, SOURCE_STAGING = 0, 1
MODE_BATCH_COMPAT, MODE_PROGRESSIVE, MODE_AUTO = 0, 1, 2
NORM_INPUT, NO_OUTPUT = 1, 2
BATCH_MMA_SYNC = 1 << 8  # ls_b200_batch_args.flags: legacy warp-level MMA instead of tcgen05
STATUS_ERROR, STATUS_ERROR_EPOCH, STATUS_ERROR_DETAIL, STATUS_LAUNCHES, STATUS_WORDS = 0, 1, 2, 3, 4
TP_HANDLE_BYTES = 64
DEV_OK, DEV_QUEUE_ERROR, DEV_TIMEOUT_EPOCH, DEV_TIMEOUT_READY, DEV_TIMEOUT_SYNC, DEV_BAD_DESCRIPTOR, DEV_BAD_PLAN = range(7)


class ExecDesc(C.Structure):
    """ExecDesc, include/leanstream/types.h:16-20."""
    _fields_ = [("logical_group", C.c_uint32), ("physical_group", C.c_uint32), ("source_slot", C.c_uint32),
                ("dest_slot", C.c_uint32), ("source_kind", C.c_uint32)]


class QueueControl(C.Structure):
    """QueueControl, include/leanstream/execution_queue.h:5-12 (128 bytes)."""
    _fields_ = [("ready_count", C.c_uint32), ("reserved", C.c_uint32), ("total_count", C.c_uint32),
                ("epoch", C.c_uint32), ("batch_epoch", C.c_uint32), ("error", C.c_uint32),
                ("consumer_path", C.c_uint32), ("init_arrived", C.c_uint32), ("init_epoch", C.c_uint32),
                ("pad0", C.c_uint32 * 7), ("claim_count", C.c_uint32), ("pad1", C.c_uint32 * 15)]


class DeviceExecQueue(C.Structure):
    """DeviceExecQueue, execution_queue.h:13-18."""
    _fields_ = [("descriptors", C.c_void_p), ("ready_indices", C.c_void_p), ("control", C.c_void_p),
                ("capacity", C.c_uint32)]


class ExecSpan(C.Structure):
    _fields_ = [("data", C.c_void_p), ("size", C.c_size_t)]


class GroupSpan(C.Structure):
    _fields_ = [("data", C.c_void_p), ("size", C.c_size_t)]


ENQUEUE_FN = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_uint32, C.c_void_p, C.c_void_p, C.c_void_p, ExecSpan,
                         DeviceExecQueue, C.c_uint32, C.c_uint8)
COMPLETE_FN = C.CFUNCTYPE(C.c_bool, C.c_void_p, C.c_uint32)
COMMIT_FN = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_uint32, GroupSpan)
CANCEL_FN = C.CFUNCTYPE(None, C.c_void_p, C.c_uint32, C.c_uint32)


class ComputeBackend(C.Structure):
    """ComputeBackend, include/leanstream/runtime.h:10-22."""
    _fields_ = [("context", C.c_void_p), ("enqueue", ENQUEUE_FN), ("complete", COMPLETE_FN), ("commit", COMMIT_FN),
                ("defer_commit", C.c_void_p), ("cancel", CANCEL_FN)]


class KernelCandidate(C.Structure):
    """KernelCandidate, include/leanstream/kernel_selector.h:6-12."""
    _fields_ = [("id", C.c_uint32), ("workers", C.c_uint32), ("name", C.c_char_p), ("cta_count", C.c_uint32),
                ("tile_size", C.c_uint32), ("unroll", C.c_uint32), ("group_batch", C.c_uint32),
                ("entry_point", C.c_uint32), ("available", C.c_bool)]


class Geometry(C.Structure):
    _fields_ = [("hidden", C.c_uint32), ("group_size", C.c_uint32), ("group_count", C.c_uint32),
                ("max_layers", C.c_uint32), ("cache_slots", C.c_uint32), ("staging_slots", C.c_uint32),
                ("physical_groups", C.c_uint32), ("timeout_us", C.c_uint32), ("rms_eps", C.c_float)]


class LayerArgs(C.Structure):
    _fields_ = [("input", C.c_void_p), ("output", C.c_void_p), ("cache", C.c_void_p), ("staging", C.c_void_p),
                ("scales", C.c_void_p), ("core", C.c_void_p), ("core_count", C.c_uint32), ("epoch", C.c_uint32),
                ("queue", DeviceExecQueue), ("mode", C.c_uint8), ("pad", C.c_uint8 * 3), ("flags", C.c_uint32),
                ("candidate", C.c_int32), ("layer", C.c_uint32), ("activations", C.c_void_p),
                ("executions", C.c_void_p), ("first_compute", C.c_void_p), ("residual", C.c_void_p),
                ("hidden_out", C.c_void_p), ("output_f32", C.c_void_p), ("norm_weight", C.c_void_p),
                ("trace", C.c_void_p), ("importance", C.c_void_p), ("importance_flag", C.c_void_p)]


class Queue(C.Structure):
    """ls_b200_queue: host producer state over a DeviceExecQueue view."""
    _fields_ = [("view", DeviceExecQueue), ("tail", C.c_uint32), ("epoch", C.c_uint32), ("total", C.c_uint32)]


class IOCompletion(C.Structure):
    """IOCompletion, include/leanstream/weight_manager.h:8-11."""
    _fields_ = [("epoch", C.c_uint32), ("logical_group", C.c_int32), ("staging_slot", C.c_int32),
                ("error", C.c_int32), ("slot_sequence", C.c_uint64)]


IO_COMPLETION_FN = C.CFUNCTYPE(None, C.c_void_p, C.POINTER(IOCompletion))


class IOBackend(C.Structure):
    """IOBackend, include/leanstream/weight_manager.h:14-24."""
    _fields_ = [("context", C.c_void_p), ("begin", C.c_void_p), ("update", C.c_void_p), ("consume", C.c_void_p),
                ("retire", C.c_void_p), ("ready_slot", C.c_void_p), ("requests", C.c_void_p), ("wait", C.c_void_p)]


class StreamConfig(C.Structure):
    _fields_ = [("host_base", C.c_void_p), ("host_offsets", C.c_void_p), ("staging", C.c_void_p),
                ("staging_stride", C.c_uint64), ("group_bytes", C.c_uint64), ("io_states", C.c_void_p),
                ("group_count", C.c_uint32), ("queue_depth", C.c_uint32), ("device", C.c_int32),
                ("delay_mean_us", C.c_float), ("delay_seed", C.c_uint64), ("file_path", C.c_char_p),
                ("file_offsets", C.c_void_p), ("read_workers", C.c_uint32), ("o_direct", C.c_uint32),
                ("file_alignment", C.c_uint32)]


class StreamStats(C.Structure):
    _fields_ = [("admissions", C.c_uint64), ("completions", C.c_uint64), ("bytes", C.c_uint64),
                ("first_issue_ns", C.c_uint64), ("last_land_ns", C.c_uint64), ("copy_ns", C.c_uint64),
                ("error", C.c_int32), ("outstanding", C.c_uint32), ("direct", C.c_uint32), ("reserved", C.c_uint32),
                ("read_bytes", C.c_uint64), ("read_ns", C.c_uint64)]


IO_EMPTY, IO_INFLIGHT, IO_READY, IO_ERROR = 0, 1, 2, 3


class BatchArgs(C.Structure):
    """ls_b200_batch_args: up to 8 tokens over the union of their groups."""
    _fields_ = [("hidden", C.c_uint32), ("group_size", C.c_uint32), ("union_count", C.c_uint32),
                ("tokens", C.c_uint32), ("x", C.c_void_p), ("output", C.c_void_p), ("output_f32", C.c_void_p),
                ("residual", C.c_void_p), ("hidden_out", C.c_void_p), ("cache", C.c_void_p),
                ("staging", C.c_void_p), ("scales", C.c_void_p), ("union_descs", C.c_void_p), ("mask", C.c_void_p),
                ("scratch", C.c_void_p), ("scratch_bytes", C.c_uint64), ("flags", C.c_uint32),
                ("rms_eps", C.c_float), ("norm_weight", C.c_void_p), ("error", C.c_void_p),
                ("timeout_ns", C.c_uint64)]

assert C.sizeof(IOCompletion) == 24 and C.sizeof(IOBackend) == 64 and C.sizeof(StreamConfig) == 104
assert C.sizeof(ExecDesc) == 20 and C.sizeof(QueueControl) == 128 and C.sizeof(DeviceExecQueue) == 32

# name -> (restype, argtypes); every entry point declared in include/leanstream_b200.h
SIGNATURES = {
    "ls_b200_create": (C.c_void_p, []),
    "ls_b200_create_table": (C.c_void_p, [C.c_void_p, C.c_uint32, C.c_uint32]),
    "ls_b200_destroy": (None, [C.c_void_p]),
    "ls_b200_configure": (C.c_int, [C.c_void_p, C.POINTER(Geometry)]),
    "ls_b200_set_buffers": (C.c_int, [C.c_void_p, C.POINTER(LayerArgs)]),
    "ls_b200_set_state": (None, [C.c_void_p, C.c_uint32, C.c_uint32]),
    "ls_b200_launch": (C.c_int, [C.c_void_p, C.POINTER(LayerArgs), C.c_void_p]),
    "ls_b200_launch_static": (C.c_int, [C.POINTER(Geometry), C.POINTER(LayerArgs), C.c_void_p, C.c_void_p]),
    "ls_b200_enqueue": (C.c_int, [C.c_void_p, C.c_uint32, C.c_uint32, C.c_uint32, C.c_void_p]),
    "ls_b200_plan_size": (C.c_uint32, []),
    "ls_b200_encode_plan": (C.c_int, [C.c_void_p, C.POINTER(LayerArgs), C.c_void_p]),
    "ls_b200_launch_plans": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint32, C.c_void_p, C.c_int32, C.c_void_p,
                                       C.c_void_p]),
    "ls_b200_view": (C.c_int, [C.c_void_p, C.POINTER(ComputeBackend)]),
    "ls_b200_completed_epoch": (C.c_int, [C.c_void_p, C.c_uint32, C.POINTER(C.c_uint32)]),
    "ls_b200_status": (C.c_int, [C.c_void_p, C.POINTER(C.c_uint32), C.c_uint32]),
    "ls_b200_clear_status": (C.c_int, [C.c_void_p]),
    "ls_b200_scratch_bytes": (C.c_uint64, [C.c_void_p]),
    "ls_b200_quantize_io_load": (C.c_uint32, [C.c_uint32, C.c_uint32, C.c_uint32]),
    "ls_b200_select": (C.c_uint32, [C.c_void_p, C.c_uint32, C.c_uint32]),
    "ls_b200_candidate": (C.c_int, [C.c_void_p, C.c_uint32, C.POINTER(KernelCandidate)]),
    "ls_b200_catalog_size": (C.c_uint32, []),
    "ls_b200_default_candidate": (C.c_uint32, []),
    "ls_b200_queue_bind": (None, [C.POINTER(Queue), DeviceExecQueue]),
    "ls_b200_queue_reset": (C.c_int, [C.POINTER(Queue), C.c_uint32]),
    "ls_b200_queue_prepare": (C.c_int, [C.POINTER(Queue), C.c_uint32]),
    "ls_b200_queue_append_unpublished": (C.c_int, [C.POINTER(Queue), C.c_uint32]),
    "ls_b200_queue_activate": (C.c_int, [C.POINTER(Queue)]),
    "ls_b200_queue_seal": (C.c_int, [C.POINTER(Queue), C.c_uint32]),
    "ls_b200_queue_publish_all": (C.c_int, [C.POINTER(Queue)]),
    "ls_b200_queue_publish": (C.c_int, [C.POINTER(Queue), C.c_uint32]),
    "ls_b200_queue_fail": (C.c_int, [C.POINTER(Queue), C.c_uint32]),
    "ls_b200_build_info": (C.c_char_p, []),
    "ls_b200_tp_epilogue": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint32, C.c_void_p]),
    "ls_b200_tp_setup": (C.c_int, [C.c_void_p, C.c_uint32, C.c_uint32, C.c_void_p]),
    "ls_b200_tp_connect": (C.c_int, [C.c_void_p, C.c_void_p]),
    "ls_b200_spin": (C.c_int, [C.c_uint64, C.c_void_p]),
    "ls_b200_batch_scratch_bytes": (C.c_uint64, [C.c_uint32, C.c_uint32, C.c_uint32]),
    "ls_b200_batch_mlp": (C.c_int, [C.POINTER(BatchArgs), C.c_void_p]),
    "ls_b200_stream_create": (C.c_void_p, [C.POINTER(StreamConfig)]),
    "ls_b200_stream_view": (C.c_int, [C.c_void_p, C.POINTER(IOBackend)]),
    "ls_b200_stream_stats": (C.c_int, [C.c_void_p, C.POINTER(StreamStats)]),
    "ls_b200_stream_issue_log": (C.c_uint32, [C.c_void_p, C.c_void_p, C.c_uint32]),
    "ls_b200_stream_destroy": (None, [C.c_void_p]),
}

_lib = None


def load() -> C.CDLL:
    """Loads the in-tree sm_100a library, failing loudly when it is absent."""
    global _lib
    if _lib is None:
        if not LIBRARY.exists():
            raise RuntimeError(f"{LIBRARY} is missing: run `python -m leanstream_b200.build` (no CPU fallback)")
        lib = C.CDLL(str(LIBRARY), use_errno=True)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib
