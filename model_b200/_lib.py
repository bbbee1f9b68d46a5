"""ctypes binding of ``include/memlayer.h`` (the library's C ABI).

The structures below mirror the header field for field.  Loading fails
loudly if ``libmemlayer.so`` has not been built: there is no fallback.
"""

from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libmemlayer.so")

OK, ERR_BAD_SHAPE, ERR_BAD_POINTER, ERR_UNSUPPORTED, ERR_WORKSPACE, ERR_CUDA, ERR_PEER_TIMEOUT = range(7)
F32, F16, BF16 = 0, 1, 2


class MemlayerConfig(C.Structure):
    _fields_ = [
        ("tokens", C.c_int64),
        ("heads", C.c_int32),
        ("n_sub_keys", C.c_int32),
        ("d_key", C.c_int32),
        ("d_value", C.c_int32),
        ("top_k", C.c_int32),
        ("d_model", C.c_int32),
        ("values_dtype", C.c_int32),
        ("routing_noise", C.c_float),
        ("min_temperature", C.c_float),
        ("max_temperature", C.c_float),
        ("query_scale", C.c_int32),
        ("balance_temperature_grad", C.c_int32),
    ]


STAGE_EVENTS = 6
MAX_SHARDS = 8
IPC_HANDLE_BYTES = 64
PHASE_ROUTE, PHASE_GATHER, PHASE_REDUCE, PHASE_ALL, PHASE_SPLIT = 1, 2, 4, 7, 8


class MemlayerStageEvents(C.Structure):
    _fields_ = [("events", C.c_void_p * STAGE_EVENTS)]


class MemlayerPoolArgs(C.Structure):
    _fields_ = [
        ("queries", C.c_void_p),
        ("sub_keys", C.c_void_p),
        ("log_temperature", C.c_void_p),
        ("values", C.c_void_p),
        ("gumbel", C.c_void_p),
        ("noise_scale", C.c_float),
        ("train", C.c_int32),
        ("shuffle_reads", C.c_int32),
        ("out", C.c_void_p),
        ("slots", C.c_void_p),
        ("weights", C.c_void_p),
        ("queries_unit", C.c_void_p),
        ("subkey_counts", C.c_void_p),
        ("slot_counts", C.c_void_p),
        ("balance_loss", C.c_void_p),
        ("top1_weight", C.c_void_p),
        ("temperature", C.c_void_p),
        ("stage_events", C.POINTER(MemlayerStageEvents)),
    ]


class MemlayerLayerArgs(C.Structure):
    _fields_ = [
        ("h", C.c_void_p),
        ("w_router", C.c_void_p),
        ("b_router", C.c_void_p),
        ("w_gate", C.c_void_p),
        ("b_gate", C.c_void_p),
        ("w_out", C.c_void_p),
        ("b_out", C.c_void_p),
        ("y", C.c_void_p),
        ("mem", C.c_void_p),
        ("pool", MemlayerPoolArgs),
    ]


class MemlayerStagedArgs(C.Structure):
    _fields_ = [
        ("all_slots", C.c_void_p),
        ("all_weights", C.c_void_p),
        ("route_stride", C.c_int64),
        ("partials", C.c_void_p),
        ("mem", C.c_void_p),
        ("rank", C.c_int32),
        ("world", C.c_int32),
    ]


MAX_LAYERS = 32


class MemlayerModelConfig(C.Structure):
    _fields_ = [
        ("vocab_size", C.c_int32),
        ("max_len", C.c_int32),
        ("d_model", C.c_int32),
        ("n_layers", C.c_int32),
        ("n_heads", C.c_int32),
        ("ffn_mult", C.c_int32),
        ("memory_layers", C.c_uint32),
        ("memory_ffn", C.c_int32),
        ("pool", MemlayerConfig),
    ]


class MemlayerBlockParams(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in (
        "ln_attn_scale", "ln_attn_bias", "w_qkv", "b_qkv", "w_attn_out", "b_attn_out", "ln_ffn_scale",
        "ln_ffn_bias", "w_ffn_in", "b_ffn_in", "w_ffn_out", "b_ffn_out", "w_router", "b_router", "w_gate",
        "b_gate", "w_out", "b_out")]


class MemlayerModelParams(C.Structure):
    _fields_ = [
        ("embedding", C.c_void_p),
        ("pos_embed", C.c_void_p),
        ("layers", C.POINTER(MemlayerBlockParams)),
        ("ln_final_scale", C.c_void_p),
        ("ln_final_bias", C.c_void_p),
        ("sub_keys", C.c_void_p),
        ("log_temperature", C.c_void_p),
        ("values", C.c_void_p),
    ]


MAX_READS = 8


class MemlayerRead(C.Structure):
    _fields_ = [("slots", C.c_void_p), ("weights", C.c_void_p), ("grad", C.c_void_p), ("tokens", C.c_int64)]


class MemlayerAdagradArgs(C.Structure):
    _fields_ = [
        ("values", C.c_void_p),
        ("accum", C.c_void_p),
        ("lr", C.c_float),
        ("grad_clip", C.c_float),
        ("rest_sq_norm", C.c_void_p),
        ("clip_scale", C.c_void_p),
        ("n_unique", C.c_void_p),
    ]


class MemlayerReviveArgs(C.Structure):
    _fields_ = [
        ("sub_keys", C.c_void_p),
        ("usage", C.c_void_p),
        ("queries", C.c_void_p),
        ("query_tokens", C.c_int64),
        ("pick", C.c_void_p),
        ("noise", C.c_void_p),
        ("threshold", C.c_float),
        ("noise_scale", C.c_float),
        ("dead", C.c_void_p),
        ("moment0", C.c_void_p),
        ("moment1", C.c_void_p),
    ]


class MemlayerLayerGrads(C.Structure):
    _fields_ = [
        ("dy", C.c_void_p),
        ("balance_coef", C.c_float),
        ("route_through_pool", C.c_int32),
        ("forward_workspace", C.c_void_p),
        ("dh", C.c_void_p),
        ("dw_router", C.c_void_p),
        ("db_router", C.c_void_p),
        ("dsub_keys", C.c_void_p),
        ("dlog_temperature", C.c_void_p),
        ("dw_gate", C.c_void_p),
        ("db_gate", C.c_void_p),
        ("dw_out", C.c_void_p),
        ("db_out", C.c_void_p),
        ("probe", C.c_void_p),
    ]


DEVICE_ERRORS = {11: "producer wait timed out", 12: "MMA wait timed out", 13: "MMA wait timed out",
                 14: "epilogue wait timed out", 15: "epilogue pair wait timed out",
                 21: "sub-key id out of range", 22: "sharded row id out of range",
                 23: "fetched slot id out of range", 24: "row push beyond inbox capacity",
                 25: "host-table row id out of range", 26: "token id or position out of range",
                 31: "peer inbox wait timed out", 32: "peer partial-sum wait timed out",
                 33: "row-gradient inbox wait timed out", 34: "norm partial wait timed out",
                 35: "peer probe-row wait timed out", 36: "peer dot wait timed out"}


class MemlayerError(RuntimeError):
    """A non-zero memlayer_status."""

    def __init__(self, status: int, where: str):
        self.status = status
        super().__init__(f"{where}: {status_string(status)} (status {status})")


_lib = None


def lib() -> C.CDLL:
    """The loaded library (raises if it was not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `python -m model_b200.build`")
        L = C.CDLL(LIB_PATH)
        L.memlayer_abi_version.restype = C.c_int32
        L.memlayer_status_string.restype = C.c_char_p
        L.memlayer_status_string.argtypes = [C.c_int32]
        for name in ("memlayer_pool_workspace_size", "memlayer_layer_workspace_size"):
            f = getattr(L, name)
            f.restype = C.c_int32
            f.argtypes = [C.POINTER(MemlayerConfig), C.POINTER(C.c_size_t)]
        L.memlayer_pool_forward.restype = C.c_int32
        L.memlayer_pool_forward.argtypes = [C.POINTER(MemlayerConfig), C.POINTER(MemlayerPoolArgs), C.c_void_p,
                                            C.c_size_t, C.c_void_p]
        L.memlayer_layer_forward.restype = C.c_int32
        L.memlayer_layer_forward.argtypes = [C.POINTER(MemlayerConfig), C.POINTER(MemlayerLayerArgs), C.c_void_p,
                                             C.c_size_t, C.c_void_p]
        L.memlayer_workspace_status.restype = C.c_int32
        L.memlayer_workspace_status.argtypes = [C.POINTER(MemlayerConfig), C.c_void_p, C.POINTER(C.c_int32),
                                                C.c_void_p]
        L.memlayer_kernel_launch_count.restype = C.c_int64
        L.memlayer_shard_rows.restype = C.c_int64
        L.memlayer_shard_rows.argtypes = [C.c_int64, C.c_int32, C.c_int32]
        L.memlayer_shard_comm_create.restype = C.c_int32
        L.memlayer_shard_comm_create.argtypes = [C.POINTER(MemlayerConfig), C.c_int32, C.c_int32,
                                                 C.POINTER(C.c_void_p)]
        L.memlayer_shard_comm_info.restype = C.c_int32
        L.memlayer_shard_comm_info.argtypes = [C.c_void_p, C.POINTER(C.c_int32), C.POINTER(C.c_int32),
                                               C.POINTER(C.c_int32), C.POINTER(C.c_size_t)]
        L.memlayer_shard_comm_ipc_handle.restype = C.c_int32
        L.memlayer_shard_comm_ipc_handle.argtypes = [C.c_void_p, C.c_void_p]
        L.memlayer_shard_comm_open_peers.restype = C.c_int32
        L.memlayer_shard_comm_open_peers.argtypes = [C.c_void_p, C.c_void_p]
        L.memlayer_shard_comm_set_peer.restype = C.c_int32
        L.memlayer_shard_comm_set_peer.argtypes = [C.c_void_p, C.c_int32, C.c_void_p]
        L.memlayer_shard_comm_set_wait_budget.restype = C.c_int32
        L.memlayer_shard_comm_set_wait_budget.argtypes = [C.c_void_p, C.c_int64]
        L.memlayer_layer_forward_staged.restype = C.c_int32
        L.memlayer_layer_forward_staged.argtypes = [C.POINTER(MemlayerConfig), C.POINTER(MemlayerLayerArgs),
                                                    C.POINTER(MemlayerStagedArgs), C.c_int32, C.c_void_p,
                                                    C.c_size_t, C.c_void_p]
        L.memlayer_model_workspace_size.restype = C.c_int32
        L.memlayer_model_workspace_size.argtypes = [C.POINTER(MemlayerModelConfig), C.c_int64, C.POINTER(C.c_size_t)]
        L.memlayer_model_cache_size.restype = C.c_int32
        L.memlayer_model_cache_size.argtypes = [C.POINTER(MemlayerModelConfig), C.c_int64, C.POINTER(C.c_size_t)]
        L.memlayer_model_forward.restype = C.c_int32
        L.memlayer_model_forward.argtypes = [C.POINTER(MemlayerModelConfig), C.POINTER(MemlayerModelParams),
                                             C.c_void_p, C.c_int64, C.c_int64, C.c_void_p, C.c_void_p, C.c_size_t,
                                             C.c_void_p]
        L.memlayer_model_decode_step.restype = C.c_int32
        L.memlayer_model_decode_step.argtypes = [C.POINTER(MemlayerModelConfig), C.POINTER(MemlayerModelParams),
                                                 C.c_void_p, C.c_int64, C.c_void_p, C.c_void_p, C.c_void_p,
                                                 C.c_void_p, C.c_size_t, C.c_void_p]
        L.memlayer_shard_comm_destroy.restype = C.c_int32
        L.memlayer_shard_comm_destroy.argtypes = [C.c_void_p]
        L.memlayer_shard_workspace_size.restype = C.c_int32
        L.memlayer_shard_workspace_size.argtypes = [C.POINTER(MemlayerConfig), C.c_int32, C.c_int32,
                                                    C.POINTER(C.c_size_t)]
        L.memlayer_pool_forward_sharded.restype = C.c_int32
        L.memlayer_pool_forward_sharded.argtypes = [C.POINTER(MemlayerConfig), C.POINTER(MemlayerPoolArgs),
                                                    C.c_void_p, C.c_int32, C.c_void_p, C.c_size_t, C.c_void_p]
        L.memlayer_layer_forward_sharded.restype = C.c_int32
        L.memlayer_layer_forward_sharded.argtypes = [C.POINTER(MemlayerConfig), C.POINTER(MemlayerLayerArgs),
                                                     C.c_void_p, C.c_int32, C.c_void_p, C.c_size_t, C.c_void_p]
        L.memlayer_layer_host_workspace_size.restype = C.c_int32
        L.memlayer_layer_host_workspace_size.argtypes = [C.POINTER(MemlayerConfig), C.c_int32, C.POINTER(C.c_size_t)]
        L.memlayer_layer_forward_host.restype = C.c_int32
        L.memlayer_layer_forward_host.argtypes = [C.POINTER(MemlayerConfig), C.POINTER(MemlayerLayerArgs), C.c_int32,
                                                  C.c_void_p, C.c_size_t, C.c_void_p]
        L.memlayer_rowgrad_workspace_size.restype = C.c_int32
        L.memlayer_rowgrad_workspace_size.argtypes = [C.POINTER(MemlayerConfig), C.c_int64, C.POINTER(C.c_size_t)]
        L.memlayer_fetched_row_grads.restype = C.c_int32
        L.memlayer_fetched_row_grads.argtypes = [C.POINTER(MemlayerConfig), C.POINTER(MemlayerRead), C.c_int32,
                                                 C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                                 C.c_size_t, C.c_void_p]
        L.memlayer_row_adagrad.restype = C.c_int32
        L.memlayer_row_adagrad.argtypes = [C.POINTER(MemlayerConfig), C.POINTER(MemlayerRead), C.c_int32,
                                           C.POINTER(MemlayerAdagradArgs), C.c_void_p, C.c_size_t, C.c_void_p]
        L.memlayer_key_diversity_workspace_size.restype = C.c_int32
        L.memlayer_key_diversity_workspace_size.argtypes = [C.POINTER(MemlayerConfig), C.POINTER(C.c_size_t)]
        L.memlayer_key_diversity.restype = C.c_int32
        L.memlayer_key_diversity.argtypes = [C.POINTER(MemlayerConfig), C.c_void_p, C.c_void_p, C.c_void_p, C.c_float,
                                             C.c_void_p, C.c_size_t, C.c_void_p]
        L.memlayer_revive_dead_keys.restype = C.c_int32
        L.memlayer_revive_dead_keys.argtypes = [C.POINTER(MemlayerConfig), C.POINTER(MemlayerReviveArgs), C.c_void_p]
        L.memlayer_shard_comm_create_rowgrad.restype = C.c_int32
        L.memlayer_shard_comm_create_rowgrad.argtypes = [C.POINTER(MemlayerConfig), C.c_int32, C.c_int32, C.c_int32,
                                                         C.POINTER(C.c_void_p)]
        L.memlayer_shard_rowgrad_workspace_size.restype = C.c_int32
        L.memlayer_shard_rowgrad_workspace_size.argtypes = [C.c_void_p, C.c_int64, C.POINTER(C.c_size_t)]
        L.memlayer_row_adagrad_sharded.restype = C.c_int32
        L.memlayer_row_adagrad_sharded.argtypes = [C.POINTER(MemlayerConfig), C.POINTER(MemlayerRead), C.c_int32,
                                                   C.POINTER(MemlayerAdagradArgs), C.c_void_p, C.c_int32, C.c_void_p,
                                                   C.c_size_t, C.c_void_p]
        L.memlayer_host_table_workspace_size.restype = C.c_int32
        L.memlayer_host_table_workspace_size.argtypes = [C.POINTER(MemlayerConfig), C.POINTER(C.c_size_t)]
        L.memlayer_pool_forward_host_table.restype = C.c_int32
        L.memlayer_pool_forward_host_table.argtypes = [C.POINTER(MemlayerConfig), C.POINTER(MemlayerPoolArgs),
                                                       C.c_void_p, C.c_size_t, C.c_void_p]
        L.memlayer_layer_forward_prepared.restype = C.c_int32
        L.memlayer_layer_forward_prepared.argtypes = [C.POINTER(MemlayerConfig), C.POINTER(MemlayerLayerArgs),
                                                      C.c_void_p, C.c_size_t, C.c_void_p]
        L.memlayer_layer_backward_workspace_size.restype = C.c_int32
        L.memlayer_layer_backward_workspace_size.argtypes = [C.POINTER(MemlayerConfig), C.c_int32,
                                                             C.POINTER(C.c_size_t)]
        L.memlayer_layer_backward.restype = C.c_int32
        L.memlayer_layer_backward.argtypes = [C.POINTER(MemlayerConfig), C.POINTER(MemlayerLayerArgs),
                                              C.POINTER(MemlayerLayerGrads), C.c_void_p, C.c_size_t, C.c_void_p]
        L.memlayer_layer_backward_sharded.restype = C.c_int32
        L.memlayer_layer_backward_sharded.argtypes = [C.POINTER(MemlayerConfig), C.POINTER(MemlayerLayerArgs),
                                                      C.POINTER(MemlayerLayerGrads), C.c_void_p, C.c_int32,
                                                      C.c_void_p, C.c_size_t, C.c_void_p]
        if L.memlayer_abi_version() != 1:
            raise ImportError("libmemlayer.so ABI version mismatch; rebuild")
        _lib = L
    return _lib


def status_string(status: int) -> str:
    return lib().memlayer_status_string(status).decode()


def check(status: int, where: str) -> None:
    if status != OK:
        raise MemlayerError(status, where)


def device_status(cfg, workspace_ptr: int, stream_ptr: int) -> int:
    """The device status word of the last call on this workspace (syncs)."""
    code = C.c_int32(0)
    check(lib().memlayer_workspace_status(C.byref(cfg), workspace_ptr, C.byref(code), stream_ptr),
          "memlayer_workspace_status")
    return code.value


class DeviceError(RuntimeError):
    """A kernel recorded a failure in the workspace status word."""
