"""ctypes binding of libvxk.so (include/vxk.h) for tests, smoke() and bench.py.

The binding only marshals arguments: every computation happens in libvxk.so.
Loading fails loudly when the library has not been built; there is no
fallback path.  Device buffers are passed as integer device addresses
(e.g. ``tensor.data_ptr()``), streams as integer cudaStream_t handles.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libvxk.so"

STATUS = {
    0: "ok", 1: "invalid_argument", 2: "invalid_state", 3: "out_of_memory", 5: "not_ready",
    9: "backend_error", 10: "internal_error", 11: "buffer_too_small", 12: "timeout",
}
OK, INVALID_ARGUMENT, INVALID_STATE, OUT_OF_MEMORY = 0, 1, 2, 3
NOT_READY, BACKEND_ERROR, INTERNAL_ERROR, BUFFER_TOO_SMALL, TIMEOUT = 5, 9, 10, 11, 12
DTYPE_F16, DTYPE_Q8_0, DTYPE_BF16 = 1, 8, 30


class VxkError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS.get(status, status)}: {message}")
        self.status = status


class DecoderKvRing(C.Structure):
    _fields_ = [("capacity", C.c_int64), ("used", C.c_int64),
                ("oldest_absolute_position", C.c_int64), ("next_absolute_position", C.c_int64),
                ("wraps", C.c_int64), ("evictions", C.c_int64), ("bytes_moved", C.c_int64),
                ("full_buffer_moves", C.c_int64)]


class KvSeg(C.Structure):
    _fields_ = [("slot", C.c_int32), ("len", C.c_int32)]


class DecoderKvPlan(C.Structure):
    _fields_ = [("absolute_start", C.c_int64), ("n_new", C.c_int32), ("write_nseg", C.c_int32),
                ("write_seg", KvSeg * 2), ("read_seg", KvSeg * 2), ("read_nseg", C.c_int32),
                ("wrapped", C.c_int32), ("used_after", C.c_int64), ("oldest_after", C.c_int64),
                ("next_after", C.c_int64), ("evicted", C.c_int64)]


class EncKvPlan(C.Structure):
    _fields_ = [("q_start", C.c_int64), ("n_new", C.c_int32), ("win_len", C.c_int32),
                ("win_start", C.c_int64), ("win_end", C.c_int64), ("read_seg", KvSeg * 2),
                ("read_nseg", C.c_int32), ("read_wraps", C.c_int32), ("write_seg", KvSeg * 2),
                ("write_nseg", C.c_int32), ("write_wraps", C.c_int32),
                ("conv_mel_start", C.c_int64), ("conv_mel_end", C.c_int64),
                ("conv_slice_start", C.c_int32), ("reserved", C.c_int32), ("evicted", C.c_int64)]


class PoolConfig(C.Structure):
    _fields_ = [("struct_size", C.c_uint32), ("api_version", C.c_uint32), ("device", C.c_int32),
                ("n_layers", C.c_int32), ("n_q_heads", C.c_int32), ("n_kv_heads", C.c_int32),
                ("head_dim", C.c_int32), ("block_tokens", C.c_int32), ("n_blocks", C.c_int32),
                ("capacity", C.c_int32), ("max_streams", C.c_int32), ("max_rows", C.c_int32),
                ("max_position", C.c_int32), ("dtype", C.c_int32), ("rope_theta", C.c_float),
                ("alloc_seed", C.c_uint32), ("split_pages", C.c_int32)]


class PoolStats(C.Structure):
    _fields_ = [("pages_total", C.c_int64), ("pages_used", C.c_int64),
                ("pages_high_water", C.c_int64), ("streams_open", C.c_int64),
                ("compactions", C.c_int64), ("pages_moved", C.c_int64),
                ("bytes_moved", C.c_int64), ("device_bytes", C.c_int64),
                ("kernel_launches", C.c_int64)]


class EncConfig(C.Structure):
    _fields_ = [("struct_size", C.c_uint32), ("api_version", C.c_uint32), ("device", C.c_int32),
                ("n_layers", C.c_int32), ("n_heads", C.c_int32), ("head_dim", C.c_int32),
                ("window", C.c_int32), ("capacity", C.c_int32), ("max_streams", C.c_int32),
                ("max_new", C.c_int32), ("max_position", C.c_int32), ("dtype", C.c_int32),
                ("rope_theta", C.c_float), ("reserved", C.c_int32)]


class HeadConfig(C.Structure):
    _fields_ = [("struct_size", C.c_uint32), ("api_version", C.c_uint32), ("device", C.c_int32),
                ("dim", C.c_int32), ("vocab", C.c_int32), ("dtype", C.c_int32)]


class QWeightConfig(C.Structure):
    _fields_ = [("struct_size", C.c_uint32), ("api_version", C.c_uint32), ("device", C.c_int32),
                ("type", C.c_int32), ("n_rows", C.c_int32), ("n_cols", C.c_int32), ("max_batch", C.c_int32),
                ("reserved", C.c_int32)]


QTYPE_Q8_0, QTYPE_Q4_K, QTYPE_Q6_K = 8, 12, 14


class GgufTensor(C.Structure):
    _fields_ = [("name", C.c_char_p), ("type", C.c_int32), ("n_dims", C.c_int32), ("ne", C.c_int64 * 4),
                ("offset", C.c_uint64), ("n_bytes", C.c_uint64)]

class DecoderConfig(C.Structure):
    _fields_ = [("struct_size", C.c_uint32), ("api_version", C.c_uint32), ("audio_capacity", C.c_int32),
                ("enc_capacity", C.c_int32), ("time_value", C.c_float), ("reserved", C.c_int32 * 3)]


class DecoderInfo(C.Structure):
    _fields_ = [(n, C.c_int32) for n in ("n_layers", "dim", "hidden", "n_q_heads", "n_kv_heads", "head_dim",
                                         "vocab", "ada_dim", "emb_type", "max_rows", "max_streams",
                                         "audio_capacity", "enc_capacity", "enc_dim")] + [("device_bytes", C.c_int64)]


class EncoderInfo(C.Structure):
    _fields_ = [(n, C.c_int32) for n in ("n_layers", "dim", "hidden", "n_heads", "head_dim", "n_mel", "max_rows",
                                         "reserved")] + [("device_bytes", C.c_int64)]


class BatcherConfig(C.Structure):
    _fields_ = [("struct_size", C.c_uint32), ("api_version", C.c_uint32), ("max_rows", C.c_int32),
                ("max_wait_us", C.c_int32), ("expected", C.c_int32), ("timeout_ms", C.c_int32)]


class BatcherStats(C.Structure):
    _fields_ = [("batches", C.c_int64), ("rows", C.c_int64), ("max_rows_seen", C.c_int64),
                ("failed_batches", C.c_int64), ("timeouts", C.c_int64), ("mean_wait_us", C.c_double)]


BATCH_FN = C.CFUNCTYPE(C.c_int32, C.c_void_p, C.c_int32, C.POINTER(C.c_int32), C.POINTER(C.c_int32),
                       C.POINTER(C.c_int32), C.POINTER(C.c_int32))

_P = C.c_void_p
_I32 = C.c_int32
_I64 = C.c_int64
_I32P = C.POINTER(C.c_int32)
_I64P = C.POINTER(C.c_int64)

# name -> (restype, argtypes); every symbol declared in include/vxk.h
SIGNATURES = {
    "vxk_status_string": (C.c_char_p, [_I32]),
    "vxk_api_version": (C.c_uint32, []),
    "vxk_decoder_kv_plan_make": (_I32, [C.POINTER(DecoderKvRing), _I64, _I32, C.POINTER(DecoderKvPlan)]),
    "vxk_decoder_kv_plan_commit": (_I32, [C.POINTER(DecoderKvRing), C.POINTER(DecoderKvPlan)]),
    "vxk_enc_kv_plan_make": (_I32, [_I64, _I32, _I32, _I32, C.POINTER(EncKvPlan)]),
    "vxk_enc_kv_mask_allows": (_I32, [_I64, _I64, _I32]),
    "vxk_pool_default_config": (PoolConfig, []),
    "vxk_pool_create": (_I32, [C.POINTER(PoolConfig), C.POINTER(_P)]),
    "vxk_pool_destroy": (None, [_P]),
    "vxk_pool_last_error": (_I32, [_P, C.c_char_p, C.c_size_t]),
    "vxk_pool_get_stats": (_I32, [_P, C.POINTER(PoolStats)]),
    "vxk_stream_open": (_I32, [_P, _I32P]),
    "vxk_stream_close": (_I32, [_P, _I32]),
    "vxk_stream_reset": (_I32, [_P, _I32]),
    "vxk_stream_get_ring": (_I32, [_P, _I32, C.POINTER(DecoderKvRing)]),
    "vxk_stream_evict": (_I32, [_P, _I32, _I64]),
    "vxk_batch_plan": (_I32, [_P, _I32P, _I32P, _I32, _P]),
    "vxk_batch_rows": (_I32, [_P, _I32P]),
    "vxk_batch_commit": (_I32, [_P]),
    "vxk_batch_abort": (_I32, [_P]),
    "vxk_decode_layer": (_I32, [_P, _I32, _P, _P, _P, _P, _P]),
    "vxk_decode_layer_static_scratch": (_I32, [_P, _I32, _P, _P, _P, _P, _P]),
    "vxk_append_layer": (_I32, [_P, _I32, _P, _P, _P]),
    "vxk_attend_layer": (_I32, [_P, _I32, _P, _P, _P]),
    "vxk_decode_step_host": (_I32, [_P, _I32P, _I32, _P, _P, _P, _P, _P]),
    "vxk_sync": (_I32, [_P, _P, _I32]),
    "vxk_pool_compact": (_I32, [_P, _P, _I64P, _I64P]),
    "vxk_read_rows": (_I32, [_P, _I32, _I32, _I64, _I32, _P, _P, _P]),
    "vxk_pool_row_bytes": (_I64, [_P]),
    "vxk_enc_default_config": (EncConfig, []),
    "vxk_enc_create": (_I32, [C.POINTER(EncConfig), C.POINTER(_P)]),
    "vxk_enc_destroy": (None, [_P]),
    "vxk_enc_last_error": (_I32, [_P, C.c_char_p, C.c_size_t]),
    "vxk_enc_stream_open": (_I32, [_P, _I32P]),
    "vxk_enc_stream_close": (_I32, [_P, _I32]),
    "vxk_enc_stream_reset": (_I32, [_P, _I32]),
    "vxk_enc_stream_position": (_I32, [_P, _I32, _I64P, _I64P]),
    "vxk_enc_batch_plan": (_I32, [_P, _I32P, _I32P, _I32, _P]),
    "vxk_enc_batch_rows": (_I32, [_P, _I32P]),
    "vxk_enc_batch_commit": (_I32, [_P]),
    "vxk_enc_layer": (_I32, [_P, _I32, _P, _P, _P, _P, _P]),
    "vxk_enc_read_slots": (_I32, [_P, _I32, _I32, _I32, _I32, _P, _P, _P]),
    "vxk_pool_probe_wait_timeout": (_I32, [_P, _I32, _P]),
    "vxk_head_default_config": (HeadConfig, []),
    "vxk_head_create": (_I32, [C.POINTER(HeadConfig), C.POINTER(C.c_void_p)]),
    "vxk_head_destroy": (None, [_P]),
    "vxk_head_last_error": (_I32, [_P, C.c_char_p, C.c_size_t]),
    "vxk_head_logits_argmax": (_I32, [_P, _P, _P, _I32, _P, _P, _P]),
    "vxk_head_sync": (_I32, [_P, _P, _I32]),
    "vxk_head_logits_argmax_q": (_I32, [_P, _P, _P, _I32, _P, _P, _P]),
    "vxk_qweight_default_config": (QWeightConfig, []),
    "vxk_qweight_packed_bytes": (_I32, [_I32, _I32, _I32, C.POINTER(C.c_size_t)]),
    "vxk_qweight_repack": (_I32, [_I32, _I32, _I32, _P, C.c_size_t, _P, C.c_size_t]),
    "vxk_qweight_create": (_I32, [C.POINTER(QWeightConfig), _P, C.c_size_t, C.POINTER(C.c_void_p)]),
    "vxk_qweight_destroy": (None, [_P]),
    "vxk_qweight_last_error": (_I32, [_P, C.c_char_p, C.c_size_t]),
    "vxk_qweight_matmul": (_I32, [_P, _P, _I32, _P, _P]),
    "vxk_qweight_matmul_group": (_I32, [C.POINTER(C.c_void_p), _I32, _P, _I32, C.POINTER(C.c_void_p), _P]),
    "vxk_qweight_sync": (_I32, [_P, _P, _I32]),
    "vxk_gguf_open": (_I32, [C.c_char_p, C.POINTER(C.c_void_p)]),
    "vxk_gguf_close": (None, [_P]),
    "vxk_gguf_last_error": (_I32, [_P, C.c_char_p, C.c_size_t]),
    "vxk_gguf_version": (C.c_uint32, [_P]),
    "vxk_gguf_n_tensors": (_I64, [_P]),
    "vxk_gguf_get_tensor": (_I32, [_P, _I64, C.POINTER(GgufTensor)]),
    "vxk_gguf_find_tensor": (_I64, [_P, C.c_char_p]),
    "vxk_gguf_tensor_data": (_P, [_P, _I64]),
    "vxk_gguf_n_keys": (_I64, [_P]),
    "vxk_gguf_key": (C.c_char_p, [_P, _I64]),
    "vxk_gguf_key_type": (_I32, [_P, C.c_char_p]),
    "vxk_gguf_get_int": (_I32, [_P, C.c_char_p, _I64P]),
    "vxk_gguf_get_float": (_I32, [_P, C.c_char_p, C.POINTER(C.c_double)]),
    "vxk_gguf_get_str": (_I32, [_P, C.c_char_p, C.POINTER(C.c_char_p)]),
    "vxk_gguf_get_array": (_I32, [_P, C.c_char_p, _I32P, _I64P, C.POINTER(C.c_void_p)]),
    "vxk_gguf_get_array_str": (_I32, [_P, C.c_char_p, _I64, C.POINTER(C.c_char_p)]),
    "vxk_qweight_create_from_gguf": (_I32, [_P, C.c_char_p, _I32, _I32, C.POINTER(C.c_void_p)]),
    "vxk_decoder_default_config": (DecoderConfig, []),
    "vxk_decoder_create": (_I32, [_P, _P, C.POINTER(DecoderConfig), C.POINTER(C.c_void_p)]),
    "vxk_decoder_destroy": (None, [_P]),
    "vxk_decoder_last_error": (_I32, [_P, C.c_char_p, C.c_size_t]),
    "vxk_decoder_get_info": (_I32, [_P, C.POINTER(DecoderInfo)]),
    "vxk_decoder_forward": (_I32, [_P, _I32P, _I32P, _P, _P, _P, _P]),
    "vxk_decoder_write_enc": (_I32, [_P, _I32, _I64, _I32, _P, _P]),
    "vxk_decoder_write_audio": (_I32, [_P, _I32, _I64, _I32, _P, _P]),
    "vxk_decoder_adapt": (_I32, [_P, _I32, _I32P, _I64P, _I64P, _P]),
    "vxk_decoder_read_audio": (_I32, [_P, _I32, _I64, _I32, _P, _P]),
    "vxk_decoder_sync": (_I32, [_P, _P, _I32]),
    "vxk_encoder_create": (_I32, [_P, _P, _I32, C.POINTER(C.c_void_p)]),
    "vxk_encoder_destroy": (None, [_P]),
    "vxk_encoder_last_error": (_I32, [_P, C.c_char_p, C.c_size_t]),
    "vxk_encoder_get_info": (_I32, [_P, C.POINTER(EncoderInfo)]),
    "vxk_encoder_forward": (_I32, [_P, _P, _P, _P]),
    "vxk_encoder_stem": (_I32, [_P, _P, _P, _P]),
    "vxk_encoder_sync": (_I32, [_P, _P, _I32]),
    "vxk_batcher_default_config": (BatcherConfig, []),
    "vxk_batcher_create": (_I32, [C.POINTER(BatcherConfig), BATCH_FN, _P, C.POINTER(C.c_void_p)]),
    "vxk_batcher_create_for_decoder": (_I32, [C.POINTER(BatcherConfig), _P, _P, _P, C.POINTER(C.c_void_p)]),
    "vxk_batcher_destroy": (None, [_P]),
    "vxk_batcher_step": (_I32, [_P, _I32, _I32, _I32, _I32P]),
    "vxk_batcher_get_stats": (_I32, [_P, C.POINTER(BatcherStats)]),
}

_lib = None


def load(path: str | os.PathLike | None = None) -> C.CDLL:
    """Loads libvxk.so; raises if it is missing (build it with build.py)."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise ImportError(f"{p} is not built; run voxtral.cpp_b200/build.py")
    lib = C.CDLL(str(p))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = lib
    return lib


def _i32_array(values):
    arr = (C.c_int32 * len(values))(*values)
    return arr


class Pool:
    """Owns one vxk_pool (decoder paged KV cache on one device)."""

    def __init__(self, **cfg):
        self.lib = load()
        c = self.lib.vxk_pool_default_config()
        for k, v in cfg.items():
            if not hasattr(c, k):
                raise AttributeError(k)
            setattr(c, k, v)
        self.config = c
        h = C.c_void_p()
        st = self.lib.vxk_pool_create(C.byref(c), C.byref(h))
        if st != OK:
            raise VxkError(st, self.last_error(None))
        self.h = h

    def last_error(self, handle="self") -> str:
        buf = C.create_string_buffer(1024)
        hv = self.h if handle == "self" else handle
        self.lib.vxk_pool_last_error(hv, buf, 1024)
        return buf.value.decode()

    def _check(self, st: int):
        if st != OK:
            raise VxkError(st, self.last_error())

    def close(self):
        if getattr(self, "h", None):
            self.lib.vxk_pool_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def open_stream(self) -> int:
        sid = C.c_int32()
        self._check(self.lib.vxk_stream_open(self.h, C.byref(sid)))
        return sid.value

    def close_stream(self, sid: int):
        self._check(self.lib.vxk_stream_close(self.h, sid))

    def reset_stream(self, sid: int):
        self._check(self.lib.vxk_stream_reset(self.h, sid))

    def ring(self, sid: int) -> DecoderKvRing:
        r = DecoderKvRing()
        self._check(self.lib.vxk_stream_get_ring(self.h, sid, C.byref(r)))
        return r

    def evict(self, sid: int, new_oldest: int):
        self._check(self.lib.vxk_stream_evict(self.h, sid, new_oldest))

    def plan(self, stream_ids, n_new, cuda_stream=0) -> int:
        ids = _i32_array(list(stream_ids))
        nn = _i32_array(list(n_new))
        self._check(self.lib.vxk_batch_plan(self.h, ids, nn, len(stream_ids), C.c_void_p(cuda_stream)))
        rows = C.c_int32()
        self._check(self.lib.vxk_batch_rows(self.h, C.byref(rows)))
        return rows.value

    def commit(self):
        self._check(self.lib.vxk_batch_commit(self.h))

    def abort(self):
        self._check(self.lib.vxk_batch_abort(self.h))

    def decode_layer(self, layer, q, k, v, out, cuda_stream=0):
        self._check(self.lib.vxk_decode_layer(self.h, layer, q, k, v, out, C.c_void_p(cuda_stream)))

    def decode_layer_static_scratch(self, layer, q, k, v, out, cuda_stream=0):
        """decode_layer whose split scratch is the library's fixed device array
        (no device allocation behind the call)."""
        self._check(self.lib.vxk_decode_layer_static_scratch(self.h, layer, q, k, v, out,
                                                             C.c_void_p(cuda_stream)))

    def append_layer(self, layer, k, v, cuda_stream=0):
        self._check(self.lib.vxk_append_layer(self.h, layer, k, v, C.c_void_p(cuda_stream)))

    def attend_layer(self, layer, q, out, cuda_stream=0):
        self._check(self.lib.vxk_attend_layer(self.h, layer, q, out, C.c_void_p(cuda_stream)))

    def decode_step_host(self, stream_ids, h_q, h_k, h_v, h_out, cuda_stream=0):
        ids = _i32_array(list(stream_ids))
        self._check(self.lib.vxk_decode_step_host(self.h, ids, len(stream_ids), h_q, h_k, h_v, h_out,
                                                  C.c_void_p(cuda_stream)))

    def sync(self, cuda_stream=0, timeout_ms=60000):
        self._check(self.lib.vxk_sync(self.h, C.c_void_p(cuda_stream), timeout_ms))

    def probe_wait_timeout(self, limit_ms, cuda_stream=0):
        self._check(self.lib.vxk_pool_probe_wait_timeout(self.h, limit_ms, C.c_void_p(cuda_stream)))

    def compact(self, cuda_stream=0):
        pm, bm = C.c_int64(), C.c_int64()
        self._check(self.lib.vxk_pool_compact(self.h, C.c_void_p(cuda_stream), C.byref(pm), C.byref(bm)))
        return pm.value, bm.value

    def stats(self) -> PoolStats:
        s = PoolStats()
        self._check(self.lib.vxk_pool_get_stats(self.h, C.byref(s)))
        return s

    def row_bytes(self) -> int:
        return int(self.lib.vxk_pool_row_bytes(self.h))

    def read_rows(self, layer, sid, pos_start, n, cuda_stream=0):
        import numpy as np
        rb = self.row_bytes()
        k = np.zeros((n, rb), dtype=np.uint8)
        v = np.zeros((n, rb), dtype=np.uint8)
        self._check(self.lib.vxk_read_rows(self.h, layer, sid, pos_start, n, k.ctypes.data, v.ctypes.data,
                                           C.c_void_p(cuda_stream)))
        return k, v


class EncPool:
    """Owns one vxk_enc_pool (streaming-encoder KV rings on one device)."""

    def __init__(self, **cfg):
        self.lib = load()
        c = self.lib.vxk_enc_default_config()
        for k, v in cfg.items():
            if not hasattr(c, k):
                raise AttributeError(k)
            setattr(c, k, v)
        self.config = c
        h = C.c_void_p()
        st = self.lib.vxk_enc_create(C.byref(c), C.byref(h))
        if st != OK:
            raise VxkError(st, self.last_error(None))
        self.h = h

    def last_error(self, handle="self") -> str:
        buf = C.create_string_buffer(1024)
        hv = self.h if handle == "self" else handle
        self.lib.vxk_enc_last_error(hv, buf, 1024)
        return buf.value.decode()

    def _check(self, st):
        if st != OK:
            raise VxkError(st, self.last_error())

    def close(self):
        if getattr(self, "h", None):
            self.lib.vxk_enc_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def open_stream(self) -> int:
        sid = C.c_int32()
        self._check(self.lib.vxk_enc_stream_open(self.h, C.byref(sid)))
        return sid.value

    def position(self, sid):
        nx, ev = C.c_int64(), C.c_int64()
        self._check(self.lib.vxk_enc_stream_position(self.h, sid, C.byref(nx), C.byref(ev)))
        return nx.value, ev.value

    def plan(self, stream_ids, n_new, cuda_stream=0) -> int:
        ids = _i32_array(list(stream_ids))
        nn = _i32_array(list(n_new))
        self._check(self.lib.vxk_enc_batch_plan(self.h, ids, nn, len(stream_ids), C.c_void_p(cuda_stream)))
        rows = C.c_int32()
        self._check(self.lib.vxk_enc_batch_rows(self.h, C.byref(rows)))
        return rows.value

    def commit(self):
        self._check(self.lib.vxk_enc_batch_commit(self.h))

    def layer(self, layer, q, k, v, out, cuda_stream=0):
        self._check(self.lib.vxk_enc_layer(self.h, layer, q, k, v, out, C.c_void_p(cuda_stream)))

    def read_slots(self, layer, sid, slot0, n, cuda_stream=0):
        import numpy as np
        c = self.config
        k = np.zeros((n, c.n_heads * c.head_dim), dtype=np.uint32 if c.dtype == 0 else np.uint16)
        v = np.zeros_like(k)
        self._check(self.lib.vxk_enc_read_slots(self.h, layer, sid, slot0, n, k.ctypes.data, v.ctypes.data,
                                                C.c_void_p(cuda_stream)))
        return k, v


class Head:
    """Owns one vxk_head (greedy head: tied logits and argmax on one device)."""

    def __init__(self, **cfg):
        self.lib = load()
        c = self.lib.vxk_head_default_config()
        for k, v in cfg.items():
            if not hasattr(c, k):
                raise AttributeError(k)
            setattr(c, k, v)
        self.config = c
        h = C.c_void_p()
        st = self.lib.vxk_head_create(C.byref(c), C.byref(h))
        if st != OK:
            raise VxkError(st, self.last_error(None))
        self.h = h

    def last_error(self, handle="self") -> str:
        buf = C.create_string_buffer(1024)
        hv = self.h if handle == "self" else handle
        self.lib.vxk_head_last_error(hv, buf, 1024)
        return buf.value.decode()

    def _check(self, st):
        if st != OK:
            raise VxkError(st, self.last_error())

    def close(self):
        if getattr(self, "h", None):
            self.lib.vxk_head_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def logits_argmax(self, w_ptr, x_ptr, rows, argmax_ptr, logits_ptr=0, cuda_stream=0):
        self._check(self.lib.vxk_head_logits_argmax(self.h, C.c_void_p(w_ptr), C.c_void_p(x_ptr), rows,
                                                    C.c_void_p(argmax_ptr), C.c_void_p(logits_ptr or None),
                                                    C.c_void_p(cuda_stream)))

    def logits_argmax_q(self, qweight, x_ptr, rows, argmax_ptr, logits_ptr=0, cuda_stream=0):
        """Greedy head over quantized embeddings (vxk_head_logits_argmax_q)."""
        self._check(self.lib.vxk_head_logits_argmax_q(self.h, qweight.h, C.c_void_p(x_ptr), rows,
                                                      C.c_void_p(argmax_ptr), C.c_void_p(logits_ptr or None),
                                                      C.c_void_p(cuda_stream)))

    def sync(self, cuda_stream=0, timeout_ms=10000):
        self._check(self.lib.vxk_head_sync(self.h, C.c_void_p(cuda_stream), timeout_ms))


# ---- planners (host only) -------------------------------------------------

def decoder_plan(ring: DecoderKvRing, start: int, n_new: int):
    lib = load()
    p = DecoderKvPlan()
    st = lib.vxk_decoder_kv_plan_make(C.byref(ring), start, n_new, C.byref(p))
    return st, p


def decoder_commit(ring: DecoderKvRing, plan: DecoderKvPlan):
    lib = load()
    return lib.vxk_decoder_kv_plan_commit(C.byref(ring), C.byref(plan))


def enc_plan(q_start: int, n_new: int, capacity: int, window: int):
    lib = load()
    p = EncKvPlan()
    st = lib.vxk_enc_kv_plan_make(q_start, n_new, capacity, window, C.byref(p))
    return st, p


def enc_mask_allows(kv: int, q: int, window: int) -> bool:
    return bool(load().vxk_enc_kv_mask_allows(kv, q, window))


class QWeight:
    """Owns one vxk_qweight: a GGUF Q8_0 / Q4_K / Q6_K matrix on one device
    and the scratch of its products (ggml_mul_mat with ggml's CPU
    arithmetic)."""

    def __init__(self, gguf_blocks, **cfg):
        import numpy as np

        self.lib = load()
        c = self.lib.vxk_qweight_default_config()
        for k, v in cfg.items():
            if not hasattr(c, k):
                raise AttributeError(k)
            setattr(c, k, v)
        self.config = c
        blocks = np.ascontiguousarray(gguf_blocks, dtype=np.uint8)
        h = C.c_void_p()
        st = self.lib.vxk_qweight_create(C.byref(c), blocks.ctypes.data, blocks.nbytes, C.byref(h))
        if st != OK:
            raise VxkError(st, self.last_error(None))
        self.h = h

    def last_error(self, handle="self") -> str:
        buf = C.create_string_buffer(1024)
        hv = self.h if handle == "self" else handle
        self.lib.vxk_qweight_last_error(hv, buf, 1024)
        return buf.value.decode()

    def _check(self, st):
        if st != OK:
            raise VxkError(st, self.last_error())

    def close(self):
        if getattr(self, "h", None):
            self.lib.vxk_qweight_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def matmul(self, x_ptr, rows, y_ptr, cuda_stream=0):
        self._check(self.lib.vxk_qweight_matmul(self.h, C.c_void_p(x_ptr), rows, C.c_void_p(y_ptr),
                                                C.c_void_p(cuda_stream)))

    def sync(self, cuda_stream=0, timeout_ms=10000):
        self._check(self.lib.vxk_qweight_sync(self.h, C.c_void_p(cuda_stream), timeout_ms))


def qweight_matmul_group(mats, x_ptr, rows, y_ptrs, cuda_stream=0):
    """vxk_qweight_matmul_group: one quantization of x, one launch for all of
    `mats` (QWeight objects sharing n_cols and the activation family)."""
    lib = load()
    n = len(mats)
    ws = (C.c_void_p * n)(*[m.h.value for m in mats])
    ys = (C.c_void_p * n)(*y_ptrs)
    st = lib.vxk_qweight_matmul_group(ws, n, C.c_void_p(x_ptr), rows, ys, C.c_void_p(cuda_stream))
    if st != OK:
        raise VxkError(st, mats[0].last_error() if n else "")


def qweight_repack(qtype: int, n_rows: int, n_cols: int, gguf_blocks):
    """Host repack of GGUF rows into the device record layout (vxk_qweight_repack)."""
    import numpy as np

    lib = load()
    size = C.c_size_t()
    st = lib.vxk_qweight_packed_bytes(qtype, n_rows, n_cols, C.byref(size))
    if st != OK:
        raise VxkError(st, "packed_bytes")
    blocks = np.ascontiguousarray(gguf_blocks, dtype=np.uint8)
    out = np.empty(size.value, np.uint8)
    st = lib.vxk_qweight_repack(qtype, n_rows, n_cols, blocks.ctypes.data, blocks.nbytes, out.ctypes.data, out.nbytes)
    if st != OK:
        raise VxkError(st, "repack")
    return out


class Gguf:
    """A GGUF file opened by vxk_gguf_open (metadata, tensor table, mapped bytes)."""

    def __init__(self, path):
        self.lib = load()
        h = C.c_void_p()
        st = self.lib.vxk_gguf_open(str(path).encode(), C.byref(h))
        if st != OK:
            buf = C.create_string_buffer(1024)
            self.lib.vxk_gguf_last_error(None, buf, 1024)
            raise VxkError(st, buf.value.decode())
        self.h = h

    def close(self):
        if getattr(self, "h", None):
            self.lib.vxk_gguf_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def version(self):
        return int(self.lib.vxk_gguf_version(self.h))

    def tensors(self):
        out = []
        for i in range(self.lib.vxk_gguf_n_tensors(self.h)):
            t = GgufTensor()
            if self.lib.vxk_gguf_get_tensor(self.h, i, C.byref(t)) != OK:
                raise VxkError(1, "get_tensor")
            out.append(dict(name=t.name.decode(), type=t.type, n_dims=t.n_dims, ne=list(t.ne)[: t.n_dims],
                            offset=int(t.offset), n_bytes=int(t.n_bytes)))
        return out

    def find_tensor(self, name):
        return int(self.lib.vxk_gguf_find_tensor(self.h, name.encode()))

    def tensor_bytes(self, name):
        import numpy as np

        i = self.find_tensor(name)
        if i < 0:
            raise KeyError(name)
        t = self.tensors()[i]
        ptr = self.lib.vxk_gguf_tensor_data(self.h, i)
        if not ptr:
            raise VxkError(1, "tensor data not available")
        return np.ctypeslib.as_array((C.c_uint8 * t["n_bytes"]).from_address(ptr)).copy()

    def keys(self):
        return [self.lib.vxk_gguf_key(self.h, i).decode() for i in range(self.lib.vxk_gguf_n_keys(self.h))]

    def key_type(self, key):
        return int(self.lib.vxk_gguf_key_type(self.h, key.encode()))

    def get(self, key):
        """Scalar or array value of a key (ints widened, floats as float)."""
        import numpy as np

        t = self.key_type(key)
        k = key.encode()
        if t < 0:
            raise KeyError(key)
        if t == 8:
            s = C.c_char_p()
            self.lib.vxk_gguf_get_str(self.h, k, C.byref(s))
            return s.value.decode()
        if t in (6, 12):
            d = C.c_double()
            self.lib.vxk_gguf_get_float(self.h, k, C.byref(d))
            return d.value
        if t == 9:
            et, n, p = C.c_int32(), C.c_int64(), C.c_void_p()
            self.lib.vxk_gguf_get_array(self.h, k, C.byref(et), C.byref(n), C.byref(p))
            if et.value == 8:
                out = []
                for i in range(n.value):
                    s = C.c_char_p()
                    self.lib.vxk_gguf_get_array_str(self.h, k, i, C.byref(s))
                    out.append(s.value.decode())
                return out
            dt = {0: np.uint8, 1: np.int8, 2: np.uint16, 3: np.int16, 4: np.uint32, 5: np.int32, 6: np.float32,
                  7: np.bool_, 10: np.uint64, 11: np.int64, 12: np.float64}[et.value]
            nb = n.value * np.dtype(dt).itemsize
            raw = np.ctypeslib.as_array((C.c_uint8 * nb).from_address(p.value)).copy() if nb else np.zeros(0, np.uint8)
            return raw.view(dt)
        v = C.c_int64()
        self.lib.vxk_gguf_get_int(self.h, k, C.byref(v))
        return bool(v.value) if t == 7 else int(v.value)

    def qweight(self, name, device=0, max_batch=64):
        q = QWeight.__new__(QWeight)
        q.lib = self.lib
        h = C.c_void_p()
        st = self.lib.vxk_qweight_create_from_gguf(self.h, name.encode(), device, max_batch, C.byref(h))
        if st != OK:
            raise VxkError(st, q.last_error(None))
        q.h = h
        return q


class Decoder:
    """Owns one vxk_decoder: a GGUF model's decoder, head and adapter on the
    pool's device, run over the pool's planned batch (vxk_decoder_forward)."""

    def __init__(self, gguf: "Gguf", pool: Pool, **cfg):
        self.lib = load()
        c = self.lib.vxk_decoder_default_config()
        for k, v in cfg.items():
            if not hasattr(c, k):
                raise AttributeError(k)
            setattr(c, k, v)
        self.config = c
        self.pool = pool
        h = C.c_void_p()
        st = self.lib.vxk_decoder_create(gguf.h, pool.h, C.byref(c), C.byref(h))
        if st != OK:
            raise VxkError(st, self._error(None))
        self.h = h
        info = DecoderInfo()
        self._check(self.lib.vxk_decoder_get_info(self.h, C.byref(info)))
        self.info = {n: getattr(info, n) for n, _ in DecoderInfo._fields_}

    def _error(self, h) -> str:
        buf = C.create_string_buffer(1024)
        self.lib.vxk_decoder_last_error(h, buf, 1024)
        return buf.value.decode()

    def _check(self, st: int):
        if st != OK:
            raise VxkError(st, self._error(self.h))

    def close(self):
        if getattr(self, "h", None):
            self.lib.vxk_decoder_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def forward(self, tokens, audio_slots, argmax_ptr: int, logits_ptr: int = 0, hidden_ptr: int = 0,
                cuda_stream: int = 0):
        """tokens / audio_slots: one int per row of the planned batch (host)."""
        t = _i32_array(list(tokens))
        a = _i32_array(list(audio_slots))
        self._check(self.lib.vxk_decoder_forward(self.h, t, a, argmax_ptr, logits_ptr or None, hidden_ptr or None,
                                                 cuda_stream or None))

    def write_enc(self, stream: int, frame: int, n: int, rows_ptr: int, cuda_stream: int = 0):
        self._check(self.lib.vxk_decoder_write_enc(self.h, stream, frame, n, rows_ptr, cuda_stream or None))

    def write_audio(self, stream: int, pos: int, n: int, rows_ptr: int, cuda_stream: int = 0):
        self._check(self.lib.vxk_decoder_write_audio(self.h, stream, pos, n, rows_ptr, cuda_stream or None))

    def read_audio(self, stream: int, pos: int, n: int, rows_ptr: int, cuda_stream: int = 0):
        self._check(self.lib.vxk_decoder_read_audio(self.h, stream, pos, n, rows_ptr, cuda_stream or None))

    def adapt(self, streams, enc_frames, audio_pos, cuda_stream: int = 0):
        n = len(streams)
        s = _i32_array(list(streams))
        e = (C.c_int64 * n)(*enc_frames)
        a = (C.c_int64 * n)(*audio_pos)
        self._check(self.lib.vxk_decoder_adapt(self.h, n, s, e, a, cuda_stream or None))

    def sync(self, cuda_stream: int = 0, timeout_ms: int = 10000):
        self._check(self.lib.vxk_decoder_sync(self.h, cuda_stream or None, timeout_ms))


class Batcher:
    """Owns one vxk_batcher.  `fn(streams, tokens, audio_slots) -> (status,
    out_tokens)` runs a batch on the dispatcher thread (a host executor), or
    pass decoder= / pool= for the built-in decoder executor."""

    def __init__(self, fn=None, decoder=None, pool=None, cuda_stream=0, **cfg):
        self.lib = load()
        c = self.lib.vxk_batcher_default_config()
        for k, v in cfg.items():
            if not hasattr(c, k):
                raise AttributeError(k)
            setattr(c, k, v)
        self.config = c
        h = C.c_void_p()
        if fn is not None:
            def tramp(user, n, streams, tokens, slots, outs):
                try:
                    st, res = fn([streams[i] for i in range(n)], [tokens[i] for i in range(n)],
                                 [slots[i] for i in range(n)])
                    for i, v in enumerate(res):
                        outs[i] = int(v)
                    return int(st)
                except Exception:
                    return 10
            self._cb = BATCH_FN(tramp)  # kept alive with the batcher
            st = self.lib.vxk_batcher_create(C.byref(c), self._cb, None, C.byref(h))
        else:
            st = self.lib.vxk_batcher_create_for_decoder(C.byref(c), decoder.h, pool.h, cuda_stream or None,
                                                         C.byref(h))
        if st != OK:
            raise VxkError(st, "vxk_batcher_create failed")
        self.h = h

    def step(self, stream: int, token: int, audio_slot: int) -> int:
        out = C.c_int32(-1)
        st = self.lib.vxk_batcher_step(self.h, stream, token, audio_slot, C.byref(out))
        if st != OK:
            raise VxkError(st, "vxk_batcher_step failed")
        return out.value

    def stats(self) -> dict:
        s = BatcherStats()
        st = self.lib.vxk_batcher_get_stats(self.h, C.byref(s))
        if st != OK:
            raise VxkError(st, "vxk_batcher_get_stats failed")
        return {n: getattr(s, n) for n, _ in BatcherStats._fields_}

    def close(self):
        if getattr(self, "h", None):
            self.lib.vxk_batcher_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Encoder:
    """Owns one vxk_encoder: a GGUF model's streaming encoder stack on an
    encoder pool's device, run over the pool's planned batch."""

    def __init__(self, gguf: "Gguf", pool: "EncPool", max_rows: int = 0):
        self.lib = load()
        h = C.c_void_p()
        st = self.lib.vxk_encoder_create(gguf.h, pool.h, max_rows, C.byref(h))
        if st != OK:
            raise VxkError(st, self._error(None))
        self.h = h
        info = EncoderInfo()
        self._check(self.lib.vxk_encoder_get_info(self.h, C.byref(info)))
        self.info = {n: getattr(info, n) for n, _ in EncoderInfo._fields_}

    def _error(self, h) -> str:
        buf = C.create_string_buffer(1024)
        self.lib.vxk_encoder_last_error(h, buf, 1024)
        return buf.value.decode()

    def _check(self, st: int):
        if st != OK:
            raise VxkError(st, self._error(self.h))

    def forward(self, mel_ptr: int, out_ptr: int, cuda_stream: int = 0):
        self._check(self.lib.vxk_encoder_forward(self.h, mel_ptr, out_ptr, cuda_stream or None))

    def stem(self, mel_ptr: int, out_ptr: int, cuda_stream: int = 0):
        self._check(self.lib.vxk_encoder_stem(self.h, mel_ptr, out_ptr, cuda_stream or None))

    def sync(self, cuda_stream: int = 0, timeout_ms: int = 10000):
        self._check(self.lib.vxk_encoder_sync(self.h, cuda_stream or None, timeout_ms))

    def close(self):
        if getattr(self, "h", None):
            self.lib.vxk_encoder_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

