"""ctypes binding of libcacheslide_sm100.so (the C ABI in include/cacheslide_b200.h).

Loading is strict: if the shared library is missing or cannot be loaded, every
operator raises ``RuntimeError``.  There is no CPU fallback anywhere in this
package; operators also reject CPU tensors.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libcacheslide_sm100.so"

CS_OK, CS_ERR_INVALID, CS_ERR_CUDA, CS_ERR_UNSUPPORTED, CS_ERR_TOO_LARGE = 0, 1, 2, 3, 4
CS_F32, CS_F16, CS_BF16, CS_F64 = 0, 1, 2, 3

ST_SLOT_RANGE = 1 << 0
ST_NONFINITE = 1 << 1
ST_LOGIT_NONFINITE = 1 << 2
ST_POS_RANGE = 1 << 3
ST_PATH_NEG = 1 << 4
ST_PATH_AVAIL = 1 << 5
ST_PATH_INCR = 1 << 6
ST_PATH_GAP = 1 << 7
ST_TIMEOUT = 1 << 8
ST_INPUT_NONFINITE = 1 << 9

POS_CONTEXTUAL, POS_FIXED, POS_TABLE, POS_CHUNK = 0, 1, 2, 3
LAUNCH_OVERLAP_PREV = 1

DTYPES = {
    torch.float32: CS_F32,
    torch.float16: CS_F16,
    torch.bfloat16: CS_BF16,
    torch.float64: CS_F64,
}

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int32
_f64 = ctypes.c_double


class PagedKV(ctypes.Structure):
    _fields_ = [
        ("cache", _p),
        ("num_blocks", _i64), ("kv_heads", _i64), ("block_size", _i64), ("head_dim", _i64),
        ("stride_block", _i64), ("stride_head", _i64), ("stride_offset", _i64),
        ("stride_elem", _i64),
        ("side_k", _p), ("side_v", _p), ("side_capacity", _i64),
        ("side_stride_row", _i64), ("side_stride_head", _i64), ("side_stride_elem", _i64),
        ("dtype", _i32),
    ]


class AttnParams(ctypes.Structure):
    _fields_ = [
        ("q", _p), ("q_stride_tok", _i64), ("q_stride_head", _i64),
        ("nq", _i32), ("hq", _i32), ("d", _i32),
        ("qpos", _p),
        ("k", _p), ("v", _p),
        ("k_stride_tok", _i64), ("k_stride_head", _i64),
        ("v_stride_tok", _i64), ("v_stride_head", _i64),
        ("paged", PagedKV),
        ("kv_slots", _p),
        ("nk", _i32), ("hkv", _i32), ("dv", _i32),
        ("kpos", _p),
        ("E", _p), ("e_stride_d", _i64), ("e_stride_p", _i64), ("npos", _i32),
        ("scale", _f64),
        ("pos_mode", _i32),
        ("fixed_pos", _p), ("fp_stride_h", _i64), ("fp_stride_q", _i64), ("fp_stride_k", _i64),
        ("table", _p), ("tb_stride_h", _i64), ("tb_stride_r", _i64), ("tb_stride_c", _i64),
        ("q_row", _p), ("k_ord", _p),
        ("key_chunk", _p), ("chunk_off", _p), ("co_stride_h", _i64), ("co_stride_q", _i64),
        ("nchunks", _i32),
        ("gate_mask", _p), ("gm_stride_h", _i64), ("gm_stride_q", _i64),
        ("vis_mask", _p), ("vm_stride_h", _i64), ("vm_stride_q", _i64),
        ("q_selected", _p), ("k_fixed", _p),
        ("strict", _i32), ("atol", _f64), ("positions_only", _i32),
        ("out_positions", _p), ("op_stride_h", _i64), ("op_stride_q", _i64),
        ("out", _p), ("o_stride_tok", _i64), ("o_stride_head", _i64),
        ("in_dtype", _i32), ("out_dtype", _i32),
        ("status", _p),
        ("launch_flags", _i32),
        ("nq_dev", _p),
    ]


class ScatterItem(ctypes.Structure):
    """cs_slide_scatter_item: one request of cs_slide_scatter_batch."""
    _fields_ = [
        ("slots", _p), ("rows", _p), ("n", _i64), ("k", _p), ("v", _p),
        ("in_stride_row", _i64), ("in_stride_head", _i64), ("status", _p),
    ]


class InitializeItem(ctypes.Structure):
    """cs_wca_initialize_item: one request of cs_wca_initialize_batch."""
    _fields_ = [
        ("cached", _p), ("c_stride_row", _i64), ("c_stride_head", _i64),
        ("fresh", _p), ("f_stride_row", _i64), ("f_stride_head", _i64),
        ("n", _i64), ("reused", _p), ("dev_out", _p), ("alpha_out", _p), ("candidate", _p),
        ("selected", _p), ("removed", _p), ("counts_out", _p), ("status", _p),
    ]


class UpdateItem(ctypes.Structure):
    """cs_wca_update_item: one request of cs_wca_update_batch."""
    _fields_ = [
        ("cached_k", _p), ("cached_v", _p), ("c_stride_row", _i64), ("c_stride_head", _i64),
        ("fresh_k", _p), ("fresh_v", _p), ("f_stride_row", _i64), ("f_stride_head", _i64),
        ("indices", _p), ("a", _i64), ("alpha", _p), ("mandatory", _p),
        ("fused_k", _p), ("fused_v", _p), ("next_alpha_out", _p), ("used_alpha_out", _p),
        ("cos_out", _p), ("slots", _p), ("status", _p), ("a_dev", _p),
    ]


class CommitItem(ctypes.Structure):
    """cs_wca_commit_item: one request of cs_wca_commit_batch."""
    _fields_ = [
        ("indices", _p), ("a", _i64), ("next_alpha", _p), ("cos", _p), ("n", _i64),
        ("budget", _i64), ("initial_dev", _p), ("alpha", _p), ("candidate", _p),
        ("selected", _p), ("removed", _p), ("removed_out", _p), ("promoted_out", _p),
        ("counts_out", _p), ("status", _p), ("a_dev", _p),
    ]


class QKVParams(ctypes.Structure):
    """cs_qkv_params: the selective-layer QKV projection (cs_qkv_gather_lora)."""
    _fields_ = [
        ("src0", _p), ("src0_stride", _i64), ("src0_rows", _i64),
        ("src1", _p), ("src1_stride", _i64), ("src1_rows", _i64),
        ("row_src", _p), ("row_idx", _p), ("a", _i64), ("hidden", _i64), ("n_out", _i64),
        ("w", _p), ("lora_a", _p), ("lora_b", _p), ("rank", _i32),
        ("out", _p), ("out_stride", _i64), ("dtype", _i32), ("status", _p), ("a_dev", _p),
    ]


_SIGNATURES = {
    "cs_slide_gather": [ctypes.POINTER(PagedKV), _p, _i64, _p, _p, _i64, _i64, _p, _p],
    "cs_slide_scatter": [ctypes.POINTER(PagedKV), _p, _p, _i64, _p, _p, _i64, _i64, _p, _p],
    "cs_slide_relocate": [ctypes.POINTER(PagedKV), _p, _p, _i64, _p, _p],
    "cs_slide_pack_pages": [ctypes.POINTER(PagedKV), _p, _i64, _p, _p, _p],
    "cs_slide_unpack_pages": [ctypes.POINTER(PagedKV), _p, _i64, _p, _p, _p],
    "cs_slide_scatter_batch": [ctypes.POINTER(PagedKV), ctypes.POINTER(ScatterItem), _i32, _p],
    "cs_wca_initialize_batch": [ctypes.POINTER(InitializeItem), _i32, _i64, _i64, _i32, _f64,
                                _i32, _p],
    "cs_wca_update_batch": [ctypes.POINTER(UpdateItem), _i32, _i64, _i64, _i32, _i32, _f64,
                            _i32, ctypes.POINTER(PagedKV), _p],
    "cs_wca_commit_batch": [ctypes.POINTER(CommitItem), _i32, _f64, _i32, _p],
    "cs_wca_deviation": [_p, _i64, _i64, _p, _p, _i64, _i64, _i64, _i64, _i64, _i32, _f64,
                         _i32, _p, _p, _p, _p],
    "cs_wca_cosine": [_p, _i64, _i64, _p, _i64, _i64, _p, _i64, _i64, _i64, _i32, _f64, _p,
                      _p, _p],
    "cs_wca_row_sums": [_p, _i64, _i64, _p, _p, _i64, _i64, _i64, _i64, _i64, _i32, _i64, _p,
                        _p, _p, _p, _p],
    "cs_wca_weights": [_p, _p, _i64, _f64, _i32, _p, _p, _p, _p, _p, _p],
    "cs_wca_select_topk": [_p, _p, _i64, _i64, _p, _p, _p, _p, _p],
    "cs_wca_active_rows": [_p, _p, _i64, _i64, _p, _p, _p, _p, _p],
    "cs_wca_initialize": [_p, _i64, _i64, _p, _i64, _i64, _i64, _i64, _i64, _i32, _p, _f64,
                          _i32, _p, _p, _p, _p, _p, _p, _p, _p],
    "cs_wca_update": [_p, _p, _i64, _i64, _p, _p, _i64, _i64, _p, _i64, _i64, _i64, _i32, _p,
                      _p, _i32, _f64, _i32, _p, _p, _p, _p, _p, ctypes.POINTER(PagedKV), _p,
                      _p, _p],
    "cs_wca_commit": [_p, _i64, _p, _p, _f64, _i32, _i64, _i64, _p, _p, _p, _p, _p, _p, _p,
                      _p, _p, _p],
    "cs_qkv_gather_lora": [ctypes.POINTER(QKVParams), _p],
    "cs_cope_attn": [ctypes.POINTER(AttnParams), _p],
    "cs_cope_attn_prefill": [ctypes.POINTER(AttnParams), _p],
    "cs_cope_attn_prefill_batch": [ctypes.POINTER(AttnParams), _i32, _p],
    "cs_cope_attn_decode_workspace": [ctypes.POINTER(AttnParams)],
    "cs_cope_attn_decode": [ctypes.POINTER(AttnParams), _p, _p],
    "cs_cope_attn_decode_noalloc": [ctypes.POINTER(AttnParams), _p],
    "cs_cope_attn_decode_batch_workspace": [ctypes.POINTER(AttnParams), _i32],
    "cs_cope_attn_decode_batch": [ctypes.POINTER(AttnParams), _i32, _p, _p],
    "cs_cope_positions": [_p, _i64, _i64, _p, _i64, _i64, _i32, _i64, _i64, _i32, _i32, _p,
                          _i64, _i64, _p, _p],
    "cs_cope_bias": [_p, _i64, _i64, _p, _i64, _i64, _i32, _i32, _p, _i64, _i64, _i32, _i64,
                     _i64, _i32, _p, _i64, _i64, _p, _p],
    "cs_cope_chunk_offsets": [_p, _i64, _i64, _i32, _i32, _i32, _p, _p, _p, _p, _i64, _i64,
                              _i32, _p, _p, _p, _i32, _p, _i64, _i64, _i64, _i32, _i32, _i32,
                              _p, _i64, _i64, _i32, _p, _p],
    "cs_cope_validate_path": [_p, _i64, _i64, _p, _p, _p, _i64, _i64, _i32, _i64, _i64, _f64,
                              _i32, _p, _p],
    "cs_build_info": [],
    "cs_abi_version": [],
}
_RESTYPES = {"cs_build_info": ctypes.c_char_p, "cs_abi_version": _i32,
             "cs_cope_attn_decode_workspace": _i64,
             "cs_cope_attn_decode_batch_workspace": _i64}

EXPORTED = tuple(_SIGNATURES)

_lib = None
_lock = threading.Lock()


def load() -> ctypes.CDLL:
    """Load the CUDA library once; raise RuntimeError when it is unavailable."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"{LIB_PATH.name} is not built; run `python -m cacheslide_b200.build`"
                )
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, args in _SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes = args
                fn.restype = _RESTYPES.get(name, ctypes.c_int)
            _lib = lib
    return _lib


def check(rc: int, name: str) -> None:
    if rc == CS_OK:
        return
    if rc == CS_ERR_INVALID:
        raise ValueError(f"{name}: invalid arguments for the CUDA kernel")
    if rc == CS_ERR_UNSUPPORTED:
        raise ValueError(f"{name}: shape/dtype combination is not supported on device")
    raise RuntimeError(f"{name}: CUDA launch failed (status {rc})")


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_of(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(*tensors: torch.Tensor) -> torch.device:
    device = None
    for t in tensors:
        if t is None:
            continue
        if not isinstance(t, torch.Tensor) or t.device.type != "cuda":
            raise ValueError(
                "cacheslide_b200 operators run on CUDA tensors only (no CPU fallback)"
            )
        if device is None:
            device = t.device
        elif t.device != device:
            raise ValueError("all tensors must be on the same CUDA device")
    if device is None:
        raise ValueError("cacheslide_b200 operators need at least one CUDA tensor")
    return device


class Status:
    """A device int32 status word per call; read after the stream drains."""

    def __init__(self, device: torch.device):
        self.word = torch.zeros(1, dtype=torch.int32, device=device)

    @property
    def ptr(self) -> int:
        return self.word.data_ptr()

    def read(self) -> int:
        return int(self.word.item())


def paged_view(
    cache: torch.Tensor,
    side_k: torch.Tensor | None = None,
    side_v: torch.Tensor | None = None,
) -> PagedKV:
    """Describe a [blocks, kv_heads, block_size, 2*D] view (any strides)."""
    if cache.ndim != 4 or cache.shape[-1] % 2:
        raise ValueError("cache must be [blocks, kv_heads, block_size, 2*D]")
    if cache.dtype not in DTYPES:
        raise ValueError("cache dtype must be float16/bfloat16/float32/float64")
    kv = PagedKV()
    kv.cache = cache.data_ptr()
    kv.num_blocks, kv.kv_heads, kv.block_size = cache.shape[0], cache.shape[1], cache.shape[2]
    kv.head_dim = cache.shape[3] // 2
    kv.stride_block, kv.stride_head, kv.stride_offset, kv.stride_elem = cache.stride()
    kv.dtype = DTYPES[cache.dtype]
    if side_k is not None and side_v is not None:
        if side_k.stride() != side_v.stride() or side_k.shape != side_v.shape:
            raise ValueError("sidecar K and V must share shape and strides")
        kv.side_k, kv.side_v = side_k.data_ptr(), side_v.data_ptr()
        kv.side_capacity = side_k.shape[0]
        kv.side_stride_row, kv.side_stride_head, kv.side_stride_elem = side_k.stride()
    return kv
