"""ctypes binding of the C ABI declared in include/flash_attn_b200.h.

PyTorch supplies device memory and the current CUDA stream; every kernel runs
inside ``_lib/libflash_attn_b200.so``. There is no fallback: if the library is
missing or a CUDA device is absent, calls raise ``RuntimeError``.
"""

import ctypes
import os
import threading

import torch

_LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_lib", "libflash_attn_b200.so")

FA_OK, FA_ERR_INVALID, FA_ERR_UNSUPPORTED, FA_ERR_CUDA = 0, 1, 2, 3
_DTYPES = {
    torch.float16: 1, torch.bfloat16: 2, torch.float32: 3, torch.float8_e4m3fn: 4,
    torch.int32: 5, torch.int64: 6, torch.bool: 7, torch.uint8: 8,
}


class Tensor(ctypes.Structure):
    _fields_ = [
        ("ptr", ctypes.c_void_p),
        ("dtype", ctypes.c_int32),
        ("ndim", ctypes.c_int32),
        ("shape", ctypes.c_int64 * 4),
        ("stride", ctypes.c_int64 * 4),
    ]


_TENSOR_FIELDS = (
    "q k v out lse cu_seqlens_q cu_seqlens_k seqused_k block_table leftpad_k "
    "causal_per_seq alibi_slopes s_aux q_descale k_descale v_descale mask_aux0 "
    "mask_aux1 workspace"
).split()


class AttentionArgs(ctypes.Structure):
    _fields_ = [(name, Tensor) for name in _TENSOR_FIELDS] + [
        ("batch", ctypes.c_int32),
        ("max_seqlen_q", ctypes.c_int32),
        ("max_seqlen_k", ctypes.c_int32),
        ("softmax_scale", ctypes.c_float),
        ("softcap", ctypes.c_float),
        ("causal", ctypes.c_int32),
        ("window_left", ctypes.c_int32),
        ("window_right", ctypes.c_int32),
        ("mask_kind", ctypes.c_int32),
        ("mask_window", ctypes.c_int32),
        ("mask_clamp", ctypes.c_int32),
        ("num_splits", ctypes.c_int32),
        ("deterministic", ctypes.c_int32),
        ("cp_tot_seqused_k", Tensor),
        ("cp_world_size", ctypes.c_int32),
        ("cp_rank", ctypes.c_int32),
    ]


_P = ctypes.POINTER
# (name, argtypes) of every exported entry point; tests check the header too.
_RESTYPES = {"fa_last_error": ctypes.c_char_p, "fa_build_id": ctypes.c_char_p,
             "fa_kernel_launches": ctypes.c_uint64}

SIGNATURES = {
    "fa_abi_version": [],
    "fa_last_error": [],
    "fa_build_id": [],
    "fa_pipeline_timeouts": [ctypes.c_int],
    "fa_kernel_launches": [],
    "fa_attention_workspace_size": [_P(AttentionArgs), _P(ctypes.c_size_t)],
    "fa_attention_fwd": [_P(AttentionArgs), ctypes.c_void_p],
    "fa_decode_fwd_noalloc": [_P(AttentionArgs), ctypes.c_void_p],
    "fa_store_kvcache": [_P(Tensor)] * 7 + [ctypes.c_void_p],
    "fa_append_kvcache": [_P(Tensor)] * 9 + [ctypes.c_void_p],
    "fa_rotary": [_P(Tensor)] * 5 + [ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p],
    "fa_rotary_append_kvcache": [_P(Tensor)] * 13 + [ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p],
    "fa_merge_attn_states": [_P(Tensor)] * 6 + [ctypes.c_void_p],
    "fa_merge_partials": [_P(Tensor)] * 4 + [ctypes.c_void_p],
}

FA_MAX_PEERS = 8


class PeerBuffers(ctypes.Structure):
    _fields_ = [("slots", ctypes.c_void_p * FA_MAX_PEERS), ("flags", ctypes.c_void_p * FA_MAX_PEERS)]


SIGNATURES.update({
    "fa_shard_push": [_P(Tensor), _P(PeerBuffers), ctypes.c_int32, ctypes.c_int32, ctypes.c_uint32, ctypes.c_void_p],
    "fa_shard_wait": [_P(PeerBuffers), ctypes.c_int32, ctypes.c_int32, ctypes.c_uint32, ctypes.c_void_p],
})

_lock = threading.Lock()
_lib = None


def library():
    """Load the CUDA library once; raise if it is missing."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(_LIB_PATH):
                    raise RuntimeError(
                        f"flash_attn_b200 CUDA library not built ({_LIB_PATH}); "
                        "run `python flash-attn-mps_b200/build.py`")
                lib = ctypes.CDLL(_LIB_PATH)
                for name, argtypes in SIGNATURES.items():
                    fn = getattr(lib, name)
                    fn.argtypes = argtypes
                    fn.restype = _RESTYPES.get(name, ctypes.c_int)
                _lib = lib
    return _lib


def build_id():
    """Hash of the sources the loaded library was built from (build.py source_hash)."""
    return library().fa_build_id().decode()


def kernel_launches():
    """Kernel launches the library has issued so far (graph replays not counted)."""
    return int(library().fa_kernel_launches())


def tensor(t, dtype_override=None):
    """Describe a torch tensor (or None = absent) as an fa_tensor."""
    d = Tensor()
    if t is None:
        return d
    if t.dim() > 4:
        raise ValueError("tensors passed to the CUDA library have at most 4 dimensions")
    ptr = t.data_ptr()
    d.ptr = ptr if ptr else 16  # empty tensors: non-null, never dereferenced
    d.dtype = dtype_override if dtype_override is not None else _DTYPES.get(t.dtype, 0)
    d.ndim = t.dim()
    for i, (n, s) in enumerate(zip(t.shape, t.stride())):
        d.shape[i] = n
        d.stride[i] = s
    return d


def check(rc):
    if rc == FA_OK:
        return
    message = library().fa_last_error().decode()
    if rc == FA_ERR_INVALID:
        raise ValueError(message)
    if rc == FA_ERR_UNSUPPORTED:
        raise NotImplementedError(message)
    raise RuntimeError(message)


def stream_of(device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def ref(x):
    return ctypes.byref(x)
