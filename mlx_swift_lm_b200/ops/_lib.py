"""ctypes binding of ``libb200kernels.so`` (the sm_100a kernel library).

Every CUDA op in :mod:`mlx_swift_lm_b200.ops` goes through this module. The
library is required whenever a CUDA tensor reaches an op: there is no silent
eager fallback on a GPU box. If the shared object is missing, the first CUDA
op raises :class:`KernelLibraryMissing` with the build command.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

import torch

_PKG = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
# B200LM_CHECKED=1: the bounds-checked build of the same kernels
CHECKED = os.environ.get("B200LM_CHECKED", "0") == "1"
LIB_PATH = os.path.join(_PKG, "_lib", "libb200kernels_checked.so" if CHECKED else "libb200kernels.so")

_lock = threading.Lock()
_lib = None

vp = C.c_void_p
i32 = C.c_int
i64 = C.c_int64
f32 = C.c_float
u64 = C.c_uint64
sz = C.c_size_t

# name -> (restype, argtypes)
_SIGS = {
    "b200_gemm_bf16": (i32, [vp, i32, i32, i32, vp, i32, i32, vp, i32, vp, i32, vp, i32, i32, i32, vp]),
    "b200_gemm_qkv_rope": (i32, [vp, i32, i32, i32, vp, i32, i32, vp, vp, vp, vp, vp, vp, f32, vp, vp, vp, i32, vp, vp,
                                 i32, i32, i64, i32, i32, vp]),
    "b200_gemm_num_splits": (i32, [i32, i32, i32, i32]),
    "b200_gemm_q": (i32, [vp, i32, i32, i32, vp, i32, i32, i32, vp, i32, vp, i32, vp, i32, i32, i32, vp]),
    "b200_gemm_q_num_splits": (i32, [i32, i32, i32]),
    "b200_gemm_set_ktrace": (None, [vp]),
    "b200_add_rmsnorm": (i32, [vp, vp, vp, vp, i32, i32, i32, i32, i32, f32, i32, vp]),
    "b200_qk_norm_rope_kv": (i32, [vp, i32, i32, vp, vp, vp, i32, i32, vp, vp, f32, vp, vp, vp, i32, vp, vp,
                                   i32, i32, i32, i64, vp, vp, vp]),
    "b200_embedding": (i32, [vp, vp, vp, i32, i32, i64, f32, vp]),
    "b200_silu_mul": (i32, [vp, vp, i32, i32, i32, i32, vp]),
    "b200_paged_decode": (i32, [vp, vp, vp, i32, vp, vp, vp, i32, vp, vp, vp, vp, vp, i32, i32, i32, i32, i32,
                                i32, f32, f32, i64, vp]),
    "b200_paged_decode_part_tokens": (i32, []),
    "b200_add_layernorm": (i32, [vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, f32, vp]),
    "b200_paged_prefill_mma": (i32, [vp, vp, vp, vp, i32, vp, vp, vp, i32, vp, vp, i32, i32, i32, i32, f32, f32,
                                     i64, vp]),
    "b200_paged_prefill_simt": (i32, [vp, vp, vp, vp, i32, vp, vp, vp, i32, vp, vp, i32, i32, i32, i32, f32, f32,
                                      i64, vp]),
    "b200_prefill_simt_q_tile": (i32, [i32]),
    "b200_logits_process": (i32, [vp, i64, i32, i32, vp, vp, vp, i32, vp, vp, i32, vp, vp, vp, i32, vp, vp, vp,
                                  i32, vp, vp]),
    "b200_sample": (i32, [vp, i64, i32, i32, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp]),
    "b200_argmax": (i32, [vp, i64, i32, i32, vp, vp, vp, vp]),
    "b200_argmax_conf": (i32, [vp, i64, i32, i32, vp, vp, vp, vp, i32, vp]),
    "b200_logprobs": (i32, [vp, i64, i32, i32, vp, i32, vp, vp, vp, vp]),
    "b200_philox_u32": (C.c_uint32, [u64, u64, C.c_uint32]),
    "b200_gather_tokens": (i32, [vp, vp, vp, vp, i32, vp]),
    "b200_paged_decode_mma_part": (i32, [vp, vp, vp, vp, i32, vp, vp, vp, i32, i32, i32, i32, i32, i32, f32, f32,
                                         i64, vp]),
    "b200_paged_decode_mma": (i32, [vp, vp, vp, vp, i32, vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, i32, f32, f32,
                                    i64, vp]),
    "b200_paged_decode_merge": (i32, [vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, vp]),
    "b200_paged_decode_wide_part": (i32, [vp, vp, vp, i32, vp, vp, vp, i32, vp, vp, vp, i32, i32, i32, i32, i32,
                                          i32, f32, f32, i64, vp]),
    "b200_lora_shrink": (i32, [vp, i32, vp, i32, i32, vp, i32, vp, i32, vp]),
    "b200_lora_expand": (i32, [vp, i32, vp, i32, i32, vp, vp, vp, i32, i32, vp]),
    "b200_lora_expand_glu": (i32, [vp, i32, vp, i32, i32, vp, i32, vp, vp, vp, i32, i32, i32, vp]),
    "b200_mtp_accept": (i32, [vp, vp, vp, i32, vp, i32, i32, vp, i32, vp, vp, i32, vp]),
    "b200_e2m1_pairs": (i32, [vp, vp]),
    "b200_set_pdl": (None, [i32]),
    "b200_get_pdl": (i32, []),
}

# status accessors exported per translation unit
_STATUS_TAGS = ["gemm", "norm", "attn_decode", "attn_prefill_simt", "sampling", "misc", "attn_decode_mma",
                "attn_prefill_mma", "attn_wide", "lora", "mtp"]


class KernelLibraryMissing(RuntimeError):
    pass


class KernelError(RuntimeError):
    pass


def _load():
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise KernelLibraryMissing(
                f"{LIB_PATH} is missing: build it with `python -m mlx_swift_lm_b200._build` "
                "(CUDA tensors are only served by the sm_100a kernel library)")
        lib = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(lib, name, None)
            if fn is None:
                continue
            fn.restype = res
            fn.argtypes = args
        for tag in _STATUS_TAGS + _EXTRA_STATUS_TAGS:
            fn = getattr(lib, "b200_status_" + tag, None)
            if fn is not None:
                fn.restype = i32
                fn.argtypes = [C.POINTER(C.c_uint), i32]
        _lib = lib
        return lib


_EXTRA_STATUS_TAGS: list[str] = []


def register_signatures(sigs: dict, status_tags=()):
    """Add signatures for kernels defined in other modules (called at import)."""
    _SIGS.update(sigs)
    _EXTRA_STATUS_TAGS.extend(status_tags)
    if _lib is not None:
        for name, (res, args) in sigs.items():
            fn = getattr(_lib, name, None)
            if fn is not None:
                fn.restype = res
                fn.argtypes = args
        for tag in status_tags:
            fn = getattr(_lib, "b200_status_" + tag, None)
            if fn is not None:
                fn.restype = i32
                fn.argtypes = [C.POINTER(C.c_uint), i32]


def lib():
    return _lib if _lib is not None else _load()


def available() -> bool:
    return os.path.exists(LIB_PATH)


def ptr(t: torch.Tensor | None):
    return None if t is None else t.data_ptr()


def stream_ptr(device=None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def check(rc: int, what: str):
    if rc != 0:
        raise KernelError(f"{what} failed with code {rc}")


def read_status(clear: bool = True) -> dict:
    """Device status words of every kernel unit (nonzero = a bounded wait
    expired or a bounds check failed). Synchronizes the device."""
    L = lib()
    out = {}
    for tag in _STATUS_TAGS + _EXTRA_STATUS_TAGS:
        fn = getattr(L, "b200_status_" + tag, None)
        if fn is None:
            continue
        v = C.c_uint(0)
        fn(C.byref(v), 1 if clear else 0)
        out[tag] = v.value
    return out


def timeline_start(device, cap: int = 1 << 16):
    """Install a device timeline buffer in every kernel unit: each kernel's
    block 0 records {globaltimer ns, launch signature} after its pdl_wait()
    (see b200_common.cuh). Returns the (buf, head) tensors for
    :func:`timeline_read`; :func:`timeline_stop` turns recording off."""
    L = lib()
    buf = torch.zeros(cap, 2, dtype=torch.int64, device=device)
    head = torch.zeros(1, dtype=torch.int32, device=device)
    for tag in _STATUS_TAGS + _EXTRA_STATUS_TAGS:
        fn = getattr(L, "b200_timeline_" + tag, None)
        if fn is not None:
            fn.restype = i32
            fn.argtypes = [vp, vp, C.c_uint]
            check(fn(buf.data_ptr(), head.data_ptr(), cap), f"timeline {tag}")
    return buf, head


def timeline_stop():
    L = lib()
    for tag in _STATUS_TAGS + _EXTRA_STATUS_TAGS:
        fn = getattr(L, "b200_timeline_" + tag, None)
        if fn is not None:
            fn.restype = i32
            fn.argtypes = [vp, vp, C.c_uint]
            fn(None, None, 0)


def timeline_read(tl) -> list:
    """Recorded marks in time order: (ns, (grid x, grid y, grid z, block x)) for
    kernel marks, (ns, tag) for tagged points inside kernels."""
    buf, head = tl
    torch.cuda.synchronize(buf.device)
    n = min(int(head.item()), buf.shape[0])
    rows = buf[:n].cpu().tolist()
    out = []
    for t, sig in rows:
        sig &= (1 << 63) - 1
        if sig >> 62:  # tagged point inside a kernel: the tag
            out.append((t, sig & ((1 << 62) - 1)))
            continue
        out.append((t, ((sig >> 31) & 0xFFFFF, (sig >> 19) & 0xFFF, (sig >> 11) & 0xFF, sig & 0x7FF)))
    out.sort(key=lambda m: m[0])
    return out


# Count of kernel launches issued through this binding (for bench accounting).
launch_counter = [0]


def count(n: int = 1):
    launch_counter[0] += n


register_signatures({"b200_gemm_set_trace": (None, [vp])})
