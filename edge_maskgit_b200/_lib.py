"""ctypes binding of libmgcuda.so (the C ABI declared in include/mgc.h).

The library is built in-tree by ``edge_maskgit_b200.build``.  There is no fallback: if the
shared object is missing, importing this module raises.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libmgcuda.so"

if not LIB_PATH.exists():
    raise ImportError(f"{LIB_PATH} is missing: run `python -m edge_maskgit_b200.build` "
                      "(the CUDA backend has no CPU fallback)")

lib = C.CDLL(str(LIB_PATH))

P = C.c_void_p
I = C.c_int
I64 = C.c_int64
F = C.c_float

_SIGS = {
    "mgc_last_error": (C.c_char_p, []),
    "mgc_device_error": (I, []),
    "mgc_selftest_wait_timeout": (I, [I, P]),
    "mgc_pack_q8_0": (I, [P, I64, I64, P]),
    "mgc_pack_q4_k": (I, [P, I64, I64, P]),
    "mgc_dequant": (I, [I, P, I64, I64, P]),
    "mgc_quantize_act": (I, [P, I, I, P, P, P, P]),
    "mgc_qweight_create": (I, [I, P, I, I, C.POINTER(P)]),
    "mgc_qweight_destroy": (None, [P]),
    "mgc_qgemm": (I, [P, P, I, P, I, P, P, P]),
    "mgc_qgemm_noalloc": (I, [P, P, I, P, I, P, P, P]),
    "mgc_gemm_f32": (I, [P, P, I, I, I, P, I, P, P, P]),
    "mgc_layernorm_affine": (I, [P, P, P, I, I, F, P, P]),
    "mgc_flash_attn": (I, [P, I, I, I, I, F, P, P]),
    "mgc_embed": (I, [P, I, P, I, P, I, I, P, P]),
    "mgc_runtime_create": (I, [C.c_char_p, I, I, C.POINTER(P)]),
    "mgc_runtime_destroy": (None, [P]),
    "mgc_tp_unique_id": (I, [P]),
    "mgc_runtime_create_tp": (I, [C.c_char_p, I, I, I, I, P, C.POINTER(P)]),
    "mgc_runtime_hparams": (I, [P, P]),
    "mgc_runtime_device_name": (C.c_char_p, [P]),
    "mgc_transformer_forward": (I, [P, P, I, I, P]),
    "mgc_transformer_forward_dev": (I, [P, P, I, I, P]),
    "mgc_transformer_forward_dump": (I, [P, P, I, I, P, P]),
    "mgc_runtime_sync": (I, [P]),
    "mgc_runtime_stream": (P, [P]),
    "mgc_generate": (I, [P, I, P, P, I, F, P]),
    "mgc_runtime_kernel_count": (I, [P]),
    "mgc_runtime_time_op": (I, [P, C.c_char_p, I, I, I, C.POINTER(F), C.POINTER(I)]),
    "mgc_profile_enable": (I, [P, I]),
    "mgc_profile_reset": (I, [P]),
    "mgc_profile_report": (I, [P, C.c_char_p, C.c_size_t]),
    "mgc_vqgan_create": (I, [C.c_char_p, I, I, C.POINTER(P)]),
    "mgc_vqgan_info": (I, [P, P, P, P]),
    "mgc_vqgan_decode": (I, [P, P, I, P]),
    "mgc_vqgan_decode_device": (I, [P, P, I, P, P]),
    "mgc_vqgan_decode_rgb8": (I, [P, P, I, P]),
    "mgc_generate_images": (I, [P, P, I, P, P, I, F, P, P]),
    "mgc_vqgan_launches": (I, [P]),
    "mgc_vqgan_time_op": (I, [P, C.c_char_p, I, I, C.POINTER(F), C.POINTER(I)]),
    "mgc_vqgan_destroy": (None, [P]),
}

for _name, (_res, _args) in _SIGS.items():
    _fn = getattr(lib, _name)
    _fn.restype = _res
    _fn.argtypes = _args

EXPORTED = tuple(_SIGS)


class MgcError(RuntimeError):
    pass


def check(rc: int, what: str = "") -> None:
    if rc != 0:
        msg = lib.mgc_last_error().decode(errors="replace")
        raise MgcError(f"{what}: {msg}" if what else msg)
