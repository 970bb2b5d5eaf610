"""Host-side mirror of edge_maskgit's backend interface over libmgcuda.so.

``CudaRuntime`` mirrors ``mg::OpenCLRuntime`` (include/mg-opencl.hpp:23-58) for the MaskGIT
transformer graph: construct once per device, call ``forward`` (the ``TransformerFwd``
callback of include/mg-generate.hpp:15) once per decode step, optionally profile per op type.
The kernel-level functions (``quantize_act``, ``QWeight.qgemm``, ``layernorm_affine``,
``flash_attn``, ``embed``, ``gemm_f32``) take CUDA torch tensors and call the C ABI directly;
torch is only used for device memory and streams.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from ._lib import MgcError, check, lib

__all__ = ["CudaRuntime", "VqganDecoder", "QWeight", "MgcError", "pack_q8_0", "pack_q4_k", "dequant", "tp_unique_id",
           "quantize_act", "gemm_f32", "layernorm_affine", "flash_attn", "embed", "device_error",
           "F32", "Q8_0", "Q4_K"]

F32, Q8_0, Q4_K = 0, 8, 12


def _ptr(a) -> C.c_void_p:
    if a is None:
        return None
    if isinstance(a, np.ndarray):
        return C.c_void_p(a.ctypes.data)
    return C.c_void_p(a.data_ptr())


def _stream():
    import torch
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def _cuda_f32(t, name):
    import torch
    if not (isinstance(t, torch.Tensor) and t.is_cuda and t.dtype == torch.float32 and t.is_contiguous()):
        raise MgcError(f"{name} must be a contiguous float32 CUDA tensor")
    return t


# ----------------------------------------------------------------- block formats (host)
def pack_q8_0(w: np.ndarray) -> np.ndarray:
    """[N][K] f32 -> GGUF Q8_0 bytes (tools/convert_to_gguf.py:109-124)."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    N, K = w.shape
    out = np.empty(N * K // 32 * 34, np.uint8)
    check(lib.mgc_pack_q8_0(_ptr(w), N, K, _ptr(out)), "pack_q8_0")
    return out


def pack_q4_k(w: np.ndarray) -> np.ndarray:
    """[N][K] f32 -> GGUF Q4_K bytes (tools/convert_to_gguf.py:68-106)."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    N, K = w.shape
    out = np.empty(N * K // 256 * 144, np.uint8)
    check(lib.mgc_pack_q4_k(_ptr(w), N, K, _ptr(out)), "pack_q4_k")
    return out


def dequant(wtype: int, blocks: np.ndarray, N: int, K: int) -> np.ndarray:
    """GGUF blocks -> [N][K] f32 (DEQ_Q8 / deq_q4k_elem of mg-opencl.cpp)."""
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    out = np.empty((N, K), np.float32)
    check(lib.mgc_dequant(wtype, _ptr(blocks), N, K, _ptr(out)), "dequant")
    return out


def device_error() -> int:
    """Read and clear the device error word set by kernels whose bounded waits expired."""
    return int(lib.mgc_device_error())


# ----------------------------------------------------------------- kernel-level ops
def quantize_act(x, want_sum: bool = False):
    """k_quantize_q8: x [M][K] -> (qx int8 [M][K], dx f32 [M][K/32], sumx int32 | None)."""
    import torch
    _cuda_f32(x, "x")
    M, K = x.shape
    qx = torch.empty((M, K), dtype=torch.int8, device=x.device)
    dx = torch.empty((M, K // 32), dtype=torch.float32, device=x.device)
    sx = torch.empty((M, K // 32), dtype=torch.int32, device=x.device) if want_sum else None
    check(lib.mgc_quantize_act(_ptr(x), M, K, _ptr(qx), _ptr(dx), _ptr(sx), _stream()), "quantize_act")
    return qx, dx, sx


class QWeight:
    """A Q8_0 / Q4_K (or F32) [N][K] weight resident on the current CUDA device."""

    def __init__(self, wtype: int, data: np.ndarray, N: int, K: int):
        data = np.ascontiguousarray(data)
        h = C.c_void_p()
        check(lib.mgc_qweight_create(wtype, _ptr(data), N, K, C.byref(h)), "qweight_create")
        self._h, self.wtype, self.N, self.K = h, wtype, N, K

    def qgemm(self, x, bias=None, act: int = 0, resid=None, out=None):
        """y = act(W.x + bias) + resid, the MulMat(q) dispatch of mg-opencl.cpp:1381-1399."""
        import torch
        _cuda_f32(x, "x")
        M = x.shape[0]
        if x.shape[1] != self.K:
            raise MgcError(f"x has {x.shape[1]} columns, weight K = {self.K}")
        y = out if out is not None else torch.empty((M, self.N), dtype=torch.float32, device=x.device)
        check(lib.mgc_qgemm(self._h, _ptr(x), M, _ptr(bias), act, _ptr(resid), _ptr(y), _stream()), "qgemm")
        return y

    def close(self):
        if self._h:
            lib.mgc_qweight_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def gemm_f32(w, x, bias=None, act: int = 0, resid=None):
    import torch
    N, K = w.shape
    M = x.shape[0]
    y = torch.empty((M, N), dtype=torch.float32, device=x.device)
    check(lib.mgc_gemm_f32(_ptr(w), _ptr(x), M, N, K, _ptr(bias), act, _ptr(resid), _ptr(y), _stream()),
          "gemm_f32")
    return y


def layernorm_affine(x, gamma, beta, eps: float = 1e-12):
    import torch
    rows, D = x.shape
    y = torch.empty_like(x)
    check(lib.mgc_layernorm_affine(_ptr(x), _ptr(gamma), _ptr(beta), rows, D, eps, _ptr(y), _stream()),
          "layernorm_affine")
    return y


def flash_attn(qkv, B: int, S: int, H: int, Dh: int, scale: float):
    import torch
    y = torch.empty((B * S, H * Dh), dtype=torch.float32, device=qkv.device)
    check(lib.mgc_flash_attn(_ptr(qkv), B, S, H, Dh, scale, _ptr(y), _stream()), "flash_attn")
    return y


def embed(tok, pos, tokens, B: int, S: int):
    import torch
    V, E = tok.shape
    y = torch.empty((B * S, E), dtype=torch.float32, device=tok.device)
    check(lib.mgc_embed(_ptr(tok), V, _ptr(pos), E, _ptr(tokens), B, S, _ptr(y), _stream()), "embed")
    return y


# ----------------------------------------------------------------- runtime
@dataclass
class HParams:
    n_layer: int
    n_head: int
    n_embd: int
    n_ffn: int
    head_dim: int
    vocab_size: int
    n_tokens: int
    mask_token_id: int
    codebook_size: int
    wtype: int


@dataclass
class OpProfile:   # include/mg-opencl.hpp:17-21
    op: str
    count: int
    ms: float


def tp_unique_id() -> bytes:
    """128-byte NCCL id for a tensor-parallel runtime group (make it on one rank, share it)."""
    buf = (C.c_uint8 * 128)()
    check(lib.mgc_tp_unique_id(buf), "tp_unique_id")
    return bytes(buf)


class CudaRuntime:
    """mg::OpenCLRuntime's counterpart for the MaskGIT transformer on one B200.

    tp=(rank, world, id) makes this process rank `rank` of a column-split tensor-parallel group
    of `world` GPUs (id from tp_unique_id() on one rank); all ranks then run every forward with
    the same inputs and each gets the full logits."""

    def __init__(self, gguf_path: str, max_rows: int = 257, device: int = 0, tp=None):
        h = C.c_void_p()
        if tp is None:
            check(lib.mgc_runtime_create(str(gguf_path).encode(), max_rows, device, C.byref(h)), "runtime_create")
        else:
            rank, world, uid = tp
            idb = (C.c_uint8 * 128).from_buffer_copy(uid)
            check(lib.mgc_runtime_create_tp(str(gguf_path).encode(), max_rows, device, rank, world, idb, C.byref(h)),
                  "runtime_create_tp")
        self._h = h
        hp = np.zeros(10, np.int32)
        check(lib.mgc_runtime_hparams(h, _ptr(hp)))
        self.hparams = HParams(*[int(v) for v in hp])
        self.max_rows = max_rows

    # --- OpenCLRuntime API
    def device_name(self) -> str:
        return lib.mgc_runtime_device_name(self._h).decode()

    def invalidate(self, _tensor=None) -> None:
        """Token inputs are uploaded on every forward, so nothing is cached to drop."""

    def profile_enable(self, on: bool) -> None:
        check(lib.mgc_profile_enable(self._h, int(on)))

    def profile_reset(self) -> None:
        check(lib.mgc_profile_reset(self._h))

    def kernel_count(self) -> int:
        """Kernels enqueued by the last forward."""
        return int(lib.mgc_runtime_kernel_count(self._h))

    def time_op(self, op: str, B: int, S: int, iters: int = 50) -> tuple[float, int]:
        """(ms per replay, kernels per replay) of a CUDA graph holding only the forward's
        launches of op class `op` (a profile_report name), replayed back to back."""
        ms, n = C.c_float(), C.c_int()
        check(lib.mgc_runtime_time_op(self._h, op.encode(), B, S, iters, C.byref(ms), C.byref(n)), "time_op")
        return float(ms.value), int(n.value)

    def profile_report(self) -> list[OpProfile]:
        buf = C.create_string_buffer(1 << 14)
        check(lib.mgc_profile_report(self._h, buf, len(buf)))
        rows = []
        for line in buf.value.decode().splitlines():
            name, n, ms = line.rsplit(" ", 2)
            rows.append(OpProfile(name, int(n), float(ms)))
        return rows

    # --- TransformerFwd
    def forward(self, tokens: np.ndarray, B: int | None = None, out: np.ndarray | None = None) -> np.ndarray:
        """tokens [B][S] int32 (host) -> logits [B*S][vocab] f32 (host).  `out` (optional) is a
        caller-owned C-contiguous float32 [B*S][vocab] buffer reused across calls, as the
        reference decode loop reuses its logits vector (mg-generate.cpp:55)."""
        tokens = np.ascontiguousarray(tokens, dtype=np.int32)
        if tokens.ndim == 1:
            tokens = tokens[None]
        B, S = tokens.shape
        shape = (B * S, self.hparams.vocab_size)
        if out is None:
            out = np.empty(shape, np.float32)
        elif out.shape != shape or out.dtype != np.float32 or not out.flags.c_contiguous:
            raise ValueError(f"out must be a C-contiguous float32 array of shape {shape}")
        check(lib.mgc_transformer_forward(self._h, _ptr(tokens), B, S, _ptr(out)), "forward")
        return out

    def forward_dev(self, tokens_dev, logits_dev, B: int, S: int) -> None:
        """Device-resident forward on the runtime's stream (graph replay); not synchronised."""
        check(lib.mgc_transformer_forward_dev(self._h, _ptr(tokens_dev), B, S, _ptr(logits_dev)), "forward_dev")

    def forward_dump(self, tokens: np.ndarray):
        """Forward that also returns the 51 named verification tensors (MG_DUMP_NAMED)."""
        tokens = np.ascontiguousarray(tokens, dtype=np.int32)
        if tokens.ndim == 1:
            tokens = tokens[None]
        B, S = tokens.shape
        hp = self.hparams
        R = B * S
        logits = np.empty((R, hp.vocab_size), np.float32)
        dump = np.empty(R * (hp.n_embd * (2 * hp.n_layer + 2) + hp.vocab_size), np.float32)
        check(lib.mgc_transformer_forward_dump(self._h, _ptr(tokens), B, S, _ptr(logits), _ptr(dump)),
              "forward_dump")
        return logits, split_named(dump, R, hp.n_layer, hp.n_embd, hp.vocab_size)

    def sync(self) -> None:
        check(lib.mgc_runtime_sync(self._h), "sync")

    @property
    def stream_handle(self) -> int:
        return int(lib.mgc_runtime_stream(self._h) or 0)

    def generate(self, class_ids, seeds, steps: int = 8, temperature: float = 4.5) -> np.ndarray:
        """generate() (src/mg-generate.cpp:53-123) for len(class_ids) images -> tokens [B][S]."""
        cls = np.ascontiguousarray(class_ids, dtype=np.int32)
        sd = np.ascontiguousarray(seeds, dtype=np.uint64)
        B = cls.shape[0]
        out = np.empty((B, self.hparams.n_tokens + 1), np.int32)
        check(lib.mgc_generate(self._h, B, _ptr(cls), _ptr(sd), steps, temperature, _ptr(out)), "generate")
        return out

    def generate_images(self, vq: "VqganDecoder", class_ids, seeds, steps: int = 8,
                        temperature: float = 4.5) -> tuple[np.ndarray, np.ndarray]:
        """mg::generate end to end (mgc_generate_images): uint8 images [B][R][R][3] and the
        final token sequences [B][n_tokens + 1]."""
        cls = np.ascontiguousarray(class_ids, np.int32)
        sd = np.ascontiguousarray(seeds, np.uint64)
        B, R = len(cls), vq.resolution
        rgb = np.empty((B, R, R, 3), np.uint8)
        tok = np.empty((B, self.hparams.n_tokens + 1), np.int32)
        check(lib.mgc_generate_images(self._h, vq._h, B, _ptr(cls), _ptr(sd), steps, temperature, _ptr(rgb),
                                      _ptr(tok)), "generate_images")
        return rgb, tok

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib.mgc_runtime_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class VqganDecoder:
    """The VQGAN decoder (build_vqgan_decoder, include/mg-vqgan.hpp:12) on one B200.

    ``decode(grid)`` is the reference's VqganFwd callback (include/mg-generate.hpp:17): a token
    grid [n_tokens] (or a batch [n][n_tokens]) -> HWC float image [R][R][3] (or [n][R][R][3])."""

    def __init__(self, gguf_path: str, max_images: int = 1, device: int = 0):
        h = C.c_void_p()
        check(lib.mgc_vqgan_create(str(gguf_path).encode(), max_images, device, C.byref(h)), "vqgan_create")
        self._h = h
        info = [C.c_int(), C.c_int(), C.c_int()]
        check(lib.mgc_vqgan_info(h, *[C.byref(v) for v in info]))
        self.n_tokens, self.resolution, self.codebook_size = (v.value for v in info)
        self.max_images = max_images

    def decode(self, grid, out: np.ndarray | None = None) -> np.ndarray:
        g = np.ascontiguousarray(grid, np.int32)
        single = g.ndim == 1
        g = g.reshape(-1, self.n_tokens)
        R = self.resolution
        if out is None:
            out = np.empty((g.shape[0], R, R, 3), np.float32)
        check(lib.mgc_vqgan_decode(self._h, _ptr(g), g.shape[0], _ptr(out)), "vqgan_decode")
        return out[0] if single else out

    def decode_rgb8(self, grid) -> np.ndarray:
        """The bytes of the reference's mg::Image (clamp, * 255 + 0.5, truncate): uint8 HWC."""
        g = np.ascontiguousarray(grid, np.int32)
        single = g.ndim == 1
        g = g.reshape(-1, self.n_tokens)
        R = self.resolution
        out = np.empty((g.shape[0], R, R, 3), np.uint8)
        check(lib.mgc_vqgan_decode_rgb8(self._h, _ptr(g), g.shape[0], _ptr(out)), "vqgan_decode_rgb8")
        return out[0] if single else out

    def decode_device(self, grid_dev, out_dev, n_images: int) -> None:
        """Device tensors (int32 [n][n_tokens], float32 [n][R][R][3]) on the current torch stream."""
        check(lib.mgc_vqgan_decode_device(self._h, _ptr(grid_dev), n_images, _ptr(out_dev), _stream()),
              "vqgan_decode_device")

    def launches(self) -> int:
        return lib.mgc_vqgan_launches(self._h)

    def time_op(self, op: str, n_images: int = 1, iters: int = 20) -> tuple[float, int]:
        """(ms per replay, launches) of a graph of one kernel class of the decode."""
        ms, n = C.c_float(), C.c_int()
        check(lib.mgc_vqgan_time_op(self._h, op.encode(), n_images, iters, C.byref(ms), C.byref(n)), "vqgan_time_op")
        return ms.value, n.value

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib.mgc_vqgan_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def named_tensor_names(n_layer: int) -> list[str]:
    """The 51 verification names of mg-transformer.cpp:48,91,98,105,109 in dump order."""
    names = ["embd_post_norm"]
    for i in range(n_layer):
        names += [f"blk.{i}.attn_post", f"blk.{i}.ffn_post"]
    return names + ["output_norm", "output_logits"]


def split_named(dump: np.ndarray, R: int, n_layer: int, E: int, V: int) -> dict:
    out, off = {}, 0
    for name in named_tensor_names(n_layer):
        w = V if name == "output_logits" else E
        out[name] = dump[off:off + R * w].reshape(R, w)
        off += R * w
    return out
