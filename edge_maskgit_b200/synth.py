"""Synthetic MaskGIT GGUF models (the stand-in for the reference's real checkpoints).

Writes GGUF v3 in the layout the reference loader reads (mg-model.cpp:139-201) with the
tensor names and shapes of reference/export_weights.py:51-80 and the metadata keys of
tools/convert_to_gguf.py:188-210.  Every tensor is ``0.02 * N(0, 1)`` drawn from one
``numpy.random.default_rng(seed)`` stream in export order.  Linear weights (attn_q/k/v/o,
ffn_up/down, output_proj) are packed Q8_0 ("gq8") or Q4_K ("gq4") by the library's packer,
or kept F32 ("f32"); token_embd / pos_embd / LayerNorm / biases stay F32, as the reference
converter does (convert_to_gguf.py:213-246).

With ``vqgan=VqganSpec(...)`` the file also carries a VQGAN decoder (the ``vqgan.*`` tensors of
export_weights.py and the ``maskgit.vqgan.*`` keys of convert_to_gguf.py:203-208), every conv
weight F32 as the converter keeps them (convert_to_gguf.py:217-247): conv weights
``N(0,1)/sqrt(fan_in)``, conv biases ``0.02*N(0,1)``, GroupNorm weight ``1 + 0.1*N(0,1)`` and bias
``0.1*N(0,1)``, codebook ``N(0,1)``, drawn from the same stream after the transformer tensors.

``dequant_twin`` writes the same model with every packed weight dequantised back to F32 --
the input the reference's scalar CPU executor needs (it reads weights as float only).

The packers are the library's (``runtime.pack_q8_0`` / ``pack_q4_k`` / ``dequant``) unless the
caller passes another implementation of the same three functions (``packers=``), e.g. a CPU
process that must not load the CUDA library.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass
from pathlib import Path

import numpy as np

ALIGN = 32
_LINEAR = ("attn_q.weight", "attn_k.weight", "attn_v.weight", "attn_o.weight",
           "ffn_up.weight", "ffn_down.weight")


@dataclass
class VqganSpec:
    """The decoder of maskgit/nets/vqgan_tokenizer.py as mg-vqgan.cpp builds it."""
    embedding_dim: int = 256
    filters: int = 128
    num_res_blocks: int = 2
    channel_multipliers: tuple = (1, 1, 2, 2, 4)
    group_norm_groups: int = 32


@dataclass
class ModelSpec:
    n_layer: int = 24
    n_embd: int = 768
    n_head: int = 16
    n_ffn: int = 3072
    vocab_size: int = 2025
    n_tokens: int = 256
    codebook: int = 1024
    quant: str = "gq8"        # gq8 | gq4 | f32
    seed: int = 42
    vqgan: VqganSpec | None = None

    @property
    def latent(self) -> int:
        L = 1
        while L * L < self.n_tokens:
            L += 1
        return L

    @property
    def resolution(self) -> int:
        if self.vqgan is None:
            return 256
        return self.latent * 2 ** (len(self.vqgan.channel_multipliers) - 1)

    @property
    def head_dim(self) -> int:
        return self.n_embd // self.n_head


def tensor_list(s: ModelSpec):
    """(name, numpy shape) in export order (export_weights.py:51-80)."""
    E, F, V, P = s.n_embd, s.n_ffn, s.vocab_size, s.n_tokens + 1
    out = [("token_embd.weight", (V, E)), ("pos_embd.weight", (P, E)),
           ("token_embd_norm.weight", (E,)), ("token_embd_norm.bias", (E,))]
    for i in range(s.n_layer):
        p = f"blk.{i}."
        for nm in ("q", "k", "v"):
            out += [(p + f"attn_{nm}.weight", (E, E)), (p + f"attn_{nm}.bias", (E,))]
        out += [(p + "attn_o.weight", (E, E)), (p + "attn_o.bias", (E,)),
                (p + "attn_norm.weight", (E,)), (p + "attn_norm.bias", (E,)),
                (p + "ffn_up.weight", (F, E)), (p + "ffn_up.bias", (F,)),
                (p + "ffn_down.weight", (E, F)), (p + "ffn_down.bias", (E,)),
                (p + "ffn_norm.weight", (E,)), (p + "ffn_norm.bias", (E,))]
    out += [("output_proj.weight", (E, E)), ("output_proj.bias", (E,)),
            ("output_norm.weight", (E,)), ("output_norm.bias", (E,)), ("output.bias", (V,))]
    return out


def vqgan_tensor_list(s: ModelSpec):
    """(name, numpy shape, kind) of the decoder, in the order mg-vqgan.cpp:67-108 uses them.
    kind: conv | bias | gn_w | gn_b | codebook."""
    v = s.vqgan
    out = [("vqgan.quantizer.codebook.weight", (s.codebook, v.embedding_dim), "codebook")]
    d = "vqgan.decoder."
    mult, nrb = list(v.channel_multipliers), v.num_res_blocks

    def conv(name, oc, ic, k, bias):
        out.append((name + ".weight", (oc, ic, k, k), "conv"))
        if bias:
            out.append((name + ".bias", (oc,), "bias"))

    def gn(name, c):
        out.extend([(name + ".weight", (c,), "gn_w"), (name + ".bias", (c,), "gn_b")])

    def resblock(pfx, cin, cout):
        gn(pfx + "norm0", cin)
        conv(pfx + "conv0", cout, cin, 3, False)
        gn(pfx + "norm1", cout)
        conv(pfx + "conv1", cout, cout, 3, False)
        if cin != cout:
            conv(pfx + "conv_res", cout, cout, 1, False)   # applied to the processed h

    curr = v.filters * mult[-1]
    conv(d + "conv_in", curr, v.embedding_dim, 3, True)
    for l in range(nrb):
        resblock(f"{d}res_blocks.0.{l}.", curr, curr)
    prev = curr
    for bi, i in enumerate(range(len(mult) - 1, -1, -1), start=1):
        curr = v.filters * mult[i]
        for l in range(nrb):
            resblock(f"{d}res_blocks.{bi}.{l}.", prev, curr)
            prev = curr
        if i > 0:
            conv(f"{d}res_blocks.{bi}.{nrb + 1}", curr, curr, 3, True)
    gn(d + "norm_out", curr)
    conv(d + "conv_out", 3, curr, 3, True)
    return out


def _vqgan_values(rng, shape, kind):
    z = rng.standard_normal(shape, dtype=np.float32)
    if kind == "conv":
        fan_in = int(np.prod(shape[1:]))
        return (z / np.float32(np.sqrt(fan_in))).astype(np.float32)
    if kind == "bias":
        return (z * np.float32(0.02)).astype(np.float32)
    if kind == "gn_w":
        return (np.float32(1.0) + z * np.float32(0.1)).astype(np.float32)
    if kind == "gn_b":
        return (z * np.float32(0.1)).astype(np.float32)
    return z


def _is_linear(name: str) -> bool:
    return name.endswith(_LINEAR) or name == "output_proj.weight"


class _Buf:
    def __init__(self):
        self.b = bytearray()

    def u32(self, v): self.b += struct.pack("<I", v)
    def i32(self, v): self.b += struct.pack("<i", v)
    def u64(self, v): self.b += struct.pack("<Q", v)
    def f32(self, v): self.b += struct.pack("<f", v)

    def s(self, text: str):
        raw = text.encode()
        self.u64(len(raw))
        self.b += raw


def _metadata(s: ModelSpec, quant_label: str) -> tuple[bytes, int]:
    kv = _Buf()
    n = 0

    def put(key, typ, val):
        nonlocal n
        kv.s(key)
        kv.u32(typ)
        if typ == 9:   # array of i32
            kv.u32(5)
            kv.u64(len(val))
            for x in val:
                kv.i32(int(x))
        else:
            {4: kv.u32, 5: kv.i32, 6: kv.f32, 8: kv.s}[typ](val)
        n += 1

    put("general.architecture", 8, "maskgit")
    put("general.name", 8, f"synthetic maskgit (seed {s.seed})")
    put("general.alignment", 4, ALIGN)
    put("general.file_type", 4, 0)
    put("maskgit.resolution", 4, s.resolution)
    put("maskgit.n_layer", 4, s.n_layer)
    put("maskgit.n_head", 4, s.n_head)
    put("maskgit.n_embd", 4, s.n_embd)
    put("maskgit.n_ffn", 4, s.n_ffn)
    put("maskgit.head_dim", 4, s.head_dim)
    put("maskgit.vocab_size", 4, s.vocab_size)
    put("maskgit.n_tokens", 4, s.n_tokens)
    put("maskgit.n_positions", 4, s.n_tokens + 1)
    put("maskgit.mask_token_id", 5, s.vocab_size - 1)
    put("maskgit.layernorm_eps", 6, 1e-12)
    put("maskgit.vqgan.codebook_size", 4, s.codebook)
    if s.vqgan is not None:
        v = s.vqgan
        put("maskgit.vqgan.embedding_dim", 4, v.embedding_dim)
        put("maskgit.vqgan.filters", 4, v.filters)
        put("maskgit.vqgan.num_res_blocks", 4, v.num_res_blocks)
        put("maskgit.vqgan.group_norm_groups", 4, v.group_norm_groups)
        put("maskgit.vqgan.channel_multipliers", 9, list(v.channel_multipliers))
    put("maskgit.sampling.choice_temperature", 6, 4.5)
    put("maskgit.quant", 8, quant_label)
    return bytes(kv.b), n


def _write(path: Path, s: ModelSpec, quant_label: str, tensors) -> None:
    """tensors: iterable of (name, ne innermost-first, ggml type, bytes)."""
    tensors = list(tensors)
    kv, nkv = _metadata(s, quant_label)
    info = _Buf()
    offs, cur = [], 0
    for name, ne, typ, data in tensors:
        info.s(name)
        info.u32(len(ne))
        for d in ne:
            info.u64(int(d))
        info.u32(typ)
        info.u64(cur)
        offs.append(cur)
        cur = (cur + len(data) + ALIGN - 1) // ALIGN * ALIGN
    head = struct.pack("<IIQQ", 0x46554747, 3, len(tensors), nkv) + kv + bytes(info.b)
    pad = (-len(head)) % ALIGN
    path.parent.mkdir(parents=True, exist_ok=True)
    with open(path, "wb") as f:
        f.write(head + b"\0" * pad)
        pos = 0
        for (name, ne, typ, data), off in zip(tensors, offs):
            if off > pos:
                f.write(b"\0" * (off - pos))
                pos = off
            f.write(data)
            pos += len(data)


def make_model(path, spec: ModelSpec | None = None, dequant_twin=None, packers=None) -> Path:
    """Write a synthetic GGUF (and optionally its dequantised F32 twin).  `packers`: an object
    with pack_q8_0(w), pack_q4_k(w) and dequant(wtype, blocks, N, K) (default: the library's)."""
    s = spec or ModelSpec()
    if packers is None and s.quant != "f32":
        from . import runtime as packers
    Q8_0, Q4_K = 8, 12
    rng = np.random.default_rng(s.seed)
    packed, twin = [], []
    for name, shape in tensor_list(s):
        a = (rng.standard_normal(shape, dtype=np.float32) * np.float32(0.02)).astype(np.float32)
        ne = list(reversed(shape))
        if _is_linear(name) and s.quant in ("gq8", "gq4"):
            N, K = shape
            if s.quant == "gq8":
                blob, typ = packers.pack_q8_0(a), Q8_0
            else:
                blob, typ = packers.pack_q4_k(a), Q4_K
            packed.append((name, ne, typ, blob.tobytes()))
            if dequant_twin is not None:
                twin.append((name, ne, 0, packers.dequant(typ, blob, N, K).tobytes()))
        else:
            packed.append((name, ne, 0, a.tobytes()))
            if dequant_twin is not None:
                twin.append((name, ne, 0, a.tobytes()))
    if s.vqgan is not None:
        for name, shape, kind in vqgan_tensor_list(s):
            a = _vqgan_values(rng, shape, kind)
            ent = (name, list(reversed(shape)), 0, a.tobytes())
            packed.append(ent)
            if dequant_twin is not None:
                twin.append(ent)
    path = Path(path)
    _write(path, s, s.quant, packed)
    if dequant_twin is not None:
        _write(Path(dequant_twin), s, "f32", twin)
    return path


def vqgan_spec(vq: VqganSpec | None = None, n_tokens: int = 256, seed: int = 42) -> ModelSpec:
    """A model whose VQGAN decoder is `vq` (default: the MaskGIT decoder, 256 x 256 output) next
    to a one-layer F32 transformer (the decoder tests do not need the transformer)."""
    return ModelSpec(n_layer=1, n_embd=64, n_head=2, n_ffn=128, n_tokens=n_tokens, quant="f32", seed=seed,
                     vqgan=vq or VqganSpec())


def config1_tokens(spec: ModelSpec | None = None, class_id: int = 207) -> np.ndarray:
    """Step-1 input: class token (class + codebook) then n_tokens mask ids (mg-generate.cpp:58-59)."""
    s = spec or ModelSpec()
    t = np.full(s.n_tokens + 1, s.vocab_size - 1, np.int32)
    t[0] = class_id + s.codebook
    return t
