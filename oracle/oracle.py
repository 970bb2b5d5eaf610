"""ctypes binding of the CPU oracle (oracle/libmgo.so) and of the reference's own CPU path
(oracle/_ref/libmgref.so).  TEST INFRASTRUCTURE ONLY: imported by tests/, by the smoke()
check of __graft_entry__.py and by the CPU-baseline legs of bench.py -- never by the
edge_maskgit_b200 package.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
MGO = HERE / "libmgo.so"
MGREF = HERE / "_ref" / "libmgref.so"

P, I, I64, F = C.c_void_p, C.c_int, C.c_int64, C.c_float
FWD_FN = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p)


def _p(a):
    return None if a is None else C.c_void_p(a.ctypes.data)


def build() -> None:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)


_mgo = None
_ref = None


def mgo():
    global _mgo
    if _mgo is None:
        if not MGO.exists():
            build()
        L = C.CDLL(str(MGO))
        sig = {
            "mgo_f16_to_f32": (F, [C.c_uint16]), "mgo_f32_to_f16": (C.c_uint16, [F]),
            "mgo_pack_q8_0": (None, [P, I64, I64, P]), "mgo_pack_q4_k": (None, [P, I64, I64, P]),
            "mgo_dequant": (None, [I, P, I64, I64, P]),
            "mgo_quantize_act": (None, [P, I64, I64, P, P, P]),
            "mgo_qgemm": (None, [I, P, P, P, P, I64, I64, I64, P, I, P, P, P]),
            "mgo_qgemm_fused": (None, [I, P, P, P, P, I64, I64, I64, P, I, P, P, P]),
            "mgo_gemm_f32": (None, [P, P, I64, I64, I64, P, I, P, P]),
            "mgo_layernorm_affine": (None, [P, P, P, I64, I64, F, P]),
            "mgo_flash_attn": (None, [P, I64, I64, I64, I64, F, P]),
            "mgo_embed": (None, [P, I64, P, I64, P, I64, I64, P]),
            "mgo_model_load": (P, [C.c_char_p]), "mgo_model_free": (None, [P]),
            "mgo_last_error": (C.c_char_p, []), "mgo_model_hparams": (None, [P, P]),
            "mgo_forward": (I, [P, P, I, I, P, P]),
            "mgo_generate": (I, [P, FWD_FN, P, I, P, P, I, F, P]),
        }
        for n, (r, a) in sig.items():
            f = getattr(L, n)
            f.restype, f.argtypes = r, a
        _mgo = L
    return _mgo


def ref_available() -> bool:
    return MGREF.exists()


def mgref():
    global _ref
    if _ref is None:
        L = C.CDLL(str(MGREF))
        L.mgref_last_error.restype = C.c_char_p
        L.mgref_forward.restype = I
        L.mgref_forward.argtypes = [C.c_char_p, P, I, I, P, P, I]
        L.mgref_generate.restype = I
        L.mgref_generate.argtypes = [C.c_char_p, FWD_FN, P, I, C.c_ulonglong, I, F, P]
        L.mgref_vqgan.restype = I
        L.mgref_vqgan.argtypes = [C.c_char_p, P, P]
        _ref = L
    return _ref


# ------------------------------------------------------------------ kernel-level oracle
def pack_q8_0(w):
    w = np.ascontiguousarray(w, np.float32)
    N, K = w.shape
    out = np.empty(N * K // 32 * 34, np.uint8)
    mgo().mgo_pack_q8_0(_p(w), N, K, _p(out))
    return out


def pack_q4_k(w):
    w = np.ascontiguousarray(w, np.float32)
    N, K = w.shape
    out = np.empty(N * K // 256 * 144, np.uint8)
    mgo().mgo_pack_q4_k(_p(w), N, K, _p(out))
    return out


def dequant(wtype, blocks, N, K):
    blocks = np.ascontiguousarray(blocks, np.uint8)
    out = np.empty((N, K), np.float32)
    mgo().mgo_dequant(wtype, _p(blocks), N, K, _p(out))
    return out


def quantize_act(x):
    x = np.ascontiguousarray(x, np.float32)
    M, K = x.shape
    qx = np.empty((M, K), np.int8)
    dx = np.empty((M, K // 32), np.float32)
    sx = np.empty((M, K // 32), np.int32)
    mgo().mgo_quantize_act(_p(x), M, K, _p(qx), _p(dx), _p(sx))
    return qx, dx, sx


def qgemm(wtype, wblocks, x, N, bias=None, act=0, resid=None, want_idot=False, order="reference"):
    """Full quantized linear on f32 x: quantize_act + int8-dot GEMM + epilogue.
    order "reference": Q4_K accumulated as mg-opencl.cpp:572 writes it (difference first);
    "kernel": the CUDA kernel's two fused multiply-adds (Q8_0 is the same either way)."""
    x = np.ascontiguousarray(x, np.float32)
    M, K = x.shape
    qx, dx, sx = quantize_act(x)
    y = np.empty((M, N), np.float32)
    idot = np.empty((M, N, K // 32), np.int32) if want_idot else None
    wblocks = np.ascontiguousarray(wblocks, np.uint8)
    bias = None if bias is None else np.ascontiguousarray(bias, np.float32)
    resid = None if resid is None else np.ascontiguousarray(resid, np.float32)
    fn = mgo().mgo_qgemm if order == "reference" else mgo().mgo_qgemm_fused
    fn(wtype, _p(wblocks), _p(qx), _p(dx), _p(sx), M, N, K, _p(bias), act, _p(resid), _p(y),
                    _p(idot))
    return (y, idot) if want_idot else y


def gemm_f32(w, x, bias=None, act=0, resid=None):
    w = np.ascontiguousarray(w, np.float32)
    x = np.ascontiguousarray(x, np.float32)
    N, K = w.shape
    M = x.shape[0]
    y = np.empty((M, N), np.float32)
    mgo().mgo_gemm_f32(_p(w), _p(x), M, N, K, _p(bias), act, _p(resid), _p(y))
    return y


def layernorm_affine(x, g, b, eps=1e-12):
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    mgo().mgo_layernorm_affine(_p(x), _p(np.ascontiguousarray(g, np.float32)),
                               _p(np.ascontiguousarray(b, np.float32)), x.shape[0], x.shape[1], eps, _p(y))
    return y


def flash_attn(qkv, B, S, H, Dh, scale):
    qkv = np.ascontiguousarray(qkv, np.float32)
    out = np.empty((B * S, H * Dh), np.float32)
    mgo().mgo_flash_attn(_p(qkv), B, S, H, Dh, scale, _p(out))
    return out


def embed(tok, pos, tokens, B, S):
    tok = np.ascontiguousarray(tok, np.float32)
    pos = np.ascontiguousarray(pos, np.float32)
    tokens = np.ascontiguousarray(tokens, np.int32)
    out = np.empty((B * S, tok.shape[1]), np.float32)
    mgo().mgo_embed(_p(tok), tok.shape[0], _p(pos), tok.shape[1], _p(tokens), B, S, _p(out))
    return out


# ------------------------------------------------------------------ model-level oracle
def named_tensor_names(n_layer):
    """The 51 verification names (mg-transformer.cpp:48,91,98,105,109) in dump order."""
    names = ["embd_post_norm"]
    for i in range(n_layer):
        names += [f"blk.{i}.attn_post", f"blk.{i}.ffn_post"]
    return names + ["output_norm", "output_logits"]


def split_named(dump, R, n_layer, E, V):
    out, off = {}, 0
    for name in named_tensor_names(n_layer):
        w = V if name == "output_logits" else E
        out[name] = dump[off:off + R * w].reshape(R, w)
        off += R * w
    return out

class OracleModel:
    def __init__(self, path):
        self._h = mgo().mgo_model_load(str(path).encode())
        if not self._h:
            raise RuntimeError(mgo().mgo_last_error().decode())
        hp = np.zeros(10, np.int32)
        mgo().mgo_model_hparams(self._h, _p(hp))
        (self.n_layer, self.n_head, self.n_embd, self.n_ffn, self.head_dim, self.vocab_size,
         self.n_tokens, self.mask_id, self.codebook, self.wtype) = [int(v) for v in hp]

    def forward(self, tokens, dump=False):
        tokens = np.ascontiguousarray(tokens, np.int32)
        if tokens.ndim == 1:
            tokens = tokens[None]
        B, S = tokens.shape
        R = B * S
        logits = np.empty((R, self.vocab_size), np.float32)
        d = np.empty(R * (self.n_embd * (2 * self.n_layer + 2) + self.vocab_size), np.float32) if dump else None
        if mgo().mgo_forward(self._h, _p(tokens), B, S, _p(logits), _p(d)) != 0:
            raise RuntimeError(mgo().mgo_last_error().decode())
        if not dump:
            return logits
        return logits, split_named(d, R, self.n_layer, self.n_embd, self.vocab_size)

    def generate(self, class_ids, seeds, steps=8, temperature=4.5, fwd=None):
        """Decode loop; fwd(tokens[B][S]) -> logits[B*S][V] defaults to the oracle forward."""
        cls = np.ascontiguousarray(class_ids, np.int32)
        sd = np.ascontiguousarray(seeds, np.uint64)
        B = cls.shape[0]
        out = np.empty((B, self.n_tokens + 1), np.int32)
        cb = _make_cb(fwd, self.vocab_size) if fwd else None
        if cb is None:
            native = FWD_FN(("mgo_forward_cb", mgo()))
            rc = mgo().mgo_generate(self._h, native, self._h, B, _p(cls), _p(sd), steps, temperature, _p(out))
        else:
            rc = mgo().mgo_generate(self._h, cb, None, B, _p(cls), _p(sd), steps, temperature, _p(out))
        if rc != 0:
            raise RuntimeError("oracle generate failed")
        return out

    def __del__(self):
        try:
            mgo().mgo_model_free(self._h)
        except Exception:
            pass


def _make_cb(fwd, vocab):
    def cb(_user, tok_ptr, B, S, logit_ptr):
        try:
            t = np.ctypeslib.as_array(C.cast(tok_ptr, C.POINTER(C.c_int32)), shape=(B, S)).copy()
            out = np.ctypeslib.as_array(C.cast(logit_ptr, C.POINTER(C.c_float)), shape=(B * S * vocab,))
            out[:] = np.asarray(fwd(t), np.float32).reshape(-1)
            return 0
        except Exception:
            return -1
    return FWD_FN(cb)


# ------------------------------------------------------------------ the reference itself
def ref_forward(gguf_f32, tokens, n_embd, n_layer, vocab, dump=False, n_threads=1):
    """The reference's own scalar CPU path (mg-cpu) on an F32 GGUF."""
    tokens = np.ascontiguousarray(tokens, np.int32)
    if tokens.ndim == 1:
        tokens = tokens[None]
    B, S = tokens.shape
    R = B * S
    logits = np.empty((R, vocab), np.float32)
    d = np.empty(R * (n_embd * (2 * n_layer + 2) + vocab), np.float32) if dump else None
    if mgref().mgref_forward(str(gguf_f32).encode(), _p(tokens), B, S, _p(logits), _p(d), n_threads) != 0:
        raise RuntimeError(mgref().mgref_last_error().decode())
    if not dump:
        return logits
    return logits, split_named(d, R, n_layer, n_embd, vocab)


def ref_generate(gguf, fwd, vocab, n_tokens, class_id=207, seed=42, steps=8, temperature=4.5):
    """The reference's own generate() (src/mg-generate.cpp) driving `fwd` -> final grid."""
    grid = np.empty(n_tokens, np.int32)
    cb = _make_cb(fwd, vocab)
    if mgref().mgref_generate(str(gguf).encode(), cb, None, class_id, seed, steps, temperature, _p(grid)) != 0:
        raise RuntimeError(mgref().mgref_last_error().decode())
    return grid


def ref_vqgan(gguf, grid, resolution):
    """The reference's own VQGAN decoder (src/mg-vqgan.cpp on mg-cpu) -> [R][R][3] HWC float."""
    grid = np.ascontiguousarray(grid, np.int32)
    out = np.empty((resolution, resolution, 3), np.float32)
    if mgref().mgref_vqgan(str(gguf).encode(), _p(grid), _p(out)) != 0:
        raise RuntimeError(mgref().mgref_last_error().decode())
    return out


# ------------------------------------------------------------------ VQGAN decoder (numpy)
def read_gguf(path):
    """Minimal GGUF v3 reader (the format of mg-model.cpp:139-201): scalar / string / array
    metadata and F32 tensors as numpy arrays (numpy shape = reversed ne)."""
    import struct
    b = Path(path).read_bytes()
    p = 0

    def take(fmt):
        nonlocal p
        v = struct.unpack_from("<" + fmt, b, p)
        p += struct.calcsize("<" + fmt)
        return v[0]

    def string():
        nonlocal p
        n = take("Q")
        s = b[p:p + n].decode()
        p += n
        return s

    scal = {0: "B", 1: "b", 2: "H", 3: "h", 4: "I", 5: "i", 6: "f", 7: "?", 10: "Q", 11: "q", 12: "d"}

    def value(t):
        if t == 8:
            return string()
        if t == 9:
            sub, n = take("I"), take("Q")
            return [value(sub) for _ in range(n)]
        return take(scal[t])

    assert take("I") == 0x46554747 and take("I") == 3
    nt, nkv = take("Q"), take("Q")
    kv = {}
    for _ in range(nkv):
        k = string()
        kv[k] = value(take("I"))
    infos = []
    for _ in range(nt):
        name = string()
        ne = [take("Q") for _ in range(take("I"))]
        infos.append((name, ne, take("I"), take("Q")))
    align = kv.get("general.alignment", 32)
    data0 = (p + align - 1) // align * align
    tensors = {}
    for name, ne, typ, off in infos:
        if typ == 0:
            n = int(np.prod(ne))
            tensors[name] = np.frombuffer(b, np.float32, n, data0 + off).reshape(tuple(reversed(ne)))
    return kv, tensors


def _gn_affine_silu(x, w, b, groups=32, eps=1e-5):
    """x [C][H][W]; mg-cpu.cpp:124-147 (group stats in double, two passes) + :265-276."""
    C = x.shape[0]
    cpg = C // groups
    out = np.empty_like(x)
    for g in range(groups):
        xs = x[g * cpg:(g + 1) * cpg].astype(np.float64)
        mean = xs.mean()
        var = ((xs - mean) ** 2).mean()
        inv = np.float32(1.0) / np.sqrt(np.float32(var) + np.float32(eps))
        out[g * cpg:(g + 1) * cpg] = (xs - mean).astype(np.float32) * inv
    xn = out * w[:, None, None] + b[:, None, None]
    return (xn / (np.float32(1.0) + np.exp(-xn))).astype(np.float32)


def _conv(x, w, bias=None):
    """x [IC][H][W], w [OC][IC][k][k], stride 1, pad k//2 (mg-cpu.cpp:166-187) via im2col."""
    IC, H, W = x.shape
    OC, _, k, _ = w.shape
    pd = k // 2
    xp = np.pad(x, ((0, 0), (pd, pd), (pd, pd)))
    cols = np.empty((IC, k, k, H, W), np.float32)
    for kh in range(k):
        for kw in range(k):
            cols[:, kh, kw] = xp[:, kh:kh + H, kw:kw + W]
    y = (w.reshape(OC, -1) @ cols.reshape(IC * k * k, H * W)).reshape(OC, H, W)
    if bias is not None:
        y = y + bias[:, None, None]
    return y.astype(np.float32)


def vqgan_decode(gguf, grid):
    """CPU restatement of build_vqgan_decoder (src/mg-vqgan.cpp:67-108) -> [R][R][3] HWC."""
    kv, t = read_gguf(gguf)
    filters = kv["maskgit.vqgan.filters"]
    mult = kv["maskgit.vqgan.channel_multipliers"]
    nrb = kv["maskgit.vqgan.num_res_blocks"]
    n_tok = kv["maskgit.n_tokens"]
    L = 1
    while L * L < n_tok:
        L += 1
    d = "vqgan.decoder."
    cb = t["vqgan.quantizer.codebook.weight"]
    x = cb[np.asarray(grid)].reshape(L, L, -1).transpose(2, 0, 1)     # [C][H][W], token y*L+x

    def gas(name, h):
        return _gn_affine_silu(h, t[name + ".weight"], t[name + ".bias"])

    def resblock(pfx, h, cin, cout):
        res = h
        h = _conv(gas(pfx + "norm0", h), t[pfx + "conv0.weight"])
        h = _conv(gas(pfx + "norm1", h), t[pfx + "conv1.weight"])
        if cin != cout:
            res = _conv(h, t[pfx + "conv_res.weight"])                # applied to the processed h
        return h + res

    curr = filters * mult[-1]
    x = _conv(x, t[d + "conv_in.weight"], t[d + "conv_in.bias"])
    for l in range(nrb):
        x = resblock(f"{d}res_blocks.0.{l}.", x, curr, curr)
    prev = curr
    for bi, i in enumerate(range(len(mult) - 1, -1, -1), start=1):
        curr = filters * mult[i]
        for l in range(nrb):
            x = resblock(f"{d}res_blocks.{bi}.{l}.", x, prev, curr)
            prev = curr
        if i > 0:
            x = x.repeat(2, axis=1).repeat(2, axis=2)                 # nearest, mg-cpu.cpp:190-196
            up = f"{d}res_blocks.{bi}.{nrb + 1}"
            x = _conv(x, t[up + ".weight"], t[up + ".bias"])
    x = gas(d + "norm_out", x)
    x = _conv(x, t[d + "conv_out.weight"], t[d + "conv_out.bias"])
    return np.ascontiguousarray(x.transpose(1, 2, 0))
