"""Column-split tensor parallelism for long sequences (the M=4097, batch-4 step forward).

One process per GPU (rank g of G), NCCL all-gathers over NVLink, kernels through the C ABI:

- QKV: whole heads per rank (H/G heads: rows of attn_q/k/v for those heads, fused), so
  attention runs locally with no exchange;
- the head-merged attention output, attn_o, ffn_up and ffn_down outputs are column slices that
  are all-gathered into the full [rows, width] activation the next op needs (attn_o and
  ffn_down add their residual slice in the epilogue; LayerNorm needs whole rows);
- embeddings, LayerNorms and output_proj are replicated; the MLM head is split by vocabulary
  rows and its logits gathered.

Every GEMM output element is computed exactly as on one GPU (same K order, same activation
quantization), so results match the single-GPU runtime up to the attention's key-split choice.
"""
from __future__ import annotations

import numpy as np

from . import runtime as rt
from .gguf import GGUF


def _gather_cols(t, group=None):
    """[R][w] slice per rank -> [R][G*w] (rank-major column blocks) via one all-gather."""
    import torch
    import torch.distributed as dist
    if not dist.is_initialized():
        return t
    G = dist.get_world_size(group)
    R, w = t.shape
    buf = torch.empty((G * R, w), dtype=t.dtype, device=t.device)
    dist.all_gather_into_tensor(buf, t.contiguous(), group=group)
    return buf.view(G, R, w).permute(1, 0, 2).reshape(R, G * w)


class TPForward:
    def __init__(self, gguf_path, rank: int, world: int, group=None):
        import torch
        self.g, self.G, self.group = rank, world, group
        m = GGUF(gguf_path)
        self.L = int(m.hp("n_layer"))
        self.H = int(m.hp("n_head"))
        self.E = int(m.hp("n_embd"))
        self.F = int(m.hp("n_ffn"))
        self.Dh = int(m.hp("head_dim"))
        self.V = int(m.hp("vocab_size"))
        self.eps = float(m.hp("layernorm_eps", 1e-12))
        if self.H % world or self.E % world or self.F % world:
            raise ValueError("heads / widths must divide the world size")
        self.dev = torch.device("cuda", torch.cuda.current_device())
        E, F, G, g = self.E, self.F, world, rank
        Eg, Fg = E // G, F // G

        def f32(name):
            return torch.from_numpy(np.array(m[name].f32())).to(self.dev)

        def qw(names_rows):
            """QWeight from row ranges of several [N][K] tensors of one type, stacked."""
            parts, typ, K = [], None, None
            for name, a, b in names_rows:
                t = m[name]
                typ = t.type if typ is None else typ
                K = t.ne[0]
                parts.append(np.asarray(t.rows(a, b)))
            n = sum(b - a for _, a, b in names_rows)
            data = np.concatenate(parts)
            if typ == 0:
                return rt.QWeight(0, data.view(np.float32).reshape(n, K), n, K)
            return rt.QWeight(typ, data, n, K)

        self.tok = f32("token_embd.weight")
        self.pos = f32("pos_embd.weight")
        self.g0, self.b0 = f32("token_embd_norm.weight"), f32("token_embd_norm.bias")
        self.layers = []
        for i in range(self.L):
            p = f"blk.{i}."
            L = {}
            L["qkv"] = qw([(p + f"attn_{x}.weight", g * Eg, (g + 1) * Eg) for x in "qkv"])
            L["bqkv"] = torch.cat([f32(p + f"attn_{x}.bias")[g * Eg:(g + 1) * Eg] for x in "qkv"]).contiguous()
            L["o"] = qw([(p + "attn_o.weight", g * Eg, (g + 1) * Eg)])
            L["bo"] = f32(p + "attn_o.bias")[g * Eg:(g + 1) * Eg].contiguous()
            L["up"] = qw([(p + "ffn_up.weight", g * Fg, (g + 1) * Fg)])
            L["bup"] = f32(p + "ffn_up.bias")[g * Fg:(g + 1) * Fg].contiguous()
            L["down"] = qw([(p + "ffn_down.weight", g * Eg, (g + 1) * Eg)])
            L["bdown"] = f32(p + "ffn_down.bias")[g * Eg:(g + 1) * Eg].contiguous()
            for nm in ("attn_norm", "ffn_norm"):
                L[nm] = (f32(p + nm + ".weight"), f32(p + nm + ".bias"))
            self.layers.append(L)
        self.proj = qw([("output_proj.weight", 0, E)])
        self.bproj = f32("output_proj.bias")
        self.gout, self.bout = f32("output_norm.weight"), f32("output_norm.bias")
        self.Vg = (self.V + G - 1) // G
        v0, v1 = min(self.V, g * self.Vg), min(self.V, (g + 1) * self.Vg)
        head = torch.zeros((self.Vg, E), device=self.dev)
        head[: v1 - v0] = self.tok[v0:v1]
        self.head = head
        hb = torch.zeros(self.Vg, device=self.dev)
        hb[: v1 - v0] = f32("output.bias")[v0:v1]
        self.hbias = hb

    def forward(self, tokens):
        """tokens [B][S] int32 (host) -> logits [B*S][vocab] f32 (device, every rank)."""
        import torch
        tokens = np.ascontiguousarray(tokens, np.int32)
        B, S = tokens.shape
        E, g, Eg = self.E, self.g, self.E // self.G
        tok = torch.from_numpy(tokens).to(self.dev)
        x = rt.embed(self.tok, self.pos, tok, B, S)
        x = rt.layernorm_affine(x, self.g0, self.b0, self.eps)
        scale = float(1.0 / np.sqrt(np.float32(self.Dh)))
        for L in self.layers:
            qkv = L["qkv"].qgemm(x, bias=L["bqkv"])
            att = rt.flash_attn(qkv, B, S, self.H // self.G, self.Dh, scale)
            att = _gather_cols(att, self.group)
            o = L["o"].qgemm(att, bias=L["bo"], resid=x[:, g * Eg:(g + 1) * Eg].contiguous())
            x = rt.layernorm_affine(_gather_cols(o, self.group), *L["attn_norm"], self.eps)
            ff = L["up"].qgemm(x, bias=L["bup"], act=1)
            ff = _gather_cols(ff, self.group)
            d = L["down"].qgemm(ff, bias=L["bdown"], resid=x[:, g * Eg:(g + 1) * Eg].contiguous())
            x = rt.layernorm_affine(_gather_cols(d, self.group), *L["ffn_norm"], self.eps)
        hd = self.proj.qgemm(x, bias=self.bproj, act=1)
        hd = rt.layernorm_affine(hd, self.gout, self.bout, self.eps)
        lg = rt.gemm_f32(self.head, hd, bias=self.hbias)
        return _gather_cols(lg, self.group)[:, : self.V]
