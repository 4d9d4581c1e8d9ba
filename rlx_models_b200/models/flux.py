"""FLUX.1 DiT on the sm_100a kernels, plus the rectified-flow sampler.

Layout. Both streams live in one "stream-major" row space: the B * Lt text
rows first, then the B * Li image rows. Per-stream GEMMs of the double blocks
work on contiguous row ranges; the single blocks and the joint attention see
all rows. Joint attention runs non-causally over 16-row pages: batch b's
sequence is its text pages followed by its image pages (a block table), and
the query/output rows go through the same table, so no concatenation or
split copy is ever made.

One wide activation buffer Y [rows, 3H + M + H] holds per block
    [0, 3H)        qkv (GEMM output)            -> QK-norm / RoPE kernel
    [3H, 3H + M)   MLP hidden (GELU in the GEMM epilogue)
    [3H + M, ...)  attention output
so the single block's linear2 input concat(attn, gelu(mlp)) is the slice
Y[:, 3H:] once linear2's columns are stored in [mlp | attn] order, and its
linear1 writes qkv and the GELU'd MLP hidden with one GEMM.

Sequence parallelism (Ulysses): with ``sp_size`` ranks each holds a
contiguous block of R / sp rows of the stream-major row space (weights are
replicated) and runs every GEMM, norm and modulation on its rows only (row
offsets map local rows to their batch and joint position). Around each joint
attention, q/k/v are written head-group-major and exchanged with one NCCL
all-to-all each, so every rank attends over all rows for heads / sp heads;
a second all-to-all returns the output rows. The final layer's image rows are
all-gathered so every rank holds the full velocity.

Fused epilogues carry the adaLN residual algebra: ``x += gate[b] * (y W^T + bias)``
(gated residual) and GELU-tanh; LayerNorm + modulate is one kernel. All
modulation vectors of a step come from a single GEMM over the concatenated
modulation weights. The forward is CUDA-graph captured per (B, Lt, Li).

Reference: rlx-flux1 src/transformer.rs:58-500, src/embed.rs, src/sampler.rs,
src/pipeline.rs:215-600 (which hard-codes batch 1; batching is native here).
"""
from __future__ import annotations

import math

import torch
import torch.distributed as dist
import torch.nn.functional as F

from .. import ops
from ..config import FluxConfig
from ..ops._ext import ext
from .flux_common import (deinterleave_perm, euler, pack, position_ids, rope_tables, schedule,
                          timestep_embedding, unpack)


class FluxDiT:
    def __init__(self, cfg: FluxConfig, weights, device="cuda", sp_rank: int = 0, sp_size: int = 1, sp_group=None):
        assert cfg.head_dim == 128, "the DiT QK-norm/RoPE kernel is written for head_dim 128"
        self.cfg = cfg
        self.sp_rank, self.sp_size, self.sp_group = sp_rank, sp_size, sp_group
        self.device = torch.device(device)
        H, M = cfg.hidden_size, cfg.mlp_hidden
        dev, bf = self.device, torch.bfloat16

        def g(name):
            t = weights[name] if not hasattr(weights, "take") else weights.take(name)
            return t.to(dev, bf).contiguous()

        perm = deinterleave_perm(cfg.head_dim).to(dev)
        # q/k rows of a fused qkv weight: de-interleave within each head
        qk_rows = torch.arange(2 * H, device=dev).view(2 * cfg.num_heads, cfg.head_dim)[:, perm].reshape(-1)
        row_order = torch.cat([qk_rows, torch.arange(2 * H, 3 * H, device=dev)])

        def qkv_w(name, extra_rows=0):
            w = g(name + ".weight")
            b = g(name + ".bias") if (name + ".bias") in weights else None
            order = torch.cat([row_order, torch.arange(3 * H, 3 * H + extra_rows, device=dev)])
            return w[order].contiguous(), (b[order].contiguous() if b is not None else None)

        def scales(prefix):
            return torch.stack([g(prefix + "query_norm.scale")[perm], g(prefix + "key_norm.scale")[perm]]).contiguous()

        self.w = {}
        for n in ("img_in", "txt_in", "time_in.in_layer", "time_in.out_layer", "vector_in.in_layer",
                  "vector_in.out_layer", "final_layer.linear") + (
                ("guidance_in.in_layer", "guidance_in.out_layer") if cfg.guidance_embed else ()):
            self.w[n] = (g(n + ".weight"), g(n + ".bias"))
        mod_w, mod_b, self.mod_off = [], [], {}
        off = 0

        def add_mod(key, name, n):
            nonlocal off
            mod_w.append(g(name + ".weight"))
            mod_b.append(g(name + ".bias"))
            self.mod_off[key] = off
            off += n * H

        self.double = []
        for i in range(cfg.depth):
            blk = {}
            for s in ("txt", "img"):
                p = f"double_blocks.{i}.{s}"
                add_mod((i, s), p + "_mod.lin", 6)
                blk[s] = dict(qkv=qkv_w(p + "_attn.qkv"), proj=(g(p + "_attn.proj.weight"), g(p + "_attn.proj.bias")),
                              mlp0=(g(p + "_mlp.0.weight"), g(p + "_mlp.0.bias")),
                              mlp2=(g(p + "_mlp.2.weight"), g(p + "_mlp.2.bias")),
                              scales=scales(p + "_attn.norm."))
            self.double.append(blk)
        self.single = []
        for i in range(cfg.depth_single_blocks):
            p = f"single_blocks.{i}"
            add_mod(("single", i), p + ".modulation.lin", 3)
            w1, b1 = qkv_w(p + ".linear1", extra_rows=M)
            w2 = g(p + ".linear2.weight")
            w2 = torch.cat([w2[:, H:], w2[:, :H]], 1).contiguous()  # inputs ordered [mlp | attn]
            self.single.append(dict(l1=(w1, b1), l2=(w2, g(p + ".linear2.bias")), scales=scales(p + ".norm.")))
        add_mod("final", "final_layer.adaLN_modulation.1", 2)
        self.mod_w = torch.cat(mod_w).contiguous()
        self.mod_b = torch.cat(mod_b).contiguous()
        self.n_mod = off
        self._bufs = None
        self._graph = None

    # -- buffers -----------------------------------------------------------------
    def _prepare(self, B: int, Lt: int, Li: int, h: int, w: int):
        key = (B, Lt, Li, h, w)
        if self._bufs is not None and self._bufs["key"] == key:
            return self._bufs
        c, dev, sp = self.cfg, self.device, self.sp_size
        assert Lt % 16 == 0 and Li % 16 == 0, "text and image lengths must be multiples of 16"
        H, M = c.hidden_size, c.mlp_hidden
        R = B * (Lt + Li)
        Lj = Lt + Li
        assert R % (16 * sp) == 0 and c.num_heads % sp == 0, "rows / heads must split evenly over the SP ranks"
        Rl = R // sp
        row0 = self.sp_rank * Rl
        T = B * Lt
        t_hi = min(max(T - row0, 0), Rl)  # local rows [0, t_hi) are text, [t_hi, Rl) image
        bt = torch.empty(B, Lj // 16, dtype=torch.int32)
        for b in range(B):
            bt[b, :Lt // 16] = torch.arange(Lt // 16) + b * Lt // 16
            bt[b, Lt // 16:] = torch.arange(Li // 16) + (B * Lt + b * Li) // 16
        ids = position_ids(Lt, h, w)
        cos, sin = rope_tables(ids, c.axes_dim, c.theta)
        z = lambda *s, dt=torch.bfloat16: torch.zeros(*s, dtype=dt, device=dev)
        hpg = c.num_heads // sp
        S = dict(
            key=key, B=B, Lt=Lt, Li=Li, R=R, Rl=Rl, row0=row0, T=T, t_hi=t_hi, hpg=hpg,
            img=z(B * Li, c.in_channels), txt=z(B * Lt, c.context_in_dim), y=z(B, c.vec_in_dim),
            temb=z(B, 256), gemb=z(B, 256), X=z(Rl, H), Xm=z(Rl, H), Y=z(Rl, 4 * H + M),
            mods=z(B, self.n_mod), vel=z(B * Li, c.out_channels),
            btab=bt.to(dev), ctx=torch.full((B,), Lj, dtype=torch.int32, device=dev),
            cu=(torch.arange(B + 1, dtype=torch.int32) * Lj).to(dev),
            cos=cos.to(dev).contiguous(), sin=sin.to(dev).contiguous())
        if sp == 1:
            S.update(Q=z(R, c.num_heads, 128), K=z(R // 16, c.num_heads, 16, 128), V=z(R // 16, c.num_heads, 16, 128))
        else:
            # head-group-major per-rank q/k/v [sp][Rl][hpg][128] -> all-to-all -> [R][hpg][128]
            S.update(Qg=z(sp, Rl, hpg, 128), Kg=z(sp, Rl, hpg, 128), Vg=z(sp, Rl, hpg, 128),
                     Qa=z(R, hpg, 128), Ka=z(R, hpg, 128), Va=z(R, hpg, 128), Oa=z(R, hpg, 128),
                     Ob=z(sp, Rl, hpg * 128), vel_all=z(R, c.out_channels), vel_loc=z(Rl, c.out_channels))
        self._bufs = S
        self._graph = None
        return S

    # -- one velocity evaluation (reads the static input buffers) -----------------
    def _forward_static(self):
        c, S = self.cfg, self._bufs
        B, Lt, Li, Rl, row0, T, t_hi = S["B"], S["Lt"], S["Li"], S["Rl"], S["row0"], S["T"], S["t_hi"]
        H, M = c.hidden_size, c.mlp_hidden
        X, Xm, Y, mods = S["X"], S["Xm"], S["Y"], S["mods"]
        sp = self.sp_size

        def lin(x, wb, **kw):
            return ops.linear(x, wb[0], bias=wb[1], **kw)

        def mlp_embed(name, x):
            h = lin(x, self.w[name + ".in_layer"])
            return lin(F.silu(h), self.w[name + ".out_layer"])

        vec = mlp_embed("time_in", S["temb"])
        if c.guidance_embed:
            vec = vec + mlp_embed("guidance_in", S["gemb"])
        vec = vec + mlp_embed("vector_in", S["y"])
        lin(F.silu(vec), (self.mod_w, self.mod_b), out=mods)
        # local rows: text rows [0, t_hi) = global text rows row0.., image rows [t_hi, Rl)
        i0 = row0 + t_hi - T  # first global image row held here
        if t_hi > 0:
            lin(S["txt"][row0:row0 + t_hi], self.w["txt_in"], out=X[:t_hi])
        if t_hi < Rl:
            lin(S["img"][i0:i0 + Rl - t_hi], self.w["img_in"], out=X[t_hi:])
        # per-stream local ranges: (r0, r1, stream length, global stream-row offset of r0)
        rows = {"txt": (0, t_hi, Lt, row0), "img": (t_hi, Rl, Li, i0)}
        attn_out = Y[:, 3 * H + M:]

        def attention(scales_txt, scales_img):
            ops._count(1)
            if sp == 1:
                ext().dit_qk_rope(Y[:, :3 * H], c.num_heads, scales_txt, scales_img, S["cos"], S["sin"], T, Lt, Li,
                                  c.eps, S["Q"], S["K"], S["V"])
                ops.prefill_attention(S["Q"], S["K"], S["V"], S["btab"], S["ctx"], S["cu"], Lt + Li,
                                      scale=1.0 / math.sqrt(128), causal=False, q_paged=True, out=attn_out)
                return
            # Ulysses: rows -> heads all-to-all, joint attention over all rows for hpg heads, back
            ext().dit_qk_rope(Y[:, :3 * H], c.num_heads, scales_txt, scales_img, S["cos"], S["sin"], T, Lt, Li,
                              c.eps, S["Qg"], S["Kg"], S["Vg"], row_off=row0, kv_groups=sp)
            for src, dst in (("Qg", "Qa"), ("Kg", "Ka"), ("Vg", "Va")):
                dist.all_to_all_single(S[dst], S[src], group=self.sp_group)
            ops.prefill_attention(S["Qa"], S["Ka"], S["Va"], S["btab"], S["ctx"], S["cu"], Lt + Li,
                                  scale=1.0 / math.sqrt(128), causal=False, q_paged=True, out=S["Oa"])
            dist.all_to_all_single(S["Ob"], S["Oa"], group=self.sp_group)
            attn_out.copy_(S["Ob"].transpose(0, 1).reshape(Rl, H))

        def ln_mod(r0, r1, off, split, ra, rb, row_off):
            if r1 > r0:
                ext().ln_modulate(X[r0:r1], Xm[r0:r1], mods, off, off + H, c.eps, split, ra, rb, row_off)
                ops._count(1)

        for i, blk in enumerate(self.double):
            for st in ("txt", "img"):
                r0, r1, L, goff = rows[st]
                if r1 > r0:
                    o = self.mod_off[(i, st)]
                    ln_mod(r0, r1, o, 0, 1, L, goff)
                    lin(Xm[r0:r1], blk[st]["qkv"], out=Y[r0:r1, :3 * H])
            attention(blk["txt"]["scales"], blk["img"]["scales"])
            for st in ("txt", "img"):
                r0, r1, L, goff = rows[st]
                if r1 <= r0:
                    continue
                o = self.mod_off[(i, st)]
                lin(attn_out[r0:r1], blk[st]["proj"], out=X[r0:r1], residual=X[r0:r1],
                    gate=mods[:, o + 2 * H:o + 3 * H], gate_rows=(0, 1, L, goff))
                ln_mod(r0, r1, o + 3 * H, 0, 1, L, goff)
                lin(Xm[r0:r1], blk[st]["mlp0"], out=Y[r0:r1, 3 * H:3 * H + M], gelu_from=0)
                lin(Y[r0:r1, 3 * H:3 * H + M], blk[st]["mlp2"], out=X[r0:r1], residual=X[r0:r1],
                    gate=mods[:, o + 5 * H:o + 6 * H], gate_rows=(0, 1, L, goff))
        for i, blk in enumerate(self.single):
            o = self.mod_off[("single", i)]
            ln_mod(0, Rl, o, T, Lt, Li, row0)
            lin(Xm, blk["l1"], out=Y[:, :3 * H + M], gelu_from=3 * H)
            attention(blk["scales"], blk["scales"])
            lin(Y[:, 3 * H:], blk["l2"], out=X, residual=X, gate=mods[:, o + 2 * H:o + 3 * H],
                gate_rows=(T, Lt, Li, row0))
        o = self.mod_off["final"]
        if sp == 1:
            ln_mod(T, Rl, o, 0, 1, Li, 0)
            lin(Xm[T:], self.w["final_layer.linear"], out=S["vel"])
            return S["vel"]
        # every local row through the final layer (text rows are discarded), then gather the image rows
        ln_mod(0, Rl, o, T, Lt, Li, row0)
        lin(Xm, self.w["final_layer.linear"], out=S["vel_loc"])
        dist.all_gather_into_tensor(S["vel_all"], S["vel_loc"], group=self.sp_group)
        S["vel"].copy_(S["vel_all"][T:])
        return S["vel"]

    # -- public ------------------------------------------------------------------
    def forward(self, img: torch.Tensor, txt: torch.Tensor, timesteps: torch.Tensor, y: torch.Tensor,
                guidance: torch.Tensor | None = None, h: int | None = None, w: int | None = None,
                graph: bool = True) -> torch.Tensor:
        """img [B, Li, in], txt [B, Lt, ctx], timesteps/guidance [B], y [B, vec];
        (h, w) the packed image grid (h * w = Li). Returns the velocity [B, Li, out] (bf16)."""
        B, Li, _ = img.shape
        Lt = txt.shape[1]
        if h is None:
            h = w = int(round(math.sqrt(Li)))
        S = self._prepare(B, Lt, Li, h, w)
        S["img"].copy_(img.reshape(B * Li, -1), non_blocking=True)
        S["txt"].copy_(txt.reshape(B * Lt, -1), non_blocking=True)
        S["y"].copy_(y, non_blocking=True)
        S["temb"].copy_(timestep_embedding(timesteps.float().cpu()), non_blocking=True)
        if self.cfg.guidance_embed:
            gv = guidance if guidance is not None else torch.full((B,), 3.5)
            S["gemb"].copy_(timestep_embedding(gv.float().cpu()), non_blocking=True)
        if not graph:
            return self._forward_static().view(B, Li, -1)
        if self._graph is None:
            s = torch.cuda.Stream(self.device)
            s.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(s):
                self._forward_static()  # warm-up (lazy allocations, attribute setup)
            torch.cuda.current_stream(self.device).wait_stream(s)
            g = torch.cuda.CUDAGraph()
            n0 = ops.launch_count()
            with torch.cuda.graph(g):
                self._forward_static()
            self._graph_launches = ops.launch_count() - n0
            ops._count(-self._graph_launches)  # capture does not execute; replays are counted
            self._graph = g
        self._graph.replay()
        ops._count(self._graph_launches)
        return S["vel"].view(B, Li, -1)


def generate_latents(model: FluxDiT, txt: torch.Tensor, pooled: torch.Tensor, *, height: int = 1024,
                     width: int = 1024, steps: int = 28, guidance: float = 3.5, seed: int = 0,
                     noise: torch.Tensor | None = None) -> torch.Tensor:
    """Text embeddings [B, Lt, ctx] + pooled [B, vec] -> denoised latents [B, 16, H/8, W/8]
    by Euler integration of the rectified-flow velocity over the shifted schedule."""
    B = txt.shape[0]
    c = model.cfg
    lh, lw = 2 * math.ceil(height / 16), 2 * math.ceil(width / 16)
    ch = c.in_channels // 4
    if noise is None:
        gen = torch.Generator().manual_seed(seed)
        noise = torch.randn(B, ch, lh, lw, generator=gen)
    x = pack(noise).to(model.device, torch.float32)
    Li = x.shape[1]
    ts = schedule(steps, Li, shift=c.guidance_embed)
    gvec = torch.full((B,), float(guidance))

    def velocity(xc, t, i):
        return model.forward(xc.to(torch.bfloat16), txt, torch.full((B,), t), pooled, gvec, lh // 2, lw // 2).float()

    x = euler(x, ts, velocity)
    return unpack(x, ch, lh, lw)
