"""Building blocks shared by the convolutional audio codecs (DAC, EnCodec):
weight-norm folding, channels-last convolutions as GEMMs, and the LSTM.

Layout: activations are channels-last [B, T, C] (bf16 on the GPU, fp32 on
CPU). A convolution is ``act_im2col`` (the preceding activation, the padding
-- zero or reflected -- and the dilation folded into the GEMM operand) followed
by one tcgen05 linear whose epilogue adds the bias and, for residual blocks,
the skip input; a transposed convolution is one linear into fp32 taps followed
by ``convt_fold`` (overlap-add, bias, crop). An LSTM layer projects every
time step's input in one GEMM, then per step accumulates h W_hh^T into that
step's gate row (``linear_acc``) and applies the cell (``lstm_cell``). On CPU
the same code runs on the fp32 torch statements of the kernels
(``ops/reference.py``), which the tests compare against transformers.

Reference: crates/rlx-dac/src/layers.rs:7-60 (weight-normalised convs) and
crates/rlx-encodec (SEANet convs, LSTM) in the reference.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from ..ops import reference as R


def fold_weight_norm(named: dict) -> dict:
    """fp32 tensors with weight normalisation folded, w = g * v / ||v|| (the
    norm over every axis but the one ``g`` keeps: the first, or e.g. the kernel
    axis of wav2vec2's positional conv), from either serialisation:
    ``X.weight_g`` / ``X.weight_v`` or ``X.parametrizations.weight.original0`` / ``original1``."""
    raw = {}
    for k, t in named.items():
        n = k.replace("parametrizations.weight.original0", "weight_g").replace(
            "parametrizations.weight.original1", "weight_v")
        raw[n] = t.float()
    out = {}
    for n, t in raw.items():
        if n.endswith(".weight_g"):
            base = n[:-len(".weight_g")]
            v = raw[base + ".weight_v"]
            keep = [d for d in range(v.dim()) if t.dim() == v.dim() and t.shape[d] != 1] or [0]
            axes = [d for d in range(v.dim()) if d not in keep]
            norm = v.pow(2).sum(dim=axes, keepdim=True).sqrt() if axes else v.abs()
            out[base + ".weight"] = t * v / norm
        elif not n.endswith(".weight_v"):
            out[n] = t
    return out


class GemmConv:
    """One convolution prepared as a GEMM operand: ``w`` [N_pad, round_up(k * C, 8)]
    (column j * C + c = tap j of input channel c; output rows padded to a multiple
    of 8). Transposed convs: ``w`` [k * O, C], row j * O + o = tap j of output o."""

    def __init__(self, W: torch.Tensor, b: torch.Tensor | None, transposed: bool, dt, dev):
        if transposed:
            C, O, k = W.shape
            w = W.permute(2, 1, 0).reshape(k * O, C)
        else:
            O, C, k = W.shape
            w = W.permute(0, 2, 1).reshape(O, k * C)
            w = F.pad(w, (0, (-w.shape[1]) % 8))
            w = F.pad(w, (0, 0, 0, (-O) % 8))
        self.k, self.C, self.O, self.transposed = k, C, O, transposed
        self.w = w.to(dev, dt).contiguous()
        bp = None if b is None else (b if transposed else F.pad(b, (0, (-O) % 8)))
        self.b = None if bp is None else bp.to(dev, dt).contiguous()   # GEMM epilogue bias (bf16 on the GPU)
        self.b32 = None if b is None else b.to(dev, torch.float32).contiguous()


class ConvRunner:
    """Runs ``GemmConv``s on the package's kernels (``fast``, CUDA bf16) or on
    their fp32 torch statements (CPU)."""

    def __init__(self, device):
        self.device = torch.device(device)
        self.fast = self.device.type == "cuda"
        self.dtype = torch.bfloat16 if self.fast else torch.float32
        if self.fast:
            from .. import ops
            self.ops = ops

    def conv(self, x: torch.Tensor, L: GemmConv, *, act: str | None = None, alpha=None, stride: int = 1,
             pad: int = 0, pad_right: int | None = None, dil: int = 1, reflect: bool = False,
             residual: torch.Tensor | None = None) -> torch.Tensor:
        """x [B, T, C] -> [B, T_out, O]: act, pad (left ``pad``, right
        ``pad_right``, zero or reflected), conv, + bias (+ residual [B, T_out, O])."""
        B = x.shape[0]
        fuse_res = residual is not None and L.w.shape[0] == L.O
        if self.fast:
            cols = self.ops.act_im2col(x, L.k, stride=stride, pad=pad, pad_right=pad_right, dil=dil, act=act,
                                       alpha=alpha, reflect=reflect)
            res = residual.reshape(-1, L.O) if fuse_res else None
            y = self.ops.linear(cols, L.w, bias=L.b, residual=res)
        else:
            cols = R.act_im2col(x, L.k, stride, pad, pad_right, dil, act, alpha, reflect)
            y = cols @ L.w.t()
            if L.b is not None:
                y = y + L.b
            if fuse_res:
                y = y + residual.reshape(-1, L.O)
        if y.shape[1] != L.O:
            y = y[:, :L.O]
        y = y.reshape(B, -1, L.O)
        if residual is not None and not fuse_res:
            y = y + residual
        return y

    def conv_t(self, x: torch.Tensor, L: GemmConv, *, stride: int, pad: int, pad_right: int | None = None,
               act: str | None = None, alpha=None) -> torch.Tensor:
        """Transposed conv of x [B, T, C] (after ``act``), cropped by ``pad`` /
        ``pad_right`` samples -> [B, (T - 1) * stride + k - pad - pad_right, O]."""
        B, T, _ = x.shape
        if self.fast:
            cols = self.ops.act_im2col(x, 1, act=act, alpha=alpha) if act is not None else x.reshape(B * T, -1)
            Y = self.ops.linear(cols.contiguous(), L.w, out_dtype=torch.float32)
            return self.ops.convt_fold(Y.view(B, T, -1), L.b32, L.O, stride=stride, pad=pad, pad_right=pad_right)
        xa = R.act_im2col(x, 1, act=act, alpha=alpha)[:, :x.shape[2]] if act is not None else x.reshape(B * T, -1)
        Y = xa.float() @ L.w.t()
        return R.convt_fold(Y.view(B, T, -1), L.b32, L.O, stride, pad, pad_right)

    def lstm(self, x: torch.Tensor, layers: list) -> torch.Tensor:
        """Stacked unidirectional LSTM over x [B, T, H] from zero state;
        ``layers`` = [(W_ih [4H, H], W_hh [4H, H], b_ih + b_hh fp32 [4H])]. -> [B, T, H]."""
        B, T, H = x.shape
        inp = x.transpose(0, 1).contiguous()                # time-major rows t * B + b
        for wih, whh, b in layers:
            if self.fast:
                G = self.ops.linear(inp.view(T * B, H), wih, out_dtype=torch.float32)
                G.add_(b)
                G = G.view(T, B, 4 * H)
                h = torch.zeros(B, H, dtype=torch.bfloat16, device=self.device)
                c = torch.zeros(B, H, dtype=torch.float32, device=self.device)
                out = torch.empty(T, B, H, dtype=torch.bfloat16, device=self.device)
                for t in range(T):
                    if t > 0:
                        self.ops.linear_acc(h, whh, acc=G[t])
                    self.ops.lstm_cell(G[t], c, h, out[t])
            else:
                G = (inp.reshape(T * B, H).float() @ wih.t() + b).view(T, B, 4 * H)
                h = torch.zeros(B, H)
                c = torch.zeros(B, H)
                rows = []
                for t in range(T):
                    h, c = R.lstm_cell(G[t] + h @ whh.t(), c)
                    rows.append(h)
                out = torch.stack(rows)
            inp = out
        return inp.transpose(0, 1)
