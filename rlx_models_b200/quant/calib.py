"""Post-training quantisation: formats and calibration algorithms.

Formats (weights W [out, in], quantised along ``in``):
  * MXFP4  - E2M1 codes, one E8M0 power-of-two scale per 32 (gpt-oss layout;
             ``quant.mxfp4``), the format the grouped / dense MXFP4 kernels read;
  * NVFP4  - E2M1 codes, one E4M3 scale per 16 and one fp32 scale per tensor;
  * FP8    - E4M3 with one fp32 scale per output channel.

Algorithms (each returns the dequantised weight it chose plus the packed form):
  * RTN   - round to nearest on the raw weights;
  * AWQ   - activation-aware per-input-channel scaling s = mean|x|^a, grid
            search over a in [0, 1] for the lowest output error on calibration
            activations; the weight is quantised as W * s and 1/s must be
            folded into whatever produces x (returned);
  * GPTQ  - column-by-column quantisation with second-order error feedback
            from H = X^T X (Cholesky of the damped inverse), group-wise scales
            chosen when a group starts.

Reference: rlx-quant-calib (RTN / AWQ / GPTQ / BitNet, GGUF sink),
rlx-models-core src/mxfp4_pack.rs.
"""
from __future__ import annotations


import torch

from .mxfp4 import E2M1, dequantize_mxfp4, quantize_mxfp4

# -- formats --------------------------------------------------------------------

_MAGS = E2M1[:8]


def _e2m1_round(a: torch.Tensor) -> torch.Tensor:
    """Nearest E2M1 code (0..15) of a (already scaled) float tensor."""
    mags = _MAGS.to(a.device)
    idx = torch.bucketize(a.abs(), (mags[1:] + mags[:-1]) / 2)
    return (idx + torch.where(a < 0, 8, 0)).to(torch.uint8)


def quantize_nvfp4(w: torch.Tensor):
    """[..., K] (K % 16 == 0) -> (codes uint8 [..., K] (one code per byte, low 4 bits),
    block scales e4m3 [..., K/16], tensor scale fp32). Value = E2M1 * block * tensor."""
    x = w.float().reshape(*w.shape[:-1], -1, 16)
    amax = x.abs().amax()
    tscale = (amax / (6.0 * 448.0)).clamp_min(1e-30)
    bamax = x.abs().amax(-1)
    bscale = (bamax / (6.0 * tscale)).clamp(max=448.0).to(torch.float8_e4m3fn)
    bs = bscale.float().clamp_min(1e-30)
    codes = _e2m1_round(x / (bs[..., None] * tscale))
    return codes.reshape(w.shape), bscale, tscale.float()


def dequantize_nvfp4(codes, bscale, tscale) -> torch.Tensor:
    vals = E2M1.to(codes.device)[codes.long()].reshape(*codes.shape[:-1], -1, 16)
    return (vals * bscale.float()[..., None] * tscale).reshape(codes.shape)


def quantize_fp8(w: torch.Tensor):
    """Per-output-channel E4M3: (fp8 [out, in], scale fp32 [out])."""
    s = (w.float().abs().amax(-1) / 448.0).clamp_min(1e-12)
    return (w.float() / s[:, None]).to(torch.float8_e4m3fn), s


def dequantize_fp8(q, s) -> torch.Tensor:
    return q.float() * s[:, None]


def mxfp4_rtn(w: torch.Tensor) -> torch.Tensor:
    b, s = quantize_mxfp4(w)
    return dequantize_mxfp4(b, s)


def quantize_int_group(w: torch.Tensor, bits: int = 4, group: int = 128):
    """Group-wise symmetric integer RTN: per group of ``group`` input columns
    scale = amax / (2^(bits-1) - 1), codes in [-(2^(bits-1) - 1), 2^(bits-1) - 1]
    -> (int8 codes [out, in], fp32 scales [out, in / group])."""
    out_f, in_f = w.shape
    g = min(group, in_f)
    qmax = (1 << (bits - 1)) - 1
    wg = w.float().view(out_f, in_f // g, g)
    scale = (wg.abs().amax(-1) / qmax).clamp_min(1e-12)
    q = (wg / scale.unsqueeze(-1)).round().clamp(-qmax, qmax).to(torch.int8)
    return q.view(out_f, in_f), scale


def dequantize_int_group(q: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    out_f, in_f = q.shape
    g = in_f // scale.shape[1]
    return (q.float().view(out_f, -1, g) * scale.unsqueeze(-1)).view(out_f, in_f)


def quantize_bitnet(w: torch.Tensor):
    """BitNet b1.58 weights (Ma et al. 2024): ternary codes round(W / mean|W|)
    clipped to {-1, 0, 1} with the per-tensor absmean as the scale."""
    scale = w.float().abs().mean().clamp_min(1e-8)
    q = (w.float() / scale).round().clamp(-1, 1).to(torch.int8)
    return q, scale


def dequantize_bitnet(q: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    return q.float() * scale


def pack_ternary(q: torch.Tensor) -> torch.Tensor:
    """{-1, 0, 1} codes -> 2-bit fields (code + 1), four per byte, low bits first."""
    u = (q.to(torch.int16) + 1).to(torch.uint8).view(q.shape[0], -1, 4)
    return u[..., 0] | (u[..., 1] << 2) | (u[..., 2] << 4) | (u[..., 3] << 6)


def unpack_ternary(p: torch.Tensor) -> torch.Tensor:
    f = torch.stack([(p >> s) & 3 for s in (0, 2, 4, 6)], -1).to(torch.int8) - 1
    return f.view(p.shape[0], -1)


def bitnet_activation_quant(x: torch.Tensor):
    """Per-token int8 absmax activations of BitNet b1.58: (int8 codes, fp32 scale [tokens, 1])."""
    s = (x.float().abs().amax(-1, keepdim=True) / 127).clamp_min(1e-8)
    return (x.float() / s).round().clamp(-128, 127).to(torch.int8), s


FORMATS = {
    "mxfp4": mxfp4_rtn,
    "nvfp4": lambda w: dequantize_nvfp4(*quantize_nvfp4(w)),
    "fp8": lambda w: dequantize_fp8(*quantize_fp8(w)),
    "int4": lambda w: dequantize_int_group(*quantize_int_group(w, 4)),
    "int8": lambda w: dequantize_int_group(*quantize_int_group(w, 8)),
    "bitnet": lambda w: dequantize_bitnet(*quantize_bitnet(w)),
}


# -- calibration ---------------------------------------------------------------

def output_error(w: torch.Tensor, wq: torch.Tensor, x: torch.Tensor) -> float:
    """Relative error of the layer output on calibration activations x [n, in]."""
    ref = x.float() @ w.float().t()
    return float((x.float() @ wq.float().t() - ref).norm() / ref.norm().clamp_min(1e-12))


def awq(w: torch.Tensor, x: torch.Tensor, fmt: str = "mxfp4", grid: int = 20):
    """Returns (dequantised W' = Q(W s) / s, s [in], chosen alpha). The quantised
    weight to store is Q(W s); the caller folds 1/s into the producer of x."""
    q = FORMATS[fmt]
    act = x.float().abs().mean(0).clamp_min(1e-8)
    best = (float("inf"), None, None, None)
    for i in range(grid + 1):
        a = i / grid
        s = act.pow(a)
        s = s / (s.max() * s.min()).sqrt()  # keep scales centred around 1
        wq = q(w.float() * s[None, :]) / s[None, :]
        err = output_error(w, wq, x)
        if err < best[0]:
            best = (err, wq, s, a)
    return best[1], best[2], best[3]


def _group_scale(fmt: str, grp: torch.Tensor) -> torch.Tensor:
    """Per-row scale of a column group, fixed when the group starts."""
    amax = grp.abs().amax(1).clamp_min(1e-30)
    if fmt == "mxfp4":
        return torch.pow(2.0, torch.ceil(torch.log2(amax / 6.0)))
    if fmt == "nvfp4":
        return (amax / 6.0).to(torch.float8_e4m3fn).float().clamp_min(1e-30)
    if fmt == "fp8":
        return amax / 448.0
    if fmt in ("int4", "int8"):
        return amax / ((1 << ((4 if fmt == "int4" else 8) - 1)) - 1)
    raise ValueError(fmt)


def _quant_col(fmt: str, col: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    if fmt == "fp8":
        return (col / scale).clamp(-448, 448).to(torch.float8_e4m3fn).float() * scale
    if fmt in ("int4", "int8"):
        qmax = (1 << ((4 if fmt == "int4" else 8) - 1)) - 1
        return (col / scale).round().clamp(-qmax, qmax) * scale
    v = (col / scale).clamp(-6.0, 6.0)
    return E2M1.to(col.device)[_e2m1_round(v).long()] * scale


def gptq(w: torch.Tensor, x: torch.Tensor, fmt: str = "mxfp4", group: int | None = None, block: int = 128,
         damp: float = 0.01) -> torch.Tensor:
    """Group-wise GPTQ (Frantar et al. 2022): columns in order, each quantised
    with its group's scale (fixed at the group's first column from the
    error-corrected weights), the rounding error spread over the remaining
    columns through the upper Cholesky factor of the damped inverse Hessian."""
    if fmt == "bitnet":
        raise ValueError("GPTQ needs a group-wise format; BitNet ternary weights use RTN (per-tensor absmean)")
    group = group or {"mxfp4": 32, "nvfp4": 16, "fp8": w.shape[1], "int4": 128, "int8": 128}[fmt]
    group = min(group, w.shape[1])
    W = w.float().clone()
    out_f, in_f = W.shape
    H = x.float().t() @ x.float()
    dead = torch.diag(H) == 0
    H[dead, dead] = 1
    W[:, dead] = 0
    H += damp * torch.mean(torch.diag(H)) * torch.eye(in_f, device=H.device)
    Hinv = torch.linalg.cholesky(torch.cholesky_inverse(torch.linalg.cholesky(H)), upper=True)
    Q = torch.zeros_like(W)
    scale = None
    for b0 in range(0, in_f, block):
        b1 = min(b0 + block, in_f)
        W1 = W[:, b0:b1].clone()
        E1 = torch.zeros_like(W1)
        Hb = Hinv[b0:b1, b0:b1]
        for j in range(b1 - b0):
            c = b0 + j
            if c % group == 0:
                scale = _group_scale(fmt, W1[:, j:j + group] if j + group <= b1 - b0 else
                                     torch.cat([W1[:, j:], W[:, b1:b1 + group - (b1 - b0 - j)]], 1))
            qcol = _quant_col(fmt, W1[:, j], scale)
            Q[:, c] = qcol
            err = (W1[:, j] - qcol) / Hb[j, j]
            W1[:, j:] -= err[:, None] * Hb[j, j:][None, :]
            E1[:, j] = err
        W[:, b1:] -= E1 @ Hinv[b0:b1, b1:]
    return Q.to(w.dtype)


def quantize_weight(w, x=None, algo: str = "rtn", fmt: str = "mxfp4"):
    """One entry point: returns the dequantised weight chosen by ``algo``
    (plus AWQ's input scales, else None)."""
    if algo == "rtn" or x is None:
        return FORMATS[fmt](w).to(w.dtype), None
    if algo == "awq":
        wq, s, _ = awq(w, x, fmt)
        return wq.to(w.dtype), s
    if algo == "gptq":
        return gptq(w, x, fmt), None
    raise ValueError(f"unknown algorithm {algo}")
