"""MXFP4 (OCP microscaling FP4): E2M1 elements, E8M0 power-of-two scale per
group of 32 along the reduction dimension.

Storage matches the gpt-oss checkpoints (and the reference's pack,
rlx-models-core src/mxfp4_pack.rs:60-290): ``blocks`` uint8 [..., G, 16] with
two codes per byte (low nibble first), ``scales`` uint8 [..., G] holding the
biased exponent (value 2^(s-127)).

Quantisation rule (same as the reference's packer): per group the scale
exponent is the smallest e with 6 * 2^e >= amax (6 is the largest E2M1
magnitude, so nothing saturates); each element rounds to the nearest E2M1
value of x / 2^e (ties to the larger magnitude index as in a searchsorted).
"""
from __future__ import annotations

import torch

E2M1 = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0])
GROUP = 32


def dequantize_mxfp4(blocks: torch.Tensor, scales: torch.Tensor, dtype=torch.float32) -> torch.Tensor:
    """blocks [..., G, 16] uint8, scales [..., G] uint8 -> [..., G*32] ``dtype``."""
    lut = E2M1.to(blocks.device)
    lo = (blocks & 0x0F).long()
    hi = (blocks >> 4).long()
    vals = torch.stack([lut[lo], lut[hi]], dim=-1).reshape(*blocks.shape[:-1], 32)
    exp = scales.to(torch.int32) - 127
    out = vals * torch.pow(2.0, exp.float())[..., None]
    return out.reshape(*blocks.shape[:-2], blocks.shape[-2] * 32).to(dtype)


def quantize_mxfp4(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """[..., K] float (K % 32 == 0) -> (blocks [..., K/32, 16], scales [..., K/32])."""
    K = w.shape[-1]
    assert K % GROUP == 0
    x = w.float().reshape(*w.shape[:-1], K // GROUP, GROUP)
    amax = x.abs().amax(-1)
    e = torch.ceil(torch.log2(torch.clamp(amax, min=1e-30) / 6.0))
    e = torch.where(amax > 0, e, torch.full_like(e, -127.0)).clamp(-127, 127)
    scaled = x / torch.pow(2.0, e)[..., None]
    mags = E2M1[:8].to(w.device)
    a = scaled.abs()
    # nearest magnitude: midpoints between consecutive E2M1 magnitudes
    mids = (mags[1:] + mags[:-1]) / 2
    idx = torch.bucketize(a, mids)
    code = idx + torch.where(scaled < 0, 8, 0)
    code = code.to(torch.uint8)
    pairs = code.reshape(*code.shape[:-1], 16, 2)
    blocks = (pairs[..., 0] | (pairs[..., 1] << 4)).to(torch.uint8)
    scales = (e + 127).to(torch.uint8)
    return blocks, scales


def mxfp4_roundtrip(w: torch.Tensor) -> torch.Tensor:
    b, s = quantize_mxfp4(w)
    return dequantize_mxfp4(b, s)


TILE_ROWS, TILE_K = 128, 64
TILE_BYTES = TILE_ROWS * TILE_K // 2 + TILE_ROWS * TILE_K // GROUP  # 4096 code bytes + 256 scale bytes


def tile_mxfp4(blocks: torch.Tensor, scales: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Grouped-GEMM weight layout: blocks [E, N, K/32, 16] (or [E, N, K/2]) and
    scales [E, N, K/32] -> (tiles uint8 [E, ceil(N/128), K/64, 4352],
    row_exp uint8 [E, ceil(N/128) * 128]).

    Each (expert, 128-row tile, 64-wide k tile) is one contiguous block:
    [2 k-halves][128 rows][16 code bytes] then [2 k-halves][128 rows] scale
    offsets (a kernel thread owns one row and one half). A scale offset
    is row_exp - s, with row_exp the largest E8M0 exponent of the weight row,
    so the kernel multiplies codes by 2^-(offset) <= 1 and applies
    2^(row_exp - 127) to the accumulator row. Rows past N are zero."""
    E, N = blocks.shape[0], blocks.shape[1]
    b = blocks.reshape(E, N, -1)
    K = b.shape[2] * 2
    assert K % TILE_K == 0 and scales.shape == (E, N, K // GROUP)
    NT, KT = (N + TILE_ROWS - 1) // TILE_ROWS, K // TILE_K
    pad = NT * TILE_ROWS - N
    row_exp = scales.amax(-1)                                   # [E, N]
    s = (row_exp[..., None] - scales).to(torch.uint8)           # offsets >= 0
    if pad:
        b = torch.cat([b, b.new_zeros(E, pad, b.shape[2])], 1)
        s = torch.cat([s, s.new_zeros(E, pad, s.shape[2])], 1)
        row_exp = torch.cat([row_exp, row_exp.new_zeros(E, pad)], 1)
    # [E, NT, 128 rows, KT, 2 halves, 16 bytes] -> [E, NT, KT, half, row, 16]
    bt = b.reshape(E, NT, TILE_ROWS, KT, 2, 16).permute(0, 1, 3, 4, 2, 5).reshape(E, NT, KT, TILE_ROWS * 32)
    st = s.reshape(E, NT, TILE_ROWS, KT, 2).permute(0, 1, 3, 4, 2).reshape(E, NT, KT, TILE_ROWS * 2)
    return torch.cat([bt, st], -1).contiguous(), row_exp.contiguous()


def untile_mxfp4(t: torch.Tensor, row_exp: torch.Tensor, N: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Inverse of ``tile_mxfp4``: -> (blocks [E, N, K/32, 16], scales [E, N, K/32])."""
    E, NT, KT, _ = t.shape
    b = t[..., :TILE_ROWS * 32].reshape(E, NT, KT, 2, TILE_ROWS, 16).permute(0, 1, 4, 2, 3, 5)
    s = t[..., TILE_ROWS * 32:].reshape(E, NT, KT, 2, TILE_ROWS).permute(0, 1, 4, 2, 3)
    b = b.reshape(E, NT * TILE_ROWS, KT * 32)[:, :N]
    s = s.reshape(E, NT * TILE_ROWS, KT * 2)[:, :N]
    s = (row_exp[:, :N, None].to(torch.int16) - s.to(torch.int16)).to(torch.uint8)
    return b.reshape(E, N, KT * 2, 16).contiguous(), s.contiguous()
