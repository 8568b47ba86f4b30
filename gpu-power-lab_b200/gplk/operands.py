"""Seeded GEMM operands for the FP8 and NVFP4 rungs, quantised on the device.

The rungs' inputs are N(0,1) matrices quantised the way the rung
configuration states:

  FP8   per-tensor scale = amax / 448; q = E4M3(x / scale), round to nearest
        even, saturating at +-448.
  NVFP4 global scale g = amax / (6 * 448); per 16 consecutive K-elements a
        UE4M3 block scale s = E4M3(block_amax / 6 / g); q = E2M1(x / (s * g)),
        round to nearest even (ties to the even mantissa), saturating at +-6;
        two elements per byte, element 2j in the low nibble. The block
        scales are laid out in cuBLASLt's VEC16_UE4M3 order (128-row x
        4-scale blocks of 512 bytes), the order gplk_gemm_nvfp4_tn reads.

Every step is an elementwise IEEE single-precision operation in the same
order as the C restatement of these rules, so the bytes are identical to it
on the same input (checked by the tests on CPU and GPU tensors). Works on
any torch device.
"""
from __future__ import annotations

import torch

E4M3_MAX = 448.0
E2M1_MAX = 6.0


def normal(rows: int, cols: int, seed: int, device) -> torch.Tensor:
    """rows x cols float32 N(0,1) from torch's generator seeded with `seed`."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return torch.randn(rows, cols, device=device, generator=g, dtype=torch.float32)


def _e4m3_bits(v: torch.Tensor) -> torch.Tensor:
    """float32 -> E4M3 (fn) byte, round to nearest even, saturating."""
    return v.clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn).view(torch.uint8)


def quantize_fp8(x: torch.Tensor) -> tuple[torch.Tensor, float]:
    """Per-tensor E4M3: returns (uint8 codes of x's shape, scale)."""
    amax = float(x.abs().max())
    scale = torch.tensor(amax, dtype=torch.float32) / E4M3_MAX if amax > 0.0 else torch.tensor(1.0)
    scale = float(scale)
    return _e4m3_bits(x / torch.tensor(scale, dtype=torch.float32, device=x.device)), scale


def e2m1_codes(v: torch.Tensor) -> torch.Tensor:
    """float32 -> E2M1 nibble (sign in bit 3), round to nearest even on the
    grid 0, 0.5, 1, 1.5, 2, 3, 4, 6 and saturating at 6. NaN encodes as 0."""
    a = v.abs()
    code = ((a > 0.25).to(torch.uint8) + (a >= 0.75).to(torch.uint8) + (a > 1.25).to(torch.uint8)
            + (a >= 1.75).to(torch.uint8) + (a > 2.5).to(torch.uint8) + (a >= 3.5).to(torch.uint8)
            + (a > 5.0).to(torch.uint8))
    code = code | (torch.signbit(v).to(torch.uint8) << 3)
    return torch.where(torch.isnan(v), torch.zeros_like(code), code)


def sf_bytes(rows: int, k: int) -> int:
    """Bytes of one VEC16_UE4M3 scale array for `rows` rows and K = k."""
    return ((rows + 127) // 128) * ((k // 16 + 3) // 4) * 512


def sf_layout(s8: torch.Tensor) -> torch.Tensor:
    """rows x (k/16) scale bytes -> the flat VEC16_UE4M3 block layout: block
    (r/128, kb/4) at ((r/128) * ceil(kb_n/4) + kb/4) * 512, and inside it
    (r % 32) * 16 + ((r % 128) / 32) * 4 + kb % 4. Padding is zero."""
    rows, kb_n = s8.shape
    R, KB = (rows + 127) // 128 * 128, (kb_n + 3) // 4 * 4
    p = torch.zeros(R, KB, dtype=torch.uint8, device=s8.device)
    p[:rows, :kb_n] = s8
    # r = rb*128 + rq*32 + r32, kb = kb4*4 + kk  ->  [rb, kb4, r32, rq, kk]
    p = p.view(R // 128, 4, 32, KB // 4, 4).permute(0, 3, 2, 1, 4)
    return p.contiguous().view(-1)


def quantize_nvfp4(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, float]:
    """rows x k float32 (k a multiple of 16) -> (packed rows x k/2 uint8,
    VEC16_UE4M3 scale bytes, global scale)."""
    rows, k = x.shape
    assert k % 16 == 0
    amax = float(x.abs().max())
    one = torch.tensor(1.0, dtype=torch.float32)
    g = float(torch.tensor(amax, dtype=torch.float32) / (6.0 * 448.0)) if amax > 0.0 else float(one)
    gt = torch.tensor(g, dtype=torch.float32, device=x.device)
    xb = x.view(rows, k // 16, 16)
    bmax = xb.abs().amax(dim=2)
    want = bmax / 6.0 / gt
    s8 = torch.where(want > 0, _e4m3_bits(want) & 0x7F, torch.zeros_like(want, dtype=torch.uint8))
    bs = s8.view(torch.float8_e4m3fn).to(torch.float32) * gt
    q = torch.where(bs.unsqueeze(2) > 0, e2m1_codes(xb / bs.unsqueeze(2)), torch.zeros_like(xb, dtype=torch.uint8))
    q = q.view(rows, k // 2, 2)
    packed = (q[..., 0] | (q[..., 1] << 4)).contiguous()
    return packed, sf_layout(s8), g
