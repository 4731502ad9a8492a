"""Writer of the FP8 KV cache layout read by ``forward_fp8``.

One 656-byte row per token (DeepSeek-V3.2's FP8 MLA cache layout): 512
float8 e4m3 latent values, 4 FP32 scales (scale k = max |kv| over latent
dims [128k, 128k + 128) / 448, the e4m3 maximum; 1 for an all-zero block),
then the 64 rope dims as BF16. The reference keeps kv in BF16 only; this
module is the cache writer a serving engine would call, not part of the
forward.
"""
from __future__ import annotations

import torch

ROW_BYTES = 656
E4M3_MAX = 448.0


def quantize_kv_fp8(kv: torch.Tensor, k_rope: torch.Tensor) -> torch.Tensor:
    """kv BF16 ``[B, L, 1, 512]`` and k_rope BF16 ``[B, L, 1, 64]`` ->
    uint8 ``[B, L, 1, 656]`` in the layout above (on kv's device)."""
    if kv.shape[-1] != 512 or k_rope.shape[-1] != 64 or kv.shape[:-1] != k_rope.shape[:-1]:
        raise ValueError("need kv[..., 512] and k_rope[..., 64] with the same leading shape")
    lead = kv.shape[:-1]
    blocks = kv.float().reshape(*lead, 4, 128)
    amax = blocks.abs().amax(-1)
    scale = torch.where(amax > 0, amax / E4M3_MAX, torch.ones_like(amax))
    q8 = (blocks / scale[..., None]).clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn)
    out = torch.empty((*lead, ROW_BYTES), dtype=torch.uint8, device=kv.device)
    out[..., :512] = q8.reshape(*lead, 512).view(torch.uint8)
    out[..., 512:528] = scale.contiguous().view(torch.uint8).reshape(*lead, 16)
    out[..., 528:] = k_rope.contiguous().view(torch.uint8).reshape(*lead, 128)
    return out
