"""CPU restatement of NF4 blockwise quantisation (test infrastructure only).

The reference gets its 4-bit base layers from bitsandbytes 0.50.2
(``Linear4bit`` with NF4, blocksize 64; the reference loads adapters over them in
``harness/eval_adapter.py:21-69``), which is not installed here and is not
pinned by any reference test: parity with bitsandbytes is unpinned, and this
restatement is the checker for the CUDA kernels in ``csrc/nf4.cu``.

Code values: the NF4 construction of the QLoRA paper (Dettmers et al. 2023,
arXiv 2305.14314, Appendix E). The positive half takes the 8 standard-normal
quantiles at probabilities evenly spaced from ``offset`` down to 0.5
(exclusive); the negative half the 7 quantiles of the mirrored range; zero is
exact. ``offset`` = 1 - (1/(2*15) + 1/(2*16)) / 2 keeps the extreme quantiles
finite. The 16 values are normalised by their maximum to [-1, 1].
"""

from __future__ import annotations

import numpy as np
import torch


def nf4_code() -> torch.Tensor:
    """The 16 NF4 code values, ascending, fp32."""
    from scipy.stats import norm

    offset = 1.0 - 0.5 * (1.0 / 30.0 + 1.0 / 32.0)
    pos = norm.ppf(np.linspace(offset, 0.5, 9)[:-1])
    neg = -norm.ppf(np.linspace(offset, 0.5, 8)[:-1])
    vals = np.sort(np.concatenate([pos, [0.0], neg]))
    vals = vals / np.abs(vals).max()
    return torch.tensor(vals, dtype=torch.float32)


def nf4_quantize(w: torch.Tensor, code: torch.Tensor, blocksize: int = 64):
    """Return (packed uint8 [n/2], absmax fp32 [n/blocksize]); nearest code, ties -> lower index."""
    x = w.detach().reshape(-1).float().cpu()
    assert x.numel() % blocksize == 0
    blocks = x.view(-1, blocksize)
    absmax = blocks.abs().amax(dim=1)
    inv = torch.where(absmax > 0, 1.0 / absmax, torch.zeros_like(absmax))
    normed = blocks * inv[:, None]
    dist = (normed[..., None] - code.view(1, 1, 16)).abs()
    idx = dist.argmin(dim=-1).reshape(-1).to(torch.uint8)  # first minimum = lower index
    packed = (idx[0::2] << 4) | idx[1::2]
    return packed, absmax


def nf4_dequantize(packed: torch.Tensor, absmax: torch.Tensor, code: torch.Tensor,
                   blocksize: int = 64, dtype=torch.bfloat16) -> torch.Tensor:
    p = packed.cpu().to(torch.int64)
    idx = torch.stack([p >> 4, p & 0xF], dim=1).reshape(-1)
    vals = code[idx].view(-1, blocksize) * absmax.cpu().view(-1, 1)
    return vals.reshape(-1).to(dtype)
