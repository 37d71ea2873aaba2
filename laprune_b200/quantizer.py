"""Drop-in for the encode surface of the reference's ``AdditiveQuantizer``
(laprune/quantizer.py:319-374) with pretrained codebooks.

``encode(X, method="icm", icm_iters=2)`` returns the reference's tuple
``(codes int64 [N, M], average loss, None)``: greedy residual codes from
this package's tcgen05 encoder, refined by up to ``icm_iters`` ICM sweeps
(both equal to the CPU arithmetic's), and, with ``return_loss``, the mean L2
norm of the final residual (``sqrt(sum((X - recon)^2, 1)).mean()``,
quantizer.py:372-373).  Codebook training (``fit``) is outside the decode
path and is not provided.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import ops

__all__ = ["AdditiveQuantizer"]


class AdditiveQuantizer:
    """M codebooks of K codewords of dimension d, encoding only."""

    def __init__(self, M: int, K: int, d: int, init: str = "pretrained", reg: float = 1e-4,
                 device: Optional[torch.device] = None, dtype: torch.dtype = torch.float32,
                 codebooks: Optional[torch.Tensor] = None, **kwargs) -> None:
        if codebooks is None:
            raise NotImplementedError(f"init={init!r} without codebooks: codebook training is not on the decode path")
        if tuple(codebooks.shape) != (M, K, d):
            raise ValueError(f"codebooks {tuple(codebooks.shape)} do not match (M, K, d) = {(M, K, d)}")
        self.M, self.K, self.d = M, K, d
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.dtype = dtype
        self.codebooks = codebooks.detach().to(device=self.device, dtype=torch.float32).contiguous()

    @torch.no_grad()
    def encode(self, X: torch.Tensor, method: str = "icm", icm_iters: int = 2, batch_size: int = 3000000,
               return_loss: bool = True):
        """``(codes, avg_loss, None)`` for ``X [N, d]`` (quantizer.py:319-344)."""
        if method != "icm":
            raise NotImplementedError("Only ICM method is implemented in this LUT version.")
        X = X.to(self.device)
        if X.dtype not in (torch.float32, torch.float16, torch.bfloat16):
            X = X.to(self.dtype)
        if X.stride(-1) != 1:
            X = X.contiguous()
        codes = ops.encode_keys(X, self.codebooks, icm_iters=int(icm_iters)).long()
        if not return_loss or X.shape[0] == 0:
            return codes, 0.0, None
        recon = torch.zeros((X.shape[0], self.d), dtype=torch.float32, device=self.device)
        for m in range(self.M):
            recon += self.codebooks[m][codes[:, m]]
        loss = torch.sqrt(((X.float() - recon) ** 2).sum(dim=1)).mean()
        return codes, float(loss), None
