"""Final norm + lm_head + cross-entropy on the device, forward and backward.

FitLLM seeds the backward of each micro-batch from its lm_head loss
(fitllm/backward.py:188-198): h_last -> final RMSNorm -> lm_head (bf16,
vocab 152,064, no bias) -> CrossEntropyLoss (mean over labels != -100) ->
(loss * loss_scale).backward() gives grad_h; the logged loss is the same mean
(fitllm/trainer.py:506-522, there on fp32 logits moved to the CPU).

Here, per micro-batch: RMSNorm (fitq_rmsnorm_fwd) -> logits = x.W^T on the
tcgen05 GEMM (bf16 [S, V]) -> fitq_cross_entropy turns the logits in place
into d(loss_scale * loss)/dlogits and writes the mean loss to a device scalar
-> dx = dlogits.W on the same GEMM (against Wᵀ, materialised once: the
lm_head is frozen) -> fitq_rmsnorm_bwd.  Nothing leaves the device and no
per-micro-batch synchronisation is needed; the losses stay on the device
until the caller reads them.
"""
from __future__ import annotations

from typing import List, Optional, Tuple

import torch

from . import _lib, ops


class LMHeadLoss:
    """Frozen final norm + lm_head with the reference's loss.

    norm_weight: [H] bf16; weight: [V, H] bf16 (nn.Linear layout)."""

    def __init__(self, norm_weight: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6,
                 ignore_index: int = -100):
        if weight.dtype != torch.bfloat16 or norm_weight.dtype != torch.bfloat16:
            raise TypeError("LMHeadLoss: bf16 norm weight and lm_head weight expected")
        self.norm_weight = norm_weight.contiguous()
        self.weight = weight.contiguous()
        self.weight_t = self.weight.t().contiguous()  # [H, V] for dx = dlogits . W
        self.eps = float(eps)
        self.ignore_index = int(ignore_index)

    @property
    def vocab(self) -> int:
        return int(self.weight.shape[0])

    def _norm(self, h2: torch.Tensor) -> torch.Tensor:
        L = _lib.load()
        y = torch.empty_like(h2)
        _lib.check(L.fitq_rmsnorm_fwd(h2.data_ptr(), self.norm_weight.data_ptr(), y.data_ptr(),
                                      h2.shape[0], h2.shape[1], self.eps, ops._stream(h2.device)),
                   "fitq_rmsnorm_fwd")
        return y

    def _norm_bwd(self, dy: torch.Tensor, h2: torch.Tensor) -> torch.Tensor:
        L = _lib.load()
        dx = torch.empty_like(h2)
        _lib.check(L.fitq_rmsnorm_bwd(dy.data_ptr(), h2.data_ptr(), self.norm_weight.data_ptr(),
                                      dx.data_ptr(), h2.shape[0], h2.shape[1], self.eps,
                                      ops._stream(h2.device)), "fitq_rmsnorm_bwd")
        return dx

    def logits(self, h: torch.Tensor) -> torch.Tensor:
        """[..., V] bf16 logits of the final hidden states (forward only)."""
        h2 = h.reshape(-1, h.shape[-1]).contiguous()
        return ops.gemm_bf16_tn(self._norm(h2), self.weight).view(*h.shape[:-1], self.vocab)

    def loss_and_grad(self, h: torch.Tensor, labels: torch.Tensor,
                      loss_scale: float = 1.0) -> Tuple[torch.Tensor, torch.Tensor]:
        """One micro-batch: h [B, S, H] bf16 (last layer output), labels [B, S]
        int64 (already shifted, -100 ignored).  Returns (mean CE loss as a
        device fp32 scalar, grad of loss * loss_scale w.r.t. h, bf16)."""
        L = _lib.load()
        dev = h.device
        h2 = h.reshape(-1, h.shape[-1]).contiguous()
        rows = h2.shape[0]
        lab = labels.reshape(-1).to(device=dev, dtype=torch.int64).contiguous()
        if lab.numel() != rows:
            raise ValueError("loss_and_grad: labels must have one entry per token")
        with torch.cuda.device(dev):
            x = self._norm(h2)
            logits = ops.gemm_bf16_tn(x, self.weight)
            del x
            loss = torch.empty((), dtype=torch.float32, device=dev)
            nbytes = L.fitq_cross_entropy_workspace(rows)
            ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
            _lib.check(L.fitq_cross_entropy(logits.data_ptr(), lab.data_ptr(), rows, self.vocab,
                                            self.ignore_index, float(loss_scale), loss.data_ptr(),
                                            ws.data_ptr(), nbytes, ops._stream(dev)),
                       "fitq_cross_entropy")
            dx = ops.gemm_bf16_tn(logits, self.weight_t)  # logits now hold dlogits
            del logits
            grad = self._norm_bwd(dx, h2)
        return loss, grad.view_as(h)

    def loss_and_grad_microbatches(self, h: torch.Tensor, labels: torch.Tensor,
                                   loss_scale: float) -> Tuple[List[torch.Tensor], torch.Tensor]:
        """h [nmb, S, H], labels [nmb, S]: the reference's per-micro-batch loop
        (each micro-batch its own mean).  Returns (losses, grad_h [nmb, S, H])."""
        grad = torch.empty_like(h)
        losses = []
        for i in range(h.shape[0]):
            loss, g = self.loss_and_grad(h[i:i + 1], labels[i:i + 1], loss_scale)
            grad[i:i + 1] = g
            losses.append(loss)
        return losses, grad


def random_lm_head(hidden: int, vocab: int, device, seed: int = 0, std: float = 0.02,
                   eps: float = 1e-6) -> LMHeadLoss:
    """Seeded N(0, std) bf16 lm_head with a unit final norm (synthetic workloads)."""
    g = torch.Generator(device=device).manual_seed(seed)
    w = (torch.randn(vocab, hidden, generator=g, device=device) * std).bfloat16()
    return LMHeadLoss(torch.ones(hidden, dtype=torch.bfloat16, device=device), w, eps=eps)
