"""AdamW over a stage's flat parameter buffer.

One update pass over the flat fp32 master buffer implements
``torch.optim.AdamW`` (decoupled weight decay, bias-corrected moments; the
reference constructs it with torch's defaults, ``nano_megatron/train.py:85``).
On CUDA the pass is one multi-tensor kernel that also applies the
gradient-clipping coefficient on load and rewrites the bf16 compute copy, so
clip, step and cast cost one read of each buffer. On CPU it runs the same
update with torch ops.

The moments are flat buffers with the parameter buffer's layout; the state
dict stores them flat together with the step count and hyperparameters.
"""

from __future__ import annotations

import torch

from . import ops
from .ops import reference as ref


class FusedAdamW:
    def __init__(self, model, lr: float = 1e-3, betas=(0.9, 0.999), eps: float = 1e-8,
                 weight_decay: float = 0.01):
        if lr < 0 or eps < 0 or weight_decay < 0:
            raise ValueError("lr, eps and weight_decay must be non-negative")
        buffers = getattr(model, "flat_buffers", None)
        if buffers is None:
            raise ValueError("FusedAdamW needs a model with flat buffers")
        self.flat = buffers
        self.param_groups = [dict(lr=lr, betas=tuple(betas), eps=eps, weight_decay=weight_decay)]
        self.step_count = 0
        self.exp_avg = torch.zeros_like(buffers.data)
        self.exp_avg_sq = torch.zeros_like(buffers.data)

    def zero_grad(self, set_to_none: bool = True) -> None:
        """Zero the flat gradient buffer (parameters keep their grad views)."""
        self.flat.zero_grad()

    @torch.no_grad()
    def step(self, grad_scale: torch.Tensor | float | None = None) -> None:
        """One AdamW step; ``grad_scale`` (e.g. a clip coefficient) multiplies the gradient."""
        group = self.param_groups[0]
        self.step_count += 1
        b = self.flat
        beta1, beta2 = group["betas"]
        if b.data.is_cuda:
            scale = grad_scale if isinstance(grad_scale, torch.Tensor) else torch.tensor(
                1.0 if grad_scale is None else float(grad_scale), device=b.data.device)
            ops.cuda_ops().adamw_flat(b.data, b.grad, self.exp_avg, self.exp_avg_sq, b.compute,
                                      scale.float(), lr=group["lr"], beta1=beta1, beta2=beta2,
                                      eps=group["eps"], weight_decay=group["weight_decay"],
                                      step=self.step_count)
        else:
            g = b.grad if grad_scale is None else b.grad * grad_scale
            ref.adamw_(b.data, g, self.exp_avg, self.exp_avg_sq, lr=group["lr"], beta1=beta1,
                       beta2=beta2, eps=group["eps"], weight_decay=group["weight_decay"],
                       step=self.step_count, compute_copy=b.compute)

    def state_dict(self) -> dict:
        return {
            "state": {"step": self.step_count, "exp_avg": self.exp_avg.clone(),
                      "exp_avg_sq": self.exp_avg_sq.clone()},
            "param_groups": [dict(g) for g in self.param_groups],
        }

    def load_state_dict(self, state: dict) -> None:
        s = state["state"]
        if s["exp_avg"].shape != self.exp_avg.shape:
            raise ValueError("optimizer state does not match the parameter buffer layout")
        self.step_count = int(s["step"])
        self.exp_avg.copy_(s["exp_avg"])
        self.exp_avg_sq.copy_(s["exp_avg_sq"])
        self.param_groups = [dict(g) for g in state["param_groups"]]
        for g in self.param_groups:
            g["betas"] = tuple(g["betas"])
