"""Flat, persistent parameter / gradient / compute-copy buffers for one stage.

Every parameter of a stage becomes a view into one fp32 ``data`` buffer and
its gradient a view into one fp32 ``grad`` buffer (``param.main_grad`` and
``param.grad`` are that view). Parameters that one fused GEMM consumes
together (q/k/v, gate/up) share one region ``[K, sum(N_i)]`` and are column
slices of it, so the fused kernel reads a single ``[K, 3N]`` weight while the
state dict still has the separate ``q.weight``/``k.weight``/``v.weight``
entries of the reference layout (``tests/reference.py:17-27``).

On CUDA a bf16 ``compute`` mirror with the same layout holds the weights the
GEMMs read in bf16 mode; the fused optimizer refreshes it in the same pass that
updates the fp32 master, so no per-step cast kernels run.

Regions start on 64-element boundaries (256 B of fp32, 128 B of bf16), which
satisfies TMA's 16-byte alignment rule for every tensor the kernels load.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn as nn

_ALIGN = 64


def _round_up(n: int, a: int) -> int:
    return (n + a - 1) // a * a


@dataclass
class Region:
    offset: int
    shape: tuple[int, ...]
    params: tuple[nn.Parameter, ...]
    names: tuple[str, ...]

    @property
    def numel(self) -> int:
        n = 1
        for s in self.shape:
            n *= s
        return n


class FlatBuffers:
    """Owns the flat buffers of one module tree and re-points its parameters."""

    def __init__(self, module: nn.Module, fused_groups: list[list[str]],
                 compute_dtype: torch.dtype | None):
        named = list(module.named_parameters())  # shared parameters appear once
        if not named:
            raise ValueError("module has no parameters")
        device = named[0][1].device
        by_name = dict(named)
        group_of = {}
        for group in fused_groups:
            for name in group:
                group_of[name] = tuple(group)

        regions: list[Region] = []
        done: set[str] = set()
        offset = 0
        for name, param in named:
            if name in done:
                continue
            members = group_of.get(name, (name,))
            params = tuple(by_name[n] for n in members)
            if len(params) > 1:
                k = params[0].shape[0]
                if any(p.dim() != 2 or p.shape[0] != k for p in params):
                    raise ValueError(f"fused group {members} needs 2-D weights with equal dim 0")
                shape = (k, sum(p.shape[1] for p in params))
            else:
                shape = tuple(param.shape)
            region = Region(offset, shape, params, members)
            regions.append(region)
            done.update(members)
            offset = _round_up(offset + region.numel, _ALIGN)

        self.numel = offset
        self.device = device
        self.regions = regions
        self.data = torch.zeros(offset, dtype=torch.float32, device=device)
        self.grad = torch.zeros(offset, dtype=torch.float32, device=device)
        self.compute = (torch.empty(offset, dtype=compute_dtype, device=device)
                        if compute_dtype is not None and compute_dtype != torch.float32 else None)
        self._region_of: dict[int, Region] = {}
        for region in regions:
            self._bind(region)

    def _views(self, flat: torch.Tensor, region: Region):
        block = flat[region.offset: region.offset + region.numel].view(region.shape)
        if len(region.params) == 1:
            return block, [block]
        views, col = [], 0
        for p in region.params:
            views.append(block[:, col: col + p.shape[1]])
            col += p.shape[1]
        return block, views

    def _bind(self, region: Region) -> None:
        data_block, data_views = self._views(self.data, region)
        grad_block, grad_views = self._views(self.grad, region)
        comp_block, comp_views = (self._views(self.compute, region) if self.compute is not None
                                  else (None, [None] * len(region.params)))
        for p, dv, gv, cv in zip(region.params, data_views, grad_views, comp_views):
            dv.copy_(p.data)
            p.data = dv
            p.main_grad = gv
            p.grad = gv
            p.compute_copy = cv
            self._region_of[id(p)] = region
        region.data_block, region.grad_block, region.compute_block = data_block, grad_block, comp_block
        if comp_block is not None:
            comp_block.copy_(data_block)

    def region_of(self, param: nn.Parameter) -> Region:
        return self._region_of[id(param)]

    def refresh_compute(self) -> None:
        """Re-derive the compute mirror from the fp32 master (after loads/broadcasts)."""
        if self.compute is not None:
            self.compute.copy_(self.data)

    def rehome_grad(self, new_grad: torch.Tensor) -> None:
        """Move the flat gradient into ``new_grad`` (same numel, fp32, same device),
        e.g. a symmetric-memory allocation that peers map, and re-point every view."""
        if new_grad.numel() != self.numel or new_grad.dtype != self.grad.dtype:
            raise ValueError("replacement gradient buffer has the wrong size or dtype")
        new_grad.copy_(self.grad)
        self.grad = new_grad
        for region in self.regions:
            region.grad_block, _ = self._views(self.grad, region)
        self.reattach_grads()

    def reattach_grads(self) -> None:
        """Point ``param.grad`` back at the flat views (after ``zero_grad(set_to_none)``)."""
        for region in self.regions:
            _, grad_views = self._views(self.grad, region)
            for p, gv in zip(region.params, grad_views):
                p.main_grad = gv
                p.grad = gv

    def zero_grad(self) -> None:
        self.grad.zero_()
        self.reattach_grads()
