"""Device time per op class of a training step, from CUDA events.

    with OpProfile() as prof:
        trainer.train_step(batches)
    print(prof.report(step_ms))

While active, every CUDA op of the op layer (:mod:`..ops.cuda`,
:mod:`..ops.fused_tp`, the data-parallel averaging of :mod:`..ops.dp_reduce`)
is bracketed by two CUDA events on the stream it is launched on; the wrappers
are removed on exit. :meth:`OpProfile.report` synchronizes once and sums the
elapsed times per op class. Everything else that runs on the device (ATen
element-wise kernels, NCCL point-to-point and control collectives, idle gaps
between launches) is the difference between the step time and the sum of the
compute-stream classes, reported as ``other``. Classes that run on a side
stream (the data-parallel buckets) overlap the compute stream and are listed
separately.

The events themselves cost a few microseconds of host time per op, so take
the step time for the report from an unprofiled run.
"""

from __future__ import annotations

from collections import defaultdict

import torch

# op-layer function -> class in the report
_CUDA_OPS = {
    "mm_nn": "gemm", "mm_nt": "gemm", "mm_tn_acc": "gemm (weight gradient)",
    "mm_swiglu": "gemm + swiglu epilogue",
    "rmsnorm": "rmsnorm", "rmsnorm_bwd": "rmsnorm backward", "add_rmsnorm": "residual add + rmsnorm",
    "attention": "attention forward", "attention_bwd": "attention backward",
    "swiglu": "swiglu", "swiglu_bwd": "swiglu backward",
    "embedding": "embedding", "embedding_bwd": "embedding backward",
    "ce_local_stats": "cross entropy", "ce_grad": "cross entropy",
    "lm_head_ce_fwd": "lm head + cross entropy", "lm_head_ce_grad": "lm head + cross entropy (grad)",
    "adamw_flat": "adamw", "weighted_sq_norm": "grad norm",
}
_FUSED_OPS = {
    "all_gather_matmul": "fused all-gather -> gemm",
    "matmul_reduce_scatter": "fused gemm -> reduce-scatter",
    "lm_head_cross_entropy": "lm head + cross entropy",
}
SIDE_STREAM_CLASSES = ("data-parallel averaging",)


class OpProfile:
    """Context manager that times op classes with CUDA events."""

    def __init__(self):
        self.events: dict[str, list] = defaultdict(list)
        self._patched: list[tuple[object, str, object]] = []

    def _wrap(self, module, name: str, label: str) -> None:
        fn = getattr(module, name, None)
        if fn is None:
            return
        events = self.events

        def timed(*args, **kwargs):
            start = torch.cuda.Event(enable_timing=True)
            end = torch.cuda.Event(enable_timing=True)
            start.record()
            out = fn(*args, **kwargs)
            end.record()
            events[label].append((start, end))
            return out

        self._patched.append((module, name, fn))
        setattr(module, name, timed)

    def __enter__(self) -> "OpProfile":
        from ..ops import cuda, dp_reduce, fused_tp
        for name, label in _CUDA_OPS.items():
            self._wrap(cuda, name, label)
        for name, label in _FUSED_OPS.items():
            self._wrap(fused_tp, name, label)
        self._wrap(dp_reduce.DPWorkspace, "all_reduce_avg", SIDE_STREAM_CLASSES[0])
        return self

    def __exit__(self, *exc) -> None:
        for module, name, fn in reversed(self._patched):
            setattr(module, name, fn)
        self._patched.clear()

    def report(self, step_ms: float | None = None, steps: int = 1) -> dict:
        """``{class: {"calls", "ms"}}`` per step, plus ``other`` when ``step_ms`` is given."""
        torch.cuda.synchronize()
        out = {}
        for label, pairs in self.events.items():
            total = sum(s.elapsed_time(e) for s, e in pairs)
            out[label] = {"calls": len(pairs) // steps, "ms": round(total / steps, 3)}
        if step_ms is not None:
            on_compute = sum(v["ms"] for k, v in out.items() if k not in SIDE_STREAM_CLASSES)
            out["other (ATen, NCCL, gaps)"] = {"calls": None, "ms": round(step_ms - on_compute, 3)}
        return dict(sorted(out.items(), key=lambda kv: -kv[1]["ms"]))
