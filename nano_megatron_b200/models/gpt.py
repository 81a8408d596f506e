"""One pipeline stage of a decoder-only GPT: RMSNorm, RoPE, causal MHA, SwiGLU.

A stage builds only its own layers: the embedding on the first stage, the final
norm and LM head on the last. A non-first stage takes a hidden state, a
non-last stage returns one, so the pipeline schedule stays outside the model.

Layout: inside a stage the residual stream is sequence-first and token-major,
``[s*b, H]`` (``s = S/tp`` under sequence parallelism), so a sequence shard is
a contiguous row range. At the stage's edges everything is batch-first as in
the reference: token ids and labels ``[b, S]``, hidden states ``[b, s, H]``
(for one sequence per microbatch the two layouts are the same memory).

Attention uses one fused ``[H, 3H/tp]`` QKV weight and the MLP one fused
``[H, 2F/tp]`` gate|up weight; the separate ``q``/``k``/``v`` and ``gate``/``up``
Parameters (reference state-dict keys and shapes) are column views of them.

Parity: ``nano_megatron/model.py:35-281``.
"""

from __future__ import annotations

import contextlib

import torch
import torch.nn as nn
from torch.utils.checkpoint import checkpoint

from ..parallel.context import ParallelContext
from .. import ops
from .buffers import FlatBuffers
from .config import GPTConfig, divide
from .functional import (WeightRef, add_rms_norm, causal_attention, column_linear, discarded_forward,
                         gate_up_swiglu, gate_up_swiglu_supported, lm_head_cross_entropy,
                         lm_head_logits, row_linear, swiglu)
from .layers import (ColumnParallelLinear, RMSNorm, RowParallelLinear,
                     VocabParallelEmbedding)


def build_rope_cache(seq_len, head_dim, device, base=10000.0):
    """fp32 ``(cos, sin)`` tables ``[seq_len, head_dim/2]``; ``base`` is RoPE theta."""
    return ops.rope_cache(seq_len, head_dim, base, device)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """NeoX rotary embedding of ``x [..., s, head_dim]`` (positions on dim -2).

    The two halves ``(a, b)`` of the last dimension become
    ``(a cos - b sin, b cos + a sin)`` with the first ``s`` rows of the
    ``[seq, head_dim/2]`` tables of :func:`build_rope_cache`; the result has the
    promoted dtype of ``x`` and the tables. The model itself rotates q/k inside
    its attention op (and un-rotates the gradient inside the backward kernels);
    this is the standalone form for callers that hold separate q/k tensors
    (reference ``nano_megatron/model.py:84-89``, ``[b, heads, s, head_dim]``).
    """
    s, half = x.shape[-2], x.shape[-1] // 2
    dt = torch.promote_types(x.dtype, cos.dtype)
    c = cos[:s].to(dt)
    sn = sin[:s].to(dt)
    a = x[..., :half].to(dt)
    b = x[..., half:].to(dt)
    out = torch.empty(x.shape, dtype=dt, device=x.device)
    torch.addcmul(a * c, b, sn, value=-1.0, out=out[..., :half])
    torch.addcmul(b * c, a, sn, out=out[..., half:])
    return out


def cuda_shape_problems(config: GPTConfig, ctx: ParallelContext) -> list[str]:
    """What keeps ``config`` at this layout off the CUDA kernels, as messages
    (empty when it fits): per-rank GEMM widths must be multiples of 8 (16-byte
    rows for TMA), the RMSNorm kernels take up to 8192 columns, and the RoPE
    kernel rotates 8-element chunks of each half of a head. Attention itself
    takes any head size and length (sizes the flash kernels do not cover run
    the exact materialized path)."""
    problems = []
    t = ctx.tp_size
    if config.n_embd % 8 or (config.n_embd // t) % 8:
        problems.append(f"n_embd {config.n_embd} (per rank {config.n_embd // t}) must be a multiple of 8")
    if config.n_embd > 8192:
        problems.append(f"n_embd {config.n_embd} is above the RMSNorm kernels' 8192 columns")
    if (config.ffn_size // t) % 8:
        problems.append(f"the SwiGLU width per rank ({config.ffn_size // t}) must be a multiple of 8")
    if (config.vocab_size // t) % 8:
        pad = -(-config.vocab_size // (8 * t)) * 8 * t
        problems.append(f"the vocabulary shard per rank ({config.vocab_size // t}) must be a multiple of 8: "
                        f"pad vocab_size to {pad}")
    if config.head_dim % 16:
        problems.append(f"head_dim {config.head_dim} must be a multiple of 16 for the RoPE kernel")
    return problems


def layers_for_stage(n_layer: int, pp_size: int, pp_rank: int) -> tuple[int, int]:
    """Contiguous, equal split of the layers over the pipeline stages."""
    per_stage = divide(n_layer, pp_size)
    return pp_rank * per_stage, (pp_rank + 1) * per_stage


def _fused_ref(buffers: FlatBuffers, params) -> WeightRef:
    region = buffers.region_of(params[0])
    return WeightRef(region.data_block, params, region.compute_block, region.grad_block)


def _column_group(x, linears, buffers: FlatBuffers | None, ctx: ParallelContext, mode: str,
                  dtype: torch.dtype):
    """``x @ [W_1 | W_2 | ...]`` for column-parallel layers that share an input:
    one GEMM over the fused region inside a model; each layer on its own (one
    GEMM and one input collective each) for modules built outside one."""
    weights = tuple(lin.weight for lin in linears)
    if buffers is not None:
        return column_linear(x, _fused_ref(buffers, weights), ctx, mode, dtype)
    return torch.cat([column_linear(x, WeightRef.of(w), ctx, mode, dtype) for w in weights], dim=1)


def _compute_dtype(x: torch.Tensor) -> torch.dtype:
    """The dtype a module called in the reference's form computes in: the
    autocast dtype when autocast is on for ``x``'s device, else ``x``'s."""
    kind = x.device.type
    if torch.is_autocast_enabled(kind):
        return torch.get_autocast_dtype(kind)
    return x.dtype if x.is_floating_point() else torch.float32


def _batch_first_call(fn, x: torch.Tensor, *args):
    """Run ``fn(rows, batch, *args)`` on ``x [b, s, H]`` as sequence-major rows
    ``[s*b, H]`` and return its rows ``[s'*b, N]`` as ``[b, s', N]``."""
    b = x.shape[0]
    rows = x.transpose(0, 1).reshape(-1, x.shape[-1])
    y = fn(rows, b, *args)
    return y.view(-1, b, y.shape[-1]).transpose(0, 1).contiguous()


class ParallelAttention(nn.Module):
    """MHA sharded over heads; one fused QKV GEMM, one row-parallel output GEMM.

    Parity: ``nano_megatron/model.py:92-128``. ``forward(x, cos, sin)`` is the
    reference's call (batch-first ``[b, s, H]``); the model calls
    ``forward(rows, cos, sin, batch, dtype)`` on its sequence-major token rows
    (:meth:`forward_rows`), so module hooks see both.
    """

    def __init__(self, config: GPTConfig, ctx: ParallelContext):
        super().__init__()
        self.ctx = ctx
        self.n_head_local = divide(config.n_head, ctx.tp_size)
        self.head_dim = config.head_dim
        self.sequence_parallel = config.sequence_parallel
        std = config.init_std
        h = config.n_embd
        self.q = ColumnParallelLinear(h, h, ctx, bias=False, init_std=std)
        self.k = ColumnParallelLinear(h, h, ctx, bias=False, init_std=std)
        self.v = ColumnParallelLinear(h, h, ctx, bias=False, init_std=std)
        self.proj = RowParallelLinear(h, h, ctx, bias=False, init_std=std)
        self.flat_buffers: FlatBuffers | None = None

    def fused_groups(self, prefix: str):
        return [[f"{prefix}q.weight", f"{prefix}k.weight", f"{prefix}v.weight"]]

    def forward(self, x, cos, sin, *rows_form):
        """``x [b, s, H]`` (``s = S/tp`` under sequence parallelism) -> ``[b, s, H]``;
        with ``rows_form = (batch, dtype)``, :meth:`forward_rows`."""
        if rows_form:
            return self.forward_rows(x, rows_form[0], cos, sin, rows_form[1])
        return _batch_first_call(self.forward_rows, x, cos, sin, _compute_dtype(x))

    def forward_rows(self, x, batch, cos, sin, dtype):
        """``x [s*b, H]`` (already normed, sequence-major rows) -> ``[s*b, H]``."""
        sp = self.sequence_parallel and self.ctx.tp_size > 1
        qkv = _column_group(x, (self.q, self.k, self.v), self.flat_buffers, self.ctx,
                            "ag" if sp else "f", dtype)
        o = causal_attention(qkv, batch, self.n_head_local, self.head_dim, cos, sin)
        return row_linear(o, WeightRef.of(self.proj.weight), self.ctx, "rs" if sp else "g", dtype)


class ParallelMLP(nn.Module):
    """SwiGLU: fused gate|up column-parallel GEMM, row-parallel down GEMM.

    Parity: ``nano_megatron/model.py:131-153`` (with a configurable width;
    the reference's is ``4 * n_embd``). ``forward(x)`` is the reference's call
    (batch-first ``[b, s, H]``); the model calls ``forward(rows, dtype)``
    (:meth:`forward_rows`).
    """

    def __init__(self, config: GPTConfig, ctx: ParallelContext):
        super().__init__()
        self.ctx = ctx
        self.sequence_parallel = config.sequence_parallel
        h, f, std = config.n_embd, config.ffn_size, config.init_std
        self.gate = ColumnParallelLinear(h, f, ctx, bias=False, init_std=std)
        self.up = ColumnParallelLinear(h, f, ctx, bias=False, init_std=std)
        self.down = RowParallelLinear(f, h, ctx, bias=False, init_std=std)
        self.flat_buffers: FlatBuffers | None = None

    def fused_groups(self, prefix: str):
        return [[f"{prefix}gate.weight", f"{prefix}up.weight"]]

    def forward(self, x, *rows_form):
        """``x [b, s, H]`` (``s = S/tp`` under sequence parallelism) -> ``[b, s, H]``;
        with ``rows_form = (dtype,)``, :meth:`forward_rows`."""
        if rows_form:
            return self.forward_rows(x, rows_form[0])
        return _batch_first_call(lambda rows, _b, dtype: self.forward_rows(rows, dtype), x,
                                 _compute_dtype(x))

    def forward_rows(self, x, dtype):
        """``x [s*b, H]`` (sequence-major rows) -> ``[s*b, H]``."""
        sp = self.sequence_parallel and self.ctx.tp_size > 1
        mode = "ag" if sp else "f"
        if (self.flat_buffers is not None and dtype == torch.bfloat16
                and gate_up_swiglu_supported(x, self.gate.weight.shape[1], self.ctx, mode)):
            gu_ref = _fused_ref(self.flat_buffers, (self.gate.weight, self.up.weight))
            a = gate_up_swiglu(x, gu_ref, self.ctx, mode, dtype)
        else:
            a = swiglu(_column_group(x, (self.gate, self.up), self.flat_buffers, self.ctx, mode, dtype))
        return row_linear(a, WeightRef.of(self.down.weight), self.ctx, "rs" if sp else "g", dtype)


class TransformerLayer(nn.Module):
    """Pre-norm block: ``x + attn(norm(x))`` then ``x + mlp(norm(x))``.

    Parity: ``nano_megatron/model.py:156-166``. ``forward(x, cos, sin)`` is the
    reference's call (batch-first ``[b, s, H]``); the model calls
    ``forward(rows, cos, sin, batch, dtype)`` (:meth:`forward_rows`), where the
    first residual add and the MLP's norm are one kernel.
    """

    def __init__(self, config: GPTConfig, ctx: ParallelContext):
        super().__init__()
        self.attn_norm = RMSNorm(config.n_embd)
        self.attn = ParallelAttention(config, ctx)
        self.mlp_norm = RMSNorm(config.n_embd)
        self.mlp = ParallelMLP(config, ctx)

    def forward(self, x, cos, sin, *rows_form):
        """``x [b, s, H]`` -> ``[b, s, H]``; with ``rows_form = (batch, dtype)``,
        :meth:`forward_rows`."""
        if rows_form:
            return self.forward_rows(x, rows_form[0], cos, sin, rows_form[1])
        return _batch_first_call(self.forward_rows, x, cos, sin, _compute_dtype(x))

    def forward_rows(self, x, batch, cos, sin, dtype):
        """``x [s*b, H]`` (sequence-major rows) -> ``[s*b, H]``."""
        a = self.attn(self.attn_norm(x), cos, sin, batch, dtype)
        # residual add and the MLP's norm in one pass
        x, h = add_rms_norm(x, a.reshape(-1, a.shape[-1]), self.mlp_norm.weight, self.mlp_norm.eps)
        return x + self.mlp(h, dtype)


class ParallelLMHead(nn.Module):
    """Vocab-sharded output projection ``[V/tp, H]`` (the embedding's layout, so they can tie).

    Parity: ``nano_megatron/model.py:169-192``. The model's last stage uses the
    fused LM head + cross entropy instead of :meth:`forward` when it has labels.
    """

    def __init__(self, config: GPTConfig, ctx: ParallelContext):
        super().__init__()
        self.ctx = ctx
        per_partition = divide(config.vocab_size, ctx.tp_size)
        self.weight = nn.Parameter(torch.empty(per_partition, config.n_embd))
        self.weight.tensor_parallel_sharded = True
        self.sequence_parallel = config.sequence_parallel
        nn.init.normal_(self.weight, std=config.init_std)

    def forward(self, x):
        """``x [b, s, H]`` -> vocab-sharded logits ``[b, S, V/tp]``: the sequence
        is all-gathered first under sequence parallelism, else f applies."""
        mode = "ag" if self.sequence_parallel and self.ctx.tp_size > 1 else "f"
        return _batch_first_call(
            lambda rows, _b, dtype: lm_head_logits(rows, WeightRef.of(self.weight), self.ctx, mode, dtype),
            x, _compute_dtype(x))


class GPT(nn.Module):
    """This rank's pipeline stage of the model.

    Parity: ``nano_megatron/model.py:200-281`` (size checks, stage split, tie
    at one stage, RoPE tables as non-persistent buffers, whole-block
    recompute in training). Differences: parameters are views of flat fp32
    buffers (``flat_buffers``), and compute is in ``config.activation_dtype``
    without autocast.
    """

    def __init__(self, config: GPTConfig, ctx: ParallelContext | None = None,
                 device: torch.device | str | None = None):
        super().__init__()
        ctx = ctx or ParallelContext.single()
        self.config = config
        self.ctx = ctx
        self.first_stage = ctx.is_first_stage
        self.last_stage = ctx.is_last_stage
        config.activation_dtype  # validate before allocating parameters
        for name in ("vocab_size", "n_layer", "n_head", "n_embd", "seq_len"):
            if getattr(config, name) <= 0:
                raise ValueError(f"{name} must be positive")
        if config.ffn_hidden_size is not None and config.ffn_hidden_size <= 0:
            raise ValueError("ffn_hidden_size must be positive")
        divide(config.n_layer, ctx.pp_size)
        divide(config.n_embd, ctx.tp_size)
        divide(config.n_head, ctx.tp_size)
        divide(config.vocab_size, ctx.tp_size)
        divide(config.ffn_size, ctx.tp_size)
        if config.head_dim % 2:
            raise ValueError("RoPE requires an even attention head dimension")
        if config.sequence_parallel:
            divide(config.seq_len, ctx.tp_size)

        with torch.device(device) if device is not None else contextlib.nullcontext():
            start, end = layers_for_stage(config.n_layer, ctx.pp_size, ctx.pp_rank)
            self.layers = nn.ModuleList([TransformerLayer(config, ctx) for _ in range(start, end)])
            if self.first_stage:
                self.embedding = VocabParallelEmbedding(config.vocab_size, config.n_embd, ctx,
                                                        init_std=config.init_std)
            if self.last_stage:
                self.final_norm = RMSNorm(config.n_embd)
                self.lm_head = ParallelLMHead(config, ctx)
            # One stage: the tie is one shared tensor. Split across stages the
            # two copies are kept equal by the tied-group broadcast/all-reduce.
            if config.tie_word_embeddings and self.first_stage and self.last_stage:
                self.lm_head.weight = self.embedding.weight
            cos, sin = build_rope_cache(config.seq_len, config.head_dim, None, config.rope_theta)
        self.register_buffer("rope_cos", cos, persistent=False)
        self.register_buffer("rope_sin", sin, persistent=False)
        self.flat_buffers: FlatBuffers | None = None
        self._cuda_checked = False
        self._build_buffers()

    # ---------------------------------------------------------- flat buffers
    def _build_buffers(self) -> None:
        groups = []
        for name, module in self.named_modules():
            if hasattr(module, "fused_groups"):
                groups.extend(module.fused_groups(f"{name}." if name else ""))
        compute = self.config.activation_dtype
        on_cuda = next(self.parameters()).is_cuda
        self.flat_buffers = FlatBuffers(self, groups, compute if on_cuda else None)
        for module in self.modules():
            if isinstance(module, (ParallelAttention, ParallelMLP)):
                module.flat_buffers = self.flat_buffers

    def _apply(self, fn, recurse=True):
        # Moving or casting re-creates each parameter separately; rebuild the
        # flat buffers so parameters stay views of one allocation.
        result = super()._apply(fn, recurse)
        if getattr(self, "flat_buffers", None) is not None:
            self._build_buffers()
        return result

    def zero_grad(self, set_to_none: bool = True) -> None:
        """Zero the flat gradient buffer; ``param.grad`` stays a view of it."""
        self.flat_buffers.zero_grad()

    def refresh_compute_copies(self) -> None:
        self.flat_buffers.refresh_compute()

    def load_state_dict(self, state_dict, strict: bool = True, assign: bool = False):
        if assign:
            raise ValueError("assign=True would detach parameters from the flat buffers")
        result = super().load_state_dict(state_dict, strict=strict)
        self.refresh_compute_copies()
        return result

    # --------------------------------------------------------------- forward
    def vocab_range(self) -> tuple[int, int]:
        per = divide(self.config.vocab_size, self.ctx.tp_size)
        return self.ctx.tp_rank * per, (self.ctx.tp_rank + 1) * per

    def _layer_call(self, layer, h, batch, dtype):
        cos, sin = self.rope_cos, self.rope_sin
        if self.config.recompute and self.training:
            calls = [0]

            def run(h, batch, cos, sin, dtype):
                # the first call is the forward whose saved tensors checkpoint
                # drops; the second is the recomputation before backward
                calls[0] += 1
                with discarded_forward(calls[0] == 1):
                    return layer(h, cos, sin, batch, dtype)

            return checkpoint(run, h, batch, cos, sin, dtype, use_reentrant=False)
        return layer(h, cos, sin, batch, dtype)

    def forward(self, x, labels=None):
        """Token ids ``[b, S]`` on the first stage, hidden ``[b, s, H]`` elsewhere.

        Returns the mean loss on the last stage when ``labels [b, S]`` is
        given, the vocab-sharded logits ``[b, S, V/tp]`` when it is not, and
        the hidden state ``[b, s, H]`` on every other stage.
        """
        cfg, ctx = self.config, self.ctx
        dtype = cfg.activation_dtype
        sp = cfg.sequence_parallel and ctx.tp_size > 1
        if x.is_cuda and not self._cuda_checked:
            problems = cuda_shape_problems(cfg, ctx)
            if problems:
                raise ValueError("this configuration does not fit the CUDA kernels: " + "; ".join(problems))
            self._cuda_checked = True
        if self.first_stage:
            batch = x.shape[0]
            ids = x.t().reshape(-1)  # sequence-major token order: 1-D ids are token rows
            h = self.embedding(ids, sequence_parallel=sp, out_dtype=dtype)
        else:
            s_local = cfg.seq_len // ctx.tp_size if sp else cfg.seq_len
            if x.dim() != 3 or x.shape[1] != s_local or x.shape[2] != cfg.n_embd:
                raise ValueError(f"a non-first pipeline stage takes its hidden state batch-first "
                                 f"[batch, {s_local}, {cfg.n_embd}]; got {tuple(x.shape)}")
            batch = x.shape[0]
            h = x.transpose(0, 1).reshape(-1, cfg.n_embd)  # a view for one sequence per microbatch
        if h.dtype != dtype:
            h = h.to(dtype)

        for layer in self.layers:
            h = self._layer_call(layer, h, batch, dtype)

        if not self.last_stage:
            return h.view(-1, batch, cfg.n_embd).transpose(0, 1)

        hn = self.final_norm(h)
        head = WeightRef.of(self.lm_head.weight)
        mode = "ag" if sp else "f"
        if labels is None:
            logits = lm_head_logits(hn, head, ctx, mode, dtype)
            return logits.view(cfg.seq_len, batch, -1).transpose(0, 1)
        start, end = self.vocab_range()
        labels_sf = labels.t().reshape(-1)
        return lm_head_cross_entropy(hn, labels_sf, head, ctx, mode, dtype, start, end)
