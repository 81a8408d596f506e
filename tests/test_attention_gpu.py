"""Flash attention kernels (forward and backward, with RoPE) against the
plain-PyTorch fp32 computation of the same causal attention."""

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA GPU", allow_module_level=True)

from nano_megatron_b200.ops import cuda as KC  # noqa: E402
from nano_megatron_b200.ops import reference as R  # noqa: E402

DEV = torch.device("cuda", 0)


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


@pytest.mark.parametrize("S,b,h", [(64, 1, 1), (128, 2, 2), (512, 1, 4), (1024, 2, 3), (2048, 1, 2)])
def test_flash_attention_fwd_bwd(S, b, h):
    torch.manual_seed(S + b + h)
    d = 128
    cos, sin = R.rope_cache(S, d, 10000.0, DEV)
    qkv = torch.randn(S * b, 3 * h * d, device=DEV).bfloat16()
    o, saved = KC.attention(qkv, b, h, d, cos, sin)
    o_ref, saved_ref = R.attention(qkv.float(), b, h, d, cos, sin)
    assert _rel(o, o_ref) < 1.5e-2, _rel(o, o_ref)
    do = torch.randn(S * b, h * d, device=DEV).bfloat16()
    dqkv = KC.attention_bwd(do, saved, b, h, d, cos, sin)
    dqkv_ref = R.attention_bwd(do.float(), saved_ref, b, h, d, cos, sin)
    q, k, v = R.split_qkv(dqkv, b, h, d)
    qr, kr, vr = R.split_qkv(dqkv_ref, b, h, d)
    assert _rel(v, vr) < 2e-2, _rel(v, vr)
    assert _rel(k, kr) < 3e-2, _rel(k, kr)
    assert _rel(q, qr) < 3e-2, _rel(q, qr)


def test_attention_leaves_input_untouched():
    S, b, h, d = 128, 1, 2, 128
    cos, sin = R.rope_cache(S, d, 10000.0, DEV)
    qkv = torch.randn(S * b, 3 * h * d, device=DEV).bfloat16()
    before = qkv.clone()
    KC.attention(qkv, b, h, d, cos, sin)
    assert torch.equal(qkv, before)


def test_lse_is_log_sum_exp_of_scaled_scores():
    torch.manual_seed(0)
    S, b, h, d = 128, 1, 1, 128
    qkv = torch.randn(S * b, 3 * h * d, device=DEV).bfloat16()
    from nano_megatron_b200 import _C
    o, lse = _C.flash_attn_fwd(qkv.contiguous(), b, h, d)
    q, k, _ = R.split_qkv(qkv.float(), b, h, d)
    s = (q[:, 0, 0] @ k[:, 0, 0].t()) / d ** 0.5
    s = s.masked_fill(torch.triu(torch.ones(S, S, device=DEV, dtype=torch.bool), 1), float("-inf"))
    torch.testing.assert_close(lse[0], torch.logsumexp(s, -1), rtol=1e-3, atol=1e-3)


@pytest.mark.parametrize("S,b,h,amp", [(128, 1, 1, 1.0), (384, 1, 2, 1.0), (1024, 2, 2, 1.0), (2048, 1, 3, 1.0),
                                       (640, 2, 1, 6.0), (1024, 1, 2, 12.0)])
def test_tcgen05_forward_matches_mma_sync_forward(S, b, h, amp):
    """The tcgen05 forward and the mma.sync forward agree (output and lse).

    Odd tile counts (384, 640) leave the second query tile of a CTA empty;
    large amplitudes make row maxima jump across key blocks, which exercises
    the rescaling of the output accumulator."""
    from nano_megatron_b200 import _C
    torch.manual_seed(S * h)
    qkv = (torch.randn(S * b, 3 * h * 128, device=DEV) * amp).bfloat16()
    o1, l1 = _C.flash_attn_fwd(qkv, b, h, 128)
    o2, l2 = _C.flash_attn_fwd_tc(qkv, b, h, 128, KC.status_word(DEV))
    KC.check_status(DEV)
    assert _rel(o2, o1) < 1e-2, _rel(o2, o1)
    torch.testing.assert_close(l2, l1, rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("S,b,h", [(128, 1, 1), (512, 2, 2), (2048, 1, 3)])
def test_tcgen05_backward_matches_mma_sync_backward(S, b, h):
    """The tcgen05 backward (dK/dV + dQ kernels) and the mma.sync backward agree."""
    from nano_megatron_b200 import _C
    torch.manual_seed(S + h)
    qkv = torch.randn(S * b, 3 * h * 128, device=DEV).bfloat16()
    o, lse = _C.flash_attn_fwd(qkv, b, h, 128)
    do = torch.randn(S * b, h * 128, device=DEV).bfloat16()
    d1 = _C.flash_attn_bwd(do, qkv, o, lse, b, h, 128)
    d2 = _C.flash_attn_bwd_tc(do, qkv, o, lse, b, h, 128, KC.status_word(DEV))
    KC.check_status(DEV)
    for i, name in enumerate("qkv"):
        a_ = d1.view(S * b, 3, -1)[:, i]
        b_ = d2.view(S * b, 3, -1)[:, i]
        assert _rel(b_, a_) < 2e-2, (name, _rel(b_, a_))


@pytest.mark.parametrize("S,d", [(256, 32), (256, 64), (100, 128), (72, 128)])
def test_attention_other_head_sizes(S, d):
    """bf16 attention the flash kernels do not cover (head size other than 128,
    or a length that is not a multiple of 64) runs the exact materialized path
    and matches the fp32 reference, forward and backward."""
    torch.manual_seed(d + S)
    b, h = 2, 3
    cos, sin = R.rope_cache(S, d, 10000.0, DEV)
    qkv = torch.randn(S * b, 3 * h * d, device=DEV).bfloat16()
    o, saved = KC.attention(qkv, b, h, d, cos, sin)
    o_ref, saved_ref = R.attention(qkv.float(), b, h, d, cos, sin)
    assert o.dtype == torch.bfloat16 and _rel(o, o_ref) < 1e-2, _rel(o, o_ref)
    do = torch.randn(S * b, h * d, device=DEV).bfloat16()
    dqkv = KC.attention_bwd(do, saved, b, h, d, cos, sin)
    dqkv_ref = R.attention_bwd(do.float(), saved_ref, b, h, d, cos, sin)
    assert dqkv.dtype == torch.bfloat16 and dqkv.shape == qkv.shape
    assert _rel(dqkv, dqkv_ref) < 1e-2, _rel(dqkv, dqkv_ref)
