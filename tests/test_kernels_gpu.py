"""sm_100a kernels against plain-PyTorch fp32 references of the same op.

Each test builds inputs on the GPU, runs our kernel through the op layer and
compares with the fp32 torch computation of the same math (inputs rounded to
the kernel's storage dtype first). Shapes include partial tiles.
"""

import math

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


# shapes with M >= 2048, N >= 4096, K >= 2048 run the CTA-pair kernel (ragged ones too)
PAIR_SHAPES = [(2048, 4096, 2048), (2304, 4360, 2112)]


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (512, 768, 1024), (300, 264, 200), (2048, 3072, 4096),
                                   (8, 8, 8), (1000, 1032, 72)] + PAIR_SHAPES)
def test_gemm_nn(M, N, K):
    torch.manual_seed(0)
    a = torch.randn(M, K, device=DEV).bfloat16()
    b = torch.randn(K, N, device=DEV).bfloat16()
    got = KC.mm_nn(a, b)
    ref = a.float() @ b.float()
    assert got.shape == (M, N) and got.dtype == torch.bfloat16
    assert _rel(got, ref) < 5e-3, _rel(got, ref)


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (512, 768, 1024), (300, 264, 200), (4096, 4096, 1024)]
                         + PAIR_SHAPES)
def test_gemm_nt(M, N, K):
    torch.manual_seed(1)
    a = torch.randn(M, K, device=DEV).bfloat16()
    b = torch.randn(N, K, device=DEV).bfloat16()
    got = KC.mm_nt(a, b)
    ref = a.float() @ b.float().t()
    assert _rel(got, ref) < 5e-3


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (512, 768, 1024), (264, 392, 200), (4096, 1024, 2048),
                                   (8192, 1024, 1024), (8192, 4096, 1024), (6000, 392, 264),
                                   (2048, 4096, 2048), (2112, 4360, 2304), (8192, 4096, 2048)])
def test_gemm_tn_accumulate(M, N, K):
    """out[K,N] += a[M,K]^T b[M,N] in fp32 (weight-gradient accumulation). The
    last three shapes have few output tiles and a long reduction, so the kernel
    splits K into pieces whose partial tiles are summed by the reduce-add."""
    torch.manual_seed(2)
    a = torch.randn(M, K, device=DEV).bfloat16()
    b = torch.randn(M, N, device=DEV).bfloat16()
    out = torch.randn(K, N, device=DEV)
    start = out.clone()
    KC.mm_tn_acc(a, b, out)
    ref = start + a.float().t() @ b.float()
    assert _rel(out, ref) < 1e-5 * math.sqrt(M) + 1e-6
    KC.mm_tn_acc(a, b, out)  # accumulates again
    assert _rel(out, ref + a.float().t() @ b.float()) < 1e-4


def test_gemm_strided_column_slice_accumulate():
    """Accumulating into a column slice of a wider fp32 buffer (fused q|k|v grads)."""
    torch.manual_seed(3)
    a = torch.randn(256, 128, device=DEV).bfloat16()
    b = torch.randn(256, 64, device=DEV).bfloat16()
    big = torch.zeros(128, 192, device=DEV)
    KC.mm_tn_acc(a, b, big[:, 64:128])
    ref = a.float().t() @ b.float()
    assert _rel(big[:, 64:128], ref) < 1e-5
    assert big[:, :64].abs().max() == 0 and big[:, 128:].abs().max() == 0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("rows,cols", [(1000, 256), (4096, 4096), (77, 2560), (300, 8192), (64, 12288)])
def test_rmsnorm(dtype, rows, cols):
    torch.manual_seed(4)
    x = torch.randn(rows, cols, device=DEV).to(dtype)
    w = torch.rand(cols, device=DEV) + 0.5
    y, rstd = KC.rmsnorm(x, w, 1e-6)
    yr, rr = R.rmsnorm(x, w, 1e-6)
    tol = 1e-2 if dtype == torch.bfloat16 else 1e-5
    assert _rel(y, yr) < tol and _rel(rstd, rr) < 1e-5
    if cols > 8192:  # the backward kernel takes rows of up to 8192 columns
        return
    dy = torch.randn_like(x)
    wg = torch.zeros(cols, device=DEV)
    dx, _ = KC.rmsnorm_bwd(dy, x, w, rstd, wg)
    wr = torch.zeros(cols, device=DEV)
    dxr, _ = R.rmsnorm_bwd(dy, x, w, rr, wr)
    assert _rel(dx, dxr) < tol and _rel(wg, wr) < (1e-2 if dtype == torch.bfloat16 else 1e-5)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("rows,cols", [(2048, 4096), (77, 2560)])
def test_add_rmsnorm_and_residual_gradient(dtype, rows, cols):
    """Residual add fused with the norm (forward), and the norm backward with
    the residual-stream gradient added to dx, against the unfused reference."""
    torch.manual_seed(6)
    x = torch.randn(rows, cols, device=DEV).to(dtype)
    a = torch.randn(rows, cols, device=DEV).to(dtype)
    w = torch.rand(cols, device=DEV) + 0.5
    s, y, rstd = KC.add_rmsnorm(x, a, w, 1e-6)
    assert torch.equal(s, x + a)  # the same rounding as a separate add
    yr, rr = R.rmsnorm(x + a, w, 1e-6)
    tol = 1e-2 if dtype == torch.bfloat16 else 1e-5
    assert _rel(y, yr) < tol and _rel(rstd, rr) < 1e-5
    dy, ds = torch.randn_like(x), torch.randn_like(x)
    wg, wr = torch.zeros(cols, device=DEV), torch.zeros(cols, device=DEV)
    dx, _ = KC.rmsnorm_bwd(dy, s, w, rstd, wg, dres=ds)
    dxr, _ = R.rmsnorm_bwd(dy, s, w, rr, wr, dres=ds)
    assert _rel(dx, dxr) < tol and _rel(wg, wr) < tol


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_swiglu(dtype):
    torch.manual_seed(5)
    gu = torch.randn(333, 2 * 344, device=DEV).to(dtype)
    a = KC.swiglu(gu)
    assert _rel(a, R.swiglu(gu.float())) < (1e-2 if dtype == torch.bfloat16 else 1e-6)
    da = torch.randn(333, 344, device=DEV).to(dtype)
    d = KC.swiglu_bwd(da, gu)
    assert _rel(d, R.swiglu_bwd(da.float(), gu.float())) < (1e-2 if dtype == torch.bfloat16 else 1e-5)


@pytest.mark.parametrize("M,K,F,save", [(1024, 512, 1024, True), (384, 256, 704, True),
                                         (256, 128, 344, False), (2048, 1024, 3584, False),
                                         (2048, 2048, 2048, True), (2304, 2112, 2184, True)])
def test_swiglu_gemm_epilogue(M, K, F, save):
    """One GEMM with the SwiGLU epilogue against the GEMM + SwiGLU kernels
    (same rounding points) and against fp32 torch; ragged feature counts
    exercise the partial last tile of each half."""
    torch.manual_seed(M + F)
    x = (torch.randn(M, K, device=DEV) * 0.5).bfloat16()
    w = (torch.randn(K, 2 * F, device=DEV) / K ** 0.5).bfloat16()
    a, gu = KC.mm_swiglu(x, w, save_gu=save)
    gu_ref = KC.mm_nn(x, w)
    a_ref = KC.swiglu(gu_ref)
    assert (gu is None) == (not save)
    if save:
        assert _rel(gu, gu_ref) < 1e-4, _rel(gu, gu_ref)
    assert _rel(a, a_ref) < 1e-4, _rel(a, a_ref)
    g32 = x.float() @ w.float()
    want = torch.nn.functional.silu(g32[:, :F]) * g32[:, F:]
    assert _rel(a, want) < 1e-2


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_rope_roundtrip(dtype):
    from nano_megatron_b200 import _C
    torch.manual_seed(6)
    S, b, h, d = 64, 2, 4, 128
    cos, sin = R.rope_cache(S, d, 500000.0, DEV)
    qkv = torch.randn(S * b, 3 * h * d, device=DEV).to(dtype)
    x = qkv.clone()
    _C.rope_inplace(x, cos, sin, b, h, d, 1.0)
    q, k, v = R.split_qkv(qkv.float(), b, h, d)
    ref = torch.stack([R._rotate(q, cos, sin, 1.0), R._rotate(k, cos, sin, 1.0), v], dim=2).reshape(qkv.shape)
    assert _rel(x, ref) < (1e-2 if dtype == torch.bfloat16 else 1e-6)
    _C.rope_inplace(x, cos, sin, b, h, d, -1.0)
    assert _rel(x, qkv) < (2e-2 if dtype == torch.bfloat16 else 1e-6)


def test_embedding_and_bounds_flag():
    torch.manual_seed(7)
    V, H = 1000, 256
    w = torch.randn(V // 2, H, device=DEV)
    ids = torch.randint(0, V, (517,), device=DEV)
    out = KC.embedding(ids, w, 500, 1000, torch.bfloat16, V)
    ref = R.embedding(ids, w, 500, 1000)
    assert _rel(out, ref) < 1e-2
    dy = torch.randn(517, H, device=DEV)
    g = torch.zeros_like(w)
    KC.embedding_bwd(dy, ids, g, 500, 1000)
    gr = torch.zeros_like(w)
    R.embedding_bwd(dy, ids, gr, 500, 1000)
    assert _rel(g, gr) < 1e-6
    KC.check_status(DEV)
    bad = ids.clone()
    bad[3] = V + 5
    KC.embedding(bad, w, 500, 1000, torch.bfloat16, V)
    with pytest.raises(RuntimeError, match="vocabulary"):
        KC.check_status(DEV)


def test_cross_entropy_stats_and_grad():
    torch.manual_seed(8)
    T, V, start = 300, 1032, 1032
    logits = (torch.randn(T, V, device=DEV) * 3).bfloat16()
    target = torch.randint(0, 3 * V, (T,), device=DEV)
    mx, se, tl, owned = KC.ce_local_stats(logits, target, start, start + V)
    rm, rs, rt, ro = R.ce_local_stats(logits.float(), target, start, start + V)
    assert _rel(mx, rm) < 1e-6 and _rel(se, rs) < 1e-5 and _rel(tl, rt) < 1e-6
    gm, gs = rm + 0.5, rs * 2
    scale = torch.tensor(0.37, device=DEV)
    d = KC.ce_grad(logits, target, start, gm, gs, scale, torch.bfloat16)
    dr = R.ce_grad(logits.float(), target, start, gm, gs, scale.expand(T), torch.float32)
    assert _rel(d, dr) < 1e-2


@pytest.mark.parametrize("rows,hidden,vocab,start", [(256, 512, 1000, 0), (384, 256, 4096, 0), (128, 128, 520, 480)])
def test_fused_lm_head_cross_entropy(rows, hidden, vocab, start):
    """GEMM + CE-statistics epilogue + merge (one GPU) against torch on the same bf16 logits."""
    import torch.nn.functional as F
    from nano_megatron_b200.ops import fused_tp
    from nano_megatron_b200.parallel.context import ParallelContext
    torch.manual_seed(rows + vocab)
    x = torch.randn(rows, hidden, device=DEV).bfloat16()
    w = (torch.randn(vocab, hidden, device=DEV) * 0.1).bfloat16()
    labels = torch.randint(0, start + vocab + 40, (rows,), device=DEV)  # some outside the shard
    loss, logits, gm, gs, X = fused_tp.lm_head_cross_entropy(x, w, labels, start, start + vocab,
                                                             ParallelContext.single(), gather=False)
    KC.check_status(DEV)
    ref_logits = x.float() @ w.float().t()
    assert _rel(logits, ref_logits) < 5e-3
    lf = logits.float()
    rm = lf.max(dim=1).values
    rs = torch.exp(lf - rm[:, None]).sum(dim=1)
    local = labels - start
    owned = (local >= 0) & (local < vocab)
    rt = torch.where(owned, lf.gather(1, local.clamp(0, vocab - 1)[:, None])[:, 0], torch.zeros_like(rm))
    assert torch.equal(gm, rm)
    assert _rel(gs, rs) < 1e-5
    assert (loss - (rs.log() + rm - rt)).abs().max().item() < 1e-4
    if start == 0 and bool(owned.all()):
        assert (loss - F.cross_entropy(lf, labels, reduction="none")).abs().max().item() < 1e-4
    # backward: (softmax - onehot) * g/n, in place in the logits buffer
    g = torch.tensor(0.7, device=DEV)
    saved = logits.clone()
    d = KC.lm_head_ce_grad(X, w, labels, start, (logits, gm, gs), g / rows, inplace=True)
    assert d.data_ptr() == logits.data_ptr()
    p = torch.exp(saved.float() - gm[:, None]) / gs[:, None]
    p[owned, local[owned]] -= 1.0
    assert _rel(d, p * (0.7 / rows)) < 1e-2


def test_adamw_flat_matches_reference():
    torch.manual_seed(9)
    n = 4096 + 64
    p = torch.randn(n, device=DEV)
    g = torch.randn(n, device=DEV)
    m = torch.zeros(n, device=DEV)
    v = torch.zeros(n, device=DEV)
    comp = torch.empty(n, device=DEV, dtype=torch.bfloat16)
    pr, mr, vr = p.clone(), m.clone(), v.clone()
    for step in (1, 2, 3):
        KC.adamw_flat(p, g, m, v, comp, torch.tensor(0.5, device=DEV), lr=1e-2, beta1=0.9, beta2=0.999,
                     eps=1e-8, weight_decay=0.01, step=step)
        R.adamw_(pr, g * 0.5, mr, vr, lr=1e-2, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.01, step=step)
    assert _rel(p, pr) < 1e-6 and _rel(m, mr) < 1e-6 and _rel(v, vr) < 1e-6
    assert torch.equal(comp, p.bfloat16())


def test_weighted_sq_norm():
    torch.manual_seed(10)
    ts = [torch.randn(n, device=DEV) for n in (100, 5000, (1 << 24) + 17)]
    ws = [1.0, 0.5, 0.25]
    got = KC.weighted_sq_norm(ts, ws)
    ref = sum(w * t.double().pow(2).sum() for t, w in zip(ts, ws))
    assert abs(got.item() - ref.item()) / ref.item() < 1e-6


def test_bounded_peer_wait_times_out_into_the_status_word():
    """A cross-GPU flag wait whose flag nothing sets gives up after its bound,
    records "cross-GPU flag wait timed out" in the status word and returns; the
    context stays usable. Both "ranks" of the DP averaging kernel here are
    buffers of this one GPU, and the second never announces itself."""
    import time
    from nano_megatron_b200 import _C
    n = 1024
    bufs = [torch.ones(n, device=DEV), torch.ones(n, device=DEV)]
    flags = [torch.zeros(_C.dp_flag_bytes() // 4, dtype=torch.int32, device=DEV) for _ in range(2)]
    KC.check_status(DEV)
    t0 = time.monotonic()
    _C.dp_allreduce([b.data_ptr() for b in bufs], [f.data_ptr() for f in flags], 0, 0, n, 1,
                    KC.status_word(DEV), 0.25)
    torch.cuda.synchronize()
    waited = time.monotonic() - t0
    assert 0.2 < waited < 30.0, waited
    with pytest.raises(RuntimeError, match="cross-GPU flag wait timed out"):
        KC.check_status(DEV)
    assert torch.equal(bufs[0], torch.ones(n, device=DEV))  # gave up before touching data
    KC.check_status(DEV)  # cleared; the context still works
    assert float((bufs[0] + 1).sum()) == 2.0 * n


def test_tcgen05_mma_cycle_probe():
    """The one-SM tcgen05.mma cycle probe runs and orders the shapes sensibly:
    a wider product never takes fewer cycles, and N=128 is near its 64-cycle
    arithmetic time."""
    from nano_megatron_b200 import _C
    err = KC.status_word(DEV)
    for ts in (False, True):
        c64, c128, c256 = (_C.mma_cycles(n, ts, 1024, err) for n in (64, 128, 256))
        assert 32 <= c64 <= c128 <= c256, (ts, c64, c128, c256)
        assert 60 <= c128 <= 90, (ts, c128)
    KC.check_status(DEV)
