// Bindings of the memory-bound kernels (kernels.cu).

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "attention.cuh"
#include "fp32.cuh"
#include "kernels.cuh"

namespace {

int dtype_tag(const at::Tensor& t) {
  if (t.scalar_type() == at::kBFloat16) return 1;
  TORCH_CHECK(t.scalar_type() == at::kFloat, "expected bf16 or fp32, got ", t.scalar_type());
  return 0;
}

void need(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.is_contiguous(), name, " must be a contiguous CUDA tensor");
}

void ok(cudaError_t e, const char* what) { TORCH_CHECK(e == cudaSuccess, what, ": ", cudaGetErrorString(e)); }

cudaStream_t stream() { return at::cuda::getCurrentCUDAStream(); }

int* err_ptr(const c10::optional<at::Tensor>& err) {
  return err.has_value() ? err->data_ptr<int>() : nullptr;
}

void rmsnorm_fwd(const at::Tensor& x, const at::Tensor& w, at::Tensor& y, at::Tensor& rstd, double eps) {
  need(x, "x"); need(w, "w"); need(y, "y"); need(rstd, "rstd");
  TORCH_CHECK(w.scalar_type() == at::kFloat && rstd.scalar_type() == at::kFloat, "w, rstd must be fp32");
  const at::cuda::CUDAGuard g(x.device());
  ok(nmb::rmsnorm_fwd(x.data_ptr(), w.data_ptr<float>(), y.data_ptr(), rstd.data_ptr<float>(), x.size(0), x.size(1),
                      (float)eps, dtype_tag(x), stream()),
     "rmsnorm_fwd");
}

// s = x + a, y = rmsnorm(s) * w in one pass (s, y, x, a of one dtype; w, rstd fp32)
void add_rmsnorm_fwd(const at::Tensor& x, const at::Tensor& a, at::Tensor& s_out, const at::Tensor& w, at::Tensor& y,
                     at::Tensor& rstd, double eps) {
  need(x, "x"); need(a, "a"); need(s_out, "s"); need(w, "w"); need(y, "y"); need(rstd, "rstd");
  TORCH_CHECK(w.scalar_type() == at::kFloat && rstd.scalar_type() == at::kFloat, "w, rstd must be fp32");
  TORCH_CHECK(a.scalar_type() == x.scalar_type() && s_out.scalar_type() == x.scalar_type() &&
                  y.scalar_type() == x.scalar_type() && a.sizes() == x.sizes() && s_out.sizes() == x.sizes(),
              "x, a, s and y must match");
  const at::cuda::CUDAGuard g(x.device());
  ok(nmb::add_rmsnorm_fwd(x.data_ptr(), a.data_ptr(), s_out.data_ptr(), w.data_ptr<float>(), y.data_ptr(),
                          rstd.data_ptr<float>(), x.size(0), x.size(1), (float)eps, dtype_tag(x), stream()),
     "add_rmsnorm_fwd");
}

int64_t rmsnorm_bwd_blocks(int64_t rows, int64_t max_blocks) {
  return nmb::rmsnorm_bwd_blocks((int)rows, (int)max_blocks);
}

// dx = rmsnorm backward of dy (+ dres when given); weight-gradient partials per block
void rmsnorm_bwd(const at::Tensor& dy, const at::Tensor& x, const at::Tensor& w, const at::Tensor& rstd, at::Tensor& dx,
                 at::Tensor& partial, const c10::optional<at::Tensor>& dres) {
  need(dy, "dy"); need(x, "x"); need(w, "w"); need(rstd, "rstd"); need(dx, "dx"); need(partial, "partial");
  TORCH_CHECK(partial.size(0) >= nmb::rmsnorm_bwd_blocks(x.size(0)) && partial.size(1) == x.size(1),
              "partial buffer too small");
  const void* res = nullptr;
  if (dres.has_value()) {
    need(*dres, "dres");
    TORCH_CHECK(dres->scalar_type() == x.scalar_type() && dres->sizes() == x.sizes(), "dres must match x");
    res = dres->data_ptr();
  }
  const at::cuda::CUDAGuard g(x.device());
  ok(nmb::rmsnorm_bwd(dy.data_ptr(), x.data_ptr(), w.data_ptr<float>(), rstd.data_ptr<float>(), dx.data_ptr(),
                      partial.data_ptr<float>(), x.size(0), x.size(1), dtype_tag(x), stream(), res),
     "rmsnorm_bwd");
}

void reduce_rows_add(const at::Tensor& partial, int64_t nrows, at::Tensor& out) {
  need(partial, "partial");
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == at::kFloat && out.stride(-1) == 1, "out must be fp32 CUDA");
  TORCH_CHECK(out.numel() == partial.size(1), "out size mismatch");
  ok(nmb::reduce_rows_add(partial.data_ptr<float>(), out.data_ptr<float>(), (int)nrows, partial.size(1), stream()),
     "reduce_rows_add");
}

void swiglu_fwd(const at::Tensor& gu, at::Tensor& a) {
  need(gu, "gu"); need(a, "a");
  ok(nmb::swiglu_fwd(gu.data_ptr(), a.data_ptr(), gu.size(0), a.size(1), dtype_tag(gu), stream()), "swiglu_fwd");
}

void swiglu_bwd(const at::Tensor& da, const at::Tensor& gu, at::Tensor& dgu) {
  need(da, "da"); need(gu, "gu"); need(dgu, "dgu");
  ok(nmb::swiglu_bwd(da.data_ptr(), gu.data_ptr(), dgu.data_ptr(), gu.size(0), da.size(1), dtype_tag(gu), stream()),
     "swiglu_bwd");
}

void rope_inplace(at::Tensor& qkv, const at::Tensor& cos, const at::Tensor& sin, int64_t batch, int64_t heads,
                  int64_t hd, double sign) {
  need(qkv, "qkv"); need(cos, "cos"); need(sin, "sin");
  TORCH_CHECK(qkv.size(1) == 3 * heads * hd, "qkv width mismatch");
  TORCH_CHECK(cos.size(0) * batch >= qkv.size(0), "rope table shorter than the sequence");
  ok(nmb::rope_inplace(qkv.data_ptr(), cos.data_ptr<float>(), sin.data_ptr<float>(), qkv.size(0), (int)batch,
                       (int)heads, (int)hd, (float)sign, dtype_tag(qkv), stream()),
     "rope_inplace");
}

void embedding_fwd(const at::Tensor& ids, const at::Tensor& w, at::Tensor& out, int64_t vstart, int64_t vend,
                   int64_t vocab, const c10::optional<at::Tensor>& err) {
  need(ids, "ids"); need(w, "w"); need(out, "out");
  TORCH_CHECK(ids.scalar_type() == at::kLong && w.scalar_type() == at::kFloat, "ids int64, w fp32");
  ok(nmb::embedding_fwd(ids.data_ptr<int64_t>(), w.data_ptr<float>(), out.data_ptr(), ids.numel(), w.size(1), vstart,
                        vend, vocab, dtype_tag(out), err_ptr(err), stream()),
     "embedding_fwd");
}

void embedding_bwd(const at::Tensor& dy, const at::Tensor& ids, at::Tensor& wgrad, int64_t vstart, int64_t vend) {
  need(dy, "dy"); need(ids, "ids");
  TORCH_CHECK(wgrad.is_cuda() && wgrad.is_contiguous() && wgrad.scalar_type() == at::kFloat, "wgrad fp32 contiguous");
  ok(nmb::embedding_bwd(dy.data_ptr(), ids.data_ptr<int64_t>(), wgrad.data_ptr<float>(), ids.numel(), dy.size(1),
                        vstart, vend, dtype_tag(dy), stream()),
     "embedding_bwd");
}

void ce_stats(const at::Tensor& logits, const at::Tensor& target, at::Tensor& mx, at::Tensor& se, at::Tensor& tl,
              int64_t vstart) {
  TORCH_CHECK(logits.is_cuda() && logits.stride(1) == 1, "logits must be row-major CUDA");
  need(target, "target"); need(mx, "mx"); need(se, "se"); need(tl, "tl");
  ok(nmb::ce_stats(logits.data_ptr(), target.data_ptr<int64_t>(), mx.data_ptr<float>(), se.data_ptr<float>(),
                   tl.data_ptr<float>(), logits.size(0), logits.size(1), logits.stride(0), vstart, dtype_tag(logits),
                   stream()),
     "ce_stats");
}

void ce_grad(const at::Tensor& logits, const at::Tensor& target, const at::Tensor& gmax, const at::Tensor& gsum,
             const at::Tensor& gscale, double inv_n, at::Tensor& dlogits, int64_t vstart) {
  TORCH_CHECK(logits.is_cuda() && logits.stride(1) == 1, "logits must be row-major CUDA");
  need(target, "target"); need(gmax, "gmax"); need(gsum, "gsum"); need(dlogits, "dlogits");
  TORCH_CHECK(gscale.is_cuda() && gscale.scalar_type() == at::kFloat, "gscale fp32 CUDA");
  TORCH_CHECK(dlogits.scalar_type() == logits.scalar_type(), "dlogits dtype");
  ok(nmb::ce_grad(logits.data_ptr(), target.data_ptr<int64_t>(), gmax.data_ptr<float>(), gsum.data_ptr<float>(),
                  gscale.data_ptr<float>(), (float)inv_n, dlogits.data_ptr(), logits.size(0), logits.size(1),
                  logits.stride(0), vstart, dtype_tag(logits), stream()),
     "ce_grad");
}

void adamw_flat(at::Tensor& p, const at::Tensor& g, at::Tensor& m, at::Tensor& v,
                const c10::optional<at::Tensor>& compute, const at::Tensor& scale, double lr, double beta1,
                double beta2, double eps, double wd, int64_t step) {
  need(p, "p"); need(g, "g"); need(m, "m"); need(v, "v");
  TORCH_CHECK(p.numel() == g.numel() && p.numel() == m.numel() && p.numel() == v.numel(), "size mismatch");
  __nv_bfloat16* c = nullptr;
  if (compute.has_value()) {
    need(*compute, "compute");
    TORCH_CHECK(compute->scalar_type() == at::kBFloat16 && compute->numel() == p.numel(), "compute copy");
    c = reinterpret_cast<__nv_bfloat16*>(compute->data_ptr());
  }
  const double bc1 = 1.0 - std::pow(beta1, (double)step);
  const double bc2 = 1.0 - std::pow(beta2, (double)step);
  ok(nmb::adamw_flat(p.data_ptr<float>(), g.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(), c,
                     scale.data_ptr<float>(), p.numel(), lr, beta1, beta2, eps, wd, bc1, std::sqrt(bc2), stream()),
     "adamw_flat");
}

void weighted_sq_norm(const at::Tensor& ptrs, const at::Tensor& numels, const at::Tensor& weights, at::Tensor& out) {
  need(ptrs, "ptrs"); need(numels, "numels"); need(weights, "weights");
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == at::kDouble, "out fp64 CUDA");
  ok(nmb::weighted_sq_norm(ptrs.data_ptr<int64_t>(), numels.data_ptr<int64_t>(), weights.data_ptr<double>(),
                           ptrs.numel(), out.data_ptr<double>(), stream()),
     "weighted_sq_norm");
}

std::vector<at::Tensor> flash_attn_fwd(const at::Tensor& qkv, int64_t batch, int64_t heads, int64_t hd) {
  need(qkv, "qkv");
  TORCH_CHECK(qkv.scalar_type() == at::kBFloat16, "flash attention runs in bf16");
  TORCH_CHECK(qkv.size(1) == 3 * heads * hd && qkv.size(0) % batch == 0, "qkv shape");
  const int S = qkv.size(0) / batch;
  auto out = at::empty({qkv.size(0), heads * hd}, qkv.options());
  auto lse = at::empty({batch * heads, S}, qkv.options().dtype(at::kFloat));
  const at::cuda::CUDAGuard g(qkv.device());
  ok(nmb::flash_attn_fwd(reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()),
                         reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), lse.data_ptr<float>(), S, batch, heads, hd,
                         stream()),
     "flash_attn_fwd");
  return {out, lse};
}

std::vector<at::Tensor> flash_attn_fwd_tc(const at::Tensor& qkv, int64_t batch, int64_t heads, int64_t hd,
                                          const at::Tensor& err) {
  need(qkv, "qkv");
  TORCH_CHECK(qkv.scalar_type() == at::kBFloat16, "flash attention runs in bf16");
  TORCH_CHECK(qkv.size(1) == 3 * heads * hd && qkv.size(0) % batch == 0, "qkv shape");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(qkv.data_ptr()) % 16 == 0, "qkv must be 16-byte aligned");
  const int S = qkv.size(0) / batch;
  auto out = at::empty({qkv.size(0), heads * hd}, qkv.options());
  auto lse = at::empty({batch * heads, S}, qkv.options().dtype(at::kFloat));
  const at::cuda::CUDAGuard g(qkv.device());
  ok(nmb::flash_attn_fwd_tc(reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()),
                            reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), lse.data_ptr<float>(), S, batch, heads,
                            hd, err.data_ptr<int>(), stream()),
     "flash_attn_fwd_tc");
  return {out, lse};
}

at::Tensor flash_attn_bwd(const at::Tensor& dout, const at::Tensor& qkv, const at::Tensor& out, const at::Tensor& lse,
                          int64_t batch, int64_t heads, int64_t hd) {
  need(dout, "dout"); need(qkv, "qkv"); need(out, "out"); need(lse, "lse");
  TORCH_CHECK(dout.scalar_type() == at::kBFloat16 && qkv.scalar_type() == at::kBFloat16, "bf16 only");
  const int S = qkv.size(0) / batch;
  auto dqkv = at::empty_like(qkv);
  auto dvec = at::empty({batch * heads * S}, qkv.options().dtype(at::kFloat));
  auto dq_acc = at::empty({batch * heads * S * hd}, qkv.options().dtype(at::kFloat));
  const at::cuda::CUDAGuard g(qkv.device());
  ok(nmb::flash_attn_bwd(reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()),
                         reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()),
                         reinterpret_cast<const __nv_bfloat16*>(out.data_ptr()), lse.data_ptr<float>(),
                         dvec.data_ptr<float>(), dq_acc.data_ptr<float>(),
                         reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr()), S, batch, heads, hd, stream()),
     "flash_attn_bwd");
  return dqkv;
}

at::Tensor flash_attn_bwd_tc(const at::Tensor& dout, const at::Tensor& qkv, const at::Tensor& out,
                             const at::Tensor& lse, int64_t batch, int64_t heads, int64_t hd, const at::Tensor& err,
                             const c10::optional<at::Tensor>& cos, const c10::optional<at::Tensor>& sin) {
  need(dout, "dout"); need(qkv, "qkv"); need(out, "out"); need(lse, "lse");
  TORCH_CHECK(cos.has_value() == sin.has_value(), "cos and sin go together");
  const float* cosp = nullptr;
  const float* sinp = nullptr;
  if (cos.has_value()) {
    need(*cos, "cos"); need(*sin, "sin");
    TORCH_CHECK(cos->scalar_type() == at::kFloat && sin->scalar_type() == at::kFloat, "fp32 rotary tables");
    TORCH_CHECK(cos->size(0) * batch >= qkv.size(0) && cos->size(1) == hd / 2 && sin->sizes() == cos->sizes(),
                "rotary tables [S][head_dim/2]");
    cosp = cos->data_ptr<float>();
    sinp = sin->data_ptr<float>();
    TORCH_CHECK(reinterpret_cast<uintptr_t>(cosp) % 16 == 0 && reinterpret_cast<uintptr_t>(sinp) % 16 == 0,
                "rotary tables must be 16-byte aligned");
  }
  TORCH_CHECK(dout.scalar_type() == at::kBFloat16 && qkv.scalar_type() == at::kBFloat16, "bf16 only");
  const int S = qkv.size(0) / batch;
  auto dqkv = at::empty_like(qkv);
  auto dvec = at::empty({2 * batch * heads * S}, qkv.options().dtype(at::kFloat));  // D | lse*log2(e)
  const at::cuda::CUDAGuard g(qkv.device());
  auto bf = [](const at::Tensor& t) { return reinterpret_cast<const __nv_bfloat16*>(t.data_ptr()); };
  ok(nmb::flash_attn_bwd_dot(bf(dout), bf(out), dvec.data_ptr<float>(), S, batch, heads, stream()),
     "flash_attn_bwd_dot");
  ok(nmb::flash_attn_bwd_tc(bf(dout), bf(qkv), lse.data_ptr<float>(), dvec.data_ptr<float>(),
                            reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr()), S, batch, heads, hd, cosp, sinp,
                            err.data_ptr<int>(), stream()),
     "flash_attn_bwd_tc");
  return dqkv;
}

// fp32 GEMM on strided views: C (+)= op(A) op(B); A is [M,K] (or [K,M] with
// a_t), B is [K,N] (or [N,K] with b_t). Any element strides.
void gemm_f32(const at::Tensor& A, const at::Tensor& B, at::Tensor& C, bool a_t, bool b_t, double beta) {
  TORCH_CHECK(A.is_cuda() && B.is_cuda() && C.is_cuda(), "CUDA tensors");
  TORCH_CHECK(A.scalar_type() == at::kFloat && B.scalar_type() == at::kFloat && C.scalar_type() == at::kFloat,
              "fp32 only");
  const int M = a_t ? A.size(1) : A.size(0), K = a_t ? A.size(0) : A.size(1);
  const int N = b_t ? B.size(0) : B.size(1);
  TORCH_CHECK((b_t ? B.size(1) : B.size(0)) == K && C.size(0) == M && C.size(1) == N && C.stride(1) == 1, "shapes");
  const long sam = a_t ? A.stride(1) : A.stride(0), sak = a_t ? A.stride(0) : A.stride(1);
  const long sbk = b_t ? B.stride(1) : B.stride(0), sbn = b_t ? B.stride(0) : B.stride(1);
  ok(nmb::gemm_f32(M, N, K, A.data_ptr<float>(), sam, sak, B.data_ptr<float>(), sbk, sbn, C.data_ptr<float>(),
                   C.stride(0), (float)beta, stream()),
     "gemm_f32");
}

void causal_softmax_f32(const at::Tensor& S, at::Tensor& P, double scale) {
  need(S, "S"); need(P, "P");
  ok(nmb::causal_softmax_f32(S.data_ptr<float>(), P.data_ptr<float>(), S.size(0), (float)scale, stream()),
     "causal_softmax_f32");
}

void softmax_bwd_f32(const at::Tensor& P, const at::Tensor& dP, at::Tensor& dS, double scale) {
  need(P, "P"); need(dP, "dP"); need(dS, "dS");
  ok(nmb::softmax_bwd_f32(P.data_ptr<float>(), dP.data_ptr<float>(), dS.data_ptr<float>(), P.size(0), (float)scale,
                          stream()),
     "softmax_bwd_f32");
}

}  // namespace

// Cycles per tcgen05.mma (M=128, N=n, A from TMEM when ts) over a chain of
// `iters` products on one SM; synchronizes.
double mma_cycles(int64_t n, bool ts, int64_t iters, const at::Tensor& err) {
  need(err, "err");
  const at::cuda::CUDAGuard g(err.device());
  auto out = at::zeros({1}, err.options().dtype(at::kLong));
  ok(nmb::tc_mma_cycles((int)n, ts, (int)iters, reinterpret_cast<long long*>(out.data_ptr<int64_t>()),
                        err.data_ptr<int>(), stream()),
     "tc_mma_cycles");
  const long long cycles = out.item<int64_t>();
  TORCH_CHECK(cycles > 0, "mma_cycles: the probe's wait ran out");
  return (double)cycles / (double)(iters / 8 * 8);
}

void register_elementwise(pybind11::module& m) {
  m.def("rmsnorm_fwd", &rmsnorm_fwd);
  m.def("rmsnorm_bwd", &rmsnorm_bwd, pybind11::arg("dy"), pybind11::arg("x"), pybind11::arg("w"),
        pybind11::arg("rstd"), pybind11::arg("dx"), pybind11::arg("partial"), pybind11::arg("dres") = pybind11::none());
  m.def("add_rmsnorm_fwd", &add_rmsnorm_fwd);
  m.def("rmsnorm_bwd_blocks", &rmsnorm_bwd_blocks, pybind11::arg("rows"),
        pybind11::arg("max_blocks") = nmb::kNormBwdMaxBlocks);
  m.def("reduce_rows_add", &reduce_rows_add);
  m.def("swiglu_fwd", &swiglu_fwd);
  m.def("swiglu_bwd", &swiglu_bwd);
  m.def("rope_inplace", &rope_inplace);
  m.def("embedding_fwd", &embedding_fwd, pybind11::arg("ids"), pybind11::arg("w"), pybind11::arg("out"),
        pybind11::arg("vstart"), pybind11::arg("vend"), pybind11::arg("vocab"), pybind11::arg("err") = pybind11::none());
  m.def("embedding_bwd", &embedding_bwd);
  m.def("ce_stats", &ce_stats);
  m.def("ce_grad", &ce_grad);
  m.def("adamw_flat", &adamw_flat);
  m.def("weighted_sq_norm", &weighted_sq_norm);
  m.def("gemm_f32", &gemm_f32);
  m.def("causal_softmax_f32", &causal_softmax_f32);
  m.def("softmax_bwd_f32", &softmax_bwd_f32);
  m.def("flash_attn_fwd", &flash_attn_fwd);
  m.def("flash_attn_fwd_tc", &flash_attn_fwd_tc);
  m.def("flash_attn_bwd", &flash_attn_bwd);
  m.def("mma_cycles", &mma_cycles, pybind11::arg("n"), pybind11::arg("ts"), pybind11::arg("iters") = 2048,
        pybind11::arg("err"));
  m.def("flash_attn_bwd_tc", &flash_attn_bwd_tc, pybind11::arg("dout"), pybind11::arg("qkv"), pybind11::arg("out"),
        pybind11::arg("lse"), pybind11::arg("batch"), pybind11::arg("heads"), pybind11::arg("hd"), pybind11::arg("err"),
        pybind11::arg("cos") = pybind11::none(), pybind11::arg("sin") = pybind11::none());
}
