// Python bindings of the sm_100a kernels (torch extension ``nano_megatron_b200._C``).
//
// Every entry point validates device, dtype, contiguity/strides and alignment,
// then launches on the current torch CUDA stream. Shape logic that differs
// per call site (which operand is transposed, what the output is) lives in
// ``nano_megatron_b200/ops/cuda.py``.

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "dp_reduce.cuh"
#include "fused_tp.cuh"
#include "gemm.cuh"
#include "kernels.cuh"

namespace {

void check_cuda(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
}

void check_ok(cudaError_t e, const char* what) {
  TORCH_CHECK(e == cudaSuccess, what, " failed: ", cudaGetErrorString(e));
}

int* err_ptr(const c10::optional<at::Tensor>& err) {
  if (!err.has_value()) return nullptr;
  TORCH_CHECK(err->is_cuda() && err->scalar_type() == at::kInt, "err must be a CUDA int32 tensor");
  return err->data_ptr<int>();
}

int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

long row_stride(const at::Tensor& t) {
  TORCH_CHECK(t.dim() == 2 && t.stride(1) == 1, "expected a 2-D tensor with unit inner stride");
  return t.stride(0);
}

// C (op)= A x B on tcgen05. A is [M,K] (a_mn=False) or [K,M] (a_mn=True);
// B is [N,K] (b_mn=False) or [K,N] (b_mn=True); C is [M,N].
// out_mode: 0 bf16 store, 1 fp32 store, 2 fp32 accumulate.
void gemm(const at::Tensor& A, const at::Tensor& B, at::Tensor& C, bool a_mn, bool b_mn, int64_t out_mode,
          const c10::optional<at::Tensor>& err) {
  check_cuda(A, "A");
  check_cuda(B, "B");
  check_cuda(C, "C");
  TORCH_CHECK(A.scalar_type() == at::kBFloat16 && B.scalar_type() == at::kBFloat16, "A and B must be bf16");
  TORCH_CHECK(out_mode == 0 ? C.scalar_type() == at::kBFloat16 : C.scalar_type() == at::kFloat,
              "C dtype does not match out_mode");
  const int M = a_mn ? A.size(1) : A.size(0);
  const int K = a_mn ? A.size(0) : A.size(1);
  const int N = b_mn ? B.size(1) : B.size(0);
  const int Kb = b_mn ? B.size(0) : B.size(1);
  TORCH_CHECK(K == Kb, "inner dimensions differ: ", K, " vs ", Kb);
  TORCH_CHECK(C.size(0) == M && C.size(1) == N, "C has the wrong shape");
  nmb::GemmArgs g{};
  g.A = A.data_ptr();
  g.B = B.data_ptr();
  g.C = C.data_ptr();
  g.lda = row_stride(A);
  g.ldb = row_stride(B);
  g.ldc = row_stride(C);
  TORCH_CHECK(g.lda % 8 == 0 && g.ldb % 8 == 0, "bf16 row strides must be multiples of 8 elements");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(g.A) % 16 == 0 && reinterpret_cast<uintptr_t>(g.B) % 16 == 0 &&
                  reinterpret_cast<uintptr_t>(g.C) % 16 == 0,
              "operands must be 16-byte aligned");
  TORCH_CHECK(N % 8 == 0 && g.ldc % 8 == 0, "N and ldc must be multiples of 8");
  g.M = M;
  g.N = N;
  g.K = K;
  g.a_mn = a_mn;
  g.b_mn = b_mn;
  g.out = static_cast<nmb::OutMode>(out_mode);
  g.err = err_ptr(err);
  g.num_sms = num_sms();
  const at::cuda::CUDAGuard guard(A.device());
  check_ok(nmb::gemm_bf16(g, at::cuda::getCurrentCUDAStream()), "gemm_bf16");
}

// Fused gate|up projection with the SwiGLU epilogue (gemm.cu, OutMode::kSwiGLU):
// a[M,F] = silu(X W_gate) * (X W_up) for X [M,K] and W_gu [K,2F] (gate | up
// column halves); `gu` [M,2F] receives the bf16 pre-activation when given.
void gemm_swiglu(const at::Tensor& X, const at::Tensor& W, at::Tensor& a, const c10::optional<at::Tensor>& gu,
                 const c10::optional<at::Tensor>& err) {
  check_cuda(X, "X");
  check_cuda(W, "W");
  check_cuda(a, "a");
  TORCH_CHECK(X.scalar_type() == at::kBFloat16 && W.scalar_type() == at::kBFloat16 &&
                  a.scalar_type() == at::kBFloat16,
              "X, W and a must be bf16");
  const int M = X.size(0), K = X.size(1), N = W.size(1);
  TORCH_CHECK(W.size(0) == K, "inner dimensions differ");
  TORCH_CHECK(N % 16 == 0, "2F must be a multiple of 16");
  TORCH_CHECK(a.size(0) == M && a.size(1) == N / 2, "a has the wrong shape");
  nmb::GemmArgs g{};
  g.A = X.data_ptr();
  g.B = W.data_ptr();
  g.C = a.data_ptr();
  g.lda = row_stride(X);
  g.ldb = row_stride(W);
  g.ldc = row_stride(a);
  TORCH_CHECK(g.lda % 8 == 0 && g.ldb % 8 == 0 && g.ldc % 8 == 0, "row strides must be multiples of 8");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(g.A) % 16 == 0 && reinterpret_cast<uintptr_t>(g.B) % 16 == 0 &&
                  reinterpret_cast<uintptr_t>(g.C) % 16 == 0,
              "operands must be 16-byte aligned");
  if (gu.has_value()) {
    check_cuda(*gu, "gu");
    TORCH_CHECK(gu->scalar_type() == at::kBFloat16 && gu->size(0) == M && gu->size(1) == N, "gu must be bf16 [M, 2F]");
    g.gu = gu->data_ptr();
    g.ldgu = row_stride(*gu);
    TORCH_CHECK(g.ldgu % 8 == 0 && reinterpret_cast<uintptr_t>(g.gu) % 16 == 0, "gu must be 16-byte aligned");
  }
  g.M = M;
  g.N = N;
  g.K = K;
  g.a_mn = false;
  g.b_mn = true;
  g.out = nmb::OutMode::kSwiGLU;
  g.err = err_ptr(err);
  g.num_sms = num_sms();
  const at::cuda::CUDAGuard guard(X.device());
  check_ok(nmb::gemm_bf16(g, at::cuda::getCurrentCUDAStream()), "gemm_swiglu");
}

// One fused tensor-parallel GEMM + collective (see fused_tp.cu). `ws` holds every
// rank's workspace pointer (mapped in this process); offsets are in bytes.
void fused_tp_gemm(int64_t mode, const at::Tensor& a_local, const at::Tensor& B, bool b_mn, at::Tensor& out,
                   const std::vector<int64_t>& ws, int64_t rank, int64_t M, int64_t gather_off, int64_t recv_off,
                   int64_t flags_off, int64_t epoch, bool copy_own, const at::Tensor& err, double timeout_s,
                   const c10::optional<at::Tensor>& save_out, const c10::optional<at::Tensor>& labels,
                   int64_t vocab_start, const c10::optional<at::Tensor>& ce_part,
                   const c10::optional<at::Tensor>& ce_target, const c10::optional<at::Tensor>& gu) {
  check_cuda(a_local, "a_local");
  check_cuda(B, "B");
  check_cuda(out, "out");
  TORCH_CHECK(a_local.scalar_type() == at::kBFloat16 && B.scalar_type() == at::kBFloat16 &&
                  out.scalar_type() == at::kBFloat16,
              "fused TP GEMMs run in bf16");
  TORCH_CHECK(a_local.is_contiguous() && B.stride(1) == 1 && out.stride(1) == 1, "layout");
  const int world = (int)ws.size();
  TORCH_CHECK(world >= 1 && world <= nmb::kMaxRanks && rank >= 0 && rank < world, "bad group");
  nmb::FusedTpArgs a{};
  a.M = (int)M;
  a.K = (int)a_local.size(1);
  a.N = (int)(b_mn ? B.size(1) : B.size(0));
  TORCH_CHECK((b_mn ? B.size(0) : B.size(1)) == a.K, "inner dimensions differ");
  a.rank = (int)rank;
  a.world = world;
  a.m_chunk = (int)(M / world);
  TORCH_CHECK(M % world == 0 && a.m_chunk % 128 == 0, "rows per rank must be a multiple of 128");
  const bool ag = mode != nmb::kReduceScatterGemm;
  TORCH_CHECK(ag ? a_local.size(0) == a.m_chunk : a_local.size(0) == M, "A rows");
  const bool swiglu = mode == nmb::kAllGatherGemmSwiGLU;
  TORCH_CHECK(out.size(0) == (ag ? M : a.m_chunk) && out.size(1) == (swiglu ? a.N / 2 : a.N), "out shape");
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.ldo = out.stride(0);
  for (int r = 0; r < world; ++r) a.ws[r] = reinterpret_cast<uint8_t*>(ws[r]);
  a.gather_off = gather_off;
  a.recv_off = recv_off;
  a.flags_off = flags_off;
  a.a_local = reinterpret_cast<const __nv_bfloat16*>(a_local.data_ptr());
  a.lda_local = a_local.stride(0);
  a.epoch = (uint32_t)epoch;
  a.copy_own = copy_own ? 1 : 0;
  a.err = err.data_ptr<int>();
  a.timeout_ns = (uint64_t)(timeout_s * 1e9);
  if (save_out.has_value()) {
    TORCH_CHECK(ag && save_out->is_cuda() && save_out->scalar_type() == at::kBFloat16 && save_out->is_contiguous() &&
                    save_out->size(0) == M && save_out->size(1) == a.K,
                "save_out must be a contiguous bf16 [M, K] tensor of an all-gather call");
    a.save_out = reinterpret_cast<__nv_bfloat16*>(save_out->data_ptr());
  }
  if (mode == nmb::kAllGatherGemmCE) {
    TORCH_CHECK(labels.has_value() && ce_part.has_value() && ce_target.has_value(), "CE mode needs its buffers");
    const int num_n = (a.N + 255) / 256;
    TORCH_CHECK(labels->scalar_type() == at::kLong && labels->is_contiguous() && labels->numel() == M, "labels");
    TORCH_CHECK(ce_part->scalar_type() == at::kFloat && ce_part->is_contiguous() &&
                    ce_part->numel() == 2L * num_n * M,
                "ce_part must be fp32 [num_n, M, 2]");
    TORCH_CHECK(ce_target->scalar_type() == at::kFloat && ce_target->numel() == M, "ce_target");
    TORCH_CHECK(!b_mn, "the LM-head weight is [V/t, H] (K-major)");
    a.labels = labels->data_ptr<int64_t>();
    a.vocab_start = vocab_start;
    a.ce_part = reinterpret_cast<float2*>(ce_part->data_ptr<float>());
    a.ce_target = ce_target->data_ptr<float>();
  }
  if (swiglu && gu.has_value()) {
    TORCH_CHECK(gu->is_cuda() && gu->scalar_type() == at::kBFloat16 && gu->stride(1) == 1 && gu->size(0) == M &&
                    gu->size(1) == a.N && gu->stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(gu->data_ptr()) % 16 == 0,
                "gu must be a 16-byte aligned bf16 [M, 2F] tensor");
    a.gu = reinterpret_cast<__nv_bfloat16*>(gu->data_ptr());
    a.ldgu = gu->stride(0);
  }
  const at::cuda::CUDAGuard guard(a_local.device());
  check_ok(nmb::fused_tp_gemm((int)mode, a, B.data_ptr(), row_stride(B), b_mn, num_sms(),
                              at::cuda::getCurrentCUDAStream()),
           "fused_tp_gemm");
}

int64_t fused_tp_flag_bytes() { return nmb::kFlagInts * 4; }

// Cross-entropy merge over tiles and TP ranks (see fused_tp.cuh). `ws` is empty
// for a group of one.
void ce_merge(const at::Tensor& part, const at::Tensor& target_logit, const at::Tensor& labels, int64_t vocab_start,
              int64_t vocab_end, const std::vector<int64_t>& ws, int64_t rank, int64_t data_off, int64_t flags_off,
              int64_t epoch, const at::Tensor& err, double timeout_s, at::Tensor& loss, at::Tensor& gmax,
              at::Tensor& gsum) {
  check_cuda(part, "part");
  TORCH_CHECK(part.scalar_type() == at::kFloat && part.is_contiguous() && part.dim() == 3 && part.size(2) == 2,
              "part must be fp32 [num_n, T, 2]");
  const int64_t T = part.size(1);
  TORCH_CHECK(labels.scalar_type() == at::kLong && labels.is_contiguous() && labels.numel() == T, "labels");
  TORCH_CHECK(target_logit.scalar_type() == at::kFloat && target_logit.numel() == T, "target_logit");
  for (const at::Tensor* t : {&loss, &gmax, &gsum})
    TORCH_CHECK(t->scalar_type() == at::kFloat && t->is_contiguous() && t->numel() == T, "outputs: fp32 [T]");
  nmb::CeMergeArgs a{};
  a.part = reinterpret_cast<const float2*>(part.data_ptr<float>());
  a.target_logit = target_logit.data_ptr<float>();
  a.labels = labels.data_ptr<int64_t>();
  a.vocab_start = vocab_start;
  a.vocab_end = vocab_end;
  a.T = (int)T;
  a.num_n = (int)part.size(0);
  a.world = ws.empty() ? 1 : (int)ws.size();
  TORCH_CHECK(a.world <= nmb::kMaxRanks && rank >= 0 && rank < a.world, "bad group");
  a.rank = (int)rank;
  for (size_t r = 0; r < ws.size(); ++r) a.ws[r] = reinterpret_cast<uint8_t*>(ws[r]);
  a.data_off = data_off;
  a.flags_off = flags_off;
  a.epoch = (uint32_t)epoch;
  a.err = err.data_ptr<int>();
  a.timeout_ns = (uint64_t)(timeout_s * 1e9);
  a.loss = loss.data_ptr<float>();
  a.gmax = gmax.data_ptr<float>();
  a.gsum = gsum.data_ptr<float>();
  const at::cuda::CUDAGuard guard(part.device());
  check_ok(nmb::ce_merge(a, at::cuda::getCurrentCUDAStream()), "ce_merge");
}

// Data-parallel averaging of one span of the flat gradient buffer (see
// dp_reduce.cu); `bufs` / `flags` hold every DP rank's mapped pointers.
void dp_allreduce(const std::vector<int64_t>& bufs, const std::vector<int64_t>& flags, int64_t rank,
                  int64_t offset, int64_t n, int64_t epoch, const at::Tensor& err, double timeout_s) {
  const int world = (int)bufs.size();
  TORCH_CHECK(world >= 1 && world <= nmb::kDpMaxRanks && (int)flags.size() == world, "bad DP group");
  TORCH_CHECK(rank >= 0 && rank < world, "bad rank");
  TORCH_CHECK(offset % 4 == 0 && n % 4 == 0, "span must be a multiple of 4 elements");
  nmb::DpReduceArgs a{};
  for (int r = 0; r < world; ++r) {
    a.buf[r] = reinterpret_cast<float*>(bufs[r]);
    a.flags[r] = reinterpret_cast<int*>(flags[r]);
  }
  a.offset = offset;
  a.n = n;
  a.rank = (int)rank;
  a.world = world;
  a.epoch = (int)epoch;
  a.scale = 1.0f / (float)world;
  a.err = err.data_ptr<int>();
  a.timeout_ns = (uint64_t)(timeout_s * 1e9);
  const at::cuda::CUDAGuard guard(err.device());
  const int sms = at::cuda::getCurrentDeviceProperties()->multiProcessorCount;
  check_ok(nmb::dp_allreduce(a, sms, at::cuda::getCurrentCUDAStream()), "dp_allreduce");
}

int64_t dp_flag_bytes() { return nmb::kDpFlagInts * 4; }

}  // namespace

void register_elementwise(pybind11::module& m);

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "nano_megatron_b200 sm_100a kernels";
  m.def("gemm", &gemm, "tcgen05 bf16 GEMM", pybind11::arg("A"), pybind11::arg("B"), pybind11::arg("C"),
        pybind11::arg("a_mn"), pybind11::arg("b_mn"), pybind11::arg("out_mode"), pybind11::arg("err") = pybind11::none());
  m.def("gemm_swiglu", &gemm_swiglu, "tcgen05 gate|up GEMM with the SwiGLU epilogue", pybind11::arg("X"),
        pybind11::arg("W"), pybind11::arg("a"), pybind11::arg("gu") = c10::nullopt,
        pybind11::arg("err") = c10::nullopt);
  m.def("fused_tp_gemm", &fused_tp_gemm, pybind11::arg("mode"), pybind11::arg("a_local"), pybind11::arg("B"),
        pybind11::arg("b_mn"), pybind11::arg("out"), pybind11::arg("ws"), pybind11::arg("rank"), pybind11::arg("M"),
        pybind11::arg("gather_off"), pybind11::arg("recv_off"), pybind11::arg("flags_off"), pybind11::arg("epoch"),
        pybind11::arg("copy_own"), pybind11::arg("err"), pybind11::arg("timeout_s"),
        pybind11::arg("save_out") = pybind11::none(), pybind11::arg("labels") = pybind11::none(),
        pybind11::arg("vocab_start") = 0, pybind11::arg("ce_part") = pybind11::none(),
        pybind11::arg("ce_target") = pybind11::none(), pybind11::arg("gu") = pybind11::none());
  m.def("ce_merge", &ce_merge);
  m.def("dp_allreduce", &dp_allreduce);
  m.def("dp_flag_bytes", &dp_flag_bytes);
  m.def("fused_tp_flag_bytes", &fused_tp_flag_bytes);
  register_elementwise(m);
}
