// Python bindings of the sm_100a kernels.  Every entry point checks device, dtype, contiguity and
// alignment, then launches on the current CUDA stream; nothing here allocates except where an
// output is returned.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "gemm_sm100.cuh"
#include "ops.h"

namespace {

using trida::bf16;

#define CHECK_CUDA(x) TORCH_CHECK((x).is_cuda(), #x " must be a CUDA tensor")
#define CHECK_BF16(x) TORCH_CHECK((x).scalar_type() == at::kBFloat16, #x " must be bfloat16")
#define CHECK_F32(x) TORCH_CHECK((x).scalar_type() == at::kFloat, #x " must be float32")
#define CHECK_ROWMAJOR(x) TORCH_CHECK((x).dim() == 2 && (x).stride(1) == 1, #x " must be a row-major matrix")

int sm_count() {
  static int n = 0;
  if (!n) n = at::cuda::getCurrentDeviceProperties()->multiProcessorCount;
  return n;
}

cudaStream_t stream() { return at::cuda::getCurrentCUDAStream(); }

const bf16* cbf(const at::Tensor& t) { return reinterpret_cast<const bf16*>(t.data_ptr()); }
bf16* mbf(const at::Tensor& t) { return reinterpret_cast<bf16*>(t.data_ptr()); }

// D = alpha * op(A) op(B) + beta * C.  layout: 0 = TN (A[M,K], B[N,K]), 1 = TT (A[M,K], B[K,N]),
// 2 = NT (A[K,M], B[K,N]).  All operands row-major 2-D views; D bf16 or fp32.
void gemm(int64_t layout, const at::Tensor& A, const at::Tensor& B, const at::Tensor& D,
          const c10::optional<at::Tensor>& C, double alpha, double beta, int64_t tile) {
  CHECK_CUDA(A); CHECK_CUDA(B); CHECK_CUDA(D);
  CHECK_BF16(A); CHECK_BF16(B);
  CHECK_ROWMAJOR(A); CHECK_ROWMAJOR(B); CHECK_ROWMAJOR(D);
  const bool f32 = D.scalar_type() == at::kFloat;
  TORCH_CHECK(f32 || D.scalar_type() == at::kBFloat16, "D must be bf16 or fp32");
  trida::GemmArgs a{};
  int M, N, K;
  if (layout == 0) { M = A.size(0); K = A.size(1); N = B.size(0); TORCH_CHECK(B.size(1) == K, "K mismatch"); }
  else if (layout == 1) { M = A.size(0); K = A.size(1); N = B.size(1); TORCH_CHECK(B.size(0) == K, "K mismatch"); }
  else { K = A.size(0); M = A.size(1); N = B.size(1); TORCH_CHECK(B.size(0) == K, "K mismatch"); }
  TORCH_CHECK(D.size(0) == M && D.size(1) == N, "D shape mismatch");
  a.M = M; a.N = N; a.K = K;
  a.A = A.data_ptr(); a.lda = A.stride(0);
  a.B = B.data_ptr(); a.ldb = B.stride(0);
  a.D = D.data_ptr(); a.ldd = D.stride(0);
  if (C.has_value() && C->defined()) {
    CHECK_CUDA((*C)); CHECK_ROWMAJOR((*C));
    TORCH_CHECK(C->scalar_type() == D.scalar_type(), "C dtype must match D");
    TORCH_CHECK(C->size(0) == M && C->size(1) == N, "C shape mismatch");
    a.C = C->data_ptr(); a.ldc = C->stride(0);
    TORCH_CHECK((a.ldc * (f32 ? 4 : 2)) % 16 == 0 && (uintptr_t)a.C % 16 == 0,
                "GEMM C operand must be 16-byte aligned with a 16-byte-multiple leading dimension");
  } else {
    TORCH_CHECK(beta == 0.0, "beta != 0 needs a C operand");
    a.C = nullptr; a.ldc = a.ldd;
  }
  a.alpha = (float)alpha; a.beta = (float)beta;
  a.batch = 1;
  a.strideA_batch = a.strideB_batch = a.strideC_batch = a.strideD_batch = 0;
  if (M == 0 || N == 0) return;
  TORCH_CHECK(K > 0, "K must be positive");
  const int elemD = f32 ? 4 : 2;
  TORCH_CHECK((a.lda * 2) % 16 == 0 && (a.ldb * 2) % 16 == 0 && (a.ldd * elemD) % 16 == 0,
              "GEMM leading dimensions must be 16-byte multiples");
  TORCH_CHECK(((uintptr_t)a.A % 16 == 0) && ((uintptr_t)a.B % 16 == 0) && ((uintptr_t)a.D % 16 == 0),
              "GEMM operands must be 16-byte aligned");
  c10::cuda::CUDAGuard g(A.device());
  const int splits = trida::gemm_splitk(M, N, K, sm_count());
  at::Tensor ws;
  if (splits > 1) ws = at::empty({(int64_t)splits * M * N}, A.options().dtype(at::kFloat));
  const int rc = trida::gemm_bf16((trida::GemmLayout)layout, f32, a, (int)tile, sm_count(), stream(), splits,
                                  splits > 1 ? ws.data_ptr<float>() : nullptr);
  TORCH_CHECK(rc == 0, "sm100 GEMM failed with code ", rc, " (M=", M, " N=", N, " K=", K, " layout=", layout, ")");
}

// ---------------------------------------------------------------------------------------------
// symmetric peer memory (symm.cu).  Buffers are raw cudaMalloc allocations (IPC-exportable),
// wrapped as non-owning tensors; pointers travel as Python ints.
// ---------------------------------------------------------------------------------------------
int64_t symm_malloc(int64_t bytes) {
  void* p = nullptr;
  TORCH_CHECK(cudaMalloc(&p, bytes) == cudaSuccess, "symmetric buffer allocation of ", bytes, " bytes failed");
  TORCH_CHECK(cudaMemset(p, 0, bytes) == cudaSuccess, "symmetric buffer clear failed");
  return reinterpret_cast<int64_t>(p);
}

void symm_free(int64_t p) { cudaFree(reinterpret_cast<void*>(p)); }

py::bytes symm_handle(int64_t p) {
  unsigned char h[64];
  TORCH_CHECK(trida::symm_ipc_handle(reinterpret_cast<void*>(p), h) == 0, "cudaIpcGetMemHandle failed");
  return py::bytes(reinterpret_cast<const char*>(h), 64);
}

int64_t symm_open(py::bytes handle) {
  std::string h = handle;
  TORCH_CHECK(h.size() == 64, "IPC handle must be 64 bytes");
  void* p = trida::symm_ipc_open(reinterpret_cast<const unsigned char*>(h.data()));
  TORCH_CHECK(p != nullptr, "cudaIpcOpenMemHandle failed");
  return reinterpret_cast<int64_t>(p);
}

void symm_close(int64_t p) { trida::symm_ipc_close(reinterpret_cast<void*>(p)); }

at::Tensor symm_tensor(int64_t p, int64_t numel, at::ScalarType dtype, int64_t device) {
  return torch::from_blob(reinterpret_cast<void*>(p), {numel}, [](void*) {},
                          at::TensorOptions().dtype(dtype).device(at::kCUDA, device));
}

struct PtrArrays {
  void* bufs[8];
  unsigned* flags[8];
};

static PtrArrays ptr_arrays(const std::vector<int64_t>& bufs, const std::vector<int64_t>& flags) {
  TORCH_CHECK(bufs.size() == flags.size() && bufs.size() >= 1 && bufs.size() <= 8, "1..8 ranks");
  PtrArrays a{};
  for (size_t i = 0; i < bufs.size(); ++i) {
    a.bufs[i] = reinterpret_cast<void*>(bufs[i]);
    a.flags[i] = reinterpret_cast<unsigned*>(flags[i]);
  }
  return a;
}

// ctr_done: int32 [2] on this rank's device (epoch counter, finished-CTA counter), zero at start.
void symm_allreduce(const std::vector<int64_t>& bufs, const std::vector<int64_t>& flags, int64_t rank,
                    const at::Tensor& ctr_done, int64_t off, int64_t n, const c10::optional<at::Tensor>& residual,
                    const at::Tensor& out, const at::Tensor& err) {
  TORCH_CHECK(ctr_done.scalar_type() == at::kInt && ctr_done.numel() >= 2, "ctr_done must be int32 [2]");
  unsigned* cd = reinterpret_cast<unsigned*>(ctr_done.data_ptr<int>());
  auto a = ptr_arrays(bufs, flags);
  CHECK_BF16(out); TORCH_CHECK(out.is_contiguous() && out.numel() == n, "out must hold n elements");
  const bf16* res = nullptr;
  if (residual.has_value() && residual->defined()) {
    CHECK_BF16((*residual)); TORCH_CHECK(residual->is_contiguous() && residual->numel() == n, "residual shape");
    res = cbf(*residual);
  }
  const int rc = trida::symm_allreduce_bf16(a.bufs, a.flags, rank, bufs.size(), cd, cd + 1, off, n, res, mbf(out),
                                            err.data_ptr<int>(), sm_count(), stream());
  TORCH_CHECK(rc == 0, "symm_allreduce failed with code ", rc);
}

// Sequence-parallel boundary (tensor-parallel serving): parts / gather are every rank's symmetric
// partial [M, D] and gather [M, D] bf16 buffers; xs [nrows, D] bf16 is this rank's residual rows
// starting at row0 (updated in place); ctr_done int32 [2], zero at start.
void symm_rs_norm_ag(const std::vector<int64_t>& parts, const std::vector<int64_t>& gather,
                     const std::vector<int64_t>& flags, int64_t rank, const at::Tensor& ctr_done, int64_t row0,
                     const at::Tensor& xs, const at::Tensor& w, double eps, const at::Tensor& err) {
  TORCH_CHECK(ctr_done.scalar_type() == at::kInt && ctr_done.numel() >= 2, "ctr_done must be int32 [2]");
  TORCH_CHECK(gather.size() == parts.size(), "one gather buffer per rank");
  auto a = ptr_arrays(parts, flags);
  void* g[8] = {};
  for (size_t i = 0; i < gather.size(); ++i) g[i] = reinterpret_cast<void*>(gather[i]);
  CHECK_BF16(xs); CHECK_BF16(w);
  TORCH_CHECK(xs.dim() == 2 && xs.is_contiguous() && w.is_contiguous() && w.numel() == xs.size(1),
              "xs [rows, D] contiguous, w [D]");
  TORCH_CHECK((uintptr_t)xs.data_ptr() % 16 == 0 && (uintptr_t)w.data_ptr() % 16 == 0, "16-byte aligned rows");
  unsigned* cd = reinterpret_cast<unsigned*>(ctr_done.data_ptr<int>());
  const int rc = trida::symm_rs_norm_ag(a.bufs, g, a.flags, rank, parts.size(), cd, xs.size(1), row0, xs.size(0),
                                        mbf(xs), cbf(w), (float)eps, err.data_ptr<int>(), sm_count(), stream());
  TORCH_CHECK(rc == 0, "symm_rs_norm_ag failed with code ", rc, " (D must be a multiple of 8, at most 8192)");
}

// Row-parallel GEMM with the tensor-parallel all-reduce in its epilogue:
// D = sum over ranks of A_r B_r^T (+ residual).  recv / flags: every rank's receive buffer
// ([2][world][mcap][N] bf16) and counters ([2][tiles_cap][4] u32); ctr_done: int32 [2], zero at start.
// gu = A . B^T with B = [gate; up] ([2F, K]) and act = silu(gate) * up, one kernel (TN, bf16)
void gemm_swiglu(const at::Tensor& A, const at::Tensor& B, const at::Tensor& D, const at::Tensor& act,
                 int64_t tile) {
  CHECK_CUDA(A); CHECK_CUDA(B); CHECK_CUDA(D); CHECK_CUDA(act);
  CHECK_BF16(A); CHECK_BF16(B); CHECK_BF16(D); CHECK_BF16(act);
  CHECK_ROWMAJOR(A); CHECK_ROWMAJOR(B); CHECK_ROWMAJOR(D); CHECK_ROWMAJOR(act);
  const int M = A.size(0), K = A.size(1), N = B.size(0), F = N / 2;
  TORCH_CHECK(B.size(1) == K && N % 128 == 0, "B must be [2F, K] with F a multiple of 64");
  TORCH_CHECK(D.size(0) == M && D.size(1) == N && act.size(0) == M && act.size(1) == F, "output shapes");
  if (M == 0) return;
  trida::GemmArgs a{};
  a.M = M; a.N = N; a.K = K;
  a.A = A.data_ptr(); a.lda = A.stride(0);
  a.B = B.data_ptr(); a.ldb = B.stride(0);
  a.D = D.data_ptr(); a.ldd = D.stride(0);
  a.C = nullptr; a.ldc = a.ldd;
  a.alpha = 1.f; a.beta = 0.f; a.batch = 1;
  TORCH_CHECK((a.lda * 2) % 16 == 0 && (a.ldb * 2) % 16 == 0 && (a.ldd * 2) % 16 == 0 && (act.stride(0) * 2) % 16 == 0,
              "GEMM leading dimensions must be 16-byte multiples");
  TORCH_CHECK((uintptr_t)a.A % 16 == 0 && (uintptr_t)a.B % 16 == 0 && (uintptr_t)a.D % 16 == 0 &&
                  (uintptr_t)act.data_ptr() % 16 == 0, "GEMM operands must be 16-byte aligned");
  c10::cuda::CUDAGuard g(A.device());
  const int rc = trida::gemm_bf16_swiglu(a, act.data_ptr(), act.stride(0), F, (int)tile, sm_count(), stream());
  TORCH_CHECK(rc == 0, "gemm_bf16_swiglu failed (code ", rc, ")");
}

void gemm_allreduce(const at::Tensor& A, const at::Tensor& B, const at::Tensor& D,
                    const c10::optional<at::Tensor>& residual, const std::vector<int64_t>& recv,
                    const std::vector<int64_t>& flags, int64_t rank, const at::Tensor& ctr_done, int64_t mcap,
                    int64_t tiles_cap, const c10::optional<at::Tensor>& ws,
                    const c10::optional<at::Tensor>& tile_ctr) {
  CHECK_CUDA(A); CHECK_CUDA(B); CHECK_CUDA(D);
  CHECK_BF16(A); CHECK_BF16(B); CHECK_BF16(D);
  CHECK_ROWMAJOR(A); CHECK_ROWMAJOR(B); CHECK_ROWMAJOR(D);
  TORCH_CHECK(ctr_done.scalar_type() == at::kInt && ctr_done.numel() >= 2, "ctr_done must be int32 [2]");
  auto pa = ptr_arrays(recv, flags);
  trida::GemmArgs a{};
  a.M = A.size(0); a.K = A.size(1); a.N = B.size(0);
  TORCH_CHECK(B.size(1) == a.K && D.size(0) == a.M && D.size(1) == a.N, "shape mismatch");
  a.A = A.data_ptr(); a.lda = A.stride(0);
  a.B = B.data_ptr(); a.ldb = B.stride(0);
  a.D = D.data_ptr(); a.ldd = D.stride(0);
  a.alpha = 1.f; a.beta = 0.f; a.C = nullptr; a.ldc = a.ldd;
  if (residual.has_value() && residual->defined()) {
    CHECK_BF16((*residual)); CHECK_ROWMAJOR((*residual));
    TORCH_CHECK(residual->size(0) == a.M && residual->size(1) == a.N, "residual shape");
    a.C = residual->data_ptr(); a.ldc = residual->stride(0); a.beta = 1.f;
  }
  a.batch = 1;
  if (a.M == 0) return;
  TORCH_CHECK((a.lda * 2) % 16 == 0 && (a.ldb * 2) % 16 == 0 && (a.ldd * 2) % 16 == 0 && (a.ldc * 2) % 16 == 0,
              "GEMM leading dimensions must be 16-byte multiples");
  c10::cuda::CUDAGuard g(A.device());
  unsigned* cd = reinterpret_cast<unsigned*>(ctr_done.data_ptr<int>());
  float* wsp = nullptr;
  int64_t ws_units = 0;
  unsigned* tc = nullptr;
  if (ws.has_value() && ws->defined() && tile_ctr.has_value() && tile_ctr->defined()) {
    TORCH_CHECK(ws->scalar_type() == at::kFloat && ws->is_contiguous(), "ws must be contiguous fp32");
    TORCH_CHECK(tile_ctr->scalar_type() == at::kInt && tile_ctr->numel() >= tiles_cap * 4, "tile_ctr int32 [tiles_cap*4]");
    wsp = ws->data_ptr<float>();
    ws_units = ws->numel() / (128 * 256);
    tc = reinterpret_cast<unsigned*>(tile_ctr->data_ptr<int>());
  }
  trida::GemmAllreduce ar{(int)recv.size(), (int)rank, (int)tiles_cap, mcap, pa.bufs, pa.flags, cd, cd + 1,
                          wsp, ws_units, tc};
  const int rc = trida::gemm_bf16_allreduce(a, ar, sm_count(), stream());
  TORCH_CHECK(rc == 0, "fused GEMM + all-reduce failed with code ", rc, " (M=", a.M, " N=", a.N, " K=", a.K, ")");
}

void symm_rs_sumsq(const std::vector<int64_t>& bufs, const std::vector<int64_t>& flags, int64_t rank, int64_t epoch,
                   int64_t shard_off, int64_t shard_len, double scale, const at::Tensor& shard_out,
                   const at::Tensor& partial, const at::Tensor& err, bool accumulate,
                   const c10::optional<at::Tensor>& done, int64_t close_slot) {
  auto a = ptr_arrays(bufs, flags);
  TORCH_CHECK(shard_out.scalar_type() == at::kFloat && shard_out.numel() == shard_len, "shard_out");
  TORCH_CHECK(partial.scalar_type() == at::kFloat, "partial fp32");
  unsigned* dn = nullptr;
  if (done.has_value() && done->defined()) {
    TORCH_CHECK(done->scalar_type() == at::kInt && done->numel() >= 1, "done must be int32");
    dn = reinterpret_cast<unsigned*>(done->data_ptr<int>());
  }
  const int rc = trida::symm_rs_sumsq(a.bufs, a.flags, rank, bufs.size(), (unsigned)epoch, shard_off, shard_len,
                                      (float)scale, shard_out.data_ptr<float>(), partial.data_ptr<float>(),
                                      partial.numel(), accumulate ? 1 : 0, err.data_ptr<int>(), dn, (int)close_slot,
                                      stream());
  TORCH_CHECK(rc == 0, "symm_rs_sumsq failed with code ", rc);
}

void symm_norm_coef(const std::vector<int64_t>& partials, const std::vector<int64_t>& flags, int64_t rank,
                    int64_t epoch, int64_t nblocks, double max_norm, const at::Tensor& norm, const at::Tensor& coef,
                    const at::Tensor& err) {
  auto a = ptr_arrays(partials, flags);
  const int rc = trida::symm_norm_coef(a.bufs, a.flags, rank, partials.size(), (unsigned)epoch, nblocks,
                                       (float)max_norm, norm.data_ptr<float>(), coef.data_ptr<float>(),
                                       err.data_ptr<int>(), stream());
  TORCH_CHECK(rc == 0, "symm_norm_coef failed with code ", rc);
}

void symm_adamw_ag(const std::vector<int64_t>& bufs, const std::vector<int64_t>& flags, int64_t rank, int64_t epoch,
                   int64_t shard_off, int64_t shard_len, const at::Tensor& grad, const c10::optional<at::Tensor>& master,
                   const at::Tensor& m, const at::Tensor& v, double lr, double b1, double b2, double eps, double wd,
                   int64_t step, const c10::optional<at::Tensor>& coef, const at::Tensor& done, const at::Tensor& err) {
  auto a = ptr_arrays(bufs, flags);
  TORCH_CHECK(grad.numel() == shard_len && m.numel() == shard_len && v.numel() == shard_len, "shard sizes");
  float* pm = (master.has_value() && master->defined()) ? master->data_ptr<float>() : nullptr;
  const float* pc = (coef.has_value() && coef->defined()) ? coef->data_ptr<float>() : nullptr;
  const int rc = trida::symm_adamw_ag(a.bufs, a.flags, rank, bufs.size(), (unsigned)epoch, shard_off, shard_len,
                                      grad.data_ptr<float>(), pm, m.data_ptr<float>(), v.data_ptr<float>(), (float)lr,
                                      (float)b1, (float)b2, (float)eps, (float)wd, (int)step, pc,
                                      reinterpret_cast<unsigned*>(done.data_ptr<int>()), err.data_ptr<int>(),
                                      sm_count(), stream());
  TORCH_CHECK(rc == 0, "symm_adamw_ag failed with code ", rc);
}

// Full-shard parameter all-gather: every rank's bf16 shard (bufs[r], shard_len elements) into this
// rank's dst (world * shard_len elements) over NVLink.
void symm_gather(const std::vector<int64_t>& bufs, int64_t rank, int64_t shard_len, const at::Tensor& dst,
                 int64_t blocks) {
  TORCH_CHECK(bufs.size() >= 1 && bufs.size() <= 8, "1..8 ranks");
  CHECK_BF16(dst);
  TORCH_CHECK(dst.is_contiguous() && dst.numel() >= (int64_t)bufs.size() * shard_len, "dst too small");
  void* b[8];
  for (size_t i = 0; i < bufs.size(); ++i) b[i] = reinterpret_cast<void*>(bufs[i]);
  const int rc = trida::symm_gather_bf16(b, rank, bufs.size(), shard_len, mbf(dst), (int)blocks, stream());
  TORCH_CHECK(rc == 0, "symm_gather failed with code ", rc);
}

// The same gather on the copy engines: one peer-to-peer cudaMemcpyAsync per rank's shard (the IPC
// mapping makes every shard addressable), so no SM is taken from the compute kernels it overlaps.
void symm_gather_copy(const std::vector<int64_t>& bufs, int64_t rank, int64_t shard_len, const at::Tensor& dst) {
  TORCH_CHECK(bufs.size() >= 1 && bufs.size() <= 8, "1..8 ranks");
  CHECK_BF16(dst);
  TORCH_CHECK(dst.is_contiguous() && dst.numel() >= (int64_t)bufs.size() * shard_len, "dst too small");
  const int world = (int)bufs.size();
  for (int k = 0; k < world; ++k) {
    const int r = (int)((k + rank) % world);     // stagger the peers each rank reads first
    const cudaError_t e = cudaMemcpyAsync(mbf(dst) + (int64_t)r * shard_len, reinterpret_cast<const void*>(bufs[r]),
                                          (size_t)shard_len * 2, cudaMemcpyDeviceToDevice, stream());
    TORCH_CHECK(e == cudaSuccess, "symm_gather_copy: ", cudaGetErrorString(e));
  }
}

void symm_barrier(const std::vector<int64_t>& flags, int64_t rank, int64_t epoch, int64_t slot, const at::Tensor& err) {
  TORCH_CHECK(flags.size() >= 1 && flags.size() <= 8, "1..8 ranks");
  unsigned* f[8];
  for (size_t i = 0; i < flags.size(); ++i) f[i] = reinterpret_cast<unsigned*>(flags[i]);
  const int rc = trida::symm_barrier(f, rank, flags.size(), (unsigned)epoch, (int)slot, err.data_ptr<int>(), stream());
  TORCH_CHECK(rc == 0, "symm_barrier failed with code ", rc);
}

// Reads and clears the GEMM's device error word (host sync); 0 = no timed-out wait.
int64_t gemm_error() {
  int* w = trida::gemm_error_word();
  if (!w) return 0;
  int v = 0;
  cudaMemcpy(&v, w, sizeof(int), cudaMemcpyDeviceToHost);
  if (v) cudaMemset(w, 0, sizeof(int));
  return v;
}

// ---------------------------------------------------------------------------------------------
// gated-delta-rule layers (gdn.cu).  Matrices are row-major 2-D views (row stride free, unit
// column stride); `doc` is an optional uint8 [B, Lc] document-start mask of the clean stream.
// ---------------------------------------------------------------------------------------------
static trida::GdnParams gdn_params(const at::Tensor& mixed, const at::Tensor& ga, const at::Tensor& gb,
                                   const at::Tensor& A_log, const at::Tensor& dt_bias,
                                   const c10::optional<at::Tensor>& doc, int64_t B, int64_t T, int64_t Hk, int64_t Hv,
                                   int64_t mode, int64_t L, int64_t V, int64_t bd, bool causal_clean, bool causal_noisy,
                                   double scale) {
  CHECK_CUDA(mixed); CHECK_BF16(mixed); CHECK_ROWMAJOR(mixed);
  CHECK_BF16(ga); CHECK_BF16(gb); CHECK_ROWMAJOR(ga); CHECK_ROWMAJOR(gb);
  TORCH_CHECK(ga.stride(0) == gb.stride(0), "gate views must share a row stride");
  TORCH_CHECK(A_log.scalar_type() == at::kFloat && dt_bias.scalar_type() == at::kFloat, "A_log/dt_bias fp32");
  TORCH_CHECK(mixed.size(0) == B * T && ga.size(0) == B * T && ga.size(1) == Hv, "GDN shape mismatch");
  TORCH_CHECK(mixed.size(1) >= 2 * Hk * 128 + Hv * 128, "mixed too narrow");
  TORCH_CHECK(mixed.stride(0) % 4 == 0, "mixed row stride must be a multiple of 4");
  if (mode) TORCH_CHECK(T == (1 + V) * L, "two-stream rows must be (1 + V) * L tokens");
  trida::GdnParams p{};
  p.B = B; p.T = T; p.Hk = Hk; p.Hv = Hv; p.dk = 128; p.dvh = 128;
  p.mode = mode; p.L = L; p.V = V; p.bd = bd; p.causal_clean = causal_clean; p.causal_noisy = causal_noisy;
  if (doc.has_value() && doc->defined()) {
    TORCH_CHECK(doc->scalar_type() == at::kByte && doc->is_contiguous(), "doc must be contiguous uint8");
    TORCH_CHECK(doc->numel() == B * (mode ? L : T), "doc must be [B, Lc]");
    p.doc = doc->data_ptr<uint8_t>();
  }
  p.mixed = cbf(mixed); p.ldm = mixed.stride(0);
  p.ga = cbf(ga); p.gb = cbf(gb); p.ldg = ga.stride(0);
  p.A_log = A_log.data_ptr<float>(); p.dt_bias = dt_bias.data_ptr<float>();
  p.scale = (float)scale;
  return p;
}

int64_t gdn_state_numel(int64_t B, int64_t T, int64_t Hv, int64_t mode, int64_t L, int64_t bd) {
  trida::GdnParams p{};
  p.B = B; p.T = T; p.Hv = Hv; p.mode = mode; p.L = L; p.bd = bd;
  return trida::gdn_state_floats(p);
}

void gdn_fwd(const at::Tensor& mixed, const at::Tensor& ga, const at::Tensor& gb, const at::Tensor& A_log,
             const at::Tensor& dt_bias, const c10::optional<at::Tensor>& doc, const at::Tensor& o, const at::Tensor& ckpt,
             int64_t B, int64_t T, int64_t Hk, int64_t Hv, int64_t mode, int64_t L, int64_t V, int64_t bd,
             bool causal_clean, bool causal_noisy, double scale, const c10::optional<at::Tensor>& final_state) {
  auto p = gdn_params(mixed, ga, gb, A_log, dt_bias, doc, B, T, Hk, Hv, mode, L, V, bd, causal_clean, causal_noisy, scale);
  CHECK_BF16(o); TORCH_CHECK(o.is_contiguous() && o.numel() == B * T * Hv * 128, "o must be [B*T, Hv*128]");
  TORCH_CHECK(ckpt.scalar_type() == at::kFloat && ckpt.numel() >= trida::gdn_state_floats(p), "ckpt too small");
  p.ckpt = ckpt.data_ptr<float>(); p.o = mbf(o);
  at::Tensor prep = at::empty({trida::gdn_prep_floats(B * T, Hk, Hv)}, mixed.options().dtype(at::kFloat));
  p.prep = prep.data_ptr<float>();
  if (final_state.has_value() && final_state->defined()) {
    TORCH_CHECK(final_state->scalar_type() == at::kFloat && final_state->is_contiguous() &&
                final_state->numel() == B * Hv * 128 * 128, "final_state must be fp32 [B, Hv, 128, 128]");
    p.final_state = final_state->data_ptr<float>();
  }
  c10::cuda::CUDAGuard g(mixed.device());
  const int rc = trida::gdn_fwd(p, stream());
  TORCH_CHECK(rc == 0, "gdn_fwd failed with code ", rc);
}

void gdn_bwd(const at::Tensor& mixed, const at::Tensor& ga, const at::Tensor& gb, const at::Tensor& A_log,
             const at::Tensor& dt_bias, const c10::optional<at::Tensor>& doc, const at::Tensor& ckpt,
             const at::Tensor& d_o, const at::Tensor& dmixed, const at::Tensor& dga, const at::Tensor& dgb,
             const at::Tensor& dA_log, const at::Tensor& ddt_bias, int64_t B, int64_t T, int64_t Hk, int64_t Hv,
             int64_t mode, int64_t L, int64_t V, int64_t bd, bool causal_clean, bool causal_noisy, double scale) {
  auto p = gdn_params(mixed, ga, gb, A_log, dt_bias, doc, B, T, Hk, Hv, mode, L, V, bd, causal_clean, causal_noisy, scale);
  CHECK_BF16(d_o); TORCH_CHECK(d_o.is_contiguous() && d_o.numel() == B * T * Hv * 128, "d_o must be [B*T, Hv*128]");
  CHECK_BF16(dmixed); CHECK_ROWMAJOR(dmixed); CHECK_BF16(dga); CHECK_BF16(dgb); CHECK_ROWMAJOR(dga);
  TORCH_CHECK(dga.stride(0) == dgb.stride(0), "gate-gradient views must share a row stride");
  TORCH_CHECK(dmixed.stride(0) % 4 == 0, "dmixed row stride must be a multiple of 4");
  TORCH_CHECK(dA_log.scalar_type() == at::kFloat && ddt_bias.scalar_type() == at::kFloat, "fp32 gate grads");
  const int64_t ns = trida::gdn_state_floats(p);
  TORCH_CHECK(ckpt.numel() >= ns, "ckpt too small");
  auto f32 = mixed.options().dtype(at::kFloat);
  at::Tensor dpart = at::empty({trida::gdn_part_floats(p)}, f32);
  at::Tensor dinit = mode ? at::empty({ns}, f32) : at::Tensor();
  p.ckpt = ckpt.data_ptr<float>();
  p.d_o = cbf(d_o);
  p.dpart = dpart.data_ptr<float>();
  p.dv = mbf(dmixed) + 2 * Hk * 128; p.lddv = dmixed.stride(0);
  p.dinit = mode ? dinit.data_ptr<float>() : nullptr;
  at::Tensor prep = at::empty({trida::gdn_prep_floats(B * T, Hk, Hv)}, mixed.options().dtype(at::kFloat));
  p.prep = prep.data_ptr<float>();
  c10::cuda::CUDAGuard g(mixed.device());
  const int rc = trida::gdn_bwd(p, mbf(dmixed), dmixed.stride(0), mbf(dga), mbf(dgb), dga.stride(0),
                                dA_log.data_ptr<float>(), ddt_bias.data_ptr<float>(), stream());
  TORCH_CHECK(rc == 0, "gdn_bwd failed with code ", rc);
}

// ---------------------------------------------------------------------------------------------
// serving decode step (serve.cu, gdn.cu canvas/commit)
// ---------------------------------------------------------------------------------------------
static void check_i32(const at::Tensor& t, int64_t n, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kInt && t.is_contiguous() && t.numel() == n, name,
              " must be a contiguous int32 CUDA tensor of ", n, " elements");
}

// ptab (optional): int32 [slots, maxpages] page table of a paged cache kc / vc [pages, 64, Hkv, D]
// (position p of slot s lives in page ptab[s, p / 64], row p % 64); without it the cache is dense
// [slots, maxlen, Hkv, D].
static int paged_maxlen(const at::Tensor& kc, const c10::optional<at::Tensor>& ptab, int64_t& maxpages) {
  maxpages = 0;
  if (!ptab.has_value() || !ptab->defined()) return kc.size(1);
  TORCH_CHECK(ptab->scalar_type() == at::kInt && ptab->is_contiguous() && ptab->dim() == 2, "ptab int32 [slots, pages]");
  TORCH_CHECK(kc.size(1) == 64, "a paged cache holds 64 positions per page");
  maxpages = ptab->size(1);
  return (int)(maxpages * 64);
}

// With `err` (the device error word) the tensor-core kernel runs; without it the warp-MMA kernel.
void canvas_attention(const at::Tensor& q, const at::Tensor& kc, const at::Tensor& vc, const at::Tensor& slot,
                      const at::Tensor& pos, const at::Tensor& out, int64_t blk, int64_t n_clean, int64_t max_keys,
                      double scale, const c10::optional<at::Tensor>& ptab, const c10::optional<at::Tensor>& err) {
  CHECK_BF16(q); CHECK_BF16(kc); CHECK_BF16(vc); CHECK_BF16(out);
  TORCH_CHECK(q.dim() == 3 && q.is_contiguous() && out.is_contiguous() && kc.dim() == 4 && kc.is_contiguous() &&
              vc.is_contiguous(), "canvas attention layouts");
  const int64_t B = q.size(0) / blk;
  check_i32(slot, B, "slot"); check_i32(pos, B, "pos");
  int64_t maxpages = 0;
  const int Hq = q.size(1), D = q.size(2), Hkv = kc.size(2), maxlen = paged_maxlen(kc, ptab, maxpages);
  TORCH_CHECK(max_keys <= maxlen, "max_keys exceeds the cache length");
  c10::cuda::CUDAGuard g(q.device());
  if (err.has_value() && err->defined()) {
    TORCH_CHECK(err->scalar_type() == at::kInt && err->is_cuda(), "err must be a CUDA int32 word");
    const int64_t nw = trida::canvas_tc_work_floats(B, blk, Hq, Hkv, D, max_keys);
    at::Tensor work = nw > 0 ? at::empty({nw}, q.options().dtype(at::kFloat)) : at::Tensor();
    const int n_slots = maxpages ? (int)ptab->size(0) : (int)kc.size(0);
    const int rc = trida::canvas_attention_tc(cbf(q), cbf(kc), cbf(vc), kc.size(0) * kc.size(1), n_slots, slot.data_ptr<int>(),
                                              pos.data_ptr<int>(), mbf(out), nw > 0 ? work.data_ptr<float>() : nullptr,
                                              B, blk, n_clean, Hq, Hkv, D, maxlen, max_keys, (float)scale,
                                              err->data_ptr<int>(), stream(), maxpages ? ptab->data_ptr<int>() : nullptr,
                                              (int)maxpages);
    TORCH_CHECK(rc == 0, "canvas_attention_tc failed with code ", rc);
    return;
  }
  at::Tensor work = at::empty({trida::canvas_work_floats(B, blk, Hq, D, max_keys)}, q.options().dtype(at::kFloat));
  const int rc = trida::canvas_attention(cbf(q), cbf(kc), cbf(vc), slot.data_ptr<int>(), pos.data_ptr<int>(), mbf(out),
                                         work.data_ptr<float>(), B, blk, n_clean, Hq, Hkv, D, maxlen, max_keys,
                                         (float)scale, stream(), maxpages ? ptab->data_ptr<int>() : nullptr,
                                         (int)maxpages);
  TORCH_CHECK(rc == 0, "canvas_attention failed with code ", rc);
}

void kv_append(const at::Tensor& k, const at::Tensor& v, const at::Tensor& kc, const at::Tensor& vc,
               const at::Tensor& slot, const at::Tensor& pos, int64_t blk, const c10::optional<at::Tensor>& ptab) {
  CHECK_BF16(k); CHECK_BF16(v); CHECK_ROWMAJOR(v);
  TORCH_CHECK(k.is_contiguous() && kc.is_contiguous() && vc.is_contiguous() && kc.dim() == 4, "kv_append layouts");
  const int Hkv = kc.size(2), D = kc.size(3);
  const int64_t B = k.numel() / (blk * Hkv * D);
  TORCH_CHECK(v.size(0) == B * blk && v.size(1) == Hkv * D && v.stride(0) % 8 == 0, "v rows");
  check_i32(slot, B, "slot"); check_i32(pos, B, "pos");
  c10::cuda::CUDAGuard g(k.device());
  int64_t maxpages = 0;
  const int maxlen = paged_maxlen(kc, ptab, maxpages);
  trida::kv_append(cbf(k), cbf(v), v.stride(0), mbf(kc), mbf(vc), slot.data_ptr<int>(), pos.data_ptr<int>(), B, blk,
                   Hkv, D, maxlen, stream(), maxpages ? ptab->data_ptr<int>() : nullptr, (int)maxpages);
}

void canvas_conv(const at::Tensor& x, const at::Tensor& win, const at::Tensor& w, const at::Tensor& y,
                 const at::Tensor& slot, int64_t blk) {
  CHECK_BF16(x); CHECK_ROWMAJOR(x); CHECK_BF16(win); CHECK_BF16(w); CHECK_ROWMAJOR(y);
  const int C = x.size(1), K = w.size(1);
  TORCH_CHECK(win.is_contiguous() && win.size(1) == K - 1 && win.size(2) == C && K <= 4, "conv window layout");
  TORCH_CHECK(C % 8 == 0 && x.stride(0) % 8 == 0 && y.stride(0) % 8 == 0, "conv alignment");
  const int64_t B = x.size(0) / blk;
  check_i32(slot, B, "slot");
  c10::cuda::CUDAGuard g(x.device());
  trida::canvas_conv(cbf(x), x.stride(0), cbf(win), cbf(w), mbf(y), y.stride(0), slot.data_ptr<int>(), B, blk, C, K,
                     stream());
}

void conv_commit(const at::Tensor& x, int64_t rows_per, const at::Tensor& win, const at::Tensor& slot,
                 const at::Tensor& adv) {
  CHECK_BF16(x); CHECK_ROWMAJOR(x); CHECK_BF16(win);
  const int C = x.size(1), K = win.size(1) + 1;
  TORCH_CHECK(win.is_contiguous() && win.size(2) == C && K <= 4 && x.stride(0) % 8 == 0, "conv window layout");
  const int64_t B = slot.numel();
  check_i32(slot, B, "slot"); check_i32(adv, B, "adv");
  c10::cuda::CUDAGuard g(x.device());
  trida::conv_commit(cbf(x), x.stride(0), rows_per, mbf(win), slot.data_ptr<int>(), adv.data_ptr<int>(), B, C, K,
                     stream());
}

int64_t gdn_prep_numel(int64_t rows, int64_t Hk, int64_t Hv) { return trida::gdn_prep_floats(rows, Hk, Hv); }

// State cache: fp32 [slots, Hv, 128 * 128] in the kernels' thread-native order.
void gdn_canvas(const at::Tensor& mixed, const at::Tensor& ga, const at::Tensor& gb, const at::Tensor& A_log,
                const at::Tensor& dt_bias, const at::Tensor& o, const at::Tensor& prep, const at::Tensor& ssm,
                const at::Tensor& slot, int64_t blk, int64_t Hk, int64_t Hv, int64_t n_clean, double scale) {
  const int64_t B = mixed.size(0) / blk;
  auto p = gdn_params(mixed, ga, gb, A_log, dt_bias, c10::nullopt, B, blk, Hk, Hv, 0, blk, 0, 32, true, false, scale);
  CHECK_BF16(o); TORCH_CHECK(o.is_contiguous() && o.numel() == B * blk * Hv * 128, "o layout");
  TORCH_CHECK(ssm.scalar_type() == at::kFloat && ssm.is_contiguous() && ssm.size(1) == Hv, "state cache layout");
  TORCH_CHECK(prep.scalar_type() == at::kFloat && prep.numel() >= trida::gdn_prep_floats(B * blk, Hk, Hv), "prep size");
  check_i32(slot, B, "slot");
  p.o = mbf(o);
  c10::cuda::CUDAGuard g(mixed.device());
  TORCH_CHECK(trida::gdn_canvas(p, prep.data_ptr<float>(), ssm.data_ptr<float>(), slot.data_ptr<int>(), n_clean,
                                stream()) == 0, "gdn_canvas failed");
}

void gdn_commit(const at::Tensor& mixed, const at::Tensor& ga, const at::Tensor& gb, const at::Tensor& A_log,
                const at::Tensor& dt_bias, const at::Tensor& prep, const at::Tensor& ssm, const at::Tensor& slot,
                const at::Tensor& adv, int64_t blk, int64_t Hk, int64_t Hv, double scale) {
  const int64_t B = mixed.size(0) / blk;
  auto p = gdn_params(mixed, ga, gb, A_log, dt_bias, c10::nullopt, B, blk, Hk, Hv, 0, blk, 0, 32, true, false, scale);
  TORCH_CHECK(ssm.scalar_type() == at::kFloat && ssm.is_contiguous() && ssm.size(1) == Hv, "state cache layout");
  TORCH_CHECK(prep.scalar_type() == at::kFloat && prep.numel() >= trida::gdn_prep_floats(B * blk, Hk, Hv), "prep size");
  check_i32(slot, B, "slot"); check_i32(adv, B, "adv");
  c10::cuda::CUDAGuard g(mixed.device());
  TORCH_CHECK(trida::gdn_commit(p, prep.data_ptr<float>(), ssm.data_ptr<float>(), slot.data_ptr<int>(),
                                adv.data_ptr<int>(), stream()) == 0, "gdn_commit failed");
}

// Tensor-core canvas step: state cache fp32 [slots, Hv, 128, 128] (k rows, v columns); writes o and the
// commit inputs kbuf / ubuf (bf16 [B * blk, Hv, 128]) and gbuf (fp32 [B * blk, Hv]).
void gdn_canvas_tc(const at::Tensor& mixed, const at::Tensor& ga, const at::Tensor& gb, const at::Tensor& A_log,
                   const at::Tensor& dt_bias, const at::Tensor& o, const at::Tensor& kbuf, const at::Tensor& ubuf,
                   const at::Tensor& gbuf, const at::Tensor& ssm, const at::Tensor& slot, int64_t blk, int64_t Hk,
                   int64_t Hv, int64_t n_clean, double scale, const at::Tensor& err,
                   const c10::optional<at::Tensor>& z, const c10::optional<at::Tensor>& gnorm_w, double eps) {
  const int64_t M = mixed.size(0), B = M / blk;
  CHECK_BF16(mixed); CHECK_BF16(ga); CHECK_BF16(gb); CHECK_BF16(o); CHECK_BF16(kbuf); CHECK_BF16(ubuf);
  TORCH_CHECK(M == B * blk && mixed.stride(1) == 1 && (mixed.stride(0) % 8) == 0 && (uintptr_t)mixed.data_ptr() % 16 == 0,
              "mixed: rows of 16-byte aligned bf16");
  TORCH_CHECK(mixed.size(1) >= (2 * Hk + Hv) * 128, "mixed: q | k | v columns");
  TORCH_CHECK(ga.stride(1) == 1 && gb.stride(1) == 1 && ga.stride(0) == gb.stride(0) && ga.size(0) == M, "gate layout");
  TORCH_CHECK(o.is_contiguous() && o.numel() == M * Hv * 128, "o layout");
  TORCH_CHECK(kbuf.is_contiguous() && ubuf.is_contiguous() && kbuf.numel() == M * Hv * 128 && ubuf.numel() == M * Hv * 128,
              "kbuf / ubuf layout");
  TORCH_CHECK(gbuf.scalar_type() == at::kFloat && gbuf.is_contiguous() && gbuf.numel() == M * Hv, "gbuf layout");
  TORCH_CHECK(ssm.scalar_type() == at::kFloat && ssm.is_contiguous() && ssm.dim() == 4 && ssm.size(1) == Hv &&
                  ssm.size(2) == 128 && ssm.size(3) == 128, "state cache [slots, Hv, 128, 128] fp32");
  TORCH_CHECK(A_log.scalar_type() == at::kFloat && dt_bias.scalar_type() == at::kFloat, "fp32 A_log / dt_bias");
  check_i32(slot, B, "slot");
  // optional fused gated RMSNorm: o receives rmsnorm(o) * w * silu(z) per value head
  const bf16* pz = nullptr; const bf16* pw = nullptr; int64_t ldz = 0;
  if (z.has_value() && z->defined()) {
    TORCH_CHECK(gnorm_w.has_value() && gnorm_w->defined(), "the fused gated norm needs its weight");
    CHECK_BF16((*z)); CHECK_BF16((*gnorm_w));
    TORCH_CHECK(z->stride(1) == 1 && z->size(0) == M && z->size(1) >= Hv * 128 && z->stride(0) % 8 == 0 &&
                    (uintptr_t)z->data_ptr() % 16 == 0, "z rows of 16-byte aligned bf16");
    TORCH_CHECK(gnorm_w->is_contiguous() && gnorm_w->numel() == 128, "gated norm weight [128]");
    pz = cbf(*z); pw = cbf(*gnorm_w); ldz = z->stride(0);
  }
  c10::cuda::CUDAGuard g(mixed.device());
  TORCH_CHECK(trida::gdn_canvas_tc(cbf(mixed), mixed.stride(0), cbf(ga), cbf(gb), ga.stride(0), A_log.data_ptr<float>(),
                                   dt_bias.data_ptr<float>(), ssm.data_ptr<float>(), slot.data_ptr<int>(), mbf(o),
                                   mbf(kbuf), mbf(ubuf), gbuf.data_ptr<float>(), (int)B, (int)blk, (int)n_clean, (int)Hk,
                                   (int)Hv, (float)scale, err.data_ptr<int>(), stream(), pz, ldz, pw, (float)eps) == 0,
              "gdn_canvas_tc failed (canvas rows must be 1..64)");
}

void gdn_commit_tc(const at::Tensor& kbuf, const at::Tensor& ubuf, const at::Tensor& gbuf, const at::Tensor& ssm,
                   const at::Tensor& slot, const at::Tensor& adv, int64_t blk, int64_t Hv, const at::Tensor& err) {
  const int64_t M = gbuf.numel() / Hv, B = M / blk;
  TORCH_CHECK(ssm.scalar_type() == at::kFloat && ssm.is_contiguous() && ssm.dim() == 4 && ssm.size(1) == Hv,
              "state cache layout");
  check_i32(slot, B, "slot"); check_i32(adv, B, "adv");
  c10::cuda::CUDAGuard g(ssm.device());
  TORCH_CHECK(trida::gdn_commit_tc(cbf(kbuf), cbf(ubuf), gbuf.data_ptr<float>(), ssm.data_ptr<float>(),
                                   slot.data_ptr<int>(), adv.data_ptr<int>(), (int)B, (int)blk, (int)Hv,
                                   err.data_ptr<int>(), stream()) == 0, "gdn_commit_tc failed");
}

// Sampled self-speculative step for a batch (see sampler.cu): candidate lists [B, blk, kc] (sorted
// top-k of the canvas logits), per-request sampling parameters, per-slot draw counters and q lists.
void spec_sample(const at::Tensor& vals, const at::Tensor& idx, const at::Tensor& temp, const at::Tensor& topk,
                 const at::Tensor& topp, const at::Tensor& seed, const at::Tensor& counter, const at::Tensor& slot,
                 const at::Tensor& specs, const at::Tensor& has_specs, const at::Tensor& q_idx,
                 const at::Tensor& q_prob, const at::Tensor& out, int64_t n) {
  TORCH_CHECK(vals.scalar_type() == at::kFloat && vals.is_contiguous() && vals.dim() == 3, "vals [B, blk, kc] fp32");
  TORCH_CHECK(idx.scalar_type() == at::kLong && idx.is_contiguous() && idx.sizes() == vals.sizes(), "idx like vals");
  const int64_t B = vals.size(0), blk = vals.size(1), kc = vals.size(2), K = n - 1;
  TORCH_CHECK(temp.scalar_type() == at::kFloat && topp.scalar_type() == at::kFloat && temp.numel() == B &&
                  topp.numel() == B, "temp / topp fp32 [B]");
  check_i32(topk, B, "topk"); check_i32(slot, B, "slot"); check_i32(has_specs, B, "has_specs");
  TORCH_CHECK(seed.scalar_type() == at::kLong && seed.numel() == B, "seed int64 [B]");
  TORCH_CHECK(counter.scalar_type() == at::kLong && counter.is_contiguous(), "counter int64 [slots]");
  TORCH_CHECK(specs.scalar_type() == at::kInt && specs.is_contiguous() && specs.numel() >= B * std::max<int64_t>(K, 1),
              "specs int32 [B, K]");
  TORCH_CHECK(q_idx.scalar_type() == at::kInt && q_prob.scalar_type() == at::kFloat && q_idx.dim() == 3 &&
                  q_idx.size(1) == K && q_idx.size(2) == 64 && q_prob.sizes() == q_idx.sizes(),
              "q lists [slots, K, 64]");
  TORCH_CHECK(out.scalar_type() == at::kInt && out.is_contiguous() && out.numel() == B * (3 + K), "out int32 [B, 3 + K]");
  c10::cuda::CUDAGuard g(vals.device());
  TORCH_CHECK(trida::spec_sample(vals.data_ptr<float>(), idx.data_ptr<int64_t>(), (int)kc, temp.data_ptr<float>(),
                                 topk.data_ptr<int>(), topp.data_ptr<float>(), seed.data_ptr<int64_t>(),
                                 counter.data_ptr<int64_t>(), slot.data_ptr<int>(), specs.data_ptr<int>(),
                                 has_specs.data_ptr<int>(), q_idx.data_ptr<int>(), q_prob.data_ptr<float>(),
                                 out.data_ptr<int>(), (int)B, (int)blk, (int)n, stream()) == 0,
              "spec_sample failed (1 <= candidates <= 64, n <= canvas rows)");
}

// Greedy tokens of h W^T (the LM head) without materialising the logits: out int64 [M].
void gemm_argmax(const at::Tensor& A, const at::Tensor& B, const at::Tensor& out) {
  CHECK_BF16(A); CHECK_BF16(B); CHECK_ROWMAJOR(A); CHECK_ROWMAJOR(B);
  TORCH_CHECK(A.size(1) == B.size(1), "K mismatch");
  TORCH_CHECK(out.scalar_type() == at::kLong && out.is_contiguous() && out.numel() == A.size(0), "out int64 [M]");
  const int M = A.size(0), N = B.size(0), K = A.size(1);
  const int nt = trida::gemm_argmax_tiles(N);
  auto val = at::empty({M, nt}, A.options().dtype(at::kFloat));
  auto idx = at::empty({M, nt}, A.options().dtype(at::kInt));
  trida::GemmArgs a{};
  a.M = M; a.N = N; a.K = K; a.A = A.data_ptr(); a.lda = A.stride(0); a.B = B.data_ptr(); a.ldb = B.stride(0);
  a.C = nullptr; a.ldc = 0; a.D = nullptr; a.ldd = 0; a.alpha = 1.f; a.beta = 0.f; a.batch = 1;
  c10::cuda::CUDAGuard g(A.device());
  const int rc = trida::gemm_bf16_argmax(a, val.data_ptr<float>(), idx.data_ptr<int>(), out.data_ptr<int64_t>(),
                                         sm_count(), stream());
  TORCH_CHECK(rc == 0, "gemm_argmax failed with code ", rc);
}

void argmax_rows(const at::Tensor& logits, const at::Tensor& out) {
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.dim() == 2 && logits.stride(1) == 1, "fp32 logits rows");
  TORCH_CHECK(out.scalar_type() == at::kLong && out.is_contiguous() && out.numel() == logits.size(0), "out int64");
  c10::cuda::CUDAGuard g(logits.device());
  trida::argmax_rows(logits.data_ptr<float>(), logits.stride(0), logits.size(0), logits.size(1), out.data_ptr<int64_t>(),
                     stream());
}

// logits [B, R, V] fp32 (any batch / row strides, unit vocab stride) -> idx int64 [B, R], row max and
// sum(exp(x - max)) fp32 [B, R]
void conf_argmax_rows(const at::Tensor& logits, const at::Tensor& idx, const at::Tensor& mx, const at::Tensor& sum) {
  TORCH_CHECK(logits.is_cuda() && logits.scalar_type() == at::kFloat && logits.dim() == 3 && logits.stride(2) == 1,
              "fp32 logits [B, R, V] with unit vocabulary stride");
  const int64_t B = logits.size(0), R = logits.size(1);
  TORCH_CHECK(idx.scalar_type() == at::kLong && idx.is_contiguous() && idx.numel() == B * R, "idx int64 [B, R]");
  TORCH_CHECK(mx.scalar_type() == at::kFloat && mx.is_contiguous() && mx.numel() == B * R, "max fp32 [B, R]");
  TORCH_CHECK(sum.scalar_type() == at::kFloat && sum.is_contiguous() && sum.numel() == B * R, "sum fp32 [B, R]");
  c10::cuda::CUDAGuard g(logits.device());
  trida::conf_argmax_rows(logits.data_ptr<float>(), (int)(B * R), (int)std::max<int64_t>(R, 1), logits.stride(0),
                          logits.stride(1), (int)logits.size(2), idx.data_ptr<int64_t>(), mx.data_ptr<float>(),
                          sum.data_ptr<float>(), stream());
}

static trida::ConvParams conv_params(const at::Tensor& x, const at::Tensor& w, const c10::optional<at::Tensor>& doc,
                                     int64_t B, int64_t T, int64_t mode, int64_t L, int64_t V, int64_t bd) {
  CHECK_CUDA(x); CHECK_BF16(x); CHECK_ROWMAJOR(x); CHECK_BF16(w);
  TORCH_CHECK(w.is_contiguous() && w.dim() == 2 && w.size(0) == x.size(1), "conv weight must be [C, K]");
  TORCH_CHECK(x.size(0) == B * T && x.size(1) % 8 == 0 && x.stride(0) % 8 == 0, "conv input shape / stride");
  trida::ConvParams p{};
  p.B = B; p.T = T; p.C = x.size(1); p.K = w.size(1);
  p.mode = mode; p.L = L; p.V = V; p.bd = bd;
  if (doc.has_value() && doc->defined()) {
    TORCH_CHECK(doc->scalar_type() == at::kByte && doc->is_contiguous(), "doc must be contiguous uint8");
    p.doc = doc->data_ptr<uint8_t>();
  }
  p.x = cbf(x); p.ldx = x.stride(0); p.w = cbf(w);
  return p;
}

void gdn_conv_fwd(const at::Tensor& x, const at::Tensor& w, const at::Tensor& y, const c10::optional<at::Tensor>& doc,
                  int64_t B, int64_t T, int64_t mode, int64_t L, int64_t V, int64_t bd) {
  auto p = conv_params(x, w, doc, B, T, mode, L, V, bd);
  CHECK_BF16(y); CHECK_ROWMAJOR(y);
  TORCH_CHECK(y.size(0) == x.size(0) && y.size(1) == x.size(1) && y.stride(0) % 8 == 0, "conv output shape");
  p.y = mbf(y); p.ldy = y.stride(0);
  c10::cuda::CUDAGuard g(x.device());
  TORCH_CHECK(trida::gdn_conv_fwd(p, stream()) == 0, "gdn_conv_fwd failed");
}

void gdn_conv_bwd(const at::Tensor& dy, const at::Tensor& x, const at::Tensor& w, const at::Tensor& dx,
                  const at::Tensor& dw, const c10::optional<at::Tensor>& doc, int64_t B, int64_t T, int64_t mode,
                  int64_t L, int64_t V, int64_t bd) {
  auto p = conv_params(x, w, doc, B, T, mode, L, V, bd);
  CHECK_BF16(dy); CHECK_ROWMAJOR(dy); CHECK_BF16(dx); CHECK_ROWMAJOR(dx);
  TORCH_CHECK(dy.stride(0) % 8 == 0 && dx.stride(0) % 8 == 0, "conv gradient strides");
  TORCH_CHECK(dw.scalar_type() == at::kFloat && dw.numel() == w.numel(), "dw must be fp32 like w");
  at::Tensor dpre = at::empty({x.size(0), x.size(1)}, x.options().dtype(at::kFloat));
  c10::cuda::CUDAGuard g(x.device());
  TORCH_CHECK(trida::gdn_conv_bwd(p, cbf(dy), dy.stride(0), dpre.data_ptr<float>(), mbf(dx), dx.stride(0),
                                  dw.data_ptr<float>(), stream()) == 0, "gdn_conv_bwd failed");
}

void gdn_gnorm_fwd(const at::Tensor& o, const at::Tensor& z, const at::Tensor& w, const at::Tensor& y, int64_t H,
                   double eps) {
  CHECK_BF16(o); CHECK_BF16(z); CHECK_BF16(w); CHECK_BF16(y); CHECK_ROWMAJOR(z);
  TORCH_CHECK(o.is_contiguous() && y.is_contiguous() && w.numel() == 128, "gated norm shapes");
  const int64_t rows = z.size(0);
  TORCH_CHECK(o.numel() == rows * H * 128 && z.size(1) == H * 128, "gated norm shapes");
  c10::cuda::CUDAGuard g(o.device());
  TORCH_CHECK(trida::gdn_gnorm_fwd(cbf(o), cbf(z), z.stride(0), cbf(w), mbf(y), rows, H, (float)eps, stream()) == 0,
              "gdn_gnorm_fwd failed");
}

void gdn_gnorm_bwd(const at::Tensor& dy, const at::Tensor& o, const at::Tensor& z, const at::Tensor& w,
                   const at::Tensor& d_o, const at::Tensor& dz, const at::Tensor& dw, int64_t H, double eps) {
  CHECK_BF16(dy); CHECK_BF16(o); CHECK_BF16(z); CHECK_BF16(d_o); CHECK_BF16(dz); CHECK_ROWMAJOR(z);
  CHECK_ROWMAJOR(dz);
  TORCH_CHECK(dy.is_contiguous() && o.is_contiguous() && d_o.is_contiguous(), "gated norm grads contiguous");
  TORCH_CHECK(dw.scalar_type() == at::kFloat && dw.numel() == 128, "dw fp32 [128]");
  const int64_t rows = z.size(0);
  c10::cuda::CUDAGuard g(o.device());
  TORCH_CHECK(trida::gdn_gnorm_bwd(cbf(dy), cbf(o), cbf(z), z.stride(0), cbf(w), mbf(d_o), mbf(dz), dz.stride(0),
                                   dw.data_ptr<float>(), rows, H, (float)eps, sm_count(), stream()) == 0,
              "gdn_gnorm_bwd failed");
}

std::vector<at::Tensor> rmsnorm_fwd(const at::Tensor& x, const at::Tensor& w, double eps, const at::Tensor& out) {
  CHECK_CUDA(x); CHECK_BF16(x); CHECK_BF16(w); CHECK_ROWMAJOR(x); CHECK_ROWMAJOR(out);
  const int M = x.size(0), D = x.size(1);
  TORCH_CHECK(D % 8 == 0, "hidden size must be a multiple of 8");
  auto rstd = at::empty({M}, x.options().dtype(at::kFloat));
  trida::rmsnorm_fwd(cbf(x), x.stride(0), cbf(w), mbf(out), out.stride(0), rstd.data_ptr<float>(), M, D, (float)eps,
                     stream());
  return {out, rstd};
}

void rmsnorm_bwd(const at::Tensor& dy, const at::Tensor& x, const at::Tensor& w, const at::Tensor& rstd,
                 const c10::optional<at::Tensor>& dres, const at::Tensor& dx, const c10::optional<at::Tensor>& dw) {
  CHECK_BF16(dy); CHECK_BF16(x); CHECK_ROWMAJOR(dy); CHECK_ROWMAJOR(x); CHECK_ROWMAJOR(dx);
  const int M = x.size(0), D = x.size(1);
  const bf16* pr = nullptr; int64_t ldr = 0;
  if (dres.has_value() && dres->defined()) { CHECK_ROWMAJOR((*dres)); pr = cbf(*dres); ldr = dres->stride(0); }
  float* pdw = nullptr;
  if (dw.has_value() && dw->defined()) { CHECK_F32((*dw)); pdw = dw->data_ptr<float>(); }
  trida::rmsnorm_bwd(cbf(dy), dy.stride(0), cbf(x), x.stride(0), cbf(w), rstd.data_ptr<float>(), pr, ldr, mbf(dx),
                     dx.stride(0), pdw, M, D, sm_count(), stream());
}

// qw / kw None: RoPE without the per-head RMSNorm
at::Tensor qk_norm_rope_fwd(const at::Tensor& qkv, const c10::optional<at::Tensor>& qw,
                            const c10::optional<at::Tensor>& kw, const at::Tensor& cos_t, const at::Tensor& sin_t,
                            const at::Tensor& pos, const at::Tensor& q, const at::Tensor& k, int64_t Hq, int64_t Hkv,
                            int64_t d, int64_t rd, double eps, int64_t qstride) {
  CHECK_BF16(qkv); CHECK_ROWMAJOR(qkv); CHECK_F32(cos_t); CHECK_F32(sin_t);
  TORCH_CHECK(pos.scalar_type() == at::kInt && pos.is_contiguous(), "pos must be contiguous int32");
  TORCH_CHECK(q.is_contiguous() && k.is_contiguous(), "q/k outputs must be contiguous");
  const bool has_q = qw.has_value() && qw->defined(), has_k = kw.has_value() && kw->defined();
  TORCH_CHECK(has_q == has_k, "q and k norm weights must both be given or both be None");
  const int M = qkv.size(0);
  auto rstd = at::empty({M, Hq + Hkv}, qkv.options().dtype(at::kFloat));
  trida::qk_norm_rope_fwd(cbf(qkv), qkv.stride(0), has_q ? cbf(*qw) : nullptr, has_k ? cbf(*kw) : nullptr,
                          cos_t.data_ptr<float>(),
                          sin_t.data_ptr<float>(), pos.data_ptr<int>(), mbf(q), mbf(k), rstd.data_ptr<float>(), M,
                          Hq, Hkv, d, rd, (float)eps, qstride ? qstride : d, stream());
  return rstd;
}

void qk_norm_rope_bwd(const at::Tensor& dq, const at::Tensor& dk, const at::Tensor& qkv, const at::Tensor& qw,
                      const at::Tensor& kw, const at::Tensor& cos_t, const at::Tensor& sin_t, const at::Tensor& pos,
                      const at::Tensor& rstd, const at::Tensor& dqkv, const c10::optional<at::Tensor>& dqw,
                      const c10::optional<at::Tensor>& dkw, int64_t Hq, int64_t Hkv, int64_t d, int64_t rd,
                      int64_t qstride) {
  CHECK_ROWMAJOR(qkv); CHECK_ROWMAJOR(dqkv);
  TORCH_CHECK(dq.is_contiguous() && dk.is_contiguous(), "dq/dk must be contiguous");
  const int M = qkv.size(0);
  float* pq = (dqw.has_value() && dqw->defined()) ? dqw->data_ptr<float>() : nullptr;
  float* pk = (dkw.has_value() && dkw->defined()) ? dkw->data_ptr<float>() : nullptr;
  trida::qk_norm_rope_bwd(cbf(dq), cbf(dk), cbf(qkv), qkv.stride(0), cbf(qw), cbf(kw), cos_t.data_ptr<float>(),
                          sin_t.data_ptr<float>(), pos.data_ptr<int>(), rstd.data_ptr<float>(), mbf(dqkv),
                          dqkv.stride(0), pq, pk, M, Hq, Hkv, d, rd, qstride ? qstride : d, sm_count(), stream());
}

// y = o * sigmoid(gate) with the gate heads interleaved in qkv (head h: [q (d) | gate (d)]).
void attn_gate_fwd(const at::Tensor& o, const at::Tensor& qkv, const at::Tensor& y, int64_t Hq, int64_t d) {
  CHECK_BF16(o); CHECK_BF16(qkv); CHECK_ROWMAJOR(qkv);
  TORCH_CHECK(o.is_contiguous() && y.is_contiguous() && d % 8 == 0 && qkv.stride(0) % 8 == 0, "gate shapes");
  trida::attn_gate_fwd(cbf(o), cbf(qkv), qkv.stride(0), mbf(y), qkv.size(0), Hq, d, sm_count(), stream());
}

void attn_gate_bwd(const at::Tensor& dy, const at::Tensor& o, const at::Tensor& qkv, const at::Tensor& d_o,
                   const at::Tensor& dqkv, int64_t Hq, int64_t d) {
  CHECK_ROWMAJOR(qkv); CHECK_ROWMAJOR(dqkv);
  TORCH_CHECK(dy.is_contiguous() && o.is_contiguous() && d_o.is_contiguous() && dqkv.stride(0) % 8 == 0, "gate shapes");
  trida::attn_gate_bwd(cbf(dy), cbf(o), cbf(qkv), qkv.stride(0), mbf(d_o), mbf(dqkv), dqkv.stride(0), qkv.size(0), Hq,
                       d, sm_count(), stream());
}

void swiglu_fwd(const at::Tensor& gu, const at::Tensor& out) {
  CHECK_BF16(gu); CHECK_ROWMAJOR(gu); CHECK_ROWMAJOR(out);
  const int M = gu.size(0), F = gu.size(1) / 2;
  TORCH_CHECK(F % 8 == 0, "FFN size must be a multiple of 8");
  trida::swiglu_fwd(cbf(gu), gu.stride(0), mbf(out), out.stride(0), M, F, sm_count(), stream());
}

void swiglu_bwd(const at::Tensor& da, const at::Tensor& gu, const at::Tensor& dgu) {
  CHECK_ROWMAJOR(da); CHECK_ROWMAJOR(gu); CHECK_ROWMAJOR(dgu);
  const int M = gu.size(0), F = gu.size(1) / 2;
  trida::swiglu_bwd(cbf(da), da.stride(0), cbf(gu), gu.stride(0), mbf(dgu), dgu.stride(0), M, F, sm_count(),
                    stream());
}

void embed_fwd(const at::Tensor& ids, const at::Tensor& table, const at::Tensor& out) {
  TORCH_CHECK(ids.scalar_type() == at::kLong && ids.is_contiguous(), "ids must be contiguous int64");
  CHECK_BF16(table); CHECK_ROWMAJOR(table);
  TORCH_CHECK(out.is_contiguous(), "out must be contiguous");
  trida::embed_fwd(ids.data_ptr<int64_t>(), cbf(table), mbf(out), ids.numel(), table.size(1), stream());
}

void embed_bwd(const at::Tensor& ids, const at::Tensor& dout, const at::Tensor& dtable) {
  CHECK_F32(dtable);
  TORCH_CHECK(dout.is_contiguous(), "dout must be contiguous");
  trida::embed_bwd(ids.data_ptr<int64_t>(), cbf(dout), dtable.data_ptr<float>(), ids.numel(), dtable.size(1),
                   stream());
}

// meta: [B, T, 4] int32.  Returns (cls, fwd_list, fwd_cnt, bwd_list, bwd_cnt).
std::vector<at::Tensor> bd_attn_plan(const at::Tensor& meta, int64_t flags) {
  TORCH_CHECK(meta.scalar_type() == at::kInt && meta.is_contiguous() && meta.dim() == 3 && meta.size(2) == 4,
              "meta must be contiguous int32 [B, T, 4]");
  const int B = meta.size(0), T = meta.size(1);
  const int nt = (T + 63) / 64, nq2 = (nt + 1) / 2;
  TORCH_CHECK(nt < (1 << 14), "sequence too long for the tile lists");
  auto o8 = meta.options().dtype(at::kByte);
  auto o16 = meta.options().dtype(at::kShort);
  auto o32 = meta.options().dtype(at::kInt);
  auto cls = at::empty({B, nt, nt}, o8);
  auto fl = at::empty({B, nq2, nt}, o16);
  auto fc = at::empty({B, nq2}, o32);
  auto bl = at::empty({B, nt, nt}, o16);
  auto bc = at::empty({B, nt}, o32);
  trida::bd_attn_plan(reinterpret_cast<const int4*>(meta.data_ptr<int>()), B, T, (int)flags, cls.data_ptr<uint8_t>(),
                      fl.data_ptr<int16_t>(), fc.data_ptr<int>(), bl.data_ptr<int16_t>(), bc.data_ptr<int>(),
                      stream());
  return {cls, fl, fc, bl, bc};
}

// q [B,T,Hq,D], k [B,T,Hkv,D], v [B,T,Hkv,D] (token stride may differ: strided views allowed when
// the innermost two dims are dense), o [B,T,Hq,D], lse [B,Hq,T].
trida::AttnTensors attn_tensors(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& o,
                                const at::Tensor& lse) {
  for (auto* t : {&q, &k, &v, &o}) {
    TORCH_CHECK(t->dim() == 4 && t->stride(3) == 1 && t->stride(2) == t->size(3), "attention operand layout");
    CHECK_BF16((*t));
    TORCH_CHECK(((uintptr_t)t->data_ptr() % 16) == 0 && (t->stride(1) % 8) == 0, "attention operand alignment");
  }
  CHECK_F32(lse);
  trida::AttnTensors a;
  a.q = cbf(q); a.k = cbf(k); a.v = cbf(v);
  a.q_tok = q.stride(1); a.k_tok = k.stride(1); a.v_tok = v.stride(1);
  a.q_b = q.stride(0); a.k_b = k.stride(0); a.v_b = v.stride(0);
  a.o = mbf(o); a.o_tok = o.stride(1); a.o_b = o.stride(0);
  a.lse = lse.data_ptr<float>();
  a.B = q.size(0); a.T = q.size(1); a.Hq = q.size(2); a.Hkv = k.size(2); a.D = q.size(3);
  TORCH_CHECK(a.Hq % a.Hkv == 0, "Hq must be a multiple of Hkv");
  return a;
}

void bd_attn_fwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& o,
                 const at::Tensor& lse, const at::Tensor& meta, const at::Tensor& fwd_list, const at::Tensor& fwd_cnt,
                 int64_t flags, double scale) {
  auto a = attn_tensors(q, k, v, o, lse);
  const int rc = trida::bd_attn_fwd(a, reinterpret_cast<const int4*>(meta.data_ptr<int>()),
                                    fwd_list.data_ptr<int16_t>(), fwd_cnt.data_ptr<int>(), (int)flags, (float)scale,
                                    stream());
  TORCH_CHECK(rc == 0, "bd_attn_fwd: unsupported head_dim ", a.D);
}

void bd_attn_bwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& o,
                 const at::Tensor& lse, const at::Tensor& dout, const at::Tensor& dq, const at::Tensor& dk,
                 const at::Tensor& dv, const at::Tensor& meta, const at::Tensor& bwd_list, const at::Tensor& bwd_cnt,
                 int64_t flags, double scale) {
  auto a = attn_tensors(q, k, v, o, lse);
  for (auto* t : {&dout, &dq, &dk, &dv})
    TORCH_CHECK(t->dim() == 4 && t->stride(3) == 1 && t->stride(2) == t->size(3), "attention grad layout");
  auto dsum = at::empty({a.B, a.Hq, a.T}, lse.options());
  auto dq_acc = at::empty({a.B, a.T, a.Hq, a.D}, lse.options());
  const int rc = trida::bd_attn_bwd(a, cbf(dout), dout.stride(1), dout.stride(0), dsum.data_ptr<float>(),
                                    dq_acc.data_ptr<float>(), mbf(dq), dq.stride(1), dq.stride(0), mbf(dk),
                                    dk.stride(1), dk.stride(0), mbf(dv), dv.stride(1), dv.stride(0),
                                    reinterpret_cast<const int4*>(meta.data_ptr<int>()), bwd_list.data_ptr<int16_t>(),
                                    bwd_cnt.data_ptr<int>(), (int)flags, (float)scale, sm_count(), stream());
  TORCH_CHECK(rc == 0, "bd_attn_bwd: unsupported head_dim ", a.D);
}

std::vector<at::Tensor> bd_attn_lists128(const at::Tensor& cls, int64_t T, int64_t transpose) {
  TORCH_CHECK(cls.scalar_type() == at::kByte && cls.is_contiguous() && cls.dim() == 3, "cls must be uint8 [B,nt,nt]");
  const int B = cls.size(0), n = (T + 127) / 128;
  auto list = at::empty({B, n, n}, cls.options().dtype(at::kShort));
  auto cnt = at::empty({B, n}, cls.options().dtype(at::kInt));
  trida::bd_attn_lists128(cls.data_ptr<uint8_t>(), B, T, list.data_ptr<int16_t>(), cnt.data_ptr<int>(), (int)transpose,
                          stream());
  return {list, cnt};
}

// Row / column bit masks of the PARTIAL 128x128 tiles: ([B, n, n, 128, 4], [B, n, n, 128, 4]) int32.
std::vector<at::Tensor> bd_attn_tile_masks(const at::Tensor& meta, const at::Tensor& cls, int64_t flags) {
  const int B = meta.size(0), T = meta.size(1), n = (T + 127) / 128;
  auto rm = at::empty({B, n, n, 128, 4}, meta.options().dtype(at::kInt));
  auto cm = at::empty({B, n, n, 128, 4}, meta.options().dtype(at::kInt));
  trida::bd_attn_tile_masks(reinterpret_cast<const int4*>(meta.data_ptr<int>()), cls.data_ptr<uint8_t>(), B, T,
                            (int)flags, reinterpret_cast<uint4*>(rm.data_ptr<int>()),
                            reinterpret_cast<uint4*>(cm.data_ptr<int>()), stream());
  return {rm, cm};
}

void bd_attn_fwd_sm100(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& o,
                       const at::Tensor& lse, const at::Tensor& meta, const at::Tensor& list128,
                       const at::Tensor& cnt128, const at::Tensor& rowmask, int64_t flags, double scale,
                       const at::Tensor& err,
                       const c10::optional<at::Tensor>& dbg) {
  auto a = attn_tensors(q, k, v, o, lse);
  TORCH_CHECK(err.scalar_type() == at::kInt && err.is_cuda(), "err must be a CUDA int32 tensor");
  long long* pdbg = nullptr;
  if (dbg.has_value() && dbg->defined()) {
    TORCH_CHECK(dbg->scalar_type() == at::kLong && dbg->numel() >= 8 * 64, "dbg must be int64 [>= 512]");
    pdbg = reinterpret_cast<long long*>(dbg->data_ptr<int64_t>());
  }
  for (auto* t : {&q, &k, &v})
    TORCH_CHECK((t->stride(0) * 2) % 16 == 0 && (t->stride(1) * 2) % 16 == 0, "TMA strides must be 16-byte multiples");
  const int rc = trida::bd_attn_fwd_sm100(a, reinterpret_cast<const int4*>(meta.data_ptr<int>()),
                                          list128.data_ptr<int16_t>(), cnt128.data_ptr<int>(),
                                          reinterpret_cast<const uint4*>(rowmask.data_ptr<int>()), (int)flags,
                                          (float)scale, err.data_ptr<int>(), stream(), pdbg);
  TORCH_CHECK(rc == 0, "bd_attn_fwd_sm100 failed (code ", rc, ", head_dim ", a.D, ")");
}

void bd_attn_bwd_sm100(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& o,
                       const at::Tensor& lse, const at::Tensor& dout, const at::Tensor& dq, const at::Tensor& dk,
                       const at::Tensor& dv, const at::Tensor& meta, const at::Tensor& list128t,
                       const at::Tensor& cnt128t, const at::Tensor& colmask, int64_t flags, double scale,
                       const at::Tensor& err,
                       const c10::optional<at::Tensor>& dbg,
                       const c10::optional<at::Tensor>& list128, const c10::optional<at::Tensor>& cnt128,
                       const c10::optional<at::Tensor>& rowmask) {
  auto a = attn_tensors(q, k, v, o, lse);
  if (a.D == 256) {
    // dK / dV kernel over the transposed lists + dQ kernel over the forward lists (bf16 dq directly)
    TORCH_CHECK(list128.has_value() && cnt128.has_value() && rowmask.has_value(),
                "head_dim 256 backward needs the forward tile lists and row masks");
    for (auto* t : {&dout, &dq, &dk, &dv})
      TORCH_CHECK(t->dim() == 4 && t->stride(3) == 1 && t->stride(2) == t->size(3), "attention grad layout");
    for (auto* t : {&dout, &dq})
      TORCH_CHECK((t->stride(0) * 2) % 16 == 0 && (t->stride(1) * 2) % 16 == 0 && ((uintptr_t)t->data_ptr() % 16) == 0,
                  "dout / dq must be TMA-compatible");
    auto dsum = at::empty({a.B, a.Hq, a.T}, lse.options());
    auto dkv_acc = at::empty({2, a.B, a.T, a.Hkv, a.D}, lse.options());
    float* dk_acc = dkv_acc.data_ptr<float>();
    float* dv_acc = dk_acc + (int64_t)a.B * a.T * a.Hkv * a.D;
    trida::bd_attn_bwd_prep(a, cbf(dout), dout.stride(1), dout.stride(0), dsum.data_ptr<float>(), nullptr, dk_acc,
                            dv_acc, sm_count(), stream());
    const int rc = trida::bd_attn_bwd_d256(
        a, cbf(dout), dout.stride(1), dout.stride(0), dsum.data_ptr<float>(), dk_acc, dv_acc, mbf(dq), dq.stride(1),
        dq.stride(0), list128t.data_ptr<int16_t>(), cnt128t.data_ptr<int>(),
        reinterpret_cast<const uint4*>(colmask.data_ptr<int>()), list128->data_ptr<int16_t>(), cnt128->data_ptr<int>(),
        reinterpret_cast<const uint4*>(rowmask->data_ptr<int>()), (float)scale, err.data_ptr<int>(), stream());
    TORCH_CHECK(rc == 0, "bd_attn_bwd_d256 failed (code ", rc, ")");
    trida::bd_attn_dq_convert(dk_acc, mbf(dk), dk.stride(1), dk.stride(0), a.B, a.T, a.Hkv, a.D, sm_count(), stream());
    trida::bd_attn_dq_convert(dv_acc, mbf(dv), dv.stride(1), dv.stride(0), a.B, a.T, a.Hkv, a.D, sm_count(), stream());
    return;
  }
  long long* pdbg = nullptr;
  if (dbg.has_value() && dbg->defined()) pdbg = reinterpret_cast<long long*>(dbg->data_ptr<int64_t>());
  for (auto* t : {&dout, &dq, &dk, &dv})
    TORCH_CHECK(t->dim() == 4 && t->stride(3) == 1 && t->stride(2) == t->size(3), "attention grad layout");
  TORCH_CHECK((dout.stride(0) * 2) % 16 == 0 && (dout.stride(1) * 2) % 16 == 0 &&
                  ((uintptr_t)dout.data_ptr() % 16) == 0, "dout must be TMA-compatible");
  auto dsum = at::empty({a.B, a.Hq, a.T}, lse.options());
  auto dq_acc = at::empty({a.B, a.T, a.Hq, a.D}, lse.options());
  // dK / dV partials of the GQA group's query heads meet in fp32 (one CTA per key tile and query head)
  // (zeroed, with dQ's accumulator, by the prologue kernel that computes Dsum)
  auto dkv_acc = at::empty({2, a.B, a.T, a.Hkv, a.D}, lse.options());
  float* dk_acc = dkv_acc.data_ptr<float>();
  float* dv_acc = dk_acc + (int64_t)a.B * a.T * a.Hkv * a.D;
  trida::bd_attn_bwd_prep(a, cbf(dout), dout.stride(1), dout.stride(0), dsum.data_ptr<float>(),
                          dq_acc.data_ptr<float>(), dk_acc, dv_acc, sm_count(), stream());
  const int rc = trida::bd_attn_bwd_sm100(a, cbf(dout), dout.stride(1), dout.stride(0), dsum.data_ptr<float>(),
                                          dq_acc.data_ptr<float>(), dk_acc, dv_acc, mbf(dk), dk.stride(1), dk.stride(0),
                                          mbf(dv), dv.stride(1), dv.stride(0),
                                          reinterpret_cast<const int4*>(meta.data_ptr<int>()),
                                          list128t.data_ptr<int16_t>(), cnt128t.data_ptr<int>(),
                                          reinterpret_cast<const uint4*>(colmask.data_ptr<int>()), (int)flags,
                                          (float)scale, err.data_ptr<int>(), stream(), pdbg);
  TORCH_CHECK(rc == 0, "bd_attn_bwd_sm100 failed (code ", rc, ", head_dim ", a.D, ")");
  trida::bd_attn_dq_convert(dq_acc.data_ptr<float>(), mbf(dq), dq.stride(1), dq.stride(0), a.B, a.T, a.Hq, a.D,
                            sm_count(), stream());
  trida::bd_attn_dq_convert(dk_acc, mbf(dk), dk.stride(1), dk.stride(0), a.B, a.T, a.Hkv, a.D, sm_count(), stream());
  trida::bd_attn_dq_convert(dv_acc, mbf(dv), dv.stride(1), dv.stride(0), a.B, a.T, a.Hkv, a.D, sm_count(), stream());
}

void ce_rows(const at::Tensor& logits, const at::Tensor& target, const c10::optional<at::Tensor>& weight,
             double grad_scale, const at::Tensor& loss, const c10::optional<at::Tensor>& dlogits) {
  CHECK_F32(logits); CHECK_ROWMAJOR(logits);
  TORCH_CHECK(target.scalar_type() == at::kLong && target.is_contiguous(), "target must be contiguous int64");
  TORCH_CHECK((logits.stride(0) % 4) == 0 && (logits.size(1) % 4) == 0, "logit rows must be float4-aligned");
  const float* pw = (weight.has_value() && weight->defined()) ? weight->data_ptr<float>() : nullptr;
  bf16* pd = nullptr; int64_t ldd = 0;
  if (dlogits.has_value() && dlogits->defined()) { CHECK_ROWMAJOR((*dlogits)); pd = mbf(*dlogits); ldd = dlogits->stride(0); }
  trida::ce_rows_fwd_bwd(logits.data_ptr<float>(), logits.stride(0), target.data_ptr<int64_t>(), pw,
                         (float)grad_scale, logits.size(0), logits.size(1), loss.data_ptr<float>(), pd, ldd,
                         stream());
}

// Global-norm clip: writes norm and clip coefficient (device scalars) from a list of fp32 buffers.
void grad_norm(const std::vector<at::Tensor>& grads, double max_norm, const at::Tensor& norm_out,
               const at::Tensor& coef_out) {
  const int per = 256;
  auto partial = at::empty({(int64_t)grads.size() * per}, norm_out.options());
  for (size_t i = 0; i < grads.size(); ++i) {
    CHECK_F32(grads[i]);
    TORCH_CHECK(grads[i].is_contiguous(), "grad buffers must be contiguous");
    trida::sumsq_partial(grads[i].data_ptr<float>(), grads[i].numel(), partial.data_ptr<float>() + i * per, per,
                         stream());
  }
  trida::clip_coef(partial.data_ptr<float>(), (int)grads.size() * per, (float)max_norm, norm_out.data_ptr<float>(),
                   coef_out.data_ptr<float>(), stream());
}

void adamw(const at::Tensor& param, const c10::optional<at::Tensor>& master, const at::Tensor& grad,
           const at::Tensor& m, const at::Tensor& v, double lr, double beta1, double beta2, double eps, double wd,
           int64_t step, const c10::optional<at::Tensor>& coef) {
  CHECK_F32(grad); CHECK_F32(m); CHECK_F32(v);
  TORCH_CHECK(grad.numel() == param.numel() && m.numel() == param.numel() && v.numel() == param.numel(), "size");
  const float* pc = (coef.has_value() && coef->defined()) ? coef->data_ptr<float>() : nullptr;
  if (master.has_value() && master->defined()) {
    CHECK_F32((*master));
    bf16* pb = param.scalar_type() == at::kBFloat16 ? mbf(param) : nullptr;
    trida::adamw_step(master->data_ptr<float>(), pb, grad.data_ptr<float>(), m.data_ptr<float>(),
                      v.data_ptr<float>(), param.numel(), lr, beta1, beta2, eps, wd, (int)step, pc, stream());
  } else if (param.scalar_type() == at::kFloat) {
    trida::adamw_step(param.data_ptr<float>(), nullptr, grad.data_ptr<float>(), m.data_ptr<float>(),
                      v.data_ptr<float>(), param.numel(), lr, beta1, beta2, eps, wd, (int)step, pc, stream());
  } else {
    CHECK_BF16(param);
    trida::adamw_step_bf16(mbf(param), grad.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(),
                           param.numel(), lr, beta1, beta2, eps, wd, (int)step, pc, stream());
  }
}

}  // namespace

static trida::GdnChunkParams chunk_params(const at::Tensor& mixed, const at::Tensor& ga, const at::Tensor& gb,
                                          const at::Tensor& A_log, const at::Tensor& dt_bias,
                                          const c10::optional<at::Tensor>& doc, const at::Tensor& o,
                                          std::vector<at::Tensor>& bufs, const at::Tensor& err,
                                          const std::vector<int64_t>& geo, double scale) {
  TORCH_CHECK(geo.size() == 10 && bufs.size() == 8, "gdn_chunk: geo / bufs size");
  const int64_t B = geo[0], T = geo[1], Hk = geo[2], Hv = geo[3], mode = geo[4], L = geo[5], V = geo[6], C = geo[7];
  auto q = gdn_params(mixed, ga, gb, A_log, dt_bias, doc, B, T, Hk, Hv, mode, L, V, C, geo[8] != 0, geo[9] != 0,
                      scale);
  TORCH_CHECK(C == 16 || C == 32 || C == 64, "chunk length must be 16, 32 or 64");
  const int64_t Lc = mode ? L : T;
  TORCH_CHECK(!mode || L % C == 0, "two-stream: the stream length must be a multiple of the block");
  TORCH_CHECK(mixed.stride(0) % 8 == 0, "mixed row stride must be a multiple of 8 (TMA)");
  TORCH_CHECK(Hv % Hk == 0, "value heads must be a multiple of key heads");
  const int64_t nch = (Lc + C - 1) / C;
  const int64_t rows = B * T;
  auto need = [&](const at::Tensor& t, at::ScalarType ty, int64_t n, const char* what) {
    CHECK_CUDA(t);
    TORCH_CHECK(t.scalar_type() == ty && t.is_contiguous() && t.numel() >= n, "gdn_chunk: bad buffer ", what);
  };
  need(bufs[0], at::kBFloat16, rows * Hk * 2 * 128, "qk");
  need(bufs[1], at::kFloat, rows * Hv * 2, "gb");
  for (int i = 2; i < 6; ++i) need(bufs[i], at::kBFloat16, rows * Hv * 128, "rows");
  need(bufs[6], at::kFloat, B * Hv * nch, "gamma");
  need(bufs[7], at::kBFloat16, B * Hv * nch * 128 * 128, "ckpt");
  CHECK_BF16(o); TORCH_CHECK(o.is_contiguous() && o.numel() == rows * Hv * 128, "o must be [B*T, Hv*128]");
  TORCH_CHECK(err.scalar_type() == at::kInt && err.is_cuda(), "err must be an int32 CUDA word");
  trida::GdnChunkParams p{};
  p.B = B; p.T = T; p.Hk = Hk; p.Hv = Hv; p.mode = mode; p.L = L; p.V = V; p.C = C; p.nch = nch;
  p.causal_clean = geo[8]; p.causal_noisy = geo[9];
  p.doc = q.doc; p.mixed = q.mixed; p.ldm = q.ldm; p.ga = q.ga; p.gbeta = q.gb; p.ldg = q.ldg;
  p.A_log = q.A_log; p.dt_bias = q.dt_bias; p.scale = (float)scale;
  p.qk = mbf(bufs[0]); p.gb = bufs[1].data_ptr<float>();
  p.wn = mbf(bufs[2]); p.ut = mbf(bufs[3]); p.kt = mbf(bufs[4]); p.u = mbf(bufs[5]);
  p.gamma = bufs[6].data_ptr<float>(); p.ckpt = mbf(bufs[7]); p.o = mbf(o);
  p.err = err.data_ptr<int>();
  return p;
}

// Chunked gated-delta forward (gdn_chunk.cu).  bufs = [qk (bf16 [B*T, Hk, 2, 128]), gb (fp32
// [B*T, Hv, 2]), wn, ut, kt, u (bf16 [B*T, Hv, 128] each), gamma (fp32 [B, Hv, nch]), ckpt (bf16
// [B, Hv, nch, 128, 128])]; geo = [B, T, Hk, Hv, mode, L, V, C, causal_clean, causal_noisy].
void gdn_chunk_fwd(const at::Tensor& mixed, const at::Tensor& ga, const at::Tensor& gb, const at::Tensor& A_log,
                   const at::Tensor& dt_bias, const c10::optional<at::Tensor>& doc, const at::Tensor& o,
                   std::vector<at::Tensor> bufs, const at::Tensor& err, std::vector<int64_t> geo, double scale,
                   const c10::optional<at::Tensor>& final_state) {
  auto p = chunk_params(mixed, ga, gb, A_log, dt_bias, doc, o, bufs, err, geo, scale);
  if (final_state.has_value() && final_state->defined()) {
    TORCH_CHECK(final_state->scalar_type() == at::kFloat && final_state->is_contiguous() &&
                final_state->numel() == (int64_t)p.B * p.Hv * 128 * 128, "final_state must be fp32 [B, Hv, 128, 128]");
    p.final_state = final_state->data_ptr<float>();
  }
  c10::cuda::CUDAGuard g(mixed.device());
  const int rc = trida::gdn_chunk_fwd(p, stream());
  TORCH_CHECK(rc == 0, "gdn_chunk_fwd failed with code ", rc);
}

// Chunked gated-delta backward (gdn_chunk_bwd.cu) from the forward's saved buffers.  Writes the
// q / k / v gradient columns of dmixed and the gate pre-activation gradients; accumulates dA_log /
// ddt_bias (fp32).
void gdn_chunk_bwd(const at::Tensor& mixed, const at::Tensor& ga, const at::Tensor& gb, const at::Tensor& A_log,
                   const at::Tensor& dt_bias, const c10::optional<at::Tensor>& doc, const at::Tensor& o,
                   std::vector<at::Tensor> bufs, const at::Tensor& err, std::vector<int64_t> geo, double scale,
                   const at::Tensor& d_o, const at::Tensor& dmixed, const at::Tensor& dga, const at::Tensor& dgb,
                   const at::Tensor& dA_log, const at::Tensor& ddt_bias) {
  trida::GdnChunkBwdParams p{};
  p.fwd = chunk_params(mixed, ga, gb, A_log, dt_bias, doc, o, bufs, err, geo, scale);
  const int64_t rows = (int64_t)p.fwd.B * p.fwd.T, Hv = p.fwd.Hv;
  CHECK_BF16(d_o); TORCH_CHECK(d_o.is_contiguous() && d_o.numel() == rows * Hv * 128, "d_o must be [B*T, Hv*128]");
  CHECK_BF16(dmixed); CHECK_ROWMAJOR(dmixed); CHECK_BF16(dga); CHECK_BF16(dgb); CHECK_ROWMAJOR(dga);
  TORCH_CHECK(dga.stride(0) == dgb.stride(0), "gate-gradient views must share a row stride");
  TORCH_CHECK(dA_log.scalar_type() == at::kFloat && ddt_bias.scalar_type() == at::kFloat, "fp32 gate grads");
  auto bf = mixed.options().dtype(at::kBFloat16);
  auto f32 = mixed.options().dtype(at::kFloat);
  const int64_t nstate = (int64_t)p.fwd.B * Hv * p.fwd.nch * 128 * 128;
  std::vector<at::Tensor> rowbufs;
  for (int i = 0; i < 7; ++i) rowbufs.push_back(at::empty({rows * Hv * 128}, bf));
  at::Tensor ds0 = at::empty({nstate}, bf), dckpt = at::empty({nstate}, bf);
  at::Tensor sc = at::empty({rows * Hv * 2}, f32), dpart = at::empty({rows * Hv * 260}, f32);
  p.d_o = cbf(d_o);
  p.du0 = mbf(rowbufs[0]); p.du = mbf(rowbufs[1]); p.qg = mbf(rowbufs[2]); p.dpe = mbf(rowbufs[3]);
  p.dae = mbf(rowbufs[4]); p.dw = mbf(rowbufs[5]); p.tt = mbf(rowbufs[6]);
  p.ds0 = mbf(ds0); p.dckpt = mbf(dckpt); p.sc = sc.data_ptr<float>(); p.dpart = dpart.data_ptr<float>();
  p.dmixed = mbf(dmixed); p.lddm = dmixed.stride(0);
  p.dga = mbf(dga); p.dgb = mbf(dgb); p.lddg = dga.stride(0);
  p.dA_log = dA_log.data_ptr<float>(); p.ddt_bias = ddt_bias.data_ptr<float>();
  c10::cuda::CUDAGuard g(mixed.device());
  const int rc = trida::gdn_chunk_bwd(p, stream());
  TORCH_CHECK(rc == 0, "gdn_chunk_bwd failed with code ", rc);
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "trida_stack_b200 sm_100a kernels";
  m.def("gemm", &gemm);
  m.def("gemm_swiglu", &gemm_swiglu, py::arg("A"), py::arg("B"), py::arg("D"), py::arg("act"),
        py::arg("tile") = 0);
  m.def("rmsnorm_fwd", &rmsnorm_fwd);
  m.def("rmsnorm_bwd", &rmsnorm_bwd);
  m.def("qk_norm_rope_fwd", &qk_norm_rope_fwd, py::arg("qkv"), py::arg("qw"), py::arg("kw"), py::arg("cos_t"),
        py::arg("sin_t"), py::arg("pos"), py::arg("q"), py::arg("k"), py::arg("Hq"), py::arg("Hkv"), py::arg("d"),
        py::arg("rd"), py::arg("eps"), py::arg("qstride") = 0);
  m.def("qk_norm_rope_bwd", &qk_norm_rope_bwd, py::arg("dq"), py::arg("dk"), py::arg("qkv"), py::arg("qw"),
        py::arg("kw"), py::arg("cos_t"), py::arg("sin_t"), py::arg("pos"), py::arg("rstd"), py::arg("dqkv"),
        py::arg("dqw"), py::arg("dkw"), py::arg("Hq"), py::arg("Hkv"), py::arg("d"), py::arg("rd"),
        py::arg("qstride") = 0);
  m.def("attn_gate_fwd", &attn_gate_fwd);
  m.def("attn_gate_bwd", &attn_gate_bwd);
  m.def("swiglu_fwd", &swiglu_fwd);
  m.def("swiglu_bwd", &swiglu_bwd);
  m.def("embed_fwd", &embed_fwd);
  m.def("embed_bwd", &embed_bwd);
  m.def("bd_attn_plan", &bd_attn_plan);
  m.def("bd_attn_fwd", &bd_attn_fwd);
  m.def("bd_attn_bwd", &bd_attn_bwd);
  m.def("bd_attn_lists128", &bd_attn_lists128);
  m.def("bd_attn_fwd_sm100", &bd_attn_fwd_sm100, py::arg("q"), py::arg("k"), py::arg("v"), py::arg("o"),
        py::arg("lse"), py::arg("meta"), py::arg("list128"), py::arg("cnt128"), py::arg("rowmask"), py::arg("flags"),
        py::arg("scale"), py::arg("err"), py::arg("dbg") = py::none());
  m.def("bd_attn_tile_masks", &bd_attn_tile_masks);
  m.def("gemm_error", &gemm_error);
  m.def("symm_malloc", &symm_malloc);
  m.def("symm_free", &symm_free);
  m.def("symm_handle", &symm_handle);
  m.def("symm_open", &symm_open);
  m.def("symm_close", &symm_close);
  m.def("symm_tensor", &symm_tensor);
  m.def("symm_rs_norm_ag", &symm_rs_norm_ag);
  m.def("symm_allreduce", &symm_allreduce);
  m.def("gemm_allreduce", &gemm_allreduce, py::arg("A"), py::arg("B"), py::arg("D"), py::arg("residual"),
        py::arg("recv"), py::arg("flags"), py::arg("rank"), py::arg("ctr_done"), py::arg("mcap"),
        py::arg("tiles_cap"), py::arg("ws") = py::none(), py::arg("tile_ctr") = py::none());
  m.def("symm_rs_sumsq", &symm_rs_sumsq, py::arg("bufs"), py::arg("flags"), py::arg("rank"), py::arg("epoch"),
        py::arg("shard_off"), py::arg("shard_len"), py::arg("scale"), py::arg("shard_out"), py::arg("partial"),
        py::arg("err"), py::arg("accumulate") = false, py::arg("done") = py::none(), py::arg("close_slot") = -1);
  m.def("symm_norm_coef", &symm_norm_coef);
  m.def("symm_adamw_ag", &symm_adamw_ag);
  m.def("symm_gather", &symm_gather);
  m.def("symm_gather_copy", &symm_gather_copy);
  m.def("symm_barrier", &symm_barrier);
  m.def("gdn_state_numel", &gdn_state_numel);
  m.def("gdn_chunk_fwd", &gdn_chunk_fwd);
  m.def("gdn_chunk_bwd", &gdn_chunk_bwd);
  m.def("gdn_fwd", &gdn_fwd, py::arg("mixed"), py::arg("ga"), py::arg("gb"), py::arg("A_log"), py::arg("dt_bias"),
        py::arg("doc"), py::arg("o"), py::arg("ckpt"), py::arg("B"), py::arg("T"), py::arg("Hk"), py::arg("Hv"),
        py::arg("mode"), py::arg("L"), py::arg("V"), py::arg("bd"), py::arg("causal_clean"), py::arg("causal_noisy"),
        py::arg("scale"), py::arg("final_state") = py::none());
  m.def("canvas_attention", &canvas_attention, py::arg("q"), py::arg("kc"), py::arg("vc"), py::arg("slot"),
        py::arg("pos"), py::arg("out"), py::arg("blk"), py::arg("n_clean"), py::arg("max_keys"), py::arg("scale"),
        py::arg("ptab") = py::none(), py::arg("err") = py::none());
  m.def("kv_append", &kv_append, py::arg("k"), py::arg("v"), py::arg("kc"), py::arg("vc"), py::arg("slot"),
        py::arg("pos"), py::arg("blk"), py::arg("ptab") = py::none());
  m.def("canvas_conv", &canvas_conv);
  m.def("conv_commit", &conv_commit);
  m.def("gdn_prep_numel", &gdn_prep_numel);
  m.def("gdn_canvas", &gdn_canvas);
  m.def("gdn_commit", &gdn_commit);
  m.def("gdn_canvas_tc", &gdn_canvas_tc, py::arg("mixed"), py::arg("ga"), py::arg("gb"), py::arg("A_log"),
        py::arg("dt_bias"), py::arg("o"), py::arg("kbuf"), py::arg("ubuf"), py::arg("gbuf"), py::arg("ssm"),
        py::arg("slot"), py::arg("blk"), py::arg("Hk"), py::arg("Hv"), py::arg("n_clean"), py::arg("scale"),
        py::arg("err"), py::arg("z") = py::none(), py::arg("gnorm_w") = py::none(), py::arg("eps") = 1e-6);
  m.def("spec_sample", &spec_sample);
  m.def("gemm_argmax", &gemm_argmax);
  m.def("gdn_commit_tc", &gdn_commit_tc);
  m.def("argmax_rows", &argmax_rows);
  m.def("conf_argmax_rows", &conf_argmax_rows);
  m.def("gdn_bwd", &gdn_bwd);
  m.def("gdn_conv_fwd", &gdn_conv_fwd);
  m.def("gdn_conv_bwd", &gdn_conv_bwd);
  m.def("gdn_gnorm_fwd", &gdn_gnorm_fwd);
  m.def("gdn_gnorm_bwd", &gdn_gnorm_bwd);
  m.def("bd_attn_bwd_sm100", &bd_attn_bwd_sm100, py::arg("q"), py::arg("k"), py::arg("v"), py::arg("o"),
        py::arg("lse"), py::arg("dout"), py::arg("dq"), py::arg("dk"), py::arg("dv"), py::arg("meta"),
        py::arg("list128t"), py::arg("cnt128t"), py::arg("colmask"), py::arg("flags"), py::arg("scale"), py::arg("err"),
        py::arg("dbg") = py::none(), py::arg("list128") = py::none(), py::arg("cnt128") = py::none(),
        py::arg("rowmask") = py::none());
  m.def("ce_rows", &ce_rows);
  m.def("grad_norm", &grad_norm);
  m.def("adamw", &adamw);
}
