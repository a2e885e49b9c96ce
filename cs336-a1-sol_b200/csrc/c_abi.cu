// extern "C" entry points of libb2o (declared in include/b2o.h) and the
// library-wide plumbing: error text, launch counter, device error word.
#include "b2o_common.cuh"
#include "b2o_internal.h"

#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

namespace b2o {

std::atomic<int64_t> g_launches{0};
thread_local int64_t* t_capture_launches = nullptr;
static thread_local std::string t_last_error;

void set_error(const std::string& msg) { t_last_error = msg; }

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("B2O_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error(std::string(what) + ": " + cudaGetErrorString(e));
    return static_cast<int>(e);
  }
  return 0;
}

// The device error word lives in statically allocated device memory (no
// cudaMalloc); kernels receive its address as an argument.
__device__ int g_device_error;

constexpr int kMaxDevices = 64;
static int* g_err_ptr[kMaxDevices];
static int g_sms[kMaxDevices];
static std::mutex g_mu;

int* device_error_word() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_err_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) return nullptr;
    g_err_ptr[dev] = static_cast<int*>(p);
  }
  return g_err_ptr[dev];
}

int num_sms() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_sms[dev]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    g_sms[dev] = n;
  }
  return g_sms[dev];
}

}  // namespace b2o

using namespace b2o;

extern "C" {

int b2o_version(void) { return 1; }

int b2o_last_error(char* buf, int buflen) {
  if (!buf || buflen <= 0) return static_cast<int>(t_last_error.size());
  const int n = std::min<int>(buflen - 1, static_cast<int>(t_last_error.size()));
  memcpy(buf, t_last_error.data(), n);
  buf[n] = 0;
  return n;
}

int64_t b2o_launch_count(void) { return g_launches.load(); }

int b2o_num_sms(void) { return num_sms(); }

int b2o_launch_graphs(int enable) { return set_launch_graphs(enable); }

int b2o_launch_graph_stats(int64_t* captures, int64_t* replays, int64_t* failures) {
  launch_graph_stats(captures, replays, failures);
  return 0;
}

int b2o_gemm_timing(int enable) {
  GemmTimer::instance().enabled = enable != 0;
  return 0;
}

int b2o_gemm_timing_read(double* ms, double* flops, int64_t* launches) {
  return GemmTimer::instance().read(ms, flops, launches);
}

int b2o_check_device_error(void* stream) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) { set_error(std::string("sync: ") + cudaGetErrorString(e)); return -static_cast<int>(e); }
  int* w = device_error_word();
  if (!w) { set_error("no device error word"); return -1; }
  int val = 0;
  e = cudaMemcpyAsync(&val, w, sizeof(int), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) { set_error(std::string("read error word: ") + cudaGetErrorString(e)); return -static_cast<int>(e); }
  if (val) {
    const int zero = 0;
    cudaMemcpyAsync(w, &zero, sizeof(int), cudaMemcpyHostToDevice, st);
    cudaStreamSynchronize(st);
    set_error("device error word = " + std::to_string(val));
  }
  return val;
}

int b2o_adamw_step(const b2o_adamw_tensor* tensors, int ntensors, const b2o_adamw_group* groups, int ngroups,
                   int param_dtype, int state_dtype, float ema_weight, void* stream) {
  return adamw_step(tensors, ntensors, groups, ngroups, param_dtype, state_dtype, ema_weight,
                    static_cast<cudaStream_t>(stream));
}

int b2o_ema_update(float* const* shadows, const void* const* params, const int64_t* numels, int ntensors,
                   int param_dtype, float weight, void* stream) {
  return ema_update(shadows, params, numels, ntensors, param_dtype, weight, static_cast<cudaStream_t>(stream));
}

int b2o_ema_copy_to_params(const float* const* shadows, void* const* params, const int64_t* numels, int ntensors,
                           int param_dtype, void* stream) {
  return ema_copy_to_params(shadows, params, numels, ntensors, param_dtype, static_cast<cudaStream_t>(stream));
}

int b2o_normuon_front_parts(int64_t rc) { return normuon_front_parts(rc); }

int b2o_normuon_front(const void* const* d_grads, void* const* d_bufs, int S, int r, int c, int dtype,
                      float w_small, float w_large, int nesterov, uint16_t* d_u, float* d_partial, void* stream) {
  return normuon_front(d_grads, d_bufs, S, r, c, dtype, w_small, w_large, nesterov, d_u, d_partial,
                       static_cast<cudaStream_t>(stream));
}

int64_t b2o_ortho_workspace_bytes(int S, int r, int c) { return ortho_workspace_bytes(S, r, c); }

int b2o_orthogonalize(const uint16_t* d_u, const float* d_partial, int S, int r, int c, int mode,
                      const float* coeffs, int T, const int* resets, int nresets, float norm_eps, float norm_safety,
                      void* d_ws, int64_t ws_bytes, uint16_t* d_out, float* d_rowsq, void* stream) {
  return orthogonalize(d_u, d_partial, S, r, c, mode, coeffs, T, resets, nresets, norm_eps, norm_safety, d_ws,
                       ws_bytes, d_out, d_rowsq, static_cast<cudaStream_t>(stream));
}

static std::vector<OrthoGroup> to_groups(const b2o_ortho_group* g, int ng) {
  std::vector<OrthoGroup> v;
  for (int i = 0; i < ng; ++i)
    v.push_back(OrthoGroup{g[i].u, g[i].partial, g[i].out, g[i].rowsq, g[i].S, g[i].r, g[i].c, g[i].xscale});
  return v;
}

int64_t b2o_ortho_workspace_bytes_multi(const b2o_ortho_group* groups, int ngroups) {
  if (!groups || ngroups <= 0) return -1;
  auto v = to_groups(groups, ngroups);
  return ortho_workspace_bytes_multi(v.data(), ngroups);
}

int b2o_orthogonalize_multi(const b2o_ortho_group* groups, int ngroups, int mode, const float* coeffs, int T,
                            const int* resets, int nresets, float norm_eps, float norm_safety, void* d_ws,
                            int64_t ws_bytes, void* stream) {
  if (!groups || ngroups <= 0) { set_error("orthogonalize: no groups"); return -1; }
  auto v = to_groups(groups, ngroups);
  return orthogonalize_multi_cached(v.data(), ngroups, mode, coeffs, T, resets, nresets, norm_eps, norm_safety,
                                    d_ws, ws_bytes, static_cast<cudaStream_t>(stream));
}

int64_t b2o_normuon_apply_scratch_floats(int S, int r) {
  return static_cast<int64_t>(S) * (static_cast<int64_t>(r) + 4);
}

int b2o_normuon_apply(const uint16_t* d_o, const float* d_rowsq, int S, int r, int c, void* const* params,
                      uint16_t* const* rems, float* const* emas, float* const* vrows, int param_dtype, float neg_lr,
                      float lr_wd, float wd_factor, int wd_on, int cautious, float shape_scale, float w_beta2,
                      float ema_weight, float* d_scratch, void* stream) {
  return normuon_apply(d_o, d_rowsq, S, r, c, params, rems, emas, vrows, param_dtype, neg_lr, lr_wd, wd_factor,
                       wd_on, cautious, shape_scale, w_beta2, ema_weight, d_scratch,
                       static_cast<cudaStream_t>(stream));
}

int b2o_normuon_front_multi(const b2o_normuon_batch* batches, int nbatches, int dtype, float w_small,
                            float w_large, int nesterov, const float* d_grad_scale, void* stream) {
  return normuon_front_multi(batches, nbatches, dtype, w_small, w_large, nesterov, d_grad_scale,
                             static_cast<cudaStream_t>(stream));
}

int b2o_normuon_prescale(const b2o_normuon_batch* batches, int nbatches, int dtype, float w_small, float w_large,
                         int nesterov, const float* d_grad_scale, float norm_eps, float norm_safety, void* stream) {
  return normuon_prescale(batches, nbatches, dtype, w_small, w_large, nesterov, d_grad_scale, norm_eps, norm_safety,
                          static_cast<cudaStream_t>(stream));
}

int64_t b2o_clip_scratch_floats(const int64_t* numels, int n) { return clip_scratch_floats(numels, n); }

int b2o_clip_grad_norm(const void* const* d_grads, const int64_t* numels, const int* dtypes, int n,
                       float max_norm, float* d_scratch, float* d_out, void* stream) {
  return clip_grad_norm(d_grads, numels, dtypes, n, max_norm, d_scratch, d_out, static_cast<cudaStream_t>(stream));
}

int b2o_clip_scale(void* const* d_grads, const int64_t* numels, const int* dtypes, int n, const float* d_coef,
                   void* stream) {
  return clip_scale(d_grads, numels, dtypes, n, d_coef, static_cast<cudaStream_t>(stream));
}

int b2o_normuon_apply_multi(const b2o_normuon_batch* batches, int nbatches, int param_dtype, float neg_lr,
                            float lr_wd, float wd_factor, int wd_on, int cautious, float w_beta2, float ema_weight,
                            void* stream) {
  return normuon_apply_multi(batches, nbatches, param_dtype, neg_lr, lr_wd, wd_factor, wd_on, cautious, w_beta2,
                             ema_weight, static_cast<cudaStream_t>(stream));
}

int64_t b2o_normuon_apply_static_max_floats(void) { return normuon_apply_static_max_floats(); }

int b2o_normuon_apply_static(const uint16_t* d_o, const float* d_rowsq, int S, int r, int c, void* const* params,
                             uint16_t* const* rems, float* const* emas, float* const* vrows, int param_dtype,
                             float neg_lr, float lr_wd, float wd_factor, int wd_on, int cautious, float shape_scale,
                             float w_beta2, float ema_weight, void* stream) {
  return normuon_apply_static(d_o, d_rowsq, S, r, c, params, rems, emas, vrows, param_dtype, neg_lr, lr_wd,
                              wd_factor, wd_on, cautious, shape_scale, w_beta2, ema_weight,
                              static_cast<cudaStream_t>(stream));
}

int b2o_gemm(const uint16_t* d_A, int64_t lda, int64_t strideA, int a_kmajor, const uint16_t* d_B, int64_t ldb,
             int64_t strideB, int b_kmajor, uint16_t* d_D, int64_t ldd, int64_t strideD, const uint16_t* d_C,
             int64_t ldc, int64_t strideC, int M, int N, int K, int batch, int in_dtype, int out_dtype, int epi, int sym,
             float alpha, float beta, float gamma, const float* d_scale, float* d_rowsq, void* stream) {
  if ((in_dtype != B2O_BF16 && in_dtype != B2O_F16) || (out_dtype != B2O_BF16 && out_dtype != B2O_F16)) {
    set_error("gemm: dtypes must be B2O_BF16 or B2O_F16"); return -1;
  }
  Operand A{d_A, lda, strideA, a_kmajor ? 1 : 0, in_dtype == B2O_F16};
  Operand B{d_B, ldb, strideB, b_kmajor ? 1 : 0, in_dtype == B2O_F16};
  Epilogue e;
  memset(&e, 0, sizeof(e));
  e.kind = epi; e.alpha = alpha; e.beta = beta; e.gamma = gamma; e.scale = d_scale;
  e.C = d_C; e.ldc = ldc; e.strideC = strideC; e.D = d_D; e.ldd = ldd; e.strideD = strideD; e.rowsq = d_rowsq;
  e.d_half = out_dtype == B2O_F16;
  return gemm(A, B, e, M, N, K, batch, sym, static_cast<cudaStream_t>(stream));
}

int b2o_gemm_bf16(const uint16_t* d_A, int64_t lda, int64_t strideA, int a_kmajor, const uint16_t* d_B, int64_t ldb,
                  int64_t strideB, int b_kmajor, uint16_t* d_D, int64_t ldd, int64_t strideD, const uint16_t* d_C,
                  int64_t ldc, int64_t strideC, int M, int N, int K, int batch, int epi, int sym, float alpha,
                  float beta, float gamma, const float* d_scale, float* d_rowsq, void* stream) {
  return b2o_gemm(d_A, lda, strideA, a_kmajor, d_B, ldb, strideB, b_kmajor, d_D, ldd, strideD, d_C, ldc, strideC, M,
                  N, K, batch, B2O_BF16, B2O_BF16, epi, sym, alpha, beta, gamma, d_scale, d_rowsq, stream);
}

/* Test hook: the same GEMM on the CUDA-core path (no tensor cores). */
int b2o_gemm_bf16_simt(const uint16_t* d_A, int64_t lda, int64_t strideA, int a_kmajor, const uint16_t* d_B,
                       int64_t ldb, int64_t strideB, int b_kmajor, uint16_t* d_D, int64_t ldd, int64_t strideD,
                       const uint16_t* d_C, int64_t ldc, int64_t strideC, int M, int N, int K, int batch, int epi,
                       float alpha, float beta, float gamma, const float* d_scale, float* d_rowsq, void* stream) {
  Operand A{d_A, lda, strideA, a_kmajor ? 1 : 0};
  Operand B{d_B, ldb, strideB, b_kmajor ? 1 : 0};
  Epilogue e;
  memset(&e, 0, sizeof(e));
  e.kind = epi; e.alpha = alpha; e.beta = beta; e.gamma = gamma; e.scale = d_scale;
  e.C = d_C; e.ldc = ldc; e.strideC = strideC; e.D = d_D; e.ldd = ldd; e.strideD = strideD; e.rowsq = d_rowsq;
  if (M <= 0 || N <= 0 || K <= 0 || batch <= 0 || !d_A || !d_B || !d_D) { set_error("gemm_simt: bad args"); return -1; }
  return gemm_simt(A, B, e, M, N, K, batch, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
