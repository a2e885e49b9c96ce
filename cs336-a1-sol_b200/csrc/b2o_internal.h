// Internal (C++) interfaces shared by the translation units of libb2o.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>
#include <vector>

#include "../../include/b2o.h"

namespace b2o {

int num_sms();

// ---- streaming.cu
int adamw_step(const b2o_adamw_tensor* tensors, int ntensors, const b2o_adamw_group* groups,
               int ngroups, int param_dtype, int state_dtype, float ema_weight, cudaStream_t stream);
int ema_update(float* const* shadows, const void* const* params, const int64_t* numels, int nt,
               int param_dtype, float w, cudaStream_t stream);
int ema_copy_to_params(const float* const* shadows, void* const* params, const int64_t* numels, int nt,
                       int param_dtype, cudaStream_t stream);
int normuon_front_parts(int64_t rc);
int normuon_front(const void* const* grads, void* const* bufs, int S, int r, int c, int dtype,
                  float w_small, float w_large, int nesterov, uint16_t* U, float* partial,
                  cudaStream_t stream);
int normuon_apply(const uint16_t* O, const float* rowsq, int S, int r, int c, void* const* params,
                  uint16_t* const* rems, float* const* emas, float* const* vrows, int param_dtype,
                  float neg_lr, float lr_wd, float wd_factor, int wd_on, int cautious, float shape_scale,
                  float w_beta2, float ema_weight, float* scratch, cudaStream_t stream);
int normuon_front_multi(const b2o_normuon_batch* batches, int nb, int dtype, float w_small, float w_large,
                        int nesterov, const float* grad_scale, cudaStream_t stream);
int normuon_prescale(const b2o_normuon_batch* batches, int nb, int dtype, float w_small, float w_large,
                     int nesterov, const float* grad_scale, float norm_eps, float norm_safety, cudaStream_t stream);
// ---- clip.cu
int64_t clip_scratch_floats(const int64_t* numels, int n);
int clip_grad_norm(const void* const* grads, const int64_t* numels, const int* dtypes, int n, float max_norm,
                   float* scratch, float* out, cudaStream_t stream);
int clip_scale(void* const* grads, const int64_t* numels, const int* dtypes, int n, const float* coef,
               cudaStream_t stream);
int normuon_apply_multi(const b2o_normuon_batch* batches, int nb, int param_dtype, float neg_lr, float lr_wd,
                        float wd_factor, int wd_on, int cautious, float w_beta2, float ema_weight,
                        cudaStream_t stream);
int64_t normuon_apply_static_max_floats();
int normuon_apply_static(const uint16_t* O, const float* rowsq, int S, int r, int c, void* const* params,
                         uint16_t* const* rems, float* const* emas, float* const* vrows, int param_dtype,
                         float neg_lr, float lr_wd, float wd_factor, int wd_on, int cautious, float shape_scale,
                         float w_beta2, float ema_weight, cudaStream_t stream);

// ---- gemm.cu
// Operand view: element (row i, k) of an op(A) that is M x K (or op(B) that is N x K).
struct Operand {
  const uint16_t* ptr;
  int64_t ld;       // elements between consecutive stored rows
  int64_t stride;   // elements between batch entries
  int kmajor;       // 1: stored [i][k] (k contiguous); 0: stored [k][i] (i contiguous)
  int half;         // element type: 0 = bfloat16, 1 = binary16 (A and B must agree)
};
struct Epilogue {
  int kind;          // 0 scale, 1 poly (alpha*I + beta*C + gamma*acc), 2 quintic-B, 3 quintic-X
  float alpha, beta, gamma;
  const float* scale;  // per-batch factor on acc (kind 0), may be null
  const uint16_t* C;   // addend (kinds 1..3)
  int64_t ldc, strideC;
  uint16_t* D;
  int64_t ldd, strideD;
  int d_half;          // D (and C) element type: 0 = bfloat16, 1 = binary16
  float* rowsq;        // per-row partial sums of bf16(D)^2: [b][tile_n (256 wide)][M]
};
int gemm(const Operand& A, const Operand& B, const Epilogue& E, int M, int N, int K, int batch,
         int sym, cudaStream_t stream);
// Forces the CUDA-core path (tests compare both paths).
int gemm_simt(const Operand& A, const Operand& B, const Epilogue& E, int M, int N, int K, int batch,
              cudaStream_t stream);
bool gemm_tc_supported(const Operand& A, const Operand& B, const Epilogue& E, int M, int N, int K);

struct GemmTimer {
  static GemmTimer& instance();
  void before(cudaStream_t st, double flops);
  void after(cudaStream_t st);
  int read(double* ms, double* flops, int64_t* launches);
  bool enabled = false;
  struct Pair { cudaEvent_t a, b; double flops; };
  std::vector<Pair> pending;
  std::mutex mu;
};

// ---- ortho.cu
struct OrthoGroup {
  const uint16_t* U;       // front output (S, r, c): bf16 u, or binary16 X0 when xscale is set
  const float* partial;    // front sum-of-squares partials
  uint16_t* out;           // o (S, r, c) bf16
  float* rowsq;            // per-row partial sums of o^2
  int S, r, c;
  const float* xscale;     // Gram mode, prescaled X0: [S] s_norm / k, [S, 2S) squares; else null
};
int64_t ortho_workspace_bytes(int S, int r, int c);
int64_t ortho_workspace_bytes_multi(const OrthoGroup* g, int ng);
int orthogonalize_multi(const OrthoGroup* groups, int ng, int mode, const float* coeffs, int T, const int* resets,
                        int nresets, float norm_eps, float norm_safety, void* ws, int64_t ws_bytes,
                        cudaStream_t stream);
// orthogonalize_multi through the launch-graph cache (what the C ABI calls).
int orthogonalize_multi_cached(const OrthoGroup* groups, int ng, int mode, const float* coeffs, int T,
                               const int* resets, int nresets, float norm_eps, float norm_safety, void* ws,
                               int64_t ws_bytes, cudaStream_t stream);
int set_launch_graphs(int enable);  // returns the previous setting
void launch_graph_stats(int64_t* captures, int64_t* replays, int64_t* failures);
int orthogonalize(const uint16_t* U, const float* partial, int S, int r, int c, int mode,
                  const float* coeffs, int T, const int* resets, int nresets, float norm_eps,
                  float norm_safety, void* ws, int64_t ws_bytes, uint16_t* out, float* rowsq,
                  cudaStream_t stream);

}  // namespace b2o
