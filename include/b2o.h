/*
 * b2o.h — C ABI of the B200 optimizer-step engine (libb2o.so).
 *
 * The engine replaces the optimizer step that the reference training loop runs
 * after loss.backward() (transformer_lm/train_sol.py:500-507):
 *   muon.step()   -> NorMuonGNS.step            transformer_lm/sol_modules.py:372-425
 *   adamw.step()  -> torch.optim.AdamW(fused)   transformer_lm/sol_modules.py:476
 *   ema.update()  -> EmaWeights.update          transformer_lm/sol_modules.py:1255-1268
 *
 * Conventions
 *   - Every pointer argument named d_* is a device pointer owned by the caller
 *     (PyTorch's caching allocator in the Python host layer). The library never
 *     allocates, frees or synchronises device memory on its own, except inside
 *     b2o_check_device_error(), which synchronises the given stream.
 *   - `stream` is a cudaStream_t passed as void*; work is enqueued on it and the
 *     call returns without waiting.
 *   - Return value: 0 = ok; negative = invalid argument detected on the host
 *     (nothing was launched; b2o_last_error() has the message); positive = a
 *     CUDA launch/runtime error code.
 *   - Device-side failures (a bounded wait that ran out) set a device error word
 *     instead of trapping; b2o_check_device_error() reads and clears it.
 *   - dtype codes: B2O_F32 = 0, B2O_BF16 = 1, B2O_F16 = 2 (IEEE binary16).
 */
#ifndef B2O_H_
#define B2O_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define B2O_F32 0
#define B2O_BF16 1
#define B2O_F16 2

/* Error/status plumbing (no reference counterpart: the reference raises Python
 * exceptions from torch; these carry the same information across the C ABI). */
int b2o_version(void);
int b2o_last_error(char* buf, int buflen);
/* Number of kernels this library has launched since load (monotonic). */
int64_t b2o_launch_count(void);
/* Synchronises `stream`, returns the device error word (0 = none) and clears it. */
int b2o_check_device_error(void* stream);
/* Number of SMs of the current device (used by the host layer for grid sizing). */
int b2o_num_sms(void);
/* Measurement hooks (no reference counterpart): when enabled, every
 * tensor-core GEMM launch is bracketed by CUDA events on its stream;
 * b2o_gemm_timing_read synchronises on them and returns the summed device
 * time, the launches' algorithmic FLOPs (symmetric outputs at half) and the
 * number of launches since the previous read. */
/* Launch graphs (no reference counterpart): the second orthogonaliser call
 * with a given argument set is captured into a CUDA graph and later calls with
 * the same arguments replay it (same kernels, arguments and order; one host
 * launch instead of ~30). b2o_launch_graphs(0) turns this off (as does
 * B2O_GRAPHS=0 in the environment) and returns the previous setting;
 * b2o_launch_graph_stats reports graphs captured, replays and failed captures
 * (whose argument sets then launch directly). */
int b2o_launch_graphs(int enable);
int b2o_launch_graph_stats(int64_t* captures, int64_t* replays, int64_t* failures);
int b2o_gemm_timing(int enable);
int b2o_gemm_timing_read(double* ms, double* flops, int64_t* launches);

/* ------------------------------------------------------------------------ *
 * Fused AdamW (+ optional EMA) over a list of tensors.
 * Replaces torch.optim.AdamW(groups, betas, eps, fused=True)
 * (transformer_lm/sol_modules.py:468-476; math torch/optim/adam.py:347-547 and
 * the fused kernel formula in ATen/native/cuda/fused_adam_utils.cuh) and, when
 * `ema` is non-NULL, EmaWeights.update for the same tensors
 * (transformer_lm/sol_modules.py:1267-1268).
 * ------------------------------------------------------------------------ */
typedef struct {
  void* param;          /* param_dtype, numel elements                       */
  uint16_t* rem;        /* bf16 bit pattern of the low-mantissa remainder or NULL */
  const void* grad;     /* param_dtype                                        */
  void* exp_avg;        /* state_dtype                                        */
  void* exp_avg_sq;     /* state_dtype                                        */
  float* ema;           /* fp32 EMA shadow or NULL                            */
  int64_t numel;
  int32_t group;        /* index into the group table                         */
  int32_t _pad;
  float* step_out;      /* 0-d fp32 step tensor (torch's state["step"]) that the
                           pass sets to the group's step, or NULL             */
} b2o_adamw_tensor;

typedef struct {
  float lr;
  float beta1;
  float beta2;
  float eps;
  float weight_decay;
  float lr_wd;          /* fp32(lr * weight_decay), rounded once on the host  */
  float step;           /* step count after increment (torch's state["step"]) */
  int32_t cautious;     /* 1: decay only where update * w > 0                 */
  const float* grad_scale;  /* device pointer to a gradient-clip coefficient
                               (b2o_clip_grad_norm's d_out + 1) applied as
                               g = dtype(g * coef) before the update, or NULL */
} b2o_adamw_group;

/* param_dtype: B2O_F32 or B2O_BF16. state_dtype: B2O_F32 or B2O_BF16 (must equal
 * param_dtype unless param is bf16 and state is fp32). rem must be NULL unless
 * param_dtype is bf16. ema_weight = fp32(1 - decay); ignored where ema == NULL. */
int b2o_adamw_step(const b2o_adamw_tensor* tensors, int ntensors,
                   const b2o_adamw_group* groups, int ngroups,
                   int param_dtype, int state_dtype, float ema_weight, void* stream);

/* Stand-alone EMA: shadow = lerp(shadow, float(param), weight) for each tensor.
 * Replaces EmaWeights.update/_update_slow (transformer_lm/sol_modules.py:1255-1268). */
int b2o_ema_update(float* const* shadows, const void* const* params, const int64_t* numels,
                   int ntensors, int param_dtype, float weight, void* stream);

/* EMA swap for evaluation: param = param_dtype(shadow) for each tensor
 * (EmaWeights.averaged, transformer_lm/sol_modules.py:1270-1280; the backup and
 * restore are plain device copies done by the caller). */
int b2o_ema_copy_to_params(const float* const* shadows, void* const* params,
                           const int64_t* numels, int ntensors, int param_dtype,
                           void* stream);

/* ------------------------------------------------------------------------ *
 * NorMuon, one shape-batch of S matrices of shape (r, c).
 * Replaces the per-shape body of NorMuonGNS.step (transformer_lm/sol_modules.py:384-424).
 * ------------------------------------------------------------------------ */

/* Front: buf = lerp(buf, g, 1-beta); u = nesterov ? lerp(g, buf, beta) : buf
 * (sol_modules.py:390-394). Writes d_u (S, r, c) bf16 in the original layout and
 * per-matrix partial sums of bf16(u)^2 into d_partial (S * nparts floats, nparts
 * from b2o_normuon_front_parts). dtype is the param/grad/momentum dtype. */
int b2o_normuon_front_parts(int64_t rc);
int b2o_normuon_front(const void* const* d_grads, void* const* d_bufs, int S, int r, int c,
                      int dtype, float w_small, float w_large, int nesterov,
                      uint16_t* d_u, float* d_partial, void* stream);

/* Workspace needed by b2o_orthogonalize for a batch (bytes). */
int64_t b2o_ortho_workspace_bytes(int S, int r, int c);

/* Orthogonaliser (sol_modules.py:366-370; fallback 278-293).
 *   mode 0 = quintic Newton-Schulz restated from the reference's fallback
 *            (zeropower_via_newtonschulz5): coefficients[0..2] used every step;
 *   mode 1 = Gram Newton-Schulz on the m x m Gram matrix with a per-step
 *            coefficient table coeffs[3*T] and restart steps `resets`.
 * d_u (S, r, c) bf16 is the front output (read only); d_partial is the front's
 * sum-of-squares partials; the result o (S, r, c) bf16, original layout, goes to
 * d_out, and per-row partial sums of o^2 go to d_rowsq (S * r * ceil(c/256)).
 * norm_eps is added to the Frobenius norm; norm_safety multiplies it. */
int b2o_orthogonalize(const uint16_t* d_u, const float* d_partial, int S, int r, int c,
                      int mode, const float* coeffs, int T, const int* resets, int nresets,
                      float norm_eps, float norm_safety,
                      void* d_ws, int64_t ws_bytes, uint16_t* d_out, float* d_rowsq,
                      void* stream);

/* Several shape-batches that share m = min(r, c) in one call: the m x m
 * products of every group run as single batched GEMMs (the reference calls
 * its orthogonaliser once per exact shape, sol_modules.py:380-395; grouping by
 * m only changes launch granularity, not any matrix's arithmetic). */
typedef struct {
  const uint16_t* u;      /* front output (S, r, c): bf16 u, or binary16 X0 (xscale != NULL) */
  const float* partial;   /* front sum-of-squares partials          */
  uint16_t* out;          /* o (S, r, c) bf16                        */
  float* rowsq;           /* S * r * ceil(c/256) floats              */
  int32_t S, r, c, _pad;
  const float* xscale;    /* Gram mode: u holds X0 = binary16(u * k) with a per-matrix power of two k
                             (b2o_normuon_prescale); xscale[s] = s_norm / k, xscale[S + s] = its square;
                             NULL: u is the bf16 front output */
} b2o_ortho_group;
int64_t b2o_ortho_workspace_bytes_multi(const b2o_ortho_group* groups, int ngroups);
int b2o_orthogonalize_multi(const b2o_ortho_group* groups, int ngroups, int mode,
                            const float* coeffs, int T, const int* resets, int nresets,
                            float norm_eps, float norm_safety, void* d_ws, int64_t ws_bytes,
                            void* stream);

/* Finish + apply (sol_modules.py:396-424): v_row lerp, row/matrix scaling,
 * shape scale, cautious weight decay, update, bf16 mantissa split, EMA.
 *   params/rems/emas/vrows: S pointers each (rems/emas may be NULL arrays)
 *   param_dtype: B2O_F32 or B2O_BF16; rems non-NULL only for bf16 (bf16_master)
 *   neg_lr = fp32(-lr); lr_wd = fp32(lr*wd) (cautious factor 1 - lr_wd*mask);
 *   wd_factor = fp32(1 - lr*wd) (plain decay); wd_on, cautious flags;
 *   shape_scale = fp32(sqrt(max(1, r/c))); w_beta2 = fp32(1-beta2);
 *   ema_weight = fp32(1-decay)
 *   d_scratch: S * (r + 4) floats of scratch. */
int64_t b2o_normuon_apply_scratch_floats(int S, int r);
int b2o_normuon_apply(const uint16_t* d_o, const float* d_rowsq, int S, int r, int c,
                      void* const* params, uint16_t* const* rems, float* const* emas,
                      float* const* vrows, int param_dtype,
                      float neg_lr, float lr_wd, float wd_factor, int wd_on, int cautious,
                      float shape_scale, float w_beta2, float ema_weight,
                      float* d_scratch, void* stream);

/* All shape batches of one NorMuon parameter group in one call each (one
 * launch for the front, one each for the finish and apply passes, instead of
 * one per batch). Same per-matrix arithmetic as b2o_normuon_front and
 * b2o_normuon_apply; the reference's per-shape loop is
 * transformer_lm/sol_modules.py:380-424. Up to 16 batches and 128 matrices
 * per call; the apply call needs a remainder for every batch or for none. */
typedef struct b2o_normuon_batch {
  int S, r, c;                  /* S matrices of r x c */
  float shape_scale;            /* apply: sqrt(max(1, r / c)) (sol_modules.py:401) */
  const void* const* grads;     /* front: S gradients (param dtype) */
  void* const* bufs;            /* front: S momentum buffers */
  uint16_t* u;                  /* front output: S*r*c bf16 */
  float* partial;               /* front output: S * b2o_normuon_front_parts(r*c) */
  const uint16_t* o;            /* apply input: S*r*c bf16 orthogonaliser output */
  const float* rowsq;           /* apply input: [S][ceil(c/256)][r] row sums of o^2 */
  void* const* params;          /* apply: S params */
  uint16_t* const* rems;        /* apply: S bf16 remainders, or NULL */
  float* const* emas;           /* apply: S fp32 EMA shadows, or NULL */
  float* const* vrows;          /* apply: S fp32 (r, 1) second moments */
  float* scratch;               /* apply: b2o_normuon_apply_scratch_floats(S, r) floats */
  float* prescale;              /* front, x0_half: S per-matrix powers of two k (kept across steps; 0 = none) */
  float* xscale;                /* b2o_normuon_prescale output: 2 * S factors for b2o_ortho_group.xscale */
  int32_t* flags;               /* b2o_normuon_prescale scratch: S ints */
  int32_t x0_half;              /* front: write X0 = binary16(bf16(u) * k) instead of bf16 u */
  int32_t _pad;
} b2o_normuon_batch;
/* d_grad_scale: device pointer to a gradient-clip coefficient applied as
 * g = dtype(g * coef) when the gradients are read, or NULL. */
int b2o_normuon_front_multi(const b2o_normuon_batch* batches, int nbatches, int dtype, float w_small,
                            float w_large, int nesterov, const float* d_grad_scale, void* stream);
/* Gram-mode input without a conversion pass: a front call with x0_half writes
 * X0 = binary16(bf16(u) * k), k = prescale[s] (a power of two near 256 / ||u||
 * of the previous step, so the conversion is exact); this call then computes
 * this step's s_norm = 1 / (||u|| * safety + eps) from the partials, the
 * factors s_norm / k for the orthogonaliser, and next step's k, and rewrites
 * X0 of every matrix whose norm left k's range (factor 64 either way; every
 * matrix on the first step) from its gradient and momentum buffer. Arguments
 * as for the front call that preceded it. */
int b2o_normuon_prescale(const b2o_normuon_batch* batches, int nbatches, int dtype, float w_small, float w_large,
                         int nesterov, const float* d_grad_scale, float norm_eps, float norm_safety, void* stream);
int b2o_normuon_apply_multi(const b2o_normuon_batch* batches, int nbatches, int param_dtype, float neg_lr,
                            float lr_wd, float wd_factor, int wd_on, int cautious, float w_beta2,
                            float ema_weight, void* stream);

/* Allocation-free form of b2o_normuon_apply. No counterpart in the reference
 * (its optimizer allocates its temporaries through PyTorch).
 * For hosts that cannot hand the library a scratch buffer: a caller whose
 * device memory is entirely reserved up front by another allocator, or a
 * runtime that forbids allocating while its step is in flight. The
 * S * (r + 4) floats of scratch come from a 1 MiB array inside the library
 * (b2o_normuon_apply_static_max_floats() = 262144 floats); larger batches are
 * rejected with a negative status and a message, nothing launched. The library
 * allocates nothing: the first call on a device looks up the array's device
 * address (cudaGetSymbolAddress, once per device, with that device current),
 * so make that first call before any stream capture. The address is cached
 * for the life of the device's primary context: after a cudaDeviceReset in
 * the same process, do not call this entry point again. All calls share the one
 * array per device: two calls whose kernels overlap on the GPU (different
 * streams, no ordering between them) race on it. Every scratch value the
 * kernels read is written earlier in the same call, so no clearing is needed.
 * Arguments and results are those of b2o_normuon_apply without d_scratch. */
int64_t b2o_normuon_apply_static_max_floats(void);
int b2o_normuon_apply_static(const uint16_t* d_o, const float* d_rowsq, int S, int r, int c,
                             void* const* params, uint16_t* const* rems, float* const* emas,
                             float* const* vrows, int param_dtype,
                             float neg_lr, float lr_wd, float wd_factor, int wd_on, int cautious,
                             float shape_scale, float w_beta2, float ema_weight, void* stream);

/* ------------------------------------------------------------------------ *
 * Batched bf16 GEMM on tcgen05 (exposed for tests and the micro-benchmark).
 * D[b] = epilogue(op(A[b]) * op(B[b])), fp32 accumulation in tensor memory.
 *   A is M x K: a_kmajor=1 -> stored row-major (M rows, K contiguous, lda);
 *                a_kmajor=0 -> stored as K x M (M contiguous, lda).
 *   B is N x K: b_kmajor=1 -> stored N rows with K contiguous (D = A * B^T);
 *                b_kmajor=0 -> stored K x N (N contiguous, D = A * B).
 *   epi: 0 = D = alpha * acc; 1 = D = alpha*I + beta*C + gamma*acc (P polynomial);
 *        2 = D = bf16(bf16(beta*C) + bf16(gamma*bf16(acc)))  (quintic B);
 *        3 = D = bf16(bf16(alpha*C) + bf16(acc))             (quintic X update).
 *   sym: 1 -> output is symmetric, only tiles touching the upper triangle are
 *        computed and each is mirrored (M must equal N).
 *   d_scale: optional per-batch multiplier on acc (NULL = 1).
 *   d_rowsq: optional per-row partial sums of bf16(D)^2, layout [b][tile_n][M].
 * ------------------------------------------------------------------------ */
int b2o_gemm_bf16(const uint16_t* d_A, int64_t lda, int64_t strideA, int a_kmajor,
                  const uint16_t* d_B, int64_t ldb, int64_t strideB, int b_kmajor,
                  uint16_t* d_D, int64_t ldd, int64_t strideD,
                  const uint16_t* d_C, int64_t ldc, int64_t strideC,
                  int M, int N, int K, int batch, int epi, int sym,
                  float alpha, float beta, float gamma, const float* d_scale,
                  float* d_rowsq, void* stream);

/* General form: in_dtype (A, B and C) and out_dtype (D) are B2O_BF16 or
 * B2O_F16; epilogues 2 and 3 need bf16 throughout. b2o_gemm_bf16 is this call
 * with both dtypes bf16. No reference counterpart (the reference multiplies
 * with torch.matmul / the gram-newton-schulz package). */
int b2o_gemm(const uint16_t* d_A, int64_t lda, int64_t strideA, int a_kmajor,
             const uint16_t* d_B, int64_t ldb, int64_t strideB, int b_kmajor,
             uint16_t* d_D, int64_t ldd, int64_t strideD,
             const uint16_t* d_C, int64_t ldc, int64_t strideC,
             int M, int N, int K, int batch, int in_dtype, int out_dtype, int epi, int sym,
             float alpha, float beta, float gamma, const float* d_scale,
             float* d_rowsq, void* stream);

/* The same product on CUDA cores (no tensor cores, no mirroring); a test hook
 * that checks the tensor-core path against an independent kernel. No
 * reference counterpart. */
int b2o_gemm_bf16_simt(const uint16_t* d_A, int64_t lda, int64_t strideA, int a_kmajor,
                       const uint16_t* d_B, int64_t ldb, int64_t strideB, int b_kmajor,
                       uint16_t* d_D, int64_t ldd, int64_t strideD,
                       const uint16_t* d_C, int64_t ldc, int64_t strideC,
                       int M, int N, int K, int batch, int epi,
                       float alpha, float beta, float gamma, const float* d_scale,
                       float* d_rowsq, void* stream);

/* ------------------------------------------------------------------------ *
 * Gradient-norm clip: torch.nn.utils.clip_grad_norm_(params, max_norm,
 * foreach=True) as the reference calls it before the optimizer steps
 * (transformer_lm/train_sol.py:498-499), with torch's dtype semantics: each
 * tensor's norm rounded to its gradient dtype, the total and the coefficient
 * min(max_norm / (total + 1e-6), 1) rounded to the promoted dtype.
 * b2o_clip_scratch_floats: scratch floats a call needs (one per 32768 elements).
 * b2o_clip_grad_norm: d_out[0] = total norm, d_out[1] = clip coefficient.
 * b2o_clip_scale: g = dtype(g * d_coef[0]) in place (torch._foreach_mul_);
 *   or hand d_out + 1 to the optimizers' grad_scale arguments instead.
 * dtypes: B2O_F32 or B2O_BF16 per tensor; at most 1024 tensors per call. */
int64_t b2o_clip_scratch_floats(const int64_t* numels, int n);
int b2o_clip_grad_norm(const void* const* d_grads, const int64_t* numels, const int* dtypes, int n,
                       float max_norm, float* d_scratch, float* d_out, void* stream);
int b2o_clip_scale(void* const* d_grads, const int64_t* numels, const int* dtypes, int n, const float* d_coef,
                   void* stream);

/* ------------------------------------------------------------------------ *
 * Peer exchange for the sharded step on the GPUs of one node (no reference
 * counterpart: the reference is single-GPU, transformer_lm/train_sol.py has no
 * torch.distributed call). Each rank pushes the parameter rows it updated into
 * the same offsets of every other rank's copy with copy-engine transfers over
 * NVLink, replacing an all-gather kernel that would occupy SMs next to the
 * NorMuon GEMMs. The exchange of handles between processes and the completion
 * barrier stay with the host's process group.
 *
 * b2o_ipc_export: writes the 64-byte CUDA IPC handle of the allocation holding
 *   d_ptr and d_ptr's byte offset inside it (memory from cudaMalloc, which is
 *   what PyTorch's caching allocator uses by default).
 * b2o_ipc_import: maps another process's allocation into this process (current
 *   device, peer access enabled on first use) and returns its base; open each
 *   handle once per process and close it with b2o_ipc_close before the owner
 *   frees the memory.
 * b2o_copy_async: enqueues n device-to-device copies d_dst[i] <- d_src[i] of
 *   bytes[i] bytes on `stream`, one cudaMemcpyAsync each, in order. */
#define B2O_IPC_HANDLE_BYTES 64
int b2o_ipc_export(const void* d_ptr, void* handle_out, uint64_t* offset_out);
int b2o_ipc_import(const void* handle, void** d_base_out);
int b2o_ipc_close(void* d_base);
int b2o_copy_async(void* const* d_dst, const void* const* d_src, const int64_t* bytes, int n, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* B2O_H_ */
