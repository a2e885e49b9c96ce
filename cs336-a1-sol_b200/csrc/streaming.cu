// HBM-bound streaming kernels of the optimizer step (sm_100a):
//   * fused AdamW (+ EMA)                 torch.optim.AdamW(fused=True), sol_modules.py:468-476
//   * stand-alone EMA and EMA->param copy EmaWeights.update/averaged, sol_modules.py:1255-1280
//   * NorMuon front (momentum, Nesterov)  sol_modules.py:390-394
//   * NorMuon finish + apply              sol_modules.py:396-424
// All kernels move 16-byte vectors, size their grids in multiples of the SM
// count and take tensor lists by value as kernel parameters (no host->device
// copies of pointer tables).
#include "b2o_common.cuh"
#include "b2o_internal.h"

#include <algorithm>
#include <cstdio>
#include <mutex>
#include <string>
#include <vector>

namespace b2o {

// ------------------------------------------------------------ vector I/O ---
struct alignas(16) U16x8 { uint16_t v[8]; };
struct alignas(16) F32x4 { float v[4]; };

template <typename T> struct Elem;
template <> struct Elem<float> {
  __device__ static void load8(const float* p, float* o) {
    F32x4 a = *reinterpret_cast<const F32x4*>(p);
    F32x4 b = *reinterpret_cast<const F32x4*>(p + 4);
#pragma unroll
    for (int i = 0; i < 4; ++i) { o[i] = a.v[i]; o[4 + i] = b.v[i]; }
  }
  __device__ static void store8(float* p, const float* x) {
    F32x4 a, b;
#pragma unroll
    for (int i = 0; i < 4; ++i) { a.v[i] = x[i]; b.v[i] = x[4 + i]; }
    *reinterpret_cast<F32x4*>(p) = a;
    *reinterpret_cast<F32x4*>(p + 4) = b;
  }
  __device__ static float load1(const float* p) { return *p; }
  __device__ static void store1(float* p, float x) { *p = x; }
  // value after rounding to the storage type
  __device__ static float rnd(float x) { return x; }
};
template <> struct Elem<uint16_t> {  // bf16 stored as raw bits
  __device__ static void load8(const uint16_t* p, float* o) {
    U16x8 a = *reinterpret_cast<const U16x8*>(p);
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = bf16_to_f32(a.v[i]);
  }
  __device__ static void store8(uint16_t* p, const float* x) {
    U16x8 a;
#pragma unroll
    for (int i = 0; i < 8; ++i) a.v[i] = f32_to_bf16(x[i]);
    *reinterpret_cast<U16x8*>(p) = a;
  }
  __device__ static float load1(const uint16_t* p) { return bf16_to_f32(*p); }
  __device__ static void store1(uint16_t* p, float x) { *p = f32_to_bf16(x); }
  __device__ static float rnd(float x) { return round_bf16(x); }
};

static inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ================================================================ AdamW ===
constexpr int kAdamMaxTensors = 96;
constexpr int kAdamMaxGroups = 8;
constexpr int kAdamThreads = 256;
constexpr int kAdamChunk = kAdamThreads * 8 * 4;  // elements per block iteration

struct AdamTable {
  b2o_adamw_tensor t[kAdamMaxTensors];
  b2o_adamw_group g[kAdamMaxGroups];
  int chunk_start[kAdamMaxTensors + 1];  // prefix sum of chunks per tensor
  int vec_ok[kAdamMaxTensors];           // 1 when every pointer is 16-byte aligned
  int ntensors;
  float ema_weight;
};

// One element of torch's fused AdamW (ATen/native/cuda/fused_adam_utils.cuh,
// adam_math with ADAMW mode), extended by the cautious mask and the bf16
// remainder of NorMuonGNS (sol_modules.py:406-424).
struct AdamCoef {
  float lr, b1, b2, eps, lr_wd, step_size, bc2_sqrt;
  int wd_on, cautious;
};

__device__ __forceinline__ AdamCoef make_coef(const b2o_adamw_group& g) {
  AdamCoef c;
  c.lr = g.lr; c.b1 = g.beta1; c.b2 = g.beta2; c.eps = g.eps; c.lr_wd = g.lr_wd;
  const float bc1 = 1.0f - powf(g.beta1, g.step);
  const float bc2 = 1.0f - powf(g.beta2, g.step);
  c.bc2_sqrt = sqrtf(bc2);
  c.step_size = g.lr / bc1;
  c.wd_on = g.weight_decay != 0.0f;
  c.cautious = g.cautious;
  return c;
}

__device__ __forceinline__ void adam_elem(const AdamCoef& c, float& w, float grad, float& m, float& v) {
  m = fmaf(c.b1, m, fmaf(-c.b1, grad, grad));
  const float g2 = grad * grad;
  v = fmaf(c.b2, v, fmaf(-c.b2, g2, g2));
  if (c.wd_on) {
    if (c.cautious) {
      // the update subtracted is step_size*m/denom with positive factors, so
      // its sign is the sign of m (sol_modules.py:414-418)
      const float mask = (m * w) > 0.0f ? 1.0f : 0.0f;
      w = w * (1.0f - c.lr_wd * mask);
    } else {
      w = w - c.lr_wd * w;
    }
  }
  const float denom = sqrtf(v) / c.bc2_sqrt + c.eps;
  w = w - (c.step_size * m) / denom;
}

template <typename PT, typename ST>
__global__ void __launch_bounds__(kAdamThreads) adamw_kernel(const __grid_constant__ AdamTable tab) {
  pdl_wait();
  const int total_chunks = tab.chunk_start[tab.ntensors];
  for (int chunk = blockIdx.x; chunk < total_chunks; chunk += gridDim.x) {
    // locate the tensor owning this chunk (<= kAdamMaxTensors entries)
    int lo = 0, hi = tab.ntensors - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (tab.chunk_start[mid] <= chunk) lo = mid; else hi = mid - 1;
    }
    const b2o_adamw_tensor& T = tab.t[lo];
    const AdamCoef c = make_coef(tab.g[T.group]);
    // torch's fused AdamW keeps state["step"] on the device: the CTA of the
    // tensor's first chunk writes it
    if (T.step_out && chunk == tab.chunk_start[lo] && threadIdx.x == 0) *T.step_out = tab.g[T.group].step;
    const int64_t base = static_cast<int64_t>(chunk - tab.chunk_start[lo]) * kAdamChunk;
    const int64_t end = min(T.numel, base + kAdamChunk);
    PT* __restrict__ P = reinterpret_cast<PT*>(T.param);
    const PT* __restrict__ G = reinterpret_cast<const PT*>(T.grad);
    ST* __restrict__ M = reinterpret_cast<ST*>(T.exp_avg);
    ST* __restrict__ V = reinterpret_cast<ST*>(T.exp_avg_sq);
    uint16_t* __restrict__ R = T.rem;
    float* __restrict__ E = T.ema;
    const float ew = tab.ema_weight;
    // clipped gradient g = dtype(g * coef), as torch._foreach_mul_ leaves it
    const float* gsp = tab.g[T.group].grad_scale;
    const float gs = gsp ? *gsp : 1.0f;
    if (tab.vec_ok[lo]) {
      for (int64_t i = base + static_cast<int64_t>(threadIdx.x) * 8; i + 8 <= end; i += kAdamThreads * 8) {
        float w[8], g[8], m[8], v[8];
        Elem<PT>::load8(P + i, w);
        Elem<PT>::load8(G + i, g);
        if (gsp) {
#pragma unroll
          for (int k = 0; k < 8; ++k) g[k] = Elem<PT>::rnd(g[k] * gs);
        }
        Elem<ST>::load8(M + i, m);
        Elem<ST>::load8(V + i, v);
        if (R) {
          float r[8];
          Elem<uint16_t>::load8(R + i, r);
#pragma unroll
          for (int k = 0; k < 8; ++k) w[k] = w[k] + r[k];
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) adam_elem(c, w[k], g[k], m[k], v[k]);
        float pn[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) pn[k] = Elem<PT>::rnd(w[k]);
        Elem<PT>::store8(P + i, pn);
        if (R) {
          float r[8];
#pragma unroll
          for (int k = 0; k < 8; ++k) r[k] = w[k] - pn[k];
          Elem<uint16_t>::store8(R + i, r);
        }
        Elem<ST>::store8(M + i, m);
        Elem<ST>::store8(V + i, v);
        if (E) {
          float e[8];
          Elem<float>::load8(E + i, e);
#pragma unroll
          for (int k = 0; k < 8; ++k) e[k] = torch_lerp(e[k], pn[k], ew);
          Elem<float>::store8(E + i, e);
        }
      }
      // ragged tail of the tensor (fewer than 8 elements)
      const int64_t tail = base + ((end - base) / 8) * 8;
      for (int64_t i = tail + threadIdx.x; i < end; i += kAdamThreads) {
        float w = Elem<PT>::load1(P + i), g = Elem<PT>::load1(G + i);
        if (gsp) g = Elem<PT>::rnd(g * gs);
        float m = Elem<ST>::load1(M + i), v = Elem<ST>::load1(V + i);
        if (R) w = w + bf16_to_f32(R[i]);
        adam_elem(c, w, g, m, v);
        const float pn = Elem<PT>::rnd(w);
        Elem<PT>::store1(P + i, pn);
        if (R) R[i] = f32_to_bf16(w - pn);
        Elem<ST>::store1(M + i, m);
        Elem<ST>::store1(V + i, v);
        if (E) E[i] = torch_lerp(E[i], pn, ew);
      }
    } else {
      for (int64_t i = base + threadIdx.x; i < end; i += kAdamThreads) {
        float w = Elem<PT>::load1(P + i), g = Elem<PT>::load1(G + i);
        if (gsp) g = Elem<PT>::rnd(g * gs);
        float m = Elem<ST>::load1(M + i), v = Elem<ST>::load1(V + i);
        if (R) w = w + bf16_to_f32(R[i]);
        adam_elem(c, w, g, m, v);
        const float pn = Elem<PT>::rnd(w);
        Elem<PT>::store1(P + i, pn);
        if (R) R[i] = f32_to_bf16(w - pn);
        Elem<ST>::store1(M + i, m);
        Elem<ST>::store1(V + i, v);
        if (E) E[i] = torch_lerp(E[i], pn, ew);
      }
    }
  }
}

int adamw_step(const b2o_adamw_tensor* tensors, int ntensors, const b2o_adamw_group* groups,
               int ngroups, int param_dtype, int state_dtype, float ema_weight, cudaStream_t stream) {
  if (ntensors < 0 || (ntensors > 0 && !tensors)) { set_error("adamw: bad tensor list"); return -1; }
  if (ngroups <= 0 || ngroups > kAdamMaxGroups || !groups) { set_error("adamw: 1..8 groups required"); return -1; }
  if (param_dtype != B2O_F32 && param_dtype != B2O_BF16) { set_error("adamw: bad param dtype"); return -1; }
  if (state_dtype != B2O_F32 && state_dtype != B2O_BF16) { set_error("adamw: bad state dtype"); return -1; }
  if (param_dtype == B2O_F32 && state_dtype != B2O_F32) { set_error("adamw: fp32 params need fp32 state"); return -1; }
  for (int i = 0; i < ntensors; ++i) {
    const b2o_adamw_tensor& t = tensors[i];
    if (t.numel < 0 || (t.numel > 0 && (!t.param || !t.grad || !t.exp_avg || !t.exp_avg_sq))) {
      set_error("adamw: tensor " + std::to_string(i) + " has a null pointer"); return -1;
    }
    if (t.group < 0 || t.group >= ngroups) { set_error("adamw: tensor group out of range"); return -1; }
    if (t.rem && param_dtype != B2O_BF16) { set_error("adamw: remainder needs bf16 params"); return -1; }
  }
  int done = 0;
  while (done < ntensors) {
    AdamTable tab;
    memset(&tab, 0, sizeof(tab));
    int n = 0, chunks = 0;
    while (done + n < ntensors && n < kAdamMaxTensors) {
      const b2o_adamw_tensor& t = tensors[done + n];
      const int64_t ch = (t.numel + kAdamChunk - 1) / kAdamChunk;
      if (static_cast<int64_t>(chunks) + ch > (1ll << 30)) break;
      tab.t[n] = t;
      tab.chunk_start[n] = chunks;
      tab.vec_ok[n] = aligned16(t.param) && aligned16(t.grad) && aligned16(t.exp_avg) &&
                      aligned16(t.exp_avg_sq) && (!t.rem || aligned16(t.rem)) &&
                      (!t.ema || aligned16(t.ema));
      chunks += static_cast<int>(ch);
      ++n;
    }
    if (n == 0) { set_error("adamw: tensor too large"); return -1; }
    tab.chunk_start[n] = chunks;
    tab.ntensors = n;
    for (int g = 0; g < ngroups; ++g) tab.g[g] = groups[g];
    tab.ema_weight = ema_weight;
    if (chunks > 0) {
      const int grid = std::min(chunks, num_sms() * 8);
      if (param_dtype == B2O_F32)
        launch_pdl(adamw_kernel<float, float>, dim3(grid), dim3(kAdamThreads), 0, stream, tab);
      else if (state_dtype == B2O_F32)
        launch_pdl(adamw_kernel<uint16_t, float>, dim3(grid), dim3(kAdamThreads), 0, stream, tab);
      else
        launch_pdl(adamw_kernel<uint16_t, uint16_t>, dim3(grid), dim3(kAdamThreads), 0, stream, tab);
      count_launch();
      if (int e = check_launch("adamw")) return e;
    }
    done += n;
  }
  return 0;
}

// ================================================================== EMA ===
constexpr int kEmaMax = 128;
struct EmaTable {
  float* s[kEmaMax];
  const void* p[kEmaMax];
  int64_t n[kEmaMax];
  int chunk_start[kEmaMax + 1];
  int vec_ok[kEmaMax];
  int count;
  float w;
};
constexpr int kEmaChunk = 256 * 8 * 4;

template <typename PT, bool TO_PARAM>
__global__ void __launch_bounds__(256) ema_kernel(const __grid_constant__ EmaTable tab) {
  pdl_wait();
  const int total = tab.chunk_start[tab.count];
  for (int chunk = blockIdx.x; chunk < total; chunk += gridDim.x) {
    int lo = 0, hi = tab.count - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (tab.chunk_start[mid] <= chunk) lo = mid; else hi = mid - 1;
    }
    float* S = tab.s[lo];
    PT* P = reinterpret_cast<PT*>(const_cast<void*>(tab.p[lo]));
    const int64_t base = static_cast<int64_t>(chunk - tab.chunk_start[lo]) * kEmaChunk;
    const int64_t end = min(tab.n[lo], base + kEmaChunk);
    int64_t scalar_from = base;
    if (tab.vec_ok[lo]) {
      for (int64_t i = base + threadIdx.x * 8; i + 8 <= end; i += 256 * 8) {
        float s[8], p[8];
        Elem<float>::load8(S + i, s);
        if (TO_PARAM) {
          Elem<PT>::store8(P + i, s);
        } else {
          Elem<PT>::load8(P + i, p);
#pragma unroll
          for (int k = 0; k < 8; ++k) s[k] = torch_lerp(s[k], p[k], tab.w);
          Elem<float>::store8(S + i, s);
        }
      }
      scalar_from = base + ((end - base) / 8) * 8;
    }
    for (int64_t i = scalar_from + threadIdx.x; i < end; i += 256) {
      if (TO_PARAM) Elem<PT>::store1(P + i, S[i]);
      else S[i] = torch_lerp(S[i], Elem<PT>::load1(P + i), tab.w);
    }
  }
}

template <bool TO_PARAM>
static int ema_launch(float* const* shadows, const void* const* params, const int64_t* numels, int nt,
                      int param_dtype, float w, cudaStream_t stream) {
  if (nt < 0 || (nt > 0 && (!shadows || !params || !numels))) { set_error("ema: bad lists"); return -1; }
  if (param_dtype != B2O_F32 && param_dtype != B2O_BF16) { set_error("ema: bad dtype"); return -1; }
  int done = 0;
  while (done < nt) {
    EmaTable tab;
    memset(&tab, 0, sizeof(tab));
    int n = 0, chunks = 0;
    while (done + n < nt && n < kEmaMax) {
      const int i = done + n;
      if (numels[i] > 0 && (!shadows[i] || !params[i])) { set_error("ema: null pointer"); return -1; }
      tab.s[n] = shadows[i];
      tab.p[n] = params[i];
      tab.n[n] = numels[i];
      tab.chunk_start[n] = chunks;
      tab.vec_ok[n] = aligned16(shadows[i]) && aligned16(params[i]);
      chunks += static_cast<int>((numels[i] + kEmaChunk - 1) / kEmaChunk);
      ++n;
    }
    tab.chunk_start[n] = chunks;
    tab.count = n;
    tab.w = w;
    if (chunks > 0) {
      const int grid = std::min(chunks, num_sms() * 8);
      if (param_dtype == B2O_F32) launch_pdl(ema_kernel<float, TO_PARAM>, dim3(grid), dim3(256), 0, stream, tab);
      else launch_pdl(ema_kernel<uint16_t, TO_PARAM>, dim3(grid), dim3(256), 0, stream, tab);
      count_launch();
      if (int e = check_launch("ema")) return e;
    }
    done += n;
  }
  return 0;
}

int ema_update(float* const* shadows, const void* const* params, const int64_t* numels, int nt,
               int param_dtype, float w, cudaStream_t stream) {
  return ema_launch<false>(shadows, params, numels, nt, param_dtype, w, stream);
}
int ema_copy_to_params(const float* const* shadows, void* const* params, const int64_t* numels, int nt,
                       int param_dtype, cudaStream_t stream) {
  return ema_launch<true>(const_cast<float* const*>(shadows), const_cast<const void* const*>(params),
                          numels, nt, param_dtype, 0.0f, stream);
}

// ======================================================= NorMuon front ===
// Every kernel of the NorMuon pass takes all shape batches of one parameter
// group at once (one launch each for front, finish and apply, instead of one
// per batch): a CTA finds its batch in a small prefix table and its matrix and
// 8192/16384-element part inside it.
constexpr int kMaxBatch = 64;          // matrices per batch (orthogonaliser kernel tables)
constexpr int kMaxMultiMats = 128;     // matrices per multi-batch launch
constexpr int kMaxMultiBatches = 16;   // batches per multi-batch launch
constexpr int kFrontThreads = 256;
constexpr int kFrontPart = kFrontThreads * 8 * 8;  // elements per partial sum
constexpr int kApplyThreads = 256;
constexpr int64_t kApplyPart = kApplyThreads * 8 * 4;  // elements per apply CTA

int normuon_front_parts(int64_t rc) { return static_cast<int>((rc + kFrontPart - 1) / kFrontPart); }

struct MultiBatchInfo {
  int64_t rc;
  int r, c, S, nparts;   // nparts: CTAs per matrix
  int mat0;              // index of the batch's first matrix in the pointer tables
  int cta0;              // first CTA of the batch
  int vec_ok, has_rem, has_ema;
  float shape_scale;
  uint16_t* u;           // front output / apply input o
  float* partial;        // front: norm partials; apply: scratch (S * (r + 4))
  const float* rowsq;    // apply: [S][ceil(c/256)][r]
  int x0_half;           // front: write binary16 X0 = bf16(u) * prescale[s] instead of bf16 u
  float* prescale;       // [S] powers of two (0 = none yet)
  float* xscale;         // [2S] s_norm / k and its square
  int* flags;            // [S] 1 = X0 needs rewriting with the new k
};
struct MultiHeader {
  int nb;
  MultiBatchInfo b[kMaxMultiBatches];
};

// batch of CTA `cta` (batches are ordered by cta0)
__device__ __forceinline__ int find_batch_cta(const MultiHeader& h, int cta) {
  int k = 0;
  while (k + 1 < h.nb && cta >= h.b[k + 1].cta0) ++k;
  return k;
}

struct FrontTable {
  MultiHeader h;
  const void* g[kMaxMultiMats];
  void* buf[kMaxMultiMats];
  const float* gscale;  // gradient-clip coefficient, or null
};

// Stores 8 values of u as bf16, or as binary16 X0 = bf16(u) * k (exact: k is a power of two).
__device__ __forceinline__ void store_u8(uint16_t* dst, const float* u, bool x0, float k) {
  if (x0) {
    U16x8 a;
#pragma unroll
    for (int i = 0; i < 8; ++i) a.v[i] = f32_to_f16(u[i] * k);
    *reinterpret_cast<U16x8*>(dst) = a;
  } else {
    Elem<uint16_t>::store8(dst, u);
  }
}

// REPAIR = false: the front pass (momentum update, u, norm partials).
// REPAIR = true: rewrites X0 of the matrices flagged by the prescale pass from
// the gradient and the already updated momentum buffer (no state changes).
template <typename T, bool REPAIR>
__device__ __forceinline__ void front_body(const FrontTable& tab, int cta, float w_small, float w_large,
                                           int nesterov) {
  const MultiBatchInfo& bi = tab.h.b[find_batch_cta(tab.h, cta)];
  const int local = cta - bi.cta0;
  const int s = local / bi.nparts;
  const int part = local - s * bi.nparts;
  if (REPAIR && (!bi.x0_half || !bi.flags[s])) return;
  const int64_t rc = bi.rc;
  const T* G = reinterpret_cast<const T*>(tab.g[bi.mat0 + s]);
  T* B = reinterpret_cast<T*>(tab.buf[bi.mat0 + s]);
  uint16_t* Us = bi.u + static_cast<int64_t>(s) * rc;
  const bool x0 = bi.x0_half != 0;
  const float k = x0 ? bi.prescale[s] : 1.0f;
  const int64_t base = static_cast<int64_t>(part) * kFrontPart;
  const int64_t end = min(rc, base + kFrontPart);
  // clipped gradient g = dtype(g * coef), as torch._foreach_mul_ leaves it
  const bool clip = tab.gscale != nullptr;
  const float gs = clip ? *tab.gscale : 1.0f;
  float pacc = 0.f;
  int64_t scalar_from = base;
  if (bi.vec_ok) {
    for (int64_t i = base + threadIdx.x * 8; i + 8 <= end; i += kFrontThreads * 8) {
      float g[8], b[8], u[8];
      Elem<T>::load8(G + i, g);
      Elem<T>::load8(B + i, b);
      if (clip) {
#pragma unroll
        for (int q = 0; q < 8; ++q) g[q] = Elem<T>::rnd(g[q] * gs);
      }
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        if (!REPAIR) b[q] = Elem<T>::rnd(torch_lerp(b[q], g[q], w_small));  // buf.lerp_(g, 1-beta)
        u[q] = nesterov ? Elem<T>::rnd(torch_lerp(g[q], b[q], w_large)) : b[q];  // g.lerp(buf, beta)
        u[q] = round_bf16(u[q]);                                                  // X = u.bfloat16()
        pacc = fmaf(u[q], u[q], pacc);
      }
      if (!REPAIR) Elem<T>::store8(B + i, b);
      store_u8(Us + i, u, x0, k);
    }
    scalar_from = base + ((end - base) / 8) * 8;
  }
  for (int64_t i = scalar_from + threadIdx.x; i < end; i += kFrontThreads) {
    float g = Elem<T>::load1(G + i);
    if (clip) g = Elem<T>::rnd(g * gs);
    float b = Elem<T>::load1(B + i);
    if (!REPAIR) b = Elem<T>::rnd(torch_lerp(b, g, w_small));
    float u = nesterov ? Elem<T>::rnd(torch_lerp(g, b, w_large)) : b;
    u = round_bf16(u);
    pacc = fmaf(u, u, pacc);
    if (!REPAIR) Elem<T>::store1(B + i, b);
    Us[i] = x0 ? f32_to_f16(u * k) : f32_to_bf16(u);
  }
  if (REPAIR) return;
  // deterministic block reduction of this part
  __shared__ float red[kFrontThreads / 32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) pacc += __shfl_xor_sync(0xffffffffu, pacc, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = pacc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int q = 0; q < kFrontThreads / 32; ++q) t += red[q];
    bi.partial[static_cast<int64_t>(s) * bi.nparts + part] = t;
  }
}

template <typename T>
__global__ void __launch_bounds__(kFrontThreads) normuon_front_kernel(const __grid_constant__ FrontTable tab,
                                                                      float w_small, float w_large, int nesterov) {
  pdl_wait();
  front_body<T, false>(tab, blockIdx.x, w_small, w_large, nesterov);
}

// kRepairCtas CTAs per matrix: an unflagged matrix (almost all of them)
// costs each CTA one flag load; a flagged one is rewritten by its CTAs.
constexpr int kRepairCtas = 8;
template <typename T>
__global__ void __launch_bounds__(kFrontThreads) normuon_x0_repair_kernel(const __grid_constant__ FrontTable tab,
                                                                          float w_small, float w_large,
                                                                          int nesterov) {
  pdl_wait();
  const int m = blockIdx.x / kRepairCtas;
  const int sub = blockIdx.x - m * kRepairCtas;
  int kb = 0;
  while (kb + 1 < tab.h.nb && m >= tab.h.b[kb + 1].mat0) ++kb;
  const MultiBatchInfo& bi = tab.h.b[kb];
  const int s = m - bi.mat0;
  if (!bi.x0_half || !bi.flags[s]) return;
  for (int part = sub; part < bi.nparts; part += kRepairCtas)
    front_body<T, true>(tab, bi.cta0 + s * bi.nparts + part, w_small, w_large, nesterov);
}

// One warp per matrix of the x0_half batches: this step's norm scale, the
// factor s_norm / k for the orthogonaliser and next step's k = 2^(8 + e) with
// s_norm in [2^(e-1), 2^e): ||X0|| ~ 2^8 keeps X0's entries far from both ends
// of binary16. A matrix whose ||X0|| = k / s_norm left [2^2, 2^14] (or that had
// no k yet) is flagged and rewritten with the new k.
__global__ void __launch_bounds__(128) normuon_prescale_kernel(const __grid_constant__ MultiHeader h, int nmats,
                                                               float eps, float safety) {
  pdl_wait();
  const int m = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (m >= nmats) return;
  int kb = 0;
  while (kb + 1 < h.nb && m >= h.b[kb + 1].mat0) ++kb;
  const MultiBatchInfo& bi = h.b[kb];
  if (!bi.x0_half) return;
  const int s = m - bi.mat0;
  float acc = 0.f;  // lane-strided partial sums, then a fixed-order butterfly
  for (int i = lane; i < bi.nparts; i += 32) acc += bi.partial[static_cast<int64_t>(s) * bi.nparts + i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane != 0) return;
  const float sn = 1.0f / (sqrtf(acc) * safety + eps);
  int e = 0;
  frexpf(sn, &e);
  const float k_new = ldexpf(1.0f, e + 8);
  const float k_old = bi.prescale[s];
  const float x0norm = k_old / sn;  // ||X0|| written with k_old
  const bool ok = k_old > 0.f && x0norm >= 4.0f && x0norm <= 16384.0f;
  const float k = ok ? k_old : k_new;
  bi.flags[s] = ok ? 0 : 1;
  bi.prescale[s] = k_new;
  const float f = sn / k;
  bi.xscale[s] = f;
  bi.xscale[bi.S + s] = f * f;
}

// Checks the batch list shared by the multi-batch calls and fills the header
// (matrix and CTA offsets); parts_of(rc) = CTAs per matrix.
template <typename PartsFn>
static int fill_header(const b2o_normuon_batch* batches, int nb, const char* what, PartsFn parts_of, MultiHeader& h,
                       int& nmats, int& ncta) {
  if (nb <= 0 || nb > kMaxMultiBatches || !batches) {
    set_error(std::string(what) + ": 1.." + std::to_string(kMaxMultiBatches) + " batches per call");
    return -1;
  }
  memset(&h, 0, sizeof(h));
  h.nb = nb;
  nmats = 0;
  int64_t ctas = 0;
  for (int k = 0; k < nb; ++k) {
    const b2o_normuon_batch& b = batches[k];
    if (b.S <= 0 || b.S > kMaxBatch || b.r <= 0 || b.c <= 0) {
      set_error(std::string(what) + ": batch " + std::to_string(k) + " needs 1..64 matrices of positive shape");
      return -1;
    }
    MultiBatchInfo& bi = h.b[k];
    bi.rc = static_cast<int64_t>(b.r) * b.c;
    bi.r = b.r; bi.c = b.c; bi.S = b.S;
    bi.nparts = parts_of(bi.rc);
    bi.mat0 = nmats;
    bi.cta0 = static_cast<int>(ctas);
    bi.shape_scale = b.shape_scale;
    nmats += b.S;
    ctas += static_cast<int64_t>(b.S) * bi.nparts;
  }
  if (nmats > kMaxMultiMats) {
    set_error(std::string(what) + ": at most " + std::to_string(kMaxMultiMats) + " matrices per call");
    return -1;
  }
  if (ctas > (1ll << 30)) { set_error(std::string(what) + ": too many elements"); return -1; }
  ncta = static_cast<int>(ctas);
  return 0;
}

// repair = false: the front pass; true: the prescale pass that follows it
// (same batches and arguments).
static int front_launch(const b2o_normuon_batch* batches, int nb, int dtype, float w_small, float w_large,
                        int nesterov, const float* grad_scale, bool repair, float norm_eps, float norm_safety,
                        cudaStream_t stream) {
  if (dtype != B2O_F32 && dtype != B2O_BF16) { set_error("normuon_front: bad dtype"); return -1; }
  FrontTable tab;
  int nmats = 0, ncta = 0;
  if (int e = fill_header(batches, nb, "normuon_front", normuon_front_parts, tab.h, nmats, ncta)) return e;
  memset(tab.g, 0, sizeof(tab.g));
  memset(tab.buf, 0, sizeof(tab.buf));
  tab.gscale = grad_scale;
  for (int k = 0; k < nb; ++k) {
    const b2o_normuon_batch& b = batches[k];
    MultiBatchInfo& bi = tab.h.b[k];
    if (!b.grads || !b.bufs || !b.u || !b.partial) { set_error("normuon_front: bad args"); return -1; }
    int vec_ok = aligned16(b.u) && ((bi.rc * 2) % 16 == 0);
    for (int s = 0; s < b.S; ++s) {
      if (!b.grads[s] || !b.bufs[s]) { set_error("normuon_front: null matrix pointer"); return -1; }
      tab.g[bi.mat0 + s] = b.grads[s];
      tab.buf[bi.mat0 + s] = b.bufs[s];
      vec_ok = vec_ok && aligned16(b.grads[s]) && aligned16(b.bufs[s]);
    }
    bi.vec_ok = vec_ok;
    bi.u = b.u;
    bi.partial = b.partial;
    bi.x0_half = b.x0_half;
    bi.prescale = b.prescale;
    bi.xscale = b.xscale;
    bi.flags = b.flags;
    if (b.x0_half && (!b.prescale || !b.xscale || !b.flags)) {
      set_error("normuon_front: x0_half needs prescale, xscale and flags"); return -1;
    }
  }
  if (repair) {
    // this step's scales, next step's k, flags; then X0 of the flagged matrices
    launch_pdl(normuon_prescale_kernel, dim3((nmats * 32 + 127) / 128), dim3(128), 0, stream, tab.h, nmats,
               norm_eps, norm_safety);
    count_launch();
    if (int e = check_launch("normuon_prescale")) return e;
    const int rgrid = nmats * kRepairCtas;
    if (dtype == B2O_F32)
      launch_pdl(normuon_x0_repair_kernel<float>, dim3(rgrid), dim3(kFrontThreads), 0, stream, tab, w_small,
                 w_large, nesterov);
    else
      launch_pdl(normuon_x0_repair_kernel<uint16_t>, dim3(rgrid), dim3(kFrontThreads), 0, stream, tab, w_small,
                 w_large, nesterov);
    count_launch();
    return check_launch("normuon_x0_repair");
  }
  if (dtype == B2O_F32)
    launch_pdl(normuon_front_kernel<float>, dim3(ncta), dim3(kFrontThreads), 0, stream, tab, w_small, w_large,
               nesterov);
  else
    launch_pdl(normuon_front_kernel<uint16_t>, dim3(ncta), dim3(kFrontThreads), 0, stream, tab, w_small,
               w_large, nesterov);
  count_launch();
  return check_launch("normuon_front");
}

int normuon_front_multi(const b2o_normuon_batch* batches, int nb, int dtype, float w_small, float w_large,
                        int nesterov, const float* grad_scale, cudaStream_t stream) {
  return front_launch(batches, nb, dtype, w_small, w_large, nesterov, grad_scale, false, 0.f, 1.f, stream);
}

int normuon_prescale(const b2o_normuon_batch* batches, int nb, int dtype, float w_small, float w_large,
                     int nesterov, const float* grad_scale, float norm_eps, float norm_safety, cudaStream_t stream) {
  return front_launch(batches, nb, dtype, w_small, w_large, nesterov, grad_scale, true, norm_eps, norm_safety,
                      stream);
}

int normuon_front(const void* const* grads, void* const* bufs, int S, int r, int c, int dtype,
                  float w_small, float w_large, int nesterov, uint16_t* U, float* partial,
                  cudaStream_t stream) {
  b2o_normuon_batch b;
  memset(&b, 0, sizeof(b));
  b.S = S; b.r = r; b.c = c;
  b.grads = grads; b.bufs = bufs; b.u = U; b.partial = partial;
  return normuon_front_multi(&b, 1, dtype, w_small, w_large, nesterov, nullptr, stream);
}

// ====================================================== NorMuon finish ===
// One CTA per matrix. Reduces the GEMM's per-tile row partials of o^2 into
// row sums, updates v_row (sol_modules.py:398) and produces the per-row factor
// 1/(sqrt(v_row)+1e-10) (:399) and the per-matrix norm-restoring factor
// vnorm/(||o*inv||+1e-10) (:397, :400).
struct FinishTable {
  MultiHeader h;
  float* v[kMaxMultiMats];
};

__device__ float block_sum_1024(float x, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = x;
  __syncthreads();
  float t = 0.f;
  if (threadIdx.x == 0) {
    for (int k = 0; k < (int)(blockDim.x >> 5); ++k) t += red[k];
    red[32] = t;
  }
  __syncthreads();
  t = red[32];
  __syncthreads();
  return t;
}

__global__ void __launch_bounds__(1024) normuon_finish_kernel(const __grid_constant__ FinishTable tab,
                                                              float w_beta2) {
  pdl_wait();
  __shared__ float red[33];
  // one CTA per matrix: the batch is the last one whose first matrix is <= blockIdx.x
  int k = 0;
  while (k + 1 < tab.h.nb && static_cast<int>(blockIdx.x) >= tab.h.b[k + 1].mat0) ++k;
  const MultiBatchInfo& bi = tab.h.b[k];
  const int s = blockIdx.x - bi.mat0;
  const int r = bi.r, c = bi.c, ntn = (c + 255) / 256;
  float* inv = bi.partial + static_cast<int64_t>(s) * (r + 4);
  const float* part = bi.rowsq + static_cast<int64_t>(s) * ntn * r;
  float* vrow = tab.v[blockIdx.x];
  float sumsq = 0.f, n1 = 0.f;
  for (int i = threadIdx.x; i < r; i += blockDim.x) {
    float rs = 0.f;
    for (int t = 0; t < ntn; ++t) rs += part[static_cast<int64_t>(t) * r + i];
    sumsq += rs;
    const float mean = rs / static_cast<float>(c);
    const float v = torch_lerp(vrow[i], mean, w_beta2);
    vrow[i] = v;
    const float iv = __frcp_rn(sqrtf(v) + 1e-10f);
    inv[i] = iv;
    n1 = fmaf(rs * iv, iv, n1);
  }
  const float tot = block_sum_1024(sumsq, red);
  const float tot1 = block_sum_1024(n1, red);
  if (threadIdx.x == 0) inv[r] = sqrtf(tot) / (sqrtf(tot1) + 1e-10f);
}

// ======================================================= NorMuon apply ===
struct ApplyTable {
  MultiHeader h;
  void* p[kMaxMultiMats];
  uint16_t* rem[kMaxMultiMats];
  float* ema[kMaxMultiMats];
};

struct ApplyArgs {
  int wd_on, cautious;
  float neg_lr, lr_wd, wd_factor, ema_w;
};

// mode: 0 = fp32 params; 1 = bf16 params with remainder (bf16_master);
//       2 = bf16 params without remainder (every op rounds to bf16 as torch does).
template <int MODE>
__device__ __forceinline__ void apply_elem(const ApplyArgs& a, float o3, float& w, float& rem_out) {
  if (MODE == 2) {
    // w is the bf16 param; torch evaluates each op in fp32 and rounds to bf16
    if (a.wd_on) {
      // mask = (o * w) > 0 in fp32; factor = bf16(1 - bf16(lr*wd*mask)) (sol_modules.py:417)
      // without the cautious mask the factor is the Python double 1 - lr*wd (:420)
      const float f = a.cautious ? round_bf16(1.0f - round_bf16(a.lr_wd * ((o3 * w) > 0.f ? 1.f : 0.f)))
                                 : a.wd_factor;
      w = round_bf16(w * f);
    }
    w = round_bf16(fmaf(a.neg_lr, round_bf16(o3), w));
  } else {
    if (a.wd_on) {
      const float f = a.cautious ? (1.0f - a.lr_wd * ((o3 * w) > 0.f ? 1.f : 0.f)) : a.wd_factor;
      w = w * f;
    }
    w = fmaf(a.neg_lr, o3, w);
    if (MODE == 1) {
      const float pn = round_bf16(w);
      rem_out = w - pn;   // exact in fp32; rounded to bf16 on store
      w = pn;
    }
  }
}

template <int MODE>
__global__ void __launch_bounds__(kApplyThreads) normuon_apply_kernel(const __grid_constant__ ApplyTable tab,
                                                                      const __grid_constant__ ApplyArgs a) {
  pdl_wait();
  const MultiBatchInfo& bi = tab.h.b[find_batch_cta(tab.h, blockIdx.x)];
  const int local = blockIdx.x - bi.cta0;
  const int s = local / bi.nparts;
  const int part = local - s * bi.nparts;
  const int64_t rc = bi.rc;
  const int c = bi.c;
  const float* inv = bi.partial + static_cast<int64_t>(s) * (bi.r + 4);
  const float f = inv[bi.r];
  const float sscale = bi.shape_scale;
  const uint16_t* Os = bi.u + static_cast<int64_t>(s) * rc;
  float* E = bi.has_ema ? tab.ema[bi.mat0 + s] : nullptr;
  uint16_t* R = bi.has_rem ? tab.rem[bi.mat0 + s] : nullptr;
  using PT = typename std::conditional<MODE == 0, float, uint16_t>::type;
  PT* P = reinterpret_cast<PT*>(tab.p[bi.mat0 + s]);
  const int64_t base = static_cast<int64_t>(part) * kApplyPart;
  const int64_t end = min(rc, base + kApplyPart);
  int64_t scalar_from = base;
  if (bi.vec_ok) {
    for (int64_t i = base + threadIdx.x * 8; i + 8 <= end; i += kApplyThreads * 8) {
      float o[8], w[8], rm[8];
      Elem<uint16_t>::load8(Os + i, o);
      Elem<PT>::load8(P + i, w);
      if (MODE == 1) {
        float r0[8];
        Elem<uint16_t>::load8(R + i, r0);
#pragma unroll
        for (int k = 0; k < 8; ++k) w[k] = w[k] + r0[k];
      }
      // 8 consecutive elements may straddle a row boundary when c % 8 != 0
      // (excluded by vec_ok), so one row index serves all 8.
      const int row = static_cast<int>(i / c);
      const float iv = inv[row];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float o3 = ((o[k] * iv) * f) * sscale;
        apply_elem<MODE>(a, o3, w[k], rm[k]);
      }
      Elem<PT>::store8(P + i, w);
      if (MODE == 1) Elem<uint16_t>::store8(R + i, rm);
      if (E) {
        float e[8];
        Elem<float>::load8(E + i, e);
#pragma unroll
        for (int k = 0; k < 8; ++k) e[k] = torch_lerp(e[k], w[k], a.ema_w);
        Elem<float>::store8(E + i, e);
      }
    }
    scalar_from = base + ((end - base) / 8) * 8;
  }
  for (int64_t i = scalar_from + threadIdx.x; i < end; i += kApplyThreads) {
    float w = Elem<PT>::load1(P + i), rm = 0.f;
    if (MODE == 1) w = w + bf16_to_f32(R[i]);
    const int row = static_cast<int>(i / c);
    const float o3 = ((bf16_to_f32(Os[i]) * inv[row]) * f) * sscale;
    apply_elem<MODE>(a, o3, w, rm);
    Elem<PT>::store1(P + i, w);
    if (MODE == 1) R[i] = f32_to_bf16(rm);
    if (E) E[i] = torch_lerp(E[i], w, a.ema_w);
  }
}

static int apply_parts(int64_t rc) { return static_cast<int>((rc + kApplyPart - 1) / kApplyPart); }

int normuon_apply_multi(const b2o_normuon_batch* batches, int nb, int param_dtype, float neg_lr, float lr_wd,
                        float wd_factor, int wd_on, int cautious, float w_beta2, float ema_weight,
                        cudaStream_t stream) {
  if (param_dtype != B2O_F32 && param_dtype != B2O_BF16) { set_error("normuon_apply: bad dtype"); return -1; }
  ApplyTable tab;
  int nmats = 0, ncta = 0;
  if (int e = fill_header(batches, nb, "normuon_apply", apply_parts, tab.h, nmats, ncta)) return e;
  memset(tab.p, 0, sizeof(tab.p));
  memset(tab.rem, 0, sizeof(tab.rem));
  memset(tab.ema, 0, sizeof(tab.ema));
  FinishTable ft;
  memset(&ft, 0, sizeof(ft));
  const bool with_rem = batches[0].rems != nullptr;
  for (int k = 0; k < nb; ++k) {
    const b2o_normuon_batch& b = batches[k];
    MultiBatchInfo& bi = tab.h.b[k];
    if (!b.o || !b.rowsq || !b.params || !b.vrows || !b.scratch) { set_error("normuon_apply: bad args"); return -1; }
    if ((b.rems != nullptr) != with_rem) {
      set_error("normuon_apply: every batch of one call needs a remainder, or none"); return -1;
    }
    if (b.rems && param_dtype != B2O_BF16) { set_error("normuon_apply: remainder needs bf16 params"); return -1; }
    int vec_ok = (b.c % 8 == 0) && aligned16(b.o);
    for (int s = 0; s < b.S; ++s) {
      if (!b.params[s] || !b.vrows[s] || (b.rems && !b.rems[s]) || (b.emas && !b.emas[s])) {
        set_error("normuon_apply: null matrix pointer"); return -1;
      }
      tab.p[bi.mat0 + s] = b.params[s];
      tab.rem[bi.mat0 + s] = b.rems ? b.rems[s] : nullptr;
      tab.ema[bi.mat0 + s] = b.emas ? b.emas[s] : nullptr;
      ft.v[bi.mat0 + s] = b.vrows[s];
      vec_ok = vec_ok && aligned16(b.params[s]) && (!b.rems || aligned16(b.rems[s])) &&
               (!b.emas || aligned16(b.emas[s]));
    }
    bi.vec_ok = vec_ok;
    bi.has_rem = b.rems != nullptr;
    bi.has_ema = b.emas != nullptr;
    bi.u = const_cast<uint16_t*>(b.o);
    bi.partial = b.scratch;
    bi.rowsq = b.rowsq;
  }
  ft.h = tab.h;
  ApplyArgs a;
  memset(&a, 0, sizeof(a));
  a.wd_on = wd_on; a.cautious = cautious;
  a.neg_lr = neg_lr; a.lr_wd = lr_wd; a.wd_factor = wd_factor; a.ema_w = ema_weight;
  launch_pdl(normuon_finish_kernel, dim3(nmats), dim3(1024), 0, stream, ft, w_beta2);
  count_launch();
  if (int e = check_launch("normuon_finish")) return e;
  if (param_dtype == B2O_F32)
    launch_pdl(normuon_apply_kernel<0>, dim3(ncta), dim3(kApplyThreads), 0, stream, tab, a);
  else if (with_rem)
    launch_pdl(normuon_apply_kernel<1>, dim3(ncta), dim3(kApplyThreads), 0, stream, tab, a);
  else
    launch_pdl(normuon_apply_kernel<2>, dim3(ncta), dim3(kApplyThreads), 0, stream, tab, a);
  count_launch();
  return check_launch("normuon_apply");
}

int normuon_apply(const uint16_t* O, const float* rowsq, int S, int r, int c, void* const* params,
                  uint16_t* const* rems, float* const* emas, float* const* vrows, int param_dtype,
                  float neg_lr, float lr_wd, float wd_factor, int wd_on, int cautious, float shape_scale,
                  float w_beta2, float ema_weight, float* scratch, cudaStream_t stream) {
  b2o_normuon_batch b;
  memset(&b, 0, sizeof(b));
  b.S = S; b.r = r; b.c = c;
  b.o = O; b.rowsq = rowsq; b.params = params; b.rems = rems; b.emas = emas; b.vrows = vrows;
  b.shape_scale = shape_scale; b.scratch = scratch;
  return normuon_apply_multi(&b, 1, param_dtype, neg_lr, lr_wd, wd_factor, wd_on, cautious, w_beta2, ema_weight,
                             stream);
}

// ----------------------------------------------- allocation-free variant ---
// Scratch of b2o_normuon_apply_static: file-scope device memory, reserved by
// every GPU that loads the library (1 MiB each) for the life of the process.
// Its address is taken once per device with cudaGetSymbolAddress (the array's
// name in host code is only a stand-in for the symbol, never a device address)
// and cached for the life of that device's primary context: a process that
// resets the device (cudaDeviceReset) must not call this entry point again.
constexpr int64_t kStaticApplyScratchFloats = int64_t(1) << 18;
static __device__ __align__(256) float g_static_apply_scratch[kStaticApplyScratchFloats];

constexpr int kStaticMaxDevices = 64;
static float* g_static_scratch_ptr[kStaticMaxDevices];
static std::mutex g_static_scratch_mu;

int64_t normuon_apply_static_max_floats() { return kStaticApplyScratchFloats; }

int normuon_apply_static(const uint16_t* O, const float* rowsq, int S, int r, int c, void* const* params,
                         uint16_t* const* rems, float* const* emas, float* const* vrows, int param_dtype,
                         float neg_lr, float lr_wd, float wd_factor, int wd_on, int cautious, float shape_scale,
                         float w_beta2, float ema_weight, cudaStream_t stream) {
  if (S <= 0 || r <= 0) { set_error("normuon_apply_static: bad args"); return -1; }
  const int64_t need = static_cast<int64_t>(S) * (static_cast<int64_t>(r) + 4);
  if (need > kStaticApplyScratchFloats) {
    set_error("normuon_apply_static: needs " + std::to_string(need) + " scratch floats (S*(r+4)); the static " +
              "scratch holds " + std::to_string(kStaticApplyScratchFloats) + "; split the batch or use " +
              "b2o_normuon_apply with caller scratch");
    return -1;
  }
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kStaticMaxDevices) {
    set_error(std::string("normuon_apply_static: no usable current device: ") + cudaGetErrorString(e));
    return -1;
  }
  float* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_static_scratch_mu);
    if (!g_static_scratch_ptr[dev]) {
      // set-up on the first call on this device, with the device current
      void* ptr = nullptr;
      e = cudaGetSymbolAddress(&ptr, g_static_apply_scratch);
      if (e != cudaSuccess || !ptr) {
        set_error(std::string("normuon_apply_static: cudaGetSymbolAddress failed: ") + cudaGetErrorString(e));
        return -1;
      }
      g_static_scratch_ptr[dev] = static_cast<float*>(ptr);
    }
    scratch = g_static_scratch_ptr[dev];
  }
  // The finish kernel writes every scratch float that the apply kernel reads
  // (per-row factors and the per-matrix factor), so nothing needs clearing.
  return normuon_apply(O, rowsq, S, r, c, params, rems, emas, vrows, param_dtype, neg_lr, lr_wd, wd_factor, wd_on,
                       cautious, shape_scale, w_beta2, ema_weight, scratch, stream);
}

}  // namespace b2o
