// Gradient-norm clip: torch.nn.utils.clip_grad_norm_(params, max_norm,
// foreach=True) as the reference calls it before the optimizer steps
// (transformer_lm/train_sol.py:498-499; semantics of torch/nn/utils/clip_grad.py).
//
//   n_i   = ||g_i||_2 from an fp32 sum of squares, rounded to g_i's dtype
//           (torch._foreach_norm returns each norm in the gradient's dtype)
//   total = ||(n_1, ..., n_k)||_2 in fp32, rounded to the promoted dtype of the
//           norms (torch.linalg.vector_norm of torch.stack(norms))
//   coef  = min(max_norm * (1 / (total + 1e-6)), 1), each op rounded to that
//           dtype (a Python scalar divided by a tensor is reciprocal(t) * scalar)
//   g_i  <- dtype(g_i * coef)                         (torch._foreach_mul_)
//
// Three launches: a deterministic multi-tensor sum of squares (one partial per
// CTA), a one-CTA finalisation that writes {total, coef} to device memory, and
// the in-place scaling. The optimizers can instead read coef in their own
// passes (deferred clipping), which saves the scaling pass's read and write.
#include "b2o_common.cuh"
#include "b2o_internal.h"

#include <algorithm>
#include <cstring>
#include <string>

namespace b2o {

constexpr int kClipMaxTensors = 1024;       // tensors per call
constexpr int kClipLaunchTensors = 256;     // tensors per sum-of-squares / scale launch
constexpr int64_t kClipChunk = 256 * 8 * 16;  // elements per CTA

static int64_t clip_chunks(int64_t n) { return (n + kClipChunk - 1) / kClipChunk; }

int64_t clip_scratch_floats(const int64_t* numels, int n) {
  if (n <= 0 || n > kClipMaxTensors || !numels) return -1;
  int64_t total = 0;
  for (int i = 0; i < n; ++i) total += clip_chunks(numels[i]);
  return std::max<int64_t>(1, total);
}

struct ClipTable {
  const void* g[kClipLaunchTensors];
  int64_t n[kClipLaunchTensors];
  int part0[kClipLaunchTensors];     // first partial of the tensor in the scratch buffer
  int cta0[kClipLaunchTensors + 1];  // prefix of CTAs per tensor
  unsigned char half[kClipLaunchTensors];  // 1: bf16, 0: fp32
  unsigned char vec[kClipLaunchTensors];
  int count;
};

__device__ __forceinline__ int clip_find(const ClipTable& t, int cta) {
  int lo = 0, hi = t.count - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (t.cta0[mid] <= cta) lo = mid; else hi = mid - 1;
  }
  return lo;
}

__global__ void __launch_bounds__(256) grad_sumsq_kernel(const __grid_constant__ ClipTable t,
                                                         float* __restrict__ partial) {
  pdl_wait();
  const int i = clip_find(t, blockIdx.x);
  const int chunk = blockIdx.x - t.cta0[i];
  const int64_t base = chunk * kClipChunk;
  const int64_t end = min(t.n[i], base + kClipChunk);
  float acc = 0.f;
  if (t.half[i]) {
    const uint16_t* g = static_cast<const uint16_t*>(t.g[i]);
    int64_t from = base;
    if (t.vec[i]) {
      for (int64_t k = base + threadIdx.x * 8; k + 8 <= end; k += 256 * 8) {
        const uint4 v = *reinterpret_cast<const uint4*>(g + k);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          const float a = bf16_to_f32(static_cast<uint16_t>(w[h] & 0xFFFFu));
          const float b = bf16_to_f32(static_cast<uint16_t>(w[h] >> 16));
          acc = fmaf(a, a, acc);
          acc = fmaf(b, b, acc);
        }
      }
      from = base + ((end - base) / 8) * 8;
    }
    for (int64_t k = from + threadIdx.x; k < end; k += 256) {
      const float a = bf16_to_f32(g[k]);
      acc = fmaf(a, a, acc);
    }
  } else {
    const float* g = static_cast<const float*>(t.g[i]);
    int64_t from = base;
    if (t.vec[i]) {
      for (int64_t k = base + threadIdx.x * 4; k + 4 <= end; k += 256 * 4) {
        const float4 v = *reinterpret_cast<const float4*>(g + k);
        acc = fmaf(v.x, v.x, acc);
        acc = fmaf(v.y, v.y, acc);
        acc = fmaf(v.z, v.z, acc);
        acc = fmaf(v.w, v.w, acc);
      }
      from = base + ((end - base) / 4) * 4;
    }
    for (int64_t k = from + threadIdx.x; k < end; k += 256) acc = fmaf(g[k], g[k], acc);
  }
  __shared__ float red[8];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.f;
    for (int k = 0; k < 8; ++k) s += red[k];
    partial[t.part0[i] + chunk] = s;
  }
}

struct ClipMeta {
  int part0[kClipMaxTensors + 1];
  unsigned char half[kClipMaxTensors];
  int count, out_half;
  float max_norm;
};

__device__ __forceinline__ float round_to(float x, int half) { return half ? round_bf16(x) : x; }

// one CTA: per-tensor norms in their dtypes, the total and the coefficient
__global__ void __launch_bounds__(1024) grad_norm_finalize_kernel(const __grid_constant__ ClipMeta m,
                                                                  const float* __restrict__ partial,
                                                                  float* __restrict__ out) {
  pdl_wait();
  __shared__ float red[32];
  float acc = 0.f;
  for (int i = threadIdx.x; i < m.count; i += blockDim.x) {
    float s = 0.f;
    for (int p = m.part0[i]; p < m.part0[i + 1]; ++p) s += partial[p];
    const float ni = round_to(sqrtf(s), m.half[i]);
    acc = fmaf(ni, ni, acc);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.f;
    for (int k = 0; k < static_cast<int>(blockDim.x >> 5); ++k) s += red[k];
    const int h = m.out_half;
    const float total = round_to(sqrtf(s), h);
    const float denom = round_to(total + 1e-6f, h);
    const float recip = round_to(__frcp_rn(denom), h);
    const float coef = round_to(recip * m.max_norm, h);
    out[0] = total;
    out[1] = fminf(coef, 1.0f);
  }
}

__global__ void __launch_bounds__(256) grad_scale_kernel(const __grid_constant__ ClipTable t,
                                                         const float* __restrict__ coef) {
  pdl_wait();
  const int i = clip_find(t, blockIdx.x);
  const int chunk = blockIdx.x - t.cta0[i];
  const int64_t base = chunk * kClipChunk;
  const int64_t end = min(t.n[i], base + kClipChunk);
  const float c = *coef;
  if (t.half[i]) {
    uint16_t* g = const_cast<uint16_t*>(static_cast<const uint16_t*>(t.g[i]));
    int64_t from = base;
    if (t.vec[i]) {
      for (int64_t k = base + threadIdx.x * 8; k + 8 <= end; k += 256 * 8) {
        uint4 v = *reinterpret_cast<const uint4*>(g + k);
        uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          const uint16_t a = f32_to_bf16(bf16_to_f32(static_cast<uint16_t>(w[h] & 0xFFFFu)) * c);
          const uint16_t b = f32_to_bf16(bf16_to_f32(static_cast<uint16_t>(w[h] >> 16)) * c);
          w[h] = a | (static_cast<uint32_t>(b) << 16);
        }
        *reinterpret_cast<uint4*>(g + k) = make_uint4(w[0], w[1], w[2], w[3]);
      }
      from = base + ((end - base) / 8) * 8;
    }
    for (int64_t k = from + threadIdx.x; k < end; k += 256) g[k] = f32_to_bf16(bf16_to_f32(g[k]) * c);
  } else {
    float* g = const_cast<float*>(static_cast<const float*>(t.g[i]));
    for (int64_t k = base + threadIdx.x; k < end; k += 256) g[k] = g[k] * c;
  }
}

static int check_clip_args(const void* const* grads, const int64_t* numels, const int* dtypes, int n,
                           const char* what) {
  if (n <= 0 || n > kClipMaxTensors || !grads || !numels || !dtypes) {
    set_error(std::string(what) + ": 1.." + std::to_string(kClipMaxTensors) + " tensors");
    return -1;
  }
  for (int i = 0; i < n; ++i) {
    if (numels[i] < 0 || (numels[i] > 0 && !grads[i])) { set_error(std::string(what) + ": bad tensor"); return -1; }
    if (dtypes[i] != B2O_F32 && dtypes[i] != B2O_BF16) {
      set_error(std::string(what) + ": gradients must be fp32 or bf16"); return -1;
    }
  }
  return 0;
}

// Launches `kernel` over the tensors in tables of kClipLaunchTensors; part0
// advances by each tensor's partial slots (one per CTA; none when empty).
template <typename Kernel, typename Arg>
static int clip_launch(Kernel kernel, const char* what, const void* const* grads, const int64_t* numels,
                       const int* dtypes, int n, Arg arg, cudaStream_t stream) {
  int part = 0;
  for (int i0 = 0; i0 < n; i0 += kClipLaunchTensors) {
    ClipTable t;
    memset(&t, 0, sizeof(t));
    t.count = std::min(kClipLaunchTensors, n - i0);
    int64_t ctas = 0;
    for (int k = 0; k < t.count; ++k) {
      const int i = i0 + k;
      t.g[k] = grads[i];
      t.n[k] = numels[i];
      t.half[k] = dtypes[i] == B2O_BF16;
      t.vec[k] = (reinterpret_cast<uintptr_t>(grads[i]) & 15u) == 0;
      t.part0[k] = part;
      t.cta0[k] = static_cast<int>(ctas);
      ctas += clip_chunks(numels[i]);
      part += static_cast<int>(clip_chunks(numels[i]));
    }
    t.cta0[t.count] = static_cast<int>(ctas);
    if (ctas > (1ll << 30)) { set_error(std::string(what) + ": too many elements"); return -1; }
    if (ctas == 0) continue;
    launch_pdl(kernel, dim3(static_cast<unsigned>(ctas)), dim3(256), 0, stream, t, arg);
    count_launch();
    if (int e = check_launch(what)) return e;
  }
  return 0;
}

int clip_grad_norm(const void* const* grads, const int64_t* numels, const int* dtypes, int n, float max_norm,
                   float* scratch, float* out, cudaStream_t stream) {
  if (int e = check_clip_args(grads, numels, dtypes, n, "clip_grad_norm")) return e;
  if (!scratch || !out) { set_error("clip_grad_norm: null scratch or output"); return -1; }
  ClipMeta m;
  memset(&m, 0, sizeof(m));
  int part = 0;
  bool any_f32 = false;
  for (int i = 0; i < n; ++i) {
    m.part0[i] = part;
    m.half[i] = dtypes[i] == B2O_BF16;
    any_f32 = any_f32 || dtypes[i] == B2O_F32;
    part += static_cast<int>(clip_chunks(numels[i]));  // an empty tensor has no partial (norm 0)
  }
  m.part0[n] = part;
  m.count = n;
  m.out_half = any_f32 ? 0 : 1;  // torch.stack promotes the norms to a common dtype
  m.max_norm = max_norm;
  if (int e = clip_launch(grad_sumsq_kernel, "grad_sumsq", grads, numels, dtypes, n, scratch, stream)) return e;
  launch_pdl(grad_norm_finalize_kernel, dim3(1), dim3(1024), 0, stream, m, static_cast<const float*>(scratch), out);
  count_launch();
  return check_launch("grad_norm_finalize");
}

int clip_scale(void* const* grads, const int64_t* numels, const int* dtypes, int n, const float* coef,
               cudaStream_t stream) {
  if (int e = check_clip_args(const_cast<const void* const*>(grads), numels, dtypes, n, "clip_scale")) return e;
  if (!coef) { set_error("clip_scale: null coefficient"); return -1; }
  return clip_launch(grad_scale_kernel, "grad_scale", const_cast<const void* const*>(grads), numels, dtypes, n,
                     coef, stream);
}

}  // namespace b2o
