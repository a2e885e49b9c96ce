// Shared device/host helpers for libb2o (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <atomic>
#include <string>
#include <utility>

namespace b2o {

// ---------------------------------------------------------------- status ---
// Host-side error text for the last failing call on this thread.
void set_error(const std::string& msg);
// Counts kernel launches made by the library (reported by the benchmark).
// While this thread captures a launch graph, launches are counted into
// *t_capture_launches instead (they run only when the graph is replayed).
extern std::atomic<int64_t> g_launches;
extern thread_local int64_t* t_capture_launches;
inline void count_launch(int n = 1) {
  if (t_capture_launches) *t_capture_launches += n;
  else g_launches.fetch_add(n, std::memory_order_relaxed);
}

// Device error word (one per device, lazily allocated by the library at load
// of the first device call; see c_abi.cu). Kernels OR error bits into it.
int* device_error_word();

enum DeviceError : int {
  kErrWaitTimeout = 1,     // a bounded mbarrier wait ran out
  kErrBadTile = 2,         // a tile index outside the problem (never expected)
};

// Returns 0 or the CUDA error of the last launch (and records the message).
int check_launch(const char* what);

// ------------------------------------------------------------- numerics ---
// bf16 <-> fp32 with round-to-nearest-even (the rounding torch uses for
// .to(torch.bfloat16) and for bf16 tensor arithmetic).
__device__ __forceinline__ float bf16_to_f32(uint16_t h) {
  return __uint_as_float(static_cast<uint32_t>(h) << 16);
}
__device__ __forceinline__ uint16_t f32_to_bf16(float f) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}
__device__ __forceinline__ float round_bf16(float f) { return bf16_to_f32(f32_to_bf16(f)); }
// IEEE binary16 stored as raw bits (round-to-nearest-even).
__device__ __forceinline__ float f16_to_f32(uint16_t h) { return __half2float(__ushort_as_half(h)); }
__device__ __forceinline__ uint16_t f32_to_f16(float f) { return __half_as_ushort(__float2half_rn(f)); }
// 16-bit storage of either kind: half != 0 selects binary16, else bfloat16.
__device__ __forceinline__ float h16_to_f32(uint16_t h, int half) { return half ? f16_to_f32(h) : bf16_to_f32(h); }
__device__ __forceinline__ uint16_t f32_to_h16(float f, int half) { return half ? f32_to_f16(f) : f32_to_bf16(f); }

// ------------------------------------------- programmatic dependent launch ---
// Every library kernel is launched with programmatic stream serialisation: it
// lets its dependents launch early (trigger) and waits for its predecessor to
// complete and flush before touching global memory (wait), so launch latency
// and the previous kernel's tail overlap.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// B2O_PDL=0 in the environment launches every kernel in plain stream order.
bool pdl_enabled();

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// torch's lerp (ATen/native/Lerp.h): small weights interpolate from `self`,
// large ones from `end`; evaluated in fp32 opmath with fused multiply-add.
__device__ __forceinline__ float torch_lerp(float self, float end, float w) {
  return (fabsf(w) < 0.5f) ? fmaf(w, end - self, self) : fmaf(-(end - self), 1.0f - w, end);
}

}  // namespace b2o
