// Peer exchange for the sharded step: CUDA IPC mappings of other ranks'
// buffers and copy-engine pushes into them over NVLink.
//
// The sharded step ends with every rank holding every updated bf16 weight.
// Instead of an all-gather kernel (which occupies SMs while the NorMuon GEMMs
// run, and splits their one-wave grids into two waves), each rank pushes the
// rows it updated straight into the same offsets of every peer's buffers with
// one cudaMemcpyAsync per (peer, region). Device-to-device copies whose
// destination is a peer's IPC-mapped memory run on the copy engines, so the
// push overlaps the tensor-core work at no SM cost.
//
// The reference is single-GPU; none of this has a counterpart there.
#include "b2o_common.cuh"
#include "b2o_internal.h"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>
#include <string>

namespace b2o {

static PFN_cuMemGetAddressRange_v3020 address_range_fn() {
  static PFN_cuMemGetAddressRange_v3020 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(ptr);
  });
  return fn;
}

}  // namespace b2o

using namespace b2o;

extern "C" {

int b2o_ipc_export(const void* d_ptr, void* handle_out, uint64_t* offset_out) {
  if (!d_ptr || !handle_out || !offset_out) { set_error("ipc_export: null argument"); return -1; }
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
  auto fn = address_range_fn();
  if (!fn) { set_error("ipc_export: cuMemGetAddressRange unavailable"); return -1; }
  CUdeviceptr base = 0;
  size_t size = 0;
  CUresult r = fn(&base, &size, reinterpret_cast<CUdeviceptr>(d_ptr));
  if (r != CUDA_SUCCESS) {
    set_error("ipc_export: pointer is not device memory (cuMemGetAddressRange code " +
              std::to_string(static_cast<int>(r)) + ")");
    return -1;
  }
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_error(std::string("ipc_export: cudaIpcGetMemHandle: ") + cudaGetErrorString(e) +
              " (memory from cuMemCreate, e.g. expandable segments, cannot be exported this way)");
    return static_cast<int>(e);
  }
  memcpy(handle_out, &h, sizeof(h));
  *offset_out = static_cast<uint64_t>(reinterpret_cast<CUdeviceptr>(d_ptr) - base);
  return 0;
}

int b2o_ipc_import(const void* handle, void** d_base_out) {
  if (!handle || !d_base_out) { set_error("ipc_import: null argument"); return -1; }
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_error(std::string("ipc_import: cudaIpcOpenMemHandle: ") + cudaGetErrorString(e));
    return static_cast<int>(e);
  }
  *d_base_out = base;
  return 0;
}

int b2o_ipc_close(void* d_base) {
  if (!d_base) { set_error("ipc_close: null argument"); return -1; }
  cudaError_t e = cudaIpcCloseMemHandle(d_base);
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_error(std::string("ipc_close: ") + cudaGetErrorString(e));
    return static_cast<int>(e);
  }
  return 0;
}

int b2o_copy_async(void* const* d_dst, const void* const* d_src, const int64_t* bytes, int n, void* stream) {
  if (n < 0 || (n > 0 && (!d_dst || !d_src || !bytes))) { set_error("copy_async: bad argument list"); return -1; }
  for (int i = 0; i < n; ++i) {
    if (bytes[i] < 0 || (bytes[i] > 0 && (!d_dst[i] || !d_src[i]))) {
      set_error("copy_async: copy " + std::to_string(i) + " has a null pointer or a negative size");
      return -1;
    }
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  for (int i = 0; i < n; ++i) {
    if (!bytes[i]) continue;
    cudaError_t e = cudaMemcpyAsync(d_dst[i], d_src[i], static_cast<size_t>(bytes[i]), cudaMemcpyDeviceToDevice, st);
    if (e != cudaSuccess) {
      cudaGetLastError();
      set_error("copy_async: copy " + std::to_string(i) + ": " + cudaGetErrorString(e));
      return static_cast<int>(e);
    }
  }
  return 0;
}

}  // extern "C"
