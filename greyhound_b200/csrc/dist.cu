// Plumbing for the data-parallel weight-gradient reduce-scatter that the
// dW GEMM performs in its epilogue (gh_lce_dw_peers): CUDA IPC of the
// receive buffers between the ranks of one node, and the fixed-order sum of
// the received slots.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>

#include "common.cuh"

namespace gh {
namespace {

PFN_cuMemGetAddressRange_v3020 get_range_fn() {
  static PFN_cuMemGetAddressRange_v3020 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(p);
  });
  return fn;
}

// out0 = out1 = sum of nslots [rows, cols] slices (pitch ld) spaced
// slot_stride elements apart; fp32 sum in slot order, one rounding.
template <typename T>
__global__ void __launch_bounds__(256)
sum_slots_kernel(const T* __restrict__ slots, int nslots, int64_t slot_stride, int64_t rows, int64_t cols,
                 int64_t ld, T* out0, T* out1) {
  constexpr int PER = 16 / sizeof(T);
  const int64_t vpr = cols / PER;
  const int64_t n = rows * vpr;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / vpr, c = (i - r * vpr) * PER;
    float acc[PER];
#pragma unroll
    for (int k = 0; k < PER; ++k) acc[k] = 0.f;
    for (int sl = 0; sl < nslots; ++sl) {
      Vec16<T> v;
      v.raw = ld16_last(slots + sl * slot_stride + r * ld + c);
      float f[PER];
      v.to_float(f);
#pragma unroll
      for (int k = 0; k < PER; ++k) acc[k] += f[k];
    }
    Vec16<T> o;
    o.from_float(acc);
    st16(out0 + r * ld + c, o.raw);
    if (out1) st16(out1 + r * ld + c, o.raw);
  }
}

int sm_count() {
  int dev = 0, n = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
}

}  // namespace
}  // namespace gh

using namespace gh;

extern "C" int gh_sum_slots(const void* slots, int nslots, int64_t slot_stride, int64_t rows, int64_t cols,
                            int64_t ld, int dtype, void* out0, void* out1, void* stream) {
  if (dtype != GH_BF16 && dtype != GH_F16) return set_error(GH_ETYPE, "gh_sum_slots: bf16 or fp16 expected");
  if (nslots <= 0 || rows < 0 || cols < 0 || ld < cols) return set_error(GH_EINVAL, "gh_sum_slots: bad shape");
  if (rows == 0 || cols == 0) return GH_OK;
  if (!slots || !out0) return set_error(GH_EINVAL, "null pointer argument");
  const uintptr_t al = reinterpret_cast<uintptr_t>(slots) | reinterpret_cast<uintptr_t>(out0) |
                       reinterpret_cast<uintptr_t>(out1) | (uintptr_t)(ld * 2) | (uintptr_t)(slot_stride * 2) |
                       (uintptr_t)(cols * 2);
  if (al & 15) return set_error(GH_EINVAL, "gh_sum_slots: 16-byte aligned buffers, pitches and widths required");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned grid = 4 * sm_count();
  if (dtype == GH_BF16)
    sum_slots_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(slots), nslots,
                                                          slot_stride, rows, cols, ld,
                                                          static_cast<__nv_bfloat16*>(out0),
                                                          static_cast<__nv_bfloat16*>(out1));
  else
    sum_slots_kernel<__half><<<grid, 256, 0, st>>>(static_cast<const __half*>(slots), nslots, slot_stride, rows, cols,
                                                   ld, static_cast<__half*>(out0), static_cast<__half*>(out1));
  count_launch(1);
  return check_launch("gh_sum_slots");
}

extern "C" int gh_ipc_get_handle(const void* ptr, void* handle_out, size_t* offset_out) {
  if (!ptr || !handle_out || !offset_out) return set_error(GH_EINVAL, "null pointer argument");
  auto range = get_range_fn();
  if (!range) return set_error(GH_ECUDA, "cuMemGetAddressRange unavailable");
  int dev = 0;  // bind the current device's primary context for the driver call
  cudaGetDevice(&dev);
  cudaSetDevice(dev);
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return set_error(GH_ECUDA, "cuMemGetAddressRange failed");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return set_error(GH_ECUDA, "cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
  static_assert(sizeof(h) == 64, "IPC handle size");
  memcpy(handle_out, &h, sizeof(h));
  *offset_out = reinterpret_cast<uintptr_t>(ptr) - static_cast<uintptr_t>(base);
  return GH_OK;
}

extern "C" int gh_ipc_open(const void* handle, size_t offset, void** ptr_out) {
  if (!handle || !ptr_out) return set_error(GH_EINVAL, "null pointer argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return set_error(GH_ECUDA, "cudaIpcOpenMemHandle: %s", cudaGetErrorString(e));
  *ptr_out = static_cast<char*>(base) + offset;
  return GH_OK;
}

extern "C" int gh_ipc_close(void* ptr, size_t offset) {
  if (!ptr) return GH_OK;
  cudaError_t e = cudaIpcCloseMemHandle(static_cast<char*>(ptr) - offset);
  if (e != cudaSuccess) return set_error(GH_ECUDA, "cudaIpcCloseMemHandle: %s", cudaGetErrorString(e));
  return GH_OK;
}

extern "C" int gh_memcpy_async(void* dst, const void* src, size_t bytes, void* stream) {
  if (bytes == 0) return GH_OK;
  if (!dst || !src) return set_error(GH_EINVAL, "null pointer argument");
  cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return set_error(GH_ECUDA, "cudaMemcpyAsync: %s", cudaGetErrorString(e));
  return GH_OK;
}
