// Symmetric device memory across the processes of one node (one process per GPU).
//
// Every rank allocates a buffer of the same size with cudaMalloc (outside PyTorch's caching
// allocator, because an IPC handle must name the base of an allocation), exports a CUDA IPC
// handle, and opens the handles of its peers; the resulting peer pointers address the
// peers' buffers over NVLink (NVSwitch).  On top of that this file provides:
//   * peer copies on a stream (copy engines, no SM involvement) used by the ZeRO-3
//     all-gather and the fused tensor-parallel all-gather.
// The kernels that read peers' buffers directly are in zero_fused.cu (ZeRO reduce-scatter +
// AdamW) and gemm.cu / stream_sync.cu (tensor-parallel GEMM -> reduce-scatter).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda.h>

#include <cstring>
#include <string>
#include <vector>

#include "common.cuh"

namespace ft {

namespace {
void check(cudaError_t e, const char* what) {
  if (e != cudaSuccess)
    throw std::runtime_error(std::string("femtotron_b200 symm: ") + what + ": " + cudaGetErrorString(e));
}
}  // namespace

// Allocate `nbytes` (zeroed) with cudaMalloc and return it as a uint8 tensor that frees the
// memory when the tensor dies.
torch::Tensor symm_alloc(int64_t nbytes, int64_t device) {
  const c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(device));
  void* p = nullptr;
  check(cudaMalloc(&p, static_cast<size_t>(nbytes)), "cudaMalloc");
  check(cudaMemset(p, 0, static_cast<size_t>(nbytes)), "cudaMemset");
  auto opts = torch::TensorOptions().dtype(torch::kUInt8).device(torch::kCUDA, device);
  return torch::from_blob(p, {nbytes}, [](void* q) { cudaFree(q); }, opts);
}

// 64-byte CUDA IPC handle of the allocation that starts at `t`'s data pointer.
torch::Tensor ipc_handle(const torch::Tensor& t) {
  cudaIpcMemHandle_t h;
  check(cudaIpcGetMemHandle(&h, t.data_ptr()), "cudaIpcGetMemHandle");
  auto out = torch::empty({static_cast<int64_t>(sizeof(h))}, torch::kUInt8);
  std::memcpy(out.data_ptr(), &h, sizeof(h));
  return out;
}

// Open a peer's handle; returns the device address of its buffer in this process.
int64_t ipc_open(const torch::Tensor& handle, int64_t device) {
  const c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(device));
  TORCH_CHECK(handle.numel() == static_cast<int64_t>(sizeof(cudaIpcMemHandle_t)));
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle.data_ptr(), sizeof(h));
  void* p = nullptr;
  check(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
  return reinterpret_cast<int64_t>(p);
}

void ipc_close(int64_t ptr) {
  if (ptr) cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr));
}

// A tensor view of `numel` elements of `dtype` at device address `ptr` (no ownership).
torch::Tensor tensor_at(int64_t ptr, int64_t numel, torch::ScalarType dtype, int64_t device) {
  auto opts = torch::TensorOptions().dtype(dtype).device(torch::kCUDA, device);
  return torch::from_blob(reinterpret_cast<void*>(ptr), {numel}, opts);
}

// Copy engine transfers: dst[i] <- src_ptrs[i] (bytes[i] each) on the current stream.
void copy_from_ptrs(const std::vector<int64_t>& dsts, const std::vector<int64_t>& srcs,
                    const std::vector<int64_t>& nbytes) {
  auto st = at::cuda::getCurrentCUDAStream();
  for (size_t i = 0; i < dsts.size(); ++i)
    check(cudaMemcpyAsync(reinterpret_cast<void*>(dsts[i]), reinterpret_cast<void*>(srcs[i]),
                          static_cast<size_t>(nbytes[i]), cudaMemcpyDeviceToDevice, st),
          "cudaMemcpyAsync");
}

}  // namespace ft
