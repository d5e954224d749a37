// Stream memory operations and the owner-side reduction of the fused tensor-parallel paths.
//
// cuStreamWaitValue32 / cuStreamWriteValue32 order work across GPUs without occupying any
// SM: a stream can wait for a 32-bit flag in device memory (written by a peer over NVLink)
// to reach an epoch, and can write an epoch into local or peer memory once its prior work is
// complete (the write carries a system-scope fence).  The copy-engine all-gather of the
// fused AG->GEMM and the flag protocol of the fused GEMM->RS are built on these.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda.h>

#include <stdexcept>
#include <string>

#include "common.cuh"

namespace ft {

namespace {
using WaitFn = CUresult (*)(CUstream, CUdeviceptr, cuuint32_t, unsigned int);
using WriteFn = CUresult (*)(CUstream, CUdeviceptr, cuuint32_t, unsigned int);

template <typename F>
F entry(const char* name) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess || p == nullptr)
    throw std::runtime_error(std::string("femtotron_b200: driver entry point missing: ") + name);
  return reinterpret_cast<F>(p);
}

void check_cu(CUresult r, const char* what) {
  if (r != CUDA_SUCCESS)
    throw std::runtime_error(std::string("femtotron_b200: ") + what + " failed with CUresult " +
                             std::to_string(static_cast<int>(r)));
}
}  // namespace

// Make the current stream wait until (int32)(*addr - value) >= 0.
void stream_wait_geq(int64_t addr, int64_t value) {
  static WaitFn fn = entry<WaitFn>("cuStreamWaitValue32");
  auto st = at::cuda::getCurrentCUDAStream();
  check_cu(fn(reinterpret_cast<CUstream>(st.stream()), static_cast<CUdeviceptr>(addr),
              static_cast<cuuint32_t>(value), CU_STREAM_WAIT_VALUE_GEQ),
           "cuStreamWaitValue32");
}

// Write `value` to `addr` (local or peer device memory) once the stream's prior work is done.
void stream_write(int64_t addr, int64_t value) {
  static WriteFn fn = entry<WriteFn>("cuStreamWriteValue32");
  auto st = at::cuda::getCurrentCUDAStream();
  check_cu(fn(reinterpret_cast<CUstream>(st.stream()), static_cast<CUdeviceptr>(addr),
              static_cast<cuuint32_t>(value), CU_STREAM_WRITE_VALUE_DEFAULT),
           "cuStreamWriteValue32");
}

// out[i] = sum_s parts[s][i] (+ residual[i]), bf16 in/out, fp32 sum.  parts: [S, n] contiguous.
__global__ void sum_partials_kernel(const __nv_bfloat16* __restrict__ parts, int S, int64_t n,
                                    const __nv_bfloat16* __restrict__ resid,
                                    __nv_bfloat16* __restrict__ out) {
  asm volatile("fence.acq_rel.sys;" ::: "memory");  // partials were stored by peers over NVLink
  const int64_t nv = n / 8;
  for (int64_t v = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; v < nv;
       v += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    auto add8 = [&](const __nv_bfloat16* src) {
      const uint4 q = *reinterpret_cast<const uint4*>(src + v * 8);
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&q);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(h[j]);
        acc[2 * j] += f.x;
        acc[2 * j + 1] += f.y;
      }
    };
    for (int s = 0; s < S; ++s) add8(parts + static_cast<int64_t>(s) * n);
    if (resid) add8(resid);
    uint4 o;
    uint32_t* po = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int j = 0; j < 4; ++j) po[j] = pack_bf16x2(acc[2 * j], acc[2 * j + 1]);
    *reinterpret_cast<uint4*>(out + v * 8) = o;
  }
}

void sum_partials(const torch::Tensor& parts, const c10::optional<torch::Tensor>& resid,
                  torch::Tensor& out) {
  TORCH_CHECK(parts.is_contiguous() && out.is_contiguous() && parts.scalar_type() == at::kBFloat16);
  const int S = parts.size(0);
  const int64_t n = out.numel();
  TORCH_CHECK(parts.numel() == S * n && n % 8 == 0);
  if (resid.has_value()) TORCH_CHECK(resid->is_contiguous() && resid->numel() == n);
  const c10::cuda::CUDAGuard g(out.device());
  int dev, sms;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((n / 8 + 255) / 256, sms * 4)));
  sum_partials_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(parts.data_ptr()), S, n,
      resid.has_value() ? reinterpret_cast<const __nv_bfloat16*>(resid->data_ptr()) : nullptr,
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace ft
