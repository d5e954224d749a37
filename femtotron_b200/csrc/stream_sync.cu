// Stream memory operations and the owner-side reduction of the fused tensor-parallel paths.
//
// Cross-GPU ordering for the fused tensor-parallel paths:
//   * stream_write (cuStreamWriteValue32): a stream writes an epoch into local or peer memory
//     once its prior work (kernels, copy-engine transfers) is complete, without an SM;
//   * wait_flags_geq: a one-warp kernel that waits, with a time limit, until flags written by
//     peers reach an epoch (a stream-side wait would have no limit).
// The copy-engine all-gather of the fused AG->GEMM and the flag protocol of the fused
// GEMM->RS are built on these.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda.h>

#include <stdexcept>
#include <string>
#include <vector>

#include "common.cuh"

namespace ft {

namespace {
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

// Bounded cross-GPU wait: one warp polls up to 32 flags (lane i -> addrs[i]) with
// ld.acquire.sys until every (int32)(flag - value) >= 0, backing off with __nanosleep.  After
// `timeout_ms` it writes `code` + (index of the first missing flag) into the device status
// word and returns, so a peer that never publishes ends the wait with an error the host
// reads (KernelTimeoutError) instead of a stream that waits forever.  This replaces a
// cuStreamWaitValue32, which has no time limit.
struct WaitArgs {
  const int* addrs[32];
  int n, value, code;
  int* err;
  uint64_t timeout_ns;
};

__global__ void wait_flags_kernel(const __grid_constant__ WaitArgs a) {
  const int lane = threadIdx.x;
  uint64_t t0;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  bool done = lane >= a.n;
  uint32_t backoff = 64;
  while (true) {
    if (!done) {
      int v;
      asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(a.addrs[lane]) : "memory");
      done = (v - a.value) >= 0;
    }
    const unsigned missing = __ballot_sync(0xffffffffu, !done);
    if (missing == 0) return;
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    if (t - t0 > a.timeout_ns) {
      if (lane == 0) atomicExch(a.err, a.code + (__ffs(missing) - 1));
      return;
    }
    __nanosleep(backoff);
    if (backoff < 2048) backoff <<= 1;
  }
}

void wait_flags_geq(const std::vector<int64_t>& addrs, int64_t value, torch::Tensor& err,
                    int64_t timeout_ms, int64_t code) {
  TORCH_CHECK(addrs.size() <= 32, "wait_flags_geq: at most 32 flags");
  TORCH_CHECK(timeout_ms > 0, "wait_flags_geq: timeout_ms must be positive");
  TORCH_CHECK(err.scalar_type() == at::kInt && err.is_cuda());
  if (addrs.empty()) return;
  WaitArgs a{};
  for (size_t i = 0; i < addrs.size(); ++i) {
    TORCH_CHECK((addrs[i] & 3) == 0, "wait_flags_geq: flags must be 4-byte aligned");
    a.addrs[i] = reinterpret_cast<const int*>(addrs[i]);
  }
  a.n = static_cast<int>(addrs.size());
  a.value = static_cast<int>(value);
  a.code = static_cast<int>(code);
  a.err = err.data_ptr<int>();
  a.timeout_ns = static_cast<uint64_t>(timeout_ms) * 1000000ull;
  wait_flags_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
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
