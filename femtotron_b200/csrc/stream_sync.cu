// Stream memory operations of the fused tensor-parallel paths.
//
// Cross-GPU ordering for the fused tensor-parallel paths:
//   * stream_write (cuStreamWriteValue32): a stream writes an epoch into local or peer memory
//     once its prior work (kernels, copy-engine transfers) is complete, without an SM;
//   * wait_flags_geq: a one-warp kernel that waits, with a time limit, until flags written by
//     peers reach an epoch (a stream-side wait would have no limit).
// The flag protocols of the fused AG->GEMM and GEMM->RS (tp_comm.cu, fused.py) are built on
// these.
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

}  // namespace ft
