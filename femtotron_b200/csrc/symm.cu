// Symmetric device memory across the processes of one node (one process per GPU).
//
// Every rank allocates a buffer of the same size with cudaMalloc (outside PyTorch's caching
// allocator, because an IPC handle must name the base of an allocation), exports a CUDA IPC
// handle, and opens the handles of its peers; the resulting peer pointers address the
// peers' buffers over NVLink (NVSwitch).  On top of that this file provides:
//   * peer copies on a stream (copy engines, no SM involvement) used by the ZeRO-3
//     all-gather;
//   * device flags written by the stream (cuStreamWriteValue32) so a kernel can wait for a
//     copy without the host;
//   * a reduce-scatter kernel that reads every peer's slice of a gradient buffer directly
//     (P2P loads), averages in fp32 and adds into the local fp32 shard (reduce + cast +
//     accumulate in one pass), with bounded cross-rank flag waits.
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

// ------------------------------------------------------------------------------------------
// P2P reduce-scatter with fused cast/scale/accumulate
// ------------------------------------------------------------------------------------------
// Protocol (one flag array of `world` int32 per buffer, in symmetric memory):
//   p2p_publish (compute stream, after the kernels that wrote this rank's bf16 buffer):
//       flags_of_rank_r[this rank] = epoch for every r (release, system scope);
//   p2p_reduce_scatter (communication stream): wait (bounded) until every peer's flag in the
//       local array is >= epoch, then read slice [rank*shard, (rank+1)*shard) of every peer's
//       buffer over NVLink and write  acc[i] (+)= scale * sum_r buf_r[rank*shard + i]  in fp32
//       (the buffers hold bf16 or fp32 gradients).
// Peers may reuse their buffers only after every rank's reduction has finished; the caller
// provides that ordering (a device-side barrier between steps).
struct RSArgs {
  const void* bufs[8];           // every rank's full gradient buffer (peer addresses), bf16 or fp32
  volatile int* flags_local;     // this rank's flag array [world]
  int* flags_remote[8];          // flag arrays of every rank (peer addresses)
  float* acc;                    // local fp32 shard accumulator
  int64_t shard;
  int64_t base;                  // element offset of the reduced slice inside every buffer
  int world, rank, epoch, accumulate, wait;
  float scale;
  int* err;
  uint64_t timeout_ns;           // bound of the flag wait
};

__device__ __forceinline__ uint64_t global_ns_() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__global__ void p2p_publish_kernel(RSArgs a) {
  // one thread: tell every rank that this rank's buffer for `epoch` is complete
  __threadfence_system();
  for (int r = 0; r < a.world; ++r) {
    asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(a.flags_remote[r] + a.rank), "r"(a.epoch)
                 : "memory");
  }
}

// Bounded wait for all peers' flags >= epoch (the caller's bound, 20 s by default: a peer
// that is that late has failed).  On timeout: error code 100 + the first missing rank.
__device__ __forceinline__ bool wait_peers(const RSArgs& a) {
  const uint64_t t0 = global_ns_();
  for (int r = 0; r < a.world; ++r) {
    while (true) {
      int v;
      asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(a.flags_local + r) : "memory");
      if (v - a.epoch >= 0) break;
      if (global_ns_() - t0 > a.timeout_ns) {
        atomicExch(a.err, 100 + r);
        return false;
      }
      __nanosleep(512);
    }
  }
  return true;
}

// Load 8 consecutive elements (bf16 or fp32) as fp32.
__device__ __forceinline__ void load8(const void* p, int64_t i, float (&f)[8], bool f32) {
  if (f32) {
    const float4* q = reinterpret_cast<const float4*>(static_cast<const float*>(p) + i);
    const float4 a = q[0], b = q[1];
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  } else {
    const uint4 q = *reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(p) + i);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&q);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 t = __bfloat1622float2(h[j]);
      f[2 * j] = t.x;
      f[2 * j + 1] = t.y;
    }
  }
}

template <bool F32>
__global__ void p2p_reduce_scatter_kernel(RSArgs a) {
  if (a.wait) {
    __shared__ int ok;
    if (threadIdx.x == 0) ok = wait_peers(a) ? 1 : 0;
    __syncthreads();
    if (!ok) return;
  }
  const int64_t base = a.base;
  const int64_t nvec = a.shard / 8;
  for (int64_t v = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; v < nvec;
       v += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float s[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      if (r >= a.world) break;
      if (!FT_DCHECK(a.bufs[r] != nullptr, a.err, 91)) break;
      float f[8];
      load8(a.bufs[r], base + v * 8, f, F32);
#pragma unroll
      for (int j = 0; j < 8; ++j) s[j] += f[j];
    }
    float4* d = reinterpret_cast<float4*>(a.acc + v * 8);
    float4 o0 = make_float4(s[0] * a.scale, s[1] * a.scale, s[2] * a.scale, s[3] * a.scale);
    float4 o1 = make_float4(s[4] * a.scale, s[5] * a.scale, s[6] * a.scale, s[7] * a.scale);
    if (a.accumulate) {
      const float4 p0 = d[0], p1 = d[1];
      o0.x += p0.x; o0.y += p0.y; o0.z += p0.z; o0.w += p0.w;
      o1.x += p1.x; o1.y += p1.y; o1.z += p1.z; o1.w += p1.w;
    }
    d[0] = o0;
    d[1] = o1;
  }
}

void launch_reduce(const RSArgs& a, bool f32, int grid) {
  auto st = at::cuda::getCurrentCUDAStream();
  if (f32)
    p2p_reduce_scatter_kernel<true><<<grid, 256, 0, st>>>(a);
  else
    p2p_reduce_scatter_kernel<false><<<grid, 256, 0, st>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

namespace {
RSArgs make_rs_args(const std::vector<int64_t>& buf_ptrs, const std::vector<int64_t>& flag_ptrs,
                    int64_t rank, int64_t epoch) {
  const int world = static_cast<int>(flag_ptrs.size());
  TORCH_CHECK(world >= 1 && world <= 8, "p2p: 1..8 ranks");
  TORCH_CHECK(buf_ptrs.empty() || static_cast<int>(buf_ptrs.size()) == world);
  RSArgs a{};
  for (int r = 0; r < world; ++r) {
    if (!buf_ptrs.empty()) a.bufs[r] = reinterpret_cast<const void*>(buf_ptrs[r]);
    a.flags_remote[r] = reinterpret_cast<int*>(flag_ptrs[r]);
  }
  a.world = world;
  a.rank = static_cast<int>(rank);
  a.epoch = static_cast<int>(epoch);
  return a;
}
}  // namespace

// Publish this rank's buffer for `epoch` to every rank (flag_ptrs[r] = rank r's flag array).
void p2p_publish(const std::vector<int64_t>& flag_ptrs, int64_t rank, int64_t epoch) {
  RSArgs a = make_rs_args({}, flag_ptrs, rank, epoch);
  p2p_publish_kernel<<<1, 1, 0, at::cuda::getCurrentCUDAStream()>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void p2p_reduce_scatter(const std::vector<int64_t>& buf_ptrs, int64_t flags_local,
                        const std::vector<int64_t>& flag_ptrs, torch::Tensor& acc, int64_t shard,
                        int64_t rank, int64_t epoch, double scale, bool accumulate,
                        torch::Tensor& err, bool src_f32, int64_t timeout_ms) {
  TORCH_CHECK(timeout_ms > 0, "p2p_reduce_scatter: timeout_ms must be positive");
  TORCH_CHECK(acc.scalar_type() == at::kFloat && acc.is_contiguous() && acc.numel() >= shard);
  TORCH_CHECK(shard % 8 == 0, "p2p_reduce_scatter: shard must be a multiple of 8 elements");
  RSArgs a = make_rs_args(buf_ptrs, flag_ptrs, rank, epoch);
  for (int r = 0; r < a.world; ++r)
    TORCH_CHECK((reinterpret_cast<uintptr_t>(a.bufs[r]) & 15) == 0,
                "p2p_reduce_scatter: buffers must be 16-byte aligned");
  a.flags_local = reinterpret_cast<volatile int*>(flags_local);
  a.acc = acc.data_ptr<float>();
  a.shard = shard;
  a.base = rank * shard;
  a.wait = 1;
  a.accumulate = accumulate ? 1 : 0;
  a.scale = static_cast<float>(scale);
  a.err = err.data_ptr<int>();
  a.timeout_ns = static_cast<uint64_t>(timeout_ms) * 1000000ull;
  int dev, sms;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t nvec = shard / 8;
  // four 256-thread blocks per SM: each thread keeps `world` 32-byte loads in flight, and the
  // peer reads need several MB in flight GPU-wide to cover NVLink latency (one block per SM
  // measured 0.39 of the HBM copy rate on local buffers, long-scoreboard bound)
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((nvec + 255) / 256, 4 * sms)));
  launch_reduce(a, src_f32, grid);
}

// Local reduction of `world` bf16 slices (already in this GPU's memory, e.g. pulled from the
// peers by copy engines) into the fp32 shard: acc (+)= scale * sum_r src_r.  No waits.
void reduce_slices_f32(const std::vector<int64_t>& src_ptrs, torch::Tensor& acc, int64_t n,
                       double scale, bool accumulate, bool src_f32) {
  TORCH_CHECK(acc.scalar_type() == at::kFloat && acc.is_contiguous() && acc.numel() >= n);
  TORCH_CHECK(n % 8 == 0, "reduce_slices_f32: n must be a multiple of 8");
  const int world = static_cast<int>(src_ptrs.size());
  TORCH_CHECK(world >= 1 && world <= 8);
  RSArgs a{};
  for (int r = 0; r < world; ++r) {
    a.bufs[r] = reinterpret_cast<const void*>(src_ptrs[r]);
    TORCH_CHECK((src_ptrs[r] & 15) == 0, "reduce_slices_f32: 16-byte aligned sources");
  }
  a.world = world;
  a.acc = acc.data_ptr<float>();
  a.shard = n;
  a.base = 0;
  a.wait = 0;
  a.accumulate = accumulate ? 1 : 0;
  a.scale = static_cast<float>(scale);
  int dev, sms;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t nvec = n / 8;
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((nvec + 255) / 256, 4 * sms)));
  launch_reduce(a, src_f32, grid);
}

}  // namespace ft
